"""Failure detection on the GPU without a fault.

The library's kernels bound every on-device wait; an expired wait records
SV_DEVERR_TIMEOUT and the kernel returns.  sv_selftest_wait_timeout waits on an
mbarrier nothing completes (a 2 ms limit): the error bit must reach the host,
the kernel must return past the wait, and the context must stay usable for
ordinary work afterwards.  Nothing here traps, asserts or touches a bad address.
"""
import numpy as np
import pytest
import torch

from __graft_entry__ import load_package

sv = load_package()
pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def test_bounded_wait_expires_and_reports(orc):
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    reached = torch.zeros(1, dtype=torch.int32, device=DEV)
    st = torch.cuda.current_stream().cuda_stream
    assert sv.lib().sv_selftest_wait_timeout(err.data_ptr(), reached.data_ptr(), 2000, st) == 0
    torch.cuda.synchronize()
    assert int(err.item()) & sv.DEVERR_TIMEOUT
    assert int(reached.item()) == 1
    # the context is still healthy: a normal decode step runs and is correct
    kv = sv.KvCache()
    assert kv.alloc(0, 1, 8, 128, 512)
    k = orc.normal_f16(30, 1, 100 * 1024).reshape(100, 1024)
    v = orc.normal_f16(30, 2, 100 * 1024).reshape(100, 1024)
    kv.append(0, torch.from_numpy(k.view(np.float16)).to(DEV), torch.from_numpy(v.view(np.float16)).to(DEV), base=0)
    q = orc.normal_f16(30, 3, 32 * 128).reshape(1, 32, 128)
    out = kv.attn(0, torch.from_numpy(q.view(np.float16)).to(DEV), n_past=99, scale=1 / np.sqrt(128)).cpu().numpy()
    ref = orc.attn(orc.f16_to_f32(q), kv.tensor(0, 0).cpu().numpy(), kv.tensor(0, 1).cpu().numpy(), orc.TYPE_F16, 8,
                   128, 100, 1 / np.sqrt(128), orc.MASK_CAUSAL, 99)
    assert np.abs(out - ref).max() <= 2e-3
    assert kv.error_flags() == 0


def test_selftest_rejects_bad_limits():
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    assert sv.lib().sv_selftest_wait_timeout(err.data_ptr(), None, 0, None) == -1
    assert sv.lib().sv_selftest_wait_timeout(None, None, 100, None) == -1
