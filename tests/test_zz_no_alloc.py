"""sv_flash_attn_ext_static: attention for callers that cannot allocate device memory.

An operator running inside a ggml backend graph only receives its tensors, and
code running during CUDA stream capture may not call cudaMalloc, so neither can
hand sv_flash_attn_ext a workspace.  The static entry point keeps the split-K
scratch in a fixed device array of the library.  This test calls it through
the C ABI twice in a row and checks each result against sv_flash_attn_ext with
a caller-allocated workspace and against the CPU oracle, within the attention
tolerance of the other tests; it also checks that a shape needing more scratch than the array holds
is refused.  (This file is named so that pytest collects it last.)
"""
import ctypes

import numpy as np
import pytest
import torch

from __graft_entry__ import load_package

sv = load_package()
pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
MAX_ABS, REL_L2 = 2e-3, 1e-3


def _params(q, k, v, n_kv_head, head_dim, n_keys, scale, dst):
    T, NH, HD = q.shape
    p = sv._FaParams()
    p.q = q.data_ptr()
    p.q_type = sv.TYPE_F16
    p.q_ne[:] = [HD, T, NH]
    p.q_nb[:] = [2, q.stride(0) * 2, q.stride(1) * 2]
    for name, t in (("k", k), ("v", v)):
        setattr(p, name, t.data_ptr())
        setattr(p, name + "_type", sv.TYPE_F16)
        getattr(p, name + "_ne")[:] = [head_dim, n_keys, n_kv_head]
        getattr(p, name + "_nb")[:] = [2, t.stride(0), head_dim * 2]
    p.scale = scale
    p.dst = dst.data_ptr()
    return p


def _static_fn():
    f = sv.lib().sv_flash_attn_ext_static
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.POINTER(sv._FaParams), ctypes.c_void_p]
    return f


def _check_close(got, ref):
    d = np.abs(got.astype(np.float64) - ref.astype(np.float64))
    rel = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    assert np.isfinite(got).all()
    assert d.max() <= MAX_ABS and rel <= REL_L2, (float(d.max()), float(rel))


def test_static_scratch_matches_workspace_entry_point(orc):
    NKV, HD, NH, S = 8, 128, 32, 3000          # one decode query: 8 kv heads x many key splits
    g = torch.Generator(device=DEV).manual_seed(7)
    static_fn = _static_fn()
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):                        # two calls in a row share the static array
        k = torch.randn(S, NKV * HD, generator=g, device=DEV).half()
        v = torch.randn(S, NKV * HD, generator=g, device=DEV).half()
        q = torch.randn(1, NH, HD, generator=g, device=DEV).half()
        kb, vb = k.view(torch.uint8), v.view(torch.uint8)
        out_ws = torch.zeros(1, NH, HD, dtype=torch.float32, device=DEV)
        out_st = torch.full((1, NH, HD), float("nan"), dtype=torch.float32, device=DEV)
        p_ws = _params(q, kb, vb, NKV, HD, S, 1 / np.sqrt(HD), out_ws)
        need = sv.lib().sv_flash_attn_ext_workspace(ctypes.byref(p_ws))
        assert need > 0                          # the shape really uses split-K scratch
        ws = torch.empty(need, dtype=torch.uint8, device=DEV)
        assert sv.lib().sv_flash_attn_ext(ctypes.byref(p_ws), ws.data_ptr(), need, stream) == 0
        p_st = _params(q, kb, vb, NKV, HD, S, 1 / np.sqrt(HD), out_st)
        assert static_fn(ctypes.byref(p_st), stream) == 0
        torch.cuda.synchronize()
        _check_close(out_st.cpu().numpy(), out_ws.cpu().numpy())
        # and both against the fp32-accumulated oracle (no mask: every key of the view is visible)
        ref = orc.attn(q.float().cpu().numpy(), kb.cpu().numpy(), vb.cpu().numpy(), orc.TYPE_F16, NKV, HD, S,
                       1 / np.sqrt(HD), orc.MASK_NONE)
        _check_close(out_st.cpu().numpy(), ref)
        _check_close(out_ws.cpu().numpy(), ref)


def test_static_scratch_refuses_oversized_shape():
    NKV, HD, T, S = 8, 256, 288, 200           # 144 query tiles x 2 splits of HD 256 partials > 4 MiB
    q = torch.zeros(T, NKV, HD, dtype=torch.float16, device=DEV)
    kv = torch.zeros(S, NKV * HD * 2, dtype=torch.uint8, device=DEV)
    out = torch.zeros(T, NKV, HD, dtype=torch.float32, device=DEV)
    p = _params(q, kv, kv, NKV, HD, S, 0.0625, out)
    assert sv.lib().sv_flash_attn_ext_workspace(ctypes.byref(p)) > (4 << 20)
    assert _static_fn()(ctypes.byref(p), torch.cuda.current_stream().cuda_stream) == -6
