"""Multi-rank host logic on the CPU (gloo, world size 2 and 4).

* session sharding: every config-5 session lands on exactly one rank, loads balanced;
* KV-head sharding of one long session: each rank keeps only its kv heads' cache, computes its
  query heads (oracle attention stands in for the GPU kernel here), and the all-gather of head
  outputs must equal the single-rank result bit for bit.
"""
import importlib
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from __graft_entry__ import ROOT, load_package


def _sharding():
    load_package()
    return importlib.import_module("skyvision_b200.sharding")


def test_session_shards_config5():
    sh = _sharding()
    lens = np.random.default_rng(4).integers(512, 32769, 64)
    for n in (1, 2, 4, 8):
        shards = sh.session_shards(lens, n)
        flat = sorted(i for s in shards for i in s)
        assert flat == list(range(64))
        loads = [int(lens[s].sum()) for s in shards]
        assert max(loads) - min(loads) <= int(lens.max())


def test_head_ranges():
    sh = _sharding()
    assert sh.kv_head_range(8, 3, 4) == (6, 8)
    assert sh.q_head_range(32, 8, 3, 4) == (24, 32)
    with pytest.raises(ValueError):
        sh.kv_head_range(8, 0, 3)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q, k, v, S, n_past, ref_path):
    import sys
    sys.path.insert(0, ROOT)
    import torch.distributed as dist
    from oracle import oracle as orc
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        sh = _sharding()
        NH, HD = q.shape[1], q.shape[2]
        NKV = k.shape[1] // HD
        hs = sh.HeadShardedDecode(NH, NKV, HD, rank, world)
        # this rank's cache holds only its kv heads
        kc = np.ascontiguousarray(k[:, hs.kv_lo * HD:hs.kv_hi * HD]).view(np.uint8)
        vc = np.ascontiguousarray(v[:, hs.kv_lo * HD:hs.kv_hi * HD]).view(np.uint8)

        def attend(layer, ql, kl, vl):
            out = orc.attn(ql.numpy(), kc, vc, orc.TYPE_F16, hs.kv_hi - hs.kv_lo, HD, S, 1 / np.sqrt(HD),
                           orc.MASK_CAUSAL, n_past)
            return torch.from_numpy(out)

        out_full = torch.empty(1, NH, HD, dtype=torch.float32)
        qt = torch.from_numpy(q)
        kv_rows = torch.zeros(1, NKV * HD)          # unused by attend (cache already filled)
        hs.step_layer(attend, 0, qt, kv_rows, kv_rows, out_full)
        if rank == 0:
            np.save(ref_path, out_full.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_head_sharded_gather_matches_single_rank(tmp_path, world, orc):
    NH, NKV, HD, S = 32, 8, 128, 300
    n_past = S - 1
    q = orc.f16_to_f32(orc.normal_f16(9, 1, NH * HD)).reshape(1, NH, HD)
    k = orc.normal_f16(9, 2, S * NKV * HD).reshape(S, NKV * HD)
    v = orc.normal_f16(9, 3, S * NKV * HD).reshape(S, NKV * HD)
    ref = orc.attn(q, k.view(np.uint8), v.view(np.uint8), orc.TYPE_F16, NKV, HD, S, 1 / np.sqrt(HD),
                   orc.MASK_CAUSAL, n_past)
    path = str(tmp_path / "gathered.npy")
    mp.start_processes(_worker, args=(world, _free_port(), q, k, v, S, n_past, path), nprocs=world,
                       start_method="spawn", join=True)
    got = np.load(path)
    assert np.array_equal(got, ref)
