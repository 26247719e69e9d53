"""Head-sharded decode with the all-gather fused into the attention kernel (sv_peer_* and
sv_attn_append_at_peer).

world = 1 runs in-process on one GPU (the kernel's stores and counters go to the rank's own
buffer).  world = 2 runs two spawned processes, one per GPU, when two GPUs are visible: each rank
holds half of the kv heads of one session; the gathered rows of every layer must match the oracle
of the whole, unsharded session on both ranks.  NVLS is off; the ranks exchange IPC handles over a
gloo group and exit only between steps.  The long cases give each rank few kv heads over thousands of
keys, so the kernel takes more than 48 key splits per head and runs in its one-CTA-per-SM, 6-stage
ring form, with the gather fused in the same way.
"""
import os
import socket

import numpy as np
import pytest
import torch

from __graft_entry__ import load_package

pytestmark = pytest.mark.gpu
HD, L, STEPS = 128, 2, 3
SHORT = (8, 32, 1500)         # kv heads, query heads, cached rows before the first step
LONG1 = (2, 8, 20000)         # one rank, 2 kv heads: over 48 key splits per head
LONG2 = (8, 32, 9000)         # two ranks, 4 kv heads each: over 48 key splits per head


def _session(orc, NKV, NH, N0):
    """Seeded K/V rows (n0 + steps) per layer, and per step the query and the appended K/V row."""
    ne0 = NKV * HD
    rows = [(orc.normal_f16(61, 10 + l, (N0 + STEPS) * ne0).reshape(N0 + STEPS, ne0),
             orc.normal_f16(61, 20 + l, (N0 + STEPS) * ne0).reshape(N0 + STEPS, ne0)) for l in range(L)]
    q = orc.normal_f16(61, 30, STEPS * L * NH * HD).reshape(STEPS, L, 1, NH, HD)
    return rows, q


def _run_rank(rank, world, port, result, shape=SHORT):
    import torch.distributed as dist
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    sv = load_package()
    from oracle import oracle as orc
    torch.cuda.set_device(rank)
    dev = torch.device(f"cuda:{rank}")
    if world > 1:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    NKV, NH, N0 = shape
    nkv_l, nh_l = NKV // world, NH // world
    kv_lo, q_lo = rank * nkv_l, rank * nh_l
    rows, q = _session(orc, NKV, NH, N0)
    kv = sv.KvCache()
    assert kv.alloc(rank, L, nkv_l, HD, N0 + STEPS + 8)
    td = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.float16)).to(dev)
    for l in range(L):
        k, v = rows[l]
        kv.append(l, td(k[:N0, kv_lo * HD:(kv_lo + nkv_l) * HD]), td(v[:N0, kv_lo * HD:(kv_lo + nkv_l) * HD]), base=0)
    peer = sv.Peer(rank, rank, world, L, NH * HD * 4)
    mine = peer.export()
    handles = [None] * world
    if world > 1:
        dist.all_gather_object(handles, mine)
    else:
        handles = [mine]
    peer.import_handles(handles)
    npast = torch.full((1,), N0, dtype=torch.int32, device=dev)
    epoch = torch.ones(1, dtype=torch.int32, device=dev)
    st = torch.cuda.Stream(device=dev)
    max_err = 0.0
    for i in range(STEPS):
        dq = td(q[i][:, :, q_lo:q_lo + nh_l])                       # [L, 1, nh_l, HD]
        dk = [td(rows[l][0][N0 + i:N0 + i + 1, kv_lo * HD:(kv_lo + nkv_l) * HD]) for l in range(L)]
        dv = [td(rows[l][1][N0 + i:N0 + i + 1, kv_lo * HD:(kv_lo + nkv_l) * HD]) for l in range(L)]
        with torch.cuda.stream(st):
            for l in range(L):
                kv.attn_append_at_peer(l, dq[l], dk[l], dv[l], npast, N0 + STEPS + 4, 1 / np.sqrt(HD), peer,
                                       q_lo, NH, l, l - 1, epoch, stream=st)
            peer.wait(L - 1, epoch, nkv_l * world, stream=st)
            sv.counter_add(epoch, 1, stream=st)
            sv.counter_add(npast, 1, stream=st)
        st.synchronize()
        for l in range(L):
            got = peer.slot(l, (1, NH, HD)).cpu().numpy()
            k, v = rows[l]
            ref = orc.attn(orc.f16_to_f32(q[i][l]), k[:N0 + i + 1], v[:N0 + i + 1], orc.TYPE_F16, NKV, HD,
                           N0 + i + 1, 1 / np.sqrt(HD), orc.MASK_CAUSAL, N0 + i)
            max_err = max(max_err, float(np.abs(got - ref).max()))
        if world > 1:
            dist.barrier()
    flags = kv.error_flags()
    if world > 1:
        dist.barrier()
    peer.free()
    kv.free()
    if world > 1:
        dist.destroy_process_group()
    result[rank] = (max_err, flags)


@pytest.mark.parametrize("shape", [SHORT, LONG1], ids=["short", "long_few_heads"])
def test_peer_gather_single_rank(shape):
    res = {}
    _run_rank(0, 1, 0, res, shape)
    err, flags = res[0]
    assert flags == 0
    assert err <= 2e-3


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("shape", [SHORT, LONG2], ids=["short", "long"])
def test_peer_gather_two_ranks(shape):
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    res = mgr.dict()
    procs = [ctx.Process(target=_run_rank, args=(r, 2, port, res, shape)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    for r in range(2):
        err, flags = res[r]
        assert flags == 0
        assert err <= 2e-3
