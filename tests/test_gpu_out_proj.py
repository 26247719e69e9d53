"""The head-sharded output projection with the sum over ranks fused in (sv_out_proj_peer), against a
float64 matrix product of the whole projection (qwen3vl_model.cpp:664-667, mul_mat(L.o, attn)).

world = 1 runs in-process (the partial goes to the rank's own slot); world = 2 runs two spawned
processes, one per GPU, when two GPUs are visible: each rank holds half of the heads, and both
must end with the full product, bitwise equal between the ranks.  Tolerance: relative 1e-5 of
the row norm (f16 weights and inputs are exact; f32 accumulation).  NVLS is off.  Both exchange
forms run: slots with room for a 64-bit (value, epoch) word per partial (no counters) and slots of
f32 partials with per-band counters.
"""
import os
import socket

import numpy as np
import pytest
import torch

from __graft_entry__ import load_package

pytestmark = pytest.mark.gpu
NH, HD, D, STEPS = 32, 128, 2560, 3


def _data(T):
    rng = np.random.default_rng(41)
    x = [rng.standard_normal((T, NH * HD)).astype(np.float16) for _ in range(STEPS)]
    w = (rng.standard_normal((D, NH * HD)) * 0.02).astype(np.float16)
    return x, w


def _run_rank(rank, world, port, T, result, ll=True):
    import torch.distributed as dist
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    sv = load_package()
    torch.cuda.set_device(rank)
    dev = torch.device(f"cuda:{rank}")
    if world > 1:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    x, w = _data(T)
    K = NH * HD
    kl = K // world
    peer = sv.Peer(rank, rank, world, 2, world * T * D * (8 if ll else 4))
    mine = peer.export()
    handles = [None] * world
    if world > 1:
        dist.all_gather_object(handles, mine)
    else:
        handles = [mine]
    peer.import_handles(handles)
    wd = torch.from_numpy(w).to(dev)
    epoch = torch.ones(1, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    st = torch.cuda.Stream(device=dev)
    outs = []
    for i in range(STEPS):
        # one step = two layers (slots 0 and 1, each used once per epoch), then the epoch advances
        with torch.cuda.stream(st):
            for layer in range(2):
                xi = x[i] if layer == 0 else x[(i + 1) % STEPS]
                xd = torch.from_numpy(np.ascontiguousarray(xi[:, rank * kl:(rank + 1) * kl])).to(dev)
                outs.append((xi, peer.out_proj(xd, wd, rank * kl, layer, epoch, err=err, stream=st)))
            sv.counter_add(epoch, 1, stream=st)
        st.synchronize()
    errs = []
    for xi, o in outs:
        ref = xi.astype(np.float64) @ w.astype(np.float64).T
        errs.append(float(np.abs(o.cpu().numpy() - ref).max() / np.abs(ref).max()))
    outs = [o.cpu().numpy() for _, o in outs]
    if world > 1:
        dist.barrier()
    peer.free()
    if world > 1:
        dist.destroy_process_group()
    result[rank] = (max(errs), int(err.item()), [o.tobytes() for o in outs])


@pytest.mark.parametrize("T", [1, 5])
@pytest.mark.parametrize("ll", [True, False])
def test_out_proj_single_rank(T, ll):
    res = {}
    _run_rank(0, 1, 0, T, res, ll)
    err, flags, _ = res[0]
    assert flags == 0
    assert err <= 1e-5


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("ll", [True, False])
def test_out_proj_two_ranks(ll):
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    res = mgr.dict()
    procs = [ctx.Process(target=_run_rank, args=(r, 2, port, 1, res, ll)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    for r in range(2):
        err, flags, _ = res[r]
        assert flags == 0
        assert err <= 1e-5
    assert res[0][2] == res[1][2]          # every rank sums in rank order: identical bits


def test_out_proj_wait_expires_and_reports():
    """The cross-rank wait is bounded: with the epoch set one step ahead nothing can reach the target
    count (a flag nothing sets), so every CTA gives up after the 2 s limit, the timeout bit reaches
    the host, and the context stays usable (a fresh peer group then computes the right product)."""
    sv = load_package()
    dev = torch.device("cuda:0")
    x, w = _data(1)
    xd = torch.from_numpy(x[0]).to(dev)
    wd = torch.from_numpy(w).to(dev)
    peer = sv.Peer(0, 0, 1, 1, D * 4)
    peer.import_handles([peer.export()])
    epoch = torch.full((1,), 2, dtype=torch.int32, device=dev)      # the first call is epoch 1
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    peer.out_proj(xd, wd, 0, 0, epoch, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) & sv.DEVERR_TIMEOUT
    peer.free()
    fresh = sv.Peer(0, 0, 1, 1, D * 4)
    fresh.import_handles([fresh.export()])
    epoch.fill_(1)
    out = fresh.out_proj(xd, wd, 0, 0, epoch).cpu().numpy()
    ref = x[0].astype(np.float64) @ w.astype(np.float64).T
    assert np.abs(out - ref).max() <= 1e-5 * np.abs(ref).max()
    fresh.free()
