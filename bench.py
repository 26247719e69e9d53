#!/usr/bin/env python3
"""Benchmark of the KV-cache hot path (BASELINE metric: decode attention tokens/s,
KV GB/s against HBM, prefill attention TFLOP/s; 1..8 GPUs).

Workload (the metric's configuration that fits one GPU):
the Qwen3-VL-4B text geometry -- 36 layers, 32 query / 8 KV heads, head_dim 128,
f16 KV cache of 8192 rows.  Turn 1 fills 4096 rows per layer (untimed); turn
2's prompt strictly extends turn 1, so the splice predicate holds and only the
384-token tail is chunk-prefilled against the 4096 cached rows (timed
separately -> prefill TFLOP/s); then decode steps run.  One *step* is one
decode token through all 36 layers: per layer the K/V append of the new row
and the causal GQA attention over the whole cache.  With the default
--steps 128 the timed steps are exactly config 2's 128 decode steps
(S = 4481 .. 4608).  Inputs are synthetic N(0,1) f16 from a seeded torch CUDA
generator (seed 1); every decode step reads ~670 MB of K/V, larger than the
126 MB L2, so no flush is needed between steps.

On N GPUs (torchrun, one rank per GPU) every rank serves its own independent
session (sessions shard across GPUs; no collective on the data path), so
scaling is weak and value = N * steps / max-over-ranks time.

--impl reference times the CPU implementation of the same path on the host
cores (the C restatement of the reference's ggml CPU semantics in oracle/;
the reference's ggml is not vendored and cannot be built here) for the same
metric.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

L, NH, NKV, HD, CAP = 36, 32, 8, 128, 8192
PRE, TAIL, DEC = 4096, 384, 128
SEED = 1
SCALE = 1.0 / np.sqrt(HD)
METRIC = "decode attn tokens/s & KV GB/s vs 8 TB/s; prefill attn TFLOP/s; 1/2/4/8 GPU"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=DEC)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="svkv", choices=["svkv", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-batched", action="store_true", help="skip the config-5 multi-session leg")
    ap.add_argument("--no-longctx", action="store_true", help="skip the 131072-token kv-head-sharded leg")
    ap.add_argument("--gather", default="peer", choices=["peer", "nccl", "outproj"],
                    help="longctx: how each layer's head outputs reach every rank")
    ap.add_argument("--exchange", default="words", choices=["words", "counters"],
                    help="--workload outproj: partials as 64-bit (value, epoch) words, or f32 with band counters")
    ap.add_argument("--shards", type=int, default=None,
                    help="--workload longctx on one GPU: run rank 0's shard of an N-way kv-head split alone")
    ap.add_argument("--workload", default="cfg2", choices=["cfg2", "longctx", "kernels", "outproj"],
                    help="cfg2: the headline line; longctx: one 131072-token session sharded by kv head; "
                         "kernels: one small launch set of every kernel (for ncu captures)")
    return ap.parse_args()


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def profile_traffic(name: str):
    """Per-launch DRAM bytes from a committed ncu summary (profiles/<name>.md), if present."""
    path = os.path.join(ROOT, "profiles", name + ".md")
    try:
        for line in open(path):
            if line.strip().startswith("traffic_bytes_per_launch:"):
                return float(line.split(":", 1)[1])
    except OSError:
        pass
    return None


def decode_attn_bytes(S: int) -> int:
    """Algorithmic bytes of one decode-attention launch: K and V rows of every kv head + Q + O."""
    return S * NKV * HD * 2 * 2 + NH * HD * 2 + NH * HD * 4


def append_bytes(n_rows: int) -> int:
    return n_rows * NKV * HD * 2 * 2 * 2      # read K+V source, write K+V cache


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """NVML SM clock + throttle reasons sampled in a thread during the timed region."""

    def __init__(self, device_index: int):
        self.samples = []
        self.stop_ev = threading.Event()
        self.ok = False
        self.max_mhz = None
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            self.h = None
            uuid = getattr(torch.cuda.get_device_properties(device_index), "uuid", None)
            if uuid is not None:
                try:
                    self.h = pynvml.nvmlDeviceGetHandleByUUID(f"GPU-{uuid}")
                except Exception:
                    self.h = None
            if self.h is None:
                cvd = os.environ.get("CUDA_VISIBLE_DEVICES", "")
                ids = [c for c in cvd.split(",") if c.strip().isdigit()]
                idx = int(ids[device_index]) if device_index < len(ids) else device_index
                self.h = pynvml.nvmlDeviceGetHandleByIndex(idx)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.reasons_fn = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
            self.nv = pynvml
            self.ok = True
        except Exception:
            self.ok = False

    def _run(self):
        nv = self.nv
        while not self.stop_ev.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
                rs = self.reasons_fn(self.h)
                self.samples.append((mhz, rs))
            except Exception:
                pass
            time.sleep(0.005)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        if self.ok:
            self.stop_ev.set()
            self.t.join()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"], "samples": 0}
        nv = self.nv
        names = {
            "sw_power_cap": getattr(nv, "nvmlClocksEventReasonSwPowerCap", 0x4),
            "hw_slowdown": getattr(nv, "nvmlClocksEventReasonHwSlowdown", 0x8),
            "sw_thermal_slowdown": getattr(nv, "nvmlClocksEventReasonSwThermalSlowdown", 0x20),
            "hw_thermal_slowdown": getattr(nv, "nvmlClocksEventReasonHwThermalSlowdown", 0x40),
            "hw_power_brake_slowdown": getattr(nv, "nvmlClocksEventReasonHwPowerBrakeSlowdown", 0x80),
        }
        seen = set()
        for _, rs in self.samples:
            for n, bit in names.items():
                if rs & bit:
                    seen.add(n)
        mhz = [m for m, _ in self.samples]
        return {"sm_mhz": float(np.median(mhz)), "sm_max_mhz": self.max_mhz, "reasons": sorted(seen),
                "samples": len(mhz)}


# ------------------------------------------------------------------ distributed plumbing
def dist_setup(args):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device(f"cuda:{local}"))
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------ CPU path (oracle restatement)
def cfg2_config(world: int) -> dict:
    """The `config` of the headline line, identical in both arms (same workload, same sessions)."""
    return {
        "workload": "BASELINE config 2: 36 layers, 32q/8kv, HD 128, f16 KV cap 8192; turn 2 splices a 384-token "
                    "tail onto 4096 cached rows, then decode steps at S = 4481..",
        "sessions_per_gpu": 1,
        "sessions": world,
        "step": "one decode token through 36 layers (K/V append + causal GQA attention per layer) for every session",
        "l2": "inputs larger than L2 (each step reads ~670 MB of K/V per session)",
        "parallelism": f"{world} session(s), one per GPU, no data-path collective",
    }


def host_threads() -> int:
    """Host threads this process may use (its CPU affinity), whatever OMP_NUM_THREADS says."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_decode_sample(n_sessions: int, n_tokens: int, warmup: int = 0, seed: int = SEED):
    """Config 2 decode on the host: every token of every session goes through all 36 layers (the
    oracle's set_rows of the new K and V rows + flash-attention restatement, OpenMP over every host
    thread of this process).  Each session has its own caches holding turn 1 + the splice tail
    (4480 rows per layer); the first `warmup` tokens are untimed.  Returns (seconds for the timed
    n_sessions * n_tokens session-tokens, thread count)."""
    from oracle import oracle as orc
    orc.set_num_threads(host_threads())
    ne0 = NKV * HD
    n0 = PRE + TAIL
    rows = n0 + warmup + n_tokens
    assert rows <= CAP
    base = []
    for layer in range(L):
        k = np.zeros((rows, ne0 * 2), np.uint8)
        v = np.zeros((rows, ne0 * 2), np.uint8)
        k[:n0] = orc.normal_f16(seed, 10 + layer, n0 * ne0).view(np.uint8).reshape(n0, -1)
        v[:n0] = orc.normal_f16(seed, 90 + layer, n0 * ne0).view(np.uint8).reshape(n0, -1)
        base.append((k, v))
    sessions = [base] + [[(k.copy(), v.copy()) for k, v in base] for _ in range(n_sessions - 1)]
    n_all = warmup + n_tokens
    qs = [orc.f16_to_f32(orc.normal_f16(seed, 500 + i, L * NH * HD)).reshape(L, 1, NH, HD) for i in range(n_all)]
    ks = [orc.normal_f16(seed, 700 + i, L * ne0).reshape(L, 1, ne0) for i in range(n_all)]
    vs = [orc.normal_f16(seed, 900 + i, L * ne0).reshape(L, 1, ne0) for i in range(n_all)]

    def token(i):
        n_past = n0 + i
        for caches in sessions:
            for layer in range(L):
                k, v = caches[layer]
                orc.set_rows(k, orc.TYPE_F16, ne0, ks[i][layer], orc.TYPE_F16, base=n_past)
                orc.set_rows(v, orc.TYPE_F16, ne0, vs[i][layer], orc.TYPE_F16, base=n_past)
                orc.attn(qs[i][layer], k, v, orc.TYPE_F16, NKV, HD, n_past + 1, SCALE, orc.MASK_CAUSAL, n_past)

    for i in range(warmup):
        token(i)
    t0 = time.perf_counter()
    for i in range(warmup, n_all):
        token(i)
    return time.perf_counter() - t0, orc.num_threads()


def run_reference(args, world, rank):
    """The reference arm: the CPU path (the oracle port: the reference's ggml is not vendored and
    cannot be built here), rank 0 only, on the same work as the GPU arm -- `world` sessions of config
    2, every timed step one decode token through all 36 layers of every session -- with all the host
    threads it can use."""
    if rank != 0:
        return
    from oracle import oracle as orc
    orc.build()
    K, W = args.steps, max(1, args.warmup)
    dt, cores = cpu_decode_sample(world, K, warmup=W)
    step_s = dt / K
    value = world * K / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": K, "warmup": W, "ms_per_step": step_s * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": cfg2_config(world),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"{K} timed decode tokens (after {W} untimed) of {world} session(s), all 36 "
                                   f"layers each, S = {PRE + TAIL + W + 1}..{PRE + TAIL + W + K}; no extrapolation"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU path
def run_svkv(args, world, rank, local):
    import torch
    from __graft_entry__ import load_package
    sv = load_package()
    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    stream = torch.cuda.Stream(device=dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(SEED * 1000 + rank)
    K, W = args.steps, args.warmup
    if PRE + TAIL + max(K, W) > CAP:
        raise SystemExit(f"steps beyond the {CAP}-row cache")

    kv = sv.KvCache()
    if not kv.alloc(local, L, NKV, HD, CAP):
        raise SystemExit("KvCache.alloc failed")

    def randn(*shape):
        return torch.randn(*shape, generator=gen, device=dev, dtype=torch.float32).to(torch.float16)

    ne0 = NKV * HD
    launches = 0
    with torch.cuda.stream(stream):
        # ---- turn 1: 4096 rows per layer
        for layer in range(L):
            kv.append(layer, randn(PRE, ne0), randn(PRE, ne0), base=0, stream=stream)
        ids1 = np.arange(PRE, dtype=np.int32) % 151000
        ids2 = np.concatenate([ids1, (np.arange(TAIL, dtype=np.int32) * 7) % 151000])
        skip = sv.can_splice(ids1, PRE, ids2)          # turn 2 strictly extends turn 1
        assert skip == PRE

        # ---- turn 2 tail: chunked prefill of 384 rows against the 4096 cached
        tq = [randn(TAIL, NH, HD) for _ in range(L)]
        tk = [randn(TAIL, ne0) for _ in range(L)]
        tv = [randn(TAIL, ne0) for _ in range(L)]
        tout = torch.empty(TAIL, NH, HD, dtype=torch.float32, device=dev)

        def tail_pass():
            for layer in range(L):
                kv.append(layer, tk[layer], tv[layer], base=skip, stream=stream)
                kv.attn(layer, tq[layer], n_past=skip, scale=SCALE, out=tout, stream=stream)

        tail_pass()
        stream.synchronize()
        reps = 3
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            tail_pass()
        e1.record(stream)
        e1.synchronize()
        prefill_ms = e0.elapsed_time(e1) / reps
        vis = TAIL * skip + TAIL * (TAIL + 1) // 2
        prefill_flop = 4.0 * NH * HD * vis * L
        prefill_tflops = prefill_flop / (prefill_ms * 1e-3) / 1e12

        # ---- decode: one CUDA graph per step, replayed; n_past lives on the device
        n0 = PRE + TAIL
        max_keys = n0 + max(K, W) + 1
        npast = torch.full((1,), n0, dtype=torch.int32, device=dev)
        # the step's inputs live in one device buffer, packed per layer (Q_l, K_l, V_l), so the
        # end-to-end leg moves any run of layers with one host-to-device copy
        PER = NH * HD + 2 * ne0
        dqkv = randn(L * PER)
        dq = dqkv.as_strided((L, 1, NH, HD), (PER, NH * HD, HD, 1))
        dk = dqkv.as_strided((L, 1, ne0), (PER, ne0, 1), NH * HD)
        dvv = dqkv.as_strided((L, 1, ne0), (PER, ne0, 1), NH * HD + ne0)
        dout = torch.empty(L, 1, NH, HD, dtype=torch.float32, device=dev)

        def step():
            # per layer: the fused append + attention kernel (one launch), then the n_past advance
            for layer in range(L):
                kv.attn_append_at(layer, dq[layer], dk[layer], dvv[layer], npast, max_keys, SCALE, out=dout[layer],
                                  stream=stream)
            sv.counter_add(npast, 1, stream=stream)

        step()                                     # eager run before capture (sets kernel attributes)
        stream.synchronize()
        npast.fill_(n0)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            step()
        stream.synchronize()
        for _ in range(W):
            g.replay()
        stream.synchronize()
        npast.fill_(n0)
        # clock settle (untimed) so the sampled clocks reflect steady load
        for _ in range(20):
            g.replay()
            npast.fill_(n0)
        stream.synchronize()
        barrier(world)
        torch.cuda.synchronize()
        with ClockSampler(local) as clk:
            e0.record(stream)
            for _ in range(K):
                g.replay()
            e1.record(stream)
            e1.synchronize()
            torch.cuda.synchronize()
        barrier(world)
        dec_ms = e0.elapsed_time(e1)
        launches = K * (L + 1)
        assert int(npast.item()) == n0 + K
        check_flags(kv, stream)
        S_steps = [n0 + i + 1 for i in range(K)]
        step_bytes = sum(L * (decode_attn_bytes(S) + append_bytes(1)) for S in S_steps) / K

        # ---- the decode-attention kernel alone: 36 launches per replay (roofline)
        npast.fill_(n0 + K // 2)
        ga = torch.cuda.CUDAGraph()
        with torch.cuda.graph(ga, stream=stream):
            for layer in range(L):
                kv.attn_append_at(layer, dq[layer], dk[layer], dvv[layer], npast, max_keys, SCALE, out=dout[layer],
                                  stream=stream)
        for _ in range(3):
            ga.replay()
        stream.synchronize()
        ra = 20
        e0.record(stream)
        for _ in range(ra):
            ga.replay()
        e1.record(stream)
        e1.synchronize()
        attn_launch_ms = e0.elapsed_time(e1) / (ra * L)
        S_mid = n0 + K // 2 + 1
        attn_launch_bytes = decode_attn_bytes(S_mid) + append_bytes(1)
        attn_gbs = attn_launch_bytes / (attn_launch_ms * 1e-3) / 1e9

        # ---- end to end: every step copies that step's Q/K/V (36 layers) from pinned host memory to the
        #      device, runs the 36 layers, copies the attention output back to pinned host memory and waits
        #      for it on the host.  The copies are captured into the step's CUDA graph, one copy per run of
        #      layers: layers 0-3's inputs on the compute stream ahead of layer 0, layers 4-35's on a second
        #      stream while layers 0-3 run (~20 GB/s host to device here: the rest lands before layer 4),
        #      layers 0-31's outputs on the second stream while layers 32-35 run, layers 32-35's after the
        #      chain.  Every byte crosses PCIe in every step.  Each cross-stream join in the kernel chain
        #      costs a few us (the kernel after it starts without its programmatic early launch), so the
        #      chain has one join for the inputs and none for the outputs.  Measured per step: 259-262 us;
        #      more, smaller chunks (more joins) 263-269 us; every copy outside the chain 271-281 us; the
        #      inputs as separate Q, K, V copies of layers 0-1 and 2-35, 267-287 us.
        hqkv = torch.empty((L * PER,), dtype=torch.float16).pin_memory()       # one step's Q, K, V per layer
        hqkv.copy_(torch.randn(hqkv.shape, generator=torch.Generator().manual_seed(SEED)).half())
        hout = torch.empty((L, 1, NH, HD), dtype=torch.float32).pin_memory()
        hlay, dlay = hqkv.view(L, PER), dqkv.view(L, PER)
        cs = torch.cuda.Stream(device=dev)
        L_IN, L_OUT = 4, L - 4          # inputs [0, L_IN) on the compute stream; outputs [0, L_OUT) early

        def e2e_step():
            ev_in1 = torch.cuda.Event()
            ev_mid, ev_out0 = torch.cuda.Event(), torch.cuda.Event()
            dlay[:L_IN].copy_(hlay[:L_IN], non_blocking=True)
            cs.wait_stream(stream)
            with torch.cuda.stream(cs):
                dlay[L_IN:].copy_(hlay[L_IN:], non_blocking=True)
                ev_in1.record(cs)
            for layer in range(L):
                if layer == L_IN:
                    stream.wait_event(ev_in1)
                if layer == L_OUT:
                    ev_mid.record(stream)
                    with torch.cuda.stream(cs):
                        cs.wait_event(ev_mid)
                        hout[:L_OUT].copy_(dout[:L_OUT], non_blocking=True)
                        ev_out0.record(cs)
                kv.attn_append_at(layer, dq[layer], dk[layer], dvv[layer], npast, max_keys, SCALE, out=dout[layer],
                                  stream=stream)
            sv.counter_add(npast, 1, stream=stream)
            hout[L_OUT:].copy_(dout[L_OUT:], non_blocking=True)
            stream.wait_event(ev_out0)

        npast.fill_(n0)
        stream.synchronize()
        ge = torch.cuda.CUDAGraph()
        with torch.cuda.graph(ge, stream=stream):
            e2e_step()
        stream.synchronize()
        for _ in range(2):
            ge.replay()
            stream.synchronize()
        npast.fill_(n0)
        stream.synchronize()
        barrier(world)
        e0.record(stream)
        for i in range(K):
            ge.replay()
            stream.synchronize()
        e1.record(stream)
        e1.synchronize()
        barrier(world)
        e2e_ms = e0.elapsed_time(e1)
        h2d = hqkv.numel() * 2
        d2h = hout.numel() * 4
        assert np.isfinite(hout.numpy()).all()
        check_flags(kv, stream)
        # ---- parity of the timed kernel (outside every timed region): one more fused decode of the last
        #      layer at the next row, against the CPU oracle over the same cache
        check = decode_check(kv, L - 1, dq[L - 1], dk[L - 1], dvv[L - 1], npast, max_keys, stream)

    dec_ms_max = max_over_ranks(dec_ms, world)
    check_max_abs = max_over_ranks(check["max_abs"], world)
    e2e_ms_max = max_over_ranks(e2e_ms, world)
    prefill_ms_max = max_over_ranks(prefill_ms, world)
    clocks = clk.summary()
    kv.free()
    del kv
    torch.cuda.empty_cache()
    batched = None if args.no_batched else run_batched(sv, dev, stream, rank, world, K, W)
    # the path with a data-path exchange: one 131072-token session sharded by kv head over the same GPUs
    longctx = None if args.no_longctx else longctx_leg(sv, world, rank, local, K, max(3, W))
    # the same session with each layer's attention followed by the row-parallel output projection, the
    # rank sum fused into it (one exchange per layer, no all-gather of the attention rows)
    longctx_proj = None if args.no_longctx else longctx_leg(sv, world, rank, local, K, max(3, W), gather="outproj")
    extras = {}
    if world == 1 and not args.no_batched:
        for name, fn in (("config1", run_cfg1), ("config3_eviction", run_cfg3), ("config4_q8_0", run_cfg4),
                         ("qk_norm_rope_append", run_rope)):
            try:
                extras[name] = fn(sv, dev, stream)
            except Exception as ex:          # an extra leg never takes the headline line down
                extras[name] = {"error": f"{type(ex).__name__}: {ex}"}
    if rank != 0:
        return

    hbm, tflops_peak, peak_kind = measured_peaks()
    value = world * K / (dec_ms_max * 1e-3)
    traffic = profile_traffic("decode_attn_cfg2")
    line = {
        "metric": METRIC,
        "value": value,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": K,
        "warmup": W,
        "ms_per_step": dec_ms_max / K,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f16",
        "data": "synthetic",
        "config": cfg2_config(world),
        "kv_gbs": world * step_bytes / (dec_ms_max / K * 1e-3) / 1e9,
        "prefill": {
            "tflops": world * prefill_flop / (prefill_ms_max * 1e-3) / 1e12,
            "ms_per_turn": prefill_ms_max,
            "work": "384-token tail vs 4096 cached rows, 36 layers, 4*NH*HD*sum(visible) = %.3f TFLOP" % (prefill_flop / 1e12),
            "frac_of_bf16_peak": prefill_tflops / tflops_peak,
        },
        "roofline": {
            "kernel": "fa_decode_gqa_kernel<128> fused append + attention (sv_attn_append_at)",
            "bound": "hbm",
            "achieved": attn_gbs,
            "peak": hbm,
            "unit": "GB/s",
            "frac": attn_gbs / hbm,
            "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)",
            "bytes_per_launch": attn_launch_bytes,
            "launch_us": attn_launch_ms * 1e3,
            "traffic": traffic,
        },
        "e2e": {"value": world * K / (e2e_ms_max * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "how": "per step, one CUDA graph: pinned H2D of 36 layers' Q/K/V (layers 4-35 overlapping layers "
                       "0-3), the 36 layers, D2H of the attention output (layers 0-31 overlapping layers 32-35); "
                       "host waits for it"},
        "gpu_launches": launches,
        "clocks": clocks,
        "decode_check_max_abs": check_max_abs,
        "decode_check": dict(check, max_abs=check_max_abs,
                             gate="max-abs <= 2e-3 and rel-L2 <= 1e-3 vs the fp32-accumulated CPU oracle; "
                                  "appended K/V rows bit-exact; max-abs is the max over ranks"),
    }
    if batched is not None:
        line["batched"] = batched
    if longctx is not None:
        line["longctx"] = longctx
    if longctx_proj is not None:
        line["longctx_proj"] = longctx_proj
    line.update(extras)
    if world == 1 and not args.no_cpu_baseline:
        n_tok = max(K, 64)
        dt, cores = cpu_decode_sample(1, n_tok, warmup=2)
        line["cpu_baseline"] = {
            "value": n_tok / dt, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"{n_tok} decode tokens (after 2 untimed) of one config 2 session through all 36 layers, "
                      f"S = {PRE + TAIL + 3}..{PRE + TAIL + 2 + n_tok}; no extrapolation",
        }
    print(json.dumps(line), flush=True)


def cfg5_shards(n_gpus: int = 8):
    """64 session lengths U[512, 32768] (numpy default_rng(4)), balanced over
    n_gpus by longest-first greedy assignment on total context."""
    lens = np.random.default_rng(4).integers(512, 32769, 64)
    order = np.argsort(-lens, kind="stable")
    loads = [0] * n_gpus
    shards = [[] for _ in range(n_gpus)]
    for i in order:
        g = int(np.argmin(loads))
        shards[g].append(int(i))
        loads[g] += int(lens[i])
    return lens, shards


def run_batched(sv, dev, stream, rank, world, K, W):
    """Config-5 multi-session decode: this GPU's eighth of the 64 sessions (8 sessions, ~150k cached
    rows, ~22 GB of K/V over 36 layers) in one shared cache with per-session slot ranges; each step
    appends one row per session and runs the windowed attention for all sessions per layer
    (vc3_batch.inc's batched step), captured once as a CUDA graph.  Weak scaling: every rank serves
    its own shard (rank r takes shard r mod 8)."""
    import torch
    lens, shards = cfg5_shards(8)
    mine = shards[rank % 8]
    ctx = [int(lens[i]) for i in mine]
    n = len(ctx)
    room = K + W + 64
    caps = [c + room for c in ctx]
    base = np.concatenate([[0], np.cumsum(caps)[:-1]]).astype(np.int32)
    n_ctx = int(sum(caps))
    kv = sv.KvCache()
    if not kv.alloc(dev.index, L, NKV, HD, n_ctx):
        raise SystemExit("KvCache.alloc failed (config 5 shard)")
    gen = torch.Generator(device=dev)
    gen.manual_seed(4000 + rank)
    with torch.cuda.stream(stream):
        for layer in range(L):
            for isv in (0, 1):
                kv.tensor(layer, isv).view(torch.float16).normal_(generator=gen)
        lo = torch.tensor(base, dtype=torch.int32, device=dev)
        own0 = lo + torch.tensor(ctx, dtype=torch.int32, device=dev)
        own = own0.clone()
        hi = own + 1
        q = torch.randn(L, n, NH, HD, generator=gen, device=dev).half()
        knew = torch.randn(L, n, NKV * HD, generator=gen, device=dev).half()
        vnew = torch.randn(L, n, NKV * HD, generator=gen, device=dev).half()
        out = torch.empty(L, n, NH, HD, dtype=torch.float32, device=dev)
        max_span = max(ctx) + room

        def reset():
            own.copy_(own0)
            hi.copy_(own0 + 1)

        def step():
            for layer in range(L):
                kv.append(layer, knew[layer], vnew[layer], rows=own, stream=stream)
                kv.attn_window(layer, q[layer], lo, hi, own, max_span, SCALE, out=out[layer], stream=stream)
            sv.counter_add(hi, 1, stream=stream)
            sv.counter_add(own, 1, stream=stream)

        step()
        stream.synchronize()
        reset()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            step()
        for _ in range(W):
            g.replay()
        reset()
        stream.synchronize()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(K):
            g.replay()
        e1.record(stream)
        e1.synchronize()
        barrier(world)
        ms = e0.elapsed_time(e1)
        check_flags(kv, stream)
        # the windowed attention kernel alone (36 launches per replay) at the middle step
        own.copy_(own0 + K // 2)
        hi.copy_(own + 1)
        ga = torch.cuda.CUDAGraph()
        with torch.cuda.graph(ga, stream=stream):
            for layer in range(L):
                kv.attn_window(layer, q[layer], lo, hi, own, max_span, SCALE, out=out[layer], stream=stream)
        ga.replay()
        stream.synchronize()
        ra = 5
        e0.record(stream)
        for _ in range(ra):
            ga.replay()
        e1.record(stream)
        e1.synchronize()
        attn_ms = e0.elapsed_time(e1) / (ra * L)
    ms_max = max_over_ranks(ms, world)
    kv.free()
    row_b = NKV * HD * 2 * 2                     # K + V bytes of one cached row
    step_bytes = sum(L * ((c + i + 1) * row_b + NH * HD * 6) for c in ctx for i in range(K)) / K + L * n * append_bytes(1)
    attn_bytes = sum((c + K // 2 + 1) * row_b + NH * HD * 6 for c in ctx)
    hbm, _, peak_kind = measured_peaks()
    return {
        "workload": f"BASELINE config 5 shard: {n} of 64 sessions per GPU (ctx {min(ctx)}..{max(ctx)}, "
                    f"sum {sum(ctx)}), 36 layers, 32q/8kv HD 128 f16, one shared cache with slot ranges",
        "tokens_per_s": world * n * K / (ms_max * 1e-3),
        "ms_per_step": ms_max / K,
        "kv_gbs": world * step_bytes / (ms_max / K * 1e-3) / 1e9,
        "roofline": {"kernel": "fa_decode_kernel<128, f16> window mode (sv_attn_window)", "bound": "hbm",
                     "achieved": attn_bytes / (attn_ms * 1e-3) / 1e9, "peak": hbm, "unit": "GB/s",
                     "frac": attn_bytes / (attn_ms * 1e-3) / 1e9 / hbm,
                     "peak_source": f"{peak_kind} hbm_gbs", "bytes_per_launch": attn_bytes,
                     "launch_us": attn_ms * 1e3},
        "gpu_launches": K * (2 * L + 2),
    }


def run_cfg1(sv, dev, stream):
    """one Qwen3-VL-4B-geometry layer (32q/8kv, HD 128, f16 cache of 4096 rows, seed
    0): append a 1024-token prefill and attend it causally (timed -> prefill TFLOP/s), then 64 decode
    steps at S = 1025..1088, each one fused append + attention launch and the n_past advance, captured
    once as a CUDA graph and replayed.  One layer moves ~4.35 MB per step (~0.7 us of HBM time), so a
    step is bound by launch and dependency latency, not by HBM."""
    import torch
    P, DEC1, CAP1 = 1024, 64, 4096
    kv = sv.KvCache()
    assert kv.alloc(dev.index, 1, NKV, HD, CAP1)
    gen = torch.Generator(device=dev)
    gen.manual_seed(0)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        kp = torch.randn(P, NKV * HD, generator=gen, device=dev).half()
        vp = torch.randn(P, NKV * HD, generator=gen, device=dev).half()
        qp = torch.randn(P, NH, HD, generator=gen, device=dev).half()
        out = torch.empty(P, NH, HD, dtype=torch.float32, device=dev)

        def prefill():
            kv.append(0, kp, vp, base=0, stream=stream)
            kv.attn(0, qp, n_past=0, scale=SCALE, out=out, stream=stream)

        prefill()
        stream.synchronize()
        reps = 10
        e0.record(stream)
        for _ in range(reps):
            prefill()
        e1.record(stream)
        e1.synchronize()
        pre_ms = e0.elapsed_time(e1) / reps
        pre_flop = 4.0 * NH * HD * (P * (P + 1) // 2)
        q1 = torch.randn(DEC1, 1, NH, HD, generator=gen, device=dev).half()
        k1 = torch.randn(DEC1, 1, NKV * HD, generator=gen, device=dev).half()
        v1 = torch.randn(DEC1, 1, NKV * HD, generator=gen, device=dev).half()
        o1 = torch.empty(1, NH, HD, dtype=torch.float32, device=dev)
        npast = torch.full((1,), P, dtype=torch.int32, device=dev)
        qs, ks, vs = torch.empty_like(q1[0]), torch.empty_like(k1[0]), torch.empty_like(v1[0])

        def step():
            kv.attn_append_at(0, qs, ks, vs, npast, P + DEC1 + 1, SCALE, out=o1, stream=stream)
            sv.counter_add(npast, 1, stream=stream)

        step()
        stream.synchronize()
        npast.fill_(P)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            step()
        npast.fill_(P)
        stream.synchronize()
        # the step's inputs are staged by device copies outside the timed region: time the 64 replays
        # back to back with each step's rows already in place (one input set reused per replay)
        qs.copy_(q1[0]); ks.copy_(k1[0]); vs.copy_(v1[0])
        stream.synchronize()
        e0.record(stream)
        for _ in range(DEC1):
            g.replay()
        e1.record(stream)
        e1.synchronize()
        dec_ms = e0.elapsed_time(e1)
        check_flags(kv, stream)
        del g
    kv.free()
    dec_bytes = sum(decode_attn_bytes(P + i + 1) + append_bytes(1) for i in range(DEC1))
    return {
        "workload": "BASELINE config 1: 1 layer, 32q/8kv HD 128, f16 cache 4096; prefill 1024 then 64 decode "
                    "steps (S = 1025..1088), one CUDA graph per step",
        "prefill_tflops": pre_flop / (pre_ms * 1e-3) / 1e12,
        "prefill_us": pre_ms * 1e3,
        "decode_tokens_per_s": DEC1 / (dec_ms * 1e-3),
        "decode_us_per_step": dec_ms * 1e3 / DEC1,
        "decode_kv_gbs": dec_bytes / (dec_ms * 1e-3) / 1e9,
        "bound": "launch/dependency latency: ~4.35 MB per step is ~0.7 us of HBM time",
    }


def run_cfg3(sv, dev, stream):
    """streaming session with window eviction.  12 rounds of 16 frames x 64 rows +
    96 text rows (+32 answer rows decoded), window 6 rounds, 36 layers f16.  From round 7 the oldest
    round leaves the window and the cache is compacted in place (sv_session_begin_turn); the new
    round is chunk-prefilled after the survivors, then 32 decode steps append + attend."""
    import torch
    from oracle import oracle as orc
    rpf, frames, text, answer, rounds = 64, 16, 96, 32, 12
    round_rows = frames * rpf + text + answer
    kv = sv.KvCache()
    assert kv.alloc(dev.index, L, NKV, HD, 7 * round_rows + 64)
    sess = sv.Session(kv, max_frames=6 * frames, rows_per_frame=rpf)
    ref = orc.SessionRows(6 * frames, rpf)
    gen = torch.Generator(device=dev)
    gen.manual_seed(2)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    comp_ms, moved_bytes, prefill_ms, prefill_flop, decode_ms = 0.0, 0, 0.0, 0.0, 0.0
    q1 = torch.randn(L, 1, NH, HD, generator=gen, device=dev).half()
    k1 = torch.randn(L, 1, NKV * HD, generator=gen, device=dev).half()
    with torch.cuda.stream(stream):
        for r in range(rounds):
            rows_before = len(sess.rows())
            e0.record(stream)
            first, kept = sess.begin_turn(frames, stream=stream)
            e1.record(stream)
            e1.synchronize()
            ref.begin_turn(frames)
            if first < rows_before:                       # rows left: the survivors were compacted
                comp_ms += e0.elapsed_time(e1)
                moved = first                             # every surviving row moved down
                moved_bytes += moved * NKV * HD * 2 * 2 * L * 2
            n = kept * rpf + text
            kq = torch.randn(n, NKV * HD, generator=gen, device=dev).half()
            vq = torch.randn(n, NKV * HD, generator=gen, device=dev).half()
            qq = torch.randn(n, NH, HD, generator=gen, device=dev).half()
            out = torch.empty(n, NH, HD, dtype=torch.float32, device=dev)
            e0.record(stream)
            for layer in range(L):
                kv.append(layer, kq, vq, base=first, stream=stream)
                kv.attn(layer, qq, n_past=first, scale=SCALE, out=out, stream=stream)
            e1.record(stream)
            e1.synchronize()
            prefill_ms += e0.elapsed_time(e1)
            prefill_flop += 4.0 * NH * HD * (n * first + n * (n + 1) // 2) * L
            npast = torch.full((1,), first + n, dtype=torch.int32, device=dev)
            o1 = torch.empty(L, 1, NH, HD, dtype=torch.float32, device=dev)
            e0.record(stream)
            for _ in range(answer):
                for layer in range(L):
                    kv.attn_append_at(layer, q1[layer], k1[layer], k1[layer], npast, kv.n_ctx, SCALE, out=o1[layer],
                                      stream=stream)
                sv.counter_add(npast, 1, stream=stream)
            e1.record(stream)
            e1.synchronize()
            decode_ms += e0.elapsed_time(e1)
            sess.end_turn(kept, text, answer)
            ref.end_turn(kept, text, answer)
        assert np.array_equal(sess.rows(), ref.rows()), "kept-row set differs from the window rule"
        check_flags(kv, stream)
    kv.free()
    return {
        "workload": "BASELINE config 3: 12 rounds x (16 frames x 64 rows + 96 text + 32 answer rows), window 6 "
                    "rounds, 36 layers f16, in-place compaction from round 7",
        "kept_rows_match_window_rule": True,
        "compaction_gbs": moved_bytes / (comp_ms * 1e-3) / 1e9 if comp_ms > 0 else None,
        "compaction_ms_per_eviction": comp_ms / 6,
        "prefill_tflops": prefill_flop / (prefill_ms * 1e-3) / 1e12,
        "decode_tokens_per_s_eager": rounds * answer / (decode_ms * 1e-3),
    }


def run_cfg4(sv, dev, stream):
    """6 full-attention layers, 16q/4kv, HD 256, q8_0 cache (block-32 int8 + f16
    scale); K/V f16 N(0,1) with 1% of elements x8.  Prefill 8192 tokens in 512-token chunks (each chunk
    quantised into the cache, then attends causally), then 256 decode steps (one CUDA graph per step)."""
    import torch
    Lq, NHq, NKVq, HDq = 6, 16, 4, 256
    S0, CH, DEC4 = 8192, 512, 256
    scale = 1.0 / 16.0
    kv = sv.KvCache()
    assert kv.alloc(dev.index, Lq, NKVq, HDq, S0 + DEC4 + 64, sv.TYPE_Q8_0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(3)

    def kv_rows(n):
        x = torch.randn(n, NKVq * HDq, generator=gen, device=dev)
        x = torch.where(torch.rand(x.shape, generator=gen, device=dev) < 0.01, x * 8, x)
        return x.half()

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        chunks = [(kv_rows(CH), kv_rows(CH), torch.randn(CH, NHq, HDq, generator=gen, device=dev).half())
                  for _ in range(S0 // CH)]
        out = torch.empty(CH, NHq, HDq, dtype=torch.float32, device=dev)
        stream.synchronize()
        e0.record(stream)
        for c, (kc, vc, qc) in enumerate(chunks):
            for layer in range(Lq):
                kv.append(layer, kc, vc, base=c * CH, stream=stream)
                kv.attn(layer, qc, n_past=c * CH, scale=scale, out=out, stream=stream)
        e1.record(stream)
        e1.synchronize()
        pre_ms = e0.elapsed_time(e1)
        pre_flop = 4.0 * NHq * HDq * (S0 * (S0 + 1) // 2) * Lq
        npast = torch.full((1,), S0, dtype=torch.int32, device=dev)
        q1 = torch.randn(Lq, 1, NHq, HDq, generator=gen, device=dev).half()
        k1, v1 = kv_rows(Lq).view(Lq, 1, -1), kv_rows(Lq).view(Lq, 1, -1)
        o1 = torch.empty(Lq, 1, NHq, HDq, dtype=torch.float32, device=dev)
        max_keys = S0 + DEC4 + 1

        def step():
            for layer in range(Lq):
                kv.attn_append_at(layer, q1[layer], k1[layer], v1[layer], npast, max_keys, scale, out=o1[layer],
                                  stream=stream)
            sv.counter_add(npast, 1, stream=stream)

        step()
        stream.synchronize()
        npast.fill_(S0)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            step()
        npast.fill_(S0)
        stream.synchronize()
        e0.record(stream)
        for _ in range(DEC4):
            g.replay()
        e1.record(stream)
        e1.synchronize()
        dec_ms = e0.elapsed_time(e1)
        check_flags(kv, stream)
    del g
    kv.free()
    headb = HDq // 32 * 34
    dec_bytes = sum(Lq * ((S0 + i + 1) * NKVq * headb * 2 + NHq * HDq * 6) for i in range(DEC4))
    return {
        "workload": "BASELINE config 4: 6 layers, 16q/4kv HD 256, q8_0 cache, 1% outliers x8; 8192-token prefill in "
                    "512-token chunks, 256 decode steps",
        "prefill_tflops": pre_flop / (pre_ms * 1e-3) / 1e12,
        "prefill_ms": pre_ms,
        "prefill_kernel": "per chunk and layer: q8_0_split_kernel (visible rows -> f16 hi + lo planes), then "
                          "fa_prefill_kernel<256, 1, 2> (tcgen05/TMEM, both parts of K and V through the MMA)",
        "decode_tokens_per_s": DEC4 / (dec_ms * 1e-3),
        "decode_kv_gbs": dec_bytes / (dec_ms * 1e-3) / 1e9,
    }


def run_rope(sv, dev, stream):
    """The step before the append, fused (sv_qk_norm_rope_append): per-head q/k RMSNorm * weight,
    Qwen3-VL interleaved MRoPE (theta 5e6, sections 24/20/20/0, four position streams) and the K/V
    append, on config 2's geometry over 36 layers (one CUDA graph of 36 launches): the 384-token splice
    tail and one decode token.  HBM-bound; algorithmic bytes per launch = f32 q, k, v read + f16 q_out
    and K/V rows written."""
    import torch
    out = {"workload": "config 2 geometry (32q/8kv HD 128, f16 cache), 36 layers, IMROPE 24/20/20/0, eps 1e-6"}
    kv = sv.KvCache()
    assert kv.alloc(dev.index, L, NKV, HD, CAP)
    gen = torch.Generator(device=dev)
    gen.manual_seed(11)
    qn = 1.0 + 0.1 * torch.randn(HD, generator=gen, device=dev)
    kn = 1.0 + 0.1 * torch.randn(HD, generator=gen, device=dev)
    rope = (sv.ROPE_IMROPE, HD, 5e6, (24, 20, 20, 0))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        for T, base, reps in ((TAIL, PRE, 20), (1, PRE + TAIL, 50)):
            q = torch.randn(L, T, NH, HD, generator=gen, device=dev)
            k = torch.randn(L, T, NKV, HD, generator=gen, device=dev)
            v = torch.randn(L, T, NKV, HD, generator=gen, device=dev)
            pos = torch.stack([torch.arange(base, base + T, device=dev)] * 4).to(torch.int32).contiguous()
            qo = torch.empty(L, T, NH, HD, dtype=torch.float16, device=dev)

            def layers():
                for layer in range(L):
                    kv.norm_rope_append(layer, q[layer], k[layer], v[layer], pos, rope=rope, q_norm=qn, k_norm=kn,
                                        eps=1e-6, base=base, q_out=qo[layer], stream=stream)

            layers()
            stream.synchronize()
            g = torch.cuda.CUDAGraph()          # 36 launches per replay, no host work in between
            with torch.cuda.graph(g, stream=stream):
                layers()
            g.replay()
            stream.synchronize()
            e0.record(stream)
            for _ in range(reps):
                g.replay()
            e1.record(stream)
            e1.synchronize()
            del g
            us = e0.elapsed_time(e1) * 1e3 / (reps * L)
            nbytes = T * (NH + 2 * NKV) * HD * 4 + T * NH * HD * 2 + 2 * T * NKV * HD * 2
            out[f"T{T}_us_per_layer"] = us
            out[f"T{T}_gbs"] = nbytes / (us * 1e-6) / 1e9
        check_flags(kv, stream)
    kv.free()
    return out


def decode_check(kv, layer, q, k_new, v_new, npast, max_keys, stream):
    """One fused append + decode attention of `layer` at the device-side n_past, compared with the CPU
    oracle (test infrastructure, used here only as the checker, outside the timed regions)."""
    import torch
    from oracle import oracle as orc
    out = torch.empty(1, NH, HD, dtype=torch.float32, device=q.device)
    with torch.cuda.stream(stream):
        kv.attn_append_at(layer, q, k_new, v_new, npast, max_keys, SCALE, out=out, stream=stream)
    stream.synchronize()
    n_past = int(npast.item())
    kc = kv.tensor(layer, 0).cpu().numpy()
    vc = kv.tensor(layer, 1).cpu().numpy()
    rows_ok = bool(np.array_equal(kc[n_past].view(np.uint16), k_new.cpu().numpy().view(np.uint16).reshape(-1)) and
                   np.array_equal(vc[n_past].view(np.uint16), v_new.cpu().numpy().view(np.uint16).reshape(-1)))
    qh = q.float().cpu().numpy().reshape(1, NH, HD)
    ref = orc.attn(qh, kc, vc, orc.TYPE_F16, NKV, HD, n_past + 1, SCALE, orc.MASK_CAUSAL, n_past)
    got = out.cpu().numpy()
    err = float(np.abs(got.astype(np.float64) - ref).max())
    rel = float(np.linalg.norm(got - ref) / np.linalg.norm(ref))
    assert rows_ok, "appended K/V row differs from its source"
    assert err <= 2e-3 and rel <= 1e-3, (err, rel)
    return {"layer": layer, "n_past": n_past, "keys": n_past + 1, "max_abs": err, "rel_l2": rel,
            "rows_bit_exact": rows_ok}


def check_flags(kv, stream=None):
    """Device error bits of a cache handle (row range, expired wait, bad segment) must be clear."""
    f = kv.error_flags(stream=stream)
    assert f == 0, f"device error bits 0x{f:x}"


def run_kernels(args):
    """Each kernel of the path on a small single-layer case, 3 launches each in this order:
    fused decode (config 2 geometry, S = 4481), windowed decode (2 sessions of ~19k rows),
    chunked prefill (384 over 4096), f16 and q8_0 append, compaction, fused q8_0 decode and the last q8_0
    prefill chunk (config 4 geometry: q8_0_split_kernel, then the tensor-core kernel on hi + lo parts), and
    the fused q/k norm + IMROPE + append of a config 2 splice tail (384 tokens), and the sharded output
    projection on one rank (K 4096, D 2560).  Under 1 GB on the device; used by the committed ncu
    summaries."""
    import torch
    from __graft_entry__ import load_package
    sv = load_package()
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    times = {}
    ev = lambda: torch.cuda.Event(enable_timing=True)

    def timed(name, fn, reps=3):
        fn()
        torch.cuda.synchronize()
        a, b = ev(), ev()
        a.record()
        for _ in range(reps - 1):
            fn()
        b.record()
        b.synchronize()
        times[name] = a.elapsed_time(b) / max(reps - 1, 1) * 1e3

    kv = sv.KvCache()
    assert kv.alloc(0, 1, NKV, HD, 8192)
    kv.tensor(0, 0).view(torch.float16).normal_(generator=g)
    kv.tensor(0, 1).view(torch.float16).normal_(generator=g)
    npast = torch.full((1,), PRE + TAIL, dtype=torch.int32, device=dev)
    q1 = torch.randn(1, NH, HD, generator=g, device=dev).half()
    k1 = torch.randn(1, NKV * HD, generator=g, device=dev).half()
    timed("decode_fused_us", lambda: kv.attn_append_at(0, q1, k1, k1, npast, PRE + TAIL + 8, SCALE))
    kw = sv.KvCache()
    assert kw.alloc(0, 1, NKV, HD, 40000)
    kw.tensor(0, 0).view(torch.float16).normal_(generator=g)
    kw.tensor(0, 1).view(torch.float16).normal_(generator=g)
    lo = torch.tensor([0, 20000], dtype=torch.int32, device=dev)
    own = torch.tensor([18000, 39000], dtype=torch.int32, device=dev)
    hi = own + 1
    q2 = torch.randn(2, NH, HD, generator=g, device=dev).half()
    timed("decode_window_us", lambda: kw.attn_window(0, q2, lo, hi, own, 19001, SCALE))
    qt = torch.randn(TAIL, NH, HD, generator=g, device=dev).half()
    timed("prefill_us", lambda: kv.attn(0, qt, n_past=PRE, scale=SCALE))
    kt = torch.randn(TAIL, NKV * HD, generator=g, device=dev).half()
    timed("append_f16_us", lambda: kv.append(0, kt, kt, base=PRE))
    kq = sv.KvCache()
    assert kq.alloc(0, 1, 4, 256, 8192 + 64, sv.TYPE_Q8_0)
    kt4 = torch.randn(512, 1024, generator=g, device=dev).half()
    timed("append_q8_0_us", lambda: kq.append(0, kt4, kt4, base=0))
    segs = [(0, 1152, 0), (1152, 5 * 1152, 1)]
    timed("compact_us", lambda: kv.compact(segs, 0))
    for c in range(16):
        kq.append(0, kt4, kt4, base=c * 512)
    npq = torch.full((1,), 8192, dtype=torch.int32, device=dev)
    q4 = torch.randn(1, 16, 256, generator=g, device=dev).half()
    k4 = torch.randn(1, 1024, generator=g, device=dev).half()
    timed("decode_q8_0_us", lambda: kq.attn_append_at(0, q4, k4, k4, npq, 8193, 1 / 16.0))
    q5 = torch.randn(512, 16, 256, generator=g, device=dev).half()
    timed("prefill_q8_0_us", lambda: kq.attn(0, q5, n_past=8192 - 512, scale=1 / 16.0))
    qr = torch.randn(TAIL, NH, HD, generator=g, device=dev)
    kr = torch.randn(TAIL, NKV, HD, generator=g, device=dev)
    pr = torch.stack([torch.arange(PRE, PRE + TAIL, device=dev)] * 4).to(torch.int32).contiguous()
    wr = torch.ones(HD, device=dev)
    timed("norm_rope_append_us", lambda: kv.norm_rope_append(0, qr, kr, kr, pr, rope=(sv.ROPE_IMROPE, HD, 5e6, (24, 20, 20, 0)),
                                                             q_norm=wr, k_norm=wr, base=PRE))
    # the sharded output projection on one rank (its own slot; one slot per call, each its own epoch)
    peer = sv.Peer(0, 0, 1, 3, 2560 * 4)
    peer.import_handles([peer.export()])
    wo = (torch.randn(2560, NH * HD, generator=g, device=dev) * 0.02).half()
    xo = torch.randn(1, NH * HD, generator=g, device=dev).half()
    ep = torch.ones(1, dtype=torch.int32, device=dev)
    calls = iter(range(3))
    timed("out_proj_us", lambda: peer.out_proj(xo, wo, 0, next(calls), ep))
    torch.cuda.synchronize()
    peer.free()
    torch.cuda.synchronize()
    assert kv.error_flags() == 0 and kq.error_flags() == 0 and kw.error_flags() == 0
    print(json.dumps({"workload": "kernels", "us_per_launch": times}), flush=True)


def longctx_leg(sv, world, rank, local, K, W, gather="peer", check=True, shards=None):
    """One 131072-token session (config 5's long-context run) sharded by KV head: rank g keeps kv heads
    [g*8/G, (g+1)*8/G) of all 36 layers and their query heads.  Per layer one kernel appends, attends
    on the local heads and stores its output rows straight into every rank's gathered buffer over
    NVLink (peer memory, counted on every rank's arrival counter); the next layer's kernel waits for
    the previous layer's count before it reads its query rows (gather="nccl": attention, then an
    NCCL all-gather per layer).  Strong scaling: the session's work is fixed; returns (on rank 0) the
    decode tokens/s of that session with its KV bandwidth per GPU.  With `check`, after the timed
    steps one more step runs and every rank compares (a) its own heads' rows of the last layer, as
    they landed in its gathered buffer, with the CPU oracle over its cache shard and (b) the whole
    gathered row block with every rank's own rows (bitwise).  `shards` = G > 1 on one GPU: rank 0's shard
    of a G-way split alone (its kernel without the exchange), to separate the kernel from the exchange."""
    import importlib
    import torch
    import torch.distributed as dist
    sh = importlib.import_module("skyvision_b200.sharding")
    dev = torch.device(f"cuda:{local}")
    stream = torch.cuda.Stream(device=dev)
    S0 = 131072
    G = shards or world
    emulate = G != world
    if emulate and world != 1:
        raise SystemExit("--shards emulates one rank on one GPU")
    if emulate:
        gather = "none"
    hs = sh.HeadShardedDecode(NH, NKV, HD, rank, G)
    nkv_l, nh_l = hs.kv_hi - hs.kv_lo, hs.q_hi - hs.q_lo
    kv = sv.KvCache()
    if not kv.alloc(local, L, nkv_l, HD, S0 + K + W + 64):
        raise SystemExit("KvCache.alloc failed (long context)")
    gen = torch.Generator(device=dev)
    gen.manual_seed(5000 + rank)
    g = None
    with torch.cuda.stream(stream):
        for layer in range(L):
            for isv in (0, 1):
                kv.tensor(layer, isv).view(torch.float16).normal_(generator=gen)
        npast = torch.full((1,), S0, dtype=torch.int32, device=dev)
        ql = torch.randn(L, 1, nh_l, HD, generator=gen, device=dev).half()
        kl = torch.randn(L, 1, nkv_l * HD, generator=gen, device=dev).half()
        vl = torch.randn(L, 1, nkv_l * HD, generator=gen, device=dev).half()
        out_l = torch.empty(L, 1, nh_l, HD, dtype=torch.float32, device=dev)
        out_f = torch.empty(L, 1, NH, HD, dtype=torch.float32, device=dev)
        max_keys = S0 + K + W + 1
        peer = None
        proj = gather == "outproj"
        if proj:
            # the step after each layer's attention, row-parallel: this rank's heads' rows times its column
            # slice of the output projection (D x NH/G*HD), the partials summed over ranks in the same
            # kernel through 64-bit (value, epoch) words -- no all-gather of the attention rows
            Dp = 2560
            w_l = (torch.randn(L, Dp, nh_l * HD, generator=gen, device=dev) * 0.02).half()
            hid = torch.empty(L, 1, Dp, dtype=torch.float32, device=dev)
        if gather in ("peer", "outproj"):
            peer = sv.Peer(local, rank, world, L, world * Dp * 8 if proj else NH * HD * 4)
            mine = peer.export()
            if world > 1:
                handles = [None] * world
                dist.all_gather_object(handles, mine)
            else:
                handles = [mine]
            peer.import_handles(handles)
            epoch = torch.ones(1, dtype=torch.int32, device=dev)    # steps count from 1, never rewound
            barrier(world)

        def step():
            if proj:
                for layer in range(L):
                    kv.attn_append_at(layer, ql[layer], kl[layer], vl[layer], npast, max_keys, SCALE,
                                      out=out_l[layer], stream=stream)
                    peer.out_proj(out_l[layer].view(1, nh_l * HD), w_l[layer], 0, layer, epoch, out=hid[layer],
                                  stream=stream)
                sv.counter_add(epoch, 1, stream=stream)
            elif peer is None:
                for layer in range(L):
                    kv.attn_append_at(layer, ql[layer], kl[layer], vl[layer], npast, max_keys, SCALE,
                                      out=out_l[layer], stream=stream)
                    if not emulate:
                        hs.gather(out_l[layer], out_f[layer])
            else:
                for layer in range(L):
                    kv.attn_append_at_peer(layer, ql[layer], kl[layer], vl[layer], npast, max_keys, SCALE, peer,
                                           hs.q_lo, NH, layer, layer - 1, epoch, stream=stream)
                peer.wait(L - 1, epoch, nkv_l * world, err=None, stream=stream)
                sv.counter_add(epoch, 1, stream=stream)
            sv.counter_add(npast, 1, stream=stream)

        step()
        stream.synchronize()
        npast.fill_(S0)
        try:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                step()
            run = g.replay
            how = ("one CUDA graph per step (attention kernels)" if emulate else
                   "one CUDA graph per step (attention + row-parallel output projection kernels)" if proj else
                   "one CUDA graph per step (attention kernels + NCCL all-gathers)" if peer is None else
                   "one CUDA graph per step (attention kernels storing into every rank's gathered buffer)")
        except Exception as ex:         # capture of the collective unavailable: eager steps
            g = None
            torch.cuda.synchronize()
            run = step
            how = f"eager steps (graph capture failed: {type(ex).__name__})"
        for _ in range(W):
            run()
        npast.fill_(S0)
        stream.synchronize()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clk:
            e0.record(stream)
            for _ in range(K):
                run()
            e1.record(stream)
            e1.synchronize()
        barrier(world)
        ms = e0.elapsed_time(e1)
        check_flags(kv, stream)
        chk = {"oracle_max_abs": 0.0, "oracle_rel_l2": 0.0, "gather_mismatch": 0.0}
        if check:
            # one more step at a known n_past; the gathered rows of the last layer
            npast.fill_(S0 + K)
            torch.cuda.synchronize()
            barrier(world)
            step()
            stream.synchronize()
            barrier(world)
            if proj:
                got_all = None
                got = out_l[L - 1].cpu().numpy()
                # the projection: every rank's float64 partial of the last layer, summed, against hid
                part = torch.from_numpy(out_l[L - 1].reshape(1, -1).double().cpu().numpy() @
                                        w_l[L - 1].double().cpu().numpy().T)
                parts = [None] * world
                if world > 1:
                    dist.all_gather_object(parts, part)
                else:
                    parts = [part]
                pref = sum(parts).numpy()
                chk["proj_rel_err"] = float(np.abs(hid[L - 1].double().cpu().numpy() - pref).max() /
                                            max(np.abs(pref).max(), 1e-30))
            elif peer is not None:
                got_all = peer.slot(L - 1, (1, NH, HD)).clone()
                got = got_all[:, hs.q_lo:hs.q_hi].cpu().numpy()
            elif emulate:
                got_all = None
                got = out_l[L - 1].cpu().numpy()
            else:
                got_all = out_f[L - 1].clone()
                got = got_all[:, hs.q_lo:hs.q_hi].cpu().numpy()
            # (b) every rank's own rows, gathered by NCCL, against this rank's gathered buffer
            if world > 1 and got_all is not None:
                parts = [torch.empty_like(got_all[:, hs.q_lo:hs.q_hi]) for _ in range(world)]
                dist.all_gather(parts, got_all[:, hs.q_lo:hs.q_hi].contiguous())
                whole = torch.cat(parts, dim=1)
                chk["gather_mismatch"] = float((whole != got_all).sum().item())
            # (a) this rank's heads against the oracle over its shard of the last layer
            from oracle import oracle as orc
            orc.set_num_threads(max(1, host_threads() // world))
            kc = kv.tensor(L - 1, 0).cpu().numpy()
            vc = kv.tensor(L - 1, 1).cpu().numpy()
            n_past = S0 + K
            ref = orc.attn(ql[L - 1].float().cpu().numpy(), kc, vc, orc.TYPE_F16, nkv_l, HD, n_past + 1, SCALE,
                           orc.MASK_CAUSAL, n_past)
            chk["oracle_max_abs"] = float(np.abs(got.astype(np.float64) - ref).max())
            chk["oracle_rel_l2"] = float(np.linalg.norm(got - ref) / np.linalg.norm(ref))
            check_flags(kv, stream)
    ms_max = max_over_ranks(ms, world)
    chk = {k: max_over_ranks(v, world) for k, v in chk.items()}
    del g
    if peer is not None:
        barrier(world)
        peer.free()
    kv.free()
    del kv
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    row_b = NKV * HD * 2 * 2
    step_bytes = sum(L * ((S0 + i + 1) * row_b + NH * HD * 6) for i in range(K)) / K
    if emulate:       # one G-th of the session's bytes, on one GPU
        step_bytes /= G
    if proj:          # every rank reads its slice of the projection weights
        step_bytes += L * 2560 * NH * HD * 2
    hbm, _, _ = measured_peaks()
    res = {
        "metric": ("decode attention + output projection tokens/s" if proj else "decode attn tokens/s") +
                  ", one 131072-token session sharded by kv head",
        "value": K / (ms_max * 1e-3), "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": ms_max / K, "higher_is_better": True, "scaling": "strong",
        "workload": "one session of 131072 cached rows, 36 layers, 32q/8kv HD 128 f16 "
                    f"({nkv_l} kv heads per GPU)" + (f"; rank 0's shard of a {G}-way split alone, no exchange"
                                                     if emulate else ""), "step": how,
        "parallelism": f"kv-head sharding over {world} GPU(s), " + (
            "one rank's kernel, no exchange" if emulate else
            "row-parallel output projection, rank partials summed in its kernel through NVLink (64-bit "
            "(value, epoch) words)" if proj else
            "NCCL all-gather of head outputs per layer" if gather == "nccl" else
            "head outputs stored into every rank's buffer by the attention kernel (NVLink peer memory)"),
        "kv_gbs": step_bytes / (ms_max / K * 1e-3) / 1e9,
        "kv_gbs_per_gpu": step_bytes / world / (ms_max / K * 1e-3) / 1e9,
        "hbm_frac_per_gpu": step_bytes / world / (ms_max / K * 1e-3) / 1e9 / hbm,
        "gpu_launches": K * (L + 1),
        "clocks": clk.summary(),
    }
    if check:
        res["check"] = dict(chk, layer=L - 1, n_past=S0 + K,
                            gate="own heads vs the CPU oracle over this rank's shard (max over ranks; "
                                 "max-abs <= 2e-3, rel-L2 <= 1e-3); gathered buffer vs every rank's rows, "
                                 "elements that differ (0 = bitwise equal)")
        assert chk["oracle_max_abs"] <= 2e-3 and chk["oracle_rel_l2"] <= 1e-3 and chk["gather_mismatch"] == 0, chk
        assert chk.get("proj_rel_err", 0.0) <= 1e-5, chk
    return res


def run_longctx(args, world, rank, local):
    """`--workload longctx`: the long-session leg as its own JSON line."""
    from __graft_entry__ import load_package
    sv = load_package()
    res = longctx_leg(sv, world, rank, local, args.steps, args.warmup, gather=args.gather, shards=args.shards)
    if res is None:
        return
    line = {k: res[k] for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                                "higher_is_better", "scaling")}
    line.update({"vs_baseline": None, "dtype": "f16", "data": "synthetic",
                 "config": {"workload": res["workload"], "step": res["step"], "parallelism": res["parallelism"]}})
    line.update({k: v for k, v in res.items() if k not in line and k not in ("workload", "step", "parallelism")})
    print(json.dumps(line), flush=True)


def run_outproj(args, world, rank, local):
    """The step after a head-sharded session's attention: the output projection of this rank's heads
    with the sum over ranks fused in (sv_out_proj_peer), Qwen3-VL-4B geometry (K = 32 x 128 = 4096
    attention inputs, D = 2560 outputs, f16 weights), one decode token through 36 layers per step in
    one CUDA graph.  Strong scaling: each rank reads its K/G columns of every layer's weights
    (D x K/G x 2 bytes) and the ranks exchange [1, D] f32 partials over NVLink."""
    import torch
    import torch.distributed as dist
    from __graft_entry__ import load_package
    sv = load_package()
    dev = torch.device(f"cuda:{local}")
    stream = torch.cuda.Stream(device=dev)
    K, W = args.steps, args.warmup
    Ktot, D = NH * HD, 2560
    kl = Ktot // world
    gen = torch.Generator(device=dev)
    gen.manual_seed(6000 + rank)
    w = (torch.randn(L, D, Ktot, generator=gen, device=dev) * 0.02).half()
    x = torch.randn(L, 1, kl, generator=gen, device=dev).half()
    out = torch.empty(L, 1, D, dtype=torch.float32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    # slots of 64-bit (value, epoch) words (no counters), or of f32 partials with per-band counters
    peer = sv.Peer(local, rank, world, L, world * D * (8 if args.exchange == "words" else 4))
    mine = peer.export()
    handles = [None] * world
    if world > 1:
        dist.all_gather_object(handles, mine)
    else:
        handles = [mine]
    peer.import_handles(handles)
    epoch = torch.ones(1, dtype=torch.int32, device=dev)
    barrier(world)

    def step():
        for layer in range(L):
            peer.out_proj(x[layer], w[layer], rank * kl, layer, epoch, out=out[layer], err=err, stream=stream)
        sv.counter_add(epoch, 1, stream=stream)

    with torch.cuda.stream(stream):
        step()
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            step()
        for _ in range(W):
            g.replay()
        stream.synchronize()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clk:
            e0.record(stream)
            for _ in range(K):
                g.replay()
            e1.record(stream)
            e1.synchronize()
        barrier(world)
        ms = e0.elapsed_time(e1)
    assert int(err.item()) == 0, "device wait timed out"
    ms_max = max_over_ranks(ms, world)
    del g
    barrier(world)
    peer.free()
    if rank != 0:
        return
    hbm, _, _ = measured_peaks()
    wbytes = L * D * kl * 2
    line = {
        "metric": "output projection tokens/s, head-sharded with the sum over ranks fused in",
        "value": K / (ms_max * 1e-3), "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": ms_max / K, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f16", "data": "synthetic",
        "config": {"workload": f"36 layers x (1 x {Ktot // world}) @ ({Ktot // world} x {D}) f16 per rank, partials "
                               "summed over ranks through NVLink peer memory in the same kernel",
                   "exchange": ("64-bit (value, epoch) words, polled per word" if args.exchange == "words" else
                                "f32 partials, per-band counters (release add, acquire poll)"),
                   "parallelism": f"head (column) sharding over {world} GPU(s)"},
        "us_per_layer": ms_max / K / L * 1e3,
        "weight_gbs_per_gpu": wbytes / (ms_max / K * 1e-3) / 1e9,
        "hbm_frac_per_gpu": wbytes / (ms_max / K * 1e-3) / 1e9 / hbm,
        "gpu_launches": K * (L + 1),
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    world, rank, local = (1, 0, 0)
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, world, rank)
        return
    if args.workload == "kernels":
        run_kernels(args)
        return
    world, rank, local = dist_setup(args)
    try:
        if args.workload == "longctx":
            run_longctx(args, world, rank, local)
        elif args.workload == "outproj":
            run_outproj(args, world, rank, local)
        else:
            run_svkv(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
