#!/usr/bin/env python3
"""Generate the golden fixtures that pin the CPU oracle to the reference.

Runs only where the reference checkout and gguf-py are importable (the build
container); the GPU box never runs it.  It writes tests/golden/golden.npz.

What pins what:

* q8_0 rounding -> gguf-py 0.19.0 ``gguf.quants.quantize(x, Q8_0)``, the
  encoder the reference calls at convert/_lib.py:120-130 and which states it is
  bit-exact with ggml-quants.c's reference row quantiser.
* f32 -> f16 -> numpy ``astype(np.float16)`` (IEEE round-to-nearest-even, the
  rounding of ggml_fp32_to_fp16).
* GQA attention over an f16 KV cache -> the reference's own numpy oracles:
  ``gqa_attention`` in scripts/parity_nemotronomni_seg.py:94-112 (causal, the
  ``scenario_attn`` geometry of tools/nemotronomni_seg_test.cpp:178-276:
  8q/2kv, head_dim 16, cache 16 rows, prefill 6 then decode at 6, 7, 8), the
  head-split softmax attention of scripts/parity_minicpmo_seg.py:83-101 (the
  16-query / 40-key / 8-head / dh 32 flash-attn probe of
  tools/minicpmo_seg_test.cpp:239-292, no mask) and the KV-cached GQA step of
  parity_minicpmo_seg.py:308-365 (prefill 6 + two decode steps).
  Inputs are drawn with the reference seg-test generator (src/core/test/
  seg_test.hpp:57-68, uniform [-1, 1]), restated below.
* q/k RMSNorm * weight then NEOX rotary embedding -> the reference's numpy
  ``rms_norm`` and ``rope_llm`` (scripts/parity_minicpmo_seg.py:29-30,
  368-378), theta 1e6, positions 0.. and 8190..
* interleaved MRoPE (Qwen3-VL, sections 24/20/20) -> HF transformers'
  ``Qwen3VLTextRotaryEmbedding`` + ``apply_rotary_pos_emb`` (transformers 5.5.0,
  float32), the reference's own parity anchor for the qwen3vl text stack
  (scripts/parity_onestreamer.py:1-30, 81).  ggml's IMROPE rule takes rotation
  pairs 61 and 62 from the fourth (slot) stream, which HF takes from t; the
  fixture's slot stream equals t (a text-only turn), where both agree.

Usage:  python tests/golden/make_golden.py --reference DIR   (or SVKV_REFERENCE=DIR)
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


class SegRng:
    """The reference seg-test generator (seg_test.hpp:57-68): a 32-bit
    counter hash returning uniforms in [-1, 1]."""

    def __init__(self, seed: int):
        self.s = seed & 0xFFFFFFFF or 1

    def u(self) -> float:
        M = 0xFFFFFFFF
        self.s = (self.s + 0x6D2B79F5) & M
        t = self.s
        t = ((t ^ (t >> 15)) * (t | 1)) & M
        t ^= (t + ((t ^ (t >> 7)) * (t | 61) & M)) & M
        m = (t ^ (t >> 14)) & 0x7FFFFFFF
        return float(np.float32((np.float32(m) - np.float32(1073741824.0)) / np.float32(1073741824.0)))

    def rnd(self, n: int, scale: float = 1.0) -> np.ndarray:
        return np.array([self.u() * scale for _ in range(n)], dtype=np.float32)


def load_module(path: str, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    argv = sys.argv
    sys.argv = [path, "/nonexistent"]       # the scripts read sys.argv[1] at import
    try:
        spec.loader.exec_module(mod)
    finally:
        sys.argv = argv
    return mod


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("SVKV_REFERENCE"),
                    help="the reference checkout (default: $SVKV_REFERENCE)")
    ap.add_argument("--out", default=os.path.join(HERE, "golden.npz"))
    args = ap.parse_args()

    import gguf
    from gguf.quants import quantize
    from gguf.constants import GGMLQuantizationType

    nemo = load_module(os.path.join(args.reference, "scripts/parity_nemotronomni_seg.py"), "ref_nemo")
    cpmo = load_module(os.path.join(args.reference, "scripts/parity_minicpmo_seg.py"), "ref_cpmo")

    g: dict[str, np.ndarray] = {}
    g["gguf_version"] = np.array(gguf.__version__ if hasattr(gguf, "__version__") else "0.19.0")

    # ---------------------------------------------------------------- q8_0
    rng = np.random.default_rng(1234)
    rows = []
    # seeded N(0,1) f16 values (config-4 style rows: 4 kv heads x 256)
    base = rng.standard_normal((8, 1024)).astype(np.float16).astype(np.float32)
    out_mask = rng.random(base.shape) < 0.01
    base[out_mask] *= 8
    base = base.astype(np.float16).astype(np.float32)
    rows.append(base)
    # edge blocks: zeros, ties at .5 after scaling, one hot, f16 extremes, tiny values
    e = np.zeros((8, 1024), dtype=np.float32)
    e[0, :32] = 0.0
    e[0, 32:64] = np.linspace(-127, 127, 32)                # id = 1 exactly -> integers
    e[0, 64:96] = np.arange(32) - 15.5                      # x*id lands on many .5 ties
    e[0, 96:128] = np.concatenate([[127.0], np.full(31, 0.5)])
    e[1, :32] = 65504.0 * np.sign(np.linspace(-1, 1, 32) + 1e-3)
    e[1, 32:64] = 6.1e-5 * np.arange(32)                    # around the f16 subnormal edge
    e[1, 64:96] = -np.abs(rng.standard_normal(32))
    e[1, 96:128] = np.where(np.arange(32) == 7, -3.0, 1e-8)
    e[2:] = rng.standard_normal((6, 1024)) * rng.choice([1e-3, 1.0, 300.0], size=(6, 1))
    rows.append(e.astype(np.float16).astype(np.float32))
    qin = np.concatenate(rows, axis=0)
    qout = quantize(qin, GGMLQuantizationType.Q8_0)
    g["q8_in"] = qin
    g["q8_out"] = np.ascontiguousarray(qout, dtype=np.uint8)

    # ---------------------------------------------------------------- f16
    special = np.array([0.0, -0.0, 1.0, -1.0, 65504.0, 65519.99, 65520.0, 1e9, -1e9,
                        6.103515625e-05, 6.0975552e-05, 5.9604645e-08, 2.9802322e-08,
                        2.98023259e-08, 1e-12, 0.1, 1.0 / 3.0, 2049.0, 2051.0, 4097.0,
                        np.inf, -np.inf], dtype=np.float32)
    rnd = (rng.standard_normal(4096) * np.exp(rng.uniform(-20, 12, 4096))).astype(np.float32)
    f16_in = np.concatenate([special, rnd])
    g["f16_in"] = f16_in
    g["f16_out"] = f16_in.astype(np.float16).view(np.uint16)

    # ------------------------------------------------- attention: nemotron scenario_attn
    r = SegRng(0x5EED1234)
    NH, NKV, HD, S = 8, 2, 16, 16
    # prefill q/k/v for positions 0..5, then one row per decode step 6..8
    q_all = r.rnd(9 * NH * HD).reshape(9, NH, HD)
    k_all = r.rnd(9 * NKV * HD).reshape(9, NKV, HD).astype(np.float16)
    v_all = r.rnd(9 * NKV * HD).reshape(9, NKV, HD).astype(np.float16)
    kc = np.zeros((S, NKV, HD), dtype=np.float16)
    vc = np.zeros((S, NKV, HD), dtype=np.float16)
    kc[:6] = k_all[:6]
    vc[:6] = v_all[:6]
    pre = nemo.gqa_attention(q_all[:6].astype(np.float64), kc.astype(np.float64),
                             vc.astype(np.float64), HD, NKV)
    g["nemo_q"] = q_all
    g["nemo_k"] = k_all.view(np.uint16)
    g["nemo_v"] = v_all.view(np.uint16)
    g["nemo_prefill_out"] = pre
    dec = []
    for s in range(3):
        p = 6 + s
        kc[p] = k_all[p]
        vc[p] = v_all[p]
        o = nemo.gqa_attention(q_all[p][None].astype(np.float64), kc.astype(np.float64),
                               vc.astype(np.float64), HD, NKV, q_pos=[p])[0]
        dec.append(o)
    g["nemo_decode_out"] = np.stack(dec)
    g["nemo_final_kcache"] = kc.view(np.uint16)
    g["nemo_final_vcache"] = vc.view(np.uint16)

    # ------------------------------------------- attention: minicpmo FA probe (MHA, no mask)
    r = SegRng(0xFACE0001)
    H, NQ, NK, dh = 8, 16, 40, 32
    qp = r.rnd(NQ * H * dh).reshape(NQ, H * dh)
    kk = r.rnd(NK * H * dh).reshape(NK, H * dh).astype(np.float16)
    vv = r.rnd(NK * H * dh).reshape(NK, H * dh).astype(np.float16)

    def heads(t, n):
        return t.reshape(n, H, dh).transpose(1, 0, 2)
    qh = heads(qp.astype(np.float64), NQ)
    kh = heads(kk.astype(np.float64), NK)
    vh = heads(vv.astype(np.float64), NK)
    att = cpmo.softmax(qh @ kh.transpose(0, 2, 1) / np.sqrt(dh))
    g["probe_q"] = qp.reshape(NQ, H, dh)
    g["probe_k"] = kk.view(np.uint16)
    g["probe_v"] = vv.view(np.uint16)
    g["probe_out"] = (att @ vh).transpose(1, 0, 2)                 # [NQ, H, dh]

    # ------------------------------------ attention: minicpmo KV-cached GQA (prefill 6 + 2 decode)
    r = SegRng(0xC0FFEE01)
    NH, NKV, HD = 8, 2, 16
    Tt = [6, 1, 1]
    qs = [r.rnd(t * NH * HD).reshape(t, NH, HD) for t in Tt]
    ks = [r.rnd(t * NKV * HD).reshape(t, NKV, HD).astype(np.float16) for t in Tt]
    vs = [r.rnd(t * NKV * HD).reshape(t, NKV, HD).astype(np.float16) for t in Tt]
    outs = []
    n_past = 0
    kn_all = np.zeros((NKV, 0, HD))
    vv_all = np.zeros((NKV, 0, HD))
    for step, T in enumerate(Tt):
        q = qs[step].astype(np.float64).transpose(1, 0, 2)
        kn_all = np.concatenate([kn_all, ks[step].astype(np.float64).transpose(1, 0, 2)], 1)
        vv_all = np.concatenate([vv_all, vs[step].astype(np.float64).transpose(1, 0, 2)], 1)
        kk2 = np.repeat(kn_all, NH // NKV, axis=0)
        vv2 = np.repeat(vv_all, NH // NKV, axis=0)
        a = q @ kk2.transpose(0, 2, 1) / np.sqrt(HD)
        Sx = n_past + T
        m = np.zeros((T, Sx), bool)
        for t in range(T):
            m[t, n_past + t + 1:] = True
        a = np.where(m[None], -np.inf, a)
        a = cpmo.softmax(a)
        outs.append((a @ vv2).transpose(1, 0, 2))                  # [T, NH, HD]
        n_past += T
    for i in range(3):
        g[f"cpmo_q{i}"] = qs[i]
        g[f"cpmo_k{i}"] = ks[i].view(np.uint16)
        g[f"cpmo_v{i}"] = vs[i].view(np.uint16)
        g[f"cpmo_out{i}"] = outs[i]

    # ------------------------------------------- attention: BASELINE geometry (32q/8kv, HD 128)
    r = SegRng(0x0B200001)
    NH, NKV, HD, S, T = 32, 8, 128, 80, 8
    base = S - T
    q = r.rnd(T * NH * HD).reshape(T, NH, HD)
    kc = r.rnd(S * NKV * HD).reshape(S, NKV, HD).astype(np.float16)
    vc = r.rnd(S * NKV * HD).reshape(S, NKV, HD).astype(np.float16)
    o = nemo.gqa_attention(q.astype(np.float64), kc.astype(np.float64), vc.astype(np.float64),
                           HD, NKV, q_pos=list(range(base, S)))
    g["geo_q"] = q
    g["geo_k"] = kc.view(np.uint16)
    g["geo_v"] = vc.view(np.uint16)
    g["geo_out"] = o
    g["geo_base"] = np.array(base)

    # ------------------------------------------- q/k RMSNorm + NEOX rope: the reference's numpy forms
    # rms_norm (parity_minicpmo_seg.py:29-30) and rope_llm (:368-378), theta = 1e6, at small and large
    # positions (chunk 0 and a chunk past 8k tokens)
    r = SegRng(0x0B200002)
    for tag, T, H, HD, p0 in (("a", 5, 3, 64, 0), ("b", 4, 2, 128, 8190)):
        x = r.rnd(T * H * HD, 3.0).reshape(T, H, HD)
        w = 1.0 + r.rnd(HD, 0.5)
        pos = np.arange(p0, p0 + T)
        y = cpmo.rope_llm(cpmo.rms_norm(x.astype(np.float64), w.astype(np.float64), 1e-6), pos, HD, 1e6)
        g[f"rope_{tag}_x"] = x
        g[f"rope_{tag}_w"] = w
        g[f"rope_{tag}_pos"] = pos.astype(np.int32)
        g[f"rope_{tag}_out"] = y

    # ------------------------------------------- IMROPE: HF transformers' Qwen3-VL text rotary (float32)
    from transformers.models.qwen3_vl import modeling_qwen3_vl as hfq
    from transformers.models.qwen3_vl.configuration_qwen3_vl import Qwen3VLTextConfig
    import torch
    cfg = Qwen3VLTextConfig(hidden_size=256, num_attention_heads=2, num_key_value_heads=1, head_dim=128,
                            rope_parameters={"rope_type": "default", "rope_theta": 5e6,
                                             "mrope_section": [24, 20, 20]})
    rot = hfq.Qwen3VLTextRotaryEmbedding(cfg)
    r = SegRng(0x0B200003)
    T, H, HD = 6, 3, 128
    x = r.rnd(T * H * HD, 3.0).reshape(T, H, HD).astype(np.float32)
    t = np.arange(90, 90 + T)
    hh = np.array([3, 0, 17, 39, 22, 8])
    ww = np.array([5, 31, 0, 12, 39, 26])
    xt = torch.from_numpy(x).permute(1, 0, 2)[None]                       # (1, H, T, HD)
    cos, sin = rot(xt, torch.from_numpy(np.stack([t, hh, ww]))[:, None, :])
    y, _ = hfq.apply_rotary_pos_emb(xt, xt, cos, sin)
    g["imrope_hf_x"] = x
    g["imrope_hf_pos"] = np.stack([t, hh, ww, t]).astype(np.int32)        # [t, h, w, slot]
    g["imrope_hf_out"] = y[0].permute(1, 0, 2).numpy().astype(np.float64)

    np.savez_compressed(args.out, **g)
    print(f"wrote {args.out}: {len(g)} arrays, {os.path.getsize(args.out)} bytes")


if __name__ == "__main__":
    main()
