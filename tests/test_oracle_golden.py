"""The CPU oracle against the golden fixtures (tests/golden/make_golden.py).

These pin the oracle to the reference: q8_0 bytes against gguf-py's Q8_0
encoder (the one convert/_lib.py:120-130 calls), f16 rounding against numpy's
IEEE conversion, and GQA attention against the reference's own numpy oracles
(scripts/parity_nemotronomni_seg.py:94-112, scripts/parity_minicpmo_seg.py).
"""
import numpy as np


def test_q8_0_matches_gguf(golden, orc):
    got = orc.q8_0_quantize(golden["q8_in"])
    assert got.shape == golden["q8_out"].shape
    assert np.array_equal(got, golden["q8_out"])


def test_f16_rounding_matches_ieee(golden, orc):
    got = orc.f32_to_f16(golden["f16_in"])
    assert np.array_equal(got, golden["f16_out"])
    back = orc.f16_to_f32(golden["f16_out"])
    ref = golden["f16_out"].view(np.float16).astype(np.float32)
    assert np.array_equal(back.view(np.uint32), ref.view(np.uint32))


def _cache(k_rows):
    """[S, NKV, HD] f16 bits -> cache bytes [S, NKV*HD*2]."""
    k = np.ascontiguousarray(k_rows).view(np.uint16)
    return k.reshape(k.shape[0], -1).view(np.uint8)


def _check(got, ref, tol=1e-5):
    ref = np.asarray(ref, dtype=np.float64)
    d = np.abs(got.astype(np.float64) - ref)
    rel = np.linalg.norm(d) / np.linalg.norm(ref)
    assert d.max() <= tol and rel <= tol, (d.max(), rel)


def test_attn_nemotron_scenario(golden, orc):
    """tools/nemotronomni_seg_test.cpp:178-276: 8q/2kv HD16, cache 16, prefill 6 + 3 decodes."""
    NH, NKV, HD, S = 8, 2, 16, 16
    q, k, v = golden["nemo_q"], golden["nemo_k"], golden["nemo_v"]
    row = NKV * HD * 2
    kc = np.zeros((S, row), np.uint8)
    vc = np.zeros((S, row), np.uint8)
    # prefill: set_rows of rows 0..5 then causal FA over the whole 16-row view
    assert orc.set_rows(kc, orc.TYPE_F16, NKV * HD, k[:6].reshape(6, -1), orc.TYPE_F16, rows=np.arange(6)) == 0
    assert orc.set_rows(vc, orc.TYPE_F16, NKV * HD, v[:6].reshape(6, -1), orc.TYPE_F16, rows=np.arange(6)) == 0
    out = orc.attn(q[:6], kc, vc, orc.TYPE_F16, NKV, HD, S, 1 / np.sqrt(HD), orc.MASK_CAUSAL, 0)
    _check(out, golden["nemo_prefill_out"])
    for s in range(3):
        p = 6 + s
        orc.set_rows(kc, orc.TYPE_F16, NKV * HD, k[p].reshape(1, -1), orc.TYPE_F16, rows=[p])
        orc.set_rows(vc, orc.TYPE_F16, NKV * HD, v[p].reshape(1, -1), orc.TYPE_F16, rows=[p])
        out = orc.attn(q[p][None], kc, vc, orc.TYPE_F16, NKV, HD, S, 1 / np.sqrt(HD), orc.MASK_CAUSAL, p)
        _check(out[0], golden["nemo_decode_out"][s])
    assert np.array_equal(kc.view(np.uint16).reshape(S, NKV, HD), golden["nemo_final_kcache"])
    assert np.array_equal(vc.view(np.uint16).reshape(S, NKV, HD), golden["nemo_final_vcache"])


def test_attn_minicpmo_probe(golden, orc):
    """tools/minicpmo_seg_test.cpp:239-292: 16 queries, 40 keys, 8 heads, dh 32, no mask (F16 KV)."""
    q = golden["probe_q"]
    kc = golden["probe_k"].view(np.uint8)
    vc = golden["probe_v"].view(np.uint8)
    out = orc.attn(q, kc, vc, orc.TYPE_F16, 8, 32, 40, 1 / np.sqrt(32), orc.MASK_NONE)
    _check(out, golden["probe_out"])


def test_attn_minicpmo_kv_steps(golden, orc):
    """parity_minicpmo_seg.py:308-365 GQA 8:2 HD16 through a KV cache: prefill 6 + 2 decodes."""
    NH, NKV, HD, cap = 8, 2, 16, 32
    kc = np.zeros((cap, NKV * HD * 2), np.uint8)
    vc = np.zeros_like(kc)
    n_past = 0
    for i in range(3):
        q, k, v = golden[f"cpmo_q{i}"], golden[f"cpmo_k{i}"], golden[f"cpmo_v{i}"]
        T = q.shape[0]
        orc.set_rows(kc, orc.TYPE_F16, NKV * HD, k.reshape(T, -1), orc.TYPE_F16, base=n_past)
        orc.set_rows(vc, orc.TYPE_F16, NKV * HD, v.reshape(T, -1), orc.TYPE_F16, base=n_past)
        out = orc.attn(q, kc, vc, orc.TYPE_F16, NKV, HD, n_past + T, 1 / np.sqrt(HD), orc.MASK_CAUSAL, n_past)
        _check(out, golden[f"cpmo_out{i}"])
        n_past += T


def test_attn_baseline_geometry(golden, orc):
    """32q/8kv HD128 (the Qwen3-VL-4B text geometry), 8 queries after 72 cached rows."""
    q, k, v = golden["geo_q"], golden["geo_k"], golden["geo_v"]
    base = int(golden["geo_base"])
    S = k.shape[0]
    out = orc.attn(q, _cache(k), _cache(v), orc.TYPE_F16, 8, 128, S, 1 / np.sqrt(128), orc.MASK_CAUSAL, base)
    _check(out, golden["geo_out"])


def test_qk_norm_rope_neox_matches_reference(golden, orc):
    """The oracle's RMSNorm * weight + NEOX rope against the reference's numpy forms
    (scripts/parity_minicpmo_seg.py rms_norm and rope_llm), small and large positions."""
    for tag in ("a", "b"):
        x, w, pos = golden[f"rope_{tag}_x"], golden[f"rope_{tag}_w"], golden[f"rope_{tag}_pos"]
        HD = x.shape[-1]
        got = orc.rope(orc.rms_norm(x, w, 1e-6), pos, orc.ROPE_NEOX, HD, 1e6)
        np.testing.assert_allclose(got, golden[f"rope_{tag}_out"], rtol=1e-12, atol=1e-12)


def test_imrope_matches_hf_qwen3vl(golden, orc):
    """The oracle's interleaved MRoPE (ggml's IMROPE rule, sections 24/20/20/0, theta 5e6) against HF
    transformers' Qwen3-VL text rotary, which the reference's qwen3vl parity script uses as its
    reference.  The fixture's slot stream equals t, so the two rules agree on every rotation pair;
    HF computes in float32 (angles of positions < 100, so |error| < 5e-5)."""
    x, pos = golden["imrope_hf_x"], golden["imrope_hf_pos"]
    got = orc.rope(x, pos, orc.ROPE_IMROPE, 128, 5e6, (24, 20, 20, 0))
    np.testing.assert_allclose(got, golden["imrope_hf_out"], rtol=0, atol=5e-5)
    # a misrouted stream shows: swapping h and w moves every pair i < 60 with i % 3 != 0
    swapped = orc.rope(x, pos[[0, 2, 1, 3]], orc.ROPE_IMROPE, 128, 5e6, (24, 20, 20, 0))
    assert np.abs(swapped - golden["imrope_hf_out"]).max() > 1e-2
