"""Parity at the sizes the benchmark times, against the oracle.

The other GPU test files sweep shapes at sizes the oracle finishes quickly;
this file checks the BASELINE configurations at their own sizes:

* config 4 decode: a q8_0 cache of 8192 prefilled rows (16q/4kv, HD 256, 1 %
  outliers x8), the fused append + attention at n_past 8192..8195 and at the
  last decode step, 8447 -- appended rows bit-exact, outputs within the gate;
* config 4 prefill: the last two 512-token chunks (n_past 7168 and 7680) of an
  8192-token q8_0 prompt;
* config 3: 12 rounds of 16 frames x 64 rows + 96 text + 32 answer rows with a
  6-round window, two layers: after every round the bytes of every surviving
  row equal the rows written for its original id;
* the per-GPU shard of the 131072-token session: one decode over 131073 keys
  with 1 and 2 kv heads;
* the splice (qwen3vl_model.cpp:1165-1196): turn 2 run by splicing its tail
  onto the cached turn 1, and by clearing the cache and prefilling the whole
  prompt again (the resume=false path, qwen3vl_model.cpp:972-976), gives the
  same cache bytes and the same attention outputs.

Gate: max-abs <= 2e-3 and relative L2 <= 1e-3 against the fp32-accumulated
oracle; bit-exact for every cache byte.
"""
import numpy as np
import pytest
import torch

from __graft_entry__ import load_package

sv = load_package()
pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
MAX_ABS, REL_L2 = 2e-3, 1e-3


def close(got, ref, max_abs=MAX_ABS, rel=REL_L2):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    d = np.abs(got - ref)
    r = np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30)
    assert np.isfinite(got).all()
    assert d.max() <= max_abs and r <= rel, (float(d.max()), float(r))


def td(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.float16)).to(DEV)


def attn_ref(orc, kv, layer, q_bits, n_past, scale):
    kc = kv.tensor(layer, 0).cpu().numpy()
    vc = kv.tensor(layer, 1).cpu().numpy()
    T = q_bits.shape[0]
    return orc.attn(orc.f16_to_f32(q_bits), kc, vc, kv.kv_type, kv.n_kv_head, kv.head_dim, n_past + T, scale,
                    orc.MASK_CAUSAL, n_past)


# ------------------------------------------------------------------ config 4 (q8_0, HD 256)
C4_NKV, C4_HD, C4_NH, C4_S0, C4_CH, C4_DEC = 4, 256, 16, 8192, 512, 256


def _cfg4_cache(orc, n_ctx, seed):
    """One q8_0 layer of config 4: 8192 prefilled rows appended chunk by chunk like the prefill loop."""
    kv = sv.KvCache()
    assert kv.alloc(0, 1, C4_NKV, C4_HD, n_ctx, sv.TYPE_Q8_0)
    ne0 = C4_NKV * C4_HD
    for c in range(C4_S0 // C4_CH):
        k = orc.normal_f16(seed, 100 + c, C4_CH * ne0, outlier_frac=0.01).reshape(C4_CH, ne0)
        v = orc.normal_f16(seed, 300 + c, C4_CH * ne0, outlier_frac=0.01).reshape(C4_CH, ne0)
        kv.append(0, td(k), td(v), base=c * C4_CH)
    return kv


def test_cfg4_q8_0_decode_at_baseline_size(orc):
    """Config 4 decode steps 0..3 (n_past 8192..8195) and the last step (n_past 8447) through the fused
    append + attention on the q8_0 cache, against the oracle's block_q8_0 rule and attention."""
    kv = _cfg4_cache(orc, C4_S0 + C4_DEC + 64, seed=3)
    ne0 = C4_NKV * C4_HD
    npast = torch.zeros(1, dtype=torch.int32, device=DEV)
    max_keys = C4_S0 + C4_DEC + 1
    for n_past in (8192, 8193, 8194, 8195, 8447):
        if n_past == 8447:          # rows 8196..8446 as the skipped decode steps would have left them
            gap = n_past - 8196
            kg = orc.normal_f16(3, 900, gap * ne0, outlier_frac=0.01).reshape(gap, ne0)
            vg = orc.normal_f16(3, 901, gap * ne0, outlier_frac=0.01).reshape(gap, ne0)
            kv.append(0, td(kg), td(vg), base=8196)
        q = orc.normal_f16(3, 1000 + n_past, C4_NH * C4_HD).reshape(1, C4_NH, C4_HD)
        k = orc.normal_f16(3, 2000 + n_past, ne0, outlier_frac=0.01).reshape(1, ne0)
        v = orc.normal_f16(3, 3000 + n_past, ne0, outlier_frac=0.01).reshape(1, ne0)
        npast.fill_(n_past)
        out = kv.attn_append_at(0, td(q), td(k), td(v), npast, max_keys, 1 / 16.0)
        torch.cuda.synchronize()
        kc = kv.tensor(0, 0).cpu().numpy()
        vc = kv.tensor(0, 1).cpu().numpy()
        assert np.array_equal(kc[n_past], orc.q8_0_quantize(orc.f16_to_f32(k[0])))
        assert np.array_equal(vc[n_past], orc.q8_0_quantize(orc.f16_to_f32(v[0])))
        ref = orc.attn(orc.f16_to_f32(q), kc, vc, orc.TYPE_Q8_0, C4_NKV, C4_HD, n_past + 1, 1 / 16.0,
                       orc.MASK_CAUSAL, n_past)
        close(out.cpu().numpy(), ref)
    assert kv.error_flags() == 0


def test_cfg4_q8_0_late_prefill_chunks(orc):
    """The last two 512-token chunks of config 4's 8192-token prompt (n_past 7168 and 7680): the
    chunks the bench and the committed prefill profile time."""
    kv = _cfg4_cache(orc, C4_S0 + 64, seed=4)
    for n_past in (7168, 7680):
        q = orc.normal_f16(4, 5000 + n_past, C4_CH * C4_NH * C4_HD).reshape(C4_CH, C4_NH, C4_HD)
        out = kv.attn(0, td(q), n_past=n_past, scale=1 / 16.0)
        torch.cuda.synchronize()
        close(out.cpu().numpy(), attn_ref(orc, kv, 0, q, n_past, 1 / 16.0))
    assert kv.error_flags() == 0


# ------------------------------------------------------------------ config 3 (eviction, full shape)
def test_cfg3_full_shape_surviving_bytes(orc):
    """BASELINE config 3 at its own shape on two layers: 12 rounds of 16 frames x 64 rows + 96 text
    rows + 32 answer rows, window 6 rounds.  From round 7 the oldest round leaves and the survivors
    are compacted in place; after every round each cache row holds exactly the K and V bytes written
    for the original row id the window rule keeps there."""
    rpf, frames, text, answer, rounds, L, NKV, HD = 64, 16, 96, 32, 12, 2, 8, 128
    round_rows = frames * rpf + text + answer
    ne0 = NKV * HD
    kv = sv.KvCache()
    assert kv.alloc(0, L, NKV, HD, 7 * round_rows + 64)
    sess = sv.Session(kv, max_frames=6 * frames, rows_per_frame=rpf)
    ref = orc.SessionRows(6 * frames, rpf)
    gen = torch.Generator(device=DEV)
    gen.manual_seed(2)
    written_k = [[] for _ in range(L)]      # per layer: host copies of the rows of each round, in id order
    written_v = [[] for _ in range(L)]
    for r in range(rounds):
        first, kept = sess.begin_turn(frames)
        ref.begin_turn(frames)
        n = kept * rpf + text + answer
        for layer in range(L):
            k = torch.randn(n, ne0, generator=gen, device=DEV).half()
            v = torch.randn(n, ne0, generator=gen, device=DEV).half()
            kv.append(layer, k, v, base=first)
            written_k[layer].append(k.cpu().numpy().view(np.uint16))
            written_v[layer].append(v.cpu().numpy().view(np.uint16))
        sess.end_turn(kept, text, answer)
        ref.end_turn(kept, text, answer)
        rows = sess.rows()
        assert np.array_equal(rows, ref.rows())
        torch.cuda.synchronize()
        for layer in range(L):
            all_k = np.concatenate(written_k[layer])
            all_v = np.concatenate(written_v[layer])
            kc = kv.tensor(layer, 0).cpu().numpy().view(np.uint16)[: rows.size]
            vc = kv.tensor(layer, 1).cpu().numpy().view(np.uint16)[: rows.size]
            assert np.array_equal(kc, all_k[rows]), (r, layer)
            assert np.array_equal(vc, all_v[rows]), (r, layer)
    assert sess.rows().size == 6 * round_rows
    assert kv.error_flags() == 0


# ------------------------------------------------------------------ the long session's per-GPU shard
@pytest.mark.parametrize("nkv", [1, 2])
def test_decode_131072_keys(orc, nkv):
    """One decode token of the 131072-token session on a shard of `nkv` kv heads (8 or 4 GPUs): the
    fused append at row 131072 and attention over 131073 keys, against the oracle."""
    HD, S0 = 128, 131072
    nh = 4 * nkv
    kv = sv.KvCache()
    assert kv.alloc(0, 1, nkv, HD, S0 + 8)
    g = torch.Generator(device=DEV)
    g.manual_seed(51 + nkv)
    kv.tensor(0, 0).view(torch.float16)[:S0].normal_(generator=g)
    kv.tensor(0, 1).view(torch.float16)[:S0].normal_(generator=g)
    q = orc.normal_f16(51, nkv, nh * HD).reshape(1, nh, HD)
    k = orc.normal_f16(52, nkv, nkv * HD).reshape(1, nkv * HD)
    v = orc.normal_f16(53, nkv, nkv * HD).reshape(1, nkv * HD)
    npast = torch.full((1,), S0, dtype=torch.int32, device=DEV)
    out = kv.attn_append_at(0, td(q), td(k), td(v), npast, S0 + 4, 1 / np.sqrt(HD))
    torch.cuda.synchronize()
    assert kv.error_flags() == 0
    kc = kv.tensor(0, 0).cpu().numpy()
    vc = kv.tensor(0, 1).cpu().numpy()
    assert np.array_equal(kc[S0].view(np.uint16), k[0]) and np.array_equal(vc[S0].view(np.uint16), v[0])
    ref = orc.attn(orc.f16_to_f32(q), kc, vc, orc.TYPE_F16, nkv, HD, S0 + 1, 1 / np.sqrt(HD), orc.MASK_CAUSAL, S0)
    close(out.cpu().numpy(), ref)


# ------------------------------------------------------------------ splice == re-prefill
def _turn_rows(orc, layer, lo, hi, ne0, nh, hd):
    """K, V and Q rows of token positions [lo, hi) of one layer: a function of the position only, as
    the real model's rows are a function of the (shared) prompt prefix."""
    n = hi - lo
    k = np.stack([orc.normal_f16(61, 10000 * layer + p, ne0) for p in range(lo, hi)]).reshape(n, ne0)
    v = np.stack([orc.normal_f16(62, 10000 * layer + p, ne0) for p in range(lo, hi)]).reshape(n, ne0)
    q = np.stack([orc.normal_f16(63, 10000 * layer + p, nh * hd) for p in range(lo, hi)]).reshape(n, nh, hd)
    return k, v, q


@pytest.mark.parametrize("kv_type", [sv.TYPE_F16, sv.TYPE_Q8_0])
def test_splice_equals_full_reprefill(orc, kv_type):
    """Turn 2's prompt strictly extends turn 1's.  Route A splices: the predicate gives skip = len(turn
    1), only the tail is appended and chunk-prefilled at n_past = skip.  Route B is the resume=false
    path: sv_kv_clear, then the whole prompt is appended and prefilled from n_past 0.  Both leave the
    same cache bytes, and the tail rows' attention outputs (and one decode token after the turn) agree
    with each other and with the oracle."""
    L, NKV, HD, NH, P1, T2 = 2, 8, 128, 32, 700, 300
    if kv_type == sv.TYPE_Q8_0:
        NKV, HD, NH = 4, 256, 16
    ne0 = NKV * HD
    scale = 1 / np.sqrt(HD)
    ids1 = (np.arange(P1, dtype=np.int32) * 31) % 151000
    ids2 = np.concatenate([ids1, (np.arange(T2, dtype=np.int32) * 17 + 5) % 151000])
    rows = [_turn_rows(orc, layer, 0, P1 + T2 + 1, ne0, NH, HD) for layer in range(L)]
    caches, tails, decs = [], [], []
    for route in ("splice", "reprefill"):
        kv = sv.KvCache()
        assert kv.alloc(0, L, NKV, HD, P1 + T2 + 64, kv_type)
        # turn 1 (both routes): the whole first prompt, in two chunks
        for layer in range(L):
            k, v, q = rows[layer]
            for lo, hi in ((0, 400), (400, P1)):
                kv.append(layer, td(k[lo:hi]), td(v[lo:hi]), base=lo)
                kv.attn(layer, td(q[lo:hi]), n_past=lo, scale=scale)
        if route == "splice":
            skip = sv.can_splice(ids1, P1, ids2)
            assert skip == P1
            chunks = ((P1, P1 + T2),)
        else:
            assert sv.can_splice(ids1, P1, ids2[:P1]) == 0      # not an extension: the full path
            kv.clear()
            chunks = ((0, 512), (512, P1 + T2))
        tail = []
        for layer in range(L):
            k, v, q = rows[layer]
            outs = []
            for lo, hi in chunks:
                kv.append(layer, td(k[lo:hi]), td(v[lo:hi]), base=lo)
                outs.append(kv.attn(layer, td(q[lo:hi]), n_past=lo, scale=scale).cpu().numpy())
            tail.append(np.concatenate(outs)[-T2:])
        # one decode token after the turn
        npast = torch.full((1,), P1 + T2, dtype=torch.int32, device=DEV)
        dec = []
        for layer in range(L):
            k, v, q = rows[layer]
            dec.append(kv.attn_append_at(layer, td(q[-1:]), td(k[-1:]), td(v[-1:]), npast, P1 + T2 + 8,
                                         scale).cpu().numpy())
        torch.cuda.synchronize()
        caches.append([(kv.tensor(layer, 0).cpu().numpy(), kv.tensor(layer, 1).cpu().numpy()) for layer in range(L)])
        tails.append(tail)
        decs.append(dec)
        assert kv.error_flags() == 0
        kv.free()
    n_rows = P1 + T2 + 1
    for layer in range(L):
        (ka, va), (kb, vb) = caches[0][layer], caches[1][layer]
        assert np.array_equal(ka[:n_rows], kb[:n_rows]) and np.array_equal(va[:n_rows], vb[:n_rows]), layer
        close(tails[0][layer], tails[1][layer])
        close(decs[0][layer], decs[1][layer])
        k, v, q = rows[layer]
        ref = orc.attn(orc.f16_to_f32(q[P1:P1 + T2]), ka, va, kv_type, NKV, HD, P1 + T2, scale, orc.MASK_CAUSAL, P1)
        close(tails[0][layer], ref)
        ref_d = orc.attn(orc.f16_to_f32(q[-1:]), ka, va, kv_type, NKV, HD, n_rows, scale, orc.MASK_CAUSAL, P1 + T2)
        close(decs[0][layer], ref_d)
