"""q/k RMSNorm + rotary embedding + K/V append in one kernel (sv_qk_norm_rope_append) against the
oracle's float64 restatement (RMSNorm * weight, NEOX / IMROPE rope; pinned for NEOX to the
reference's numpy rms_norm and rope_llm by the golden fixtures).

Tolerances: f32 queries within 1e-5 (absolute + relative); f16 outputs (queries, K rows) within one
f16 ulp of the float64 value plus 1e-5 absolute; q8_0 K rows within the block_q8_0 rounding bound
of it; V rows bit-exact (f16: RNE of the f32 source; q8_0: the block_q8_0 rule of sv_set_rows,
checked against the oracle's q8_0).
"""
import numpy as np
import pytest
import torch

from __graft_entry__ import load_package

sv = load_package()
pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _inputs(orc, seed, T, NH, NKV, HD):
    rng = np.random.default_rng(seed)
    q = (rng.standard_normal((T, NH, HD)) * 2.0).astype(np.float32)
    k = (rng.standard_normal((T, NKV, HD)) * 2.0).astype(np.float32)
    v = rng.standard_normal((T, NKV, HD)).astype(np.float32)
    qn = (1.0 + 0.3 * rng.standard_normal(HD)).astype(np.float32)
    kn = (1.0 + 0.3 * rng.standard_normal(HD)).astype(np.float32)
    return q, k, v, qn, kn


def _within_f16_ulp(got16, ref64):
    """One f16 ulp of the value, plus the 1e-5 absolute floor of the f32 arithmetic (a rotation
    that cancels two order-1 products to ~1e-4 leaves f32 rounding above that value's f16 ulp)."""
    ref = np.asarray(ref64, np.float64)
    g = np.asarray(got16, np.float16).astype(np.float64)
    ulp = np.spacing(np.abs(ref).astype(np.float16)).astype(np.float64)
    assert np.all(np.abs(g - ref) <= ulp + 1e-5), float(np.max(np.abs(g - ref) - ulp))


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


@pytest.mark.parametrize("mode,T,base", [(2, 37, 100), (40, 21, 3000), (2, 1, 4094)])
def test_f16_cache_neox_imrope(orc, mode, T, base):
    """Qwen3-VL geometry (32q/8kv, HD 128, eps 1e-6): NEOX with theta 1e6, IMROPE with the
    reference's theta 5e6 and sections 24/20/20/0 on four distinct position streams."""
    NH, NKV, HD, cap = 32, 8, 128, 4096
    q, k, v, qn, kn = _inputs(orc, 5 + mode + T, T, NH, NKV, HD)
    rng = np.random.default_rng(T)
    if mode == orc.ROPE_IMROPE:
        theta, sections = 5e6, (24, 20, 20, 0)
        pos = np.stack([base + np.arange(T), rng.integers(0, 40, T), rng.integers(0, 40, T),
                        base + 7 + np.arange(T)]).astype(np.int32)
    else:
        theta, sections = 1e6, (0, 0, 0, 0)
        pos = (base + np.arange(T)).astype(np.int32)
    kv = sv.KvCache()
    assert kv.alloc(0, 2, NKV, HD, cap)
    q32 = torch.empty((T, NH, HD), dtype=torch.float32, device=DEV)
    kv.norm_rope_append(1, _t(q), _t(k), _t(v), _t(pos), rope=(mode, HD, theta, sections), q_norm=_t(qn),
                        k_norm=_t(kn), eps=1e-6, base=base, q_out=q32)
    q16 = kv.norm_rope_append(1, _t(q), _t(k), _t(v), _t(pos), rope=(mode, HD, theta, sections), q_norm=_t(qn),
                              k_norm=_t(kn), eps=1e-6, base=base)
    torch.cuda.synchronize()
    rq, rk = orc.qk_norm_rope(q, k, qn, kn, 1e-6, pos, mode, HD, theta, sections)
    np.testing.assert_allclose(q32.cpu().numpy(), rq, rtol=1e-5, atol=1e-5)
    _within_f16_ulp(q16.cpu().numpy(), rq)
    kc = kv.tensor(1, 0).view(torch.float16)[base:base + T].cpu().numpy().reshape(T, NKV, HD)
    _within_f16_ulp(kc, rk)
    vc = kv.tensor(1, 1)[base:base + T].cpu().numpy()
    assert np.array_equal(vc.view(np.uint16).reshape(T, NKV, HD), orc.f32_to_f16(v))
    assert kv.error_flags() == 0


def test_q8_0_cache_half_rotation_device_base(orc):
    """Config 4 geometry (16q/4kv, HD 256, q8_0 cache), NEOX over the first 128 dims (dims 128..255
    pass through), slot base read on the device: V rows byte-identical to the block_q8_0 rule, K rows
    within the q8_0 rounding bound of the float64 result."""
    NH, NKV, HD, T, base = 16, 4, 256, 19, 1000
    q, k, v, qn, kn = _inputs(orc, 77, T, NH, NKV, HD)
    pos = (base + np.arange(T)).astype(np.int32)
    kv = sv.KvCache()
    assert kv.alloc(0, 1, NKV, HD, 2048, sv.TYPE_Q8_0)
    base_dev = torch.tensor([base], dtype=torch.int32, device=DEV)
    q32 = torch.empty((T, NH, HD), dtype=torch.float32, device=DEV)
    kv.norm_rope_append(0, _t(q), _t(k), _t(v), _t(pos), rope=(2, 128, 1e6, (0, 0, 0, 0)), q_norm=_t(qn),
                        k_norm=_t(kn), eps=1e-6, base_dev=base_dev, q_out=q32)
    torch.cuda.synchronize()
    rq, rk = orc.qk_norm_rope(q, k, qn, kn, 1e-6, pos, orc.ROPE_NEOX, 128, 1e6)
    np.testing.assert_allclose(q32.cpu().numpy(), rq, rtol=1e-5, atol=1e-5)
    ne0 = NKV * HD
    vrows = kv.tensor(0, 1)[base:base + T].cpu().numpy()
    assert np.array_equal(vrows, orc.q8_0_quantize(v.reshape(T, ne0)))
    krows = kv.tensor(0, 0)[base:base + T].cpu().numpy()
    got = orc.q8_0_dequant(krows, ne0).reshape(T, ne0)
    d = orc.f16_to_f32(krows.reshape(T, ne0 // 32, 34)[:, :, :2].copy().view(np.uint16)).reshape(T, ne0 // 32)
    quantum = np.repeat(d, 32, axis=1)
    # |x - q * f16(d)| <= d/2 from the rounding of x/d plus |q| * |f16(d) - d| <= 127 * 2^-11 * d from
    # the f16 scale (half an ulp of 10 fraction bits), plus the f32 arithmetic's 1e-5
    assert np.all(np.abs(got - rk.reshape(T, ne0)) <= quantum * (0.5 + 127 * 2.0 ** -11) + 1e-5)
    assert kv.error_flags() == 0


@pytest.mark.parametrize("kv_type", [1, 8])
def test_plain_append_matches_set_rows(orc, kv_type):
    """No norm, no rotation: the kernel is a plain f32 -> cache append and must write exactly what
    sv_set_rows writes for the same rows (f16 RNE, or the block_q8_0 bytes)."""
    NH, NKV, HD, T, base = 16, 4, 256, 9, 33
    q, k, v, _, _ = _inputs(orc, 3, T, NH, NKV, HD)
    a = sv.KvCache()
    b = sv.KvCache()
    assert a.alloc(0, 1, NKV, HD, 256, kv_type) and b.alloc(0, 1, NKV, HD, 256, kv_type)
    qo = a.norm_rope_append(0, _t(q), _t(k), _t(v), torch.zeros(T, dtype=torch.int32, device=DEV), base=base)
    b.append(0, _t(k.reshape(T, -1)), _t(v.reshape(T, -1)), base=base)
    torch.cuda.synchronize()
    for isv in (0, 1):
        assert np.array_equal(a.tensor(0, isv).cpu().numpy(), b.tensor(0, isv).cpu().numpy())
    assert np.array_equal(qo.cpu().numpy().view(np.uint16), orc.f32_to_f16(q))


def test_rows_past_the_cache_set_the_error_bit(orc):
    NH, NKV, HD, T = 8, 2, 64, 4
    q, k, v, _, _ = _inputs(orc, 9, T, NH, NKV, HD)
    kv = sv.KvCache()
    assert kv.alloc(0, 1, NKV, HD, 64)
    with pytest.raises(sv.SvError):
        kv.norm_rope_append(0, _t(q), _t(k), _t(v), None, base=62)          # host base: refused
    base_dev = torch.tensor([62], dtype=torch.int32, device=DEV)
    kv.norm_rope_append(0, _t(q), _t(k), _t(v), None, base_dev=base_dev)   # device base: rows 64, 65 skipped
    torch.cuda.synchronize()
    assert kv.error_flags() & sv.DEVERR_ROW_RANGE


def test_imrope_kernel_matches_hf_golden(orc, golden):
    """The kernel's IMROPE (no norms, f32 queries out) against the committed HF transformers Qwen3-VL
    rotary fixture (float32 reference, slot stream = t): within 5e-5 plus the kernel's 1e-5."""
    x, pos = golden["imrope_hf_x"], golden["imrope_hf_pos"]
    T, H, HD = x.shape
    kv = sv.KvCache()
    assert kv.alloc(0, 1, 1, HD, 256)
    q32 = torch.empty((T, H, HD), dtype=torch.float32, device=DEV)
    k = np.ascontiguousarray(x[:, :1])
    kv.norm_rope_append(0, _t(x), _t(k), _t(k), _t(pos), rope=(orc.ROPE_IMROPE, HD, 5e6, (24, 20, 20, 0)),
                        base=int(pos[3, 0]), q_out=q32)
    torch.cuda.synchronize()
    np.testing.assert_allclose(q32.cpu().numpy(), golden["imrope_hf_out"], rtol=0, atol=6e-5)
    assert kv.error_flags() == 0
