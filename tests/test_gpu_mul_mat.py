"""The soft_max fallback's two mul_mat legs on the GPU against the oracle.

gemma4_model.cpp:683-692 (and moondream.cpp:476-493, per head) attends with
    kq = mul_mat(kf, qf) -> soft_max_ext(kq, mask, scale) -> mul_mat(cont(transpose(vf)), kq)
when flash attention is off.  Checked here: sv_mul_mat_kq against the oracle's
scores (float64 sums of the f16 cache rows and the f16-rounded queries, as ggml
converts src1 to an f16 src0's vec-dot type), sv_mul_mat_kqv against the
oracle's P.V, and the whole triple (with sv_soft_max_ext in the middle) against
the oracle's attention and against sv_flash_attn_ext.

Tolerances: scores (magnitude ~sqrt(HD)) max-abs <= 2e-3 and relative L2 <= 1e-5
(f32 accumulation of exact f16 products); P.V and the triple's output at the
attention gate, max-abs <= 2e-3 and relative L2 <= 1e-3.
"""
import ctypes

import numpy as np
import pytest
import torch

from __graft_entry__ import load_package

sv = load_package()
pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def close(got, ref, max_abs=2e-3, rel=1e-3):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    d = np.abs(got - ref)
    r = np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30)
    assert np.isfinite(got).all()
    assert d.max() <= max_abs and r <= rel, (float(d.max()), float(r))


def cache(orc, seed, n_rows, ne0, pad=0):
    """f16 cache rows (bits) and the device tensor of rows of ne0 + pad elements."""
    k = orc.normal_f16(seed, 1, n_rows * ne0).reshape(n_rows, ne0)
    full = np.zeros((n_rows, ne0 + pad), np.uint16)
    full[:, :ne0] = k
    return full, torch.from_numpy(full.view(np.uint8)).to(DEV)


GEOMS = [  # n_kv_head, head_dim, n_head, T, S
    (8, 128, 32, 1, 1500),      # config 2 geometry, one decode token
    (8, 128, 32, 64, 700),      # a prompt chunk
    (4, 256, 16, 40, 900),      # config 4 geometry (f16 cache)
    (2, 128, 8, 130, 257),      # ragged query tiles and key tiles
    (1, 64, 1, 33, 300),        # moondream's per-head form (one head of a 2048-wide row)
]


@pytest.mark.parametrize("nkv,hd,nh,T,S", GEOMS)
@pytest.mark.parametrize("q_f32", [False, True])
def test_mul_mat_kq(orc, nkv, hd, nh, T, S, q_f32):
    kb, kd = cache(orc, 70 + hd, S, nkv * hd, pad=64)          # rows longer than the view (cache row stride)
    q16 = orc.normal_f16(71, T + nh, T * nh * hd).reshape(T, nh, hd)
    q = orc.f16_to_f32(q16)
    if q_f32:
        q = q * np.float32(1.0 + 1e-3)                          # not f16-exact: rounded like ggml's src1
    qd = torch.from_numpy(q if q_f32 else q16.view(np.float16)).to(DEV)
    got = sv.mul_mat_kq(kd, qd, nkv, hd, S).cpu().numpy()
    ref = orc.mul_mat_kq(kb.view(np.uint8), q, nkv, hd, S)
    close(got, ref, max_abs=2e-3, rel=1e-5)


@pytest.mark.parametrize("nkv,hd,nh,T,S", GEOMS)
@pytest.mark.parametrize("split", [True, False])
def test_mul_mat_kqv(orc, nkv, hd, nh, T, S, split):
    vb, vd = cache(orc, 80 + hd, S, nkv * hd, pad=64)
    rng = np.random.default_rng(hd + T)
    p = rng.random((nh, T, S)).astype(np.float32)
    p /= p.sum(-1, keepdims=True)                               # softmax-like rows
    p[:, :, ::7] *= 3.0                                         # not normalised: any f32 weights
    pd = torch.from_numpy(p).to(DEV)
    got = sv.mul_mat_kqv(vd, pd, nkv, hd, S, workspace=split).cpu().numpy()
    ref = orc.mul_mat_kqv(vb.view(np.uint8), p, nkv, hd, S)
    close(got, ref)


def test_mul_mat_kqv_ggml_layout_and_strided_kq(orc):
    """dst in ggml's own [HD, T, NH] order and kq rows with a padded stride."""
    nkv, hd, nh, T, S = 4, 128, 16, 5, 333
    vb, vd = cache(orc, 90, S, nkv * hd)
    rng = np.random.default_rng(3)
    p = rng.random((nh, T, S)).astype(np.float32)
    pad = torch.zeros((nh, T, S + 12), dtype=torch.float32, device=DEV)
    pad[:, :, :S] = torch.from_numpy(p).to(DEV)
    pv = pad[:, :, :S]
    dst = torch.zeros((nh, T, hd), dtype=torch.float32, device=DEV)
    L = sv.lib()
    rc = L.sv_mul_mat_kqv(vd.data_ptr(), vd.stride(0), nkv, hd, S, pv.data_ptr(), pv.stride(1) * 4, pv.stride(0) * 4,
                          T, nh, dst.data_ptr(), hd * 4, T * hd * 4, None, 0, None)
    assert rc == 0
    ref = orc.mul_mat_kqv(vb.view(np.uint8), p, nkv, hd, S)      # [T, NH, HD]
    close(dst.cpu().numpy(), ref.transpose(1, 0, 2))


@pytest.mark.parametrize("nkv,hd,nh,T,n_past", [(8, 128, 32, 1, 1499), (8, 128, 32, 48, 600), (4, 256, 16, 40, 860)])
def test_soft_max_fallback_triple(orc, nkv, hd, nh, T, n_past):
    """kq = mul_mat(k, q); soft_max_ext(kq, causal mask, 1/sqrt(HD)); mul_mat(v^T, kq) with the permute:
    the reference's non-FA attention, end to end, against the oracle's attention and sv_flash_attn_ext."""
    S = n_past + T
    kb, kd = cache(orc, 100 + hd, S, nkv * hd)
    vb, vd = cache(orc, 200 + hd, S, nkv * hd)
    q16 = orc.normal_f16(101, T, T * nh * hd).reshape(T, nh, hd)
    qd = torch.from_numpy(q16.view(np.float16)).to(DEV)
    mask = np.zeros((T, S), np.float32)
    for t in range(T):
        mask[t, n_past + t + 1:] = -np.inf
    m16 = torch.from_numpy(mask.astype(np.float16)).to(DEV)
    scale = 1 / np.sqrt(hd)
    kq = sv.mul_mat_kq(kd, qd, nkv, hd, S)                       # [NH, T, S]
    probs = sv.soft_max_ext(kq.view(nh * T, S), m16, scale=scale).view(nh, T, S)
    out = sv.mul_mat_kqv(vd, probs, nkv, hd, S).cpu().numpy()    # [T, NH, HD]
    ref = orc.attn(orc.f16_to_f32(q16), kb.view(np.uint8), vb.view(np.uint8), orc.TYPE_F16, nkv, hd, S, scale,
                   orc.MASK_CAUSAL, n_past)
    close(out, ref)
    fa = sv.flash_attn_ext(qd, kd, vd, m16, scale, nkv, hd, S).cpu().numpy()
    close(out, fa)


def test_mul_mat_rejects_unsupported():
    L = sv.lib()
    k = torch.zeros((64, 8 * 128), dtype=torch.float16, device=DEV)
    q = torch.zeros((1, 32, 128), dtype=torch.float16, device=DEV)
    o = torch.zeros((32, 1, 64), dtype=torch.float32, device=DEV)
    # head_dim 96 is not a multiple of 64; misaligned row stride; G > 16
    assert L.sv_mul_mat_kq(k.data_ptr(), 8 * 96 * 2, 8, 96, 64, q.data_ptr(), 1, 32 * 96 * 2, 96 * 2, 1, 32,
                           o.data_ptr(), None) == -1
    assert L.sv_mul_mat_kq(k.data_ptr(), 8 * 128 * 2 + 2, 8, 128, 64, q.data_ptr(), 1, 32 * 256, 256, 1, 32,
                           o.data_ptr(), None) == -2
    assert L.sv_mul_mat_kq(k.data_ptr(), 8 * 128 * 2, 1, 128, 64, q.data_ptr(), 1, 32 * 256, 256, 1, 32,
                           o.data_ptr(), None) == -1
    assert L.sv_mul_mat_kqv_workspace(8, 128, 1500, 1, 32) > 0
