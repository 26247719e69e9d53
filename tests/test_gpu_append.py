"""K/V append on the GPU (ggml_set_rows / cpy-into-view) against the oracle: bit-exact.

Covers f16 -> f16 (byte copy), f32 -> f16 (RNE), f16/f32 -> q8_0 (ggml block
rounding, pinned to gguf-py by test_oracle_golden), the row-scatter and the
contiguous-base forms, out-of-range rows (skipped + error bit, where ggml
asserts), ragged widths and the BASELINE geometries.
"""
import numpy as np
import pytest
import torch

from __graft_entry__ import load_package

sv = load_package()
pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _src(orc, seed, n_rows, ne0, src_type, outliers=0.0):
    bits = orc.normal_f16(seed, 7, n_rows * ne0, outlier_frac=outliers).reshape(n_rows, ne0)
    if src_type == orc.TYPE_F16:
        return bits.view(np.float16), bits.view(np.uint8).reshape(n_rows, -1)
    f = orc.f16_to_f32(bits) * np.float32(1.37)          # f32 values that are not f16-exact
    return f, f.view(np.uint8).reshape(n_rows, -1)


@pytest.mark.parametrize("dst_type", [1, 8])
@pytest.mark.parametrize("src_type", [0, 1])
@pytest.mark.parametrize("ne0,n_rows,dst_rows", [(1024, 1024, 4096), (1024, 1, 4096), (96, 37, 64), (64, 5, 9)])
def test_set_rows_scatter(orc, dst_type, src_type, ne0, n_rows, dst_rows):
    if dst_type == 8 and ne0 % 32:
        pytest.skip("q8_0 rows need ne0 % 32 == 0")
    rng = np.random.default_rng(ne0 + n_rows)
    src, src_bytes = _src(orc, n_rows, n_rows, ne0, src_type, outliers=0.01)
    rows = rng.permutation(dst_rows)[:n_rows].astype(np.int32)
    rb = orc.row_bytes(dst_type, ne0)
    init = rng.integers(0, 256, (dst_rows, rb), dtype=np.uint8)
    ref = init.copy()
    assert orc.set_rows(ref, dst_type, ne0, src_bytes, src_type, rows=rows) == 0
    dst = torch.from_numpy(init).to(DEV)
    s = torch.from_numpy(np.ascontiguousarray(src)).to(DEV)
    r = torch.from_numpy(rows).to(DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    sv.set_rows(dst, dst_type, ne0, s, rows=r, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert np.array_equal(dst.cpu().numpy(), ref)


@pytest.mark.parametrize("dst_type", [1, 8])
def test_set_rows_base_form(orc, dst_type):
    ne0, n_rows, dst_rows, base = 1024, 384, 8192, 4096
    src, src_bytes = _src(orc, 3, n_rows, ne0, 1)
    rb = orc.row_bytes(dst_type, ne0)
    ref = np.zeros((dst_rows, rb), np.uint8)
    orc.set_rows(ref, dst_type, ne0, src_bytes, 1, base=base)
    dst = torch.zeros((dst_rows, rb), dtype=torch.uint8, device=DEV)
    sv.set_rows(dst, dst_type, ne0, torch.from_numpy(src).to(DEV), base=base)
    torch.cuda.synchronize()
    assert np.array_equal(dst.cpu().numpy(), ref)


def test_set_rows_out_of_range_row_is_skipped(orc):
    ne0, dst_rows = 64, 8
    src, src_bytes = _src(orc, 4, 3, ne0, 1)
    rows = np.array([1, 8, -1], dtype=np.int32)          # two rows outside [0, 8)
    dst = torch.zeros((dst_rows, 128), dtype=torch.uint8, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    sv.set_rows(dst, 1, ne0, torch.from_numpy(src).to(DEV), rows=torch.from_numpy(rows).to(DEV), err=err)
    torch.cuda.synchronize()
    assert int(err.item()) & sv.DEVERR_ROW_RANGE
    got = dst.cpu().numpy()
    ref = np.zeros((dst_rows, 128), np.uint8)
    ref[1] = src_bytes[0]
    assert np.array_equal(got, ref)
    # the contiguous form checks on the host: overflow status
    with pytest.raises(sv.SvError) as e:
        sv.set_rows(dst, 1, ne0, torch.from_numpy(src).to(DEV), base=6)
    assert e.value.status == -5


@pytest.mark.parametrize("kv_type,nkv,hd", [(1, 8, 128), (8, 4, 256), (1, 2, 16)])
def test_kv_append_layer(orc, kv_type, nkv, hd):
    kv = sv.KvCache()
    assert kv.alloc(0, 3, nkv, hd, 512, kv_type)
    ne0 = nkv * hd
    k, kb = _src(orc, 10, 100, ne0, 1, outliers=0.01)
    v, vb = _src(orc, 11, 100, ne0, 1, outliers=0.01)
    rows = np.random.default_rng(1).permutation(512)[:100].astype(np.int32)
    kv.append(1, torch.from_numpy(k).to(DEV), torch.from_numpy(v).to(DEV), rows=torch.from_numpy(rows).to(DEV))
    # contiguous decode-style append on another layer
    kv.append(2, torch.from_numpy(k[:1]).to(DEV), torch.from_numpy(v[:1]).to(DEV), base=300)
    torch.cuda.synchronize()
    rb = orc.row_bytes(kv_type, ne0)
    for layer, isv, src, rr, base in ((1, 0, kb, rows, 0), (1, 1, vb, rows, 0), (2, 0, kb[:1], None, 300)):
        ref = np.zeros((512, rb), np.uint8)
        orc.set_rows(ref, kv_type, ne0, src, 1, rows=rr, base=base)
        assert np.array_equal(kv.tensor(layer, isv).cpu().numpy(), ref)
    assert not kv.tensor(0, 0).cpu().numpy().any()          # untouched layer stays zero
    assert kv.error_flags() == 0
    kv.clear()
    torch.cuda.synchronize()
    assert not kv.tensor(1, 0).cpu().numpy().any()
    kv.free()
