"""Eviction compaction on the GPU: bit-exact against the oracle.

* direct sv_kv_compact on random segment tables (including the many-small-
  shift case that goes through the scratch buffer) vs the oracle's sequential
  memmove (kv_shift_rows semantics, moss_vl_model.cpp:264-271);
* a BASELINE-config-3-shaped session (rounds of frames + text + answer, window
  of 6 rounds) driven through sv_session_*, whose cache must equal the oracle's
  kept rows in order, every layer, K and V.
"""
import numpy as np
import pytest
import torch

from __graft_entry__ import load_package

sv = load_package()
pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _random_cache(kv, rng):
    snap = []
    for layer in range(kv.n_layer):
        for isv in (0, 1):
            t = kv.tensor(layer, isv)
            data = torch.from_numpy(rng.integers(0, 256, tuple(t.shape), dtype=np.uint8)).to(DEV)
            t.copy_(data)
            snap.append(data.cpu().numpy())
    torch.cuda.synchronize()
    return snap


def _segments(rng, n_rows, sink):
    segs, r = [], 0
    if sink:
        segs.append((0, sink, 1))
        r = sink
    while r < n_rows:
        n = int(min(n_rows - r, rng.integers(1, 300)))
        segs.append((r, n, int(rng.random() < 0.6)))
        r += n
    return segs


@pytest.mark.parametrize("seed", range(4))
def test_compact_random_segments(orc, seed):
    rng = np.random.default_rng(seed)
    kv = sv.KvCache()
    assert kv.alloc(0, 2, 8, 128 if seed % 2 == 0 else 64, 3000, sv.TYPE_F16 if seed < 3 else sv.TYPE_Q8_0)
    snap = _random_cache(kv, rng)
    segs = _segments(rng, 2900, sink=int(rng.integers(0, 50)))
    keep = np.concatenate([np.arange(s, s + n) for s, n, k in segs if k] or [np.zeros(0, int)]).astype(np.int32)
    new_len = kv.compact(segs, 0)
    torch.cuda.synchronize()
    assert new_len == keep.size
    for i, ref in enumerate(snap):
        ref = ref.copy()
        orc.compact_rows(ref, keep, 0)
        got = kv.tensor(i // 2, i % 2).cpu().numpy()
        assert np.array_equal(got[:new_len], ref[:new_len])
    assert kv.error_flags() == 0


def test_compact_many_small_shifts_uses_scratch(orc):
    """Evicting every 7th row: shifts of 1..n give far more than 16 waves."""
    kv = sv.KvCache()
    assert kv.alloc(0, 1, 2, 64, 1000)
    rng = np.random.default_rng(9)
    snap = _random_cache(kv, rng)
    segs = []
    for r in range(0, 980, 7):
        segs.append((r, 6, 1))
        segs.append((r + 6, 1, 0))
    keep = np.concatenate([np.arange(s, s + n) for s, n, k in segs if k]).astype(np.int32)
    new_len = kv.compact(segs, 0)
    torch.cuda.synchronize()
    for i, ref in enumerate(snap):
        ref = ref.copy()
        orc.compact_rows(ref, keep, 0)
        assert np.array_equal(kv.tensor(0, i).cpu().numpy()[:new_len], ref[:new_len])


def test_session_config3_shape(orc):
    """12 rounds x (16 frames x 8 rows + 12 text + 4 answer rows), window 6 rounds, 2 layers."""
    rpf, frames, text, answer, rounds = 8, 16, 12, 4, 12
    round_rows = frames * rpf + text + answer
    kv = sv.KvCache()
    assert kv.alloc(0, 2, 8, 128, 8 * round_rows)
    sess = sv.Session(kv, max_frames=6 * frames, rows_per_frame=rpf)
    ref = orc.SessionRows(6 * frames, rpf)
    ne0 = 8 * 128
    written = {}        # original row id -> K/V source row bits per layer
    next_id = 0
    for r in range(rounds):
        first, kept = sess.begin_turn(frames)
        ref.begin_turn(frames)
        n = kept * rpf + text + answer
        for layer in range(2):
            k = orc.normal_f16(2, 1000 * r + layer, n * ne0).reshape(n, ne0)
            v = orc.normal_f16(2, 5000 * r + layer, n * ne0).reshape(n, ne0)
            kv.append(layer, torch.from_numpy(k.view(np.float16)).to(DEV), torch.from_numpy(v.view(np.float16)).to(DEV),
                      base=first)
            for i in range(n):
                written[(layer, next_id + i)] = (k[i], v[i])
        next_id += n
        sess.end_turn(kept, text, answer)
        ref.end_turn(kept, text, answer)
        rows = sess.rows()
        assert np.array_equal(rows, ref.rows())
    torch.cuda.synchronize()
    rows = sess.rows()
    assert rows.size == 6 * round_rows
    for layer in range(2):
        kc = kv.tensor(layer, 0).cpu().numpy().view(np.uint16)
        vc = kv.tensor(layer, 1).cpu().numpy().view(np.uint16)
        for i, rid in enumerate(rows):
            k, v = written[(layer, int(rid))]
            assert np.array_equal(kc[i], k) and np.array_equal(vc[i], v), (layer, i, rid)
    assert kv.error_flags() == 0
