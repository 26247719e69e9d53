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


def test_session_row_budget_stream(orc):
    """MossVL-style streaming (pinned sink + sliding window, moss_vl_model.cpp:250-292) on a real
    cache: rows are appended in bursts, sv_session_make_room evicts in 128-row quanta before each
    burst, and every layer's K and V must hold exactly the oracle's surviving rows in order."""
    rng = np.random.default_rng(7)
    L, NKV, HD, cap, sink = 2, 4, 64, 2048, 40
    kv = sv.KvCache()
    assert kv.alloc(0, L, NKV, HD, cap)
    sess = sv.Session(kv, max_frames=1, rows_per_frame=1, sink_rows=sink)
    ref = orc.RowBudgetSession(sink)
    ne0 = NKV * HD
    # every written row carries its row id as the bit pattern of all its elements (K: id, V: id + 15000,
    # both below the f16 inf/nan patterns), so the cache shows exactly which rows survive
    def write(first_slot, ids):
        bits = np.repeat(np.asarray(ids, np.int16)[:, None], ne0, axis=1)
        kb = torch.from_numpy(bits).to(DEV).view(torch.float16)
        vb = torch.from_numpy(bits + np.int16(15000)).to(DEV).view(torch.float16)
        for layer in range(L):
            kv.append(layer, kb, vb, base=first_slot)
    write(0, list(range(sink)))
    shift_total = 0
    for burst in range(40):
        need = int(rng.integers(20, 400))
        want = ref.make_room(need, cap)
        assert want is not None
        ev, shift = sess.make_room(need)
        assert ev == want and shift == ref.rdelta
        shift_total = shift
        n_past = len(ref.rows)
        write(n_past, list(range(ref.next_id, ref.next_id + need)))
        sess.push_rows(need)
        ref.push(need)
    torch.cuda.synchronize()
    rows = np.array(ref.rows)
    assert np.array_equal(sess.rows(), rows)
    assert shift_total > 0
    want = np.repeat(rows.astype(np.int16)[:, None], ne0, axis=1)
    for layer in range(L):
        k = kv.tensor(layer, 0).view(torch.int16)[: rows.size].cpu().numpy()
        v = kv.tensor(layer, 1).view(torch.int16)[: rows.size].cpu().numpy()
        assert np.array_equal(k, want)
        assert np.array_equal(v, want + np.int16(15000))
    assert kv.error_flags() == 0
