"""The session rows of the path pinned to the reference's own code (CPU).

The window rule (qwen3vl_model.cpp:1110-1124), the splice predicate
(qwen3vl_model.cpp:1169-1171) and MossVL's row budget with its row move
(moss_vl_model.cpp:264-292) are compiled from the reference's own lines by
oracle/ref_build.py.  Here the oracle's restatements and the library's host
bookkeeping (sv_can_splice, sv_session_* with no cache) are checked against

* the golden vectors that build made (tests/golden/ref_session.npz, always), and
* the build itself on fresh random cases (when oracle/_ref holds it: a
  checkout of the reference was available when the repository was built).

Row layout.  The reference rebuilds its prompt from the surviving turns; the
library keeps their cache rows instead.  A surviving frame keeps its rows
(rows_per_frame each), and a surviving turn keeps its frames' rows, then its
text and answer rows, in turn order; the expected row ids below are derived
from the reference's surviving frame ids (s_marks) and turns in that layout.
"""
import os

import numpy as np
import pytest

from __graft_entry__ import load_package

sv = load_package()
HERE = os.path.dirname(os.path.abspath(__file__))
RPF = 3          # rows per frame used to lay the reference's frames out as rows


@pytest.fixture(scope="module")
def gold():
    return np.load(os.path.join(HERE, "golden", "ref_session.npz"))


@pytest.fixture(scope="module")
def ref():
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_ref_session_golden",
                                                  os.path.join(HERE, "golden", "make_ref_session_golden.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    from oracle import ref_build
    if not os.path.exists(ref_build.LIB):
        pytest.skip("oracle/_ref/libref_session.so not built (no reference checkout when building)")
    L = m.load_ref()
    if L is None:
        pytest.skip("reference session library unavailable")
    return m, L


# ------------------------------------------------------------------ window rule
def expected_rows(turns, states, t):
    """Row ids after turn t is answered, from the reference's state after its frames arrived.

    Row ids are handed out in write order: when turn u is answered, its surviving new frames
    (the marks no earlier turn claims) get RPF rows each, then its text rows, then its answer rows."""
    rows_of_frame, text_rows, next_id = {}, {}, 0
    for u in range(t + 1):
        marks, frames, tags = states[u]
        claimed = int(frames.sum())
        for f in marks[claimed:]:
            rows_of_frame[int(f)] = list(range(next_id, next_id + RPF))
            next_id += RPF
        n_text = turns[u][1] + turns[u][2]
        text_rows[u] = list(range(next_id, next_id + n_text))
        next_id += n_text
    marks, frames, tags = states[t]
    out, pos = [], 0
    for fr, tag in zip(frames, tags):
        for f in marks[pos:pos + fr]:
            out += rows_of_frame[int(f)]
        pos += fr
        out += text_rows[int(tag)]
    for f in marks[pos:]:
        out += rows_of_frame[int(f)]
    out += text_rows[t]
    return np.array(out, np.int64)


def check_window(max_frames, turns, states, orc):
    sess = sv.Session(None, max_frames=max_frames, rows_per_frame=RPF)
    rs = orc.SessionRows(max_frames, RPF)
    for t, (n_new, text, answer) in enumerate(turns):
        marks, frames, _ = states[t]
        kept_ref = len(marks) - int(frames.sum())       # the new frames that survive the window
        first, kept = sess.begin_turn(n_new)
        assert kept == kept_ref, (t, kept, kept_ref)
        assert rs.begin_turn(n_new) == kept_ref
        sess.end_turn(kept, text, answer)
        rs.end_turn(kept, text, answer)
        want = expected_rows(turns, states, t)
        assert np.array_equal(sess.rows(), want), t
        assert np.array_equal(rs.rows(), want), t


def gold_window_states(gold, ci):
    turns = [tuple(int(x) for x in r) for r in gold[f"win{ci}_turns"]]
    states = [(gold[f"win{ci}_t{t}_marks"], gold[f"win{ci}_t{t}_frames"], gold[f"win{ci}_t{t}_tags"])
              for t in range(len(turns))]
    return int(gold[f"win{ci}_max"]), turns, states


def test_window_rule_vs_reference_vectors(gold, orc):
    for ci in range(int(gold["win_n"])):
        max_frames, turns, states = gold_window_states(gold, ci)
        check_window(max_frames, turns, states, orc)


def test_window_rule_vs_reference_build(ref, orc):
    m, L = ref
    rng = np.random.default_rng(101)
    for _ in range(60):
        max_frames = int(rng.choice([1, 2, 5, 16, 40]))
        turns = [(int(rng.integers(0, 3 * max_frames + 2)), int(rng.integers(0, 30)), int(rng.integers(0, 9)))
                 for _ in range(int(rng.integers(1, 16)))]
        check_window(max_frames, turns, m.ref_window(L, max_frames, turns), orc)


def test_reference_vectors_match_the_build(gold, ref):
    """The committed vectors are what the reference build returns (regenerated inputs)."""
    m, L = ref
    for ci in range(int(gold["win_n"])):
        max_frames, turns, states = gold_window_states(gold, ci)
        for (a, b, c), (x, y, z) in zip(m.ref_window(L, max_frames, turns), states):
            assert np.array_equal(a, x) and np.array_equal(b, y) and np.array_equal(c, z)


# ------------------------------------------------------------------ splice predicate
def test_splice_vs_reference_vectors(gold, orc):
    for ci in range(int(gold["spl_n"])):
        cached, n_past, ids = gold[f"spl{ci}_cached"], int(gold[f"spl{ci}_npast"]), gold[f"spl{ci}_ids"]
        want = int(gold[f"spl{ci}_out"])
        got = sv.can_splice(cached, n_past, ids)
        assert (got > 0) == bool(want), ci
        if want:
            assert got == cached.size
        assert orc.can_splice(cached, n_past, ids) == bool(want)


def test_splice_vs_reference_build(ref, orc):
    m, L = ref
    rng = np.random.default_rng(102)
    for _ in range(500):
        n = int(rng.integers(0, 25))
        cached = rng.integers(0, 3, n).astype(np.int32)
        ids = np.concatenate([cached, rng.integers(0, 3, int(rng.integers(0, 4)))]).astype(np.int32)
        if rng.random() < 0.3 and ids.size:
            ids = ids[: int(rng.integers(0, ids.size + 1))].copy()
        if rng.random() < 0.3 and ids.size:
            ids[int(rng.integers(0, ids.size))] ^= 1
        n_past = n if rng.random() < 0.8 else n + int(rng.integers(-2, 3))
        want = m.ref_splice(L, cached, n_past, ids)
        assert (sv.can_splice(cached, n_past, ids) > 0) == bool(want)
        assert orc.can_splice(cached, n_past, ids) == bool(want)


# ------------------------------------------------------------------ row budget (MossVL)
def check_row_budget(n_ctx, sink, bursts, ref_state, ref_rows, orc):
    """ref_state[i] = (ok, n_past, rdelta) after burst i; ref_rows = surviving ids at the end."""
    sess = sv.Session(None, max_frames=1, rows_per_frame=1, sink_rows=sink)
    rb = orc.RowBudgetSession(sink)
    rb.push(0)
    for i, need in enumerate(bursts):
        ok, n_past, rdelta = (int(x) for x in ref_state[i])
        want = rb.make_room(int(need), n_ctx)
        if not ok:
            assert want is None
            with pytest.raises(sv.SvError):
                sess.make_room(int(need), n_ctx)
            assert len(rb.rows) == n_past and rb.rdelta == rdelta
            continue
        ev, shift = sess.make_room(int(need), n_ctx)
        assert ev == want and shift == rdelta == rb.rdelta
        sess.push_rows(int(need))
        rb.push(int(need))
        assert len(rb.rows) == n_past and sess.rows().size == n_past
    assert np.array_equal(np.array(rb.rows) % 65536, ref_rows)
    assert np.array_equal(sess.rows() % 65536, ref_rows)


def test_row_budget_vs_reference_vectors(gold, orc):
    for ci in range(int(gold["rb_n"])):
        n_ctx, sink = (int(x) for x in gold[f"rb{ci}_cfg"])
        check_row_budget(n_ctx, sink, gold[f"rb{ci}_bursts"], gold[f"rb{ci}_state"], gold[f"rb{ci}_rows"], orc)


def test_row_budget_and_row_move_vs_reference_build(ref, orc):
    """session_compact_self on host tensors (kv_shift_rows as memcpy) against the restatement's
    eviction counts and kept rows, and its moved bytes against the oracle's compaction (the
    checker of the GPU compaction kernel) applied to the same tensors."""
    m, L = ref
    rng = np.random.default_rng(103)
    for n_ctx, sink in ((1500, 0), (3000, 77), (900, 300)):
        bursts = [int(rng.integers(1, 400)) for _ in range(25)]
        res, ks, vs = m.ref_row_budget(L, n_ctx, sink, bursts)
        state = np.array([(ok, n_past, rd) for ok, n_past, rd, _ in res])
        check_row_budget(n_ctx, sink, bursts, state, res[-1][3], orc)
    # the row move itself: random bytes, one session_compact_self, vs orc.compact_rows
    n_ctx, sink, row_elems = 2048, 40, 16
    ks = [rng.integers(0, 65536, (n_ctx, row_elems), dtype=np.uint16) for _ in range(2)]
    before = [k.copy() for k in ks]
    import ctypes
    kp = (ctypes.c_void_p * 2)(*[k.ctypes.data for k in ks])
    vs = [k.copy() for k in ks]
    vp = (ctypes.c_void_p * 2)(*[v.ctypes.data for v in vs])
    h = L.ref_moss_new(2, n_ctx, row_elems, kp, vp, sink)
    try:
        L.ref_moss_push(h, 2000)
        assert L.ref_moss_compact(h, 300) == 1
        n_past, rd = ctypes.c_int(), ctypes.c_int()
        L.ref_moss_state(h, ctypes.byref(n_past), ctypes.byref(rd))
    finally:
        L.ref_moss_free(h)
    evict = rd.value
    keep = np.concatenate([np.arange(sink), np.arange(sink + evict, 2000)]).astype(np.int32)
    for k_ref, k0 in zip(ks, before):
        mine = k0.copy()
        orc.compact_rows(mine.view(np.uint8).reshape(n_ctx, -1), keep, 0)
        assert np.array_equal(mine[:n_past.value], k_ref[:n_past.value])
