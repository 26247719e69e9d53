"""CPU-side checks of the product library (no GPU needed).

* libsvkv.so loads and exports every function include/svkv.h declares;
* the host-only entry points behave like the reference: the splice predicate
  (qwen3vl_model.cpp:1165-1171) and the session window rule
  (qwen3vl_model.cpp:1110-1124) against the oracle's restatement;
* creating a cache without a device fails with a status, not a crash.
"""
import ctypes

import numpy as np
import pytest

from __graft_entry__ import load_package

sv = load_package()


def test_library_exports_header():
    L = sv.lib()
    names = sv.header_functions()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    assert L.sv_version() >= 100
    assert L.sv_status_string(-5) == b"context overflow"


@pytest.mark.parametrize("case", [
    ([1, 2, 3], 3, [1, 2, 3, 4, 5], 3),    # strict extension -> splice, skip 3
    ([1, 2, 3], 3, [1, 2, 3], 0),          # not longer -> no splice
    ([1, 2, 3], 2, [1, 2, 3, 4], 0),       # kv_len != n_past
    ([1, 2, 3], 3, [1, 9, 3, 4], 0),       # prefix differs
    ([], 0, [1, 2], 0),                    # empty cache
])
def test_splice_predicate(case, orc):
    cached, n_past, ids, want = case
    assert sv.can_splice(cached, n_past, ids) == want
    assert orc.can_splice(cached, n_past, ids) == bool(want)


def test_splice_random(orc):
    rng = np.random.default_rng(5)
    for _ in range(300):
        n = int(rng.integers(0, 20))
        cached = rng.integers(0, 4, n)
        ids = np.concatenate([cached, rng.integers(0, 4, int(rng.integers(0, 5)))])
        if rng.random() < 0.3 and ids.size:
            ids[int(rng.integers(0, ids.size))] ^= 1
        n_past = n if rng.random() < 0.8 else n + 1
        got = sv.can_splice(cached, n_past, ids)
        assert (got > 0) == orc.can_splice(cached, n_past, ids)
        if got:
            assert got == n


def _drive(sess, ref, turns):
    for frames, text, answer in turns:
        first, kept = sess.begin_turn(frames)
        kept_ref = ref.begin_turn(frames)
        assert kept == kept_ref
        assert first == len(ref.rows())
        sess.end_turn(kept, text, answer)
        ref.end_turn(kept, text, answer)
        assert np.array_equal(sess.rows(), ref.rows())


def test_session_baseline_config3_kept_set(orc):
    """12 rounds of 16 frames x 64 rows + 96 text (+32 answer rows), window 6 rounds."""
    sess = sv.Session(None, max_frames=6 * 16, rows_per_frame=64)
    ref = orc.SessionRows(6 * 16, 64)
    _drive(sess, ref, [(16, 96, 32)] * 12)
    rows = sess.rows()
    assert rows.size == 6 * (16 * 64 + 96 + 32)
    assert rows[0] == 6 * 1152                      # rounds 1..6 were evicted
    assert np.all(np.diff(rows) == 1)              # the kept window is the last six rounds, in order


@pytest.mark.parametrize("seed", range(6))
def test_session_random_turns(seed, orc):
    rng = np.random.default_rng(seed)
    max_frames = int(rng.integers(1, 40))
    rpf = int(rng.integers(1, 9))
    sink = int(rng.integers(0, 12))
    turns = [(int(rng.integers(0, 25)), int(rng.integers(0, 30)), int(rng.integers(0, 20))) for _ in range(30)]
    sess = sv.Session(None, max_frames, rpf, sink)
    ref = orc.SessionRows(max_frames, rpf, sink)
    _drive(sess, ref, turns)
    sess.reset()
    ref = orc.SessionRows(max_frames, rpf, sink)
    _drive(sess, ref, turns[:5])


@pytest.mark.parametrize("seed", range(6))
def test_session_row_budget_random(seed, orc):
    """MossVL's row-budget eviction (session_compact_self) on a host-only session against the
    oracle's restatement: eviction counts, the rope-position shift and the kept-row map."""
    rng = np.random.default_rng(100 + seed)
    sink = int(rng.integers(0, 64))
    n_ctx = int(rng.integers(sink + 400, 4096))
    sess = sv.Session(None, max_frames=1, rows_per_frame=1, sink_rows=sink)
    ref = orc.RowBudgetSession(sink)
    for _ in range(60):
        need = int(rng.integers(1, 700))
        want = ref.make_room(need, n_ctx)
        if want is None:                       # the reference refuses: context overflow
            with pytest.raises(sv.SvError) as ex:
                sess.make_room(need, n_ctx)
            assert ex.value.status == -5          # SV_ERR_OVERFLOW
            break
        ev, shift = sess.make_room(need, n_ctx)
        assert ev == want and shift == ref.rdelta
        sess.push_rows(need)
        ref.push(need)
        assert np.array_equal(sess.rows(), np.array(ref.rows, dtype=np.int64))


def test_session_row_budget_refuses_turn_sessions():
    sess = sv.Session(None, max_frames=4, rows_per_frame=2)
    sess.begin_turn(1)
    with pytest.raises(sv.SvError):
        sess.make_room(10, 100)
    sess.end_turn(1, 3, 2)
    with pytest.raises(sv.SvError):
        sess.push_rows(5)
    sess.reset()
    assert sess.make_room(10, 100) == (0, 0)


def test_create_without_gpu_reports_status():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = ctypes.c_void_p()
    rc = sv.lib().sv_kv_create(0, 1, 8, 128, 64, sv.TYPE_F16, ctypes.byref(h))
    assert rc in (-3, -4)
    assert not h.value
    kv = sv.KvCache()
    assert kv.alloc(0, 1, 8, 128, 64) is False


def test_invalid_arguments_rejected():
    L = sv.lib()
    assert L.sv_kv_destroy(None) == -1
    assert L.sv_attn(None, 0, None, 1, 1, 32, 0, 1.0, None, None) == -1
    assert L.sv_set_rows(None, 1, 16, 4, 32, None, 1, 32, 1, None, 0, None, None) == -1


def test_peer_and_projection_arguments_rejected():
    """The peer-group and sharded-projection entry points refuse bad arguments before any CUDA call
    (world outside 1..8, rank outside the world, no slots, slot sizes that are not 16-byte multiples,
    null handles)."""
    L = sv.lib()
    h = ctypes.c_void_p()
    for dev, rank, world, n_slots, slot_bytes in [(0, 0, 0, 1, 16), (0, 0, 9, 1, 16), (0, 2, 2, 1, 16),
                                                  (0, -1, 2, 1, 16), (0, 0, 1, 0, 16), (0, 0, 1, 1, 10),
                                                  (0, 0, 1, 1, 0)]:
        assert L.sv_peer_create(dev, rank, world, n_slots, slot_bytes, ctypes.byref(h)) == -1
        assert not h.value
    assert L.sv_peer_create(0, 0, 1, 1, 16, None) == -1
    assert L.sv_peer_destroy(None) == 0
    assert L.sv_peer_wait(None, 0, None, 1, None, None) == -1
    assert L.sv_out_proj_peer(None, None, 1, 8192, None, 4096, 0, 4096, 2560, 1, 0, None, None, None, None) == -1
    assert L.sv_qk_norm_rope_append(None, 0, None, None, None, 1, 32, None, None, 1e-6, None, None, 0, None, None,
                                    1, None) == -1
