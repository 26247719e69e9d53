"""Golden vectors for the session rows of the path, made by the reference's own code.

Runs oracle/_ref/libref_session.so -- the reference's window loops, splice
predicate and session_compact_self compiled by oracle/ref_build.py from the
reference checkout -- on seeded random inputs and stores what it returns in
tests/golden/ref_session.npz, so the CPU tests can pin the oracle's
restatements and the library's host bookkeeping to the reference where the
reference checkout is absent.

    python tests/golden/make_ref_session_golden.py [--reference DIR]

Cases (all seeded):
  * window: sequences of turns (new frames, text rows, answer rows) under a
    max_frames window; after each turn's frames arrive the reference's loops
    run, and the surviving frame ids (s_marks) and turns (frames, tag) are
    recorded;
  * splice: cached ids / n_past / new prompt triples (empty cache, equal
    prompt, strict extension, a mismatch at a random position, a stale
    n_past) and the predicate's value;
  * row budget: bursts of `need` rows into an n_ctx cache with a sink; after
    each session_compact_self the return value, n_past, sess_rdelta and the
    ids of the surviving rows (every row's elements hold its id).
"""
from __future__ import annotations

import argparse
import ctypes
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)


def load_ref(reference: str | None = None):
    """The compiled reference session code (builds it when a checkout is given or found)."""
    from oracle import ref_build
    if reference or not os.path.exists(ref_build.LIB):
        ref = reference or os.environ.get("SVKV_REFERENCE") or os.path.join(os.path.dirname(ROOT), "reference")
        ref_build.build(ref, quiet=True)
    if not os.path.exists(ref_build.LIB):
        return None
    L = ctypes.CDLL(ref_build.LIB)
    P, I, I64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
    L.ref_win_new.restype = P
    L.ref_win_new.argtypes = [I]
    L.ref_win_free.argtypes = [P]
    L.ref_win_add_frames.argtypes = [P, P, I]
    L.ref_win_end_turn.argtypes = [P, I64]
    L.ref_win_marks.restype = I
    L.ref_win_marks.argtypes = [P, P, I]
    L.ref_win_turns.restype = I
    L.ref_win_turns.argtypes = [P, P, P, I]
    L.ref_can_splice.restype = I
    L.ref_can_splice.argtypes = [P, I64, I64, P, I64]
    L.ref_moss_new.restype = P
    L.ref_moss_new.argtypes = [I, I, I, P, P, I]
    L.ref_moss_free.argtypes = [P]
    L.ref_moss_compact.restype = I
    L.ref_moss_compact.argtypes = [P, I]
    L.ref_moss_push.argtypes = [P, I]
    L.ref_moss_state.argtypes = [P, ctypes.POINTER(I), ctypes.POINTER(I)]
    return L


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def ref_window(L, max_frames: int, turns):
    """turns: [(n_new_frames, text, answer)].  Returns per turn (marks ids, turn frames, turn tags) after
    the turn's frames arrived and the window ran (before the turn is answered)."""
    w = L.ref_win_new(max_frames)
    out, next_frame = [], 0
    try:
        for t, (n_new, _text, _ans) in enumerate(turns):
            ids = np.arange(next_frame, next_frame + n_new, dtype=np.int64)
            next_frame += n_new
            L.ref_win_add_frames(w, _p(ids), n_new)
            marks = np.zeros(max(next_frame, 1), np.int64)
            nm = L.ref_win_marks(w, _p(marks), marks.size)
            fr = np.zeros(len(turns) + 1, np.int32)
            tg = np.zeros(len(turns) + 1, np.int64)
            nt = L.ref_win_turns(w, _p(fr), _p(tg), fr.size)
            out.append((marks[:nm].copy(), fr[:nt].copy(), tg[:nt].copy()))
            L.ref_win_end_turn(w, t)
    finally:
        L.ref_win_free(w)
    return out


def ref_splice(L, cached, n_past, ids) -> int:
    c = np.ascontiguousarray(cached, np.int32)
    i = np.ascontiguousarray(ids, np.int32)
    return L.ref_can_splice(_p(c), c.size, n_past, _p(i), i.size)


def ref_row_budget(L, n_ctx: int, sink: int, bursts, n_layer: int = 2, row_elems: int = 8):
    """Rows carry their id in every element (uint16); returns per burst (ok, n_past, rdelta, surviving ids)
    and the final K and V tensors."""
    ks = [np.zeros((n_ctx, row_elems), np.uint16) for _ in range(n_layer)]
    vs = [np.zeros((n_ctx, row_elems), np.uint16) for _ in range(n_layer)]
    kp = (ctypes.c_void_p * n_layer)(*[k.ctypes.data for k in ks])
    vp = (ctypes.c_void_p * n_layer)(*[v.ctypes.data for v in vs])
    m = L.ref_moss_new(n_layer, n_ctx, row_elems, kp, vp, sink)
    out = []
    next_id = 0
    n_past = ctypes.c_int(0)
    rd = ctypes.c_int(0)

    def write(first, n):
        nonlocal next_id
        for layer in range(n_layer):
            ks[layer][first:first + n] = np.arange(next_id, next_id + n, dtype=np.uint16)[:, None]
            vs[layer][first:first + n] = (np.arange(next_id, next_id + n, dtype=np.uint16) + 20000)[:, None]
        next_id += n
        L.ref_moss_push(m, n)

    try:
        write(0, sink)
        for need in bursts:
            ok = L.ref_moss_compact(m, int(need))
            L.ref_moss_state(m, ctypes.byref(n_past), ctypes.byref(rd))
            if ok:
                write(n_past.value, int(need))
                L.ref_moss_state(m, ctypes.byref(n_past), ctypes.byref(rd))
            out.append((ok, n_past.value, rd.value, ks[0][:n_past.value, 0].astype(np.int64).copy()))
    finally:
        L.ref_moss_free(m)
    return out, ks, vs


def window_cases(seed: int = 0):
    rng = np.random.default_rng(seed)
    cases = []
    for max_frames in (1, 4, 16, 96):
        for _ in range(6):
            n = int(rng.integers(3, 14))
            turns = [(int(rng.integers(0, 3 * max_frames + 2)), int(rng.integers(0, 40)), int(rng.integers(0, 20)))
                     for _ in range(n)]
            cases.append((max_frames, turns))
    cases.append((96, [(16, 96, 32)] * 12))          # BASELINE config 3's shape (rows per frame scale it)
    return cases


def splice_cases(seed: int = 1):
    rng = np.random.default_rng(seed)
    cases = [(np.zeros(0, np.int32), 0, np.arange(5, dtype=np.int32))]
    for _ in range(40):
        n = int(rng.integers(1, 60))
        cached = rng.integers(0, 50, n).astype(np.int32)
        kind = int(rng.integers(0, 5))
        if kind == 0:
            ids = cached.copy()                                            # not strictly longer
        elif kind == 1:
            ids = np.concatenate([cached, rng.integers(0, 50, int(rng.integers(1, 30)))]).astype(np.int32)
        elif kind == 2:
            ids = np.concatenate([cached, rng.integers(0, 50, 5)]).astype(np.int32)
            ids[int(rng.integers(0, n))] += 1                              # one differing prefix id
        elif kind == 3:
            ids = cached[: int(rng.integers(0, n))].copy()                 # shorter prompt
        else:
            ids = np.concatenate([cached, [7]]).astype(np.int32)
        n_past = n if rng.random() < 0.8 else n + int(rng.integers(-3, 4))
        cases.append((cached, n_past, ids))
    return cases


def row_budget_cases(seed: int = 2):
    rng = np.random.default_rng(seed)
    cases = []
    for n_ctx, sink in ((1024, 0), (2048, 40), (4096, 300), (700, 10)):
        bursts = [int(rng.integers(1, 500)) for _ in range(30)]
        cases.append((n_ctx, sink, bursts))
    return cases


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None, help="reference checkout (else $SVKV_REFERENCE)")
    a = ap.parse_args()
    L = load_ref(a.reference)
    if L is None:
        raise SystemExit("reference session library unavailable: pass --reference")
    d = {}
    for ci, (mf, turns) in enumerate(window_cases()):
        d[f"win{ci}_max"] = np.array(mf)
        d[f"win{ci}_turns"] = np.array(turns, np.int32).reshape(-1, 3)
        for t, (marks, fr, tg) in enumerate(ref_window(L, mf, turns)):
            d[f"win{ci}_t{t}_marks"] = marks
            d[f"win{ci}_t{t}_frames"] = fr
            d[f"win{ci}_t{t}_tags"] = tg
    d["win_n"] = np.array(len(window_cases()))
    for ci, (cached, n_past, ids) in enumerate(splice_cases()):
        d[f"spl{ci}_cached"] = cached
        d[f"spl{ci}_npast"] = np.array(n_past)
        d[f"spl{ci}_ids"] = ids
        d[f"spl{ci}_out"] = np.array(ref_splice(L, cached, n_past, ids))
    d["spl_n"] = np.array(len(splice_cases()))
    for ci, (n_ctx, sink, bursts) in enumerate(row_budget_cases()):
        d[f"rb{ci}_cfg"] = np.array([n_ctx, sink])
        d[f"rb{ci}_bursts"] = np.array(bursts, np.int32)
        res, _, _ = ref_row_budget(L, n_ctx, sink, bursts)
        d[f"rb{ci}_state"] = np.array([(ok, n_past, rd) for ok, n_past, rd, _ in res], np.int64)
        d[f"rb{ci}_rows"] = res[-1][3]
    d["rb_n"] = np.array(len(row_budget_cases()))
    path = os.path.join(HERE, "ref_session.npz")
    np.savez_compressed(path, **d)
    print(f"wrote {path}: {len(d)} arrays")


if __name__ == "__main__":
    main()
