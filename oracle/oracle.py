"""ctypes view of the CPU oracle (svkv_oracle.c).

TEST INFRASTRUCTURE ONLY: the checker for the CUDA library.  Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline / reference arm import this
module; the product path (skyvision.cpp_b200/) never does.

Each function names the reference behaviour it restates; the C file carries the
file:line citations.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libsvkv_oracle.so")

TYPE_F32, TYPE_F16, TYPE_Q8_0 = 0, 1, 8
QK8_0, Q8_0_BYTES = 32, 34
MASK_NONE, MASK_CAUSAL, MASK_WINDOW, MASK_EXPLICIT = 0, 1, 2, 3

_lib = None


def build() -> str:
    """Compile the oracle with its Makefile (gcc, OpenMP)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(
                os.path.join(HERE, "svkv_oracle.c")):
            build()
        L = ctypes.CDLL(LIB_PATH)
        P, I64, I32, F32, U64 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_uint64
        L.orc_f32_to_f16.restype = ctypes.c_uint16
        L.orc_f32_to_f16.argtypes = [F32]
        L.orc_f16_to_f32.restype = F32
        L.orc_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.orc_f32_to_f16_n.argtypes = [P, P, I64]
        L.orc_f16_to_f32_n.argtypes = [P, P, I64]
        L.orc_normal_f16.argtypes = [U64, U64, U64, I64, F32, ctypes.c_double, F32, P]
        L.orc_stream_base.restype = U64
        L.orc_stream_base.argtypes = [U64, U64]
        L.orc_q8_0_row.argtypes = [P, I64, P]
        L.orc_q8_0_dequant_row.argtypes = [P, I64, P]
        L.orc_set_rows.restype = I32
        L.orc_set_rows.argtypes = [P, I32, I64, I64, ctypes.c_size_t, P, I32, ctypes.c_size_t, I64, P, I64]
        L.orc_attn.restype = I32
        L.orc_attn.argtypes = [P, I64, I32, I32, I32, P, P, I32, ctypes.c_size_t, I32, I32,
                               I32, I32, P, P, P, P, I64, F32, P]
        L.orc_soft_max_row.argtypes = [P, P, I32, F32, P]
        L.orc_can_splice.restype = I32
        L.orc_can_splice.argtypes = [P, I64, I64, P, I64]
        L.orc_evict_window.argtypes = [P, P, P, I32, P, P]
        L.orc_compact_rows.restype = I32
        L.orc_compact_rows.argtypes = [P, ctypes.c_size_t, I64, P, I64, I64]
        L.orc_num_threads.restype = I32
        L.orc_set_num_threads.argtypes = [I32]
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


def num_threads() -> int:
    return lib().orc_num_threads()


def set_num_threads(n: int) -> None:
    lib().orc_set_num_threads(int(n))


# ----------------------------------------------------------------- numbers
def f32_to_f16(x) -> np.ndarray:
    """f32 -> f16 bits, round-to-nearest-even (ggml_fp32_to_fp16)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().orc_f32_to_f16_n(_p(x), _p(out), x.size)
    return out


def f16_to_f32(h) -> np.ndarray:
    h = np.ascontiguousarray(h).view(np.uint16)
    out = np.empty(h.shape, dtype=np.float32)
    lib().orc_f16_to_f32_n(_p(h), _p(out), h.size)
    return out


def normal_f16(seed: int, stream: int, n: int, scale: float = 1.0, offset: int = 0,
               outlier_frac: float = 0.0, outlier_mul: float = 8.0) -> np.ndarray:
    """Seeded synthetic values: splitmix64 counter stream + Box-Muller, f16 bits.

    The reference names no generator for the BASELINE configs; this one is the
    documented stand-in (config 4 adds 1% outliers x8)."""
    out = np.empty(int(n), dtype=np.uint16)
    lib().orc_normal_f16(seed, stream, offset, int(n), scale, outlier_frac, outlier_mul, _p(out))
    return out


# ----------------------------------------------------------------- q8_0
def row_bytes(type_: int, ne0: int) -> int:
    if type_ == TYPE_F32:
        return 4 * ne0
    if type_ == TYPE_F16:
        return 2 * ne0
    if type_ == TYPE_Q8_0:
        return ne0 // QK8_0 * Q8_0_BYTES
    raise ValueError(type_)


def q8_0_quantize(x) -> np.ndarray:
    """x f32 [..., ne0] -> ggml block_q8_0 bytes [..., ne0/32*34]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    ne0 = x.shape[-1]
    rows = x.reshape(-1, ne0)
    out = np.empty((rows.shape[0], row_bytes(TYPE_Q8_0, ne0)), dtype=np.uint8)
    L = lib()
    for i in range(rows.shape[0]):
        L.orc_q8_0_row(_p(rows[i]), ne0, _p(out[i]))
    return out.reshape(x.shape[:-1] + (out.shape[-1],))


def q8_0_dequant(b, ne0: int) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint8)
    rows = b.reshape(-1, b.shape[-1])
    out = np.empty((rows.shape[0], ne0), dtype=np.float32)
    L = lib()
    for i in range(rows.shape[0]):
        L.orc_q8_0_dequant_row(_p(rows[i]), ne0, _p(out[i]))
    return out.reshape(b.shape[:-1] + (ne0,))


def dequant_rows(cache: np.ndarray, type_: int, ne0: int) -> np.ndarray:
    """cache bytes [rows, row_bytes] -> f32 [rows, ne0]."""
    if type_ == TYPE_F16:
        return f16_to_f32(np.ascontiguousarray(cache).view(np.uint16).reshape(cache.shape[0], ne0))
    if type_ == TYPE_F32:
        return np.ascontiguousarray(cache).view(np.float32).reshape(cache.shape[0], ne0).copy()
    return q8_0_dequant(cache, ne0)


# ----------------------------------------------------------------- set_rows
def set_rows(dst: np.ndarray, dst_type: int, ne0: int, src: np.ndarray, src_type: int,
             rows=None, base: int = 0) -> int:
    """ggml_set_rows into dst (uint8 [dst_rows, row_bytes], modified in place).

    src: uint8/f16/f32 rows [n_rows, ...] packed; rows None = cpy-into-view at base."""
    dst_rows = dst.shape[0]
    src = np.ascontiguousarray(src)
    n_rows = src.shape[0]
    src_nb1 = src.nbytes // max(n_rows, 1)
    r = None if rows is None else np.ascontiguousarray(rows, dtype=np.int32)
    return lib().orc_set_rows(_p(dst), dst_type, ne0, dst_rows, dst.strides[0],
                              _p(src), src_type, src_nb1, n_rows, _p(r), base)


# ----------------------------------------------------------------- attention
def attn(q: np.ndarray, k: np.ndarray, v: np.ndarray, kv_type: int, n_kv_head: int, head_dim: int,
         n_keys: int, scale: float, mask_mode: int = MASK_CAUSAL, causal_base: int = 0,
         lo=None, hi=None, own=None, mask=None) -> np.ndarray:
    """ggml_flash_attn_ext over a cache view.

    q f32 [T, NH, HD]; k/v cache bytes [rows >= n_keys, row_bytes] (token-major
    [NKV*HD] rows, ggml's [NKV*HD, n_ctx] tensor); returns f32 [T, NH, HD]."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    T, NH, HD = q.shape
    assert HD == head_dim
    k = np.ascontiguousarray(k)
    v = np.ascontiguousarray(v)
    assert k.strides[0] == v.strides[0]
    out = np.empty((T, NH, HD), dtype=np.float32)
    lo_ = None if lo is None else np.ascontiguousarray(lo, dtype=np.int32)
    hi_ = None if hi is None else np.ascontiguousarray(hi, dtype=np.int32)
    own_ = None if own is None else np.ascontiguousarray(own, dtype=np.int32)
    m = None if mask is None else np.ascontiguousarray(mask).view(np.uint16)
    m_nb1 = 0 if m is None else m.shape[-1]
    rc = lib().orc_attn(_p(q), NH * HD, T, NH, HD, _p(k), _p(v), kv_type, k.strides[0],
                        n_kv_head, n_keys, mask_mode, causal_base, _p(lo_), _p(hi_), _p(own_),
                        _p(m), m_nb1, scale, _p(out))
    if rc != 0:
        raise ValueError(f"orc_attn failed: {rc}")
    return out


def soft_max_row(x, mask=None, scale: float = 1.0) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    m = None if mask is None else np.ascontiguousarray(mask).view(np.uint16)
    lib().orc_soft_max_row(_p(x), _p(m), x.size, scale, _p(y))
    return y


def _kv_heads_f64(cache, n_kv_head: int, head_dim: int, n_keys: int) -> np.ndarray:
    """An f16 cache's first n_keys rows as float64 [S, NKV, HD] (exact)."""
    rows = np.ascontiguousarray(cache[:n_keys]).view(np.uint8)
    h = rows[:, : n_kv_head * head_dim * 2].copy().view(np.float16)
    return h.astype(np.float64).reshape(n_keys, n_kv_head, head_dim)


def mul_mat_kq(k, q, n_kv_head: int, head_dim: int, n_keys: int) -> np.ndarray:
    """kq = ggml_mul_mat(kf, qf) of the soft_max fallback (gemma4_model.cpp:685): the raw scores
    kq[h, t, s] = sum_e k[s, h // (NH // NKV), e] * q[t, h, e] -- ggml broadcasts src0's third
    dimension over src1's.  q (f32 [T, NH, HD]) is rounded to f16 first, as ggml converts src1 to
    the vec-dot type of an f16 src0; the sum is taken in float64.  k: f16 cache bytes [rows,
    row_bytes].  Returns f32 [NH, T, S] (ggml's [S, T, NH])."""
    kf = _kv_heads_f64(k, n_kv_head, head_dim, n_keys)
    qf = np.asarray(q, np.float32).astype(np.float16).astype(np.float64)
    T, NH, HD = qf.shape
    g = NH // n_kv_head
    out = np.empty((NH, T, n_keys), np.float64)
    for h in range(NH):
        out[h] = qf[:, h, :] @ kf[:, h // g, :].T
    return out.astype(np.float32)


def mul_mat_kqv(v, kq, n_kv_head: int, head_dim: int, n_keys: int) -> np.ndarray:
    """kqv = ggml_mul_mat(ggml_cont(ggml_transpose(vf)), kq) (gemma4_model.cpp:689-690), then the
    permute to [HD, NH, T] (:691): out[t, h, e] = sum_s v[s, h // (NH // NKV), e] * kq[h, t, s], in
    float64.  v: f16 cache bytes; kq f32 [NH, T, S].  Returns f32 [T, NH, HD]."""
    vf = _kv_heads_f64(v, n_kv_head, head_dim, n_keys)
    p = np.asarray(kq, np.float64)
    NH, T, S = p.shape
    g = NH // n_kv_head
    out = np.empty((T, NH, head_dim), np.float64)
    for h in range(NH):
        out[:, h, :] = p[h] @ vf[:, h // g, :]
    return out.astype(np.float32)


# ----------------------------------------------------------------- q/k norm + rotary embedding
ROPE_NONE, ROPE_NEOX, ROPE_IMROPE = 0, 2, 40


def rms_norm(x, w, eps: float) -> np.ndarray:
    """ggml_rms_norm over the last axis, then ggml_mul by w (qwen3vl_model.cpp:638-642), in float64:
    y = x / sqrt(mean(x^2) + eps) * w (the reference's numpy form, scripts/parity_minicpmo_seg.py:29-30)."""
    x = np.asarray(x, np.float64)
    return x / np.sqrt((x * x).mean(-1, keepdims=True) + eps) * np.asarray(w, np.float64)


def imrope_axis(i: int, sections) -> int:
    """Position stream of rotation pair i in ggml's interleaved MRoPE (GGML_ROPE_TYPE_IMROPE, the
    Qwen3-VL rope of qwen3vl_model.cpp:644-650; ggml-cpu's mrope cache rule, ggml-org/ggml master):
    h when i % 3 == 1 and i < 3*s[1], w when i % 3 == 2 and i < 3*s[2], t when i % 3 == 0 and
    i < 3*s[0], else the fourth stream; i is taken modulo the section sum."""
    sd = sum(sections)
    sec = i % sd if sd > 0 else i
    if sec % 3 == 1 and sec < 3 * sections[1]:
        return 1
    if sec % 3 == 2 and sec < 3 * sections[2]:
        return 2
    if sec % 3 == 0 and sec < 3 * sections[0]:
        return 0
    return 3


def rope(x, pos, mode: int, n_dims: int, freq_base: float, sections=(0, 0, 0, 0)) -> np.ndarray:
    """Rotary embedding of x [T, H, HD] in float64, NEOX pairing (i, i + n_dims/2) as ggml_rope_ext with
    GGML_ROPE_TYPE_NEOX (the reference's numpy form: rope_llm, scripts/parity_minicpmo_seg.py:368-378)
    and ggml_rope_multi with IMROPE.  theta = p * freq_base^(-2i/n_dims) exactly (ggml accumulates it
    by repeated f32 multiplication).  pos: [T] (NEOX) or [4, T] (IMROPE)."""
    x = np.array(x, np.float64)
    if mode == ROPE_NONE:
        return x
    T = x.shape[0]
    half = n_dims // 2
    i = np.arange(half)
    inv = float(freq_base) ** (-2.0 * i / n_dims)
    pos = np.asarray(pos, np.float64)
    if mode == ROPE_IMROPE:
        axis = np.array([imrope_axis(int(k), sections) for k in i])
        p = pos.reshape(4, T)[axis, :].T                 # [T, half]
    else:
        p = np.repeat(pos.reshape(T, 1), half, axis=1)
    th = p * inv[None, :]
    c, s = np.cos(th)[:, None, :], np.sin(th)[:, None, :]
    a, b = x[..., :half].copy(), x[..., half:n_dims].copy()
    x[..., :half] = a * c - b * s
    x[..., half:n_dims] = a * s + b * c
    return x


def qk_norm_rope(q, k, q_norm, k_norm, eps, pos, mode, n_dims, freq_base, sections=(0, 0, 0, 0)):
    """The chain of qwen3vl_model.cpp:636-650 on one chunk: per-head RMSNorm * weight, then rope."""
    qn = rms_norm(q, q_norm, eps) if q_norm is not None else np.asarray(q, np.float64)
    kn = rms_norm(k, k_norm, eps) if k_norm is not None else np.asarray(k, np.float64)
    return (rope(qn, pos, mode, n_dims, freq_base, sections), rope(kn, pos, mode, n_dims, freq_base, sections))


# ----------------------------------------------------------------- session logic
def can_splice(cached_ids, n_past: int, ids) -> bool:
    c = np.ascontiguousarray(cached_ids, dtype=np.int32)
    i = np.ascontiguousarray(ids, dtype=np.int32)
    return bool(lib().orc_can_splice(_p(c), c.size, n_past, _p(i), i.size))


def evict_window(turn_frames, n_marks: int, max_frames: int):
    """qwen3vl window rule -> (kept turn frames, n_marks, drop_turns, drop_frames)."""
    tf = np.ascontiguousarray(turn_frames, dtype=np.int32).copy()
    nt = ctypes.c_int(tf.size)
    nm = ctypes.c_int(n_marks)
    dt = ctypes.c_int(0)
    df = ctypes.c_int(0)
    lib().orc_evict_window(_p(tf) if tf.size else None, ctypes.byref(nt), ctypes.byref(nm), max_frames,
                           ctypes.byref(dt), ctypes.byref(df))
    return tf[: nt.value].copy(), nm.value, dt.value, df.value


class SessionRows:
    """Which cache rows a streaming session keeps, turn by turn.

    Restates Qwen3VL::ask_session's window (qwen3vl_model.cpp:1110-1124,
    likewise MageVL::session_evict, mage_model.cpp:1827-1841) on a KV row
    layout: a pinned prefix of sink rows, then per completed turn its frames
    (rows_per_frame rows each), its text rows and its answer rows.  Dropping a
    turn drops all its rows; trimming a frame (the reference erases the oldest
    mark and decrements the front turn's frame count, clamped at 0) drops that
    frame's rows, or a not-yet-written frame of the new turn when the front
    turn has none left.  Row ids are the order in which rows were first written.
    """

    def __init__(self, max_frames: int, rows_per_frame: int, sink_rows: int = 0):
        self.max_frames = max_frames
        self.rpf = rows_per_frame
        self.sink = list(range(sink_rows))
        self.next_id = sink_rows
        self.turns = []          # dicts: frames (list of row-id lists), text, answer (row-id lists)
        self.marks = 0           # s_marks.size()
        self.pending_new = 0

    def begin_turn(self, n_new: int) -> int:
        self.marks += n_new
        new_kept = n_new
        while self.marks > self.max_frames and len(self.turns) > 1:
            self.marks -= len(self.turns[0]["frames"])
            del self.turns[0]
        while self.marks > self.max_frames:
            self.marks -= 1
            if self.turns and len(self.turns[0]["frames"]) > 0:
                del self.turns[0]["frames"][0]
            else:
                new_kept -= 1
        self.pending_new = new_kept
        return new_kept

    def end_turn(self, frames: int, text: int, answer: int) -> None:
        t = {"frames": [], "text": [], "answer": []}
        for _ in range(frames):
            t["frames"].append(list(range(self.next_id, self.next_id + self.rpf)))
            self.next_id += self.rpf
        t["text"] = list(range(self.next_id, self.next_id + text))
        self.next_id += text
        t["answer"] = list(range(self.next_id, self.next_id + answer))
        self.next_id += answer
        self.marks -= self.pending_new - min(frames, self.pending_new)
        self.turns.append(t)

    def rows(self) -> np.ndarray:
        out = list(self.sink)
        for t in self.turns:
            for f in t["frames"]:
                out += f
            out += t["text"] + t["answer"]
        return np.array(out, dtype=np.int64)


class RowBudgetSession:
    """MossVL's streaming self-KV budget (moss_vl_model.cpp:250-292), restated on a row-id list.

    rows[i] is the original id of cache row i; rows [0, sink) are pinned.  make_room(need, n_ctx)
    follows session_compact_self (:275-292): nothing happens while n_past + need fits; otherwise
    needed_free = n_past + need - n_ctx, evictable = n_past - sink - 256 (recent_floor, :278), and
    evict = min(evictable, needed_free rounded up to 128) rows right after the sink leave
    (kv_shift_rows moves the rest down, :282-285), n_past -= evict, rdelta += evict (:287).  Returns
    the eviction count, or None where the reference returns false (evictable < needed_free).
    """

    def __init__(self, sink_rows: int = 0):
        self.sink = sink_rows
        self.rows = list(range(sink_rows))
        self.next_id = sink_rows
        self.rdelta = 0

    def make_room(self, need: int, n_ctx: int):
        n_past = len(self.rows)
        if n_past + need <= n_ctx:
            return 0
        needed_free = n_past + need - n_ctx
        evictable = n_past - self.sink - 256
        if evictable < needed_free:
            return None
        evict = min(evictable, (needed_free + 127) // 128 * 128)
        del self.rows[self.sink:self.sink + evict]
        self.rdelta += evict
        return evict

    def push(self, n: int) -> None:
        self.rows += list(range(self.next_id, self.next_id + n))
        self.next_id += n


def compact_rows(cache: np.ndarray, keep, dst_base: int) -> None:
    """Order-preserving in-place move of kept rows to dst_base.. (moss_vl kv_shift_rows)."""
    k = np.ascontiguousarray(keep, dtype=np.int32)
    rc = lib().orc_compact_rows(_p(cache), cache.strides[0], cache.shape[0], _p(k), k.size, dst_base)
    if rc != 0:
        raise ValueError("invalid kept-row list")
