"""skyvision.cpp_b200 -- B200 (sm_100a) text-decoder KV-cache path of SkyVision.cpp.

Python view of the C ABI in include/svkv.h (libsvkv.so, built in-tree by
``make -C skyvision.cpp_b200``).  The classes mirror the reference's host
interface for this path:

* ``KvCache``     -> vqa::KvCache (src/core/engine/attention.hpp:19-56):
                     ``alloc`` returns False on failure like the reference, ``clear``, ``free``;
                     ``append`` is the pair of ggml_set_rows of a layer (qwen3vl_model.cpp:652-655);
                     ``attn`` the ggml_flash_attn_ext over the cache (qwen3vl_model.cpp:657-663).
* ``set_rows``    -> ggml_set_rows / ggml_cpy into a view (llm_block.hpp:227-233).
* ``flash_attn_ext`` -> ggml_flash_attn_ext(q, k, v, mask, scale, 0, 0) (llm_block.hpp:268-277).
* ``soft_max_ext``   -> ggml_soft_max_ext of the mul_mat fallback (gemma4_model.cpp:683-692).
* ``Session``     -> Qwen3VL's session bookkeeping: window eviction + compaction
                     (qwen3vl_model.cpp:1110-1124, moss_vl_model.cpp:264-291).
* ``can_splice``  -> the KV splice predicate (qwen3vl_model.cpp:1165-1171).

Device memory, streams and process groups come from PyTorch; the C ABI only
sees raw pointers and sizes.  There is no CPU fallback: if libsvkv.so is
missing or a CUDA call fails, these functions raise.
"""
from __future__ import annotations

import ctypes
import os
import re
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libsvkv.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "svkv.h")

TYPE_F32, TYPE_F16, TYPE_Q8_0 = 0, 1, 8
MASK_NONE, MASK_CAUSAL, MASK_WINDOW, MASK_EXPLICIT = 0, 1, 2, 3
DEVERR_ROW_RANGE, DEVERR_TIMEOUT, DEVERR_SEGMENT = 1, 2, 4
OK = 0
STATUS = {0: "ok", -1: "invalid", -2: "unsupported", -3: "cuda", -4: "nomem", -5: "overflow",
          -6: "workspace", -7: "device"}

_lib = None


class SvError(RuntimeError):
    def __init__(self, fn: str, status: int):
        super().__init__(f"{fn} failed: {status} ({STATUS.get(status, '?')})")
        self.status = status


def build() -> str:
    """Compile libsvkv.so for sm_100a (nvcc cross-compiles without a GPU)."""
    subprocess.run(["make", "-s", "-C", HERE, "-j8"], check=True)
    return LIB_PATH


def header_functions() -> list[str]:
    """Every function the public header declares."""
    txt = open(HEADER).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(sv_[a-z0-9_]+)\s*\(", txt)))


class _Seg(ctypes.Structure):
    _fields_ = [("src", ctypes.c_int32), ("n_rows", ctypes.c_int32), ("keep", ctypes.c_int32)]


class _Rope(ctypes.Structure):
    _fields_ = [("mode", ctypes.c_int), ("n_dims", ctypes.c_int), ("freq_base", ctypes.c_float),
                ("sections", ctypes.c_int * 4)]


ROPE_NONE, ROPE_NEOX, ROPE_IMROPE = 0, 2, 40


class _FaParams(ctypes.Structure):
    _fields_ = [
        ("q", ctypes.c_void_p), ("q_type", ctypes.c_int), ("q_ne", ctypes.c_int64 * 3), ("q_nb", ctypes.c_size_t * 3),
        ("k", ctypes.c_void_p), ("k_type", ctypes.c_int), ("k_ne", ctypes.c_int64 * 3), ("k_nb", ctypes.c_size_t * 3),
        ("v", ctypes.c_void_p), ("v_type", ctypes.c_int), ("v_ne", ctypes.c_int64 * 3), ("v_nb", ctypes.c_size_t * 3),
        ("mask", ctypes.c_void_p), ("mask_ne1", ctypes.c_int64), ("mask_nb1", ctypes.c_size_t),
        ("scale", ctypes.c_float), ("max_bias", ctypes.c_float), ("logit_softcap", ctypes.c_float),
        ("dst", ctypes.c_void_p),
    ]


def lib() -> ctypes.CDLL:
    """Load libsvkv.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is missing: run `make -C {HERE}` (no CPU fallback exists)")
    L = ctypes.CDLL(LIB_PATH)
    P, I, I64, SZ, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t, ctypes.c_float
    sig = {
        "sv_status_string": (ctypes.c_char_p, [I]),
        "sv_version": (I, []),
        "sv_kv_create": (I, [I, I, I, I, I, I, ctypes.POINTER(P)]),
        "sv_kv_destroy": (I, [P]),
        "sv_kv_clear": (I, [P, P]),
        "sv_kv_tensor": (I, [P, I, I, ctypes.POINTER(P), ctypes.POINTER(SZ)]),
        "sv_kv_info": (I, [P, P, P, P, P, P]),
        "sv_kv_error": (I, [P, ctypes.POINTER(I), P]),
        "sv_set_rows": (I, [P, I, I64, I64, SZ, P, I, SZ, I64, P, I64, P, P]),
        "sv_kv_append": (I, [P, I, P, P, I, I, P, I, P]),
        "sv_kv_append_at": (I, [P, I, P, P, I, I, P, P]),
        "sv_counter_add": (I, [P, I, I, P]),
        "sv_attn_at": (I, [P, I, P, I, I, I, P, I, F, P, P]),
        "sv_attn_append_at": (I, [P, I, P, I, P, P, I, I, P, I, F, P, P]),
        "sv_flash_attn_ext_workspace": (SZ, [ctypes.POINTER(_FaParams)]),
        "sv_flash_attn_ext": (I, [ctypes.POINTER(_FaParams), P, SZ, P]),
        "sv_attn": (I, [P, I, P, I, I, I, I, F, P, P]),
        "sv_attn_window": (I, [P, I, P, I, I, I, P, P, P, I, F, P, P]),
        "sv_soft_max_ext": (I, [P, I64, I64, SZ, P, I64, SZ, F, P, SZ, P]),
        "sv_mul_mat_kq": (I, [P, SZ, I, I, I, P, I, SZ, SZ, I, I, P, P]),
        "sv_mul_mat_kqv_workspace": (SZ, [I, I, I, I, I]),
        "sv_mul_mat_kqv": (I, [P, SZ, I, I, I, P, SZ, SZ, I, I, P, SZ, SZ, P, SZ, P]),
        "sv_kv_compact": (I, [P, ctypes.POINTER(_Seg), I, I, ctypes.POINTER(I), P]),
        "sv_can_splice": (I, [P, I64, I64, P, I64, ctypes.POINTER(I64)]),
        "sv_session_create": (I, [P, I, I, I, ctypes.POINTER(P)]),
        "sv_session_destroy": (I, [P]),
        "sv_session_reset": (I, [P]),
        "sv_session_begin_turn": (I, [P, I, ctypes.POINTER(I), ctypes.POINTER(I), P]),
        "sv_session_end_turn": (I, [P, I, I, I]),
        "sv_session_rows": (I, [P, ctypes.POINTER(I), P, I]),
        "sv_qk_norm_rope_append": (I, [P, I, P, P, P, I, I, P, P, ctypes.c_float, P, P, I, P, P, I, P]),
        "sv_session_make_room": (I, [P, I, I, ctypes.POINTER(I), ctypes.POINTER(ctypes.c_int64), P]),
        "sv_session_push_rows": (I, [P, I]),
        "sv_selftest_wait_timeout": (I, [P, P, ctypes.c_uint, P]),
        "sv_peer_create": (I, [I, I, I, I, SZ, ctypes.POINTER(P)]),
        "sv_peer_export": (I, [P, P]),
        "sv_peer_import": (I, [P, P]),
        "sv_peer_slot": (I, [P, I, ctypes.POINTER(P)]),
        "sv_peer_wait": (I, [P, I, P, I, P, P]),
        "sv_out_proj_peer": (I, [P, P, I, ctypes.c_int64, P, I, I, I, I, I, I, P, P, P, P]),
        "sv_peer_destroy": (I, [P]),
        "sv_attn_append_at_peer": (I, [P, I, P, I, P, P, I, I, P, I, F, P, I, I, I, I, P, P]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


def _check(fn: str, rc: int) -> None:
    if rc != OK:
        raise SvError(fn, rc)


def _ptr(x):
    """Raw address of a torch tensor / int / None."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    return x.data_ptr()


def _stream(stream):
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


class _DevBuf:
    """__cuda_array_interface__ wrapper so torch can view library-owned memory."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3}


def device_view(ptr: int, nbytes: int, device: int):
    import torch
    return torch.as_tensor(_DevBuf(ptr, nbytes), device=f"cuda:{device}")


# =================================================================== KV store
class KvCache:
    """vqa::KvCache: n_layer pairs of [n_kv_head*head_dim, n_ctx] K/V tensors."""

    def __init__(self):
        self.h = None
        self.n_layer = self.n_ctx = self.n_kv_head = self.head_dim = 0
        self.kv_type = TYPE_F16
        self.device = 0

    def alloc(self, device: int, n_layer: int, n_kv_head: int, head_dim: int, n_ctx: int,
              kv_type: int = TYPE_F16) -> bool:
        h = ctypes.c_void_p()
        rc = lib().sv_kv_create(device, n_layer, n_kv_head, head_dim, n_ctx, kv_type, ctypes.byref(h))
        if rc != OK:
            return False
        self.h = h.value
        self.device, self.n_layer, self.n_kv_head, self.head_dim, self.n_ctx = device, n_layer, n_kv_head, head_dim, n_ctx
        self.kv_type = kv_type
        return True

    def free(self) -> None:
        if self.h:
            lib().sv_kv_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass

    def clear(self, stream=None) -> None:
        _check("sv_kv_clear", lib().sv_kv_clear(self.h, _stream(stream)))

    def tensor_ptr(self, layer: int, is_v: bool):
        p = ctypes.c_void_p()
        rb = ctypes.c_size_t()
        _check("sv_kv_tensor", lib().sv_kv_tensor(self.h, layer, int(is_v), ctypes.byref(p), ctypes.byref(rb)))
        return p.value, rb.value

    def tensor(self, layer: int, is_v: bool):
        """torch uint8 view [n_ctx, row_bytes] of kv.k[layer] / kv.v[layer]."""
        p, rb = self.tensor_ptr(layer, is_v)
        return device_view(p, rb * self.n_ctx, self.device).view(self.n_ctx, rb)

    @property
    def row_bytes(self) -> int:
        return self.tensor_ptr(0, False)[1]

    def append(self, layer: int, k, v, rows=None, base: int = 0, stream=None) -> None:
        """set_rows of one layer's K and V: k/v torch [n_rows, n_kv_head*head_dim] f16/f32."""
        import torch
        st = TYPE_F32 if k.dtype == torch.float32 else TYPE_F16
        _check("sv_kv_append", lib().sv_kv_append(self.h, layer, _ptr(k), _ptr(v), st, k.shape[0], _ptr(rows), base,
                                                  _stream(stream)))

    def append_at(self, layer: int, k, v, base_dev, stream=None) -> None:
        """append with the first row read on the device from base_dev (int32 tensor [1])."""
        import torch
        st = TYPE_F32 if k.dtype == torch.float32 else TYPE_F16
        _check("sv_kv_append_at", lib().sv_kv_append_at(self.h, layer, _ptr(k), _ptr(v), st, k.shape[0],
                                                        _ptr(base_dev), _stream(stream)))

    def attn_append_at_peer(self, layer: int, q, k_new, v_new, n_past_dev, max_keys: int, scale: float, peer,
                            head_offset: int, n_head_total: int, slot: int, wait_slot: int, epoch_dev, stream=None):
        """attn_append_at for this rank's heads with the gather fused in: the output rows land at
        head_offset of `peer` slot `slot` on every rank (see Peer)."""
        import torch
        T, NH, HD = q.shape
        qt = TYPE_F32 if q.dtype == torch.float32 else TYPE_F16
        _check("sv_attn_append_at_peer",
               lib().sv_attn_append_at_peer(self.h, layer, _ptr(q), qt, _ptr(k_new), _ptr(v_new), T, NH,
                                            _ptr(n_past_dev), max_keys, scale, peer.h, head_offset, n_head_total,
                                            slot, wait_slot, _ptr(epoch_dev), _stream(stream)))

    def attn_at(self, layer: int, q, n_past_dev, max_keys: int, scale: float, out=None, stream=None):
        """attn with n_past read on the device (graph-capturable)."""
        import torch
        T, NH, HD = q.shape
        if out is None:
            out = torch.empty((T, NH, HD), dtype=torch.float32, device=q.device)
        qt = TYPE_F32 if q.dtype == torch.float32 else TYPE_F16
        _check("sv_attn_at", lib().sv_attn_at(self.h, layer, _ptr(q), qt, T, NH, _ptr(n_past_dev), max_keys, scale,
                                              _ptr(out), _stream(stream)))
        return out

    def attn_append_at(self, layer: int, q, k_new, v_new, n_past_dev, max_keys: int, scale: float, out=None,
                       stream=None):
        """Fused decode step of one layer: append k_new/v_new at *n_past_dev and attend (graph-capturable)."""
        import torch
        T, NH, HD = q.shape
        if out is None:
            out = torch.empty((T, NH, HD), dtype=torch.float32, device=q.device)
        qt = TYPE_F32 if q.dtype == torch.float32 else TYPE_F16
        _check("sv_attn_append_at", lib().sv_attn_append_at(self.h, layer, _ptr(q), qt, _ptr(k_new), _ptr(v_new), T,
                                                            NH, _ptr(n_past_dev), max_keys, scale, _ptr(out),
                                                            _stream(stream)))
        return out

    def attn(self, layer: int, q, n_past: int, scale: float, out=None, stream=None):
        """Causal attention of q [T, n_head, head_dim] over cache rows [0, n_past + t]."""
        import torch
        T, NH, HD = q.shape
        if out is None:
            out = torch.empty((T, NH, HD), dtype=torch.float32, device=q.device)
        qt = TYPE_F32 if q.dtype == torch.float32 else TYPE_F16
        _check("sv_attn", lib().sv_attn(self.h, layer, _ptr(q), qt, T, NH, n_past, scale, _ptr(out), _stream(stream)))
        return out

    def norm_rope_append(self, layer: int, q, k, v, pos, rope=None, q_norm=None, k_norm=None, eps: float = 1e-6,
                         base: int = 0, base_dev=None, q_out=None, stream=None):
        """q/k RMSNorm + rotary embedding + K/V append (sv_qk_norm_rope_append).  q [T, NH, HD],
        k/v [T, NKV, HD] f32; pos int32 [T] (NEOX) or [4, T] (IMROPE); rope = (mode, n_dims,
        freq_base, sections) or None.  Returns the rotated queries (f16 unless q_out is given)."""
        import torch
        T, NH, HD = q.shape
        if q_out is None:
            q_out = torch.empty((T, NH, HD), dtype=torch.float16, device=q.device)
        qt = TYPE_F32 if q_out.dtype == torch.float32 else TYPE_F16
        rp = None
        if rope is not None:
            mode, n_dims, freq_base, sections = rope
            rp = _Rope(mode, n_dims, freq_base, (ctypes.c_int * 4)(*sections))
        _check("sv_qk_norm_rope_append",
               lib().sv_qk_norm_rope_append(self.h, layer, _ptr(q), _ptr(k), _ptr(v), T, NH, _ptr(q_norm), _ptr(k_norm),
                                            eps, ctypes.byref(rp) if rp is not None else None, _ptr(pos), base,
                                            _ptr(base_dev), _ptr(q_out), qt, _stream(stream)))
        return q_out

    def attn_window(self, layer: int, q, lo, hi, own, max_span: int, scale: float, out=None, stream=None):
        """Per-query window attention (multi-session batch): q [n_q, n_head, head_dim]."""
        import torch
        n_q, NH, HD = q.shape
        if out is None:
            out = torch.empty((n_q, NH, HD), dtype=torch.float32, device=q.device)
        qt = TYPE_F32 if q.dtype == torch.float32 else TYPE_F16
        _check("sv_attn_window", lib().sv_attn_window(self.h, layer, _ptr(q), qt, n_q, NH, _ptr(lo), _ptr(hi), _ptr(own),
                                                      max_span, scale, _ptr(out), _stream(stream)))
        return out

    def compact(self, segments, dst_base: int = 0, stream=None) -> int:
        """segments: list of (src, n_rows, keep); returns the new row count."""
        arr = (_Seg * max(len(segments), 1))(*[_Seg(int(s), int(n), int(bool(k))) for s, n, k in segments])
        nl = ctypes.c_int()
        _check("sv_kv_compact", lib().sv_kv_compact(self.h, arr, len(segments), dst_base, ctypes.byref(nl),
                                                    _stream(stream)))
        return nl.value

    def error_flags(self, stream=None) -> int:
        f = ctypes.c_int()
        _check("sv_kv_error", lib().sv_kv_error(self.h, ctypes.byref(f), _stream(stream)))
        return f.value


PEER_HANDLE_BYTES = 64


class Peer:
    """Gathered-output buffers of a head-sharded session shared across ranks (sv_peer_*).

    p = Peer(device, rank, world, n_slots, slot_bytes); handles = all ranks' p.export() (any host
    channel, e.g. torch.distributed.all_gather_object); p.import_handles(handles); then
    KvCache.attn_append_at_peer(...) per layer and p.slot(s) views the gathered rows."""

    def __init__(self, device: int, rank: int, world: int, n_slots: int, slot_bytes: int):
        h = ctypes.c_void_p()
        _check("sv_peer_create", lib().sv_peer_create(device, rank, world, n_slots, slot_bytes, ctypes.byref(h)))
        self.h, self.device, self.rank, self.world = h.value, device, rank, world
        self.n_slots, self.slot_bytes = n_slots, slot_bytes

    def export(self) -> bytes:
        buf = (ctypes.c_char * PEER_HANDLE_BYTES)()
        _check("sv_peer_export", lib().sv_peer_export(self.h, buf))
        return bytes(buf)

    def import_handles(self, handles) -> None:
        blob = b"".join(handles)
        assert len(blob) == PEER_HANDLE_BYTES * self.world
        buf = (ctypes.c_char * len(blob)).from_buffer_copy(blob)
        _check("sv_peer_import", lib().sv_peer_import(self.h, buf))

    def slot(self, s: int, shape=None):
        """torch f32 view of slot s (shape defaults to the whole slot, flat)."""
        import torch
        p = ctypes.c_void_p()
        _check("sv_peer_slot", lib().sv_peer_slot(self.h, s, ctypes.byref(p)))
        t = device_view(p.value, self.slot_bytes, self.device).view(torch.float32)
        return t if shape is None else t[: int(np.prod(shape))].view(*shape)

    def out_proj(self, x, w, k_offset: int, slot: int, epoch_dev, out=None, err=None, stream=None):
        """This rank's output-projection partial x [T, K_local] (f16/f32) @ w[:, k_offset:k_offset+K_local]^T
        (w f16 [D, K_total]), summed over every rank through peer memory (sv_out_proj_peer) -> [T, D] f32."""
        import torch
        T, KL = x.shape
        D, KT = w.shape
        if out is None:
            out = torch.empty((T, D), dtype=torch.float32, device=x.device)
        xt = TYPE_F32 if x.dtype == torch.float32 else TYPE_F16
        _check("sv_out_proj_peer", lib().sv_out_proj_peer(self.h, _ptr(x), xt, x.stride(0) * x.element_size(), _ptr(w),
                                                          KT, k_offset, KL, D, T, slot, _ptr(epoch_dev), _ptr(out),
                                                          _ptr(err), _stream(stream)))
        return out

    def wait(self, s: int, epoch_dev, per_epoch: int, err=None, stream=None) -> None:
        _check("sv_peer_wait", lib().sv_peer_wait(self.h, s, _ptr(epoch_dev), per_epoch, _ptr(err), _stream(stream)))

    def free(self) -> None:
        if self.h:
            lib().sv_peer_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def counter_add(counter, delta: int, stream=None) -> None:
    """counter (int32 device tensor [n]) += delta elementwise, on the stream."""
    _check("sv_counter_add", lib().sv_counter_add(_ptr(counter), counter.numel(), delta, _stream(stream)))


# =================================================================== ggml-op forms
def set_rows(dst, dst_type: int, ne0: int, src, rows=None, base: int = 0, err=None, stream=None,
             dst_rows: int | None = None, dst_nb1: int | None = None) -> None:
    """ggml_set_rows(dst, src, rows): dst torch uint8 [dst_rows, row_bytes]; src torch [n_rows, ne0]."""
    import torch
    st = TYPE_F32 if src.dtype == torch.float32 else TYPE_F16
    n_rows = src.shape[0]
    src_nb1 = src.stride(0) * src.element_size()
    dr = dst.shape[0] if dst_rows is None else dst_rows
    nb1 = dst.stride(0) * dst.element_size() if dst_nb1 is None else dst_nb1
    _check("sv_set_rows", lib().sv_set_rows(_ptr(dst), dst_type, ne0, dr, nb1, _ptr(src), st, src_nb1, n_rows,
                                            _ptr(rows), base, _ptr(err), _stream(stream)))


def flash_attn_ext(q, k, v, mask, scale: float, n_kv_head: int, head_dim: int, n_keys: int, kv_type: int = TYPE_F16,
                   dst=None, workspace=None, stream=None):
    """ggml_flash_attn_ext over cache views.

    q: torch [T, NH, HD] (f16/f32; passed as the [HD, T, NH] view ggml builds)
    k, v: torch uint8 caches [rows >= n_keys, row_bytes]; mask: torch f16 [T, n_keys] or None.
    Returns f32 [T, NH, HD] (ggml's [HD, NH, T])."""
    import torch
    T, NH, HD = q.shape
    es = q.element_size()
    headb = head_dim * 2 if kv_type == TYPE_F16 else head_dim // 32 * 34
    p = _FaParams()
    p.q = _ptr(q)
    p.q_type = TYPE_F32 if q.dtype == torch.float32 else TYPE_F16
    p.q_ne[:] = [HD, T, NH]
    p.q_nb[:] = [es, q.stride(0) * es, q.stride(1) * es]
    for name, t in (("k", k), ("v", v)):
        setattr(p, name, _ptr(t))
        setattr(p, name + "_type", kv_type)
        getattr(p, name + "_ne")[:] = [head_dim, n_keys, n_kv_head]
        getattr(p, name + "_nb")[:] = [2 if kv_type == TYPE_F16 else 1, t.stride(0), headb]
    if mask is not None:
        p.mask = _ptr(mask)
        p.mask_ne1 = mask.shape[0]
        p.mask_nb1 = mask.stride(0) * 2
    p.scale = scale
    if dst is None:
        dst = torch.empty((T, NH, HD), dtype=torch.float32, device=q.device)
    p.dst = _ptr(dst)
    L = lib()
    need = L.sv_flash_attn_ext_workspace(ctypes.byref(p))
    if workspace is None and need > 0:
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    wsb = 0 if workspace is None else workspace.numel() * workspace.element_size()
    _check("sv_flash_attn_ext", L.sv_flash_attn_ext(ctypes.byref(p), _ptr(workspace), wsb, _stream(stream)))
    return dst


def soft_max_ext(x, mask=None, scale: float = 1.0, out=None, stream=None):
    """ggml_soft_max_ext(x, mask, scale, 0): x torch f32 [rows, ne0], mask f16 [mask_rows, ne0]."""
    import torch
    if out is None:
        out = torch.empty_like(x)
    n_rows, ne0 = x.shape
    mrows = 0 if mask is None else mask.shape[0]
    mnb1 = 0 if mask is None else mask.stride(0) * 2
    _check("sv_soft_max_ext", lib().sv_soft_max_ext(_ptr(x), ne0, n_rows, x.stride(0) * 4, _ptr(mask), mrows, mnb1,
                                                    scale, _ptr(out), out.stride(0) * 4, _stream(stream)))
    return out


# =================================================================== session
def mul_mat_kq(k, q, n_kv_head: int, head_dim: int, n_keys: int, out=None, stream=None):
    """ggml_mul_mat(kf, qf) of the soft_max fallback: k is the cache (rows of n_kv_head*head_dim f16,
    any row stride), q [T, NH, HD] f16/f32 (the view's t and h strides are taken from the tensor);
    returns the f32 scores [NH, T, S] (ggml's [S, T, NH])."""
    import torch
    T, NH, HD = q.shape
    assert HD == head_dim
    if out is None:
        out = torch.empty((NH, T, n_keys), dtype=torch.float32, device=q.device)
    qt = TYPE_F32 if q.dtype == torch.float32 else TYPE_F16
    es = q.element_size()
    _check("sv_mul_mat_kq", lib().sv_mul_mat_kq(_ptr(k), k.stride(0) * k.element_size(), n_kv_head, head_dim, n_keys,
                                                _ptr(q), qt, q.stride(0) * es, q.stride(1) * es, T, NH, _ptr(out),
                                                _stream(stream)))
    return out


def mul_mat_kqv(v, kq, n_kv_head: int, head_dim: int, n_keys: int, out=None, stream=None, workspace=True):
    """ggml_mul_mat(ggml_cont(ggml_transpose(vf)), kq) + permute: v the cache, kq f32 [NH, T, S] (any
    t / h strides); returns f32 [T, NH, HD] (the [HD, NH, T] layout the fallback reshapes)."""
    import torch
    NH, T, S = kq.shape
    assert S == n_keys
    if out is None:
        out = torch.empty((T, NH, head_dim), dtype=torch.float32, device=kq.device)
    ws = None
    wsb = 0
    if workspace:
        wsb = lib().sv_mul_mat_kqv_workspace(n_kv_head, head_dim, n_keys, T, NH)
        if wsb:
            ws = torch.empty(wsb, dtype=torch.uint8, device=kq.device)
    _check("sv_mul_mat_kqv", lib().sv_mul_mat_kqv(_ptr(v), v.stride(0) * v.element_size(), n_kv_head, head_dim,
                                                  n_keys, _ptr(kq), kq.stride(1) * 4, kq.stride(0) * 4, T, NH,
                                                  _ptr(out), out.stride(0) * 4, out.stride(1) * 4,
                                                  _ptr(ws) if ws is not None else None, wsb, _stream(stream)))
    return out


def can_splice(cached_ids, n_past: int, ids) -> int:
    """Returns the number of cached rows to skip (0 = no splice)."""
    import numpy as np
    c = np.ascontiguousarray(cached_ids, dtype=np.int32)
    i = np.ascontiguousarray(ids, dtype=np.int32)
    skip = ctypes.c_int64()
    ok = lib().sv_can_splice(c.ctypes.data if c.size else None, c.size, n_past,
                             i.ctypes.data if i.size else None, i.size, ctypes.byref(skip))
    return int(skip.value) if ok else 0


class Session:
    """Streaming-session KV bookkeeping (window eviction + in-place compaction)."""

    def __init__(self, kv: KvCache | None, max_frames: int, rows_per_frame: int, sink_rows: int = 0):
        h = ctypes.c_void_p()
        _check("sv_session_create", lib().sv_session_create(kv.h if kv is not None else None, max_frames,
                                                            rows_per_frame, sink_rows, ctypes.byref(h)))
        self.h = h.value
        self.kv = kv

    def __del__(self):
        try:
            if self.h:
                lib().sv_session_destroy(self.h)
        except Exception:
            pass

    def reset(self) -> None:
        _check("sv_session_reset", lib().sv_session_reset(self.h))

    def begin_turn(self, n_new_frames: int, stream=None):
        fr = ctypes.c_int()
        kept = ctypes.c_int()
        st = _stream(stream) if self.kv is not None else None
        _check("sv_session_begin_turn", lib().sv_session_begin_turn(self.h, n_new_frames, ctypes.byref(fr),
                                                                    ctypes.byref(kept), st))
        return fr.value, kept.value

    def end_turn(self, frames: int, text_rows: int, answer_rows: int) -> None:
        _check("sv_session_end_turn", lib().sv_session_end_turn(self.h, frames, text_rows, answer_rows))

    def make_room(self, need: int, capacity: int = 0, stream=None):
        """Row-budget eviction before `need` new rows (MossVL's session_compact_self): returns
        (rows evicted now, total rope-position shift since the reset)."""
        ev = ctypes.c_int()
        shift = ctypes.c_int64()
        st = _stream(stream) if self.kv is not None else None
        _check("sv_session_make_room", lib().sv_session_make_room(self.h, need, capacity, ctypes.byref(ev),
                                                                  ctypes.byref(shift), st))
        return ev.value, shift.value

    def push_rows(self, n: int) -> None:
        _check("sv_session_push_rows", lib().sv_session_push_rows(self.h, n))

    def rows(self):
        import numpy as np
        n = ctypes.c_int()
        _check("sv_session_rows", lib().sv_session_rows(self.h, ctypes.byref(n), None, 0))
        out = np.zeros(n.value, dtype=np.int64)
        _check("sv_session_rows", lib().sv_session_rows(self.h, ctypes.byref(n), out.ctypes.data, n.value))
        return out
