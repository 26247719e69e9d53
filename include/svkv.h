/*
 * svkv.h - C ABI of the B200 (sm_100a) text-decoder KV-cache library.
 *
 * Drop-in for the per-layer ggml ops SkyVision.cpp's decoders emit on the KV
 * path (reference paths relative to the SkyVision.cpp checkout):
 *
 *   ggml_set_rows(kv.k[il], k2, pos_slot)      src/core/blocks/llm_block.hpp:227-233,
 *                                              src/models/qwen3vl/qwen3vl_model.cpp:652-655
 *   ggml_cpy(src, ggml_view(cache, base..))    src/core/engine/stage_buf.hpp:53-56 (view sink form)
 *   ggml_flash_attn_ext(qf, kf, vf, mask, ..)  llm_block.hpp:239-277, qwen3vl_model.cpp:657-663
 *   mul_mat / soft_max_ext / mul_mat           src/models/gemma4/gemma4_model.cpp:683-692
 *   vqa::KvCache alloc/clear/free              src/core/engine/attention.hpp:19-56
 *   set_causal_mask / set_window_mask          attention.hpp:60-83 (in-kernel predicates here)
 *   KV splice predicate                        qwen3vl_model.cpp:1165-1171
 *   window eviction + in-place compaction      qwen3vl_model.cpp:1110-1124, moss_vl_model.cpp:264-291
 *
 * Conventions
 *   - Every function returns an int status: SV_OK (0) or a negative SV_ERR_*.
 *     No exception crosses this boundary.
 *   - Device pointers are plain pointers into the device the handle lives on;
 *     `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *     Calls are asynchronous on that stream unless documented otherwise.
 *   - Nothing on the per-token path allocates: workspaces are reserved when a
 *     handle is created (or passed in by the caller for the raw ggml-op forms).
 *   - A handle is not thread-safe (vqa::Model is single-threaded per instance,
 *     src/core/vqa.hpp:121-123); distinct handles are independent.
 *   - Type ids are ggml's: F32 = 0, F16 = 1, Q8_0 = 8.
 *   - Layout is ggml's: a cache tensor is [n_kv_head*head_dim, n_ctx], i.e.
 *     token-major rows of n_kv_head*head_dim elements (q8_0: blocks of 32
 *     int8 + one f16 scale, 34 bytes per block).
 */
#ifndef SVKV_H
#define SVKV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status */
#define SV_OK 0
#define SV_ERR_INVALID (-1)      /* bad argument (null handle, bad shape, ...) */
#define SV_ERR_UNSUPPORTED (-2)  /* shape/type combination this build does not implement */
#define SV_ERR_CUDA (-3)         /* a CUDA runtime/driver call failed */
#define SV_ERR_NOMEM (-4)        /* device allocation failed (KvCache::alloc returning false) */
#define SV_ERR_OVERFLOW (-5)     /* context overflow: rows beyond n_ctx (qwen3vl_model.cpp:719) */
#define SV_ERR_WORKSPACE (-6)    /* caller workspace too small */
#define SV_ERR_DEVICE (-7)       /* a kernel reported an error bit (see sv_kv_error) */

#define SV_TYPE_F32 0
#define SV_TYPE_F16 1
#define SV_TYPE_Q8_0 8

/* mask modes of the attention entry points */
#define SV_MASK_NONE 0      /* every key of the view is visible */
#define SV_MASK_CAUSAL 1    /* key s visible to query t iff s <= base + t (set_causal_mask) */
#define SV_MASK_WINDOW 2    /* s in [lo[t], hi[t]) or s == own[t] (set_window_mask) */
#define SV_MASK_EXPLICIT 3  /* additive f16 mask [S, T] (ggml's mask argument) */

/* device error bits reported by sv_kv_error / the err_flag word */
#define SV_DEVERR_ROW_RANGE 1   /* a set_rows target row was out of range; that row was skipped */
#define SV_DEVERR_TIMEOUT 2     /* a bounded on-device wait expired; the kernel unwound */
#define SV_DEVERR_SEGMENT 4     /* a compaction segment pointed outside the cache */

/* Human-readable name of a status code. */
const char* sv_status_string(int status);
/* Library ABI version (major*10000 + minor*100 + patch). */
int sv_version(void);

/* ================================================================ KV store
 * Replaces vqa::KvCache (src/core/engine/attention.hpp:19-56): n_layer pairs
 * of [n_kv_head*head_dim, n_ctx] K/V tensors in one device buffer, zero-filled
 * at creation.  kv_type is SV_TYPE_F16 (the reference's only cache type) or
 * SV_TYPE_Q8_0 (head_dim a multiple of 32).  The handle also owns the attention
 * workspace (split-K partials) and a device error word.
 */
typedef struct sv_kv sv_kv;

/* KvCache::alloc (attention.hpp:25-46).  Prints "kv cache: %.2f GB" to stderr
 * like the reference.  SV_ERR_NOMEM when the buffer cannot be allocated. */
int sv_kv_create(int device, int n_layer, int n_kv_head, int head_dim, int n_ctx, int kv_type,
                 sv_kv** out);
/* KvCache::free (attention.hpp:52-55). */
int sv_kv_destroy(sv_kv* kv);
/* KvCache::clear (attention.hpp:48-50): zero every K/V tensor (async). */
int sv_kv_clear(sv_kv* kv, void* stream);
/* kv.k[layer] / kv.v[layer] (attention.hpp:21): device pointer and row bytes,
 * for callers that build ggml-style views themselves. */
int sv_kv_tensor(const sv_kv* kv, int layer, int is_v, void** data, size_t* row_bytes);
/* Shape of the cache. Any output pointer may be NULL. */
int sv_kv_info(const sv_kv* kv, int* n_layer, int* n_kv_head, int* head_dim, int* n_ctx, int* kv_type);
/* Read and clear the device error word (synchronises `stream`).  *flags gets
 * the SV_DEVERR_* bits raised since the last call. */
int sv_kv_error(sv_kv* kv, int* flags, void* stream);

/* ================================================================ append
 * ggml_set_rows(dst, src, rows) (llm_block.hpp:232-233) and the
 * ggml_cpy-into-view form (rows == NULL: row i goes to base + i).
 *   dst   [ne0, dst_rows] of dst_type (F16, Q8_0 or F32), row stride dst_nb1 bytes
 *   src   [ne0, n_rows]   of src_type (F16 or F32),        row stride src_nb1 bytes
 *   rows  device int32 [n_rows] or NULL
 * f16 -> f16 is a byte copy, f32 -> f16 rounds to nearest even, and any -> q8_0
 * uses ggml's block_q8_0 rounding (d = amax/127 in f32, q = round-half-away(x/d),
 * d stored as f16).  A row outside [0, dst_rows) is skipped and raises
 * SV_DEVERR_ROW_RANGE in *err_flag (device int, may be NULL) -- ggml asserts there.
 */
int sv_set_rows(void* dst, int dst_type, int64_t ne0, int64_t dst_rows, size_t dst_nb1,
                const void* src, int src_type, size_t src_nb1, int64_t n_rows,
                const int32_t* rows, int64_t base, int* err_flag, void* stream);

/* Both set_rows of one decoder layer in one launch
 * (ggml_set_rows(kv.k[il], k2, pos_slot) + ggml_set_rows(kv.v[il], v2, pos_slot),
 * qwen3vl_model.cpp:654-655).  k/v: device [n_rows][n_kv_head*head_dim] of
 * src_type; rows: device int32 [n_rows] or NULL for base + i.
 * SV_ERR_OVERFLOW when rows == NULL and base + n_rows > n_ctx. */
int sv_kv_append(sv_kv* kv, int layer, const void* k, const void* v, int src_type, int n_rows,
                 const int32_t* rows, int base, void* stream);

/* sv_kv_append with the first row read on the device from *base_dev when the
 * kernel runs (rows *base_dev .. *base_dev + n_rows - 1; a row past n_ctx is
 * skipped and raises SV_DEVERR_ROW_RANGE).  With sv_attn_at and
 * sv_counter_add this makes a whole decode step capturable in one CUDA graph
 * that is replayed unchanged every token -- the purpose of the reference's
 * static decode graph (src/core/engine/decode_graph.hpp:66-102), without its
 * 512/1024-row bucket of masked keys. */
int sv_kv_append_at(sv_kv* kv, int layer, const void* k, const void* v, int src_type, int n_rows,
                    const int32_t* base_dev, void* stream);

/* counter_dev[i] += delta for i < n, on the stream (advances device-side n_past
 * values / per-session window ends between replays of a captured step). */
int sv_counter_add(int32_t* counter_dev, int n, int delta, void* stream);

/* ================================================================ attention
 * ggml_flash_attn_ext(q, k, v, mask, scale, max_bias = 0, softcap = 0)
 * (llm_block.hpp:268-277) with the reference's views spelled out as ggml
 * ne/nb arrays:
 *   q   [HD, T, NH]   F32 or F16   (qf = view of q3 with nb1 and nb2 swapped)
 *   k,v [HD, S, NKV]  F16 or Q8_0  (nb1 = cache row stride, nb2 = one head's bytes)
 *   mask F16 [S, >=T] additive, row stride mask_nb1 bytes, or NULL
 *   dst F32 [HD, NH, T] contiguous
 * GQA maps query head h to kv head h / (NH/NKV).  A query row that sees no key
 * gets zeros.  Only max_bias == 0 and logit_softcap == 0 are supported (the
 * only values the reference passes).  The workspace holds split-K partials:
 * size it with sv_flash_attn_ext_workspace; a smaller one gives fewer splits,
 * ws_bytes == 0 runs unsplit.
 */
typedef struct sv_fa_params {
    const void* q;    int q_type;  int64_t q_ne[3];  size_t q_nb[3];
    const void* k;    int k_type;  int64_t k_ne[3];  size_t k_nb[3];
    const void* v;    int v_type;  int64_t v_ne[3];  size_t v_nb[3];
    const void* mask; int64_t mask_ne1;  size_t mask_nb1;
    float scale;
    float max_bias;
    float logit_softcap;
    float* dst;
} sv_fa_params;

size_t sv_flash_attn_ext_workspace(const sv_fa_params* p);
int sv_flash_attn_ext(const sv_fa_params* p, void* workspace, size_t ws_bytes, void* stream);

/* sv_flash_attn_ext without a workspace argument: the split-K scratch is a
 * 4 MiB static device array inside this library (held by every GPU that loads
 * it until the process exits), for callers that cannot allocate device memory
 * where attention runs -- e.g. an operator inside a ggml backend graph, which
 * receives only its tensors, or code running during CUDA stream capture.
 * No counterpart in the reference.  The first call on a device resolves the
 * array's address (cudaGetSymbolAddress) with that device current: make it
 * before any stream capture.  Shapes that need more than 4 MiB of scratch
 * return SV_ERR_WORKSPACE.  The array is shared by all calls and keeps the last
 * call's contents (the merge tickets are cleared on each call); calls that
 * overlap on the GPU race.  The cached address belongs to the device's primary
 * context: after cudaDeviceReset (or any reset of that context) the library
 * must be unloaded and loaded again before this entry point is used. */
int sv_flash_attn_ext_static(const sv_fa_params* p, void* stream);

/* Cache-level attention for one decoder layer (the FA node of
 * qwen3vl_model.cpp:657-663 with the causal mask of set_causal_mask(mask,
 * n_past, T) computed in-kernel): query t (0 <= t < T) attends cache rows
 * [0, n_past + t].  q: device [T][n_head][head_dim] of q_type (F16/F32);
 * out: device f32 [T][n_head][head_dim].  Single-token decode (T = 1) runs the
 * split-K flash-decode kernel; chunks with T > 16/(NH/NKV) queries run the
 * chunked-prefill kernel. */
int sv_attn(sv_kv* kv, int layer, const void* q, int q_type, int T, int n_head, int n_past,
            float scale, float* out, void* stream);

/* sv_attn with n_past read on the device from *n_past_dev when the kernel runs
 * (graph-stable form; see sv_kv_append_at).  max_keys >= n_past + T bounds the
 * keys any replay may attend and sizes the grid; CTAs past the live length
 * exit at once, so no masked key is read. */
int sv_attn_at(sv_kv* kv, int layer, const void* q, int q_type, int T, int n_head, const int32_t* n_past_dev,
               int max_keys, float scale, float* out, void* stream);

/* The two ops a decoder layer emits per token fused into one kernel: the K/V
 * append (ggml_set_rows of k_new/v_new at rows *n_past_dev + t,
 * qwen3vl_model.cpp:654-655) and the causal attention over the cache including
 * those rows (qwen3vl_model.cpp:657-663).  k_new/v_new: device f16
 * [T][n_kv_head*head_dim].  f16 caches with T*(n_head/n_kv_head) <= 16, and
 * q8_0 caches at head_dim 256 with T*(n_head/n_kv_head) <= 4 (16-byte aligned
 * sources), run as one kernel: the CTA that covers a new row writes it to the
 * cache (q8_0: quantised with the same steps as sv_set_rows, bytes identical)
 * and uses it from shared memory; other cases run sv_kv_append_at then
 * sv_attn_at.  Graph-stable like sv_attn_at. */
int sv_attn_append_at(sv_kv* kv, int layer, const void* q, int q_type, const void* k_new, const void* v_new, int T,
                      int n_head, const int32_t* n_past_dev, int max_keys, float scale, float* out, void* stream);

/* Multi-session attention over one shared cache (vc3_batch.inc:145-172 with
 * set_window_mask, attention.hpp:71-83): query i attends rows [lo[i], hi[i])
 * plus row own[i].  lo/hi/own: device int32 [n_q]; max_span: an upper bound
 * on max_i(hi[i] - lo[i]) (sizes the grid).  q/out as in sv_attn with T = n_q. */
int sv_attn_window(sv_kv* kv, int layer, const void* q, int q_type, int n_q, int n_head,
                   const int32_t* lo, const int32_t* hi, const int32_t* own, int max_span,
                   float scale, float* out, void* stream);

/* ggml_soft_max_ext(x, mask, scale, max_bias = 0) of the mul_mat fallback
 * (gemma4_model.cpp:685-691): y[r] = softmax(x[r]*scale + mask[r % mask_rows]).
 * x, y: f32 rows of ne0 (strides in bytes); mask: F16 rows or NULL. */
int sv_soft_max_ext(const float* x, int64_t ne0, int64_t n_rows, size_t x_nb1, const void* mask,
                    int64_t mask_rows, size_t mask_nb1, float scale, float* y, size_t y_nb1,
                    void* stream);

/* The two mul_mat legs of that fallback (gemma4_model.cpp:685-691; moondream.cpp:476-493 runs
 * them per head: n_kv_head = n_head = 1 over a one-head view), on the tensor cores.
 *
 * sv_mul_mat_kq replaces kq = ggml_mul_mat(kf, qf) (gemma4_model.cpp:685): the raw scores
 *   kq[s, t, h] = sum_e k[e, s, h / (NH/NKV)] * q[e, t, h]   (ggml's broadcast of src0 over dim 2)
 *   k   F16 cache view [HD, S, NKV]: key s of kv head g at k + s*k_nb1 + g*HD*2 (heads packed in
 *       the row; k and k_nb1 16-byte aligned)
 *   q   [HD, T, NH] of q_type (F16 or F32): element (e, t, h) at q + t*q_nb1 + h*q_nb2 + e*size
 *       (16-byte aligned rows); an F32 query is rounded to f16 first, as ggml converts src1 to
 *       the f16 vec-dot type of an F16 src0
 *   kq  F32 [S, T, NH], contiguous (ggml's mul_mat result)
 * head_dim 64, 128 or 256; n_head / n_kv_head <= 16. */
int sv_mul_mat_kq(const void* k, size_t k_nb1, int n_kv_head, int head_dim, int n_keys, const void* q, int q_type,
                  size_t q_nb1, size_t q_nb2, int T, int n_head, float* kq, void* stream);

/* sv_mul_mat_kqv replaces vt = ggml_cont(ggml_transpose(vf)); kqv = ggml_mul_mat(vt, kq)
 * (gemma4_model.cpp:689-690) and the permute + cont after it (:691), reading V in its cache
 * layout (the transposed copy is never made):
 *   kqv[e, t, h] = sum_s v[e, s, h / (NH/NKV)] * kq[s, t, h]
 *   v   F16 cache view [HD, S, NKV], laid out like k above
 *   kq  F32 [S, T, NH]: (s, t, h) at kq + t*kq_nb1 + h*kq_nb2 + 4*s (any row stride)
 *   dst F32: (e, t, h) at dst + t*dst_nb1 + h*dst_nb2 + 4*e (16-byte aligned): ggml's
 *       [HD, T, NH] result is dst_nb1 = HD*4, dst_nb2 = T*HD*4; the permuted [HD, NH, T] that
 *       gemma4 reshapes to [NH*HD, T] is dst_nb1 = NH*HD*4, dst_nb2 = HD*4
 * kq enters the tensor core as f16 hi + lo parts (~22 bits kept).  The key range is split over
 * the SMs when `workspace` holds sv_mul_mat_kqv_workspace(...) bytes (0 = unsplit; a smaller
 * workspace gives fewer splits).  head_dim 64, 128 or 256; n_head / n_kv_head <= 16. */
size_t sv_mul_mat_kqv_workspace(int n_kv_head, int head_dim, int n_keys, int T, int n_head);
int sv_mul_mat_kqv(const void* v, size_t v_nb1, int n_kv_head, int head_dim, int n_keys, const float* kq,
                   size_t kq_nb1, size_t kq_nb2, int T, int n_head, float* dst, size_t dst_nb1, size_t dst_nb2,
                   void* workspace, size_t ws_bytes, void* stream);

/* ================================================================ eviction
 * In-HBM, order-preserving compaction of every layer's K and V
 * (the row move of kv_shift_rows, moss_vl_model.cpp:264-291, driven by the
 * qwen3vl window rule, qwen3vl_model.cpp:1110-1124).  The cache rows
 * [0, n_rows_used) are described by consecutive segments {src, n_rows, keep};
 * kept segments are packed, in order, starting at dst_base (the destination of
 * each kept row is dst_base + exclusive prefix sum of kept lengths).  Rows
 * only move towards the front.  *new_len = dst_base + total kept rows.
 * The segment table is host memory (the host owns the turn table). */
typedef struct sv_segment {
    int32_t src;     /* first cache row of the segment */
    int32_t n_rows;  /* rows in the segment */
    int32_t keep;    /* nonzero: the segment survives */
} sv_segment;

int sv_kv_compact(sv_kv* kv, const sv_segment* segs, int n_segs, int dst_base, int* new_len,
                  void* stream);

/* ================================================================ session
 * Host-side KV bookkeeping of a streaming session (Qwen3VL's s_kv_ids /
 * s_turns / n_past, qwen3vl_model.cpp:167-181).  The frames of a turn occupy
 * rows_per_frame cache rows each, followed by the turn's text rows and its
 * answer rows; an optional sink prefix [0, sink_rows) is never evicted.
 */
typedef struct sv_session sv_session;

/* The splice predicate (qwen3vl_model.cpp:1167-1169): 1 if the cache holds
 * exactly `cached` (kv_len == n_past) and `ids` strictly extends it, else 0.
 * *skip (may be NULL) gets kv_len when splicing. Pure host function. */
int sv_can_splice(const int32_t* cached, int64_t kv_len, int64_t n_past, const int32_t* ids,
                  int64_t n_ids, int64_t* skip);

/* kv may be NULL: the session then only plans rows (no device work). */
int sv_session_create(sv_kv* kv, int max_frames, int rows_per_frame, int sink_rows, sv_session** out);
int sv_session_destroy(sv_session* s);
/* session_reset (qwen3vl_model.cpp:1059-1064): forget turns and rows (no device work). */
int sv_session_reset(sv_session* s);
/* Start a turn that brings n_new_frames frames: applies the window rule to the
 * completed turns plus the new frames and compacts the cache when rows leave.
 * *first_row gets the cache row where the new turn's rows start (the new
 * n_past); *kept_new_frames how many of the new frames survive the window. */
int sv_session_begin_turn(sv_session* s, int n_new_frames, int* first_row, int* kept_new_frames,
                          void* stream);
/* Close the turn: frames actually written, and the text / answer rows that
 * followed them. */
int sv_session_end_turn(sv_session* s, int frames, int text_rows, int answer_rows);
/* Current row count and the kept-row map: rows_out[i] = the original (never
 * compacted) row id of cache row i, i < *n_rows (max_rows caps the copy). */
int sv_session_rows(const sv_session* s, int* n_rows, int64_t* rows_out, int max_rows);

/* ---------------------------------------------------------------- q/k norm + RoPE fused into the append
 * Rotary modes, ggml's type ids: NEOX rotates pairs (i, i + n_dims/2) at one position per token
 * (ggml_rope_ext, e.g. gemma4_model.cpp:640-642); IMROPE is Qwen3-VL's interleaved multi-axis
 * form (ggml_rope_multi with GGML_ROPE_TYPE_IMROPE, qwen3vl_model.cpp:644-650): pair i takes its
 * position from stream h when i % 3 == 1 and i < 3*sections[1], from w when i % 3 == 2 and
 * i < 3*sections[2], from t when i % 3 == 0 and i < 3*sections[0], else from the fourth stream
 * (i counted modulo the section sum), with NEOX pairing. */
#define SV_ROPE_NONE 0
#define SV_ROPE_NEOX 2
#define SV_ROPE_IMROPE 40

typedef struct sv_rope {
    int mode;          /* SV_ROPE_NONE / SV_ROPE_NEOX / SV_ROPE_IMROPE */
    int n_dims;        /* rotated dims: head_dim, or head_dim / 2 for head_dim 128 / 256 */
    float freq_base;   /* theta = pos * freq_base^(-2i / n_dims) */
    int sections[4];   /* IMROPE: t, h, w, extra pair counts (Qwen3-VL: 24, 20, 20, 0) */
} sv_rope;

/* The ops of a decoder layer between the QKV projection and the attention
 * (qwen3vl_model.cpp:636-655): per-head RMSNorm of q and k times their weights
 * (ggml_rms_norm + ggml_mul; q_norm / k_norm NULL = no norm, eps as
 * rms_norm_eps), the rotary embedding of q and k, and ggml_set_rows of k and
 * v into the cache at rows slot_base + t (or *slot_base_dev + t when
 * slot_base_dev is set, graph-stable like sv_kv_append_at), in one launch.
 * q, k, v: device f32 [T][n_head | n_kv_head][head_dim] (the projections'
 * outputs); pos: device int32 [T] (NEOX) or [4][T] (IMROPE: t, h, w, extra
 * streams, the reference's mpos layout, qwen3vl_model.cpp:602-605);
 * rope NULL or mode SV_ROPE_NONE = no rotation.  q_out gets the rotated
 * queries, [T][n_head][head_dim] in q_out_type (SV_TYPE_F16 or SV_TYPE_F32),
 * for sv_attn*.  Cache rows are f16 (RNE) or q8_0 with sv_set_rows's exact
 * quantisation.  head_dim 64 / 128 / 256.  A row outside the cache is not
 * written and sets the device error bit SV_DEVERR_ROW_RANGE. */
int sv_qk_norm_rope_append(sv_kv* kv, int layer, const float* q, const float* k, const float* v, int T, int n_head,
                           const float* q_norm, const float* k_norm, float eps, const sv_rope* rope,
                           const int32_t* pos, int slot_base, const int32_t* slot_base_dev, void* q_out,
                           int q_out_type, void* stream);

/* Row-budget sessions (MossVL's streaming self-KV, moss_vl_model.cpp:250-292):
 * the cache holds a pinned sink prefix and a sliding window of rows, with no
 * turn table (these calls return SV_ERR_INVALID once sv_session_begin_turn has
 * been used, until sv_session_reset).
 *
 * sv_session_make_room replaces session_compact_self (moss_vl_model.cpp:275-292):
 * before `need` new rows are written, if rows + need exceed the capacity
 * (capacity rows, or the cache's n_ctx when 0), the oldest rows after the sink
 * leave in multiples of 128, never touching the newest 256 rows; the survivors
 * move down in place (sv_kv_compact, every layer's K and V) instead of the
 * reference's host round trip per tensor (kv_shift_rows, :264-271).
 * *evicted gets the rows removed now, *rope_shift the total removed since the
 * reset, which the caller adds to a new row's slot to get its rope position
 * (the reference's sess_rdelta += evict, :287).  SV_ERR_OVERFLOW when even the
 * largest eviction cannot make room (the reference's `false`).  Either pointer
 * may be NULL. */
int sv_session_make_room(sv_session* s, int need, int capacity, int* evicted, int64_t* rope_shift, void* stream);
/* Record n rows written after the current rows (n_past += n in the reference). */
int sv_session_push_rows(sv_session* s, int n);

/* ---------------------------------------------------------------- head-sharded decode, gather fused in
 * One session too long for one GPU's bandwidth shards by kv head (rank g holds kv heads
 * [g*NKV/G, (g+1)*NKV/G) and their query heads).  The reference-side design gathers each layer's
 * [T, NH/G, HD] outputs with an all-gather after attention; here the attention kernel's output
 * stores go straight into every rank's gathered buffer over NVLink (CUDA IPC peer memory) and count
 * themselves on every rank's arrival counter.  No reference counterpart (the reference runs one
 * process per model, qwen3vl_model.cpp:657-663); replaces the NCCL all-gather of this build's
 * sharded decode.
 *
 * sv_peer_create allocates this rank's gathered buffer (n_slots regions of slot_bytes, one per
 * layer, rows [T][n_head_total][HD] f32) and its counters; sv_peer_export writes its IPC handle
 * (SV_PEER_HANDLE_BYTES); after exchanging handles (any host channel), sv_peer_import opens every
 * rank's buffer (handles in rank order).  sv_attn_append_at_peer is sv_attn_append_at for this
 * rank's n_head heads whose output rows land at head_offset of slot `slot` on every rank; when
 * wait_slot >= 0 it first waits (bounded, on the device) until slot wait_slot holds the current
 * epoch's rows from every rank (the previous layer's gather).  *epoch_dev counts steps from 1 and is
 * advanced by the caller after each step (sv_counter_add).  sv_peer_wait is that wait alone.
 * f16 caches, head_dim 64/128, T * (n_head / n_kv_head) <= 8; otherwise SV_ERR_UNSUPPORTED. */
#define SV_PEER_HANDLE_BYTES 64
typedef struct sv_peer sv_peer;
int sv_peer_create(int device, int rank, int world, int n_slots, size_t slot_bytes, sv_peer** out);
int sv_peer_export(const sv_peer* p, void* handle);
int sv_peer_import(sv_peer* p, const void* handles);
int sv_peer_slot(const sv_peer* p, int slot, void** data);
int sv_peer_wait(sv_peer* p, int slot, const int32_t* epoch_dev, int per_epoch, int* err_dev, void* stream);
int sv_peer_destroy(sv_peer* p);

/* The step after attention, head-sharded (qwen3vl_model.cpp:664-667, attn = mul_mat(L.o, attn)):
 * rank g multiplies its heads' attention rows x (T rows of K_local elements, f16 or f32, row
 * stride x_nb_t bytes) by its column slice [k_offset, k_offset + K_local) of the f16 projection
 * w (D rows of K_total, 16-byte aligned), and the ranks' partials are summed into out (f32
 * [T][D]) on every rank, in rank order, so every rank gets the same bits.  One kernel: the
 * partials go into every rank's slot `slot` over peer memory.  With slot_bytes >= world * T * D * 8
 * each partial travels as one 64-bit word holding the value and the current epoch, and each rank
 * polls the words it needs until they carry this epoch (no counters, no fences); with
 * world * T * D * 4 <= slot_bytes < world * T * D * 8 the partials are f32 and counted on every
 * rank's per-band counter.  Either way each rank waits (bounded, on the device; err_dev, may be
 * NULL, gets SV_DEVERR_TIMEOUT) for the current epoch's partials of all ranks, then sums.  Every
 * rank calls it with the same D, T and slot, and the same slot_bytes.  Like the attention gather,
 * each slot is used once per epoch (one slot per layer; *epoch_dev counts steps from 1 and the
 * caller advances it after each step), so consecutive calls use different slots.  T <= 8,
 * K_local <= 4096 and multiples of 8, D <= 18944.  w is read before the kernel's dependency on
 * the previous kernel of the stream: weights written on the GPU must be complete before that
 * kernel starts.  The grid is at most one CTA per SM of the device and every CTA waits for the same
 * band of every rank, so all CTAs must be resident at once: a process restricted to a share of the
 * SMs (MPS, green contexts) gets SV_DEVERR_TIMEOUT instead of a result.  If one rank's wait for its
 * own weight rows expires, it does not count its band (or store its words) on any rank, so every
 * rank reports SV_DEVERR_TIMEOUT (no rank sums a stale partial); the peer group must then be recreated.
 * No reference counterpart (the
 * reference runs one process per model); replaces an NCCL all-gather of the attention rows
 * followed by the full projection on every rank. */
int sv_out_proj_peer(sv_peer* p, const void* x, int x_type, int64_t x_nb_t, const void* w, int K_total, int k_offset,
                     int K_local, int D, int T, int slot, const int32_t* epoch_dev, float* out, int* err_dev,
                     void* stream);
int sv_attn_append_at_peer(sv_kv* kv, int layer, const void* q, int q_type, const void* k_new, const void* v_new,
                           int T, int n_head, const int32_t* n_past_dev, int max_keys, float scale, sv_peer* peer,
                           int head_offset, int n_head_total, int slot, int wait_slot, const int32_t* epoch_dev,
                           void* stream);

/* ================================================================ failure detection
 * Every on-device wait of the library is bounded; on expiry the kernel sets
 * SV_DEVERR_TIMEOUT in its error word and unwinds instead of hanging.  This
 * self-test runs a one-warp kernel whose wait can never complete, with a limit
 * of limit_us microseconds (<= 1 s): afterwards *err_dev has SV_DEVERR_TIMEOUT
 * set and *reached_end_dev (may be NULL) is 1 (the kernel returned past the
 * expired wait).  The reference has no device-side failure detection (errors
 * are bool returns, src/core/engine/attention.hpp:38-42, qwen3vl_model.cpp:743). */
int sv_selftest_wait_timeout(int* err_dev, int* reached_end_dev, unsigned limit_us, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* SVKV_H */
