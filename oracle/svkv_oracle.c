/*
 * svkv_oracle.c -- CPU restatement of SkyVision.cpp's text-decoder KV-cache path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * library under skyvision.cpp_b200/: only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline / reference arm may load it.  Nothing in the product
 * path links or calls it.
 *
 * The reference runs this path through ggml (ggml-org/ggml, branch master,
 * unpinned, not vendored: CMakeLists.txt:8-69, Dockerfile:36-38), so ggml's
 * arithmetic is restated here from the reference's call sites:
 *
 *   orc_set_rows        ggml_set_rows(cache, src, rows)        src/core/blocks/llm_block.hpp:227-233
 *                       (f32/f16 source, f16 or q8_0 cache; out-of-range rows are
 *                       rejected like ggml's GGML_ASSERT(i1 < ne1))
 *   orc_q8_0_row        ggml block_q8_0 encoder as gguf-py runs it            convert/_lib.py:120-130
 *                       (d = amax/127 in f32, id = 1/d, q = round-half-away(x*id),
 *                       d stored as f16 RNE; pinned against gguf 0.19.0 Q8_0)
 *   orc_attn            ggml_flash_attn_ext(q, k_view, v_view, mask, scale)      llm_block.hpp:268-277,
 *                       qwen3vl_model.cpp:657-663; GQA head map kv = h / (NH/NKV);
 *                       masks: set_causal_mask attention.hpp:60-67, set_window_mask
 *                       attention.hpp:71-83, or an explicit additive f16 mask;
 *                       fp32 accumulation (two-pass softmax per query row; each q.k dot
 *                       product in 8 interleaved partial sums, as ggml's SIMD vec_dot
 *                       keeps several accumulators)
 *   orc_can_splice      KV splice predicate                                  qwen3vl_model.cpp:1165-1171
 *   orc_evict_window    sliding-window kept-set rule                         qwen3vl_model.cpp:1110-1124,
 *                                                                            mage_model.cpp:1827-1841
 *   orc_compact_rows    order-preserving row move (memmove semantics)        moss_vl_model.cpp:264-291
 *   orc_normal_f16      seeded synthetic inputs (splitmix64 + Box-Muller); the
 *                       reference names no generator for these configs, so this
 *                       one is documented and shared with the bench.
 *
 * Build: make -C oracle   (gcc -O3 -fopenmp, no fast-math, no FMA contraction; shared library)
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_TYPE_F32 0
#define ORC_TYPE_F16 1
#define ORC_TYPE_Q8_0 8
#define ORC_QK8_0 32
#define ORC_Q8_0_BYTES 34

#define ORC_MASK_NONE 0
#define ORC_MASK_CAUSAL 1
#define ORC_MASK_WINDOW 2
#define ORC_MASK_EXPLICIT 3

/* ------------------------------------------------------------------ f16 */
/* IEEE binary16 <-> binary32, round-to-nearest-even (the rounding ggml's
 * ggml_fp32_to_fp16 uses on F16C hardware).  Written from the format
 * definition: sign | 5-bit exponent (bias 15) | 10-bit mantissa. */
static inline uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

uint16_t orc_f32_to_f16(float f) {
    const uint32_t x = f32_bits(f);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ex = (x >> 23) & 0xffu;
    uint32_t man = x & 0x7fffffu;
    if (ex == 0xffu) {                       /* inf / nan */
        if (man == 0) return (uint16_t)(sign | 0x7c00u);
        return (uint16_t)(sign | 0x7e00u | (man >> 13));
    }
    const int e = (int)ex - 127 + 15;        /* rebiased exponent */
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);   /* overflow -> inf */
    if (e <= 0) {                            /* f16 subnormal or zero */
        if (e < -10) return (uint16_t)sign;  /* below half the smallest subnormal */
        man |= 0x800000u;                    /* implicit bit */
        const int shift = 14 - e;            /* 13 + (1 - e) */
        uint32_t h = man >> shift;
        const uint32_t rem = man & ((1u << shift) - 1u);
        const uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (h & 1u))) h++;
        return (uint16_t)(sign | h);
    }
    uint32_t h = ((uint32_t)e << 10) | (man >> 13);
    const uint32_t rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;  /* may carry into exponent: still correct */
    return (uint16_t)(sign | h);
}

float orc_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t ex = (h >> 10) & 0x1fu;
    const uint32_t man = h & 0x3ffu;
    if (ex == 0) {
        if (man == 0) return bits_f32(sign);
        /* subnormal: man * 2^-24 */
        float v = (float)man * (1.0f / 16777216.0f);
        return sign ? -v : v;
    }
    if (ex == 31) return bits_f32(sign | 0x7f800000u | (man << 13));
    return bits_f32(sign | ((ex + 112u) << 23) | (man << 13));
}

void orc_f32_to_f16_n(const float* x, uint16_t* y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = orc_f32_to_f16(x[i]);
}
void orc_f16_to_f32_n(const uint16_t* x, float* y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = orc_f16_to_f32(x[i]);
}

/* ------------------------------------------------------------------ rng */
/* splitmix64 finaliser (Steele, Lea, Flood 2014; public-domain constants) used
 * as a counter-based generator: value i of stream s under seed k is
 * mix(base(k, s) + i). */
static inline uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
static inline uint64_t stream_base(uint64_t seed, uint64_t stream) {
    return mix64(seed * 0x9E3779B97F4A7C15ull + stream * 0xD1B54A32D192ED03ull + 0x632BE59BD9B4E019ull);
}

uint64_t orc_stream_base(uint64_t seed, uint64_t stream) { return stream_base(seed, stream); }

/* N(0,1) element i of a stream, in double: Box-Muller on the pair i>>1. */
static double normal_at(uint64_t base, uint64_t i) {
    const uint64_t j = i >> 1;
    const uint64_t a = mix64(base + 2 * j + 1);
    const uint64_t b = mix64(base + 2 * j + 2);
    const double u1 = ((double)(a >> 11) + 1.0) * (1.0 / 9007199254740992.0);   /* (0, 1] */
    const double u2 = (double)(b >> 11) * (1.0 / 9007199254740992.0);           /* [0, 1) */
    const double r = sqrt(-2.0 * log(u1));
    const double th = 6.283185307179586476925286766559 * u2;
    return (i & 1) ? r * sin(th) : r * cos(th);
}

/* out[i] = f16( f32(z_i) * scale ), with element i multiplied by outlier_mul when
 * the stream's outlier draw for i is below outlier_frac (1%, x8). */
void orc_normal_f16(uint64_t seed, uint64_t stream, uint64_t offset, int64_t n, float scale,
                    double outlier_frac, float outlier_mul, uint16_t* out) {
    const uint64_t base = stream_base(seed, stream);
    const uint64_t obase = stream_base(seed ^ 0xA5A5A5A5A5A5A5A5ull, stream);
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < n; t++) {
        const uint64_t i = offset + (uint64_t)t;
        float v = (float)normal_at(base, i) * scale;
        if (outlier_frac > 0.0) {
            const double u = (double)(mix64(obase + i + 1) >> 11) * (1.0 / 9007199254740992.0);
            if (u < outlier_frac) v *= outlier_mul;
        }
        out[t] = orc_f32_to_f16(v);
    }
}

/* ---------------------------------------------------------------- q8_0 */
/* One ggml block_q8_0 row: n/32 blocks of { f16 d, int8 qs[32] }. */
static float round_half_away(float x) {
    /* C99 roundf: halfway cases away from zero */
    return roundf(x);
}

void orc_q8_0_row(const float* x, int64_t n, uint8_t* out) {
    const int64_t nb = n / ORC_QK8_0;
    for (int64_t b = 0; b < nb; b++) {
        const float* xb = x + b * ORC_QK8_0;
        float amax = 0.0f;
        for (int i = 0; i < ORC_QK8_0; i++) {
            const float a = fabsf(xb[i]);
            if (a > amax) amax = a;
        }
        volatile float d = amax / 127.0f;            /* keep the f32 rounding steps separate */
        volatile float id = d != 0.0f ? 1.0f / d : 0.0f;
        uint8_t* ob = out + b * ORC_Q8_0_BYTES;
        const uint16_t dh = orc_f32_to_f16(d);
        memcpy(ob, &dh, 2);
        for (int i = 0; i < ORC_QK8_0; i++) {
            volatile float p = xb[i] * id;
            const int q = (int)round_half_away(p);
            ob[2 + i] = (uint8_t)(int8_t)q;
        }
    }
}

void orc_q8_0_dequant_row(const uint8_t* in, int64_t n, float* y) {
    const int64_t nb = n / ORC_QK8_0;
    for (int64_t b = 0; b < nb; b++) {
        const uint8_t* ib = in + b * ORC_Q8_0_BYTES;
        uint16_t dh;
        memcpy(&dh, ib, 2);
        const float d = orc_f16_to_f32(dh);
        for (int i = 0; i < ORC_QK8_0; i++) y[b * ORC_QK8_0 + i] = (float)(int8_t)ib[2 + i] * d;
    }
}

static size_t row_bytes_of(int type, int64_t ne0) {
    switch (type) {
        case ORC_TYPE_F32: return (size_t)ne0 * 4;
        case ORC_TYPE_F16: return (size_t)ne0 * 2;
        case ORC_TYPE_Q8_0: return (size_t)(ne0 / ORC_QK8_0) * ORC_Q8_0_BYTES;
        default: return 0;
    }
}

static void load_row_f32(const void* src, int type, int64_t ne0, float* y) {
    if (type == ORC_TYPE_F32) memcpy(y, src, (size_t)ne0 * 4);
    else if (type == ORC_TYPE_F16) orc_f16_to_f32_n((const uint16_t*)src, y, ne0);
    else orc_q8_0_dequant_row((const uint8_t*)src, ne0, y);
}

/* ---------------------------------------------------------------- set_rows */
/* ggml_set_rows(dst [ne0, dst_rows], src [ne0, n_rows], rows i32 [n_rows]);
 * rows == NULL means the ggml_cpy-into-view form: row i -> base + i.
 * Returns 0, or -1 when a target row is outside [0, dst_rows) (nothing written). */
int orc_set_rows(void* dst, int dst_type, int64_t ne0, int64_t dst_rows, size_t dst_nb1,
                 const void* src, int src_type, size_t src_nb1, int64_t n_rows,
                 const int32_t* rows, int64_t base) {
    if (dst_type == ORC_TYPE_Q8_0 && (ne0 % ORC_QK8_0) != 0) return -2;
    for (int64_t i = 0; i < n_rows; i++) {
        const int64_t r = rows ? (int64_t)rows[i] : base + i;
        if (r < 0 || r >= dst_rows) return -1;
    }
    float* tmp = (float*)malloc((size_t)ne0 * sizeof(float));
    for (int64_t i = 0; i < n_rows; i++) {
        const int64_t r = rows ? (int64_t)rows[i] : base + i;
        const uint8_t* s = (const uint8_t*)src + (size_t)i * src_nb1;
        uint8_t* d = (uint8_t*)dst + (size_t)r * dst_nb1;
        if (src_type == dst_type && dst_type != ORC_TYPE_Q8_0) {
            memcpy(d, s, row_bytes_of(dst_type, ne0));
            continue;
        }
        load_row_f32(s, src_type, ne0, tmp);
        if (dst_type == ORC_TYPE_F32) memcpy(d, tmp, (size_t)ne0 * 4);
        else if (dst_type == ORC_TYPE_F16) orc_f32_to_f16_n(tmp, (uint16_t*)d, ne0);
        else orc_q8_0_row(tmp, ne0, d);
    }
    free(tmp);
    return 0;
}

/* ---------------------------------------------------------------- attention */
/* every f16 value as f32 (the exact conversion above, tabulated once) */
static float g_f16_f32[65536];
static pthread_once_t g_f16_once = PTHREAD_ONCE_INIT;
static void f16_table_fill(void) {
    for (uint32_t h = 0; h < 65536u; h++) g_f16_f32[h] = orc_f16_to_f32((uint16_t)h);
}

/* the dequantised K/V view, kept between calls (a fresh 2 x 37 MB buffer per decode layer spent as
 * much time in page faults as in the arithmetic); calls are serialised on its lock */
static pthread_mutex_t g_kv_mu = PTHREAD_MUTEX_INITIALIZER;
static float* g_kv_buf = NULL;
static size_t g_kv_floats = 0;
static float* kv_buffer(size_t n_floats) {
    if (n_floats > g_kv_floats) {
        free(g_kv_buf);
        g_kv_buf = (float*)malloc(n_floats * sizeof(float));
        g_kv_floats = g_kv_buf ? n_floats : 0;
    }
    return g_kv_buf;
}

/* q: f32 [T][NH][HD] (row stride q_nb1 floats between queries, NH*HD when packed)
 * k, v: cache views; key s of kv-head g starts at base + s*kv_nb1 + g*head_bytes
 *       where head_bytes = row_bytes_of(kv_type, HD).
 * S: number of keys in the view.
 * mask modes:
 *   NONE      every key < S visible
 *   CAUSAL    key s visible to query t iff s <= causal_base + t   (set_causal_mask)
 *   WINDOW    s in [lo[t], hi[t]) or s == own[t]                  (set_window_mask)
 *   EXPLICIT  additive f16 mask row t at mask + t*mask_nb1 (elements), -inf hides
 * out: f32 [T][NH][HD].  A query with no visible key gets zeros. */
int orc_attn(const float* q, int64_t q_nb1, int T, int NH, int HD,
             const void* k, const void* v, int kv_type, size_t kv_nb1, int NKV, int S,
             int mask_mode, int causal_base, const int32_t* lo, const int32_t* hi,
             const int32_t* own, const uint16_t* mask, int64_t mask_nb1,
             float scale, float* out) {
    if (NH % NKV != 0) return -2;
    const int grp = NH / NKV;
    const size_t head_bytes = row_bytes_of(kv_type, HD);
    /* dequantise the whole view once per kv head: kf/vf [NKV][S][HD] */
    pthread_once(&g_f16_once, f16_table_fill);
    pthread_mutex_lock(&g_kv_mu);
    const size_t view_floats = (size_t)NKV * S * HD;
    float* kf = kv_buffer(2 * view_floats + 1);
    if (!kf) {
        pthread_mutex_unlock(&g_kv_mu);
        return -3;
    }
    float* vf = kf + view_floats;
#pragma omp parallel for schedule(static)
    for (int64_t idx = 0; idx < (int64_t)NKV * S; idx++) {
        const int g = (int)(idx / S), s = (int)(idx % S);
        const uint8_t* kr = (const uint8_t*)k + (size_t)s * kv_nb1 + (size_t)g * head_bytes;
        const uint8_t* vr = (const uint8_t*)v + (size_t)s * kv_nb1 + (size_t)g * head_bytes;
        float* kd = kf + ((size_t)g * S + s) * HD;
        float* vd = vf + ((size_t)g * S + s) * HD;
        if (kv_type == ORC_TYPE_F16) {
            const uint16_t* kh = (const uint16_t*)kr;
            const uint16_t* vh = (const uint16_t*)vr;
            for (int e = 0; e < HD; e++) {
                kd[e] = g_f16_f32[kh[e]];
                vd[e] = g_f16_f32[vh[e]];
            }
        } else {
            load_row_f32(kr, kv_type, HD, kd);
            load_row_f32(vr, kv_type, HD, vd);
        }
    }
#pragma omp parallel
    {
        float* sc = (float*)malloc((size_t)(S > 0 ? S : 1) * sizeof(float));
        float* acc = (float*)malloc((size_t)HD * sizeof(float));
#pragma omp for schedule(dynamic, 4)
        for (int64_t th = 0; th < (int64_t)T * NH; th++) {
            const int t = (int)(th / NH), h = (int)(th % NH);
            const int g = h / grp;
            const float* qr = q + (size_t)t * q_nb1 + (size_t)h * HD;
            float m = -INFINITY;
            for (int s = 0; s < S; s++) {
                int vis = 1;
                float add = 0.0f;
                if (mask_mode == ORC_MASK_CAUSAL) vis = s <= causal_base + t;
                else if (mask_mode == ORC_MASK_WINDOW) vis = (s >= lo[t] && s < hi[t]) || s == own[t];
                else if (mask_mode == ORC_MASK_EXPLICIT) {
                    add = orc_f16_to_f32(mask[(size_t)t * mask_nb1 + s]);
                    vis = add != -INFINITY;
                }
                if (!vis) { sc[s] = -INFINITY; continue; }
                const float* kr = kf + ((size_t)g * S + s) * HD;
                float a8[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
                int e = 0;
                for (; e + 8 <= HD; e += 8)
                    for (int j = 0; j < 8; j++) a8[j] += qr[e + j] * kr[e + j];
                float dot = ((a8[0] + a8[4]) + (a8[1] + a8[5])) + ((a8[2] + a8[6]) + (a8[3] + a8[7]));
                for (; e < HD; e++) dot += qr[e] * kr[e];
                sc[s] = dot * scale + add;
                if (sc[s] > m) m = sc[s];
            }
            float* o = out + ((size_t)t * NH + h) * HD;
            for (int e = 0; e < HD; e++) acc[e] = 0.0f;
            if (m == -INFINITY) {
                for (int e = 0; e < HD; e++) o[e] = 0.0f;
                continue;
            }
            float l = 0.0f;
            for (int s = 0; s < S; s++) {
                if (sc[s] == -INFINITY) continue;
                const float p = expf(sc[s] - m);
                l += p;
                const float* vr = vf + ((size_t)g * S + s) * HD;
                for (int e = 0; e < HD; e++) acc[e] += p * vr[e];
            }
            for (int e = 0; e < HD; e++) o[e] = acc[e] / l;
        }
        free(sc);
        free(acc);
    }
    pthread_mutex_unlock(&g_kv_mu);
    return 0;
}

/* The soft_max/mul_mat fallback (gemma4_model.cpp:683-692): kq = K^T q,
 * soft_max_ext(kq, mask, scale), kqv = V kq.  Same result as orc_attn by
 * construction; kept as its own entry so the fallback op's softmax row
 * (ggml_soft_max_ext on one [S] row: softmax(x*scale + mask)) is checkable. */
void orc_soft_max_row(const float* x, const uint16_t* mask, int S, float scale, float* y) {
    float m = -INFINITY;
    for (int s = 0; s < S; s++) {
        const float v = x[s] * scale + (mask ? orc_f16_to_f32(mask[s]) : 0.0f);
        y[s] = v;
        if (v > m) m = v;
    }
    float l = 0.0f;
    for (int s = 0; s < S; s++) {
        const float p = (m == -INFINITY || y[s] == -INFINITY) ? 0.0f : expf(y[s] - m);
        y[s] = p;
        l += p;
    }
    const float inv = l > 0.0f ? 1.0f / l : 0.0f;
    for (int s = 0; s < S; s++) y[s] *= inv;
}

/* ---------------------------------------------------------------- splice */
/* qwen3vl_model.cpp:1165-1171: the cached ids are a strict prefix of the new
 * prompt and the cache holds exactly them (kv_len == n_past). */
int orc_can_splice(const int32_t* cached, int64_t kv_len, int64_t n_past,
                   const int32_t* ids, int64_t n_ids) {
    if (!(kv_len > 0 && n_ids > kv_len && kv_len == n_past)) return 0;
    for (int64_t i = 0; i < kv_len; i++)
        if (cached[i] != ids[i]) return 0;
    return 1;
}

/* ---------------------------------------------------------------- eviction */
/* qwen3vl_model.cpp:1110-1124 on the turn table.  turn_frames[n_turns] are the
 * completed turns' frame counts (oldest first); n_marks is the number of
 * retained frames including the current, not yet completed turn.  On return
 * turn_frames/n_turns describe the kept turns, *drop_turns is how many whole
 * turns left the front and *drop_frames how many single frames were trimmed
 * from the (new) front turn afterwards. */
void orc_evict_window(int32_t* turn_frames, int* n_turns, int* n_marks, int max_frames,
                      int* drop_turns, int* drop_frames) {
    int dt = 0, df = 0;
    while (*n_marks > max_frames && *n_turns > 1) {
        const int drop = turn_frames[0];
        *n_marks -= drop;
        memmove(turn_frames, turn_frames + 1, (size_t)(*n_turns - 1) * sizeof(int32_t));
        (*n_turns)--;
        dt++;
    }
    while (*n_marks > max_frames) {
        (*n_marks)--;
        if (*n_turns > 0) turn_frames[0] = turn_frames[0] > 1 ? turn_frames[0] - 1 : 0;
        df++;
    }
    *drop_turns = dt;
    *drop_frames = df;
}

/* Order-preserving compaction of one cache tensor: kept source rows
 * keep[0..n_keep) (strictly increasing) land at dst_base, dst_base+1, ...
 * Sequential memmove semantics, as kv_shift_rows (moss_vl_model.cpp:264-271)
 * applies them one contiguous run at a time. */
int orc_compact_rows(uint8_t* cache, size_t row_bytes, int64_t n_rows,
                     const int32_t* keep, int64_t n_keep, int64_t dst_base) {
    for (int64_t i = 0; i < n_keep; i++) {
        if (keep[i] < 0 || keep[i] >= n_rows) return -1;
        if (i > 0 && keep[i] <= keep[i - 1]) return -1;
        if (dst_base + i > keep[i]) return -1;     /* rows only move towards the front */
    }
    for (int64_t i = 0; i < n_keep; i++) {
        if (keep[i] != dst_base + i)
            memmove(cache + (size_t)(dst_base + i) * row_bytes, cache + (size_t)keep[i] * row_bytes, row_bytes);
    }
    return 0;
}

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void orc_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}
