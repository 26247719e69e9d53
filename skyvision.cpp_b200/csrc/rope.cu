// rope.cu - the step before the KV append, fused: per-head q/k RMSNorm with its weight, rotary
// position embedding, and the append of K and V into the cache, one launch per layer and chunk.
//
// Replaces the op chain of qwen3vl_model.cpp:636-655 (and the NEOX-mode models, e.g.
// gemma4_model.cpp:640-642, nemotronomni_model.cpp:298-300):
//   q3 = ggml_rms_norm(q3, eps) * qn;  k3 = ggml_rms_norm(k3, eps) * kn;
//   q3 = rope(q3, pos); k3 = rope(k3, pos);   (GGML_ROPE_TYPE_NEOX or GGML_ROPE_TYPE_IMROPE)
//   ggml_set_rows(kv.k[il], k3, slot); ggml_set_rows(kv.v[il], v, slot);
// The rotated queries go to q_out (f16 or f32) for the attention launch that follows.
//
// One CTA per (token, group of 8 heads), one warp per head (the q heads, the k heads, then the v
// heads).  The CTA's threads first compute the token's rotation table in shared memory: for pair
// i < n_dims/2, theta = p * inv_freq[i] in double (inv_freq[i] = base^(-2i/n_dims), computed in
// double on the host), reduced modulo 2 pi in double, then cos and sin of the reduced angle in f32
// (ggml builds theta by repeated f32 multiplication; this table is the exact angle to f32 rounding,
// so the two differ by ggml's own rounding).  Lane l of a warp holds elements l + 32j, so the rotation partner
// l + 32j + n_dims/2 of a rotated element is in the same lane (n_dims/2 is a multiple of 32), the
// RMS is one warp reduction, and a q8_0 block (32 consecutive elements) is one j across the warp.
// q8_0 rows use the append kernel's exact steps (d = amax/127, id = 1/d, q = round-half-away(x*id),
// d stored as f16), so V rows match sv_set_rows of the same f32 source byte for byte.
//
// Bound: HBM (reads the f32 q/k/v rows, writes the cache rows and q_out); tiny next to attention.
#include <cmath>

#include "common.cuh"
#include "internal.hpp"

namespace svkv {

namespace {

constexpr int kRopeThreads = 256;
constexpr int kMaxHD = 256;

struct RopeArgs {
    const float* q;          // [T][NH][HD]
    const float* k;          // [T][NKV][HD]
    const float* v;          // [T][NKV][HD]
    int T, NH, NKV, HD;
    const float* qn;         // [HD] or null (no q norm)
    const float* kn;         // [HD] or null
    float eps;
    int mode, n_dims;        // SV_ROPE_NONE / NEOX / IMROPE
    float freq_base;
    int sec[4];
    const int32_t* pos;      // NEOX: [T]; IMROPE: [4][T] (t, h, w, e)
    double inv_freq[kMaxHD / 2];
    int slot_base;
    const int32_t* slot_base_dev;
    uint8_t* kc;             // cache row r of K at kc + r * row_bytes
    uint8_t* vc;
    size_t row_bytes;
    int kv_type;
    int n_ctx;
    void* q_out;             // [T][NH][HD]
    int q_out_type;
    int* err;
};

// the position axis of rotation pair i (ggml's interleaved-MRoPE rule for Qwen3-VL: pairs cycle
// t, h, w within the first 3*sections[.] pairs of each axis; the rest use the fourth stream)
__device__ __forceinline__ int imrope_axis(int i, const int* sec) {
    const int sect_dims = sec[0] + sec[1] + sec[2] + sec[3];
    const int sector = sect_dims > 0 ? i % sect_dims : i;
    if (sector % 3 == 1 && sector < 3 * sec[1]) return 1;
    if (sector % 3 == 2 && sector < 3 * sec[2]) return 2;
    if (sector % 3 == 0 && sector < 3 * sec[0]) return 0;
    return 3;
}

// one block of 32 elements (one per lane) quantised to block_q8_0 at dst (34 bytes)
__device__ __forceinline__ void store_q8_0_block(uint8_t* dst, float x, int lane) {
    float amax = fabsf(x);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float dd = __fdiv_rn(amax, 127.0f);
    const float id = dd != 0.0f ? __fdiv_rn(1.0f, dd) : 0.0f;
    const int qv = (int)roundf(__fmul_rn(x, id));
    dst[2 + lane] = (uint8_t)(int8_t)qv;
    if (lane == 0) *reinterpret_cast<__half*>(dst) = __float2half_rn(dd);
}

// NJ = head_dim / 32 elements per lane; HALF = n_dims / 64 (0: no rotation)
template <int NJ, int HALF>
__global__ void __launch_bounds__(kRopeThreads) qk_norm_rope_append_kernel(const __grid_constant__ RopeArgs a) {
    __shared__ float2 cs[kMaxHD / 2];
    pdl_wait();
    const int t = blockIdx.x;
    const int slot = (a.slot_base_dev ? __ldg(a.slot_base_dev) : a.slot_base) + t;
    const bool slot_ok = slot >= 0 && slot < a.n_ctx;
    if (!slot_ok && threadIdx.x == 0 && blockIdx.y == 0 && a.err) atomicOr(a.err, ERRBIT_ROW_RANGE);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = blockIdx.y * (kRopeThreads / 32) + warp;
    const int kind = h < a.NH ? 0 : (h < a.NH + a.NKV ? 1 : 2);   // q, k, v
    const int hh = kind == 0 ? h : (kind == 1 ? h - a.NH : h - a.NH - a.NKV);
    const bool live = h < a.NH + 2 * a.NKV && (kind == 0 || slot_ok);
    // the head's loads first: their latency overlaps the rotation table below
    float x[NJ];
    if (live) {
        const float* src = kind == 0 ? a.q + ((size_t)t * a.NH + hh) * a.HD
                                     : (kind == 1 ? a.k : a.v) + ((size_t)t * a.NKV + hh) * a.HD;
#pragma unroll
        for (int j = 0; j < NJ; j++) x[j] = src[lane + 32 * j];
    }
    if (a.mode != SV_ROPE_NONE) {
        for (int i = threadIdx.x; i < a.n_dims / 2; i += blockDim.x) {
            const int axis = a.mode == SV_ROPE_IMROPE ? imrope_axis(i, a.sec) : 0;
            const double p = (double)__ldg(a.pos + (size_t)axis * a.T + t);
            double th = p * a.inv_freq[i];
            th = fma(-6.283185307179586, rint(th * 0.15915494309189535), th);   // th mod 2 pi, |th| <= pi
            float sn, cn;
            sincosf((float)th, &sn, &cn);
            cs[i] = make_float2(cn, sn);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) pdl_trigger();
    if (!live) return;
    {
        if (kind != 2) {
            const float* w = kind == 0 ? a.qn : a.kn;
            if (w) {   // ggml_rms_norm then ggml_mul: y = (x * (1 / sqrt(mean(x^2) + eps))) * w
                float ss = 0.0f;
#pragma unroll
                for (int j = 0; j < NJ; j++) ss = fmaf(x[j], x[j], ss);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
                const float scale = 1.0f / sqrtf(ss / (float)a.HD + a.eps);
#pragma unroll
                for (int j = 0; j < NJ; j++) x[j] = __fmul_rn(__fmul_rn(x[j], scale), __ldg(w + lane + 32 * j));
            }
            if (HALF > 0 && a.mode != SV_ROPE_NONE) {   // NEOX pairs (i, i + n_dims/2); dims >= n_dims pass through
#pragma unroll
                for (int j = 0; j < HALF; j++) {
                    const float2 c = cs[lane + 32 * j];
                    const float x0 = x[j], x1 = x[j + HALF];
                    x[j] = x0 * c.x - x1 * c.y;
                    x[j + HALF] = x0 * c.y + x1 * c.x;
                }
            }
        }
        if (kind == 0) {
            const size_t o = ((size_t)t * a.NH + hh) * a.HD + lane;
#pragma unroll
            for (int j = 0; j < NJ; j++) {
                if (a.q_out_type == SV_TYPE_F32) reinterpret_cast<float*>(a.q_out)[o + 32 * j] = x[j];
                else reinterpret_cast<__half*>(a.q_out)[o + 32 * j] = __float2half_rn(x[j]);
            }
        } else {
            uint8_t* row = (kind == 1 ? a.kc : a.vc) + (size_t)slot * a.row_bytes;
            if (a.kv_type == SV_TYPE_Q8_0) {
                uint8_t* hb = row + (size_t)hh * NJ * kQ8_0Bytes;
#pragma unroll
                for (int j = 0; j < NJ; j++) store_q8_0_block(hb + (size_t)j * kQ8_0Bytes, x[j], lane);
            } else {
                __half* hr = reinterpret_cast<__half*>(row) + (size_t)hh * a.HD + lane;
#pragma unroll
                for (int j = 0; j < NJ; j++) hr[32 * j] = __float2half_rn(x[j]);
            }
        }
    }
}

}  // namespace

cudaError_t launch_qk_norm_rope_append(const RopeLaunch& r, cudaStream_t st) {
    RopeArgs a{};
    a.q = r.q;
    a.k = r.k;
    a.v = r.v;
    a.T = r.T;
    a.NH = r.NH;
    a.NKV = r.NKV;
    a.HD = r.HD;
    a.qn = r.qn;
    a.kn = r.kn;
    a.eps = r.eps;
    a.mode = r.mode;
    a.n_dims = r.n_dims;
    a.freq_base = r.freq_base;
    for (int i = 0; i < 4; i++) a.sec[i] = r.sec[i];
    a.pos = r.pos;
    for (int i = 0; i < r.n_dims / 2 && i < kMaxHD / 2; i++)
        a.inv_freq[i] = std::pow((double)r.freq_base, -2.0 * (double)i / (double)r.n_dims);
    a.slot_base = r.slot_base;
    a.slot_base_dev = r.slot_base_dev;
    a.kc = r.kc;
    a.vc = r.vc;
    a.row_bytes = r.row_bytes;
    a.kv_type = r.kv_type;
    a.n_ctx = r.n_ctx;
    a.q_out = r.q_out;
    a.q_out_type = r.q_out_type;
    a.err = r.err;
    const int half = r.mode == SV_ROPE_NONE ? 0 : r.n_dims / 64;
    const dim3 grid((unsigned)r.T, (unsigned)ceil_div(r.NH + 2 * r.NKV, kRopeThreads / 32)), block(kRopeThreads);
#define SV_ROPE_CASE(HD_, HALF_) \
    if (r.HD == HD_ && half == HALF_) return launch_pdl(qk_norm_rope_append_kernel<HD_ / 32, HALF_>, grid, block, 0, st, a);
    SV_ROPE_CASE(64, 0) SV_ROPE_CASE(64, 1)
    SV_ROPE_CASE(128, 0) SV_ROPE_CASE(128, 1) SV_ROPE_CASE(128, 2)
    SV_ROPE_CASE(256, 0) SV_ROPE_CASE(256, 2) SV_ROPE_CASE(256, 4)
#undef SV_ROPE_CASE
    return cudaErrorInvalidValue;
}

// head sizes 64 / 128 / 256; the rotated dims (n_dims) all of them or half (128, 256), or none
bool rope_supported(int head_dim, int mode, int n_dims) {
    if (head_dim != 64 && head_dim != 128 && head_dim != 256) return false;
    if (mode == SV_ROPE_NONE) return true;
    if (mode != SV_ROPE_NEOX && mode != SV_ROPE_IMROPE) return false;
    return n_dims == head_dim || (head_dim >= 128 && n_dims == head_dim / 2);
}

}  // namespace svkv
