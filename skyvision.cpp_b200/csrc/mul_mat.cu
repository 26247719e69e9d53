// mul_mat.cu - the two ggml_mul_mat legs of the soft_max attention fallback on the
// 5th-generation tensor cores (tcgen05.mma, accumulators in TMEM), sm_100a.
//
// With flash attention off, gemma4_model.cpp:683-692 builds per layer (moondream.cpp:476-493 the
// same per head):
//     kq  = ggml_mul_mat(kf, qf)                      [S, T, NH]  raw scores
//     kq  = ggml_soft_max_ext(kq, mask, scale, 0)     sv_soft_max_ext (softmax.cu)
//     vt  = ggml_cont(ggml_transpose(vf))             [S, HD, NKV]
//     kqv = ggml_mul_mat(vt, kq)                      [HD, T, NH]
// kf / vf are views of the f16 cache ([HD, S, NKV], one cache row per key, heads packed in the
// row) and qf the f32 (or f16) queries; query head h reads kv head h / (NH/NKV), ggml's broadcast
// of src0 over src1's third dimension.
//
// mm_kq_kernel: one CTA per (tile of 128 query rows, kv head, range of keys).  The 128 rows pack
// 128/G queries x the G query heads of the kv head, so every key tile serves the whole GQA group.
// The queries are converted to f16 once per CTA (an f32 src1 is rounded to the f16 vec-dot type
// by ggml as well) into a K-major, 128-byte-swizzled B tile; 128-key tiles of K stream by TMA
// into a ring (the A operand, K-major), and one thread issues
//     S(keys x rows) = K(128 x HD) * Q^T(HD x N)      M = 128, N = the tile's rows (16..128)
// into one of two TMEM buffers, so the tensor core computes tile j + 1 while eight epilogue warps
// store tile j: TMEM lane = key, so for a fixed query row a warp writes 32 consecutive keys of the
// contiguous [S, T, NH] result (128-byte stores).  Bound: HBM, on the S x T x NH x 4 bytes of
// scores written (plus the K rows read).
//
// mm_kqv_kernel: one CTA per (tile of 128 query rows, kv head, range of keys), accumulating
//     O(rows x HD) += P(rows x 64 keys) * V(64 keys x HD)  M = 128, N = HD, K = 64 per tile
// in TMEM.  V comes by TMA straight from the cache rows (MN-major B operand), so the transposed
// copy ggml_cont makes is never built.  Eight converter warps load each tile's probabilities (f32,
// row t of head h at kq + t*nb1 + h*nb2) and write them as f16 hi + lo parts (hi = f16(p), lo =
// f16(p - hi)) into two K-major A tiles, and both parts go through the MMA into the same
// accumulator, so P keeps ~22 bits.  Key ranges split over the SMs merge through a workspace:
// every split writes its partial, the last to take the arrival ticket sums them in split order
// (deterministic) and stores.  Bound: HBM, on P (S x T x NH x 4 bytes) and V read.
//
// Every mbarrier wait is bounded (common.cuh); on expiry the kernel sets the abort flag, stops
// issuing, drains its copies and frees TMEM.
#include <algorithm>
#include <cstdio>

#include "common.cuh"
#include "internal.hpp"
#include "umma.cuh"

namespace svkv {

namespace {

struct MmArgs {
    const uint8_t* src;      // kq: queries (q_type); kqv: probabilities (f32)
    int64_t src_nb_t, src_nb_h;   // bytes between queries / heads
    int src_type;
    int T, NH, NKV, G, S;
    int qpt;                 // queries per 128-row tile
    int chunk, n_splits;     // keys per split (a multiple of the tile's keys), splits
    float* out;              // kq: [S, T, NH] contiguous; kqv: (e, t, h) at out + t*out_nb_t + h*out_nb_h
    int64_t out_nb_t, out_nb_h;   // floats
    float* ws;               // kqv split partials [tile][split][128][HD]
    int* tickets;            // kqv [tile], zero before the launch
    int* err;
};

template <int HD>
struct KqCfg {
    static constexpr int BM = 128;                     // keys per tile (M)
    static constexpr int BN = 128;                     // query rows per CTA (N, at most)
    static constexpr int SLAB_A = BM * 128;            // one 64-column slab of a key tile
    static constexpr int A_B = HD / 64 * SLAB_A;
    static constexpr int SLAB_B = BN * 128;
    static constexpr int B_B = HD / 64 * SLAB_B;
    static constexpr int STAGES = HD == 256 ? 2 : 4;
    static constexpr int OFF_B = 0;
    static constexpr int OFF_A = B_B;
    static constexpr int OFF_BAR = OFF_A + STAGES * A_B;
    static constexpr int N_BAR = 2 * STAGES + 5;       // full, empty, q_full, s_full[2], t_free[2]
    static constexpr int SMEM = OFF_BAR + N_BAR * 8 + 16;
    static constexpr int EPI_WARPS = 8;
    static constexpr int THREADS = (EPI_WARPS + 2) * 32;
    static constexpr int TMEM_COLS = 2 * BN;
    static_assert(SMEM + 1024 <= 227 * 1024, "shared memory budget");
};

template <int HD>
__global__ void __launch_bounds__(KqCfg<HD>::THREADS, 1)
mm_kq_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ MmArgs a) {
    using C = KqCfg<HD>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    uint64_t* full = bars;
    uint64_t* empty = bars + C::STAGES;
    uint64_t* q_full = bars + 2 * C::STAGES;
    uint64_t* s_full = q_full + 1;       // [2] S of tile j in TMEM buffer j & 1
    uint64_t* t_free = s_full + 2;       // [2] the epilogue has read buffer j & 1
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::N_BAR);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qt = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
    const int G = a.G;
    const int t0 = qt * a.qpt;
    const int nq = min(a.qpt, a.T - t0);
    const int rows = nq * G;                                // <= 128
    const int n_eff = max(16, (rows + 15) / 16 * 16);       // N of the MMA
    const int ks = split * a.chunk;
    const int ke = min(a.S, ks + a.chunk);
    const int nt = ke > ks ? (ke - ks + C::BM - 1) / C::BM : 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(q_full, C::EPI_WARPS);
        for (int b = 0; b < 2; b++) {
            mbar_init(&s_full[b], 1);
            mbar_init(&t_free[b], C::EPI_WARPS);
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"((uint32_t)C::TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (warp == C::EPI_WARPS && lane == 0) tma_prefetch_desc(&tmk);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();
    if (threadIdx.x == 0) pdl_trigger();

    if (warp < C::EPI_WARPS) {
        // ---- the query rows as the B tile: row r = query r / G, head r % G of the group; f16,
        // K-major, 128-byte swizzled slabs of BN rows x 64 columns; rows past the tile are zero
        const int es = a.src_type == SV_TYPE_F32 ? 4 : 2;
        for (int idx = threadIdx.x; idx < n_eff * (HD / 8); idx += C::EPI_WARPS * 32) {
            const int r = idx / (HD / 8), e = (idx % (HD / 8)) * 8;
            uint4 v = make_uint4(0, 0, 0, 0);
            if (r < rows) {
                const uint8_t* qrow = a.src + (size_t)(t0 + r / G) * a.src_nb_t + (size_t)(kvh * G + r % G) * a.src_nb_h +
                                      (size_t)e * es;
                if (es == 4) {
                    const float4 f0 = *reinterpret_cast<const float4*>(qrow);
                    const float4 f1 = *reinterpret_cast<const float4*>(qrow + 16);
                    v.x = pack_h2(f0.x, f0.y);
                    v.y = pack_h2(f0.z, f0.w);
                    v.z = pack_h2(f1.x, f1.y);
                    v.w = pack_h2(f1.z, f1.w);
                } else {
                    v = *reinterpret_cast<const uint4*>(qrow);
                }
            }
            *reinterpret_cast<uint4*>(smem + C::OFF_B + (e / 64) * C::SLAB_B + swz_off(r, e % 64, 128)) = v;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(q_full);
        // ---- epilogue: warp w reads TMEM lane quarter w % 4 (keys) and column half w / 4 (rows)
        const int quarter = warp & 3, half = warp >> 2;
        for (int j = 0; j < nt; j++) {
            if (!warp_wait(&s_full[j & 1], (j >> 1) & 1, a.err, abort_flag)) break;
            tc_fence_after();
            const int key = ks + j * C::BM + quarter * 32 + lane;
            for (int c0 = half * (C::BN / 2); c0 < (half + 1) * (C::BN / 2) && c0 < rows; c0 += 32) {
                float v[32];
                tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)((j & 1) * C::BN + c0), v);
                tmem_wait_ld();
                if (key < ke) {
#pragma unroll
                    for (int k = 0; k < 32; k++) {
                        const int c = c0 + k;
                        if (c < rows)
                            a.out[(size_t)(kvh * G + c % G) * a.out_nb_h + (size_t)(t0 + c / G) * a.out_nb_t + key] = v[k];
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&t_free[j & 1]);
        }
    } else if (warp == C::EPI_WARPS) {
        // ---- TMA producer: 128-key tiles of this kv head's columns (rows past the view are zero)
        if (lane == 0 && nt > 0) {
            int issued = 0;
            for (int j = 0; j < nt; j++) {
                const int s = j % C::STAGES;
                if (j >= C::STAGES && !wait_or_abort(&empty[s], ((j / C::STAGES) - 1) & 1, a.err, abort_flag)) break;
                mbar_arrive_expect_tx(&full[s], C::A_B);
#pragma unroll
                for (int b = 0; b < HD / 64; b++)
                    tma_load_2d(smem + C::OFF_A + s * C::A_B + b * C::SLAB_A, &tmk, kvh * HD + b * 64, ks + j * C::BM,
                                &full[s]);
                issued = j + 1;
            }
            for (int j = max(0, issued - C::STAGES); j < issued; j++)
                mbar_wait(&full[j % C::STAGES], (j / C::STAGES) & 1, a.err);
        }
    } else {
        // ---- MMA issuer (one thread)
        if (lane == 0 && nt > 0) {
            const uint32_t idesc = umma_idesc(128, n_eff, 0, 0);
            constexpr uint32_t hi = desc_hi_sw128(1024);
            const uint32_t a_lo = desc_lo(smem_u32(smem + C::OFF_A), 16);
            const uint32_t b_lo = desc_lo(smem_u32(smem + C::OFF_B), 16);
            bool ok = wait_or_abort(q_full, 0, a.err, abort_flag);
            for (int j = 0; ok && j < nt; j++) {
                const int s = j % C::STAGES;
                if (!wait_or_abort(&full[s], (j / C::STAGES) & 1, a.err, abort_flag)) break;
                if (j >= 2 && !wait_or_abort(&t_free[j & 1], ((j >> 1) - 1) & 1, a.err, abort_flag)) break;
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)((j & 1) * C::BN);
#pragma unroll
                for (int kk = 0; kk < HD / 16; kk++) {
                    const uint32_t a_off = (uint32_t)((s * C::A_B + (kk / 4) * C::SLAB_A + (kk % 4) * 32) >> 4);
                    const uint32_t b_off = (uint32_t)(((kk / 4) * C::SLAB_B + (kk % 4) * 32) >> 4);
                    umma_f16_w(d, a_lo + a_off, b_lo + b_off, hi, idesc, kk > 0 ? 1u : 0u);
                }
                umma_commit(&s_full[j & 1]);
                umma_commit(&empty[s]);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)C::TMEM_COLS));
    }
}

template <int HD>
struct KqvCfg {
    static constexpr int BM = 128;                     // query rows per tile (M)
    static constexpr int BK = 64;                      // keys per tile
    static constexpr int A_B = BM * 128;               // one part (hi or lo) of the P tile
    static constexpr int VBOX = BK * 128;              // one 64-column slab of a V tile
    static constexpr int V_B = HD / 64 * VBOX;
    static constexpr int STAGE_B = 2 * A_B + V_B;
    static constexpr int STAGES = 3;
    static constexpr int OFF_BAR = STAGES * STAGE_B;
    static constexpr int N_BAR = 3 * STAGES + 1;       // full_a, full_v, empty, o_done
    static constexpr int SMEM = OFF_BAR + N_BAR * 8 + 16;
    static constexpr int CONV_WARPS = 8;
    static constexpr int THREADS = (CONV_WARPS + 2) * 32;
    static constexpr int TMEM_COLS = HD;
    static_assert(SMEM + 1024 <= 227 * 1024, "shared memory budget");
};

__device__ __forceinline__ void conv_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(KqvCfg<64>::CONV_WARPS * 32) : "memory");
}

template <int HD>
__global__ void __launch_bounds__(KqvCfg<HD>::THREADS, 1)
mm_kqv_kernel(const __grid_constant__ CUtensorMap tmv, const __grid_constant__ MmArgs a) {
    using C = KqvCfg<HD>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    uint64_t* full_a = bars;
    uint64_t* full_v = bars + C::STAGES;
    uint64_t* empty = bars + 2 * C::STAGES;
    uint64_t* o_done = bars + 3 * C::STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::N_BAR);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* last_flag = abort_flag + 1;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int mt = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
    const int G = a.G;
    const int t0 = mt * a.qpt;
    const int nq = min(a.qpt, a.T - t0);
    const int rows = nq * G;
    const int ks = split * a.chunk;
    const int ke = min(a.S, ks + a.chunk);
    const int nt = ke > ks ? (ke - ks + C::BK - 1) / C::BK : 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; s++) {
            mbar_init(&full_a[s], C::CONV_WARPS);
            mbar_init(&full_v[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(o_done, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"((uint32_t)C::TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (warp == C::CONV_WARPS && lane == 0) tma_prefetch_desc(&tmv);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();
    if (threadIdx.x == 0) pdl_trigger();

    if (warp < C::CONV_WARPS) {
        // ---- converters: warp w fills rows 32*(w % 4) + lane, keys [32*(w / 4), +32) of each tile
        const int quarter = warp & 3, kh = warp >> 2;
        const int r = quarter * 32 + lane;
        const bool valid = r < rows;
        const float* prow = valid ? reinterpret_cast<const float*>(a.src + (size_t)(t0 + r / G) * a.src_nb_t +
                                                                   (size_t)(kvh * G + r % G) * a.src_nb_h)
                                  : nullptr;
        bool ok = true;
        for (int j = 0; j < nt; j++) {
            const int s = j % C::STAGES;
            if (j >= C::STAGES && !warp_wait(&empty[s], ((j / C::STAGES) - 1) & 1, a.err, abort_flag)) {
                ok = false;
                break;
            }
            const int k0 = ks + j * C::BK + kh * 32;
            float x[32];
            // 16-byte loads where the row allows them (ggml's contiguous kq has rows of S floats, so an
            // odd S leaves rows 4-byte aligned only)
            if (valid && k0 + 32 <= ke && (reinterpret_cast<uintptr_t>(prow + k0) & 15) == 0) {
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const float4 f = __ldg(reinterpret_cast<const float4*>(prow + k0) + i);
                    x[4 * i] = f.x; x[4 * i + 1] = f.y; x[4 * i + 2] = f.z; x[4 * i + 3] = f.w;
                }
            } else {
#pragma unroll
                for (int i = 0; i < 32; i++) x[i] = (valid && k0 + i < ke) ? __ldg(prow + k0 + i) : 0.0f;
            }
            uint8_t* ah = smem + s * C::STAGE_B;
            uint8_t* al = ah + C::A_B;
#pragma unroll
            for (int c = 0; c < 4; c++) {
                uint32_t h[4], l[4];
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const __half2 hh = __floats2half2_rn(x[8 * c + 2 * i], x[8 * c + 2 * i + 1]);
                    const float2 hf = __half22float2(hh);
                    h[i] = *reinterpret_cast<const uint32_t*>(&hh);
                    l[i] = pack_h2(x[8 * c + 2 * i] - hf.x, x[8 * c + 2 * i + 1] - hf.y);
                }
                const uint32_t off = swz_off(r, kh * 32 + c * 8, 128);
                *reinterpret_cast<uint4*>(ah + off) = make_uint4(h[0], h[1], h[2], h[3]);
                *reinterpret_cast<uint4*>(al + off) = make_uint4(l[0], l[1], l[2], l[3]);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&full_a[s]);
        }
        // ---- epilogue: warp w reads TMEM lane quarter w % 4 (rows), columns [HD/2 * (w / 4), +HD/2)
        const bool have = nt > 0 && ok && warp_wait(o_done, 0, a.err, abort_flag);
        tc_fence_after();
        const int c_lo = kh * (HD / 2), c_hi = c_lo + HD / 2;
        float* orow = valid ? a.out + (size_t)(t0 + r / G) * a.out_nb_t + (size_t)(kvh * G + r % G) * a.out_nb_h
                            : nullptr;
        const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16);
        if (a.n_splits == 1) {
            for (int cc = c_lo; cc < c_hi; cc += 32) {
                float o[32];
                if (have) {
                    tmem_ld32(taddr + cc, o);
                    tmem_wait_ld();
                } else {
#pragma unroll
                    for (int k = 0; k < 32; k++) o[k] = 0.0f;
                }
                if (valid)
#pragma unroll
                    for (int k = 0; k < 32; k += 4)
                        *reinterpret_cast<float4*>(orow + cc + k) = make_float4(o[k], o[k + 1], o[k + 2], o[k + 3]);
            }
        } else {
            // every split publishes its partial, then takes the arrival ticket; the last sums all
            // partials in split order (its own included) and resets the ticket
            const int unit = kvh * gridDim.x + mt;
            const int ns = a.n_splits;
            float* part = a.ws + ((size_t)(unit * ns + split) * C::BM + r) * HD;
            for (int cc = c_lo; cc < c_hi; cc += 32) {
                float o[32];
                if (have) {
                    tmem_ld32(taddr + cc, o);
                    tmem_wait_ld();
                } else {
#pragma unroll
                    for (int k = 0; k < 32; k++) o[k] = 0.0f;
                }
                if (valid)
#pragma unroll
                    for (int k = 0; k < 32; k += 4)
                        *reinterpret_cast<float4*>(part + cc + k) = make_float4(o[k], o[k + 1], o[k + 2], o[k + 3]);
            }
            __threadfence();
            conv_sync();
            if (threadIdx.x == 0) *last_flag = atomicAdd(&a.tickets[unit], 1) == ns - 1;
            conv_sync();
            if (*last_flag) {
                __threadfence();
                if (valid) {
                    const float* base = a.ws + ((size_t)unit * ns * C::BM + r) * HD;
                    for (int cc = c_lo; cc < c_hi; cc += 4) {
                        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
                        for (int sp = 0; sp < ns; sp++) {
                            const float4 v = __ldcg(reinterpret_cast<const float4*>(base + (size_t)sp * C::BM * HD + cc));
                            acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
                        }
                        *reinterpret_cast<float4*>(orow + cc) = acc;
                    }
                }
                if (threadIdx.x == 0) a.tickets[unit] = 0;
            }
        }
    } else if (warp == C::CONV_WARPS) {
        // ---- TMA producer: 64-key tiles of V (this kv head's columns), rows past the view zero
        if (lane == 0 && nt > 0) {
            int issued = 0;
            for (int j = 0; j < nt; j++) {
                const int s = j % C::STAGES;
                if (j >= C::STAGES && !wait_or_abort(&empty[s], ((j / C::STAGES) - 1) & 1, a.err, abort_flag)) break;
                mbar_arrive_expect_tx(&full_v[s], C::V_B);
#pragma unroll
                for (int b = 0; b < HD / 64; b++)
                    tma_load_2d(smem + s * C::STAGE_B + 2 * C::A_B + b * C::VBOX, &tmv, kvh * HD + b * 64, ks + j * C::BK,
                                &full_v[s]);
                issued = j + 1;
            }
            for (int j = max(0, issued - C::STAGES); j < issued; j++)
                mbar_wait(&full_v[j % C::STAGES], (j / C::STAGES) & 1, a.err);
        }
    } else {
        // ---- MMA issuer: O += P_hi V + P_lo V per 16-key step
        if (lane == 0 && nt > 0) {
            const uint32_t idesc = umma_idesc(128, HD, 0, 1);
            constexpr uint32_t hi = desc_hi_sw128(1024);
            bool ok = true;
            for (int j = 0; j < nt; j++) {
                const int s = j % C::STAGES;
                if (!wait_or_abort(&full_a[s], (j / C::STAGES) & 1, a.err, abort_flag) ||
                    !wait_or_abort(&full_v[s], (j / C::STAGES) & 1, a.err, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t ph = desc_lo(smem_u32(smem + s * C::STAGE_B), 16);
                const uint32_t pl = ph + (uint32_t)(C::A_B >> 4);
                const uint32_t vd = desc_lo(smem_u32(smem + s * C::STAGE_B + 2 * C::A_B), C::VBOX);
#pragma unroll
                for (int kk = 0; kk < C::BK / 16; kk++) {
                    const uint32_t boff = (uint32_t)((kk * 16 * 128) >> 4);
                    umma_f16_w(tmem, ph + (uint32_t)((kk * 32) >> 4), vd + boff, hi, idesc, (j > 0 || kk > 0) ? 1u : 0u);
                    umma_f16_w(tmem, pl + (uint32_t)((kk * 32) >> 4), vd + boff, hi, idesc, 1u);
                }
                umma_commit(&empty[s]);
            }
            if (ok) umma_commit(o_done);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)C::TMEM_COLS));
    }
}

// ------------------------------------------------------------------ host side
struct MmPlan {
    int qpt = 1, n_qt = 1, chunk = 0, n_splits = 1;
};

MmPlan plan_mm(int T, int G, int NKV, int S, int tile_keys, int target_ctas, int max_splits) {
    MmPlan p;
    p.qpt = std::max(1, 128 / G);
    p.n_qt = ceil_div(T, p.qpt);
    const int units = p.n_qt * NKV;
    const int tiles = std::max(1, ceil_div(S, tile_keys));
    int ns = std::min(std::min(std::max(1, ceil_div(target_ctas, units)), tiles), std::max(1, max_splits));
    p.chunk = ceil_div(ceil_div(S, ns), tile_keys) * tile_keys;
    p.n_splits = std::max(1, ceil_div(S, p.chunk));
    return p;
}

bool make_f16_view_tmap(CUtensorMap* m, const void* base, int NKV, int HD, size_t nb1, int S, int box_rows) {
    return encode_tmap_2d(m, base, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, (uint64_t)NKV * HD, (uint64_t)S, nb1, 64,
                          (uint32_t)box_rows, CU_TENSOR_MAP_SWIZZLE_128B);
}

// kernel attributes, once per device and kernel
template <int HD>
cudaError_t launch_kq_t(const CUtensorMap& tm, const MmArgs& a, dim3 grid, cudaStream_t st) {
    constexpr int smem = KqCfg<HD>::SMEM + 1024;
    static std::once_flag once[kMaxDevices];
    static cudaError_t status[kMaxDevices];
    const cudaError_t e = once_per_device(once, status, [] {
        return cudaFuncSetAttribute(mm_kq_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    });
    if (e != cudaSuccess) return e;
    return launch_pdl(mm_kq_kernel<HD>, grid, dim3(KqCfg<HD>::THREADS), (size_t)smem, st, tm, a);
}

template <int HD>
cudaError_t launch_kqv_t(const CUtensorMap& tm, const MmArgs& a, dim3 grid, cudaStream_t st) {
    constexpr int smem = KqvCfg<HD>::SMEM + 1024;
    static std::once_flag once[kMaxDevices];
    static cudaError_t status[kMaxDevices];
    const cudaError_t e = once_per_device(once, status, [] {
        return cudaFuncSetAttribute(mm_kqv_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    });
    if (e != cudaSuccess) return e;
    return launch_pdl(mm_kqv_kernel<HD>, grid, dim3(KqvCfg<HD>::THREADS), (size_t)smem, st, tm, a);
}

int status_of(cudaError_t e) {
    if (e == cudaSuccess) return SV_OK;
    fprintf(stderr, "svkv: CUDA error %s\n", cudaGetErrorString(e));
    return SV_ERR_CUDA;
}

constexpr int kKqvMaxSplits = 64;

bool mm_shape_ok(int n_kv_head, int head_dim, int n_keys, int T, int n_head) {
    return n_kv_head > 0 && n_keys > 0 && T > 0 && n_head > 0 && n_head % n_kv_head == 0 &&
           n_head / n_kv_head <= 16 && (head_dim == 64 || head_dim == 128 || head_dim == 256);
}

}  // namespace
}  // namespace svkv

using namespace svkv;

extern "C" {

int sv_mul_mat_kq(const void* k, size_t k_nb1, int n_kv_head, int head_dim, int n_keys, const void* q, int q_type,
                  size_t q_nb1, size_t q_nb2, int T, int n_head, float* kq, void* stream) {
    if (!k || !q || !kq || !mm_shape_ok(n_kv_head, head_dim, n_keys, T, n_head)) return SV_ERR_INVALID;
    if (q_type != SV_TYPE_F16 && q_type != SV_TYPE_F32) return SV_ERR_UNSUPPORTED;
    const int HD = head_dim, NKV = n_kv_head, G = n_head / n_kv_head;
    // heads packed in the cache row; 16-byte aligned rows for TMA and the vector query loads
    if (k_nb1 < (size_t)NKV * HD * 2 || (k_nb1 & 15) || (reinterpret_cast<uintptr_t>(k) & 15) ||
        (reinterpret_cast<uintptr_t>(q) & 15) || (q_nb1 & 15) || (q_nb2 & 15))
        return SV_ERR_UNSUPPORTED;
    CUtensorMap tm;
    if (!make_f16_view_tmap(&tm, k, NKV, HD, k_nb1, n_keys, 128)) return SV_ERR_UNSUPPORTED;
    const MmPlan p = plan_mm(T, G, NKV, n_keys, 128, 2 * device_sm_count(), 1 << 20);
    MmArgs a{};
    a.src = static_cast<const uint8_t*>(q);
    a.src_nb_t = (int64_t)q_nb1;
    a.src_nb_h = (int64_t)q_nb2;
    a.src_type = q_type;
    a.T = T;
    a.NH = n_head;
    a.NKV = NKV;
    a.G = G;
    a.S = n_keys;
    a.qpt = p.qpt;
    a.chunk = p.chunk;
    a.n_splits = p.n_splits;
    a.out = kq;
    a.out_nb_t = n_keys;
    a.out_nb_h = (int64_t)n_keys * T;
    const dim3 grid((unsigned)p.n_qt, (unsigned)NKV, (unsigned)p.n_splits);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    switch (HD) {
        case 64: return status_of(launch_kq_t<64>(tm, a, grid, st));
        case 128: return status_of(launch_kq_t<128>(tm, a, grid, st));
        default: return status_of(launch_kq_t<256>(tm, a, grid, st));
    }
}

size_t sv_mul_mat_kqv_workspace(int n_kv_head, int head_dim, int n_keys, int T, int n_head) {
    if (!mm_shape_ok(n_kv_head, head_dim, n_keys, T, n_head)) return 0;
    const MmPlan p = plan_mm(T, n_head / n_kv_head, n_kv_head, n_keys, 64, device_sm_count(), kKqvMaxSplits);
    if (p.n_splits <= 1) return 0;
    const size_t units = (size_t)p.n_qt * n_kv_head;
    return (units * sizeof(int) + 255) / 256 * 256 + units * p.n_splits * 128 * head_dim * sizeof(float);
}

int sv_mul_mat_kqv(const void* v, size_t v_nb1, int n_kv_head, int head_dim, int n_keys, const float* kq,
                   size_t kq_nb1, size_t kq_nb2, int T, int n_head, float* dst, size_t dst_nb1, size_t dst_nb2,
                   void* workspace, size_t ws_bytes, void* stream) {
    if (!v || !kq || !dst || !mm_shape_ok(n_kv_head, head_dim, n_keys, T, n_head)) return SV_ERR_INVALID;
    const int HD = head_dim, NKV = n_kv_head, G = n_head / n_kv_head;
    if (v_nb1 < (size_t)NKV * HD * 2 || (v_nb1 & 15) || (reinterpret_cast<uintptr_t>(v) & 15) ||
        (reinterpret_cast<uintptr_t>(kq) & 3) || (kq_nb1 & 3) || (kq_nb2 & 3) ||
        (reinterpret_cast<uintptr_t>(dst) & 15) || (dst_nb1 & 15) || (dst_nb2 & 15))
        return SV_ERR_UNSUPPORTED;
    CUtensorMap tm;
    if (!make_f16_view_tmap(&tm, v, NKV, HD, v_nb1, n_keys, 64)) return SV_ERR_UNSUPPORTED;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    MmPlan p = plan_mm(T, G, NKV, n_keys, 64, device_sm_count(), kKqvMaxSplits);
    const size_t units = (size_t)p.n_qt * NKV;
    const size_t tk_bytes = (units * sizeof(int) + 255) / 256 * 256;
    // the splits the workspace holds (none without one)
    const size_t per_split = units * 128 * HD * sizeof(float);
    int max_ns = 1;
    if (workspace && ws_bytes > tk_bytes) max_ns = (int)std::min<size_t>((ws_bytes - tk_bytes) / per_split, kKqvMaxSplits);
    if (p.n_splits > max_ns) p = plan_mm(T, G, NKV, n_keys, 64, device_sm_count(), std::max(1, max_ns));
    MmArgs a{};
    a.src = reinterpret_cast<const uint8_t*>(kq);
    a.src_nb_t = (int64_t)kq_nb1;
    a.src_nb_h = (int64_t)kq_nb2;
    a.src_type = SV_TYPE_F32;
    a.T = T;
    a.NH = n_head;
    a.NKV = NKV;
    a.G = G;
    a.S = n_keys;
    a.qpt = p.qpt;
    a.chunk = p.chunk;
    a.n_splits = p.n_splits;
    a.out = dst;
    a.out_nb_t = (int64_t)(dst_nb1 / 4);
    a.out_nb_h = (int64_t)(dst_nb2 / 4);
    if (p.n_splits > 1) {
        a.tickets = static_cast<int*>(workspace);
        a.ws = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + tk_bytes);
        const cudaError_t e = cudaMemsetAsync(a.tickets, 0, units * sizeof(int), st);
        if (e != cudaSuccess) return status_of(e);
    }
    const dim3 grid((unsigned)p.n_qt, (unsigned)NKV, (unsigned)p.n_splits);
    switch (HD) {
        case 64: return status_of(launch_kqv_t<64>(tm, a, grid, st));
        case 128: return status_of(launch_kqv_t<128>(tm, a, grid, st));
        default: return status_of(launch_kqv_t<256>(tm, a, grid, st));
    }
}

}  // extern "C"
