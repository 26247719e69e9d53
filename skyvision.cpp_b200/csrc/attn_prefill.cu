// attn_prefill.cu - chunked-prefill attention on the 5th-generation tensor
// cores (tcgen05.mma, accumulators in TMEM), sm_100a.
//
// Replaces ggml_flash_attn_ext for prompt chunks (the 512-token ubatches of
// gemma4_model.cpp:1355-1395, the splice tail of qwen3vl_model.cpp:1172-1193)
// over an f16 cache, causal mask as an in-kernel predicate
// (set_causal_mask(mask, n_past, T), attention.hpp:60-67).
//
// One CTA = one 128-row query tile x one kv head.  The 128 rows pack
// 128/G queries x the G query heads of the kv head, so each K/V tile feeds
// every head of the GQA group.  Warp roles (192 threads):
//   warps 0-3  softmax: row r = thread r = TMEM lane r.  Load Q into shared
//              memory (128-byte swizzled K-major), then per key tile read S
//              with tcgen05.ld, apply scale and the causal predicate, update
//              the running max / sum, write P (f16) into shared memory and,
//              only when a row's max grew by more than 2^8, rescale that row
//              of O in TMEM (tcgen05.ld/st); the epilogue divides O by l.
//   warp 4     TMA producer: K and V tiles of the kv head into a 2-stage ring
//              (cp.async.bulk.tensor, 128-byte swizzle, no multicast).
//   warp 5     MMA issuer (one elected thread):
//                S  = Q K^T   M=128, N=BN keys, K=HD   (A, B K-major)
//                O += P V     M=128, N=HD,      K=BN   (A K-major, B MN-major)
//              completions reach the other roles through tcgen05.commit on
//              mbarriers.
// TMEM: S in columns [0, BN), O in [128, 128 + HD).
//
// Roofline: tensor-bound.  Algorithmic FLOPs per launch = 4 * NH * HD * sum
// over queries of visible keys (masked keys do not count).
#include "common.cuh"
#include "internal.hpp"

namespace svkv {

namespace {

constexpr int kPThreads = 192;
constexpr int kSoftmaxThreads = 128;
constexpr float kRescaleLog2 = 8.0f;     // rescale O only when the max grows by > 2^8

__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;            // descriptor version (sm100)
    d |= (uint64_t)2 << 61;            // 128-byte swizzle
    return d;
}

// kind::f16 instruction descriptor: f32 accumulate, f16 A/B
__device__ __forceinline__ uint32_t umma_idesc(int M, int N, int a_mn_major, int b_mn_major) {
    return (1u << 4) | ((uint32_t)a_mn_major << 15) | ((uint32_t)b_mn_major << 16) | ((uint32_t)(N >> 3) << 17) |
           ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n"
        ".reg .pred p;\n"
        "setp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n"
        "}\n" ::"r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
    uint32_t* r = reinterpret_cast<uint32_t*>(v);
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* v) {
    const uint32_t* r = reinterpret_cast<const uint32_t*>(v);
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
        "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
        "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

template <int HD>
struct PreCfg {
    static constexpr int BN = HD >= 256 ? 64 : 128;      // keys per tile
    static constexpr int NS = 2;                          // K/V stages
    static constexpr int BOX_ROW = 128;                   // bytes per swizzled row (64 f16)
    static constexpr int QBOX = 128 * BOX_ROW;            // one 64-column slab of the Q tile
    static constexpr int Q_B = (HD / 64) * QBOX;
    static constexpr int KBOX = BN * BOX_ROW;             // one 64-column slab of a K or V tile
    static constexpr int KV_B = (HD / 64) * KBOX;         // K (or V) bytes per stage
    static constexpr int STAGE_B = 2 * KV_B;
    static constexpr int PBOX = 128 * BOX_ROW;            // 64 keys x 128 rows of P
    static constexpr int P_B = (BN / 64) * PBOX;
    static constexpr int OFF_Q = 0;
    static constexpr int OFF_ST = OFF_Q + Q_B;
    static constexpr int OFF_P = OFF_ST + NS * STAGE_B;
    static constexpr int OFF_BAR = OFF_P + P_B;
    static constexpr int N_BAR = 2 * NS + 5;
    static constexpr int SMEM = OFF_BAR + N_BAR * 8 + 16;
    static constexpr int OCOL = 128;
    static constexpr int TMEM_COLS = (OCOL + HD) <= 256 ? 256 : 512;
};

__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, int* err, volatile int* abort_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
            if (err) atomicOr(err, ERRBIT_TIMEOUT);
            *abort_flag = 1;
            return false;
        }
    }
}

template <int HD>
__global__ void __launch_bounds__(kPThreads, 1)
fa_prefill_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                  const __grid_constant__ AttnArgs a) {
    using C = PreCfg<HD>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    uint64_t* full = bars;                // [NS]
    uint64_t* empty = bars + C::NS;       // [NS]
    uint64_t* q_full = bars + 2 * C::NS;
    uint64_t* s_full = q_full + 1;
    uint64_t* p_full = q_full + 2;
    uint64_t* o_done = q_full + 3;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::N_BAR);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qt = blockIdx.x, kvh = blockIdx.y;
    const int QPT = 128 / a.G;
    const int t0 = qt * QPT;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::NS; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(q_full, kSoftmaxThreads);
        mbar_init(s_full, 1);
        mbar_init(p_full, kSoftmaxThreads);
        mbar_init(o_done, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"((uint32_t)C::TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (warp == 4 && lane == 0) {
        tma_prefetch_desc(&tmk);
        tma_prefetch_desc(&tmv);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();                      // everything above overlapped the previous kernel
    if (threadIdx.x == 0) pdl_trigger();
    const int cbase = a.causal_base_dev ? __ldg(a.causal_base_dev) : a.causal_base;
    const int nq = min(QPT, a.T - t0);
    const int kend = min(a.S, cbase + t0 + nq);                 // keys [0, kend) reach some row
    const int n_tiles = (kend + C::BN - 1) / C::BN;

    if (warp < 4) {
        // ============================ softmax warps
        const int r = threadIdx.x;                       // row = TMEM lane
        const int qi = r / a.G, g = r % a.G;
        const int t = t0 + qi;
        const bool valid = qi < nq;
        const int qpos = cbase + min(t, a.T - 1);        // invalid rows mirror the last query
        const uint32_t lane_addr = tmem + ((uint32_t)(warp * 32) << 16);
        // ---- Q row -> shared memory (128-byte swizzled, K-major)
        {
            const uint8_t* qrow = a.q + (size_t)(valid ? t : 0) * a.q_nb_t + (size_t)(kvh * a.G + g) * a.q_nb_h;
            uint8_t* qs = smem + C::OFF_Q;
#pragma unroll 4
            for (int e = 0; e < HD; e += 8) {
                uint4 v = make_uint4(0, 0, 0, 0);
                if (valid) {
                    if (a.q_type == SV_TYPE_F32) {
                        const float4 f0 = *reinterpret_cast<const float4*>(qrow + (size_t)e * 4);
                        const float4 f1 = *reinterpret_cast<const float4*>(qrow + (size_t)e * 4 + 16);
                        v.x = pack_h2(f0.x, f0.y);
                        v.y = pack_h2(f0.z, f0.w);
                        v.z = pack_h2(f1.x, f1.y);
                        v.w = pack_h2(f1.z, f1.w);
                    } else {
                        v = *reinterpret_cast<const uint4*>(qrow + (size_t)e * 2);
                    }
                }
                *reinterpret_cast<uint4*>(qs + (e / 64) * C::QBOX + swz_off(r, e % 64, 128)) = v;
            }
            fence_proxy_async_smem();
            mbar_arrive(q_full);
        }
        float m_use = -INFINITY, l = 0.0f;
        for (int j = 0; j < n_tiles; j++) {
            if (!wait_or_abort(s_full, j & 1, a.err, abort_flag)) break;
            tc_fence_after();
            const int kb = j * C::BN;
            float s[C::BN];
#pragma unroll
            for (int c = 0; c < C::BN; c += 32) tmem_ld32(lane_addr + c, s + c);
            tmem_wait_ld();
            const bool need_mask = kb + C::BN - 1 > qpos || kb + C::BN > kend;
            float mt = -INFINITY;
#pragma unroll
            for (int c = 0; c < C::BN; c++) {
                float x = s[c] * a.scale_log2;
                if (need_mask && (kb + c > qpos || kb + c >= kend)) x = -INFINITY;
                s[c] = x;
                mt = fmaxf(mt, x);
            }
            // the previous P.V must be complete before O is rescaled or P is overwritten
            if (j > 0 && !wait_or_abort(o_done, (j - 1) & 1, a.err, abort_flag)) break;
            tc_fence_after();
            float alpha = 1.0f;
            bool resc = false;
            if (j == 0) {
                m_use = mt;
            } else if (mt > m_use + kRescaleLog2) {
                alpha = fast_exp2(m_use - mt);
                m_use = mt;
                resc = true;
            }
            if (__any_sync(0xffffffffu, resc)) {
#pragma unroll 1
                for (int c = 0; c < HD; c += 32) {
                    float o[32];
                    tmem_ld32(lane_addr + C::OCOL + c, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int k = 0; k < 32; k++) o[k] *= alpha;
                    tmem_st32(lane_addr + C::OCOL + c, o);
                }
                tmem_wait_st();
            }
            const float mu = m_use == -INFINITY ? 0.0f : m_use;
            float sum = 0.0f;
            uint8_t* ps = smem + C::OFF_P;
#pragma unroll
            for (int c = 0; c < C::BN; c += 8) {
                float p[8];
#pragma unroll
                for (int k = 0; k < 8; k++) {
                    p[k] = fast_exp2(s[c + k] - mu);
                    sum += p[k];
                }
                uint4 v;
                v.x = pack_h2(p[0], p[1]);
                v.y = pack_h2(p[2], p[3]);
                v.z = pack_h2(p[4], p[5]);
                v.w = pack_h2(p[6], p[7]);
                *reinterpret_cast<uint4*>(ps + (c / 64) * C::PBOX + swz_off(r, c % 64, 128)) = v;
            }
            l = l * alpha + sum;
            fence_proxy_async_smem();
            tc_fence_before();
            mbar_arrive(p_full);
        }
        // ---- epilogue: O / l
        if (n_tiles > 0 && wait_or_abort(o_done, (n_tiles - 1) & 1, a.err, abort_flag)) {
            tc_fence_after();
            const float inv = l > 0.0f ? 1.0f / l : 0.0f;
            float* orow = valid ? a.out + (size_t)t * a.out_nb_t + (size_t)(kvh * a.G + g) * a.out_nb_h : nullptr;
#pragma unroll 1
            for (int c = 0; c < HD; c += 32) {
                float o[32];
                tmem_ld32(lane_addr + C::OCOL + c, o);
                tmem_wait_ld();
                if (valid) {
#pragma unroll
                    for (int k = 0; k < 32; k += 4)
                        *reinterpret_cast<float4*>(orow + c + k) =
                            make_float4(o[k] * inv, o[k + 1] * inv, o[k + 2] * inv, o[k + 3] * inv);
                }
            }
        } else if (n_tiles == 0 && valid) {
            float* orow = a.out + (size_t)t * a.out_nb_t + (size_t)(kvh * a.G + g) * a.out_nb_h;
            for (int c = 0; c < HD; c++) orow[c] = 0.0f;
        }
    } else if (warp == 4) {
        // ============================ TMA producer
        if (lane == 0 && n_tiles > 0) {
            int issued = 0;
            for (int j = 0; j < n_tiles; j++) {
                const int s = j % C::NS;
                if (j >= C::NS && !wait_or_abort(&empty[s], ((j / C::NS) - 1) & 1, a.err, abort_flag)) break;
                uint8_t* kst = smem + C::OFF_ST + s * C::STAGE_B;
                uint8_t* vst = kst + C::KV_B;
                mbar_arrive_expect_tx(&full[s], C::STAGE_B);
                const int y = a.row_base + j * C::BN;
#pragma unroll
                for (int b = 0; b < HD / 64; b++) {
                    tma_load_2d(kst + b * C::KBOX, &tmk, kvh * HD + b * 64, y, &full[s]);
                    tma_load_2d(vst + b * C::KBOX, &tmv, kvh * HD + b * 64, y, &full[s]);
                }
                issued = j + 1;
            }
            for (int j = max(0, issued - C::NS); j < issued; j++)
                mbar_wait(&full[j % C::NS], (j / C::NS) & 1, a.err);
        }
    } else {
        // ============================ MMA issuer
        if (lane == 0 && n_tiles > 0) {
            const uint32_t idesc_s = umma_idesc(128, C::BN, 0, 0);
            const uint32_t idesc_o = umma_idesc(128, HD, 0, 1);
            const uint32_t q_base = smem_u32(smem + C::OFF_Q);
            const uint32_t p_base = smem_u32(smem + C::OFF_P);
            bool ok = wait_or_abort(q_full, 0, a.err, abort_flag);
            tc_fence_after();
            for (int j = 0; ok && j < n_tiles; j++) {
                const int s = j % C::NS;
                if (!wait_or_abort(&full[s], (j / C::NS) & 1, a.err, abort_flag)) break;
                tc_fence_after();
                const uint32_t k_base = smem_u32(smem + C::OFF_ST + s * C::STAGE_B);
                const uint32_t v_base = k_base + C::KV_B;
                // S = Q K^T
#pragma unroll
                for (int kk = 0; kk < HD / 16; kk++) {
                    const uint64_t ad = umma_desc(q_base + (kk / 4) * C::QBOX + (kk % 4) * 32, 16, 1024);
                    const uint64_t bd = umma_desc(k_base + (kk / 4) * C::KBOX + (kk % 4) * 32, 16, 1024);
                    umma_f16(tmem, ad, bd, idesc_s, kk > 0 ? 1u : 0u);
                }
                umma_commit(s_full);
                if (!wait_or_abort(p_full, j & 1, a.err, abort_flag)) break;
                tc_fence_after();
                // O += P V
#pragma unroll
                for (int kk = 0; kk < C::BN / 16; kk++) {
                    const uint64_t ad = umma_desc(p_base + (kk / 4) * C::PBOX + (kk % 4) * 32, 16, 1024);
                    const uint64_t bd = umma_desc(v_base + kk * 16 * 128, C::KBOX, 1024);
                    umma_f16(tmem + C::OCOL, ad, bd, idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
                }
                umma_commit(o_done);
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
cudaError_t launch_t(const AttnArgs& a, const CUtensorMap* tk, const CUtensorMap* tv, cudaStream_t st) {
    using C = PreCfg<HD>;
    static bool attr_set = false;
    const int smem = C::SMEM + 1024;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(fa_prefill_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    const int QPT = 128 / a.G;
    dim3 grid((unsigned)ceil_div(a.T, QPT), (unsigned)a.NKV);
    return launch_pdl(fa_prefill_kernel<HD>, grid, dim3(kPThreads), (size_t)smem, st, *tk, *tv, a);
}

}  // namespace

bool prefill_supported(int head_dim, int kv_type, int G, size_t row_bytes) {
    return kv_type == SV_TYPE_F16 && (head_dim == 128 || head_dim == 256) && G >= 1 && G <= 16 && (128 % G) == 0 &&
           row_bytes % 16 == 0;
}

bool make_prefill_tmap(CUtensorMap* m, const void* base, int head_dim, int n_kv_head, size_t row_bytes,
                       int64_t n_rows) {
    const uint32_t bn = head_dim >= 256 ? 64 : 128;
    return encode_tmap_2d(m, base, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, (uint64_t)n_kv_head * head_dim, (uint64_t)n_rows,
                          row_bytes, 64, bn, CU_TENSOR_MAP_SWIZZLE_128B);
}

cudaError_t launch_prefill(const AttnArgs& a, int head_dim, const CUtensorMap* tk, const CUtensorMap* tv,
                           cudaStream_t st) {
    if (head_dim == 128) return launch_t<128>(a, tk, tv, st);
    if (head_dim == 256) return launch_t<256>(a, tk, tv, st);
    return cudaErrorInvalidValue;
}

}  // namespace svkv
