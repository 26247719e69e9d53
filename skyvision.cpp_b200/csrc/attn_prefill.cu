// attn_prefill.cu - chunked-prefill attention on the 5th-generation tensor
// cores (tcgen05.mma, accumulators in TMEM), sm_100a.
//
// Replaces ggml_flash_attn_ext for prompt chunks (the 512-token ubatches of
// gemma4_model.cpp:1355-1395, the splice tail of qwen3vl_model.cpp:1172-1193)
// over an f16 cache, causal mask as an in-kernel predicate
// (set_causal_mask(mask, n_past, T), attention.hpp:60-67).
//
// Work unit: one 128-row query tile x one kv head x one split of its keys.  The
// 128 rows pack 128/G queries x the G query heads of the kv head, so every K/V
// tile feeds all heads of the GQA group.  The key range of a tile is cut into
// n_splits contiguous parts; the splits of a tile run as one thread-block
// cluster and merge their partial (m, l, O) through distributed shared memory,
// so short prompts still cover every SM.  Warp roles (320 threads):
//   warps 0-7  softmax: warps w and w+4 share TMEM lane quarter w%4 (32 rows)
//              and split the columns (S columns [32h, 32h+32) of each 64-key
//              tile, O columns [h*HD/2, (h+1)*HD/2)).  Load Q into shared memory
//              (128-byte swizzled K-major); per tile read S with tcgen05.ld,
//              apply scale and the causal predicate, exchange the half-row
//              maxima (f16, mbarrier-synchronised), write P (f16) into one of
//              two shared buffers and, only when a row's max grew by more than
//              2^8, rescale that row of O in TMEM (tcgen05.ld/st).  Epilogue:
//              O / l, or the cluster merge.
//   warp 8     TMA producers: lane 0 streams K tiles, lane 1 V tiles, each into
//              its own ring (5 stages at HD 128, 2 at HD 256); a K stage is
//              refilled as soon as its S has completed, a V stage after its P.V.
//   warp 9     MMA issuer (one thread), S double-buffered in TMEM so the
//              tensor core computes S(j+1) while the softmax warps work on S(j):
//                S  = Q K^T   M=128, N=64 keys, K=HD   (A, B K-major)
//                O += P V     M=128, N=HD,      K=64   (A K-major, B MN-major)
//              completions reach the other roles through tcgen05.commit on
//              mbarriers.
// TMEM: S buffers in columns [0, 64) and [64, 128), O in [128, 128 + HD).
//
// Measured limiter (round-trip probes and ncu): with 128 query rows per K/V
// tile each SM must pull ~64 KB of K/V per 1.5 MFLOP-tile pair, and with the
// ~3 us loaded L2 latency the ring that fits beside Q and P cannot keep that in
// flight, so the tensor pipe idles (~15 % of peak).  Feeding 256 query rows per
// K/V tile (two Q tiles per CTA, or a 2-SM cta_group::2 pair) is the next step.
//
// Roofline: tensor-bound.  Algorithmic FLOPs per launch = 4 * NH * HD * sum
// over queries of visible keys (masked keys do not count).
#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "internal.hpp"

namespace svkv {

namespace {

constexpr int kPThreads = 320;          // 8 softmax warps, 1 TMA warp, 1 MMA warp
constexpr int kSoftmaxThreads = 256;
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
    static constexpr int BN = 64;                         // keys per tile (one 128-byte swizzle row of P)
    static constexpr int NS = HD >= 256 ? 2 : 5;          // K/V stages (shared memory budget)
    static constexpr int BOX_ROW = 128;                   // bytes per swizzled row (64 f16)
    static constexpr int QBOX = 128 * BOX_ROW;            // one 64-column slab of the Q tile
    static constexpr int Q_B = (HD / 64) * QBOX;
    static constexpr int KBOX = BN * BOX_ROW;             // one 64-column slab of a K or V tile
    static constexpr int KV_B = (HD / 64) * KBOX;         // K (or V) bytes per stage
    static constexpr int STAGE_B = 2 * KV_B;
    static constexpr int P_B = 128 * BOX_ROW;             // 128 rows x 64 keys of P (one of two buffers)
    static constexpr int OFF_Q = 0;
    static constexpr int OFF_ST = OFF_Q + Q_B;
    static constexpr int OFF_P = OFF_ST + NS * STAGE_B;
    static constexpr int OFF_X = OFF_P + 2 * P_B;        // row-max exchange: f16 [2 parities][2 halves][128]
    static constexpr int OFF_BAR = OFF_X + 2 * 2 * 128 * 2;
    static constexpr int N_BAR = 4 * NS + 7 + 4;         // K and V rings, + one exchange barrier per lane quarter
    static constexpr int SMEM = OFF_BAR + N_BAR * 8 + 16;
    static constexpr int OCOL = 128;                      // S buffers at columns 0 and 64
    static constexpr int TMEM_COLS = (OCOL + HD) <= 256 ? 256 : 512;
    // cluster merge staging after the main loop: partial O [128][HD] f32 over Q + the ring,
    // and (m, l) per row in the P region
    static constexpr int OFF_PO = 0;
    static constexpr int OFF_PM = OFF_P;
    static_assert(128 * HD * 4 <= OFF_P, "partial O must fit in front of the P buffer");
    static_assert(128 * 2 * 4 <= P_B, "row statistics must fit in the P buffer");
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

// wait_or_abort for a whole warp: every lane waits, and the result is the same on all lanes
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* err, volatile int* abort_flag) {
    const bool ok = wait_or_abort(bar, parity, err, abort_flag);
    return __all_sync(0xffffffffu, ok);
}

template <int HD>
__global__ void __launch_bounds__(kPThreads, 1)
fa_prefill_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                  const __grid_constant__ AttnArgs a) {
    using C = PreCfg<HD>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    // K and V rings are separate so a K stage is refilled as soon as its S = Q K^T has completed
    uint64_t* full_k = bars;              // [NS]
    uint64_t* empty_k = bars + C::NS;     // [NS]
    uint64_t* full_v = bars + 2 * C::NS;  // [NS]
    uint64_t* empty_v = bars + 3 * C::NS; // [NS]
    uint64_t* q_full = bars + 4 * C::NS;
    uint64_t* s_full = q_full + 1;        // [2] per S buffer
    uint64_t* p_full = q_full + 3;
    uint64_t* o_done = q_full + 4;        // [2] per P buffer: P.V of the tiles that used it
    uint64_t* xbar = q_full + 6;          // [4] the two softmax warps of a lane quarter exchanged their halves
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::N_BAR);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int split = blockIdx.x, qt = blockIdx.y, kvh = blockIdx.z;
    const int ns = a.n_splits;
    const int QPT = 128 / a.G;
    const int t0 = qt * QPT;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::NS; s++) {
            mbar_init(&full_k[s], 1);
            mbar_init(&empty_k[s], 1);
            mbar_init(&full_v[s], 1);
            mbar_init(&empty_v[s], 1);
        }
        // the softmax warps arrive once per warp (lane 0 after __syncwarp)
        mbar_init(q_full, kSoftmaxThreads / 32);
        mbar_init(&s_full[0], 1);
        mbar_init(&s_full[1], 1);
        mbar_init(p_full, kSoftmaxThreads / 32);
        mbar_init(&o_done[0], 1);
        mbar_init(&o_done[1], 1);
        for (int k = 0; k < 4; k++) mbar_init(&xbar[k], 2);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"((uint32_t)C::TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (warp == 8 && lane == 0) {
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
    const int nt = (kend + C::BN - 1) / C::BN;                  // tiles of the whole key range
    const int j0 = (int)((long long)nt * split / ns);           // this split's tiles [j0, j1)
    const int j1 = (int)((long long)nt * (split + 1) / ns);
    const int n = j1 - j0;
    // The query tiles of one kv head stream the same K/V tiles; each starts at a different
    // rotation of its range so they do not hit the same L2 lines in lockstep (the online
    // softmax does not depend on the order of the tiles).
    const int rot = n > 0 ? (qt * 7) % n : 0;
    auto tile_of = [&](int i) { return j0 + (i + rot) % n; };

    if (warp < 8) {
        // ============================ softmax warps
        // Warps w and w+4 read the same TMEM lane quarter (w % 4), i.e. the same 32 rows, and
        // split the columns: half ch = w / 4 owns S columns [32ch, 32ch + 32) of every tile and
        // O columns [ch*HD/2, (ch+1)*HD/2).  The two halves exchange row maxima through shared
        // memory once per tile and their partial sums once at the end.
        const int quarter = warp & 3, ch = warp >> 2;
        const int r = quarter * 32 + lane;               // row = TMEM lane
        const int qi = r / a.G, g = r % a.G;
        const int t = t0 + qi;
        const bool valid = qi < nq;
        const int qpos = cbase + min(t, a.T - 1);        // invalid rows mirror the last query
        const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16);
        const float c = a.scale_log2;
        __half* xch = reinterpret_cast<__half*>(smem + C::OFF_X);   // [2 parities][2 halves][128 rows]
        uint64_t* xb = &xbar[quarter];
        // ---- Q: each thread loads half of its row (128-byte swizzled, K-major)
        {
            const uint8_t* qrow = a.q + (size_t)(valid ? t : 0) * a.q_nb_t + (size_t)(kvh * a.G + g) * a.q_nb_h;
            uint8_t* qs = smem + C::OFF_Q;
#pragma unroll 4
            for (int e = ch * (HD / 2); e < (ch + 1) * (HD / 2); e += 8) {
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
            __syncwarp();
            if (lane == 0) mbar_arrive(q_full);
        }
        float m_use = -INFINITY, l = 0.0f;               // l: this half's partial row sum
        bool ok = true;
        for (int i = 0; i < n; i++) {
            if (!warp_wait(&s_full[i & 1], (i >> 1) & 1, a.err, abort_flag)) { ok = false; break; }
            tc_fence_after();
            const int kb = tile_of(i) * C::BN + ch * 32;  // first key of this half
            float s[32];
            tmem_ld32(lane_addr + (i & 1) * C::BN + ch * 32, s);
            tmem_wait_ld();
            // keys past the row's position (or past kend) are masked; only the last tiles have any
            if (kb + 31 > qpos || kb + 32 > kend) {
#pragma unroll
                for (int k = 0; k < 32; k++)
                    if (kb + k > qpos || kb + k >= kend) s[k] = -INFINITY;
            }
            float m8[8];
#pragma unroll
            for (int k = 0; k < 8; k++) m8[k] = fmaxf(fmaxf(s[k], s[k + 8]), fmaxf(s[k + 16], s[k + 24]));
            float mr = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                             fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7])));
            {
                // both halves use the f16-rounded maxima, so they agree on the row's offset; the
                // offset only has to be near the true maximum (p stays far below f16 overflow)
                __half* slot = xch + (i & 1) * 2 * 128;
                const __half mine = __float2half_ru(fminf(mr, 65504.0f));
                slot[ch * 128 + r] = mine;
                __syncwarp();
                if (lane == 0) mbar_arrive(xb);
                if (!warp_wait(xb, i & 1, a.err, abort_flag)) { ok = false; break; }
                mr = fmaxf(__half2float(mine), __half2float(slot[(1 - ch) * 128 + r]));
            }
            const float mt = mr * c;                     // scale > 0 commutes with max
            float alpha = 1.0f;
            bool resc = false;
            if (i == 0) {
                m_use = mt;
            } else if (mt > m_use + kRescaleLog2) {
                alpha = fast_exp2(m_use - mt);
                m_use = mt;
                resc = true;
            }
            // P buffer i&1 was last read by P.V(i-2); a rescale of O needs P.V(i-1) complete
            if (i >= 2) {
                if (!warp_wait(&o_done[i & 1], ((i - 2) >> 1) & 1, a.err, abort_flag)) { ok = false; break; }
                tc_fence_after();
            }
            const bool any_resc = __any_sync(0xffffffffu, resc);
            if (any_resc) {
                if (!warp_wait(&o_done[(i - 1) & 1], ((i - 1) >> 1) & 1, a.err, abort_flag)) { ok = false; break; }
                tc_fence_after();
#pragma unroll 1
                for (int cc = ch * (HD / 2); cc < (ch + 1) * (HD / 2); cc += 32) {
                    float o[32];
                    tmem_ld32(lane_addr + C::OCOL + cc, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int k = 0; k < 32; k++) o[k] *= alpha;
                    tmem_st32(lane_addr + C::OCOL + cc, o);
                }
                tmem_wait_st();
            }
            const float mneg = m_use == -INFINITY ? 0.0f : -m_use;
            float sum4[4] = {0.f, 0.f, 0.f, 0.f};
            uint8_t* ps = smem + C::OFF_P + (i & 1) * C::P_B;
#pragma unroll
            for (int cc = 0; cc < 32; cc += 8) {
                float p[8];
#pragma unroll
                for (int k = 0; k < 8; k++) {
                    p[k] = fast_exp2(fmaf(s[cc + k], c, mneg));
                    sum4[k & 3] += p[k];
                }
                uint4 v;
                v.x = pack_h2(p[0], p[1]);
                v.y = pack_h2(p[2], p[3]);
                v.z = pack_h2(p[4], p[5]);
                v.w = pack_h2(p[6], p[7]);
                *reinterpret_cast<uint4*>(ps + swz_off(r, ch * 32 + cc, 128)) = v;
            }
            l = l * alpha + ((sum4[0] + sum4[1]) + (sum4[2] + sum4[3]));
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full);
        }
        if (n > 0 && ok && !warp_wait(&o_done[(n - 1) & 1], ((n - 1) >> 1) & 1, a.err, abort_flag)) ok = false;
        tc_fence_after();
        // the row sum: both halves' partial sums (a slot set the last tile did not use)
        float L = l;
        if (ok) {
            // P buffer 1 is free once the last P.V has completed: it carries the f32 half sums
            float* lx = reinterpret_cast<float*>(smem + C::OFF_P + C::P_B);
            lx[ch * 128 + r] = l;
            __syncwarp();
            if (lane == 0) mbar_arrive(xb);
            if (warp_wait(xb, n & 1, a.err, abort_flag)) L = l + lx[(1 - ch) * 128 + r];
        }
        float* orow = valid ? a.out + (size_t)t * a.out_nb_t + (size_t)(kvh * a.G + g) * a.out_nb_h : nullptr;
        if (ns == 1) {
            // ---- single split: this half of O / L straight out of TMEM
            const float inv = L > 0.0f ? 1.0f / L : 0.0f;
#pragma unroll 1
            for (int cc = ch * (HD / 2); cc < (ch + 1) * (HD / 2); cc += 32) {
                float o[32];
                if (n > 0) {
                    tmem_ld32(lane_addr + C::OCOL + cc, o);
                    tmem_wait_ld();
                } else {
#pragma unroll
                    for (int k = 0; k < 32; k++) o[k] = 0.0f;
                }
                if (valid) {
#pragma unroll
                    for (int k = 0; k < 32; k += 4)
                        *reinterpret_cast<float4*>(orow + cc + k) =
                            make_float4(o[k] * inv, o[k + 1] * inv, o[k + 2] * inv, o[k + 3] * inv);
                }
            }
        } else {
            // ---- split: stage the unnormalised partial in shared memory for the cluster merge
            // (the last tile's P.V is complete, so Q, the K/V ring and P are free)
            float* po = reinterpret_cast<float*>(smem + C::OFF_PO);
            float* pm = reinterpret_cast<float*>(smem + C::OFF_PM);
#pragma unroll 1
            for (int cc = ch * (HD / 2); cc < (ch + 1) * (HD / 2); cc += 32) {
                float o[32];
                if (n > 0) {
                    tmem_ld32(lane_addr + C::OCOL + cc, o);
                    tmem_wait_ld();
                } else {
#pragma unroll
                    for (int k = 0; k < 32; k++) o[k] = 0.0f;
                }
#pragma unroll
                for (int k = 0; k < 32; k += 4)
                    *reinterpret_cast<float4*>(&po[r * HD + cc + k]) = make_float4(o[k], o[k + 1], o[k + 2], o[k + 3]);
            }
            if (ch == 0) {
                pm[r * 2] = n > 0 ? m_use : -INFINITY;
                pm[r * 2 + 1] = n > 0 ? L : 0.0f;
            }
        }
    } else if (warp == 8) {
        // ============================ TMA producers: lane 0 streams K tiles, lane 1 V tiles
        if (lane < 2 && n > 0) {
            const bool is_v = lane == 1;
            uint64_t* fullx = is_v ? full_v : full_k;
            uint64_t* emptyx = is_v ? empty_v : empty_k;
            const CUtensorMap* tm = is_v ? &tmv : &tmk;
            int issued = 0;
            for (int i = 0; i < n; i++) {
                const int s = i % C::NS;
                if (i >= C::NS && !wait_or_abort(&emptyx[s], ((i / C::NS) - 1) & 1, a.err, abort_flag)) break;
                uint8_t* dst = smem + C::OFF_ST + s * C::STAGE_B + (is_v ? C::KV_B : 0);
                mbar_arrive_expect_tx(&fullx[s], C::KV_B);
                const int y = a.row_base + tile_of(i) * C::BN;
#pragma unroll
                for (int b = 0; b < HD / 64; b++) tma_load_2d(dst + b * C::KBOX, tm, kvh * HD + b * 64, y, &fullx[s]);
                issued = i + 1;
            }
            for (int i = max(0, issued - C::NS); i < issued; i++)
                mbar_wait(&fullx[i % C::NS], (i / C::NS) & 1, a.err);
        }
    } else {
        // ============================ MMA issuer
        if (lane == 0 && n > 0) {
            const uint32_t idesc_s = umma_idesc(128, C::BN, 0, 0);
            const uint32_t idesc_o = umma_idesc(128, HD, 0, 1);
            const uint32_t q_base = smem_u32(smem + C::OFF_Q);
            const uint32_t p_base = smem_u32(smem + C::OFF_P);
            auto issue_s = [&](int i) {          // S(i) = Q K(i)^T into buffer i & 1
                const uint32_t k_base = smem_u32(smem + C::OFF_ST + (i % C::NS) * C::STAGE_B);
#pragma unroll
                for (int kk = 0; kk < HD / 16; kk++) {
                    const uint64_t ad = umma_desc(q_base + (kk / 4) * C::QBOX + (kk % 4) * 32, 16, 1024);
                    const uint64_t bd = umma_desc(k_base + (kk / 4) * C::KBOX + (kk % 4) * 32, 16, 1024);
                    umma_f16(tmem + (i & 1) * C::BN, ad, bd, idesc_s, kk > 0 ? 1u : 0u);
                }
                umma_commit(&s_full[i & 1]);
                umma_commit(&empty_k[i % C::NS]);   // the K stage is free once S(i) has completed
            };
            bool ok = wait_or_abort(q_full, 0, a.err, abort_flag);
            if (ok) ok = wait_or_abort(&full_k[0], 0, a.err, abort_flag);
            tc_fence_after();
            if (ok) issue_s(0);
            for (int i = 0; ok && i < n; i++) {
                // S(i+1) overlaps the softmax of tile i (its buffer held S(i-1), already consumed)
                if (i + 1 < n) {
                    const int s1 = (i + 1) % C::NS;
                    if (!wait_or_abort(&full_k[s1], ((i + 1) / C::NS) & 1, a.err, abort_flag)) break;
                    tc_fence_after();
                    issue_s(i + 1);
                }
                if (!wait_or_abort(p_full, i & 1, a.err, abort_flag)) break;
                if (!wait_or_abort(&full_v[i % C::NS], (i / C::NS) & 1, a.err, abort_flag)) break;
                tc_fence_after();
                const uint32_t v_base = smem_u32(smem + C::OFF_ST + (i % C::NS) * C::STAGE_B) + C::KV_B;
                const uint32_t pb = p_base + (i & 1) * C::P_B;
#pragma unroll
                for (int kk = 0; kk < C::BN / 16; kk++) {
                    const uint64_t ad = umma_desc(pb + kk * 32, 16, 1024);
                    const uint64_t bd = umma_desc(v_base + kk * 16 * 128, C::KBOX, 1024);
                    umma_f16(tmem + C::OCOL, ad, bd, idesc_o, (i > 0 || kk > 0) ? 1u : 0u);
                }
                umma_commit(&o_done[i & 1]);
                umma_commit(&empty_v[i % C::NS]);
            }
        }
    }

    if (ns > 1) {
        // ============================ cluster merge of the splits (all 192 threads of every CTA)
        __syncwarp();
        cluster_sync_all();
        const uint32_t rank = cluster_ctarank();
        const float* po = reinterpret_cast<const float*>(smem + C::OFF_PO);
        const float* pm = reinterpret_cast<const float*>(smem + C::OFF_PM);
        // rows [r0, r1) of the tile are merged by this CTA
        const int r0 = (int)(128 * rank / ns), r1 = (int)(128 * (rank + 1) / ns);
        constexpr int G4 = HD / 4;
        for (int gi = threadIdx.x; gi < (r1 - r0) * G4; gi += kPThreads) {
            const int r = r0 + gi / G4, cc = (gi % G4) * 4;
            const int qi = r / a.G, g = r % a.G;
            if (qi >= nq) continue;
            float M = -INFINITY;
            for (int sp = 0; sp < ns; sp++) M = fmaxf(M, dsmem_ld_f2(dsmem_map(smem_u32(&pm[r * 2]), sp)).x);
            float L = 0.0f;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int sp = 0; sp < ns; sp++) {
                const float2 ml = dsmem_ld_f2(dsmem_map(smem_u32(&pm[r * 2]), sp));
                if (ml.x == -INFINITY) continue;
                const float w = fast_exp2(ml.x - M);
                const float4 v = dsmem_ld_f4(dsmem_map(smem_u32(&po[r * HD + cc]), sp));
                L += ml.y * w;
                acc.x += v.x * w; acc.y += v.y * w; acc.z += v.z * w; acc.w += v.w * w;
            }
            const float inv = L > 0.0f ? 1.0f / L : 0.0f;
            float* orow = a.out + (size_t)(t0 + qi) * a.out_nb_t + (size_t)(kvh * a.G + g) * a.out_nb_h;
            *reinterpret_cast<float4*>(orow + cc) = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
        }
        cluster_sync_all();          // every CTA's partial stays valid until all merges read it
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)C::TMEM_COLS));
    }
}

template <int HD>
cudaError_t prepare_t() {
    static cudaError_t status = [] {
        using C = PreCfg<HD>;
        cudaError_t e = cudaFuncSetAttribute(fa_prefill_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             C::SMEM + 1024);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(fa_prefill_kernel<HD>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        return e;
    }();
    return status;
}

// Splits of the key range per query tile: the fewest that make the CTA count fill whole waves
// of the SMs best (one CTA per SM), at most 8 per cluster and at least 2 tiles per split.
int pick_splits(int base_ctas, int min_tiles) {
    int best = 1;
    double best_t = 1e30;
    for (int s = 1; s <= 8; s++) {
        if (s > 1 && min_tiles / s < 2) break;
        const double waves = std::ceil((double)base_ctas * s / kNumSMs);
        const double t = waves / s;
        if (t < best_t - 1e-9) {
            best_t = t;
            best = s;
        }
    }
    return best;
}

template <int HD>
cudaError_t launch_t(const AttnArgs& a_in, const CUtensorMap* tk, const CUtensorMap* tv, cudaStream_t st) {
    using C = PreCfg<HD>;
    cudaError_t e = prepare_t<HD>();
    if (e != cudaSuccess) return e;
    AttnArgs a = a_in;
    const int QPT = 128 / a.G;
    const int n_qtiles = ceil_div(a.T, QPT);
    // the first query tile sees the fewest keys: size the splits by it
    const int cb = a.causal_base;                       // host value (device-side bases use max keys)
    const int min_keys = a.causal_base_dev ? a.S : std::min(a.S, cb + std::min(QPT, a.T));
    a.n_splits = pick_splits(n_qtiles * a.NKV, (min_keys + C::BN - 1) / C::BN);
    dim3 grid((unsigned)a.n_splits, (unsigned)n_qtiles, (unsigned)a.NKV);
    return launch_pdl_cluster(fa_prefill_kernel<HD>, grid, dim3(kPThreads), (size_t)(C::SMEM + 1024), st,
                              a.n_splits, *tk, *tv, a);
}

}  // namespace

bool prefill_supported(int head_dim, int kv_type, int G, size_t row_bytes) {
    return kv_type == SV_TYPE_F16 && (head_dim == 128 || head_dim == 256) && G >= 1 && G <= 16 && (128 % G) == 0 &&
           row_bytes % 16 == 0;
}

bool make_prefill_tmap(CUtensorMap* m, const void* base, int head_dim, int n_kv_head, size_t row_bytes,
                       int64_t n_rows) {
    return encode_tmap_2d(m, base, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, (uint64_t)n_kv_head * head_dim, (uint64_t)n_rows,
                          row_bytes, 64, PreCfg<128>::BN, CU_TENSOR_MAP_SWIZZLE_128B);
}

cudaError_t launch_prefill(const AttnArgs& a, int head_dim, const CUtensorMap* tk, const CUtensorMap* tv,
                           cudaStream_t st) {
    if (head_dim == 128) return launch_t<128>(a, tk, tv, st);
    if (head_dim == 256) return launch_t<256>(a, tk, tv, st);
    return cudaErrorInvalidValue;
}

}  // namespace svkv
