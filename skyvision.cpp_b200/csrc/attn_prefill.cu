// attn_prefill.cu - chunked-prefill attention on the 5th-generation tensor
// cores (tcgen05.mma, accumulators in TMEM), sm_100a.
//
// Replaces ggml_flash_attn_ext for prompt chunks (the 512-token ubatches of
// gemma4_model.cpp:1355-1395, the splice tail of qwen3vl_model.cpp:1172-1193)
// over an f16 cache, or a q8_0 cache whose visible rows q8_0_split_kernel (end of
// this file) rewrote as f16 (hi, lo) planes: K and V tiles then enter the MMA as two
// parts each (NP = 2) and P as two parts (PL = 2), so the q8_0 values and the
// weights keep ~22 bits.  Causal mask as an in-kernel predicate
// (set_causal_mask(mask, n_past, T), attention.hpp:60-67).
//
// Work unit: NQT query tiles of 128 rows (NQT = 2 at HD 128 when the chunk has two) x one kv
// head x one split of its keys.  A tile's 128 rows pack 128/G queries x the G query heads of the
// kv head, so every K/V tile feeds all heads of the GQA group, and with NQT = 2 each K/V tile
// read from L2 feeds 256 rows.  Warp roles ((4*NQT + 3) warps):
//   softmax warps (4 per query tile; warp w reads TMEM lane quarter w % 4, one row per thread):
//              per key tile read S (BN columns) with tcgen05.ld, apply scale and the causal
//              predicate, take the row max, write P = exp2(S - m) as f16 over the first BN/2
//              columns of the same TMEM buffer (the P.V MMA reads A from TMEM), and, when the
//              row max grew, rescale the row of O in TMEM after the exponentials.  One
//              exponential in four runs on the FMA pipe (exp2_fma) to take load off the SFU
//              (two in four measured slower: the FMA pipe, not the SFU, is the tighter one).
//   TMA warps  one lane of the first loads the query tiles (a 3D map over [T][NH][HD] whose
//              {64, G, 128/G} box is one slab of a tile) and streams K tiles, one lane of the second
//              V tiles, each into its own ring (5 stages at HD 128, 2 at HD 256); a K stage is
//              refilled as soon as its S has completed, a V stage after its P.V.  The two rings have
//              a warp each: as two lanes of one warp, a V lane blocked in its slot wait held back the
//              K lane's loads (~450 cycles of the MMA thread's wait per tile, in-kernel stamps).
//   MMA warp   (one thread)
//                S  = Q K^T   M=128, N=BN keys, K=HD   (A, B K-major, shared memory)
//                O += P V     M=128, N=HD,      K=BN   (A = P from TMEM, B = V MN-major)
//              completions reach the other roles through tcgen05.commit on mbarriers (per
//              parity of the tile index where a role can run a tile ahead).
//              BN = 64 (one query tile, HD 256, q8_0 parts): S double-buffered per query tile,
//              so the tensor core computes S(j+1) while the softmax warps work on S(j).
//              BN = 128 (two query tiles of an f16 cache at HD 128): one 128-column S buffer per
//              query tile; S_q(j+1) is issued right after P.V_q(j) (it overwrites P_q(j); the
//              tensor pipe runs in order), and the query tiles alternate, so the tensor core runs
//              P.V_1(j), S_1(j+1) while query tile 0's softmax works on S_0(j+1).  N = 128 S MMAs
//              halve the S instructions per key: the tensor front end takes an N = 64 MMA about
//              every 84 cycles, barely more than the N = 128 one's ~92 cycles of work.
// TMEM per query tile: S/P buffers in columns [0, 64) and [64, 128) (BN = 64) or one buffer in
// [0, 128) (BN = 128), O in [128, 128 + HD).
// Splits: when the units (query tiles x kv heads) are fewer than the SMs, the key range of a
// unit is cut into up to 8 splits (one CTA per SM, no clusters, so every SM is usable).  The
// splits take an arrival ticket; all but the last publish their partial (O, m, l) to the
// handle's workspace, and the last waits (bounded) for them and merges with its own partial,
// which never leaves TMEM.
//
// Measured (config 2 splice tail, 384 over 4096 cached rows, one B200): 448 TFLOP/s over 36
// layers with 64-key tiles, 490 with 128-key tiles; config 4's q8_0 chunks ~297 TFLOP/s
// (algorithmic).  In-kernel clock stamps per 128-key tile (two query tiles): ~4950 cycles a
// tile.  Per query tile the softmax takes ~2900 (S load 185, max + exponentials ~1780, O rescale
// and P store ~940) and its P.V + next S MMAs ~1800 (the issuing thread blocks ~92 cycles per
// N = 128 S MMA and ~130 per P.V MMA), one after the other, so the tensor pipe idles ~30 % of a
// tile.  Measured and dropped: two threads per row (16 softmax warps: the 19-warp block gets 96
// registers and spills, 169 TFLOP/s); a two-pass softmax whose TMEM reloads overlap the
// exponentials (386); a rescale threshold of 2^8 (the dominant weights' f16 rounding then
// breaks the 2e-3 gate on x8-outlier V rows, even with the row sum taken over rounded weights).
//
// Roofline: tensor-bound.  Algorithmic FLOPs per launch = 4 * NH * HD * sum
// over queries of visible keys (masked keys do not count).
#include <algorithm>
#include <cmath>
#include <cstring>

#include "common.cuh"
#include "internal.hpp"
#include "umma.cuh"

namespace svkv {

namespace {

// O is rescaled whenever a row's max grows, so the largest weight of every tile is exactly 1 in f16.
// (A lazy rescale that lets the running max trail by up to 2^8 saves the O round trips but rounds the
// dominant weights: with x8 outlier V rows it cost ~1e-3 of max-abs error, measured on the GPU.)
constexpr float kRescaleLog2 = 0.0f;
// softmax exponentials per four that run on the FMA pipe (exp2_fma); the rest use the SFU (two in four
// measured slower: 490 -> 450 TFLOP/s on the config 2 tail)
constexpr int kExpFma = 1;
// P parts on f16 caches (1: P rounded to f16, standard flash-attention precision)
constexpr int kF16PParts = 1;

// 2^x on the FMA pipe, for part of the softmax exponentials (the SFU's ex2 rate, 16 per clock per
// SM, is below the tensor pipe's rate for 64-key tiles).  x = n + f with n = round(x), f in
// [-0.5, 0.5]; 2^f by a degree-4 polynomial fitted here for minimax relative error on that interval
// (Lawson's iteratively reweighted least squares; max relative error 2.7e-6 in f32 Horner form,
// far under the f16 rounding P gets), and 2^n added into the exponent field.  A degree-3 fit
// (7.5e-5) showed in the outputs of V rows with x8 outliers.  x is clamped at -126 (2^-126 rounds
// to 0 in f16); x <= kRescaleLog2 because P is taken against the running max.
__device__ __forceinline__ float exp2_fma(float x) {
    x = fmaxf(x, -126.0f);
    const float t = x + 12582912.0f;             // 1.5 * 2^23: round(x) lands in the low mantissa bits
    const float f = x - (t - 12582912.0f);
    const float p = fmaf(fmaf(fmaf(fmaf(0.00956530869f, f, 0.05591748655f), f, 0.2402486354f), f, 0.6931219101f), f,
                         0.9999992251f);
    return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

// NQT query tiles of 128 rows per CTA share every K/V tile (NQT = 2 at HD 128).  NP = 1: f16 cache
// tiles; NP = 2: every K and V tile arrives as two f16 parts (hi, lo) whose sum is the exact
// dequantised q8_0 value, and both parts go through the tensor core into the same accumulator.
// The K and V rings hold single parts ("entries"), so a tile takes NP consecutive entries.
// BN = keys per tile.  BN = 64: S double-buffered per Q tile (two 64-column buffers); BN = 128 (f16,
// HD 128): one 128-column S buffer per Q tile, and the two Q tiles alternate on the tensor core, so
// every S MMA is N = 128 (half the S instructions per key of BN = 64).
template <int HD, int NQT, int NP = 1, int BN_ = 64>
struct PreCfg {
    static constexpr int BN = BN_;                        // keys per tile
    static constexpr bool S2 = BN == 64;                  // S double-buffered per Q tile

    static constexpr int BOX_ROW = 128;                   // bytes per swizzled row (64 f16)
    static constexpr int QBOX = 128 * BOX_ROW;            // one 64-column slab of a Q tile
    static constexpr int Q_B = (HD / 64) * QBOX;          // one Q tile
    static constexpr int KBOX = BN * BOX_ROW;             // one 64-column slab of a K or V tile
    static constexpr int KV_B = (HD / 64) * KBOX;         // one part of a K (or V) tile: a ring entry
    static constexpr int ENT_FIT = (227 * 1024 - NQT * Q_B - 2048) / KV_B;
    // f16: up to 5 stages of (K, V) (BN = 128: the entries that fit, one more for K); hi + lo parts:
    // the entries that fit, split between K and V
    static constexpr int NEK = NP == 1 ? (BN == 128 ? (ENT_FIT + 1) / 2 : (ENT_FIT / 2 > 5 ? 5 : ENT_FIT / 2))
                                       : ((ENT_FIT + 1) / 2 > 5 * NP ? 5 * NP : (ENT_FIT + 1) / 2);
    static constexpr int NEV = NP == 1 ? (BN == 128 ? ENT_FIT / 2 : NEK) : (ENT_FIT / 2 > 5 * NP ? 5 * NP : ENT_FIT / 2);
    static_assert(NEK >= 2 && NEK >= NP && NEV >= NP && NEV >= 2, "K/V rings need two entries and a whole tile");
    static_assert(BN == 64 || (BN == 128 && NP == 1), "128-key tiles: f16 caches");
    static constexpr int OFF_Q = 0;
    static constexpr int OFF_K = OFF_Q + NQT * Q_B;
    static constexpr int OFF_V = OFF_K + NEK * KV_B;
    static constexpr int OFF_BAR = OFF_V + NEV * KV_B;
    static constexpr int N_BAR = 2 * NEK + 2 * NEV + 1 + NQT * 6;
    static constexpr int SMEM = OFF_BAR + N_BAR * 8 + 16;
    static_assert(SMEM + 1024 <= 227 * 1024, "shared memory budget");
    static constexpr int QCOLS = 128 + HD;                // per Q tile: S/P buffer(s) in [0, 128), O after
    static constexpr int TMEM_COLS = NQT * QCOLS <= 256 ? 256 : 512;
    static_assert(NQT * QCOLS <= 512, "TMEM budget");
    static constexpr int SM_WARPS = 4 * NQT;              // softmax warps: one row per thread
    static constexpr int THREADS = (SM_WARPS + 3) * 32;   // + K and V producer warps + MMA warp
    static constexpr int ROWS = NQT * 128;
};

// O += P V with P (f16, K-major) read from TMEM; B as (lo, hi) descriptor words
__device__ __forceinline__ void umma_f16_ts_w(uint32_t d_tmem, uint32_t a_tmem, uint32_t b_lo, uint32_t b_hi,
                                              uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n"
        ".reg .pred p;\n"
        ".reg .b64 db;\n"
        "setp.ne.b32 p, %5, 0;\n"
        "mov.b64 db, {%2, %3};\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], db, %4, p;\n"
        "}\n" ::"r"(d_tmem), "r"(a_tmem), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(acc));
}

// Named barrier of the softmax warps.  Code before it may have run on one lane only (a ticket,
// a bounded spin), so the warp reconverges first: the barrier instruction must be executed by
// whole warps.
template <int kSoftmaxWarps>
__device__ __forceinline__ void softmax_sync() {
    __syncwarp();
    asm volatile("barrier.sync 2, %0;" ::"n"(kSoftmaxWarps * 32) : "memory");
}

// tmk/tmv: the f16 cache tensors, or (NP = 2) the hi parts; tmk2/tmv2: the lo parts (NP = 2 only).
// PL = 2: P goes to the tensor core as f16 hi + lo parts (O += P_hi V + P_lo V_hi), so the weights
// keep ~22 bits; PL = 1: P rounded to f16.
template <int HD, int NQT, int NP, int PL, int BN>
__global__ void __launch_bounds__(PreCfg<HD, NQT, NP, BN>::THREADS, 1)
fa_prefill_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                  const __grid_constant__ CUtensorMap tmk2, const __grid_constant__ CUtensorMap tmv2,
                  const __grid_constant__ CUtensorMap tmq, const __grid_constant__ AttnArgs a) {
    using C = PreCfg<HD, NQT, NP, BN>;
    constexpr int kSoftmaxWarps = C::SM_WARPS;
    constexpr int kTmaWarp = kSoftmaxWarps;   // Q and K producer; then the V producer and the MMA issuer
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    // K and V rings are separate so a K stage is refilled as soon as its S = Q K^T has completed
    uint64_t* full_k = bars;                          // [NEK]
    uint64_t* empty_k = bars + C::NEK;                // [NEK]
    uint64_t* full_v = bars + 2 * C::NEK;             // [NEV]
    uint64_t* empty_v = bars + 2 * C::NEK + C::NEV;   // [NEV]
    uint64_t* q_full = bars + 2 * C::NEK + 2 * C::NEV;
    uint64_t* s_full = q_full + 1;        // [NQT][2] per Q tile and S buffer
    // [NQT][2] P(i) written, by the parity of i: the softmax warps can finish tile i+1 before the
    // MMA warp has taken P(i) (S(i+1) is issued first), so one barrier would be two phases ahead
    uint64_t* p_full = s_full + 2 * NQT;
    uint64_t* o_done = p_full + 2 * NQT;  // [NQT][2] P.V(i) of the Q tile, by the parity of i
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::N_BAR);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* last_flag = abort_flag + 1;   // split merge: this CTA is the last split of its unit

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int split = blockIdx.x, qp = blockIdx.y, kvh = blockIdx.z;
    const int ns = a.n_splits;
    const int QPT = 128 / a.G;
    const int t0 = qp * NQT * QPT;                       // first query of the CTA's first Q tile
    const int nq_all = min(NQT * QPT, a.T - t0);         // queries of this CTA
    const int nqt = (nq_all + QPT - 1) / QPT;            // Q tiles with any query (1..NQT)

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::NEK; s++) {
            mbar_init(&full_k[s], 1);
            mbar_init(&empty_k[s], 1);
        }
        for (int s = 0; s < C::NEV; s++) {
            mbar_init(&full_v[s], 1);
            mbar_init(&empty_v[s], 1);
        }
        // f16 queries arrive by TMA (one arrival with the byte count); f32 ones are converted by the
        // softmax warps (one arrival per warp)
        mbar_init(q_full, a.q_tma ? 1 : kSoftmaxWarps);
        for (int q = 0; q < NQT; q++) {
            mbar_init(&s_full[2 * q], 1);
            mbar_init(&s_full[2 * q + 1], 1);
            mbar_init(&p_full[2 * q], 4);
            mbar_init(&p_full[2 * q + 1], 4);
            mbar_init(&o_done[2 * q], 1);
            mbar_init(&o_done[2 * q + 1], 1);
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"((uint32_t)C::TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (warp == kTmaWarp && lane == 0) {
        tma_prefetch_desc(&tmk);
        tma_prefetch_desc(&tmv);
        if (NP == 2) {
            tma_prefetch_desc(&tmk2);
            tma_prefetch_desc(&tmv2);
        }
        if (a.q_tma) tma_prefetch_desc(&tmq);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();                      // everything above overlapped the previous kernel
    if (threadIdx.x == 0) pdl_trigger();
    const int cbase = a.causal_base_dev ? __ldg(a.causal_base_dev) : a.causal_base;
    const int kend = min(a.S, cbase + t0 + nq_all);             // keys [0, kend) reach some row
    const int nt = (kend + C::BN - 1) / C::BN;                  // tiles of the whole key range
    const int j0 = (int)((long long)nt * split / ns);           // this split's tiles [j0, j1)
    const int j1 = (int)((long long)nt * (split + 1) / ns);
    const int n = j1 - j0;
    // The CTAs of one kv head stream the same K/V tiles; each starts at a different rotation of
    // its range so they do not hit the same L2 lines in lockstep (the online softmax does not
    // depend on the order of the tiles).
    const int rot = n > 0 ? (qp * 7) % n : 0;
    auto tile_of = [&](int i) { return j0 + (i + rot) % n; };

    if (warp < kSoftmaxWarps) {
        // ============================ softmax warps: one row of one Q tile per thread
        // Q tile qtl = warp / 4, TMEM lane quarter warp % 4 (rows 32*quarter + lane).  Per key tile:
        // S (BN columns) from TMEM, scale and causal mask, row max, P = exp2(S - m) written back as
        // f16 over the first BN/2 columns of the same TMEM buffer (the P.V MMA reads it from there),
        // and, when the row max grew, O rescaled in TMEM.
        const int qtl = warp >> 2, quarter = warp & 3;
        const bool tile_live = qtl < nqt;
        const int r = quarter * 32 + lane;               // row = TMEM lane
        const int qi = qtl * QPT + r / a.G, g = r % a.G;
        const int t = t0 + qi;
        const bool valid = qi < nq_all;
        const int qpos = cbase + min(t, a.T - 1);        // invalid rows mirror the last query
        const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(qtl * C::QCOLS);
        const float c = a.scale_log2;
        uint64_t* sf = &s_full[2 * qtl];
        uint64_t* pf = &p_full[2 * qtl];
        // o_done[2q + b] completes with P.V(i) for i % 2 == b.  When S(i) is visible, P.V(i-2) has
        // completed (it was issued before S(i)), so a wait below is never two phases behind.
        uint64_t* od = &o_done[2 * qtl];
        // ---- Q: f16 queries come by TMA from the producer warp; otherwise (f32, or strides a tensor
        // map cannot describe) each thread loads and converts its row (128-byte swizzled, K-major)
        if (!a.q_tma) {
            const uint8_t* qrow = a.q + (size_t)(valid ? t : 0) * a.q_nb_t + (size_t)(kvh * a.G + g) * a.q_nb_h;
            uint8_t* qs = smem + C::OFF_Q + qtl * C::Q_B;
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
            __syncwarp();
            if (lane == 0) mbar_arrive(q_full);
        }
        float m_use = -INFINITY, l = 0.0f;
        bool ok = true;
        const int n_mine = tile_live ? n : 0;
        for (int i = 0; i < n_mine; i++) {
            if (!warp_wait(&sf[i & 1], (i >> 1) & 1, a.err, abort_flag)) { ok = false; break; }
            tc_fence_after();
            const int kb = tile_of(i) * C::BN;           // first key of the tile
            const uint32_t sbuf = lane_addr + (C::S2 ? (i & 1) * C::BN : 0);
            // keys past the row's position (or past kend) are masked; only the last tiles have any
            const bool edge = kb + C::BN - 1 > qpos || kb + C::BN > kend;
            float s[C::BN];
#pragma unroll
            for (int cc = 0; cc < C::BN; cc += 32) tmem_ld32(sbuf + cc, s + cc);
            tmem_wait_ld();
            if (edge) {
#pragma unroll
                for (int k = 0; k < C::BN; k++)
                    if (kb + k > qpos || kb + k >= kend) s[k] = -INFINITY;
            }
            // ---- the row max over the tile's BN columns
            float mr = -INFINITY;
#pragma unroll
            for (int h = 0; h < C::BN; h += 64) {
                float m8[8];
#pragma unroll
                for (int k = 0; k < 8; k++)
                    m8[k] = fmaxf(fmaxf(fmaxf(s[h + k], s[h + k + 8]), fmaxf(s[h + k + 16], s[h + k + 24])),
                                  fmaxf(fmaxf(s[h + k + 32], s[h + k + 40]), fmaxf(s[h + k + 48], s[h + k + 56])));
                mr = fmaxf(mr, fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                                     fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7]))));
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
            const float mneg = m_use == -INFINITY ? 0.0f : -m_use;
            float sum4[4] = {0.f, 0.f, 0.f, 0.f};
            // exponentials of 32 keys (register copy sv of their S columns) -> 16 packed f16 P words
            // (and the P_lo words with PL = 2)
            auto exp32 = [&](const float* sv, uint32_t* pk, uint32_t* pl) {
#pragma unroll
                for (int k = 0; k < 32; k += 4) {
                    const float* x = sv + k;   // masked keys are -inf already
                    // three of every four on the SFU, one on the FMA pipe (kExpFma of four)
                    const float p0 = fast_exp2(fmaf(x[0], c, mneg));
                    const float p1 = kExpFma >= 3 ? exp2_fma(fmaf(x[1], c, mneg)) : fast_exp2(fmaf(x[1], c, mneg));
                    const float p2 = kExpFma >= 2 ? exp2_fma(fmaf(x[2], c, mneg)) : fast_exp2(fmaf(x[2], c, mneg));
                    const float p3 = exp2_fma(fmaf(x[3], c, mneg));
                    const __half2 h01 = __floats2half2_rn(p0, p1), h23 = __floats2half2_rn(p2, p3);
                    sum4[(k >> 2) & 3] += (p0 + p1) + (p2 + p3);
                    pk[k >> 1] = *reinterpret_cast<const uint32_t*>(&h01);
                    pk[(k >> 1) + 1] = *reinterpret_cast<const uint32_t*>(&h23);
                    if constexpr (PL == 2) {
                        // p - f16(p) is exact in f32; its f16 rounding leaves ~2^-22 of p
                        const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
                        pl[k >> 1] = pack_h2(p0 - f01.x, p1 - f01.y);
                        pl[(k >> 1) + 1] = pack_h2(p2 - f23.x, p3 - f23.y);
                    }
                }
            };
            const bool any_resc = __any_sync(0xffffffffu, resc);
            {
                uint32_t pk[C::BN / 2];
                uint32_t pl[PL == 2 ? C::BN / 2 : 1];
#pragma unroll
                for (int cc = 0; cc < C::BN; cc += 32)
                    exp32(s + cc, pk + cc / 2, PL == 2 ? pl + cc / 2 : pl);
                // the exponentials above overlapped P.V(i-1) (64-key tiles; with 128-key tiles it
                // completed before S(i)); O is stable once it has completed
                if (any_resc) {
                    if (!warp_wait(&od[(i - 1) & 1], ((i - 1) >> 1) & 1, a.err, abort_flag)) { ok = false; break; }
                    tc_fence_after();
                    // 64 columns per TMEM round trip (the S registers are free by now)
#pragma unroll 1
                    for (int cc = 0; cc < HD; cc += 64) {
                        float o[64];
                        tmem_ld32(lane_addr + 128 + cc, o);
                        tmem_ld32(lane_addr + 128 + cc + 32, o + 32);
                        tmem_wait_ld();
#pragma unroll
                        for (int k = 0; k < 64; k++) o[k] *= alpha;
                        tmem_st32(lane_addr + 128 + cc, o);
                        tmem_st32(lane_addr + 128 + cc + 32, o + 32);
                    }
                }
                // P over the first BN/2 columns of this tile's S buffer (the S MMA that next writes the
                // buffer, S(i+2) or with one buffer S(i+1), is issued only after P.V(i), and the tensor
                // pipe runs in order)
#pragma unroll
                for (int cc = 0; cc < C::BN / 2; cc += 32) tmem_st32(sbuf + cc, reinterpret_cast<const float*>(pk + cc));
                if constexpr (PL == 2) tmem_st32(sbuf + 32, reinterpret_cast<const float*>(pl));   // P_lo after P_hi
            }
            l = l * alpha + ((sum4[0] + sum4[1]) + (sum4[2] + sum4[3]));
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&pf[i & 1]);
        }
        if (n_mine > 0 && ok && !warp_wait(&od[(n_mine - 1) & 1], ((n_mine - 1) >> 1) & 1, a.err, abort_flag))
            ok = false;
        tc_fence_after();
        const float L = l;
        float* orow = valid ? a.out + (size_t)t * a.out_nb_t + (size_t)(kvh * a.G + g) * a.out_nb_h : nullptr;
        if (ns == 1) {
            // ---- single split: O / L straight out of TMEM
            const float inv = L > 0.0f ? 1.0f / L : 0.0f;
            if (tile_live) {
#pragma unroll 1
                for (int cc = 0; cc < HD; cc += 32) {
                    float o[32];
                    if (n > 0) {
                        tmem_ld32(lane_addr + 128 + cc, o);
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
            }
        } else {
            // ---- split: the splits of a unit (query tiles x kv head) take an arrival ticket; all
            // but the last publish their partial (unnormalised O, m, l) to the workspace and count
            // it, and the last waits for those counts and merges them with its own partial, which
            // stays in TMEM.  Workspace layout [split][col/4][row] float4: a warp's 32 rows are one
            // coalesced 512-byte access per column group.  Counters: tickets[2u] arrivals,
            // tickets[2u + 1] published partials; the merging CTA resets both.
            const int unit = qp * a.NKV + kvh;
            const int row = qtl * 128 + r;
            const bool have = n > 0 && tile_live && ok;
            int* arrive_ctr = &a.tickets[2 * unit];
            int* pub_ctr = &a.tickets[2 * unit + 1];
            softmax_sync<kSoftmaxWarps>();
            if (threadIdx.x == 0) *last_flag = atomicAdd(arrive_ctr, 1) == ns - 1;
            softmax_sync<kSoftmaxWarps>();
            if (!*last_flag) {
                float4* wo = reinterpret_cast<float4*>(a.ws_o) + (size_t)(unit * ns + split) * (HD / 4) * C::ROWS;
                float2* wml = reinterpret_cast<float2*>(a.ws_ml) + (size_t)(unit * ns + split) * C::ROWS;
#pragma unroll 1
                for (int cc = 0; cc < HD; cc += 32) {
                    float o[32];
                    if (have) {
                        tmem_ld32(lane_addr + 128 + cc, o);
                        tmem_wait_ld();
                    } else {
#pragma unroll
                        for (int k = 0; k < 32; k++) o[k] = 0.0f;
                    }
#pragma unroll
                    for (int k = 0; k < 32; k += 4)
                        wo[(size_t)((cc + k) / 4) * C::ROWS + row] = make_float4(o[k], o[k + 1], o[k + 2], o[k + 3]);
                }
                wml[row] = make_float2(have ? m_use : -INFINITY, have ? L : 0.0f);
                __threadfence();
                softmax_sync<kSoftmaxWarps>();
                if (threadIdx.x == 0) atomicAdd(pub_ctr, 1);
            } else {
                // wait (bounded) until the other splits, all running, have published
                if (threadIdx.x == 0) {
                    const uint64_t tw = globaltimer_ns();
                    bool done = false;
                    while (!done) {
                        done = *reinterpret_cast<volatile int*>(pub_ctr) >= ns - 1;
                        if (!done && globaltimer_ns() - tw > kWaitLimitNs) {
                            if (a.err) atomicOr(a.err, ERRBIT_TIMEOUT);
                            break;
                        }
                    }
                    *last_flag = done ? 1 : 2;
                    *arrive_ctr = 0;                         // ready for the next launch
                    *pub_ctr = 0;
                }
                softmax_sync<kSoftmaxWarps>();
                __threadfence();
                // warp-uniform condition: the TMEM loads below are whole-warp instructions; only the
                // output store depends on the row being a real query
                if (*last_flag == 1 && tile_live) {
                    const float2* uml = reinterpret_cast<const float2*>(a.ws_ml) + (size_t)unit * ns * C::ROWS;
                    const float4* uo = reinterpret_cast<const float4*>(a.ws_o) + (size_t)unit * ns * (HD / 4) * C::ROWS;
                    float wsp[8];
                    float2 mls[8];
                    float M = have ? m_use : -INFINITY;
#pragma unroll
                    for (int sp = 0; sp < 8; sp++) {
                        if (sp < ns && sp != split) {
                            mls[sp] = __ldcg(&uml[(size_t)sp * C::ROWS + row]);
                            M = fmaxf(M, mls[sp].x);
                        }
                    }
                    const float w_own = (have && m_use != -INFINITY) ? fast_exp2(m_use - M) : 0.0f;
                    float LL = have ? L * w_own : 0.0f;
#pragma unroll
                    for (int sp = 0; sp < 8; sp++) {
                        if (sp < ns && sp != split) {
                            wsp[sp] = mls[sp].x == -INFINITY ? 0.0f : fast_exp2(mls[sp].x - M);
                            LL += mls[sp].y * wsp[sp];
                        }
                    }
                    const float inv = LL > 0.0f ? 1.0f / LL : 0.0f;
#pragma unroll 1
                    for (int cc = 0; cc < HD; cc += 32) {
                        float o[32];
                        if (have) {
                            tmem_ld32(lane_addr + 128 + cc, o);
                            tmem_wait_ld();
                        } else {
#pragma unroll
                            for (int k = 0; k < 32; k++) o[k] = 0.0f;
                        }
#pragma unroll
                        for (int k = 0; k < 32; k++) o[k] *= w_own;
#pragma unroll
                        for (int sp = 0; sp < 8; sp++) {
                            if (sp < ns && sp != split) {
                                float4 v[8];
#pragma unroll
                                for (int u = 0; u < 8; u++)
                                    v[u] = __ldcg(&uo[((size_t)sp * (HD / 4) + cc / 4 + u) * C::ROWS + row]);
                                const float w = wsp[sp];
#pragma unroll
                                for (int u = 0; u < 8; u++) {
                                    o[4 * u] += v[u].x * w; o[4 * u + 1] += v[u].y * w;
                                    o[4 * u + 2] += v[u].z * w; o[4 * u + 3] += v[u].w * w;
                                }
                            }
                        }
                        if (valid) {
#pragma unroll
                            for (int k = 0; k < 32; k += 4)
                                *reinterpret_cast<float4*>(orow + cc + k) =
                                    make_float4(o[k] * inv, o[k + 1] * inv, o[k + 2] * inv, o[k + 3] * inv);
                        }
                    }
                }
            }
        }
    } else if (warp == kTmaWarp || warp == kTmaWarp + 1) {
        // ============================ TMA producers: lane 0 of the first warp loads the Q tiles, then
        // streams K tiles; lane 0 of the second streams V tiles
        const bool is_v = warp == kTmaWarp + 1;
        if (!is_v && lane == 0 && a.q_tma) {
            // box {64 columns, G heads, QPT queries} = the 128 rows of a Q tile in row order qi*G + g
            mbar_arrive_expect_tx(q_full, (uint32_t)(nqt * C::Q_B));
            for (int q = 0; q < nqt; q++)
#pragma unroll
                for (int b = 0; b < HD / 64; b++)
                    tma_load_3d(smem + C::OFF_Q + q * C::Q_B + b * C::QBOX, &tmq, b * 64, kvh * a.G, t0 + q * QPT, q_full);
        }
        if (lane == 0 && n > 0) {
            // ring entries in the order the MMA warp consumes them: tile i, part p -> entry i*NP + p
            uint64_t* fullx = is_v ? full_v : full_k;
            uint64_t* emptyx = is_v ? empty_v : empty_k;
            const int NE = is_v ? C::NEV : C::NEK;
            uint8_t* ring = smem + (is_v ? C::OFF_V : C::OFF_K);
            const int n_ent = n * NP;
            int issued = 0;
            for (int e = 0; e < n_ent; e++) {
                const int s = e % NE;
                if (e >= NE && !wait_or_abort(&emptyx[s], ((e / NE) - 1) & 1, a.err, abort_flag)) break;
                const int p = NP == 1 ? 0 : e % NP;
                const CUtensorMap* tm = is_v ? (p ? &tmv2 : &tmv) : (p ? &tmk2 : &tmk);
                uint8_t* dst = ring + s * C::KV_B;
                mbar_arrive_expect_tx(&fullx[s], C::KV_B);
                const int y = a.row_base + tile_of(e / NP) * C::BN;
#pragma unroll
                for (int b = 0; b < HD / 64; b++)
#pragma unroll
                    for (int h = 0; h < C::BN / 64; h++)   // the tensor map's box is 64 rows
                        tma_load_2d(dst + b * C::KBOX + h * 64 * C::BOX_ROW, tm, kvh * HD + b * 64, y + h * 64,
                                    &fullx[s]);
                issued = e + 1;
            }
            for (int e = max(0, issued - NE); e < issued; e++)
                mbar_wait(&fullx[e % NE], (e / NE) & 1, a.err);
        }
        // never leave the Q copy in flight either (a CTA without keys does not wait for it otherwise)
        if (!is_v && lane == 0 && a.q_tma) mbar_wait(q_full, 0, a.err);
    } else {
        // ============================ MMA issuer
        if (lane == 0 && n > 0) {
            const uint32_t idesc_s = umma_idesc(128, C::BN, 0, 0);
            const uint32_t idesc_o = umma_idesc(128, HD, 0, 1);
            // descriptor words: K-major Q and K (LBO 16, SBO 1024) and MN-major V (LBO = one 64-column
            // box, SBO 1024), all 128-byte swizzled, so one hi word serves every operand
            constexpr uint32_t hi = desc_hi_sw128(1024);
            const uint32_t q_lo = desc_lo(smem_u32(smem + C::OFF_Q), 16);
            const uint32_t k_lo = desc_lo(smem_u32(smem + C::OFF_K), 16);
            const uint32_t v_lo = desc_lo(smem_u32(smem + C::OFF_V), C::KBOX);
            // S(i) = Q K(i)^T into Q tile q's S buffer (buffer i & 1 when double-buffered), summed over the
            // NP parts of K(i); the K entries of tile i must have landed (wait_k)
            auto wait_k = [&](int i) -> bool {
                for (int p = 0; p < NP; p++) {
                    const int e = i * NP + p;
                    if (!wait_or_abort(&full_k[e % C::NEK], (e / C::NEK) & 1, a.err, abort_flag)) return false;
                }
                tc_fence_after();
                return true;
            };
            auto mma_s = [&](int i, int q) {
                uint32_t kd[NP];
#pragma unroll
                for (int p = 0; p < NP; p++) kd[p] = k_lo + (uint32_t)(((i * NP + p) % C::NEK) * (C::KV_B >> 4));
                const uint32_t d_tmem = tmem + q * C::QCOLS + (C::S2 ? (i & 1) * C::BN : 0);
#pragma unroll
                for (int p = 0; p < NP; p++) {
#pragma unroll
                    for (int kk = 0; kk < HD / 16; kk++) {
                        const uint32_t a_off = (uint32_t)((q * C::Q_B + (kk / 4) * C::QBOX + (kk % 4) * 32) >> 4);
                        const uint32_t b_off = (uint32_t)(((kk / 4) * C::KBOX + (kk % 4) * 32) >> 4);
                        umma_f16_w(d_tmem, q_lo + a_off, kd[p] + b_off, hi, idesc_s, (kk > 0 || p > 0) ? 1u : 0u);
                    }
                }
                umma_commit(&s_full[2 * q + (i & 1)]);
            };
            // the K entries of tile i are free once every S(i) has completed
            auto release_k = [&](int i) {
                for (int p = 0; p < NP; p++) umma_commit(&empty_k[(i * NP + p) % C::NEK]);
            };
            // O += P(i) V(i) for Q tile q, once its softmax warps have written P(i)
            auto mma_pv = [&](int i, int q) -> bool {
                if (!wait_or_abort(&p_full[2 * q + (i & 1)], (i >> 1) & 1, a.err, abort_flag)) return false;
                tc_fence_after();
                uint32_t vd[NP];
#pragma unroll
                for (int p = 0; p < NP; p++) vd[p] = v_lo + (uint32_t)(((i * NP + p) % C::NEV) * (C::KV_B >> 4));
                // f16 P: 8 columns per 16 keys; P_lo (PL = 2) in the next 32 columns
                const uint32_t p_tmem = tmem + q * C::QCOLS + (C::S2 ? (i & 1) * C::BN : 0);
                const uint32_t o_tmem = tmem + q * C::QCOLS + 128;
#pragma unroll
                for (int p = 0; p < NP; p++) {
#pragma unroll
                    for (int pp = 0; pp < (p == 0 ? PL : 1); pp++) {   // P_lo meets V's first part only
#pragma unroll
                        for (int kk = 0; kk < C::BN / 16; kk++)
                            umma_f16_ts_w(o_tmem, p_tmem + pp * 32 + kk * 8, vd[p] + (uint32_t)(kk * 16 * 128 >> 4), hi,
                                          idesc_o, (i > 0 || p > 0 || pp > 0 || kk > 0) ? 1u : 0u);
                    }
                }
                umma_commit(&o_done[2 * q + (i & 1)]);
                return true;
            };
            auto wait_v = [&](int i) -> bool {
                for (int p = 0; p < NP; p++) {
                    const int e = i * NP + p;
                    if (!wait_or_abort(&full_v[e % C::NEV], (e / C::NEV) & 1, a.err, abort_flag)) return false;
                }
                return true;
            };
            auto release_v = [&](int i) {
                for (int p = 0; p < NP; p++) umma_commit(&empty_v[(i * NP + p) % C::NEV]);
            };
            bool ok = wait_or_abort(q_full, 0, a.err, abort_flag) && wait_k(0);
            if (ok) {
                for (int q = 0; q < nqt; q++) mma_s(0, q);
                release_k(0);
            }
            if constexpr (C::S2) {
                for (int i = 0; ok && i < n; i++) {
                    // S(i+1) overlaps the softmax of tile i (its buffer held S(i-1), whose P.V was issued)
                    if (i + 1 < n) {
                        if (!wait_k(i + 1)) break;
                        for (int q = 0; q < nqt; q++) mma_s(i + 1, q);
                        release_k(i + 1);
                    }
                    ok = wait_v(i);
                    for (int q = 0; q < nqt && ok; q++) ok = mma_pv(i, q);
                    if (!ok) break;
                    release_v(i);
                }
            } else {
                // one S buffer per Q tile: S_q(i+1) follows P.V_q(i) (it overwrites P_q(i)), and the Q
                // tiles alternate, so the tensor core runs P.V_1(i), S_1(i+1) while the softmax warps of
                // Q tile 0 work on S_0(i+1), and the other way round
                for (int i = 0; ok && i < n; i++) {
                    ok = wait_v(i);
                    for (int q = 0; q < nqt && ok; q++) {
                        ok = mma_pv(i, q);
                        if (ok && i + 1 < n) {
                            if (q == 0) ok = wait_k(i + 1);
                            if (ok) mma_s(i + 1, q);
                        }
                    }
                    if (!ok) break;
                    release_v(i);
                    if (i + 1 < n) release_k(i + 1);
                }
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

// kernel attributes, once per device
template <int HD, int NQT, int NP, int PL, int BN>
cudaError_t prepare_t() {
    static std::once_flag once[kMaxDevices];
    static cudaError_t status[kMaxDevices];
    return once_per_device(once, status, [] {
        using C = PreCfg<HD, NQT, NP, BN>;
        cudaError_t e = cudaFuncSetAttribute(fa_prefill_kernel<HD, NQT, NP, PL, BN>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM + 1024);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(fa_prefill_kernel<HD, NQT, NP, PL, BN>,
                                     cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        return e;
    });
}

// Splits of the key range per CTA (one CTA per SM, no clusters): minimise (waves) x (per-CTA
// tiles + a merge cost of ~merge_tiles tiles when split; ~6 tiles of 64 keys), at most 8 splits and
// at least 2 tiles each, within the workspace (partials) and ticket capacity.
int pick_splits(int units, int tiles, size_t per_split_floats, size_t ws_floats, int n_tickets, double merge_tiles) {
    int best = 1;
    double best_t = 1e30;
    for (int s = 1; s <= 8; s++) {
        if (s > 1 && (tiles / s < 2 || (size_t)units * s * per_split_floats > ws_floats || 2 * units > n_tickets)) break;
        const double waves = std::ceil((double)units * s / kNumSMs);
        const double t = waves * ((double)tiles / s + (s > 1 ? merge_tiles : 0.0));
        if (t < best_t - 1e-9) {
            best_t = t;
            best = s;
        }
    }
    return best;
}

template <int HD, int NQT, int NP, int PL = NP, int BN = 64>
cudaError_t launch_t(const AttnArgs& a_in, const CUtensorMap* tk, const CUtensorMap* tv, const CUtensorMap* tk2,
                     const CUtensorMap* tv2, float* ws, size_t ws_floats, int* tickets, int n_tickets, cudaStream_t st) {
    using C = PreCfg<HD, NQT, NP, BN>;
    cudaError_t e = prepare_t<HD, NQT, NP, PL, BN>();
    if (e != cudaSuccess) return e;
    AttnArgs a = a_in;
    const int QPT = 128 / a.G;
    const int n_cta_q = ceil_div(a.T, NQT * QPT);
    const int units = n_cta_q * a.NKV;
    // key tiles of a typical CTA (host value of the causal base; a device-side base uses max keys)
    const int keys = a.causal_base_dev ? a.S : std::min(a.S, a.causal_base + std::min(NQT * QPT, a.T));
    const size_t per_split = (size_t)C::ROWS * (HD + 2);
    a.n_splits = (ws && tickets) ? pick_splits(units, (keys + C::BN - 1) / C::BN, per_split, ws_floats, n_tickets,
                                               6.0 * 64 / C::BN)
                                 : 1;
    a.cluster_merge = 0;
    if (a.n_splits > 1) {
        a.ws_o = ws;
        a.ws_ml = ws + (size_t)units * a.n_splits * C::ROWS * HD;
        a.tickets = tickets;
    }
    // f16 queries: a 3D map over [T][NH][HD] whose {64, G, QPT} box is one 64-column slab of a Q tile
    CUtensorMap tq;
    memset(&tq, 0, sizeof(tq));
    a.q_tma = 0;
    if (a.q_type == SV_TYPE_F16) {
        const uint64_t dims[3] = {(uint64_t)HD, (uint64_t)a.NH, (uint64_t)a.T};
        const uint64_t strides[2] = {(uint64_t)a.q_nb_h, (uint64_t)a.q_nb_t};
        const uint32_t box[3] = {64u, (uint32_t)a.G, (uint32_t)QPT};
        a.q_tma = encode_tmap_3d(&tq, a.q, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, dims, strides, box,
                                 CU_TENSOR_MAP_SWIZZLE_128B) ? 1 : 0;
    }
    dim3 grid((unsigned)a.n_splits, (unsigned)n_cta_q, (unsigned)a.NKV);
    return launch_pdl(fa_prefill_kernel<HD, NQT, NP, PL, BN>, grid, dim3(C::THREADS), (size_t)(C::SMEM + 1024), st, *tk, *tv,
                      NP == 2 ? *tk2 : *tk, NP == 2 ? *tv2 : *tv, tq, a);
}

// q8_0 rows -> f16 (hi, lo) parts for the tensor-core prefill.  With q an 8-bit integer and d the
// block's f16 scale, hi = f16(q * d) and lo = f16(q * d - hi) (q * d - hi has at most 8 significant
// bits), so hi + lo = q * d, the value the oracle's dequantisation gives, up to f16 subnormal
// rounding of lo (< 2^-25).  Computed in f16 arithmetic, off the conversion pipe: q becomes an exact
// f16 integer by byte permutes (0x64uu = 1024 + u, u = q + 128, minus 1152), hi = HMUL2(q, d) is
// the single round-to-nearest of the exact product, and lo = HFMA2(q, d, -hi) rounds q * d - hi once.
// One thread per 8 elements of one row of K or V; planes[0..3] = K hi, K lo, V hi, V lo, each
// [row][ne0] f16.
__global__ void __launch_bounds__(256) q8_0_split_kernel(const uint8_t* __restrict__ kc, const uint8_t* __restrict__ vc,
                                                         size_t row_bytes, int ne0, int n_rows, uint16_t* planes,
                                                         size_t plane_elems) {
    pdl_wait();   // an earlier launch may still read the planes or write the rows
    if (threadIdx.x == 0) pdl_trigger();
    const int per_row = ne0 / 8;
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (int64_t)n_rows * per_row) return;
    const int row = (int)(idx / per_row), e = (int)(idx % per_row) * 8;
    const int is_v = blockIdx.y;
    const uint8_t* blk = (is_v ? vc : kc) + (size_t)row * row_bytes + (size_t)(e / kQK8_0) * kQ8_0Bytes;
    const __half2 d2 = __half2half2(__ushort_as_half(__ldg(reinterpret_cast<const uint16_t*>(blk))));
    const uint16_t* qs = reinterpret_cast<const uint16_t*>(blk + 2 + (e % kQK8_0));   // 2-byte aligned
    const __half2 k1152 = __half2half2(__ushort_as_half(0x6480u));
    uint32_t hi[4], lo[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const uint32_t u = (uint32_t)__ldg(qs + i) ^ 0x8080u;
        const uint32_t hq = __byte_perm(u, 0x64646464u, 0x4140);   // {1024 + u0, 1024 + u1}
        const __half2 q = __hsub2(*reinterpret_cast<const __half2*>(&hq), k1152);
        const __half2 h = __hmul2(q, d2);
        const __half2 l = __hfma2(q, d2, __hneg2(h));
        hi[i] = *reinterpret_cast<const uint32_t*>(&h);
        lo[i] = *reinterpret_cast<const uint32_t*>(&l);
    }
    uint16_t* dst = planes + (size_t)(2 * is_v) * plane_elems + (size_t)row * ne0 + e;
    *reinterpret_cast<uint4*>(dst) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<uint4*>(dst + plane_elems) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
}

}  // namespace

bool prefill_supported(int head_dim, int kv_type, int G, size_t row_bytes) {
    if (!(G >= 1 && G <= 16 && (128 % G) == 0 && (head_dim == 128 || head_dim == 256))) return false;
    if (kv_type == SV_TYPE_F16) return row_bytes % 16 == 0;
    // q8_0 through the f16 (hi, lo) planes (rows of 16-byte multiples), at the head size the q8_0
    // decode kernel serves
    return kv_type == SV_TYPE_Q8_0 && head_dim == 256;
}

bool make_prefill_tmap(CUtensorMap* m, const void* base, int head_dim, int n_kv_head, size_t row_bytes,
                       int64_t n_rows) {
    return encode_tmap_2d(m, base, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, (uint64_t)n_kv_head * head_dim, (uint64_t)n_rows,
                          row_bytes, 64, PreCfg<128, 1>::BN, CU_TENSOR_MAP_SWIZZLE_128B);
}

cudaError_t launch_prefill(const AttnArgs& a, int head_dim, const CUtensorMap* tk, const CUtensorMap* tv, float* ws,
                           size_t ws_floats, int* tickets, int n_tickets, cudaStream_t st, const CUtensorMap* tk_lo,
                           const CUtensorMap* tv_lo) {
    // q8_0 (hi, lo parts of K and V): P as hi + lo too; f16 caches: P rounded to f16
    const bool parts = tk_lo && tv_lo;
    // two query tiles per CTA when the chunk has them (each K/V tile then feeds 256 query rows)
    if (head_dim == 128) {
        // two query tiles of an f16 cache: 128-key tiles, the Q tiles alternating on the tensor core
        if (a.T * a.G > 128)
            return parts ? launch_t<128, 2, 2>(a, tk, tv, tk_lo, tv_lo, ws, ws_floats, tickets, n_tickets, st)
                         : launch_t<128, 2, 1, kF16PParts, 128>(a, tk, tv, tk_lo, tv_lo, ws, ws_floats, tickets,
                                                                 n_tickets, st);
        return parts ? launch_t<128, 1, 2>(a, tk, tv, tk_lo, tv_lo, ws, ws_floats, tickets, n_tickets, st)
                     : launch_t<128, 1, 1, kF16PParts>(a, tk, tv, tk_lo, tv_lo, ws, ws_floats, tickets, n_tickets, st);
    }
    if (head_dim == 256)
        return parts ? launch_t<256, 1, 2>(a, tk, tv, tk_lo, tv_lo, ws, ws_floats, tickets, n_tickets, st)
                     : launch_t<256, 1, 1, kF16PParts>(a, tk, tv, tk_lo, tv_lo, ws, ws_floats, tickets, n_tickets, st);
    return cudaErrorInvalidValue;
}

cudaError_t launch_q8_0_split(const uint8_t* kc, const uint8_t* vc, size_t row_bytes, int ne0, int n_rows,
                              uint16_t* planes, size_t plane_elems, cudaStream_t st) {
    if (n_rows <= 0) return cudaSuccess;
    const int64_t threads = (int64_t)n_rows * (ne0 / 8);
    dim3 grid((unsigned)((threads + 255) / 256), 2);
    return launch_pdl(q8_0_split_kernel, grid, dim3(256), 0, st, kc, vc, row_bytes, ne0, n_rows, planes, plane_elems);
}

}  // namespace svkv
