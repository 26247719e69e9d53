// attn_decode.cu - split-K flash-decode over the KV cache (sm_100a).
//
// Replaces ggml_flash_attn_ext for single-token decode and short query chunks
// (llm_block.hpp:268-277, qwen3vl_model.cpp:657-663), with the reference's
// masks (set_causal_mask / set_window_mask, attention.hpp:60-83) evaluated as
// in-kernel predicates instead of a host-built f16 matrix.
//
// Grid: (key splits, kv heads, query tiles).  A query tile packs up to 16 rows
// = (queries x the GQA group's query heads), so every K/V tile a CTA loads is
// shared by all query heads of its kv head.  Block: 4 consumer warps + 1 TMA
// producer warp.  The producer streams BK-key K and V tiles of one kv head
// into a STAGES-deep shared-memory ring with cp.async.bulk.tensor (128-byte
// swizzle, no multicast) and mbarrier transaction counts; each consumer warp
// owns 16 keys of every tile:
//   S = Q K^T      mma.m16n8k16 (f16 in, f32 acc), K fragments by ldmatrix
//   online softmax  row max / sum by quad shuffles, exp2 with scale*log2(e)
//   O += P V       P re-packed from the S accumulators, V by ldmatrix.trans
// The four warps' (m, l, O) merge through shared memory; with more than one
// split the CTA writes its partial and the last CTA of the (tile, kv head)
// (atomic ticket, no spinning) merges all partials and resets the ticket.
//
// q8_0 caches (config 4): each warp expands its 16 keys to exact f16
// integers plus an f32 scale table.  S sums each 32-wide block in a fresh
// accumulator and adds it scaled by the block's d; for O the block scale is
// folded into P (P*d split into f16 hi + lo parts, two MMAs), so K and V are
// used exactly as the oracle dequantises them.
//
// Roofline: HBM-bound.  Algorithmic bytes per (key, kv head) = 2 * HD * 2
// (f16 K + V) or 2 * HD/32 * 34 (q8_0), plus Q and O once per tile.
#include <algorithm>

#include "common.cuh"
#include "internal.hpp"

namespace svkv {

namespace {

constexpr int kBK = 64;            // keys per pipeline stage
constexpr int kConsumerWarps = 4;  // 16 keys each
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr float kLog2e = 1.4426950408889634f;

constexpr int align_up(int x, int a) { return (x + a - 1) / a * a; }

template <int HD, int KVT>
struct DecCfg {
    static constexpr bool Q8 = KVT == SV_TYPE_Q8_0;
    static constexpr int COLS = HD >= 64 ? 64 : HD;      // f16 columns per TMA box / staging box
    static constexpr int NB = HD / COLS;
    static constexpr int PITCH = COLS * 2;               // bytes per box row (= swizzle span)
    static constexpr int BOXB = kBK * PITCH;
    static constexpr int HEADB = Q8 ? HD / kQK8_0 * kQ8_0Bytes : HD * 2;
    static constexpr int TILE_B = Q8 ? kBK * HEADB : NB * BOXB;   // K (or V) bytes per stage
    static constexpr int STAGES = 3;                              // HD <= 128: two CTAs fit per SM
    static constexpr int MIN_BLOCKS = HD >= 256 ? 1 : 2;
    static constexpr int STAGE_B = align_up(2 * TILE_B, 1024);
    static constexpr int WBOXB = 16 * PITCH;                      // q8 staging box (16 keys)
    static constexpr int WSTAGE_B = Q8 ? 2 * NB * WBOXB : 0;      // per warp: K and V f16 tiles
    static constexpr int NBLK = HD / kQK8_0;
    static constexpr int WD_B = Q8 ? 2 * 16 * NBLK * 4 : 0;       // per warp: dK, dV tables
    static constexpr int RING_B = STAGES * STAGE_B;
    static constexpr int COMB_B = kConsumerWarps * 16 * HD * 4 + (kConsumerWarps * 16 * 2 + 16 * kConsumerWarps + 32) * 4;
    static constexpr int PO_OFF = align_up(COMB_B, 16);             // cluster merge: this CTA's partial O
    static constexpr int PM_OFF = PO_OFF + 16 * HD * 4;              //                and its (m, l) per row
    static_assert(PM_OFF + 16 * 2 * 4 <= RING_B, "cluster-merge partials must fit in the stage ring");
    static constexpr int BAR_OFF = RING_B + kConsumerWarps * (WSTAGE_B + WD_B);
    static constexpr int SMEM = BAR_OFF + 2 * STAGES * 8 + 16;
    static_assert(COMB_B <= RING_B, "combine scratch must fit in the stage ring");
};

__device__ __forceinline__ void consumer_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
}

// two signed bytes (low, high of w) -> exact f16x2
__device__ __forceinline__ uint32_t i8x2_to_h2(uint32_t w) {
    const uint32_t lo = (w & 0xffu) ^ 0x80u;
    const uint32_t hi = ((w >> 8) & 0xffu) ^ 0x80u;
    const uint32_t h = (0x6400u | lo) | ((0x6400u | hi) << 16);      // 1024 + (b + 128)
    __half2 r = __hsub2(*reinterpret_cast<const __half2*>(&h), __half2half2(__ushort_as_half(0x6480u)));  // -1152
    return *reinterpret_cast<uint32_t*>(&r);
}

template <int HD, int KVT>
__global__ void __launch_bounds__(kThreads, DecCfg<HD, KVT>::MIN_BLOCKS)
fa_decode_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                 const __grid_constant__ AttnArgs a) {
    using C = DecCfg<HD, KVT>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
    uint64_t* empty = full + C::STAGES;
    volatile int* flag = reinterpret_cast<volatile int*>(empty + C::STAGES);   // [0] abort, [1] last

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int split = blockIdx.x, kvh = blockIdx.y, qt = blockIdx.z;
    const int t0 = qt * a.qpt;
    const int nq = min(a.qpt, a.T - t0);
    const int R = nq * a.G;

    // prologue that touches no global memory overlaps the previous kernel (PDL)
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        flag[0] = 0;
        flag[1] = 0;
        fence_barrier_init();
    }
    if (threadIdx.x == kConsumerWarps * 32) {
        tma_prefetch_desc(&tmk);
        tma_prefetch_desc(&tmv);
    }
    __syncthreads();

    // one stage of K and V tiles for keys [y, y + kBK) of this kv head
    auto issue = [&](int j, int y) {
        const int s = j % C::STAGES;
        uint8_t* kst = smem + s * C::STAGE_B;
        uint8_t* vst = kst + C::TILE_B;
        mbar_arrive_expect_tx(&full[s], 2 * C::TILE_B);
        if constexpr (C::Q8) {
            tma_load_2d(kst, &tmk, kvh * (C::HEADB / 2), y, &full[s]);
            tma_load_2d(vst, &tmv, kvh * (C::HEADB / 2), y, &full[s]);
        } else {
#pragma unroll
            for (int b = 0; b < C::NB; b++) {
                tma_load_2d(kst + b * C::BOXB, &tmk, kvh * HD + b * C::COLS, y, &full[s]);
                tma_load_2d(vst + b * C::BOXB, &tmv, kvh * HD + b * C::COLS, y, &full[s]);
            }
        }
    };
    // A kernel that appends its own new rows (fused decode step) starts streaming its split's
    // first tiles before waiting for the previous kernel: the rows it reads were completed by
    // earlier steps (the host clears ring_prefill when the launch before this one wrote cache rows
    // while letting it start early), and the rows it appends are patched in from their source
    // below.  The split's start does not depend on n_past in causal mode, only its end does.
    int prefetched = 0;
    if (a.n_new > 0 && a.ring_prefill && a.mask_mode == SV_MASK_CAUSAL && threadIdx.x == kConsumerWarps * 32) {
        const int ks0 = split * a.chunk;
        const int kmax = min(a.S, ks0 + a.chunk);
        const int nt_max = kmax > ks0 ? (kmax - ks0 + kBK - 1) / kBK : 0;
        prefetched = min(nt_max, C::STAGES);
        for (int j = 0; j < prefetched; j++) issue(j, a.row_base + ks0 + j * kBK);
    }
    pdl_wait();
    if (threadIdx.x == 0) pdl_trigger();

    // ---- key range of this tile and split
    int klo = 0, khi = a.S;
    int wlo = 0, whi = 0, wown = -1;
    const int cbase = a.causal_base_dev ? __ldg(a.causal_base_dev) : a.causal_base;
    if (a.mask_mode == SV_MASK_CAUSAL) {
        khi = min(a.S, cbase + t0 + nq);
    } else if (a.mask_mode == SV_MASK_WINDOW) {
        wlo = a.lo[t0];
        whi = a.hi[t0];
        wown = a.own[t0];
        klo = whi > wlo ? wlo : wown;
        khi = whi > wlo ? whi : wown + 1;
        if (wown >= 0) {
            klo = min(klo, wown);
            khi = max(khi, wown + 1);
        }
        klo = max(klo, 0);
        khi = min(khi, a.S);
    }
    const int ks = klo + split * a.chunk;
    const int ke = min(khi, ks + a.chunk);
    const int n_tiles = ke > ks ? (ke - ks + kBK - 1) / kBK : 0;
    if (a.n_new > 0 && cbase + a.n_new > a.S && threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0 &&
        blockIdx.z == 0 && a.err)
        atomicOr(a.err, ERRBIT_ROW_RANGE);   // appended rows past the grid's key bound are not written

    if (warp == kConsumerWarps) {
        // ============================ TMA producer
        if (lane == 0 && (n_tiles > 0 || prefetched > 0)) {
            int issued = prefetched;
            for (int j = prefetched; j < n_tiles; j++) {
                const int s = j % C::STAGES;
                if (j >= C::STAGES && !mbar_wait(&empty[s], ((j / C::STAGES) - 1) & 1, a.err)) {
                    flag[0] = 1;
                    break;
                }
                if (flag[0]) break;
                issue(j, a.row_base + ks + j * kBK);
                issued = j + 1;
            }
            // never leave a bulk copy in flight into shared memory: wait (bounded) for the
            // last phase of every stage this thread filled
            for (int j = max(0, issued - C::STAGES); j < issued; j++)
                mbar_wait(&full[j % C::STAGES], (j / C::STAGES) & 1, a.err);
        }
        if (a.cluster_merge) {      // the producer warp takes part in the two cluster barriers of the merge
            __syncwarp();
            cluster_sync_all();
            cluster_sync_all();
        }
        return;
    }

    // ============================ consumers
    const int tid = threadIdx.x;   // 0..127
    const int q4 = lane & 3;
    int rrow[2] = {lane >> 2, (lane >> 2) + 8};
    bool rvalid[2];
    int rlim[2];
    const uint16_t* rmask[2];
    const uint8_t* qrow[2];
    const int q_es = a.q_type == SV_TYPE_F32 ? 4 : 2;
#pragma unroll
    for (int i = 0; i < 2; i++) {
        const int r = rrow[i];
        rvalid[i] = r < R;
        const int qi = r / a.G, g = r % a.G;
        const int t = t0 + qi;
        rlim[i] = cbase + t;
        rmask[i] = (a.mask_mode == SV_MASK_EXPLICIT && rvalid[i]) ? a.mask + (size_t)t * a.mask_nb_t : nullptr;
        qrow[i] = rvalid[i] ? a.q + (size_t)t * a.q_nb_t + (size_t)(kvh * a.G + g) * a.q_nb_h : nullptr;
    }

    // Q as A fragments (row-major 16 x HD)
    uint32_t qa[HD / 16][4];
#pragma unroll
    for (int kk = 0; kk < HD / 16; kk++) {
#pragma unroll
        for (int reg = 0; reg < 4; reg++) {
            const int i = reg & 1;
            const int e = kk * 16 + (reg >> 1) * 8 + 2 * q4;
            uint32_t v = 0;
            if (rvalid[i]) {
                if (a.q_type == SV_TYPE_F32) {
                    const float2 f = *reinterpret_cast<const float2*>(qrow[i] + (size_t)e * q_es);
                    v = pack_h2(f.x, f.y);
                } else {
                    v = *reinterpret_cast<const uint32_t*>(qrow[i] + (size_t)e * q_es);
                }
            }
            qa[kk][reg] = v;
        }
    }

    float o[HD / 8][4];
#pragma unroll
    for (int n = 0; n < HD / 8; n++) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
    float m[2] = {-INFINITY, -INFINITY};
    float l[2] = {0.0f, 0.0f};

    uint8_t* wst = smem + C::RING_B + warp * (C::WSTAGE_B + C::WD_B);   // q8 staging (this warp)
    float* dk_tab = reinterpret_cast<float*>(wst + C::WSTAGE_B);
    float* dv_tab = dk_tab + 16 * C::NBLK;

    for (int j = 0; j < n_tiles; j++) {
        const int s = j % C::STAGES;
        if (!mbar_wait(&full[s], (j / C::STAGES) & 1, a.err)) {
            flag[0] = 1;
            break;
        }
        const int kw = ks + j * kBK + 16 * warp;   // first key of this warp
        if (kw < ke) {
            const uint8_t* kst = smem + s * C::STAGE_B;
            const uint8_t* vst = kst + C::TILE_B;
            if constexpr (!C::Q8) {
                // fused append (f16 cache): a key this launch appends is written to the cache from its
                // source row and patched into the tile the TMA brought in (which may hold the old row)
                if (a.n_new > 0 && kw < cbase + a.n_new && kw + 16 > cbase) {
                    constexpr int LANES = HD * 2 / 16;             // 16-byte pieces of one head's row
                    const int k_lo = max(kw, cbase), k_hi = min(kw + 16, cbase + a.n_new);
                    for (int key = k_lo; key < k_hi; key++) {
                        if (lane < LANES) {
                            const size_t so = (size_t)(key - cbase) * a.new_nb_t + (size_t)kvh * HD * 2 + lane * 16;
                            const uint4 kvec = *reinterpret_cast<const uint4*>(a.knew + so);
                            const uint4 vvec = *reinterpret_cast<const uint4*>(a.vnew + so);
                            const size_t co = (size_t)key * a.cache_row_bytes + (size_t)kvh * HD * 2 + lane * 16;
                            *reinterpret_cast<uint4*>(a.kc_w + co) = kvec;
                            *reinterpret_cast<uint4*>(a.vc_w + co) = vvec;
                            const int row = key - (ks + j * kBK);
                            const int e = lane * 8;
                            const uint32_t off = (e / C::COLS) * C::BOXB + swz_off(row, e % C::COLS, C::PITCH);
                            *reinterpret_cast<uint4*>(const_cast<uint8_t*>(kst) + off) = kvec;
                            *reinterpret_cast<uint4*>(const_cast<uint8_t*>(vst) + off) = vvec;
                        }
                    }
                    fence_proxy_async_smem();   // order these writes before the stage's next TMA fill
                    __syncwarp();
                }
            }
            float sacc[2][4];
#pragma unroll
            for (int nt = 0; nt < 2; nt++) sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.0f;

            if constexpr (!C::Q8) {
                const int krow = 16 * warp + (lane & 7) + 8 * (lane >> 4);
                const uint32_t kbase = smem_u32(kst);
#pragma unroll
                for (int kk = 0; kk < HD / 16; kk++) {
                    const int e = kk * 16 + 8 * ((lane >> 3) & 1);
                    const uint32_t addr = kbase + (e / C::COLS) * C::BOXB + swz_off(krow, e % C::COLS, C::PITCH);
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4(addr, b0, b1, b2, b3);
                    mma_f16(sacc[0], qa[kk], b0, b1);
                    mma_f16(sacc[1], qa[kk], b2, b3);
                }
            } else {
                // expand this warp's 16 keys of K and V into exact f16 integers + scales
                const int kr0 = 16 * warp;
#pragma unroll 1
                for (int task = lane; task < 2 * 16 * C::NBLK; task += 32) {
                    const int isv = task / (16 * C::NBLK);
                    const int rem = task % (16 * C::NBLK);
                    const int kr = rem / C::NBLK, b = rem % C::NBLK;
                    const uint8_t* src = (isv ? vst : kst) + (kr0 + kr) * C::HEADB + b * kQ8_0Bytes;
                    const uint16_t* s16 = reinterpret_cast<const uint16_t*>(src);
                    (isv ? dv_tab : dk_tab)[kr * C::NBLK + b] = h2f(s16[0]);
                    uint8_t* dstb = wst + isv * C::NB * C::WBOXB;
#pragma unroll
                    for (int g = 0; g < 4; g++) {
                        uint4 v;
                        v.x = i8x2_to_h2(s16[1 + g * 4 + 0]);
                        v.y = i8x2_to_h2(s16[1 + g * 4 + 1]);
                        v.z = i8x2_to_h2(s16[1 + g * 4 + 2]);
                        v.w = i8x2_to_h2(s16[1 + g * 4 + 3]);
                        const int e = b * kQK8_0 + g * 8;
                        *reinterpret_cast<uint4*>(dstb + (e / C::COLS) * C::WBOXB + swz_off(kr, e % C::COLS, C::PITCH)) = v;
                    }
                }
                __syncwarp();
                const int krow = (lane & 7) + 8 * (lane >> 4);
                const uint32_t kbase = smem_u32(wst);
#pragma unroll
                for (int blk = 0; blk < C::NBLK; blk++) {
                    float sb[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
                    for (int kk = 2 * blk; kk < 2 * blk + 2; kk++) {
                        const int e = kk * 16 + 8 * ((lane >> 3) & 1);
                        const uint32_t addr = kbase + (e / C::COLS) * C::WBOXB + swz_off(krow, e % C::COLS, C::PITCH);
                        uint32_t b0, b1, b2, b3;
                        ldsm_x4(addr, b0, b1, b2, b3);
                        mma_f16(sb[0], qa[kk], b0, b1);
                        mma_f16(sb[1], qa[kk], b2, b3);
                    }
#pragma unroll
                    for (int nt = 0; nt < 2; nt++) {
                        const float d0 = dk_tab[(nt * 8 + 2 * q4) * C::NBLK + blk];
                        const float d1 = dk_tab[(nt * 8 + 2 * q4 + 1) * C::NBLK + blk];
                        sacc[nt][0] = fmaf(d0, sb[nt][0], sacc[nt][0]);
                        sacc[nt][1] = fmaf(d1, sb[nt][1], sacc[nt][1]);
                        sacc[nt][2] = fmaf(d0, sb[nt][2], sacc[nt][2]);
                        sacc[nt][3] = fmaf(d1, sb[nt][3], sacc[nt][3]);
                    }
                }
            }

            // ---- scale + mask (log2 domain)
#pragma unroll
            for (int nt = 0; nt < 2; nt++) {
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const int ri = i >> 1;
                    const int key = kw + nt * 8 + 2 * q4 + (i & 1);
                    float v = sacc[nt][i] * a.scale_log2;
                    bool vis = rvalid[ri] && key < ke;
                    if (a.mask_mode == SV_MASK_CAUSAL) {
                        vis = vis && key <= rlim[ri];
                    } else if (a.mask_mode == SV_MASK_WINDOW) {
                        vis = vis && ((key >= wlo && key < whi) || key == wown);
                    } else if (a.mask_mode == SV_MASK_EXPLICIT) {
                        if (vis) {
                            const float mv = h2f(rmask[ri][key]);
                            vis = mv != -INFINITY;
                            v = fmaf(mv, kLog2e, v);
                        }
                    }
                    sacc[nt][i] = vis ? v : -INFINITY;
                }
            }
            // ---- online softmax (rows r0: elements 0,1; r1: elements 2,3)
            float mx[2];
            mx[0] = fmaxf(fmaxf(sacc[0][0], sacc[0][1]), fmaxf(sacc[1][0], sacc[1][1]));
            mx[1] = fmaxf(fmaxf(sacc[0][2], sacc[0][3]), fmaxf(sacc[1][2], sacc[1][3]));
            float alpha[2], mu[2];
#pragma unroll
            for (int i = 0; i < 2; i++) {
                mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 1));
                mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 2));
                const float mn = fmaxf(m[i], mx[i]);
                alpha[i] = m[i] == -INFINITY ? 0.0f : fast_exp2(m[i] - mn);
                m[i] = mn;
                mu[i] = mn == -INFINITY ? 0.0f : mn;
            }
            float p[2][4];
#pragma unroll
            for (int nt = 0; nt < 2; nt++)
#pragma unroll
                for (int i = 0; i < 4; i++) p[nt][i] = fast_exp2(sacc[nt][i] - mu[i >> 1]);
            l[0] = l[0] * alpha[0] + (p[0][0] + p[0][1] + p[1][0] + p[1][1]);
            l[1] = l[1] * alpha[1] + (p[0][2] + p[0][3] + p[1][2] + p[1][3]);
#pragma unroll
            for (int n = 0; n < HD / 8; n++) {
                o[n][0] *= alpha[0];
                o[n][1] *= alpha[0];
                o[n][2] *= alpha[1];
                o[n][3] *= alpha[1];
            }

            // ---- O += P V
            if constexpr (!C::Q8) {
                uint32_t pa[4];
                pa[0] = pack_h2(p[0][0], p[0][1]);
                pa[1] = pack_h2(p[0][2], p[0][3]);
                pa[2] = pack_h2(p[1][0], p[1][1]);
                pa[3] = pack_h2(p[1][2], p[1][3]);
                const int vrow = 16 * warp + (lane & 7) + 8 * ((lane >> 3) & 1);
                const uint32_t vbase = smem_u32(vst);
#pragma unroll
                for (int n = 0; n < HD / 16; n++) {
                    const int e = n * 16 + 8 * (lane >> 4);
                    const uint32_t addr = vbase + (e / C::COLS) * C::BOXB + swz_off(vrow, e % C::COLS, C::PITCH);
                    uint32_t v0, v1, v2, v3;
                    ldsm_x4_t(addr, v0, v1, v2, v3);
                    mma_f16(o[2 * n], pa, v0, v1);
                    mma_f16(o[2 * n + 1], pa, v2, v3);
                }
            } else {
                const int vrow = (lane & 7) + 8 * ((lane >> 3) & 1);
                const uint32_t vbase = smem_u32(wst + C::NB * C::WBOXB);
#pragma unroll
                for (int blk = 0; blk < C::NBLK; blk++) {
                    const float d00 = dv_tab[(2 * q4) * C::NBLK + blk];
                    const float d01 = dv_tab[(2 * q4 + 1) * C::NBLK + blk];
                    const float d10 = dv_tab[(8 + 2 * q4) * C::NBLK + blk];
                    const float d11 = dv_tab[(8 + 2 * q4 + 1) * C::NBLK + blk];
                    const float x[8] = {p[0][0] * d00, p[0][1] * d01, p[0][2] * d00, p[0][3] * d01,
                                        p[1][0] * d10, p[1][1] * d11, p[1][2] * d10, p[1][3] * d11};
                    float hi[8], lo[8];
#pragma unroll
                    for (int k = 0; k < 8; k++) {
                        hi[k] = __half2float(__float2half_rn(x[k]));
                        lo[k] = x[k] - hi[k];
                    }
                    uint32_t ph[4], pl[4];
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        ph[k] = pack_h2(hi[2 * k], hi[2 * k + 1]);
                        pl[k] = pack_h2(lo[2 * k], lo[2 * k + 1]);
                    }
#pragma unroll
                    for (int n = 2 * blk; n < 2 * blk + 2; n++) {
                        const int e = n * 16 + 8 * (lane >> 4);
                        const uint32_t addr = vbase + (e / C::COLS) * C::WBOXB + swz_off(vrow, e % C::COLS, C::PITCH);
                        uint32_t v0, v1, v2, v3;
                        ldsm_x4_t(addr, v0, v1, v2, v3);
                        mma_f16(o[2 * n], ph, v0, v1);
                        mma_f16(o[2 * n], pl, v0, v1);
                        mma_f16(o[2 * n + 1], ph, v2, v3);
                        mma_f16(o[2 * n + 1], pl, v2, v3);
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }

    // ============================ merge the four warps
#pragma unroll
    for (int i = 0; i < 2; i++) {
        l[i] += __shfl_xor_sync(0xffffffffu, l[i], 1);
        l[i] += __shfl_xor_sync(0xffffffffu, l[i], 2);
    }
    consumer_sync();   // every warp is done with the stage ring: reuse it
    float* cw = reinterpret_cast<float*>(smem);               // [4][16][HD] warp partials
    float* cm = cw + kConsumerWarps * 16 * HD;                 // [4][16] warp maxima
    float* cl = cm + kConsumerWarps * 16;                      // [4][16] warp sums
    float* rs = cl + kConsumerWarps * 16;                      // [16][4] per-row warp weights (unnormalised)
    float* rm = rs + 16 * kConsumerWarps;                      // [16][2] per-row (M, L)
    if (rrow[0] < R) {
#pragma unroll
        for (int n = 0; n < HD / 8; n++)
            *reinterpret_cast<float2*>(&cw[(warp * 16 + rrow[0]) * HD + n * 8 + 2 * q4]) = make_float2(o[n][0], o[n][1]);
    }
    if (rrow[1] < R) {
#pragma unroll
        for (int n = 0; n < HD / 8; n++)
            *reinterpret_cast<float2*>(&cw[(warp * 16 + rrow[1]) * HD + n * 8 + 2 * q4]) = make_float2(o[n][2], o[n][3]);
    }
    if (q4 == 0) {
        cm[warp * 16 + rrow[0]] = m[0];
        cm[warp * 16 + rrow[1]] = m[1];
        cl[warp * 16 + rrow[0]] = l[0];
        cl[warp * 16 + rrow[1]] = l[1];
    }
    consumer_sync();
    if (tid < R) {
        float M = -INFINITY, L = 0.0f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; w++) M = fmaxf(M, cm[w * 16 + tid]);
#pragma unroll
        for (int w = 0; w < kConsumerWarps; w++) {
            const float mw = cm[w * 16 + tid];
            const float sc = mw == -INFINITY ? 0.0f : fast_exp2(mw - M);
            rs[tid * kConsumerWarps + w] = sc;
            L += cl[w * 16 + tid] * sc;
        }
        rm[tid * 2] = M;
        rm[tid * 2 + 1] = L;
    }
    consumer_sync();

    // each thread owns float4 column groups of the R live rows
    constexpr int G4 = HD / 4;
    const int tile = qt * a.NKV + kvh;
    const int n_g = R * G4;
    if (a.n_splits == 1) {
        for (int gi = tid; gi < n_g; gi += kConsumerWarps * 32) {
            const int r = gi / G4, c = (gi % G4) * 4;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int w = 0; w < kConsumerWarps; w++) {
                const float sc = rs[r * kConsumerWarps + w];
                const float4 v = *reinterpret_cast<const float4*>(&cw[(w * 16 + r) * HD + c]);
                acc.x += v.x * sc; acc.y += v.y * sc; acc.z += v.z * sc; acc.w += v.w * sc;
            }
            const float L = rm[r * 2 + 1];
            const float inv = L > 0.0f ? 1.0f / L : 0.0f;
            const int qi = r / a.G, g = r % a.G;
            float* orow = a.out + (size_t)(t0 + qi) * a.out_nb_t + (size_t)(kvh * a.G + g) * a.out_nb_h;
            *reinterpret_cast<float4*>(orow + c) = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
        }
        return;
    }
    if (a.cluster_merge) {
        // ---- split-K inside a thread-block cluster: every split keeps its partial in its own
        // shared memory; after a cluster barrier each CTA merges a slice of the columns by
        // reading all splits' partials through distributed shared memory.
        float* po = reinterpret_cast<float*>(smem + C::PO_OFF);   // [16][HD]
        float* pm = reinterpret_cast<float*>(smem + C::PM_OFF);   // [16][2]
        for (int gi = tid; gi < n_g; gi += kConsumerWarps * 32) {
            const int r = gi / G4, c = (gi % G4) * 4;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int w = 0; w < kConsumerWarps; w++) {
                const float sc = rs[r * kConsumerWarps + w];
                const float4 v = *reinterpret_cast<const float4*>(&cw[(w * 16 + r) * HD + c]);
                acc.x += v.x * sc; acc.y += v.y * sc; acc.z += v.z * sc; acc.w += v.w * sc;
            }
            *reinterpret_cast<float4*>(&po[r * HD + c]) = acc;
        }
        if (tid < R) *reinterpret_cast<float2*>(&pm[tid * 2]) = make_float2(rm[tid * 2], rm[tid * 2 + 1]);
        cluster_sync_all();
        const int ns = a.n_splits;                    // == cluster size, rank == split
        const uint32_t rank = cluster_ctarank();
        for (int gi = (int)rank + ns * tid; gi < n_g; gi += ns * kConsumerWarps * 32) {
            const int r = gi / G4, c = (gi % G4) * 4;
            float2 ml[16];
            float4 ov[16];
            float M = -INFINITY;
#pragma unroll
            for (int sp = 0; sp < 16; sp++) {
                if (sp < ns) {
                    ml[sp] = dsmem_ld_f2(dsmem_map(smem_u32(&pm[r * 2]), sp));
                    ov[sp] = dsmem_ld_f4(dsmem_map(smem_u32(&po[r * HD + c]), sp));
                    M = fmaxf(M, ml[sp].x);
                }
            }
            float L = 0.0f;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int sp = 0; sp < 16; sp++) {
                if (sp < ns && ml[sp].x != -INFINITY) {
                    const float w = fast_exp2(ml[sp].x - M);
                    L += ml[sp].y * w;
                    acc.x += ov[sp].x * w; acc.y += ov[sp].y * w; acc.z += ov[sp].z * w; acc.w += ov[sp].w * w;
                }
            }
            const float inv = L > 0.0f ? 1.0f / L : 0.0f;
            const int qi = r / a.G, g = r % a.G;
            float* orow = a.out + (size_t)(t0 + qi) * a.out_nb_t + (size_t)(kvh * a.G + g) * a.out_nb_h;
            *reinterpret_cast<float4*>(orow + c) = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
        }
        cluster_sync_all();                          // keep every CTA's partial alive until all reads are done
        return;
    }
    // ---- split-K: publish the partial, the last CTA of the tile merges
    const size_t pbase = ((size_t)tile * a.n_splits + split) * 16;
    for (int gi = tid; gi < n_g; gi += kConsumerWarps * 32) {
        const int r = gi / G4, c = (gi % G4) * 4;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int w = 0; w < kConsumerWarps; w++) {
            const float sc = rs[r * kConsumerWarps + w];
            const float4 v = *reinterpret_cast<const float4*>(&cw[(w * 16 + r) * HD + c]);
            acc.x += v.x * sc; acc.y += v.y * sc; acc.z += v.z * sc; acc.w += v.w * sc;
        }
        *reinterpret_cast<float4*>(&a.ws_o[(pbase + r) * HD + c]) = acc;
    }
    if (tid < R) *reinterpret_cast<float2*>(&a.ws_ml[(pbase + tid) * 2]) = make_float2(rm[tid * 2], rm[tid * 2 + 1]);
    __threadfence();
    consumer_sync();
    if (tid == 0) {
        const int prev = atomicAdd(&a.tickets[tile], 1);
        flag[1] = prev == a.n_splits - 1;
    }
    consumer_sync();
    if (!flag[1]) return;
    __threadfence();
    // per (row, split) weights w = exp2(m_s - M) / L, computed once into shared memory
    const int ns = a.n_splits;
    float* wgt = reinterpret_cast<float*>(smem);               // [16][ns] (the stage ring is free)
    const size_t tbase = (size_t)tile * ns * 16;
    for (int r = warp; r < R; r += kConsumerWarps) {
        float M = -INFINITY;
        for (int sp = lane; sp < ns; sp += 32) M = fmaxf(M, __ldcg(&a.ws_ml[(tbase + (size_t)sp * 16 + r) * 2]));
#pragma unroll
        for (int o2 = 16; o2 > 0; o2 >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o2));
        float L = 0.0f;
        for (int sp = lane; sp < ns; sp += 32) {
            const float2 ml = __ldcg(reinterpret_cast<const float2*>(&a.ws_ml[(tbase + (size_t)sp * 16 + r) * 2]));
            const float w = ml.x == -INFINITY ? 0.0f : fast_exp2(ml.x - M);
            wgt[r * ns + sp] = w;
            L += ml.y * w;
        }
#pragma unroll
        for (int o2 = 16; o2 > 0; o2 >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o2);
        const float inv = L > 0.0f ? 1.0f / L : 0.0f;
        __syncwarp();
        for (int sp = lane; sp < ns; sp += 32) wgt[r * ns + sp] *= inv;
    }
    consumer_sync();
    for (int gi = tid; gi < n_g; gi += kConsumerWarps * 32) {
        const int r = gi / G4, c = (gi % G4) * 4;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        int sp = 0;
        for (; sp + 4 <= ns; sp += 4) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; u++)
                v[u] = __ldcg(reinterpret_cast<const float4*>(&a.ws_o[(tbase + (size_t)(sp + u) * 16 + r) * HD + c]));
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const float w = wgt[r * ns + sp + u];
                acc.x += v[u].x * w; acc.y += v[u].y * w; acc.z += v[u].z * w; acc.w += v[u].w * w;
            }
        }
        for (; sp < ns; sp++) {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(&a.ws_o[(tbase + (size_t)sp * 16 + r) * HD + c]));
            const float w = wgt[r * ns + sp];
            acc.x += v.x * w; acc.y += v.y * w; acc.z += v.z * w; acc.w += v.w * w;
        }
        const int qi = r / a.G, g = r % a.G;
        float* orow = a.out + (size_t)(t0 + qi) * a.out_nb_t + (size_t)(kvh * a.G + g) * a.out_nb_h;
        *reinterpret_cast<float4*>(orow + c) = acc;
    }
    if (tid == 0) a.tickets[tile] = 0;
}

// kernel attributes, once per device: dynamic shared memory and clusters of up to 16 CTAs
template <int HD, int KVT>
cudaError_t prepare_t() {
    static std::once_flag once[kMaxDevices];
    static cudaError_t status[kMaxDevices];
    return once_per_device(once, status, [] {
        using C = DecCfg<HD, KVT>;
        cudaError_t e = cudaFuncSetAttribute(fa_decode_kernel<HD, KVT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             C::SMEM + 1024);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(fa_decode_kernel<HD, KVT>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        return e;
    });
}

template <int HD, int KVT>
cudaError_t launch_t(const AttnArgs& a, const CUtensorMap* tk, const CUtensorMap* tv, cudaStream_t st) {
    using C = DecCfg<HD, KVT>;
    const int smem = C::SMEM + 1024;
    cudaError_t e = prepare_t<HD, KVT>();
    if (e != cudaSuccess) return e;
    dim3 grid((unsigned)a.n_splits, (unsigned)a.NKV, (unsigned)a.n_qtiles);
    return launch_pdl_cluster(fa_decode_kernel<HD, KVT>, grid, dim3(kThreads), (size_t)smem, st,
                              a.cluster_merge ? a.n_splits : 1, *tk, *tv, a);
}

// Largest cluster of this kernel the GPU can co-schedule (capped at 16); 1 if clusters are unusable.
template <int HD, int KVT>
int max_cluster_t() {
    static int v = -1;
    if (v < 0) {
        using C = DecCfg<HD, KVT>;
        if (prepare_t<HD, KVT>() != cudaSuccess) {
            cudaGetLastError();
            v = 1;
            return v;
        }
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(16, 1, 1);
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = C::SMEM + 1024;
        int n = 0;
        if (cudaOccupancyMaxPotentialClusterSize(&n, fa_decode_kernel<HD, KVT>, &cfg) != cudaSuccess) {
            cudaGetLastError();
            n = 1;
        }
        v = n < 1 ? 1 : (n > 16 ? 16 : n);
    }
    return v;
}

}  // namespace

int decode_max_cluster(int head_dim, int kv_type) {
    if (kv_type == SV_TYPE_Q8_0) return head_dim == 256 ? max_cluster_t<256, SV_TYPE_Q8_0>() : 1;
    switch (head_dim) {
        case 16: return max_cluster_t<16, SV_TYPE_F16>();
        case 32: return max_cluster_t<32, SV_TYPE_F16>();
        case 64: return max_cluster_t<64, SV_TYPE_F16>();
        case 128: return max_cluster_t<128, SV_TYPE_F16>();
        case 256: return max_cluster_t<256, SV_TYPE_F16>();
        default: return 1;
    }
}

int decode_block_keys() { return kBK; }

size_t decode_partial_floats(int head_dim) { return (size_t)16 * head_dim + 32; }

bool decode_supported(int head_dim, int kv_type, size_t row_bytes, int n_kv_head) {
    if (row_bytes % 16 != 0) return false;
    if (kv_type == SV_TYPE_F16)
        return head_dim == 16 || head_dim == 32 || head_dim == 64 || head_dim == 128 || head_dim == 256;
    if (kv_type == SV_TYPE_Q8_0) return head_dim == 256;
    (void)n_kv_head;
    return false;
}

bool make_decode_tmap(CUtensorMap* m, const void* base, int kv_type, int head_dim, int n_kv_head,
                      size_t row_bytes, int64_t n_rows) {
    if (kv_type == SV_TYPE_Q8_0) {
        const uint32_t headb = (uint32_t)(head_dim / kQK8_0 * kQ8_0Bytes);
        return encode_tmap_2d(m, base, CU_TENSOR_MAP_DATA_TYPE_UINT16, row_bytes / 2, (uint64_t)n_rows, row_bytes,
                              headb / 2, kBK, CU_TENSOR_MAP_SWIZZLE_NONE);
    }
    const int cols = head_dim >= 64 ? 64 : head_dim;
    const CUtensorMapSwizzle swz = cols == 64   ? CU_TENSOR_MAP_SWIZZLE_128B
                                   : cols == 32 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                : CU_TENSOR_MAP_SWIZZLE_32B;
    return encode_tmap_2d(m, base, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, (uint64_t)n_kv_head * head_dim,
                          (uint64_t)n_rows, row_bytes, (uint32_t)cols, kBK, swz);
}

cudaError_t launch_decode(const AttnArgs& a, int head_dim, int kv_type, const CUtensorMap* tk,
                          const CUtensorMap* tv, cudaStream_t st) {
    if (kv_type == SV_TYPE_Q8_0) {
        if (head_dim == 256) return launch_t<256, SV_TYPE_Q8_0>(a, tk, tv, st);
        return cudaErrorInvalidValue;
    }
    switch (head_dim) {
        case 16: return launch_t<16, SV_TYPE_F16>(a, tk, tv, st);
        case 32: return launch_t<32, SV_TYPE_F16>(a, tk, tv, st);
        case 64: return launch_t<64, SV_TYPE_F16>(a, tk, tv, st);
        case 128: return launch_t<128, SV_TYPE_F16>(a, tk, tv, st);
        case 256: return launch_t<256, SV_TYPE_F16>(a, tk, tv, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace svkv
