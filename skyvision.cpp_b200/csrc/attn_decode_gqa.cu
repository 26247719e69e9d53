// attn_decode_gqa.cu - single-step decode attention over an f16 KV cache for
// grouped-query heads (sm_100a): the latency-critical form of
// ggml_flash_attn_ext at T * (NH/NKV) <= 8 query rows per kv head
// (llm_block.hpp:268-277, qwen3vl_model.cpp:657-663 with T = 1), causal or
// unmasked.
//
// Why a second decode kernel.  With one token and 4 query heads per kv head a
// 16-row MMA tile is 75 % empty when queries are the M dimension, and the
// per-tile MMA chain (not HBM) bounds each split.  Here keys are the M
// dimension and the query rows the N dimension ("swap AB"):
//   S^T(16 keys x 8 rows)  = K(16 x HD) * Q^T(HD x 8)       mma.m16n8k16, K by ldmatrix
//   O^T(HD x 8 rows)      += V^T(HD x 16 keys) * P^T(16 x 8)  V by ldmatrix.trans,
//                                                          P^T by movmatrix.trans
// which halves the MMAs per key, keeps O in 32 registers per thread and lets
// two groups of four consumer warps work on alternate K/V tiles while two CTAs
// share an SM.  Each warp owns 16 keys of every 64-key tile of its group.
//
// Latency path (a decode step is a chain of one launch per layer): before the
// programmatic grid-dependency wait the kernel only issues loads that no
// earlier kernel of the step can change: L2 prefetches of the query rows and of
// every K/V tile of the split past the shared-memory ring, and - when the
// kernel appends the step's row itself - TMA fills of the ring.  The next
// launch may start once every split has issued its last tile.  The split-K
// partials of a kv head merge inside a thread-block cluster: CTA 0 of the
// cluster does no K/V work; every split pushes its partial into CTA 0's shared
// memory with st.async (completion counted on CTA 0's mbarrier) and exits, and
// CTA 0 merges and stores, so no split waits on a cluster-wide barrier.
// Measured on config 2 (36 layers, S ~ 4.5k): 6.3 us per layer against 8.4 us
// for the general split-K kernel.
//
// Few kv heads over a long context (a long session's per-GPU shard): the
// splits outnumber a cluster and publish their partials to the workspace; the
// last split to take the kv head's ticket merges them, or, beyond 48 splits,
// the last of each group of 16 merges its group and the last group merger
// merges the groups.  With more than 48 splits per head (f16, HD 128) the plan
// runs one CTA per SM with a 6-stage ring (kDeep) instead of two CTAs with 3.
//
// Roofline: HBM-bound, 2 * HD * 2 bytes per (key, kv head) + Q and O.
#include <algorithm>

#include "common.cuh"
#include "internal.hpp"

namespace svkv {

namespace {

constexpr int kBK = 64;                    // keys per K/V tile
constexpr int kGroups = 2;                 // consumer warp groups, alternating tiles
constexpr int kWarpsPerGroup = kBK / 16;   // 16 keys per warp
constexpr int kCWarps = kGroups * kWarpsPerGroup;
constexpr int kCThreads = kCWarps * 32;
constexpr int kThreads = kCThreads + 32;   // + one TMA producer warp
constexpr int kRows = 8;                   // query rows per kv head (N of the MMA)
constexpr int kL2Ahead = 4;                // K/V tiles past the ring prefetched into L2 before the wait
constexpr int kMergeGroup = 16;            // partials one CTA merges at most (ticket merge, two levels beyond)


constexpr int align_up(int x, int a) { return (x + a - 1) / a * a; }

// DEEP (f16, long splits over few kv heads): a 6-stage ring at one CTA per SM instead of 3 stages at two
template <int HD, int KVT, bool DEEP = false>
struct GqaCfg {
    static constexpr bool Q8 = KVT == SV_TYPE_Q8_0;
    static constexpr int COLS = 64;                       // f16 columns per TMA box (128-byte swizzle span)
    static constexpr int NB = HD / COLS;
    static constexpr int PITCH = COLS * 2;
    static constexpr int BOXB = kBK * PITCH;
    static constexpr int HEADB = Q8 ? HD / kQK8_0 * kQ8_0Bytes : HD * 2;   // one kv head of one cache row
    static constexpr int TILE_B = Q8 ? kBK * HEADB : NB * BOXB;          // K (or V) bytes per tile
    static constexpr int STAGE_B = align_up(2 * TILE_B, 1024);
    // f16 HD 64/128: ~96 KB ring, two CTAs per SM; q8_0 HD 256: one CTA per SM, deeper ring
    static constexpr int STAGES = Q8 ? 4 : ((HD == 128 && !DEEP) ? 3 : 6);
    static constexpr int MIN_BLOCKS = (Q8 || DEEP) ? 1 : 2;
    static constexpr int ROWS_MAX = HD >= 256 ? 4 : kRows;              // query rows per kv head
    static constexpr int RING_B = STAGES * STAGE_B;
    static constexpr int CW_LD = HD + 4;                  // padded row of the warp-combine scratch
    static constexpr int CW_B = kCWarps * kRows * CW_LD * 4;
    static constexpr int CM_OFF = CW_B;                   // [warp][row] maxima, then sums
    static_assert(CM_OFF + 2 * kCWarps * kRows * 4 <= RING_B, "combine scratch must fit in the stage ring");
    static_assert(ROWS_MAX * (HD / 4) <= kCThreads, "one (row, 4-column) group per consumer thread");
    // cluster merge, merger CTA only: partial O [split][row][HD] and (m, l) [split][row]
    static constexpr int PUSH_O = 0;
    static constexpr int PUSH_ML = 16 * ROWS_MAX * HD * 4;
    static_assert(PUSH_ML + 16 * ROWS_MAX * 8 <= RING_B, "merge slots must fit in the stage ring");
    static constexpr int BAR_OFF = RING_B;
    // the launch's query rows of this kv head as f16, staged once per CTA (rows past R are zero);
    // the row pitch is padded by 16 bytes so the fragment reads of the 8 rows hit distinct banks
    static constexpr int QPITCH = HD * 2 + 16;
    static constexpr int Q_OFF = align_up(BAR_OFF + (2 * STAGES + 1) * 8 + 16, 128);   // after the barriers, flags
    static_assert(Q_OFF % 16 == 0 && QPITCH % 16 == 0, "16-byte stores into the query rows");
    static constexpr int SMEM = Q_OFF + kRows * QPITCH;
    static_assert(SMEM + 1024 <= 227 * 1024, "shared memory budget");
};

// Signed bytes -> exact f16 integers: with u = b ^ 0x80 = b + 128, the f16 bit pattern 0x64uu is
// 1024 + u, and subtracting 1152 leaves b.  x = the four bytes of w after the XOR; sel picks two of
// them into the low bytes of the two halves (byte_perm selector nibbles; 4 = the 0x64 byte).
template <uint32_t kSel>
__device__ __forceinline__ uint32_t u8x2_to_h2(uint32_t x) {
    const uint32_t h = __byte_perm(x, 0x64646464u, kSel);
    __half2 r = __hsub2(*reinterpret_cast<const __half2*>(&h), __half2half2(__ushort_as_half(0x6480u)));
    return *reinterpret_cast<uint32_t*>(&r);
}

// four bytes of a q8_0 row at p, which is 4-byte aligned when `aligned`, else 2-byte aligned (the
// callers' loops are unrolled, so the branch folds away)
__device__ __forceinline__ uint32_t ld_b4(const uint8_t* p, bool aligned) {
    if (aligned) return *reinterpret_cast<const uint32_t*>(p);
    return __byte_perm(*reinterpret_cast<const uint16_t*>(p), *reinterpret_cast<const uint16_t*>(p + 2), 0x5410);
}

// Fused q8_0 append: lane l quantises elements [8l, 8l + 8) of one kv head's source row (f16, 16-byte
// aligned) with the steps of the append kernel (ggml's block_q8_0 rule: d = amax / 127, id = 1 / d,
// q = round-half-away(x * id), d stored as f16), so the bytes match sv_set_rows exactly, and writes
// them both to the cache row (gdst) and into the shared-memory tile that holds the row (sdst).  The
// four lanes of a 32-element block are consecutive.  HD = 256: the warp covers the head.
__device__ __forceinline__ void quantize_head_q8_0(const uint8_t* src, uint8_t* gdst, uint8_t* sdst, int lane) {
    const uint4 u = *reinterpret_cast<const uint4*>(src + lane * 16);
    const __half2* h = reinterpret_cast<const __half2*>(&u);
    float v[8];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float2 f = __half22float2(h[i]);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
    }
    float amax = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; k++) amax = fmaxf(amax, fabsf(v[k]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const float dd = __fdiv_rn(amax, 127.0f);
    const float id = dd != 0.0f ? __fdiv_rn(1.0f, dd) : 0.0f;
    const int b = lane >> 2, sub = (lane & 3) * 8;
    const int ob = b * kQ8_0Bytes;
    if (sub == 0) {
        const __half hd = __float2half_rn(dd);
        *reinterpret_cast<__half*>(gdst + ob) = hd;   // 2-byte aligned (34 * b)
        *reinterpret_cast<__half*>(sdst + ob) = hd;
    }
#pragma unroll
    for (int k = 0; k < 8; k += 2) {
        const int q0 = (int)roundf(__fmul_rn(v[k], id));
        const int q1 = (int)roundf(__fmul_rn(v[k + 1], id));
        const uint16_t pr = (uint16_t)((uint8_t)(int8_t)q0 | ((uint16_t)(uint8_t)(int8_t)q1 << 8));
        *reinterpret_cast<uint16_t*>(gdst + ob + 2 + sub + k) = pr;   // even offsets
        *reinterpret_cast<uint16_t*>(sdst + ob + 2 + sub + k) = pr;
    }
}

__device__ __forceinline__ void consumer_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kCThreads) : "memory");
}

// transpose an 8x8 f16 fragment across the warp
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}

// asynchronous stores into another CTA's shared memory, counted on that CTA's mbarrier
__device__ __forceinline__ void st_async_f4(uint32_t caddr, float4 v, uint32_t cbar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];"
                 ::"r"(caddr), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "r"(cbar) : "memory");
}
__device__ __forceinline__ void st_async_f2(uint32_t caddr, float2 v, uint32_t cbar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];"
                 ::"r"(caddr), "f"(v.x), "f"(v.y), "r"(cbar) : "memory");
}

// One finished (row, 4-column) group of the output: to `out`, or with the gather fused in, into
// every rank's gathered buffer over NVLink (plain stores to peer memory).
template <bool kPeer>
__device__ __forceinline__ void store_out4(const AttnArgs& a, int kvh, int r, int c, float4 v) {
    const int qi = r / a.G, g = r % a.G;
    if (!kPeer) {
        float* orow = a.out + (size_t)qi * a.out_nb_t + (size_t)(kvh * a.G + g) * a.out_nb_h;
        *reinterpret_cast<float4*>(orow + c) = v;
        return;
    }
    for (int p = 0; p < a.n_peers; p++) {   // every rank's gathered buffer, this rank's own included
        float* prow = a.peer_out[p] + (size_t)qi * a.peer_nb_t + (size_t)(a.head_offset + kvh * a.G + g) * a.out_nb_h;
        *reinterpret_cast<float4*>(prow + c) = v;
    }
}

// After all of a kv head's rows were stored (by the threads that named barrier `bar_id` joins):
// make them visible system-wide, then count the head on every rank.
template <bool kPeer>
__device__ __forceinline__ void signal_peers(const AttnArgs& a, int bar_id, int n_threads) {
    if (!kPeer) return;
    __threadfence_system();
    __syncwarp();
    asm volatile("barrier.sync %0, %1;" ::"r"(bar_id), "r"(n_threads) : "memory");
    if (threadIdx.x == 0)
        for (int p = 0; p < a.n_peers; p++) atomicAdd_system(a.peer_ctr[p], 1u);
}

// Wait (bounded) for the previous layer's gather: *wait_ctr >= *epoch * per_epoch.
__device__ __forceinline__ void wait_gather(const AttnArgs& a) {
    const unsigned int target = (unsigned int)(*reinterpret_cast<const volatile int*>(a.epoch_dev)) * a.wait_per_epoch;
    const uint64_t t0 = globaltimer_ns();
    // acquire loads: the peers' rows, stored before their release of the counter, are visible to every
    // read this CTA makes after the barrier that follows
    while (ld_acquire_sys(a.wait_ctr) < target) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
            if (a.err) atomicOr(a.err, ERRBIT_TIMEOUT);
            break;
        }
    }
}

template <int HD, int KVT, bool kPeer, bool kDeep>
__global__ void __launch_bounds__(kThreads, GqaCfg<HD, KVT, kDeep>::MIN_BLOCKS)
fa_decode_gqa_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                     const __grid_constant__ AttnArgs a) {
    using C = GqaCfg<HD, KVT, kDeep>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
    uint64_t* empty = full + C::STAGES;
    uint64_t* mdata = empty + C::STAGES;                                        // leader: merge slots filled
    volatile int* flag = reinterpret_cast<volatile int*>(mdata + 1);            // [0] abort

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // with a cluster merge, CTA 0 of each kv head's cluster is the merger (no K/V work) and CTA
    // x >= 1 is split x - 1
    const int kvh = blockIdx.y;
    const bool merger = a.cluster_merge && blockIdx.x == 0;
    const int split = a.cluster_merge ? (int)blockIdx.x - 1 : (int)blockIdx.x;
    const int nq = a.T;                       // one query tile: every query of the launch
    const int R = nq * a.G;                   // <= kRows, checked by the host

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kWarpsPerGroup);
        }
        mbar_init(mdata, 1);
        flag[0] = 0;
        fence_barrier_init();
        // the other splits' partials: R rows of HD floats and an (m, l) pair each
        if (merger) mbar_arrive_expect_tx(mdata, (uint32_t)(a.n_splits * R * (HD * 4 + 8)));
    }
    if (threadIdx.x == kCThreads) {
        tma_prefetch_desc(&tmk);
        tma_prefetch_desc(&tmv);
    }
    __syncthreads();
    // every CTA of the cluster has initialised its barriers: the splits wait on this before their
    // first remote store into the merger (the wait is long satisfied by then)
    if (a.cluster_merge) cluster_arrive_relaxed();

    if (merger) {
        // ============================ merger: sum the splits' partials of this kv head
        constexpr int G4m = HD / 4;
        const int gi = threadIdx.x, n_gm = R * G4m;
        // the parameters the merge and the stores read, into the constant cache before the wait (a
        // cold line read after it would sit on the launch's critical path)
        asm volatile("" ::"l"(a.out), "l"(a.out_nb_t), "l"(a.out_nb_h), "r"(a.G), "r"(a.n_splits), "l"(a.err));
        pdl_wait();   // the output may still be in use by the previous launch
        if (threadIdx.x == 0) pdl_trigger();   // the splits decide when the next launch may start
        // every thread reaches the final signal (a named barrier when the gather is fused in)
        if (gi < n_gm && mbar_wait(mdata, 0, a.err)) {
            const int r = gi / G4m, c = (gi % G4m) * 4;
            const float* slot_o = reinterpret_cast<const float*>(smem + C::PUSH_O);
            const float* slot_ml = reinterpret_cast<const float*>(smem + C::PUSH_ML);
            const int ns = a.n_splits;
            float2 ml[16];
#pragma unroll
            for (int sp = 0; sp < 16; sp++)
                if (sp < ns) ml[sp] = *reinterpret_cast<const float2*>(&slot_ml[(sp * C::ROWS_MAX + r) * 2]);
            float MM = -INFINITY;
#pragma unroll
            for (int sp = 0; sp < 16; sp++)
                if (sp < ns) MM = fmaxf(MM, ml[sp].x);
            float LL = 0.0f;
            float4 o4 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int sp = 0; sp < 16; sp++) {
                if (sp < ns && ml[sp].x != -INFINITY) {
                    const float w = fast_exp2(ml[sp].x - MM);
                    LL += ml[sp].y * w;
                    const float4 v = *reinterpret_cast<const float4*>(&slot_o[(sp * C::ROWS_MAX + r) * HD + c]);
                    o4.x += v.x * w; o4.y += v.y * w; o4.z += v.z * w; o4.w += v.w * w;
                }
            }
            const float inv = LL > 0.0f ? 1.0f / LL : 0.0f;
            store_out4<kPeer>(a, kvh, r, c, make_float4(o4.x * inv, o4.y * inv, o4.z * inv, o4.w * inv));
        }
        signal_peers<kPeer>(a, 3, kThreads);
        return;
    }

    auto issue = [&](int j, int y) {
        const int s = j % C::STAGES;
        uint8_t* kst = smem + s * C::STAGE_B;
        uint8_t* vst = kst + C::TILE_B;
        mbar_arrive_expect_tx(&full[s], 2 * C::TILE_B);
        if constexpr (C::Q8) {     // q8_0 rows as 16-bit units, one unswizzled box per tensor
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

    // ---- before the grid dependency: loads no earlier kernel of the step can change
    const int ks0 = split * a.chunk;
    const int kmax = min(a.S, ks0 + a.chunk);
    int prefetched = 0;
    if (warp == kCWarps) {
        // L2 prefetch of the query rows (the previous kernel may still write them: only a hint)
        const int q_es = a.q_type == SV_TYPE_F32 ? 4 : 2;
        const int lines = HD * q_es / 128;
        for (int i = lane; i < R * lines; i += 32) {
            const int r = i / lines, qi = r / a.G, g = r % a.G;
            prefetch_l2(a.q + (size_t)qi * a.q_nb_t + (size_t)(kvh * a.G + g) * a.q_nb_h + (i % lines) * 128);
        }
        if (lane == 0) {
            int j0 = 0;
            if (a.n_new > 0 && a.ring_prefill) {
                // the kernel appends the step's rows itself and the launch before it wrote no cache rows
                // while letting this one start early: the rows it reads are complete (the appended ones
                // are patched in below), so the ring can fill now -- first of all, before the n_past
                // hint below is read (a global load whose latency would hold these copies back)
                const int nt_max = kmax > ks0 ? (kmax - ks0 + kBK - 1) / kBK : 0;
                prefetched = min(nt_max, C::STAGES);
                for (int j = 0; j < prefetched; j++) issue(j, a.row_base + ks0 + j * kBK);
                j0 = prefetched;
            }
            // the split's last visible key, from a possibly stale n_past (a hint for the prefetch extent only)
            int hint = a.causal_base;
            if (a.causal_base_dev) hint = *reinterpret_cast<const volatile int*>(a.causal_base_dev);
            const int pf_hi = a.mask_mode == SV_MASK_CAUSAL ? min(kmax, hint + nq + 1) : kmax;
            const int nt_pf = pf_hi > ks0 ? (pf_hi - ks0 + kBK - 1) / kBK : 0;
            // a few tiles past the ring only: long splits stream the rest (an L2 prefetch of a whole
            // long context would evict itself before use)
            const int pf_end = min(nt_pf, C::STAGES + kL2Ahead);
            for (int j = j0; j < pf_end; j++) {
                if constexpr (C::Q8) {
                    tma_prefetch_l2_2d(&tmk, kvh * (C::HEADB / 2), a.row_base + ks0 + j * kBK);
                    tma_prefetch_l2_2d(&tmv, kvh * (C::HEADB / 2), a.row_base + ks0 + j * kBK);
                } else {
#pragma unroll
                    for (int b = 0; b < C::NB; b++) {
                        tma_prefetch_l2_2d(&tmk, kvh * HD + b * C::COLS, a.row_base + ks0 + j * kBK);
                        tma_prefetch_l2_2d(&tmv, kvh * HD + b * C::COLS, a.row_base + ks0 + j * kBK);
                    }
                }
            }
        }
    }
    const bool do_gather_wait = kPeer && a.wait_ctr != nullptr;   // decided before the dependency wait
    if (warp < kCWarps) {
        // bring the launch's parameters into this SM's constant cache now: after the wait every
        // first touch of a cold parameter line would add a memory round trip to the critical path
        asm volatile("" ::"l"(a.q), "l"(a.q_nb_t), "l"(a.q_nb_h), "r"(a.G), "r"(a.q_type), "f"(a.scale_log2),
                     "l"(a.out), "l"(a.out_nb_t), "l"(a.out_nb_h), "r"(a.mask_mode), "r"(a.S), "r"(a.chunk));
        asm volatile("" ::"r"(a.n_new), "l"(a.knew), "l"(a.vnew), "l"(a.new_nb_t), "l"(a.kc_w), "l"(a.vc_w),
                     "l"(a.cache_row_bytes), "l"(a.err), "r"(a.cluster_merge), "r"(a.n_splits),
                     "l"(a.causal_base_dev), "r"(a.causal_base), "r"(a.row_base));
        if (kPeer)
            asm volatile("" ::"l"(a.peer_out), "l"(a.peer_ctr), "r"(a.head_offset), "l"(a.peer_nb_t),
                         "l"(a.wait_ctr), "l"(a.epoch_dev), "r"(a.wait_per_epoch));
    }
    pdl_wait();
    // n_past first: its load is in flight while the query rows are staged below (it bounds the key
    // range; read after the query rows it added a second dependent memory round trip per layer)
    const int cbase = a.causal_base_dev ? __ldg(a.causal_base_dev) : a.causal_base;

    // with the gather fused in, the query rows may depend on the previous layer's gathered output:
    // thread 0 waits (bounded) for its arrival count, then the consumer warps go on
    if (do_gather_wait && warp < kCWarps) {
        if (threadIdx.x == 0) wait_gather(a);
        __syncwarp();
        asm volatile("barrier.sync 1, %0;" ::"n"(kCThreads) : "memory");
    }
    // consumers: the query rows first (nothing below waits on them until the first tile).  They are
    // staged in shared memory with 16-byte loads spread over the consumer threads -- R rows of HD f16
    // are a few dozen requests, where per-thread fragment loads (16 scattered 4-byte words per
    // thread) put ~1000 sector requests per CTA into the memory system right after the dependency --
    // and each thread then reads its fragments from there.
    const int gq = lane >> 2, tq = lane & 3;     // fragment row / column-pair index
    const int q_es = a.q_type == SV_TYPE_F32 ? 4 : 2;
    // Q^T as B fragments: rows k = head-dim, column n = query row gq
    uint32_t qb[HD / 16][2];
    if (warp < kCWarps) {
        uint8_t* qs = smem + C::Q_OFF;
        for (int i = threadIdx.x; i < kRows * (HD / 8); i += kCThreads) {
            const int r = i / (HD / 8), e = (i % (HD / 8)) * 8;
            uint4 v = make_uint4(0, 0, 0, 0);
            if (r < R) {
                const uint8_t* src = a.q + (size_t)(r / a.G) * a.q_nb_t + (size_t)(kvh * a.G + r % a.G) * a.q_nb_h +
                                     (size_t)e * q_es;
                if (a.q_type == SV_TYPE_F32) {
                    if ((reinterpret_cast<uintptr_t>(src) & 15) == 0) {
                        const float4 f0 = *reinterpret_cast<const float4*>(src);
                        const float4 f1 = *reinterpret_cast<const float4*>(src + 16);
                        v = make_uint4(pack_h2(f0.x, f0.y), pack_h2(f0.z, f0.w), pack_h2(f1.x, f1.y),
                                       pack_h2(f1.z, f1.w));
                    } else {
                        const float* f = reinterpret_cast<const float*>(src);
                        v = make_uint4(pack_h2(f[0], f[1]), pack_h2(f[2], f[3]), pack_h2(f[4], f[5]), pack_h2(f[6], f[7]));
                    }
                } else if ((reinterpret_cast<uintptr_t>(src) & 15) == 0) {
                    v = *reinterpret_cast<const uint4*>(src);
                } else {
                    const uint32_t* w = reinterpret_cast<const uint32_t*>(src);
                    v = make_uint4(w[0], w[1], w[2], w[3]);
                }
            }
            *reinterpret_cast<uint4*>(qs + r * C::QPITCH + e * 2) = v;
        }
        consumer_sync();
#pragma unroll
        for (int kk = 0; kk < HD / 16; kk++) {
#pragma unroll
            for (int h = 0; h < 2; h++) {
                // q8_0: thread tq's fragment columns are the 4 consecutive elements at 4*tq of the
                // k-step (in K and Q alike, so the dot products are unchanged)
                const int e = C::Q8 ? kk * 16 + 4 * tq + 2 * h : kk * 16 + h * 8 + 2 * tq;
                qb[kk][h] = *reinterpret_cast<const uint32_t*>(qs + gq * C::QPITCH + e * 2);
            }
        }
    }

    // ---- key range of this split
    const int khi = a.mask_mode == SV_MASK_CAUSAL ? min(a.S, cbase + nq) : a.S;
    const int ks = ks0;
    const int ke = min(khi, ks + a.chunk);
    const int n_tiles = ke > ks ? (ke - ks + kBK - 1) / kBK : 0;
    if (threadIdx.x == 0 && split == 0 && kvh == 0 && a.err && a.n_new > 0 && cbase + a.n_new > a.S)
        atomicOr(a.err, ERRBIT_ROW_RANGE);   // appended rows past the grid's key bound are not written

    if (warp == kCWarps) {
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
            // The next launch of the stream may start once every split has issued its last tile: its
            // CTAs begin prefetching their own K/V at once, and triggering right after the grid
            // dependency (measured: 7.7 vs 6.9 us per layer on config 2) floods HBM while this
            // launch still waits on its query rows and last tiles.
            pdl_trigger();
            // never leave a bulk copy in flight into shared memory
            for (int j = max(0, issued - C::STAGES); j < issued; j++)
                mbar_wait(&full[j % C::STAGES], (j / C::STAGES) & 1, a.err);
        }
        return;
    }

    // ============================ consumers
    const int tid = threadIdx.x;                 // 0..255
    const int grp = warp / kWarpsPerGroup, wig = warp % kWarpsPerGroup;

    // per thread: query columns c0 = 2*tq, c1 = 2*tq + 1; visible-key limits
    int qlim[2];
    bool qvalid[2];
#pragma unroll
    for (int i = 0; i < 2; i++) {
        const int r = 2 * tq + i;
        qvalid[i] = r < R;
        qlim[i] = a.mask_mode == SV_MASK_CAUSAL ? cbase + r / a.G : a.S - 1;
    }

    float o[HD / 16][4];
#pragma unroll
    for (int n = 0; n < HD / 16; n++) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
    float m[2] = {-INFINITY, -INFINITY};
    float l[2] = {0.0f, 0.0f};

    for (int j = grp; j < n_tiles; j += kGroups) {
        const int s = j % C::STAGES;
        // The two groups share the ring, so a group can reach stage s while the other group's tile
        // j - STAGES still holds it (its fill may even be in flight).  A parity wait on full[s] alone
        // cannot tell that phase from this one; waiting first for tile j - STAGES to be released
        // (empty[s], which is at most one phase behind: this group released tile j - 2*STAGES)
        // leaves exactly one pending fill of the stage, this tile's.
        if (j >= C::STAGES && !mbar_wait(&empty[s], ((j / C::STAGES) - 1) & 1, a.err)) {
            flag[0] = 1;
            break;
        }
        if (!mbar_wait(&full[s], (j / C::STAGES) & 1, a.err)) {
            flag[0] = 1;
            break;
        }
        const int kw = ks + j * kBK + 16 * wig;   // first key of this warp
        uint8_t* kst = smem + s * C::STAGE_B;
        uint8_t* vst = kst + C::TILE_B;
        if (kw < ke) {
            // fused append (f16 caches): a key this launch appends is written to the cache from its
            // source row and patched into the tile the TMA brought in (which may hold the old row)
            if (!C::Q8 && a.n_new > 0 && kw < cbase + a.n_new && kw + 16 > cbase) {
                constexpr int LANES = HD * 2 / 16;
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
                        *reinterpret_cast<uint4*>(kst + off) = kvec;
                        *reinterpret_cast<uint4*>(vst + off) = vvec;
                    }
                }
                fence_proxy_async_smem();   // order these writes before the stage's next TMA fill
                __syncwarp();
            }
            // fused append (q8_0 caches): each appended key of this warp is quantised from its f16
            // source row into the cache and into the tile the TMA brought in
            if (C::Q8 && a.n_new > 0 && kw < cbase + a.n_new && kw + 16 > cbase) {
                static_assert(!C::Q8 || HD == 256, "one warp quantises one kv head");
                const int k_lo = max(kw, cbase), k_hi = min(kw + 16, cbase + a.n_new);
                for (int key = k_lo; key < k_hi; key++) {
                    const int row = key - (ks + j * kBK);
                    const size_t so = (size_t)(key - cbase) * a.new_nb_t + (size_t)kvh * HD * 2;
                    const size_t co = (size_t)key * a.cache_row_bytes + (size_t)kvh * C::HEADB;
                    quantize_head_q8_0(a.knew + so, a.kc_w + co, kst + row * C::HEADB, lane);
                    quantize_head_q8_0(a.vnew + so, a.vc_w + co, vst + row * C::HEADB, lane);
                }
                fence_proxy_async_smem();   // order these writes before the stage's next TMA fill
                __syncwarp();
            }
            // ---- S^T = K Q^T: four accumulator chains over the head-dim blocks
            float sacc[4][4] = {};
            if constexpr (!C::Q8) {
                const int krow = 16 * wig + (lane & 15);
                const uint32_t kbase = smem_u32(kst);
#pragma unroll
                for (int kk = 0; kk < HD / 16; kk++) {
                    const int e = kk * 16 + 8 * (lane >> 4);
                    uint32_t af[4];
                    ldsm_x4(kbase + (e / C::COLS) * C::BOXB + swz_off(krow, e % C::COLS, C::PITCH), af[0], af[1],
                            af[2], af[3]);
                    mma_f16(sacc[kk & 3], af, qb[kk][0], qb[kk][1]);
                }
            } else {
                // q8_0: the A fragments straight from the raw rows, 4 consecutive bytes per (key,
                // k-step) and thread (a0 / a1 = its first pair, a2 / a3 its second); each 32-column
                // block sums in a fresh accumulator scaled by its key's d, so K enters exactly as the
                // oracle dequantises it.  A block's bytes start 2 + 34*b into the 4-byte aligned row:
                // aligned for odd b, 2 bytes off for even b (both known at compile time).
                const uint8_t* kr0 = kst + (16 * wig + gq) * C::HEADB;     // key gq of this warp
                const uint8_t* kr1 = kr0 + 8 * C::HEADB;                    // key gq + 8
#pragma unroll
                for (int b = 0; b < HD / kQK8_0; b++) {
                    float sb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                    for (int h = 0; h < 2; h++) {
                        const int c0 = 2 + b * kQ8_0Bytes + h * 16 + 4 * tq;
                        const uint32_t x0 = ld_b4(kr0 + c0, (b & 1) == 1) ^ 0x80808080u;
                        const uint32_t x1 = ld_b4(kr1 + c0, (b & 1) == 1) ^ 0x80808080u;
                        uint32_t af[4];
                        af[0] = u8x2_to_h2<0x4140>(x0);
                        af[1] = u8x2_to_h2<0x4140>(x1);
                        af[2] = u8x2_to_h2<0x4342>(x0);
                        af[3] = u8x2_to_h2<0x4342>(x1);
                        mma_f16(sb, af, qb[2 * b + h][0], qb[2 * b + h][1]);
                    }
                    const float d0 = h2f(*reinterpret_cast<const uint16_t*>(kr0 + b * kQ8_0Bytes));
                    const float d1 = h2f(*reinterpret_cast<const uint16_t*>(kr1 + b * kQ8_0Bytes));
                    float* acc = sacc[b & 3];
                    acc[0] = fmaf(d0, sb[0], acc[0]);
                    acc[1] = fmaf(d0, sb[1], acc[1]);
                    acc[2] = fmaf(d1, sb[2], acc[2]);
                    acc[3] = fmaf(d1, sb[3], acc[3]);
                }
            }
            // ---- scale + mask (log2 domain); element i: key kw + gq + 8*(i>>1), column 2*tq + (i&1)
            float sv[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int key = kw + gq + 8 * (i >> 1);
                const int c = i & 1;
                const bool vis = qvalid[c] && key < ke && key <= qlim[c];
                sv[i] = vis ? ((sacc[0][i] + sacc[1][i]) + (sacc[2][i] + sacc[3][i])) * a.scale_log2 : -INFINITY;
            }
            // ---- online softmax per column over the warp's 16 keys (8 lanes share a column pair)
            float alpha[2], mu[2];
#pragma unroll
            for (int c = 0; c < 2; c++) {
                float mx = fmaxf(sv[c], sv[c + 2]);
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
                const float mn = fmaxf(m[c], mx);
                alpha[c] = m[c] == -INFINITY ? 0.0f : fast_exp2(m[c] - mn);
                m[c] = mn;
                mu[c] = mn == -INFINITY ? 0.0f : mn;
            }
            float p[4];
#pragma unroll
            for (int i = 0; i < 4; i++) p[i] = fast_exp2(sv[i] - mu[i & 1]);
            // per-thread partial sums (the column's lanes are summed once at the end)
            l[0] = l[0] * alpha[0] + (p[0] + p[2]);
            l[1] = l[1] * alpha[1] + (p[1] + p[3]);
#pragma unroll
            for (int n = 0; n < HD / 16; n++) {
                o[n][0] *= alpha[0];
                o[n][1] *= alpha[1];
                o[n][2] *= alpha[0];
                o[n][3] *= alpha[1];
            }
            // ---- P^T as the B fragment: transpose the two 8x8 key blocks
            const uint32_t pb0 = movmatrix_t(pack_h2(p[0], p[1]));   // keys 0-7
            const uint32_t pb1 = movmatrix_t(pack_h2(p[2], p[3]));   // keys 8-15
            // ---- O^T += V^T P^T
            if constexpr (!C::Q8) {
                const int vrow = 16 * wig + (lane & 7) + 8 * (lane >> 4);
                const uint32_t vbase = smem_u32(vst);
#pragma unroll
                for (int n = 0; n < HD / 16; n++) {
                    const int e = n * 16 + 8 * ((lane >> 3) & 1);
                    uint32_t af[4];
                    ldsm_x4_t(vbase + (e / C::COLS) * C::BOXB + swz_off(vrow, e % C::COLS, C::PITCH), af[0], af[1],
                              af[2], af[3]);
                    mma_f16(o[n], af, pb0, pb1);
                }
            } else {
                // q8_0: the A fragments of V^T straight from the raw rows.  M-row gq of m-tile n is
                // dim 16n + 2gq and M-row gq + 8 is dim 16n + 2gq + 1 (adjacent bytes of a key's row;
                // the combine below puts the outputs back in order), keys in natural order: a0 / a1 =
                // the two dims of keys 2tq, 2tq+1, a2 / a3 of keys 2tq+8, 2tq+9.  Each 32-column
                // block's d is folded into P (keys 2tq, 2tq+1, 2tq+8, 2tq+9 of the B fragment), split
                // into f16 hi + lo parts so P*d enters without a second rounding.
                const uint8_t* vr = vst + (16 * wig) * C::HEADB;
                const uint8_t* vk0 = vr + (2 * tq) * C::HEADB;
                const uint8_t* vk1 = vk0 + C::HEADB;
                const uint8_t* vk8 = vk0 + 8 * C::HEADB;
                const uint8_t* vk9 = vk8 + C::HEADB;
                const __half2 pA = *reinterpret_cast<const __half2*>(&pb0);   // keys 2tq, 2tq + 1
                const __half2 pB = *reinterpret_cast<const __half2*>(&pb1);   // keys 2tq + 8, 2tq + 9
#pragma unroll
                for (int blk = 0; blk < HD / kQK8_0; blk++) {
                    const int db = blk * kQ8_0Bytes;
                    // P * d in packed f16: hi = HMUL2 rounds the exact product once, lo = HFMA2 rounds
                    // (P * d - hi) once -- the same two roundings as in f32 then f16, in 2 instructions
                    const uint32_t dA = __byte_perm(*reinterpret_cast<const uint16_t*>(vk0 + db),
                                                    *reinterpret_cast<const uint16_t*>(vk1 + db), 0x5410);
                    const uint32_t dB = __byte_perm(*reinterpret_cast<const uint16_t*>(vk8 + db),
                                                    *reinterpret_cast<const uint16_t*>(vk9 + db), 0x5410);
                    const __half2 hA = __hmul2(pA, *reinterpret_cast<const __half2*>(&dA));
                    const __half2 hB = __hmul2(pB, *reinterpret_cast<const __half2*>(&dB));
                    const __half2 lA = __hfma2(pA, *reinterpret_cast<const __half2*>(&dA), __hneg2(hA));
                    const __half2 lB = __hfma2(pB, *reinterpret_cast<const __half2*>(&dB), __hneg2(hB));
                    const uint32_t bh0 = *reinterpret_cast<const uint32_t*>(&hA), bh1 = *reinterpret_cast<const uint32_t*>(&hB);
                    const uint32_t bl0 = *reinterpret_cast<const uint32_t*>(&lA), bl1 = *reinterpret_cast<const uint32_t*>(&lB);
#pragma unroll
                    for (int n = 2 * blk; n < 2 * blk + 2; n++) {
                        const int off = db + 2 + (n & 1) * 16 + 2 * gq;      // dims 16n + 2gq, + 1
                        // bytes [key k, dim d]: {k0 d0, k0 d1, k1 d0, k1 d1} after the first permute
                        const uint32_t x01 = __byte_perm(*reinterpret_cast<const uint16_t*>(vk0 + off),
                                                         *reinterpret_cast<const uint16_t*>(vk1 + off), 0x5410) ^
                                             0x80808080u;
                        const uint32_t x89 = __byte_perm(*reinterpret_cast<const uint16_t*>(vk8 + off),
                                                         *reinterpret_cast<const uint16_t*>(vk9 + off), 0x5410) ^
                                             0x80808080u;
                        uint32_t af[4];
                        af[0] = u8x2_to_h2<0x4240>(x01);
                        af[1] = u8x2_to_h2<0x4341>(x01);
                        af[2] = u8x2_to_h2<0x4240>(x89);
                        af[3] = u8x2_to_h2<0x4341>(x89);
                        mma_f16(o[n], af, bh0, bh1);
                        mma_f16(o[n], af, bl0, bl1);
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }

    // ============================ merge the eight warps
#pragma unroll
    for (int c = 0; c < 2; c++) {
        l[c] += __shfl_xor_sync(0xffffffffu, l[c], 4);
        l[c] += __shfl_xor_sync(0xffffffffu, l[c], 8);
        l[c] += __shfl_xor_sync(0xffffffffu, l[c], 16);
    }
    consumer_sync();   // every warp is done with the stage ring: reuse it
    float* cw = reinterpret_cast<float*>(smem);                   // [warp][row][CW_LD]
    float* cm = reinterpret_cast<float*>(smem + C::CM_OFF);       // [warp][row]
    float* cl = cm + kCWarps * kRows;                              // [warp][row]
#pragma unroll
    for (int c = 0; c < 2; c++) {
        const int r = 2 * tq + c;
        if (r < R) {
            float* dst = cw + (warp * kRows + r) * C::CW_LD;
#pragma unroll
            for (int n = 0; n < HD / 16; n++) {
                if constexpr (C::Q8) {   // the V^T M-rows gq, gq + 8 are dims 2gq, 2gq + 1 of the m-tile
                    dst[n * 16 + 2 * gq] = o[n][c];
                    dst[n * 16 + 2 * gq + 1] = o[n][c + 2];
                } else {
                    dst[n * 16 + gq] = o[n][c];
                    dst[n * 16 + gq + 8] = o[n][c + 2];
                }
            }
            if (gq == 0) {
                cm[warp * kRows + r] = m[c];
                cl[warp * kRows + r] = l[c];
            }
        }
    }
    consumer_sync();

    constexpr int G4 = HD / 4;
    const int n_g = R * G4;
    if (!a.cluster_merge && a.n_splits == 1) {   // one split: normalise and store
        for (int gi = tid; gi < n_g; gi += kCThreads) {
            const int r = gi / G4, c = (gi % G4) * 4;
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < kCWarps; w++) M = fmaxf(M, cm[w * kRows + r]);
            float L = 0.0f;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int w = 0; w < kCWarps; w++) {
                const float mw = cm[w * kRows + r];
                const float sc = mw == -INFINITY ? 0.0f : fast_exp2(mw - M);
                L += cl[w * kRows + r] * sc;
                const float4 v = *reinterpret_cast<const float4*>(&cw[(w * kRows + r) * C::CW_LD + c]);
                acc.x += v.x * sc; acc.y += v.y * sc; acc.z += v.z * sc; acc.w += v.w * sc;
            }
            const float inv = L > 0.0f ? 1.0f / L : 0.0f;
            store_out4<kPeer>(a, kvh, r, c, make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv));
        }
        signal_peers<kPeer>(a, 1, kCThreads);
        return;
    }

    if (!a.cluster_merge) {
        // ---- split-K without a cluster (many splits: few kv heads over a long context): every
        // split publishes its partial to the workspace.  Up to kMergeGroup splits, the last CTA of the
        // kv head (atomic ticket, no spinning) merges all partials.  With more splits, and ticket room
        // for the groups (merge_levels = 2), the merge has two levels, so no CTA reads more than
        // kMergeGroup partials (a 228-partial merge by one CTA took ~25 us): the last split of each group of
        // kMergeGroup merges the group into the slot of the group's first split, and the last group
        // merger of the kv head merges the groups.  Every last CTA resets the ticket it took.
        volatile int* last = flag + 1;
        const int ns = a.n_splits;
        const size_t pbase = ((size_t)kvh * ns + split) * 16;   // 16-row partial slots per split
        for (int gi = tid; gi < n_g; gi += kCThreads) {
            const int r = gi / G4, c = (gi % G4) * 4;
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < kCWarps; w++) M = fmaxf(M, cm[w * kRows + r]);
            float L = 0.0f;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int w = 0; w < kCWarps; w++) {
                const float mw = cm[w * kRows + r];
                const float sc = mw == -INFINITY ? 0.0f : fast_exp2(mw - M);
                L += cl[w * kRows + r] * sc;
                const float4 v = *reinterpret_cast<const float4*>(&cw[(w * kRows + r) * C::CW_LD + c]);
                acc.x += v.x * sc; acc.y += v.y * sc; acc.z += v.z * sc; acc.w += v.w * sc;
            }
            *reinterpret_cast<float4*>(&a.ws_o[(pbase + r) * HD + c]) = acc;
            if (c == 0) *reinterpret_cast<float2*>(&a.ws_ml[(pbase + r) * 2]) = make_float2(M, L);
        }
        const size_t tbase = (size_t)kvh * ns * 16;
        // n_g (row, 4-column) groups over the 256 consumer threads: P threads per group, each merging
        // every P-th of `cnt` partials (slot of partial u: split first + u * stride) online (running
        // max, rescaled sum) with the (m, l) pairs and partial rows of kMB partials loaded together, so
        // the merge is a few L2 round trips; then the P partial merges meet in shared memory.  Threads
        // gi < n_g return the merged (M, L, unnormalised O) of their group.
        const int P = max(1, kCThreads / n_g);
        // partials per batch of loads: 8 within the 96 registers of the two-CTAs-per-SM kernels
        // (16 spilled), 16 for the one-CTA-per-SM q8_0 kernel
        constexpr int kMB = C::MIN_BLOCKS == 1 ? 16 : 8;
        float4* part_o = reinterpret_cast<float4*>(smem);                   // [P][n_g]
        float2* part_ml = reinterpret_cast<float2*>(smem + (size_t)P * n_g * sizeof(float4));
        auto merge_partials = [&](int first, int stride, int cnt, float& Mo, float& Lo, float4& Ao) {
            if (tid < P * n_g) {
                const int gi = tid % n_g, sub = tid / n_g;
                const int r = gi / G4, c = (gi % G4) * 4;
                float M = -INFINITY, L = 0.0f;
                float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
                for (int u0 = sub; u0 < cnt; u0 += kMB * P) {
                    float2 ml[kMB];
                    float4 v[kMB];
#pragma unroll
                    for (int uu = 0; uu < kMB; uu++) {
                        const int u = u0 + uu * P;
                        if (u < cnt) {
                            const size_t slot = tbase + (size_t)(first + u * stride) * 16 + r;
                            ml[uu] = __ldcg(reinterpret_cast<const float2*>(&a.ws_ml[slot * 2]));
                            v[uu] = __ldcg(reinterpret_cast<const float4*>(&a.ws_o[slot * HD + c]));
                        } else {
                            ml[uu] = make_float2(-INFINITY, 0.0f);
                        }
                    }
                    float mb = M;
#pragma unroll
                    for (int uu = 0; uu < kMB; uu++) mb = fmaxf(mb, ml[uu].x);
                    if (mb == -INFINITY) continue;
                    const float sc = M == -INFINITY ? 0.0f : fast_exp2(M - mb);
                    L *= sc;
                    acc.x *= sc; acc.y *= sc; acc.z *= sc; acc.w *= sc;
#pragma unroll
                    for (int uu = 0; uu < kMB; uu++) {
                        if (ml[uu].x != -INFINITY) {
                            const float w = fast_exp2(ml[uu].x - mb);
                            L += ml[uu].y * w;
                            acc.x += v[uu].x * w; acc.y += v[uu].y * w; acc.z += v[uu].z * w; acc.w += v[uu].w * w;
                        }
                    }
                    M = mb;
                }
                part_o[sub * n_g + gi] = acc;
                part_ml[sub * n_g + gi] = make_float2(M, L);
            }
            consumer_sync();
            if (tid < n_g) {
                const int gi = tid;
                float M = -INFINITY;
                for (int sub = 0; sub < P; sub++) M = fmaxf(M, part_ml[sub * n_g + gi].x);
                float L = 0.0f;
                float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
                for (int sub = 0; sub < P; sub++) {
                    const float2 ml = part_ml[sub * n_g + gi];
                    if (ml.x == -INFINITY) continue;
                    const float w = fast_exp2(ml.x - M);
                    const float4 v = part_o[sub * n_g + gi];
                    L += ml.y * w;
                    acc.x += v.x * w; acc.y += v.y * w; acc.z += v.z * w; acc.w += v.w * w;
                }
                Mo = M;
                Lo = L;
                Ao = acc;
            }
        };
        float Mf = -INFINITY, Lf = 0.0f;
        float4 Af = make_float4(0.f, 0.f, 0.f, 0.f);
        const int n_grp = (ns + kMergeGroup - 1) / kMergeGroup;
        if (a.merge_levels == 2 && n_grp > 1) {
            // ---- level 1: the last split of this group of kMergeGroup merges the group
            const int grp = split / kMergeGroup, g0 = grp * kMergeGroup, gn = min(kMergeGroup, ns - g0);
            int* gticket = &a.tickets[a.NKV + kvh * n_grp + grp];
            __threadfence();
            consumer_sync();
            if (tid == 0) *last = atomicAdd(gticket, 1) == gn - 1;
            consumer_sync();
            if (!*last) return;
            __threadfence();
            merge_partials(g0, 1, gn, Mf, Lf, Af);
            // the group's partial replaces its first split's, which only this CTA reads
            if (tid < n_g) {
                const int r = tid / G4, c = (tid % G4) * 4;
                const size_t slot = tbase + (size_t)g0 * 16 + r;
                *reinterpret_cast<float4*>(&a.ws_o[slot * HD + c]) = Af;
                if (c == 0) *reinterpret_cast<float2*>(&a.ws_ml[slot * 2]) = make_float2(Mf, Lf);
            }
            if (tid == 0) *gticket = 0;
            __threadfence();
            consumer_sync();   // every thread is done with part_o / part_ml and has published
            // ---- level 2: the last group merger of the kv head merges the groups
            if (tid == 0) *last = atomicAdd(&a.tickets[kvh], 1) == n_grp - 1;
            consumer_sync();
            if (!*last) return;
            __threadfence();
            merge_partials(0, kMergeGroup, n_grp, Mf, Lf, Af);
        } else {
            __threadfence();
            consumer_sync();
            if (tid == 0) *last = atomicAdd(&a.tickets[kvh], 1) == ns - 1;
            consumer_sync();
            if (!*last) return;
            __threadfence();
            merge_partials(0, 1, ns, Mf, Lf, Af);
        }
        if (tid < n_g) {
            const int r = tid / G4, c = (tid % G4) * 4;
            const float inv = Lf > 0.0f ? 1.0f / Lf : 0.0f;
            store_out4<kPeer>(a, kvh, r, c, make_float4(Af.x * inv, Af.y * inv, Af.z * inv, Af.w * inv));
        }
        if (tid == 0) a.tickets[kvh] = 0;
        signal_peers<kPeer>(a, 1, kCThreads);
        return;
    }

    // ---- split-K inside the cluster.  Each thread owns one (row, 4-column) group of this split's
    // partial and pushes it, with its row's (m, l), into the merger's shared memory (st.async,
    // counted on the merger's mbarrier); the split CTA then exits.  No split waits for another.
    const int gi = tid;
    if (gi >= n_g) return;
    const int r = gi / G4, c = (gi % G4) * 4;
    float M = -INFINITY, L = 0.0f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int w = 0; w < kCWarps; w++) M = fmaxf(M, cm[w * kRows + r]);
#pragma unroll
    for (int w = 0; w < kCWarps; w++) {
        const float mw = cm[w * kRows + r];
        const float sc = mw == -INFINITY ? 0.0f : fast_exp2(mw - M);
        L += cl[w * kRows + r] * sc;
        const float4 v = *reinterpret_cast<const float4*>(&cw[(w * kRows + r) * C::CW_LD + c]);
        acc.x += v.x * sc; acc.y += v.y * sc; acc.z += v.z * sc; acc.w += v.w * sc;
    }
    cluster_wait_acquire();   // the merger's barrier is initialised (arrived before the grid dependency)
    const float* slot_o = reinterpret_cast<const float*>(smem + C::PUSH_O);
    const float* slot_ml = reinterpret_cast<const float*>(smem + C::PUSH_ML);
    const uint32_t bar = dsmem_map(smem_u32(mdata), 0);
    st_async_f4(dsmem_map(smem_u32(&slot_o[(split * C::ROWS_MAX + r) * HD + c]), 0), acc, bar);
    if (c == 0) st_async_f2(dsmem_map(smem_u32(&slot_ml[(split * C::ROWS_MAX + r) * 2]), 0), make_float2(M, L), bar);
}

// kernel attributes, once per device
template <int HD, int KVT, bool kPeer = false, bool kDeep = false>
cudaError_t prepare_gqa() {
    static std::once_flag once[kMaxDevices];
    static cudaError_t status[kMaxDevices];
    return once_per_device(once, status, [] {
        cudaError_t e = cudaFuncSetAttribute(fa_decode_gqa_kernel<HD, KVT, kPeer, kDeep>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             GqaCfg<HD, KVT, kDeep>::SMEM + 1024);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(fa_decode_gqa_kernel<HD, KVT, kPeer, kDeep>,
                                     cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        return e;
    });
}

template <int HD, int KVT, bool kPeer, bool kDeep = false>
cudaError_t launch_gqa_t(const AttnArgs& a, const CUtensorMap* tk, const CUtensorMap* tv, cudaStream_t st) {
    cudaError_t e = prepare_gqa<HD, KVT, kPeer, kDeep>();
    if (e != cudaSuccess) return e;
    // a cluster merge adds one merger CTA per kv head (cluster = splits + 1)
    const int nx = a.cluster_merge ? a.n_splits + 1 : a.n_splits;
    dim3 grid((unsigned)nx, (unsigned)a.NKV, 1u);
    // load-balancing cluster placement: measured 6.44 -> 6.29 us per layer on config 2 (36-layer graph;
    // the spread policy measured the same as the default)
    return launch_pdl_cluster_ex(fa_decode_gqa_kernel<HD, KVT, kPeer, kDeep>, grid, dim3(kThreads),
                                 (size_t)GqaCfg<HD, KVT, kDeep>::SMEM + 1024, st, a.cluster_merge ? nx : 1, true, *tk,
                                 *tv, a);
}

template <int HD, int KVT>
int max_cluster_gqa() {
    static int v = -1;
    if (v < 0) {
        if (prepare_gqa<HD, KVT>() != cudaSuccess) {
            cudaGetLastError();
            v = 1;
            return v;
        }
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(16, 1, 1);
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = GqaCfg<HD, KVT>::SMEM + 1024;
        int n = 0;
        if (cudaOccupancyMaxPotentialClusterSize(&n, fa_decode_gqa_kernel<HD, KVT, false, false>, &cfg) != cudaSuccess) {
            cudaGetLastError();
            n = 1;
        }
        v = n < 1 ? 1 : (n > 16 ? 16 : n);
    }
    return v;
}

}  // namespace

bool decode_gqa_applies(int head_dim, int kv_type, int T, int G, int mask_mode) {
    if (mask_mode != SV_MASK_CAUSAL && mask_mode != SV_MASK_NONE) return false;
    if (kv_type == SV_TYPE_F16 && (head_dim == 64 || head_dim == 128)) return T * G <= kRows;
    if (kv_type == SV_TYPE_Q8_0 && head_dim == 256) return T * G <= GqaCfg<256, SV_TYPE_Q8_0>::ROWS_MAX;
    return false;
}

int decode_gqa_ctas_per_sm(int kv_type) { return kv_type == SV_TYPE_Q8_0 ? 1 : 2; }

int decode_gqa_max_cluster(int head_dim, int kv_type) {
    if (kv_type == SV_TYPE_Q8_0) return head_dim == 256 ? max_cluster_gqa<256, SV_TYPE_Q8_0>() : 1;
    return head_dim == 128 ? max_cluster_gqa<128, SV_TYPE_F16>()
                           : head_dim == 64 ? max_cluster_gqa<64, SV_TYPE_F16>() : 1;
}

cudaError_t launch_decode_gqa(const AttnArgs& a, int head_dim, int kv_type, const CUtensorMap* tk,
                              const CUtensorMap* tv, cudaStream_t st) {
    if (a.n_qtiles != 1 || a.T * a.G > kRows || (a.n_splits > 1 && !a.cluster_merge && !a.tickets))
        return cudaErrorInvalidValue;
    // the fused gather is a separate instantiation, so the plain decode carries none of its code
    if (kv_type == SV_TYPE_Q8_0)
        return head_dim == 256 ? launch_gqa_t<256, SV_TYPE_Q8_0, false>(a, tk, tv, st) : cudaErrorInvalidValue;
    const bool peer = a.n_peers > 0;
    switch (head_dim) {
        case 64: return peer ? launch_gqa_t<64, SV_TYPE_F16, true>(a, tk, tv, st)
                             : launch_gqa_t<64, SV_TYPE_F16, false>(a, tk, tv, st);
        case 128:
            if (a.deep_ring)   // long splits over few kv heads: one CTA per SM, 6-stage ring
                return peer ? launch_gqa_t<128, SV_TYPE_F16, true, true>(a, tk, tv, st)
                            : launch_gqa_t<128, SV_TYPE_F16, false, true>(a, tk, tv, st);
            return peer ? launch_gqa_t<128, SV_TYPE_F16, true>(a, tk, tv, st)
                        : launch_gqa_t<128, SV_TYPE_F16, false>(a, tk, tv, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace svkv
