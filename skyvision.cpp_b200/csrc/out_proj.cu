// out_proj.cu - the step after the attention of a head-sharded session, fused with its reduction:
// the output projection of this rank's heads and the sum over ranks, in one kernel per layer.
//
// Reference step: attn = ggml_mul_mat(L.o, attn) (qwen3vl_model.cpp:664-667), with the attention
// rows of all heads.  Sharded by kv head, rank g holds the rows of its NH/G heads, i.e. columns
// [k_offset, k_offset + K_local) of the projection's input; the full output is the sum over ranks
// of x_g * W[:, k_offset : k_offset + K_local]^T (the row-parallel split of the projection).
//
// One kernel per rank and layer (every rank calls it with the same D, so CTA b covers the same band
// of output columns on every rank):
//   1. before the grid dependency, one thread issues the band's weight rows (this rank's column
//      slice of each, contiguous) as untiled bulk copies into shared memory, one mbarrier per row:
//      the weights are model constants that no kernel of the stream writes, so the whole band is in
//      flight from the first instant and the launch is one HBM read of the weights;
//   2. after the dependency it stages x in shared memory; each warp takes a row as soon as that
//      row has landed, computes y_g[t][d] (f32 accumulation) and stores it into its own region [g]
//      of slot `slot` on every rank (plain stores to peer memory over NVLink, CUDA IPC mappings);
//   3. a system-scope release add counts the band on every rank's band counter (the CTA barrier
//      before it orders every thread's stores), then the CTA waits (bounded, acquire loads) until its
//      own band counter holds the current epoch's arrivals of every rank and sums the band over the
//      ranks in rank order, so every rank ends with bitwise the same output.
// A CTA waits only for the same band of the other ranks.  The grid never exceeds one CTA per SM,
// so every CTA of a launch is resident while any of them waits; the next launch is let in once the
// whole grid runs (its CTAs take SMs as these exit and issue their own weight rows meanwhile).
// A slot holds [world][T][D] f32 partials; a slot is rewritten only after every rank has summed it
// when consecutive layers use different slots (a rank reaches layer l + 2 only after every rank
// finished layer l).
// Slots with room for 8 bytes per partial take the words form instead of steps 2-3's counters: each
// partial goes to the other ranks as one 64-bit store of (value, epoch), single-copy atomic, and the
// summing CTA polls exactly the words of its band until they carry this step's epoch -- no
// system-scope release, no counter round trip (2 GPUs: 14.8 -> 7.35 us per layer).
//
// Bound: HBM on the weights (D x K_local x 2 bytes per launch) plus two NVLink latencies.
#include "common.cuh"
#include "internal.hpp"

namespace svkv {

namespace {

constexpr int kOpThreads = 512;
constexpr int kOpWarps = kOpThreads / 32;
constexpr int kOpMaxT = 8;
constexpr int kOpMaxRows = 32;                 // weight rows staged per round (one mbarrier each)
constexpr int kOpSmemBytes = 196 * 1024;       // x (f32) + the staged weight rows
constexpr int kOpMaxBand = 128;                // output columns per CTA (D <= 148 x 128)

struct OutProjArgs {
    const uint8_t* x;            // [T] rows of K_local elements (f16 or f32), row stride x_nb_t bytes
    int x_type;
    int64_t x_nb_t;
    int x_vec;                   // rows and stride 16-byte aligned: 16-byte loads
    const uint16_t* w;           // f16 [D][K_total]
    int K_total, k_offset, K_local, D, T;
    float* const* peer_out;      // this slot's region on every rank
    unsigned int* const* peer_bctr;   // this slot's band counters on every rank
    int n_peers, rank;
    const unsigned int* my_bctr;
    const float* my_slot;        // this rank's slot: [world][T][D]
    const int32_t* epoch_dev;
    float* out;                  // [T][D] f32
    int* err;
    int rows_per_round;          // weight rows one round stages (<= kOpMaxRows)
    int ll;                      // slots of 64-bit (value, epoch) words: no counters, no fences
    uint32_t w_off;              // byte offset of the staged weight rows in dynamic shared memory
};

__global__ void __launch_bounds__(kOpThreads, 1) out_proj_peer_kernel(const __grid_constant__ OutProjArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t full[kOpMaxRows];
    __shared__ int ok_flag;
    __shared__ float own[kOpMaxBand][kOpMaxT];     // this rank's partials of the band
    __shared__ float* s_out[8];                    // the slot's region on every rank
    __shared__ unsigned int* s_bctr[8];            // the slot's band counters on every rank
    __shared__ unsigned int s_target;              // this epoch's arrival count of a band
    float* xs = reinterpret_cast<float*>(smem);   // [T][K_local]
    uint8_t* ws = smem + a.w_off;                  // [rows_per_round][K_local] f16
    const int T = a.T, KL = a.K_local, RR = a.rows_per_round;
    const uint32_t row_bytes = (uint32_t)KL * 2;
    // this CTA's band of output columns
    const int d0 = (int)((int64_t)a.D * blockIdx.x / gridDim.x);
    const int d1 = (int)((int64_t)a.D * (blockIdx.x + 1) / gridDim.x);
    const int nb = d1 - d0;
    const int n_rounds = (nb + RR - 1) / RR;
    if (threadIdx.x == 0) {
        for (int i = 0; i < RR; i++) mbar_init(&full[i], 1);
        fence_barrier_init();
        ok_flag = 1;
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // warp 0 issues a round's rows, one row per lane (RR <= 32)
    auto issue = [&](int round) {
        const int r0 = round * RR, n = min(RR, nb - r0);
        if (lane < n) {
            mbar_arrive_expect_tx(&full[lane], row_bytes);
            bulk_load_1d(ws + (size_t)lane * row_bytes, a.w + (size_t)(d0 + r0 + lane) * a.K_total + a.k_offset,
                         row_bytes, &full[lane]);
        }
    };
    if (warp == 0) issue(0);   // before the dependency: model constants only
    if (warp == 1) {
        // x may still be written by the previous kernel: an L2 prefetch is only a hint, so the loads
        // after the dependency find its lines in L2 instead of queueing behind the weight stream
        const int es = a.x_type == SV_TYPE_F32 ? 4 : 2;
        const int lines = (KL * es + 127) / 128;
        for (int i = lane; i < T * lines; i += 32)
            prefetch_l2(a.x + (size_t)(i / lines) * a.x_nb_t + (size_t)(i % lines) * 128);
    } else if (warp == 2 && lane < a.n_peers) {
        // the slot's pointer tables (written once, when the peers were imported): read now, so no
        // global round trip sits between the last row and the exchange
        s_out[lane] = a.peer_out[lane];
        s_bctr[lane] = a.peer_bctr[lane];
    }
    // the next launch may be scheduled now: this grid is resident (every CTA got here), and what a
    // launch does before its dependency wait reads only model constants
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x == 64) {   // the epoch (advanced by the kernel that ends each step), read with x
        const unsigned int ep = (unsigned int)(*reinterpret_cast<const volatile int*>(a.epoch_dev));
        s_target = a.ll ? ep : ep * (unsigned int)a.n_peers;
    }
    if (a.x_vec) {   // 8 elements per 16-byte load (K_local is a multiple of 8, so no load spans two rows)
        for (int i = threadIdx.x; i < T * KL / 8; i += blockDim.x) {
            const int e = i * 8, t = e / KL, k = e % KL;
            const uint8_t* row = a.x + (size_t)t * a.x_nb_t;
            float4 f0, f1;
            if (a.x_type == SV_TYPE_F32) {
                f0 = *reinterpret_cast<const float4*>(row + (size_t)k * 4);
                f1 = *reinterpret_cast<const float4*>(row + (size_t)k * 4 + 16);
            } else {
                const uint4 u = *reinterpret_cast<const uint4*>(row + (size_t)k * 2);
                const __half2* h = reinterpret_cast<const __half2*>(&u);
                const float2 a0 = __half22float2(h[0]), a1 = __half22float2(h[1]);
                const float2 a2 = __half22float2(h[2]), a3 = __half22float2(h[3]);
                f0 = make_float4(a0.x, a0.y, a1.x, a1.y);
                f1 = make_float4(a2.x, a2.y, a3.x, a3.y);
            }
            *reinterpret_cast<float4*>(&xs[e]) = f0;
            *reinterpret_cast<float4*>(&xs[e + 4]) = f1;
        }
    } else {
        for (int i = threadIdx.x; i < T * KL; i += blockDim.x) {
            const int t = i / KL, k = i % KL;
            const uint8_t* row = a.x + (size_t)t * a.x_nb_t;
            xs[i] = a.x_type == SV_TYPE_F32 ? reinterpret_cast<const float*>(row)[k]
                                            : __half2float(reinterpret_cast<const __half*>(row)[k]);
        }
    }
    __syncthreads();
    int last_issued = 0;   // the round whose copies were issued last (uniform across the CTA)
    for (int round = 0; round < n_rounds; round++) {
        if (round > 0) {
            __syncthreads();   // every warp is done with the previous round's rows
            if (!ok_flag) break;   // a row of that round never landed: issue nothing more
            if (warp == 0) issue(round);
            last_issued = round;
        }
        const int r0 = round * RR, n = min(RR, nb - r0);
        for (int i = warp; i < n; i += kOpWarps) {
            if (!mbar_wait(&full[i], round & 1, a.err)) {
                ok_flag = 0;
                break;
            }
            const uint8_t* wr = ws + (size_t)i * row_bytes;
            float acc[kOpMaxT];
#pragma unroll
            for (int t = 0; t < kOpMaxT; t++) acc[t] = 0.0f;
            for (int k = lane * 8; k < KL; k += 32 * 8) {
                const uint4 u = *reinterpret_cast<const uint4*>(wr + (size_t)k * 2);
                const __half2* h = reinterpret_cast<const __half2*>(&u);
                float wv[8];
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const float2 f = __half22float2(h[j]);
                    wv[2 * j] = f.x;
                    wv[2 * j + 1] = f.y;
                }
#pragma unroll
                for (int t = 0; t < kOpMaxT; t++) {
                    if (t < T) {
                        const float4 x0 = *reinterpret_cast<const float4*>(&xs[t * KL + k]);
                        const float4 x1 = *reinterpret_cast<const float4*>(&xs[t * KL + k + 4]);
                        float s = acc[t];
                        s = fmaf(wv[0], x0.x, s); s = fmaf(wv[1], x0.y, s); s = fmaf(wv[2], x0.z, s); s = fmaf(wv[3], x0.w, s);
                        s = fmaf(wv[4], x1.x, s); s = fmaf(wv[5], x1.y, s); s = fmaf(wv[6], x1.z, s); s = fmaf(wv[7], x1.w, s);
                        acc[t] = s;
                    }
                }
            }
            const int d = d0 + r0 + i;
#pragma unroll
            for (int t = 0; t < kOpMaxT; t++) {
                if (t < T) {
                    float s = acc[t];
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
                    if (lane == 0) own[d - d0][t] = s;
                    // lane p stores the value into rank p's slot, region [rank] (its own rank's term comes
                    // from shared memory); with 64-bit words the value travels with the step's epoch
                    if (lane < a.n_peers && lane != a.rank) {
                        const size_t idx = ((size_t)a.rank * T + t) * a.D + d;
                        if (a.ll)
                            st_relaxed_sys_u64(reinterpret_cast<unsigned long long*>(s_out[lane]) + idx,
                                               ((unsigned long long)s_target << 32) | __float_as_uint(s));
                        else
                            s_out[lane][idx] = s;
                    }
                }
            }
        }
    }
    // count the band on every rank once its stores are visible to that rank: the barrier orders every
    // thread's stores before thread 0's release add (release is cumulative).  System scope across
    // GPUs; with one rank nothing outside this GPU reads the slot, and GPU scope is the cheaper
    // release (measured ~0.7 vs ~2.5 us)
    __syncthreads();
    if (a.ll) {
        // ---- 64-bit words: every partial of the other ranks is valid once its word carries this
        // step's epoch (an older word is a previous step's); poll each, bounded, and sum in rank order.
        // A rank whose weight row never landed stores nothing, so the peers' polls expire and report it.
        if (!ok_flag) return;
        const unsigned int ep = s_target;
        const unsigned long long* slot = reinterpret_cast<const unsigned long long*>(a.my_slot);
        for (int i = threadIdx.x; i < T * nb; i += blockDim.x) {
            const int t = i / nb, d = d0 + i % nb;
            float s = 0.0f;
            bool ok = true;
            for (int r = 0; r < a.n_peers; r++) {
                if (r == a.rank) {
                    s += own[d - d0][t];
                    continue;
                }
                const unsigned long long* wp = slot + ((size_t)r * T + t) * a.D + d;
                unsigned long long v = ld_relaxed_sys_u64(wp);
                if ((unsigned int)(v >> 32) != ep) {
                    const uint64_t t0 = globaltimer_ns();
                    while ((unsigned int)((v = ld_relaxed_sys_u64(wp)) >> 32) != ep) {
                        if (globaltimer_ns() - t0 > kWaitLimitNs) {
                            if (a.err) atomicOr(a.err, ERRBIT_TIMEOUT);
                            ok = false;
                            break;
                        }
                    }
                }
                if (!ok) break;
                s += __uint_as_float((unsigned int)v);
            }
            if (ok) a.out[(size_t)t * a.D + d] = s;
        }
        return;
    }
    if (threadIdx.x == 0) {
        if (!ok_flag) {
            // a row never landed (the error bit is set): before the CTA leaves, wait (bounded) for the
            // last round's copies that may still be in flight into its shared memory.  The band is not
            // counted on any rank: this rank's partials in the peers' slots are stale, so the peers'
            // bounded waits expire and they report the timeout too instead of summing stale values.
            // The counters then stay one arrival short, so every later epoch of this peer group times
            // out as well: the group has to be recreated.
            const int n_last = min(RR, nb - last_issued * RR);
            for (int i = 0; i < n_last; i++) mbar_wait_limit(&full[i], last_issued & 1, nullptr, kWaitLimitNs);
        } else {
            const bool sys = a.n_peers > 1;
            for (int p = 0; p < a.n_peers; p++) {
                if (sys) red_add_release_sys(s_bctr[p] + blockIdx.x, 1u);
                else red_add_release_gpu(s_bctr[p] + blockIdx.x, 1u);
            }
            // wait (bounded) for this band of every rank of this epoch
            const unsigned int target = s_target;
            const uint64_t t0 = globaltimer_ns();
            while ((sys ? ld_acquire_sys(a.my_bctr + blockIdx.x) : ld_acquire_gpu(a.my_bctr + blockIdx.x)) < target) {
                if (globaltimer_ns() - t0 > kWaitLimitNs) {
                    if (a.err) atomicOr(a.err, ERRBIT_TIMEOUT);
                    ok_flag = 0;
                    break;
                }
            }
        }
    }
    __syncthreads();
    if (!ok_flag) return;
    // the band's sum over ranks, in rank order (identical on every rank: this rank's own term is the
    // value it stored into every slot, taken from shared memory)
    for (int i = threadIdx.x; i < T * nb; i += blockDim.x) {
        const int t = i / nb, d = d0 + i % nb;
        float s = 0.0f;
        for (int r = 0; r < a.n_peers; r++)
            s += r == a.rank ? own[d - d0][t] : __ldcv(&a.my_slot[((size_t)r * T + t) * a.D + d]);
        a.out[(size_t)t * a.D + d] = s;
    }
}

}  // namespace

cudaError_t launch_out_proj_peer(const OutProjLaunch& r, cudaStream_t st) {
    OutProjArgs a{};
    a.x = static_cast<const uint8_t*>(r.x);
    a.x_type = r.x_type;
    a.x_nb_t = r.x_nb_t;
    a.x_vec = ((reinterpret_cast<uintptr_t>(r.x) | (uintptr_t)r.x_nb_t) & 15) == 0;
    a.w = r.w;
    a.K_total = r.K_total;
    a.k_offset = r.k_offset;
    a.K_local = r.K_local;
    a.D = r.D;
    a.T = r.T;
    a.peer_out = r.peer_out;
    a.peer_bctr = r.peer_bctr;
    a.n_peers = r.n_peers;
    a.rank = r.rank;
    a.my_bctr = r.my_bctr;
    a.my_slot = r.my_slot;
    a.epoch_dev = r.epoch_dev;
    a.out = r.out;
    a.err = r.err;
    a.ll = r.ll;
    static std::once_flag once[kMaxDevices];   // the attribute, once per device
    static cudaError_t status[kMaxDevices];
    const cudaError_t attr = once_per_device(once, status, [] {
        return cudaFuncSetAttribute(out_proj_peer_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kOpSmemBytes);
    });
    if (attr != cudaSuccess) return attr;
    // one CTA per SM at most: a CTA waits for the same band of every rank, so all of them must be
    // resident at once (the device's own SM count; a share of the SMs under MPS can still time out)
    const int n_ctas = std::min(std::min(device_sm_count(), kPeerBands), std::max(1, r.D / 8));
    const int band_max = (r.D + n_ctas - 1) / n_ctas;
    // x as f32 (T x K_local x 4 <= 128 KB), then as many whole weight rows as the rest holds
    a.w_off = (uint32_t)(((size_t)r.T * r.K_local * sizeof(float) + 127) & ~(size_t)127);
    const size_t row_bytes = (size_t)r.K_local * 2;
    const size_t fit = ((size_t)kOpSmemBytes - a.w_off) / row_bytes;
    a.rows_per_round = (int)std::min(fit, (size_t)std::min(kOpMaxRows, band_max));
    const size_t smem = a.w_off + (size_t)a.rows_per_round * row_bytes;
    return launch_pdl(out_proj_peer_kernel, dim3((unsigned)n_ctas), dim3(kOpThreads), smem, st, a);
}

int out_proj_max_t() { return kOpMaxT; }
int out_proj_max_d() { return kNumSMs * kOpMaxBand; }

}  // namespace svkv

