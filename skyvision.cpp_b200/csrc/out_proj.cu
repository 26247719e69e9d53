// out_proj.cu - the step after the attention of a head-sharded session, fused with its reduction:
// the output projection of this rank's heads and the sum over ranks, in one kernel per layer.
//
// Reference step: attn = ggml_mul_mat(L.o, attn) (qwen3vl_model.cpp:664-667), with the attention
// rows of all heads.  Sharded by kv head, rank g holds the rows of its NH/G heads, i.e. columns
// [k_offset, k_offset + K_local) of the projection's input; the full output is the sum over ranks
// of x_g * W[:, k_offset : k_offset + K_local]^T (the row-parallel split of the projection).
//
// One kernel per rank and layer (every rank calls it):
//   1. each CTA computes a band of output columns d of this rank's partial y_g[t][d] (f16 weights,
//      f32 accumulation; one warp per column, 16-byte weight loads, x staged in shared memory), and
//      stores them into its own region [g] of slot `slot` on every rank (plain stores to peer memory
//      over NVLink, CUDA IPC mappings);
//   2. after a system-scope fence it adds 1 to every rank's arrival counter of the slot;
//   3. it waits (bounded, on the device) until its own counter holds the current epoch's arrivals of
//      every CTA of every rank, then sums its band over the ranks in rank order, so every rank ends
//      with bitwise the same output.
// The grid never exceeds one CTA per SM, so every CTA of a launch is resident while any of them
// waits, and the kernel lets the next launch start only when it exits.  A slot holds [world][T][D]
// f32 partials; a slot is rewritten only after every rank has summed it when consecutive layers use
// different slots (a rank reaches layer l + 2 only after every rank finished layer l).
//
// Bound: HBM on the weights (D x K_local x 2 bytes per launch) plus two NVLink latencies.
#include "common.cuh"
#include "internal.hpp"

namespace svkv {

namespace {

constexpr int kOpThreads = 512;
constexpr int kOpBatch = 16;     // 16-byte weight loads in flight per lane (a 4096-column row: all of them)
constexpr int kOpMaxT = 8;

struct OutProjArgs {
    const uint8_t* x;            // [T] rows of K_local elements (f16 or f32), row stride x_nb_t bytes
    int x_type;
    int64_t x_nb_t;
    int x_vec;                   // rows and stride 16-byte aligned: 16-byte loads
    const uint16_t* w;           // f16 [D][K_total]
    int K_total, k_offset, K_local, D, T;
    float* const* peer_out;      // this slot's region on every rank
    unsigned int* const* peer_ctr;
    int n_peers, rank;
    const unsigned int* my_ctr;
    const float* my_slot;        // this rank's slot: [world][T][D]
    const int32_t* epoch_dev;
    float* out;                  // [T][D] f32
    int* err;
};

__global__ void __launch_bounds__(kOpThreads) out_proj_peer_kernel(const __grid_constant__ OutProjArgs a) {
    extern __shared__ __align__(16) float xs[];   // [T][K_local]
    __shared__ int ok_flag;
    pdl_wait();
    const int T = a.T, KL = a.K_local;
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
    // this CTA's band of output columns
    const int d0 = (int)((int64_t)a.D * blockIdx.x / gridDim.x);
    const int d1 = (int)((int64_t)a.D * (blockIdx.x + 1) / gridDim.x);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int d = d0 + warp; d < d1; d += kOpThreads / 32) {
        const uint16_t* wr = a.w + (size_t)d * a.K_total + a.k_offset;
        float acc[kOpMaxT];
#pragma unroll
        for (int t = 0; t < kOpMaxT; t++) acc[t] = 0.0f;
        // kOpBatch weight loads per lane issued before any is used (one in flight per lane left the
        // kernel latency-bound at ~0.4 TB/s)
        for (int k0 = lane * 8; k0 < KL; k0 += 32 * 8 * kOpBatch) {
            uint4 u[kOpBatch];
#pragma unroll
            for (int c = 0; c < kOpBatch; c++) {
                const int k = k0 + c * 32 * 8;
                u[c] = k < KL ? __ldg(reinterpret_cast<const uint4*>(wr + k)) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int c = 0; c < kOpBatch; c++) {
                const int k = k0 + c * 32 * 8;
                if (k >= KL) break;
                const __half2* h = reinterpret_cast<const __half2*>(&u[c]);
                float wv[8];
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const float2 f = __half22float2(h[i]);
                    wv[2 * i] = f.x;
                    wv[2 * i + 1] = f.y;
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
        }
#pragma unroll
        for (int t = 0; t < kOpMaxT; t++) {
            if (t < T) {
                float s = acc[t];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
                if (lane < a.n_peers)   // lane p stores the value into rank p's slot, region [rank]
                    a.peer_out[lane][((size_t)a.rank * T + t) * a.D + d] = s;
            }
        }
    }
    // every rank counts this CTA once its stores are visible system-wide: the barrier makes every
    // thread's stores visible to thread 0, whose system-scope fence (cumulative) then orders them all
    // before its counter increments (one fence per CTA: a fence in every thread cost ~6 us a launch)
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        for (int p = 0; p < a.n_peers; p++) atomicAdd_system(a.peer_ctr[p], 1u);
        // wait (bounded) for every CTA of every rank of this epoch
        const unsigned int target = (unsigned int)(*reinterpret_cast<const volatile int*>(a.epoch_dev)) *
                                    (unsigned int)(a.n_peers * gridDim.x);
        const uint64_t t0 = globaltimer_ns();
        bool ok = true;
        while (*reinterpret_cast<const volatile unsigned int*>(a.my_ctr) < target) {
            __nanosleep(64);   // every CTA polls this line while the others' atomics update it: back off
            if (globaltimer_ns() - t0 > kWaitLimitNs) {
                if (a.err) atomicOr(a.err, ERRBIT_TIMEOUT);
                ok = false;
                break;
            }
        }
        __threadfence_system();
        ok_flag = ok;
    }
    __syncthreads();
    if (!ok_flag) return;
    // the band's sum over ranks, in rank order (identical on every rank)
    for (int i = threadIdx.x; i < T * (d1 - d0); i += blockDim.x) {
        const int t = i / (d1 - d0), d = d0 + i % (d1 - d0);
        float s = 0.0f;
        for (int r = 0; r < a.n_peers; r++) s += __ldcv(&a.my_slot[((size_t)r * T + t) * a.D + d]);
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
    a.peer_ctr = r.peer_ctr;
    a.n_peers = r.n_peers;
    a.rank = r.rank;
    a.my_ctr = r.my_ctr;
    a.my_slot = r.my_slot;
    a.epoch_dev = r.epoch_dev;
    a.out = r.out;
    a.err = r.err;
    const size_t smem = (size_t)r.T * r.K_local * sizeof(float);
    static cudaError_t attr = cudaFuncSetAttribute(out_proj_peer_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   kOpMaxT * 4096 * (int)sizeof(float));
    if (attr != cudaSuccess) return attr;
    const int n_ctas = std::min(kNumSMs, std::max(1, r.D / 8));
    // no programmatic early start of the next launch: this kernel's CTAs wait on one another
    return launch_pdl(out_proj_peer_kernel, dim3((unsigned)n_ctas), dim3(kOpThreads), smem, st, a);
}

int out_proj_max_t() { return kOpMaxT; }

}  // namespace svkv
