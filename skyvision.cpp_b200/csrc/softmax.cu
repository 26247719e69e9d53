// softmax.cu - ggml_soft_max_ext(kq, mask, scale, max_bias = 0) of the
// mul_mat / soft_max / mul_mat attention fallback (gemma4_model.cpp:683-692,
// moondream.cpp:476-493): y[r] = softmax(x[r] * scale + mask[r % mask_rows]).
//
// One CTA per row; the row is read once into registers/shared memory, the max
// and the sum are block reductions (warp shuffles + one shared-memory step).
// HBM-bound: algorithmic bytes per row = 4*ne0 (x) + 2*ne0 (mask) + 4*ne0 (y).
#include "common.cuh"
#include "internal.hpp"

namespace svkv {

namespace {

constexpr int kSmThreads = 256;

__device__ __forceinline__ float block_reduce(float v, bool is_max, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float w = __shfl_xor_sync(0xffffffffu, v, o);
        v = is_max ? fmaxf(v, w) : v + w;
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        v = lane < kSmThreads / 32 ? red[lane] : (is_max ? -INFINITY : 0.0f);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float w = __shfl_xor_sync(0xffffffffu, v, o);
            v = is_max ? fmaxf(v, w) : v + w;
        }
        if (lane == 0) red[0] = v;
    }
    __syncthreads();
    return red[0];
}

__global__ void __launch_bounds__(kSmThreads)
soft_max_kernel(const float* __restrict__ x, int64_t ne0, size_t x_nb1, const uint16_t* __restrict__ mask,
                int64_t mask_rows, size_t mask_nb1, float scale, float* __restrict__ y, size_t y_nb1) {
    extern __shared__ float row[];
    __shared__ float red[kSmThreads / 32];
    const int64_t r = blockIdx.x;
    const float* xr = reinterpret_cast<const float*>(reinterpret_cast<const uint8_t*>(x) + (size_t)r * x_nb1);
    const uint16_t* mr = mask ? reinterpret_cast<const uint16_t*>(reinterpret_cast<const uint8_t*>(mask) +
                                                                  (size_t)(r % mask_rows) * mask_nb1)
                              : nullptr;
    float* yr = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(y) + (size_t)r * y_nb1);
    float mx = -INFINITY;
    for (int64_t i = threadIdx.x; i < ne0; i += kSmThreads) {
        float v = xr[i] * scale;
        if (mr) v += h2f(mr[i]);
        row[i] = v;
        mx = fmaxf(mx, v);
    }
    mx = block_reduce(mx, true, red);
    float sum = 0.0f;
    for (int64_t i = threadIdx.x; i < ne0; i += kSmThreads) {
        const float p = (mx == -INFINITY || row[i] == -INFINITY) ? 0.0f : expf(row[i] - mx);
        row[i] = p;
        sum += p;
    }
    sum = block_reduce(sum, false, red);
    const float inv = sum > 0.0f ? 1.0f / sum : 0.0f;
    for (int64_t i = threadIdx.x; i < ne0; i += kSmThreads) yr[i] = row[i] * inv;
}

}  // namespace

cudaError_t launch_soft_max(const float* x, int64_t ne0, int64_t n_rows, size_t x_nb1, const uint16_t* mask,
                            int64_t mask_rows, size_t mask_nb1, float scale, float* y, size_t y_nb1,
                            cudaStream_t st) {
    const size_t smem = (size_t)ne0 * sizeof(float);
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(soft_max_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    soft_max_kernel<<<(unsigned)n_rows, kSmThreads, smem, st>>>(x, ne0, x_nb1, mask, mask_rows, mask_nb1, scale, y,
                                                               y_nb1);
    return cudaGetLastError();
}

}  // namespace svkv
