// append.cu - K/V append into the cache: ggml_set_rows and the ggml_cpy-into-view
// form (llm_block.hpp:227-233, qwen3vl_model.cpp:652-655, stage_buf.hpp:53-56).
//
// One CTA per (source row, tensor).  f16 rows move as 16-byte vectors; f32
// rows are rounded to f16 (RNE) 8 elements per thread and stored as 16 bytes;
// q8_0 rows are quantised 8 elements per thread (4 threads per 32-element
// block, amax by two shuffles), assembled in shared memory in block_q8_0 byte
// order and written back with 16-byte stores when the row allows it.
//
// Algorithmic bytes per row: src row + dst row (f16 cache: 2*ne0 + 2*ne0 for
// an f16 source; q8_0 cache: 2*ne0 + ne0/32*34).
#include "common.cuh"
#include "internal.hpp"

namespace svkv {

namespace {

constexpr int kAppendThreads = 128;

__device__ __forceinline__ float load_src(const uint8_t* s, int type, int64_t e) {
    if (type == SV_TYPE_F32) return reinterpret_cast<const float*>(s)[e];
    return __half2float(reinterpret_cast<const __half*>(s)[e]);
}

// 8 consecutive source elements as floats (vector loads when aligned)
__device__ __forceinline__ void load8(const uint8_t* s, int type, int64_t e, float* v, bool vec_ok) {
    if (type == SV_TYPE_F16) {
        if (vec_ok) {
            const uint4 u = *reinterpret_cast<const uint4*>(s + e * 2);
            const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float2 f = __half22float2(h[i]);
                v[2 * i] = f.x;
                v[2 * i + 1] = f.y;
            }
            return;
        }
    } else if (vec_ok) {
        const float4 a = *reinterpret_cast<const float4*>(s + e * 4);
        const float4 b = *reinterpret_cast<const float4*>(s + e * 4 + 16);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        return;
    }
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = load_src(s, type, e + i);
}

__global__ void __launch_bounds__(kAppendThreads)
set_rows_kernel(uint8_t* __restrict__ dst, int dst_type, int64_t ne0, int64_t dst_rows, size_t dst_nb1,
                const uint8_t* __restrict__ src, int src_type, size_t src_nb1,
                const int32_t* __restrict__ rows, int64_t base, int* err,
                size_t dst_tensor_stride, size_t src_tensor_stride, const int32_t* __restrict__ base_dev,
                int early_trigger) {
    extern __shared__ __align__(16) uint8_t qrow[];   // q8_0 row staging
    pdl_wait();
    // Letting the next launch start early is safe only when the host knows it will not read cache
    // rows before its own grid dependency resolves (cache handles track that; see run_attention);
    // otherwise dependents start when every row of this launch is written.
    if (early_trigger && threadIdx.x == 0) pdl_trigger();
    const int64_t i = blockIdx.x;
    const int z = blockIdx.y;
    const int64_t r = rows ? (int64_t)rows[i] : (base_dev ? (int64_t)__ldg(base_dev) : base) + i;
    if (r < 0 || r >= dst_rows) {
        if (threadIdx.x == 0 && err) atomicOr(err, ERRBIT_ROW_RANGE);
        return;
    }
    const uint8_t* s = src + (size_t)z * src_tensor_stride + (size_t)i * src_nb1;
    uint8_t* d = dst + (size_t)z * dst_tensor_stride + (size_t)r * dst_nb1;
    const int tid = threadIdx.x;

    if (dst_type == SV_TYPE_F16 && src_type == SV_TYPE_F16) {
        const size_t nbytes = (size_t)ne0 * 2;
        const bool vec = ((reinterpret_cast<uintptr_t>(s) | reinterpret_cast<uintptr_t>(d) | nbytes) & 15) == 0;
        if (vec) {
            const uint4* s4 = reinterpret_cast<const uint4*>(s);
            uint4* d4 = reinterpret_cast<uint4*>(d);
            for (size_t k = tid; k < nbytes / 16; k += kAppendThreads) d4[k] = s4[k];
        } else {
            const uint16_t* s2 = reinterpret_cast<const uint16_t*>(s);
            uint16_t* d2 = reinterpret_cast<uint16_t*>(d);
            for (int64_t k = tid; k < ne0; k += kAppendThreads) d2[k] = s2[k];
        }
        return;
    }
    const int es = src_type == SV_TYPE_F32 ? 4 : 2;

    if (dst_type == SV_TYPE_F16 || dst_type == SV_TYPE_F32) {
        const bool vec = (ne0 % 8 == 0) &&
                         ((reinterpret_cast<uintptr_t>(s) | reinterpret_cast<uintptr_t>(d) |
                           (uintptr_t)src_nb1) & 15) == 0;
        if (vec) {
            for (int64_t e = (int64_t)tid * 8; e < ne0; e += kAppendThreads * 8) {
                float v[8];
                load8(s, src_type, e, v, true);
                if (dst_type == SV_TYPE_F16) {
                    uint4 o;
                    o.x = pack_h2(v[0], v[1]);
                    o.y = pack_h2(v[2], v[3]);
                    o.z = pack_h2(v[4], v[5]);
                    o.w = pack_h2(v[6], v[7]);
                    *reinterpret_cast<uint4*>(d + e * 2) = o;
                } else {
                    float4* o = reinterpret_cast<float4*>(d + e * 4);
                    o[0] = make_float4(v[0], v[1], v[2], v[3]);
                    o[1] = make_float4(v[4], v[5], v[6], v[7]);
                }
            }
        } else {
            for (int64_t e = tid; e < ne0; e += kAppendThreads) {
                const float v = load_src(s, src_type, e);
                if (dst_type == SV_TYPE_F16) reinterpret_cast<__half*>(d)[e] = __float2half_rn(v);
                else reinterpret_cast<float*>(d)[e] = v;
            }
        }
        (void)es;
        return;
    }

    // ---- q8_0: ne0 % 32 == 0 (checked on the host)
    const int64_t nblk = ne0 / kQK8_0;
    const size_t qbytes = (size_t)nblk * kQ8_0Bytes;
    const bool vec_in = ((reinterpret_cast<uintptr_t>(s) & 15) == 0);
    for (int64_t e = (int64_t)tid * 8; e < ne0; e += kAppendThreads * 8) {
        float v[8];
        load8(s, src_type, e, v, vec_in);
        float amax = 0.0f;
#pragma unroll
        for (int k = 0; k < 8; k++) amax = fmaxf(amax, fabsf(v[k]));
        // the 4 lanes of one 32-element block are consecutive lanes (e = tid*8)
        // (lanes of a block are active together, so the active mask covers the xor partners)
        const unsigned am = __activemask();
        amax = fmaxf(amax, __shfl_xor_sync(am, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(am, amax, 2));
        const float dd = __fdiv_rn(amax, 127.0f);
        const float id = dd != 0.0f ? __fdiv_rn(1.0f, dd) : 0.0f;
        const int64_t b = e / kQK8_0;
        const int sub = (int)(e % kQK8_0);       // 0, 8, 16, 24
        uint8_t* ob = qrow + b * kQ8_0Bytes;
        if (sub == 0) {
            const __half hd = __float2half_rn(dd);
            *reinterpret_cast<__half*>(ob) = hd;   // 2-byte aligned (34*b)
        }
#pragma unroll
        for (int k = 0; k < 8; k += 2) {
            const int q0 = (int)roundf(__fmul_rn(v[k], id));
            const int q1 = (int)roundf(__fmul_rn(v[k + 1], id));
            const uint16_t pr = (uint16_t)((uint8_t)(int8_t)q0 | ((uint16_t)(uint8_t)(int8_t)q1 << 8));
            *reinterpret_cast<uint16_t*>(ob + 2 + sub + k) = pr;   // even offset
        }
    }
    __syncthreads();
    if ((((uintptr_t)d) & 15) == 0 && (qbytes & 15) == 0) {
        const uint4* s4 = reinterpret_cast<const uint4*>(qrow);
        uint4* d4 = reinterpret_cast<uint4*>(d);
        for (size_t k = tid; k < qbytes / 16; k += kAppendThreads) d4[k] = s4[k];
    } else {
        const uint16_t* s2 = reinterpret_cast<const uint16_t*>(qrow);
        uint16_t* d2 = reinterpret_cast<uint16_t*>(d);
        for (size_t k = tid; k < qbytes / 2; k += kAppendThreads) d2[k] = s2[k];
    }
}

__global__ void counter_add_kernel(int32_t* c, int n, int delta) {
    pdl_wait();
    for (int i = threadIdx.x; i < n; i += blockDim.x) c[i] += delta;
    pdl_trigger();
}

}  // namespace

cudaError_t launch_counter_add(int32_t* counter, int n, int delta, cudaStream_t st) {
    return launch_pdl(counter_add_kernel, dim3(1), dim3(n < 256 ? ((n + 31) / 32) * 32 : 256), 0, st, counter, n,
                      delta);
}

cudaError_t launch_set_rows(void* dst, int dst_type, int64_t ne0, int64_t dst_rows, size_t dst_nb1,
                            const void* src, int src_type, size_t src_nb1, int64_t n_rows,
                            const int32_t* rows, int64_t base, int* err, int n_tensors,
                            size_t dst_tensor_stride, size_t src_tensor_stride, cudaStream_t st,
                            const int32_t* base_dev, bool early_trigger) {
    if (n_rows <= 0) return cudaSuccess;
    const size_t smem = dst_type == SV_TYPE_Q8_0 ? row_bytes_of(SV_TYPE_Q8_0, ne0) : 0;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(set_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return e;
    }
    dim3 grid((unsigned)n_rows, (unsigned)n_tensors);
    return launch_pdl(set_rows_kernel, grid, dim3(kAppendThreads), smem, st, static_cast<uint8_t*>(dst), dst_type, ne0,
                      dst_rows, dst_nb1, static_cast<const uint8_t*>(src), src_type, src_nb1, rows, base, err,
                      dst_tensor_stride, src_tensor_stride, base_dev, early_trigger ? 1 : 0);
}

}  // namespace svkv
