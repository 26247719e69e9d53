// compact.cu - in-HBM, order-preserving compaction of a KV cache after window
// eviction (the row move of kv_shift_rows, moss_vl_model.cpp:264-291, driven by
// the qwen3vl kept-set rule, qwen3vl_model.cpp:1110-1124).
//
// The host passes the segment table {src, n_rows, keep} by value.  Each CTA
// rebuilds the exclusive prefix sum of kept segment lengths in shared memory,
// which gives every kept row j its source row (segment src + offset) and its
// destination dst_base + j, and copies whole rows with 16-byte vectors for
// every layer's K and V (blockIdx.y = tensor).
//
// In place is safe wave by wave: kept row j moves down by shift_j = src_j -
// dst_j, and shift never decreases with j.  A wave of rows [j, j + shift_j)
// writes only destinations below src_j, i.e. rows no later read touches, so
// all of its rows can be copied concurrently; consecutive waves are ordered by
// the stream.  When the shifts are so small that this needs many waves, the
// rows go through a one-tensor scratch buffer instead (gather, then copy back).
//
// Algorithmic bytes: 2 * moved rows * row_bytes * 2 * n_layer (read + write).
#include <algorithm>

#include "common.cuh"
#include "internal.hpp"

namespace svkv {

namespace {

constexpr int kMaxSegs = 1024;
constexpr int kCompactThreads = 256;
constexpr int kRowsPerCta = 8;
constexpr int kCopyUnroll = 4;
constexpr int kMaxWaves = 16;

struct CompactParams {
    uint8_t* src_base;        // tensor 0 of the source
    uint8_t* dst_base_ptr;    // tensor 0 of the destination
    size_t src_tstride, dst_tstride;   // bytes between tensors (0 for the scratch)
    size_t row_bytes;
    int src_from_segments;    // 1: source row from the segment map, 0: row (j - j_lo)
    int dst_from_base;        // 1: destination row dst_base + j, 0: row (j - j_lo)
    int dst_base;
    int j_lo, j_hi;           // kept-row index range of this launch
    int n_segs;
    int64_t n_rows_cache;     // bounds for the source rows
    int* err;
    sv_segment segs[kMaxSegs];
};

__global__ void __launch_bounds__(kCompactThreads) compact_kernel(const __grid_constant__ CompactParams p) {
    __shared__ int kept_off[kMaxSegs + 1];   // exclusive prefix of kept lengths
    __shared__ int warp_tot[kCompactThreads / 32];
    const int tid = threadIdx.x;

    // block-wide exclusive scan over kept lengths (4 segments per thread)
    constexpr int PER = kMaxSegs / kCompactThreads;
    int local[PER];
    int sum = 0;
#pragma unroll
    for (int k = 0; k < PER; k++) {
        const int s = tid * PER + k;
        const int len = (s < p.n_segs && p.segs[s].keep) ? p.segs[s].n_rows : 0;
        local[k] = sum;
        sum += len;
    }
    // inclusive warp scan of per-thread sums
    const int lane = tid & 31, w = tid >> 5;
    int inc = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += v;
    }
    if (lane == 31) warp_tot[w] = inc;
    __syncthreads();
    int wbase = 0;
    for (int k = 0; k < w; k++) wbase += warp_tot[k];
    const int excl = wbase + inc - sum;
#pragma unroll
    for (int k = 0; k < PER; k++) kept_off[tid * PER + k] = excl + local[k];
    if (tid == kCompactThreads - 1) kept_off[kMaxSegs] = excl + sum;
    __syncthreads();

    const int z = blockIdx.y;
    const uint8_t* src_t = p.src_base + (size_t)z * p.src_tstride;
    uint8_t* dst_t = p.dst_base_ptr + (size_t)z * p.dst_tstride;
    const int j0 = p.j_lo + blockIdx.x * kRowsPerCta;
    const int vec_per_row = (int)(p.row_bytes / 16);
    // the CTA's rows first (one thread per row), then every thread moves kCopyUnroll vectors with all
    // of its loads issued before its stores: rows one after another left one memory round trip per
    // row and half the threads idle on 2 KB rows.  Rows of one wave never overlap (see above), so
    // the order inside a launch is free.
    __shared__ int64_t srow[kRowsPerCta], drow[kRowsPerCta];
    if (tid < kRowsPerCta) {
        const int j = j0 + tid;
        int64_t src_row = -1, dst_row = -1;
        if (j < p.j_hi) {
            if (p.src_from_segments) {
                // last segment whose kept offset <= j among kept segments
                int lo = 0, hi = p.n_segs - 1;
                while (lo < hi) {
                    const int mid = (lo + hi + 1) >> 1;
                    if (kept_off[mid] <= j) lo = mid; else hi = mid - 1;
                }
                // skip zero-length / dropped segments that share the same offset
                while (lo < p.n_segs - 1 && !(p.segs[lo].keep && kept_off[lo] + p.segs[lo].n_rows > j)) lo++;
                src_row = (int64_t)p.segs[lo].src + (j - kept_off[lo]);
                if (src_row < 0 || src_row >= p.n_rows_cache) {
                    if (p.err) atomicOr(p.err, ERRBIT_SEGMENT);
                    src_row = -1;
                }
            } else {
                src_row = j - p.j_lo;
            }
            if (src_row >= 0) dst_row = p.dst_from_base ? (int64_t)p.dst_base + j : (int64_t)(j - p.j_lo);
        }
        srow[tid] = src_row;
        drow[tid] = dst_row;
    }
    __syncthreads();
    const int total = kRowsPerCta * vec_per_row;
    for (int base = tid; base < total; base += kCompactThreads * kCopyUnroll) {
        uint4 v[kCopyUnroll];
        int64_t dst_off[kCopyUnroll];
#pragma unroll
        for (int u = 0; u < kCopyUnroll; u++) {
            const int idx = base + u * kCompactThreads;
            dst_off[u] = -1;
            if (idx < total) {
                const int r = idx / vec_per_row, k = idx % vec_per_row;
                if (srow[r] >= 0) {
                    v[u] = reinterpret_cast<const uint4*>(src_t + (size_t)srow[r] * p.row_bytes)[k];
                    dst_off[u] = (int64_t)drow[r] * (int64_t)p.row_bytes + (int64_t)k * 16;
                }
            }
        }
#pragma unroll
        for (int u = 0; u < kCopyUnroll; u++)
            if (dst_off[u] >= 0) *reinterpret_cast<uint4*>(dst_t + dst_off[u]) = v[u];
    }
}

}  // namespace

cudaError_t launch_compact(KvHandle* kv, const int32_t*, const sv_segment* segs, int n_segs, int dst_base,
                           cudaStream_t st) {
    // kept rows in order with their shifts (host side: the table is host data)
    std::vector<int64_t> src_rows;
    for (int s = 0; s < n_segs; s++)
        if (segs[s].keep)
            for (int r = 0; r < segs[s].n_rows; r++) src_rows.push_back((int64_t)segs[s].src + r);
    const int K = (int)src_rows.size();
    int first = 0;
    while (first < K && src_rows[first] == dst_base + first) first++;   // rows already in place
    if (first >= K) return cudaSuccess;

    CompactParams p{};
    p.row_bytes = kv->row_bytes;
    p.dst_base = dst_base;
    p.n_segs = n_segs;
    p.n_rows_cache = kv->n_ctx;
    p.err = kv->err;
    for (int s = 0; s < n_segs; s++) p.segs[s] = segs[s];

    // wave plan
    std::vector<std::pair<int, int>> waves;
    for (int j = first; j < K;) {
        const int64_t shift = src_rows[j] - (dst_base + j);
        const int n = (int)std::min<int64_t>(std::max<int64_t>(shift, 1), K - j);
        waves.push_back({j, j + n});
        j += n;
    }
    const int ntensor = 2 * kv->n_layer;
    if ((int)waves.size() <= kMaxWaves) {
        p.src_base = kv->buf;
        p.dst_base_ptr = kv->buf;
        p.src_tstride = p.dst_tstride = kv->tensor_bytes;
        p.src_from_segments = 1;
        p.dst_from_base = 1;
        for (auto& w : waves) {
            p.j_lo = w.first;
            p.j_hi = w.second;
            dim3 grid((unsigned)ceil_div(w.second - w.first, kRowsPerCta), (unsigned)ntensor);
            compact_kernel<<<grid, kCompactThreads, 0, st>>>(p);
            cudaError_t e = cudaGetLastError();
            if (e != cudaSuccess) return e;
        }
        return cudaSuccess;
    }
    // many tiny shifts: per tensor, gather rows [first, K) into the scratch, then copy back
    p.j_lo = first;
    p.j_hi = K;
    for (int t = 0; t < ntensor; t++) {
        uint8_t* tensor = kv->buf + (size_t)t * kv->tensor_bytes;
        dim3 grid((unsigned)ceil_div(K - first, kRowsPerCta), 1);
        p.src_base = tensor; p.src_tstride = 0; p.src_from_segments = 1;
        p.dst_base_ptr = kv->scratch; p.dst_tstride = 0; p.dst_from_base = 0;
        compact_kernel<<<grid, kCompactThreads, 0, st>>>(p);
        p.src_base = kv->scratch; p.src_from_segments = 0;
        p.dst_base_ptr = tensor; p.dst_from_base = 1;
        compact_kernel<<<grid, kCompactThreads, 0, st>>>(p);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace svkv
