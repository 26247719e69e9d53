// capi.cpp - the extern "C" boundary (include/svkv.h): argument checking,
// KV-store ownership, tensor maps, and the choice of kernel / split plan.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "internal.hpp"

using namespace svkv;

namespace svkv {

namespace {

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

PFN_cuTensorMapEncodeTiled_v12000 encoder() {
    std::call_once(g_encode_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    return g_encode;
}

}  // namespace

bool encode_tmap_2d(CUtensorMap* m, const void* base, CUtensorMapDataType dt, uint64_t dim0, uint64_t dim1,
                    uint64_t stride1_bytes, uint32_t box0, uint32_t box1, CUtensorMapSwizzle swz) {
    auto enc = encoder();
    if (!enc) return false;
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (stride1_bytes & 15)) return false;
    const cuuint64_t dims[2] = {dim0, dim1};
    const cuuint64_t strides[1] = {stride1_bytes};
    const cuuint32_t box[2] = {box0, box1};
    const cuuint32_t es[2] = {1, 1};
    return enc(m, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool encode_tmap_3d(CUtensorMap* m, const void* base, CUtensorMapDataType dt, const uint64_t dims_in[3],
                    const uint64_t strides_bytes[2], const uint32_t box_in[3], CUtensorMapSwizzle swz) {
    auto enc = encoder();
    if (!enc) return false;
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (strides_bytes[0] & 15) || (strides_bytes[1] & 15)) return false;
    const cuuint64_t dims[3] = {dims_in[0], dims_in[1], dims_in[2]};
    const cuuint64_t strides[2] = {strides_bytes[0], strides_bytes[1]};
    const cuuint32_t box[3] = {box_in[0], box_in[1], box_in[2]};
    const cuuint32_t es[3] = {1, 1, 1};
    return enc(m, dt, 3, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

namespace {

constexpr size_t kDefaultWsBytes = 64ull << 20;   // split-K partials per handle
constexpr int kMaxTickets = 1 << 16;
constexpr int kMaxSplits = 256;

struct DeviceGuard {
    int prev = -1;
    bool ok = true;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) { ok = false; return; }
        if (prev != dev && cudaSetDevice(dev) != cudaSuccess) ok = false;
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

int cuda_status(cudaError_t e) {
    if (e == cudaSuccess) return SV_OK;
    fprintf(stderr, "svkv: CUDA error %s\n", cudaGetErrorString(e));
    return SV_ERR_CUDA;
}

// --------------------------------------------------------------- split plan
struct Plan {
    int qpt = 1, n_qtiles = 1, chunk = 64, n_splits = 1;
};

// span: keys one query tile may touch; ws_floats: capacity for partials
Plan plan_decode(int T, int G, int NKV, int span, int head_dim, bool window, size_t ws_floats, int n_tickets,
                 int target_ctas, int max_splits = kMaxSplits) {
    Plan p;
    const int BK = decode_block_keys();
    p.qpt = window ? 1 : std::max(1, 16 / G);
    p.n_qtiles = ceil_div(T, p.qpt);
    const int base = NKV * p.n_qtiles;
    span = std::max(span, 1);
    int want = std::max(1, ceil_div(target_ctas, base));
    auto set_splits = [&](int w) {
        p.chunk = std::max(BK, ceil_div(ceil_div(span, w), BK) * BK);
        p.n_splits = ceil_div(span, p.chunk);
        if (p.n_splits > max_splits) {      // bounded merge tables in shared memory / cluster size
            p.chunk = std::max(BK, ceil_div(ceil_div(span, max_splits), BK) * BK);
            p.n_splits = ceil_div(span, p.chunk);
        }
    };
    set_splits(want);
    const size_t per = decode_partial_floats(head_dim);
    while (p.n_splits > 1 && ((size_t)base * p.n_splits * per > ws_floats || base > n_tickets)) {
        want = std::max(1, want / 2);
        set_splits(want);
        if (want == 1) break;
    }
    if (p.n_splits > 1 && ((size_t)base * p.n_splits * per > ws_floats || base > n_tickets)) {
        p.chunk = ceil_div(span, BK) * BK;
        p.n_splits = 1;
    }
    return p;
}

// CTAs the split plan aims for (SVKV_DEC_CTAS overrides it for tuning runs)
int target_ctas_default() {
    static const int v = [] {
        const char* e = getenv("SVKV_DEC_CTAS");
        const int n = e ? atoi(e) : 0;
        return n > 0 ? n : kNumSMs;
    }();
    return v;
}

}  // namespace
}  // namespace svkv

// ===================================================================== C ABI
extern "C" {

const char* sv_status_string(int status) {
    switch (status) {
        case SV_OK: return "ok";
        case SV_ERR_INVALID: return "invalid argument";
        case SV_ERR_UNSUPPORTED: return "unsupported shape or type";
        case SV_ERR_CUDA: return "CUDA error";
        case SV_ERR_NOMEM: return "device allocation failed";
        case SV_ERR_OVERFLOW: return "context overflow";
        case SV_ERR_WORKSPACE: return "workspace too small";
        case SV_ERR_DEVICE: return "device-side error flag raised";
        default: return "unknown status";
    }
}

int sv_version(void) { return 100; }

int sv_kv_create(int device, int n_layer, int n_kv_head, int head_dim, int n_ctx, int kv_type, sv_kv** out) {
    if (!out || n_layer <= 0 || n_kv_head <= 0 || head_dim <= 0 || n_ctx <= 0) return SV_ERR_INVALID;
    if (kv_type != SV_TYPE_F16 && kv_type != SV_TYPE_Q8_0) return SV_ERR_UNSUPPORTED;
    if (kv_type == SV_TYPE_Q8_0 && (head_dim % kQK8_0) != 0) return SV_ERR_UNSUPPORTED;
    *out = nullptr;
    DeviceGuard g(device);
    if (!g.ok) return SV_ERR_CUDA;
    sv_kv* kv = new sv_kv();
    kv->device = device;
    kv->n_layer = n_layer;
    kv->n_kv_head = n_kv_head;
    kv->head_dim = head_dim;
    kv->n_ctx = n_ctx;
    kv->type = kv_type;
    kv->row_bytes = row_bytes_of(kv_type, (int64_t)n_kv_head * head_dim);
    kv->tensor_bytes = (kv->row_bytes * (size_t)n_ctx + 255) / 256 * 256;
    const size_t total = kv->tensor_bytes * 2 * (size_t)n_layer;
    if (cudaMalloc(&kv->buf, total) != cudaSuccess) {
        fprintf(stderr, "KV cache allocation failed (%.2f GB)\n", (double)total / 1e9);
        cudaGetLastError();
        delete kv;
        return SV_ERR_NOMEM;
    }
    bool ok = cudaMemset(kv->buf, 0, total) == cudaSuccess;
    kv->ws_bytes = kDefaultWsBytes;
    kv->n_tickets = kMaxTickets;
    ok = ok && cudaMalloc(&kv->ws, kv->ws_bytes) == cudaSuccess;
    ok = ok && cudaMalloc(&kv->tickets, sizeof(int) * kv->n_tickets) == cudaSuccess;
    ok = ok && cudaMemset(kv->tickets, 0, sizeof(int) * kv->n_tickets) == cudaSuccess;
    ok = ok && cudaMalloc(&kv->err, sizeof(int)) == cudaSuccess;
    ok = ok && cudaMemset(kv->err, 0, sizeof(int)) == cudaSuccess;
    ok = ok && cudaMalloc(&kv->scratch, kv->tensor_bytes) == cudaSuccess;
    if (!ok) {
        cudaGetLastError();
        sv_kv_destroy(kv);
        return SV_ERR_NOMEM;
    }
    if (decode_supported(head_dim, kv_type, kv->row_bytes, n_kv_head)) {
        kv->tm_dec.resize(2 * n_layer);
        for (int i = 0; i < 2 * n_layer; i++)
            if (!make_decode_tmap(&kv->tm_dec[i], kv->tensor(i / 2, i % 2), kv_type, head_dim, n_kv_head,
                                  kv->row_bytes, n_ctx)) {
                sv_kv_destroy(kv);
                return SV_ERR_CUDA;
            }
    }
    if (kv_type == SV_TYPE_Q8_0 && prefill_supported(head_dim, kv_type, 4, kv->row_bytes)) {
        // the tensor-core prefill reads a q8_0 layer as f16 (hi, lo) planes rebuilt per call
        const size_t ne0 = (size_t)n_kv_head * head_dim;
        const size_t xbytes = 4 * ne0 * (size_t)n_ctx * sizeof(uint16_t);
        // zeroed once: rows past a call's keys stay finite (masked keys meet P = 0)
        if (cudaMalloc(&kv->xbuf, xbytes) != cudaSuccess || cudaMemset(kv->xbuf, 0, xbytes) != cudaSuccess) {
            cudaGetLastError();
            sv_kv_destroy(kv);
            return SV_ERR_NOMEM;
        }
        for (int i = 0; i < 4; i++)
            if (!make_prefill_tmap(&kv->tm_x[i], kv->xbuf + (size_t)i * ne0 * n_ctx, head_dim, n_kv_head,
                                   ne0 * sizeof(uint16_t), n_ctx)) {
                sv_kv_destroy(kv);
                return SV_ERR_CUDA;
            }
    }
    if (kv_type == SV_TYPE_F16 && prefill_supported(head_dim, kv_type, 4, kv->row_bytes)) {
        kv->tm_pre.resize(2 * n_layer);
        for (int i = 0; i < 2 * n_layer; i++)
            if (!make_prefill_tmap(&kv->tm_pre[i], kv->tensor(i / 2, i % 2), head_dim, n_kv_head, kv->row_bytes,
                                   n_ctx)) {
                sv_kv_destroy(kv);
                return SV_ERR_CUDA;
            }
    }
    fprintf(stderr, "kv cache: %.2f GB (n_ctx %d)\n", (double)total / 1e9, n_ctx);
    *out = kv;
    return SV_OK;
}

int sv_kv_destroy(sv_kv* kv) {
    if (!kv) return SV_ERR_INVALID;
    DeviceGuard g(kv->device);
    if (kv->buf) cudaFree(kv->buf);
    if (kv->ws) cudaFree(kv->ws);
    if (kv->tickets) cudaFree(kv->tickets);
    if (kv->err) cudaFree(kv->err);
    if (kv->scratch) cudaFree(kv->scratch);
    if (kv->xbuf) cudaFree(kv->xbuf);
    delete kv;
    return SV_OK;
}

int sv_kv_clear(sv_kv* kv, void* stream) {
    if (!kv) return SV_ERR_INVALID;
    DeviceGuard g(kv->device);
    kv->rows_written_last = false;   // a memset is never overlapped by the next launch
    return cuda_status(cudaMemsetAsync(kv->buf, 0, kv->tensor_bytes * 2 * (size_t)kv->n_layer,
                                       static_cast<cudaStream_t>(stream)));
}

int sv_kv_tensor(const sv_kv* kv, int layer, int is_v, void** data, size_t* row_bytes) {
    if (!kv || layer < 0 || layer >= kv->n_layer) return SV_ERR_INVALID;
    if (data) *data = kv->tensor(layer, is_v ? 1 : 0);
    if (row_bytes) *row_bytes = kv->row_bytes;
    return SV_OK;
}

int sv_kv_info(const sv_kv* kv, int* n_layer, int* n_kv_head, int* head_dim, int* n_ctx, int* kv_type) {
    if (!kv) return SV_ERR_INVALID;
    if (n_layer) *n_layer = kv->n_layer;
    if (n_kv_head) *n_kv_head = kv->n_kv_head;
    if (head_dim) *head_dim = kv->head_dim;
    if (n_ctx) *n_ctx = kv->n_ctx;
    if (kv_type) *kv_type = kv->type;
    return SV_OK;
}

int sv_kv_error(sv_kv* kv, int* flags, void* stream) {
    if (!kv || !flags) return SV_ERR_INVALID;
    DeviceGuard g(kv->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int h = 0;
    cudaError_t e = cudaMemcpyAsync(&h, kv->err, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(kv->err, 0, sizeof(int), st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    *flags = h;
    return cuda_status(e);
}

// ------------------------------------------------------------------ append
int sv_set_rows(void* dst, int dst_type, int64_t ne0, int64_t dst_rows, size_t dst_nb1, const void* src,
                int src_type, size_t src_nb1, int64_t n_rows, const int32_t* rows, int64_t base, int* err_flag,
                void* stream) {
    if (!dst || (!src && n_rows > 0) || ne0 <= 0 || dst_rows <= 0 || n_rows < 0) return SV_ERR_INVALID;
    if (dst_type != SV_TYPE_F16 && dst_type != SV_TYPE_Q8_0 && dst_type != SV_TYPE_F32) return SV_ERR_UNSUPPORTED;
    if (src_type != SV_TYPE_F16 && src_type != SV_TYPE_F32) return SV_ERR_UNSUPPORTED;
    if (dst_type == SV_TYPE_Q8_0 && ne0 % kQK8_0 != 0) return SV_ERR_UNSUPPORTED;
    if (dst_type == SV_TYPE_F32 && src_type != SV_TYPE_F32 && src_type != SV_TYPE_F16) return SV_ERR_UNSUPPORTED;
    if (dst_nb1 < row_bytes_of(dst_type, ne0) || src_nb1 < row_bytes_of(src_type, ne0)) return SV_ERR_INVALID;
    if (!rows && (base < 0 || base + n_rows > dst_rows)) return SV_ERR_OVERFLOW;
    return cuda_status(launch_set_rows(dst, dst_type, ne0, dst_rows, dst_nb1, src, src_type, src_nb1, n_rows, rows,
                                       base, err_flag, 1, 0, 0, static_cast<cudaStream_t>(stream)));
}

int sv_kv_append(sv_kv* kv, int layer, const void* k, const void* v, int src_type, int n_rows, const int32_t* rows,
                 int base, void* stream) {
    if (!kv || layer < 0 || layer >= kv->n_layer || !k || !v || n_rows < 0) return SV_ERR_INVALID;
    if (src_type != SV_TYPE_F16 && src_type != SV_TYPE_F32) return SV_ERR_UNSUPPORTED;
    if (!rows && (base < 0 || base + n_rows > kv->n_ctx)) return SV_ERR_OVERFLOW;
    if (n_rows == 0) return SV_OK;
    DeviceGuard g(kv->device);
    const int64_t ne0 = (int64_t)kv->n_kv_head * kv->head_dim;
    const size_t src_nb1 = row_bytes_of(src_type, ne0);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // K and V in one launch: blockIdx.y selects the tensor; V sits one tensor after K
    // in the cache buffer, and the V source is addressed relative to the K source.
    const uint8_t* kb = static_cast<const uint8_t*>(k);
    const uint8_t* vb = static_cast<const uint8_t*>(v);
    cudaError_t e;
    if (vb > kb) {
        e = launch_set_rows(kv->tensor(layer, 0), kv->type, ne0, kv->n_ctx, kv->row_bytes, k, src_type, src_nb1,
                            n_rows, rows, base, kv->err, 2, kv->tensor_bytes, (size_t)(vb - kb), st, nullptr, true);
    } else {
        e = launch_set_rows(kv->tensor(layer, 0), kv->type, ne0, kv->n_ctx, kv->row_bytes, k, src_type, src_nb1,
                            n_rows, rows, base, kv->err, 1, 0, 0, st, nullptr, true);
        if (e == cudaSuccess)
            e = launch_set_rows(kv->tensor(layer, 1), kv->type, ne0, kv->n_ctx, kv->row_bytes, v, src_type, src_nb1,
                                n_rows, rows, base, kv->err, 1, 0, 0, st, nullptr, true);
    }
    kv->rows_written_last = true;
    return cuda_status(e);
}

int sv_kv_append_at(sv_kv* kv, int layer, const void* k, const void* v, int src_type, int n_rows,
                    const int32_t* base_dev, void* stream) {
    if (!kv || layer < 0 || layer >= kv->n_layer || !k || !v || n_rows < 0 || !base_dev) return SV_ERR_INVALID;
    if (src_type != SV_TYPE_F16 && src_type != SV_TYPE_F32) return SV_ERR_UNSUPPORTED;
    if (n_rows == 0) return SV_OK;
    DeviceGuard g(kv->device);
    const int64_t ne0 = (int64_t)kv->n_kv_head * kv->head_dim;
    const size_t src_nb1 = row_bytes_of(src_type, ne0);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const uint8_t* kb = static_cast<const uint8_t*>(k);
    const uint8_t* vb = static_cast<const uint8_t*>(v);
    cudaError_t e;
    if (vb > kb) {
        e = launch_set_rows(kv->tensor(layer, 0), kv->type, ne0, kv->n_ctx, kv->row_bytes, k, src_type, src_nb1,
                            n_rows, nullptr, 0, kv->err, 2, kv->tensor_bytes, (size_t)(vb - kb), st, base_dev, true);
    } else {
        e = launch_set_rows(kv->tensor(layer, 0), kv->type, ne0, kv->n_ctx, kv->row_bytes, k, src_type, src_nb1,
                            n_rows, nullptr, 0, kv->err, 1, 0, 0, st, base_dev, true);
        if (e == cudaSuccess)
            e = launch_set_rows(kv->tensor(layer, 1), kv->type, ne0, kv->n_ctx, kv->row_bytes, v, src_type, src_nb1,
                                n_rows, nullptr, 0, kv->err, 1, 0, 0, st, base_dev, true);
    }
    kv->rows_written_last = true;
    return cuda_status(e);
}

int sv_counter_add(int32_t* counter_dev, int n, int delta, void* stream) {
    if (!counter_dev || n <= 0) return SV_ERR_INVALID;
    return cuda_status(launch_counter_add(counter_dev, n, delta, static_cast<cudaStream_t>(stream)));
}

// ------------------------------------------------------------------ attention
static bool clusters_enabled() {
    static const bool on = [] {
        const char* e = getenv("SVKV_CLUSTER");
        return !(e && e[0] == '0');
    }();
    return on;
}

// SVKV_GQA=0 routes grouped-query decode to the general split-K kernel (A/B timing runs)
static bool gqa_enabled() {
    static const bool on = [] {
        const char* e = getenv("SVKV_GQA");
        return !(e && e[0] == '0');
    }();
    return on;
}

// tkp/tvp: prefill-box maps of the f16 cache tensors, or of the hi planes of a q8_0 layer, whose lo
// planes are then tkl/tvl
static int run_attention(sv_kv* kvh, const CUtensorMap* tk, const CUtensorMap* tv, const CUtensorMap* tkp,
                         const CUtensorMap* tvp, int head_dim, int kv_type, AttnArgs& a, int span, bool window,
                         float* ws, size_t ws_bytes, int* tickets, int n_tickets, cudaStream_t st,
                         bool allow_cluster = false, const CUtensorMap* tkl = nullptr,
                         const CUtensorMap* tvl = nullptr) {
    // A fused append + attention may fill its K/V ring before its grid dependency resolves only if
    // the launch before it on the stream did not write cache rows while letting it start early.
    a.ring_prefill = (kvh && !kvh->rows_written_last) ? 1 : 0;
    if (kvh) kvh->rows_written_last = false;
    // chunked prefill on the tensor-core kernel when it applies
    if (!window && tkp && tvp && a.mask_mode == SV_MASK_CAUSAL && a.T * a.G > 16) {
        return cuda_status(launch_prefill(a, head_dim, tkp, tvp, ws, ws ? ws_bytes / sizeof(float) : 0, tickets,
                                          tickets ? n_tickets : 0, st, tkl, tvl));
    }
    const size_t ws_floats = ws ? ws_bytes / sizeof(float) : 0;
    // grouped-query decode (one query tile of <= 8 rows per kv head) on the swap-AB kernel
    const bool gqa = !window && gqa_enabled() && decode_gqa_applies(head_dim, kv_type, a.T, a.G, a.mask_mode);
    // split-K merged inside a thread-block cluster (DSMEM) when the splits fit in one cluster
    // (the GQA kernel's cluster holds the splits plus one merger CTA)
    const int cmax = (allow_cluster && !window && clusters_enabled())
                         ? (gqa ? decode_gqa_max_cluster(head_dim, kv_type) - 1 : decode_max_cluster(head_dim, kv_type))
                         : 1;
    Plan p;
    bool use_cluster = false;
    if (cmax >= 2) {
        p = plan_decode(a.T, a.G, a.NKV, span, head_dim, window, (size_t)1 << 40, 1 << 30, target_ctas_default(), cmax);
        // a cluster caps the splits of a tile; when that leaves most SMs idle (few kv heads and a
        // long context, e.g. one kv head per GPU), the ticket merge with more splits wins
        use_cluster = (size_t)a.NKV * p.n_qtiles * p.n_splits * 2 >= (size_t)target_ctas_default();
    }
    if (use_cluster) {
        a.cluster_merge = p.n_splits > 1;
    } else {
        // per-query windows differ in length (multi-session batches): aim for several waves of
        // CTAs so the short sessions' idle splits do not leave SMs waiting on the long ones
        // (the f16 GQA kernel runs two CTAs per SM)
        const int target = window ? 8 * target_ctas_default()
                                  : (gqa ? decode_gqa_ctas_per_sm(kv_type) : 1) * target_ctas_default();
        p = plan_decode(a.T, a.G, a.NKV, span, head_dim, window, ws_floats, tickets ? n_tickets : 0, target);
        a.cluster_merge = 0;
        // long splits over few kv heads (f16, HD 128; one kv head of a 131072-token session per GPU):
        // one CTA per SM with a 6-stage ring, so more of a split's tiles are in flight (one kv head
        // 19.3 -> 17.0 us per layer), with or without the fused peer gather.
        if (gqa && kv_type == SV_TYPE_F16 && head_dim == 128 && p.n_splits > 48) {
            p = plan_decode(a.T, a.G, a.NKV, span, head_dim, window, ws_floats, tickets ? n_tickets : 0,
                            target_ctas_default());
            a.deep_ring = 1;
        }
    }
    a.qpt = p.qpt;
    a.n_qtiles = p.n_qtiles;
    a.chunk = p.chunk;
    a.n_splits = p.n_splits;
    if (a.n_splits > 1 && !a.cluster_merge) {
        const size_t n_part = (size_t)a.NKV * a.n_qtiles * a.n_splits * 16;
        a.ws_o = ws;
        a.ws_ml = ws + n_part * head_dim;
        a.tickets = tickets;
        // the GQA kernel merges more than 48 splits in two levels (groups of 16 first) when the tickets
        // have room for the groups' counters; up to 48 one CTA merges them all (config 4's 33 splits:
        // the extra ticket round trips of two levels measured slower)
        const int groups = ceil_div(a.n_splits, 16);
        a.merge_levels = (gqa && groups > 3 && (size_t)a.NKV * (1 + groups) <= (size_t)n_tickets) ? 2 : 1;
    }
    if (gqa && a.n_qtiles == 1) return cuda_status(launch_decode_gqa(a, head_dim, kv_type, tk, tv, st));
    return cuda_status(launch_decode(a, head_dim, kv_type, tk, tv, st));
}

int sv_attn(sv_kv* kv, int layer, const void* q, int q_type, int T, int n_head, int n_past, float scale, float* out,
            void* stream) {
    if (!kv || layer < 0 || layer >= kv->n_layer || !q || !out || T <= 0 || n_head <= 0 || n_past < 0)
        return SV_ERR_INVALID;
    if (q_type != SV_TYPE_F16 && q_type != SV_TYPE_F32) return SV_ERR_UNSUPPORTED;
    if (n_head % kv->n_kv_head != 0 || n_head / kv->n_kv_head > 16) return SV_ERR_UNSUPPORTED;
    if (n_past + T > kv->n_ctx) return SV_ERR_OVERFLOW;
    if (kv->tm_dec.empty()) return SV_ERR_UNSUPPORTED;
    DeviceGuard g(kv->device);
    const int HD = kv->head_dim;
    const int es = q_type == SV_TYPE_F32 ? 4 : 2;
    AttnArgs a{};
    a.q = static_cast<const uint8_t*>(q);
    a.q_type = q_type;
    a.q_nb_h = (int64_t)HD * es;
    a.q_nb_t = (int64_t)n_head * HD * es;
    a.T = T;
    a.NH = n_head;
    a.NKV = kv->n_kv_head;
    a.G = n_head / kv->n_kv_head;
    a.S = n_past + T;
    a.row_base = 0;
    a.mask_mode = SV_MASK_CAUSAL;
    a.causal_base = n_past;
    a.scale_log2 = scale * 1.4426950408889634f;
    a.out = out;
    a.out_nb_h = HD;
    a.out_nb_t = (int64_t)n_head * HD;
    a.err = kv->err;
    const CUtensorMap* tkp = kv->tm_pre.empty() ? nullptr : &kv->tm_pre[2 * layer];
    const CUtensorMap* tvp = kv->tm_pre.empty() ? nullptr : &kv->tm_pre[2 * layer + 1];
    const CUtensorMap *tkl = nullptr, *tvl = nullptr;
    if (kv->xbuf && T * a.G > 16 && prefill_supported(HD, kv->type, a.G, kv->row_bytes)) {
        // q8_0 chunk: the keys it sees, rows [0, n_past + T), as f16 (hi, lo) planes, then the
        // tensor-core kernel over the planes (each part through the MMA into the same accumulator)
        const int ne0 = kv->n_kv_head * HD;
        cudaError_t e = launch_q8_0_split(kv->tensor(layer, 0), kv->tensor(layer, 1), kv->row_bytes, ne0, n_past + T,
                                          kv->xbuf, (size_t)ne0 * kv->n_ctx, static_cast<cudaStream_t>(stream));
        if (e != cudaSuccess) return cuda_status(e);
        tkp = &kv->tm_x[0];
        tkl = &kv->tm_x[1];
        tvp = &kv->tm_x[2];
        tvl = &kv->tm_x[3];
    }
    return run_attention(kv, &kv->tm_dec[2 * layer], &kv->tm_dec[2 * layer + 1], tkp, tvp, HD, kv->type, a,
                         n_past + T, false, kv->ws, kv->ws_bytes, kv->tickets, kv->n_tickets,
                         static_cast<cudaStream_t>(stream), /*allow_cluster=*/true, tkl, tvl);
}

int sv_attn_at(sv_kv* kv, int layer, const void* q, int q_type, int T, int n_head, const int32_t* n_past_dev,
               int max_keys, float scale, float* out, void* stream) {
    if (!kv || layer < 0 || layer >= kv->n_layer || !q || !out || T <= 0 || n_head <= 0 || !n_past_dev ||
        max_keys < T)
        return SV_ERR_INVALID;
    if (q_type != SV_TYPE_F16 && q_type != SV_TYPE_F32) return SV_ERR_UNSUPPORTED;
    if (n_head % kv->n_kv_head != 0 || n_head / kv->n_kv_head > 16) return SV_ERR_UNSUPPORTED;
    if (max_keys > kv->n_ctx) return SV_ERR_OVERFLOW;
    if (kv->tm_dec.empty()) return SV_ERR_UNSUPPORTED;
    DeviceGuard g(kv->device);
    const int HD = kv->head_dim;
    const int es = q_type == SV_TYPE_F32 ? 4 : 2;
    AttnArgs a{};
    a.q = static_cast<const uint8_t*>(q);
    a.q_type = q_type;
    a.q_nb_h = (int64_t)HD * es;
    a.q_nb_t = (int64_t)n_head * HD * es;
    a.T = T;
    a.NH = n_head;
    a.NKV = kv->n_kv_head;
    a.G = n_head / kv->n_kv_head;
    a.S = max_keys;
    a.mask_mode = SV_MASK_CAUSAL;
    a.causal_base_dev = n_past_dev;
    a.scale_log2 = scale * 1.4426950408889634f;
    a.out = out;
    a.out_nb_h = HD;
    a.out_nb_t = (int64_t)n_head * HD;
    a.err = kv->err;
    // the device-side base keeps the grid fixed: always the split-K decode kernel
    return run_attention(kv, &kv->tm_dec[2 * layer], &kv->tm_dec[2 * layer + 1], nullptr, nullptr, HD, kv->type, a,
                         max_keys, false, kv->ws, kv->ws_bytes, kv->tickets, kv->n_tickets,
                         static_cast<cudaStream_t>(stream), /*allow_cluster=*/true);
}

int sv_attn_append_at(sv_kv* kv, int layer, const void* q, int q_type, const void* k_new, const void* v_new, int T,
                      int n_head, const int32_t* n_past_dev, int max_keys, float scale, float* out, void* stream) {
    if (!kv || layer < 0 || layer >= kv->n_layer || !q || !out || !k_new || !v_new || T <= 0 || n_head <= 0 ||
        !n_past_dev || max_keys < T)
        return SV_ERR_INVALID;
    if (n_head % kv->n_kv_head != 0 || n_head / kv->n_kv_head > 16) return SV_ERR_UNSUPPORTED;
    const int G = n_head / kv->n_kv_head;
    // the fused kernels cover f16 caches with one query tile, and q8_0 caches on the grouped-query
    // kernel (16-byte aligned f16 sources: each lane quantises 8 elements); otherwise append, then attend
    const bool src_aligned = ((reinterpret_cast<uintptr_t>(k_new) | reinterpret_cast<uintptr_t>(v_new)) & 15) == 0;
    const bool fused = kv->type == SV_TYPE_F16
                           ? T * G <= 16
                           : (kv->type == SV_TYPE_Q8_0 && src_aligned && gqa_enabled() &&
                              decode_gqa_applies(kv->head_dim, kv->type, T, G, SV_MASK_CAUSAL));
    if (!fused) {
        int rc = sv_kv_append_at(kv, layer, k_new, v_new, SV_TYPE_F16, T, n_past_dev, stream);
        if (rc != SV_OK) return rc;
        return sv_attn_at(kv, layer, q, q_type, T, n_head, n_past_dev, max_keys, scale, out, stream);
    }
    if (q_type != SV_TYPE_F16 && q_type != SV_TYPE_F32) return SV_ERR_UNSUPPORTED;
    if (max_keys > kv->n_ctx) return SV_ERR_OVERFLOW;
    if (kv->tm_dec.empty()) return SV_ERR_UNSUPPORTED;
    DeviceGuard g(kv->device);
    const int HD = kv->head_dim;
    const int es = q_type == SV_TYPE_F32 ? 4 : 2;
    AttnArgs a{};
    a.q = static_cast<const uint8_t*>(q);
    a.q_type = q_type;
    a.q_nb_h = (int64_t)HD * es;
    a.q_nb_t = (int64_t)n_head * HD * es;
    a.T = T;
    a.NH = n_head;
    a.NKV = kv->n_kv_head;
    a.G = G;
    a.S = max_keys;
    a.mask_mode = SV_MASK_CAUSAL;
    a.causal_base_dev = n_past_dev;
    a.scale_log2 = scale * 1.4426950408889634f;
    a.out = out;
    a.out_nb_h = HD;
    a.out_nb_t = (int64_t)n_head * HD;
    a.err = kv->err;
    a.n_new = T;
    a.knew = static_cast<const uint8_t*>(k_new);
    a.vnew = static_cast<const uint8_t*>(v_new);
    a.new_nb_t = (int64_t)kv->n_kv_head * HD * 2;
    a.kc_w = kv->tensor(layer, 0);
    a.vc_w = kv->tensor(layer, 1);
    a.cache_row_bytes = kv->row_bytes;
    return run_attention(kv, &kv->tm_dec[2 * layer], &kv->tm_dec[2 * layer + 1], nullptr, nullptr, HD, kv->type, a,
                         max_keys, false, kv->ws, kv->ws_bytes, kv->tickets, kv->n_tickets,
                         static_cast<cudaStream_t>(stream), /*allow_cluster=*/true);
}

int sv_attn_window(sv_kv* kv, int layer, const void* q, int q_type, int n_q, int n_head, const int32_t* lo,
                   const int32_t* hi, const int32_t* own, int max_span, float scale, float* out, void* stream) {
    if (!kv || layer < 0 || layer >= kv->n_layer || !q || !out || n_q <= 0 || n_head <= 0 || !lo || !hi || !own ||
        max_span < 0)
        return SV_ERR_INVALID;
    if (q_type != SV_TYPE_F16 && q_type != SV_TYPE_F32) return SV_ERR_UNSUPPORTED;
    if (n_head % kv->n_kv_head != 0 || n_head / kv->n_kv_head > 16) return SV_ERR_UNSUPPORTED;
    if (kv->tm_dec.empty()) return SV_ERR_UNSUPPORTED;
    DeviceGuard g(kv->device);
    const int HD = kv->head_dim;
    const int es = q_type == SV_TYPE_F32 ? 4 : 2;
    AttnArgs a{};
    a.q = static_cast<const uint8_t*>(q);
    a.q_type = q_type;
    a.q_nb_h = (int64_t)HD * es;
    a.q_nb_t = (int64_t)n_head * HD * es;
    a.T = n_q;
    a.NH = n_head;
    a.NKV = kv->n_kv_head;
    a.G = n_head / kv->n_kv_head;
    a.S = kv->n_ctx;
    a.mask_mode = SV_MASK_WINDOW;
    a.lo = lo;
    a.hi = hi;
    a.own = own;
    a.scale_log2 = scale * 1.4426950408889634f;
    a.out = out;
    a.out_nb_h = HD;
    a.out_nb_t = (int64_t)n_head * HD;
    a.err = kv->err;
    return run_attention(kv, &kv->tm_dec[2 * layer], &kv->tm_dec[2 * layer + 1], nullptr, nullptr, HD, kv->type, a,
                         max_span + 1, true, kv->ws, kv->ws_bytes, kv->tickets, kv->n_tickets,
                         static_cast<cudaStream_t>(stream), /*allow_cluster=*/true);
}

// ggml_flash_attn_ext with explicit views
static int check_fa(const sv_fa_params* p, int* HD, int* T, int* NH, int* S, int* NKV) {
    if (!p || !p->q || !p->k || !p->v || !p->dst) return SV_ERR_INVALID;
    if (p->max_bias != 0.0f || p->logit_softcap != 0.0f) return SV_ERR_UNSUPPORTED;
    if (p->q_type != SV_TYPE_F16 && p->q_type != SV_TYPE_F32) return SV_ERR_UNSUPPORTED;
    if (p->k_type != p->v_type || (p->k_type != SV_TYPE_F16 && p->k_type != SV_TYPE_Q8_0)) return SV_ERR_UNSUPPORTED;
    *HD = (int)p->q_ne[0];
    *T = (int)p->q_ne[1];
    *NH = (int)p->q_ne[2];
    *S = (int)p->k_ne[1];
    *NKV = (int)p->k_ne[2];
    if (p->k_ne[0] != *HD || p->v_ne[0] != *HD || p->v_ne[1] != *S || p->v_ne[2] != *NKV) return SV_ERR_INVALID;
    if (*T <= 0 || *NH <= 0 || *S <= 0 || *NKV <= 0 || *NH % *NKV != 0 || *NH / *NKV > 16) return SV_ERR_UNSUPPORTED;
    const size_t headb = row_bytes_of(p->k_type, *HD);
    // the kernel addresses a head as a column offset inside one cache row: heads packed in the row
    if (p->k_nb[2] != headb || p->v_nb[2] != headb || p->k_nb[1] != p->v_nb[1]) return SV_ERR_UNSUPPORTED;
    if (p->mask && p->mask_ne1 < *T) return SV_ERR_INVALID;
    return SV_OK;
}

size_t sv_flash_attn_ext_workspace(const sv_fa_params* p) {
    int HD, T, NH, S, NKV;
    if (check_fa(p, &HD, &T, &NH, &S, &NKV) != SV_OK) return 0;
    Plan pl = plan_decode(T, NH / NKV, NKV, S, HD, false, (size_t)1 << 40, kMaxTickets, target_ctas_default());
    if (pl.n_splits <= 1) return 0;
    const size_t tiles = (size_t)NKV * pl.n_qtiles;
    return tiles * pl.n_splits * decode_partial_floats(HD) * sizeof(float) + tiles * sizeof(int) + 256;
}

int sv_flash_attn_ext(const sv_fa_params* p, void* workspace, size_t ws_bytes, void* stream) {
    int HD, T, NH, S, NKV;
    int rc = check_fa(p, &HD, &T, &NH, &S, &NKV);
    if (rc != SV_OK) return rc;
    const size_t row_stride = p->k_nb[1];
    if (!decode_supported(HD, p->k_type, row_stride, NKV)) return SV_ERR_UNSUPPORTED;
    if ((reinterpret_cast<uintptr_t>(p->k) & 15) || (reinterpret_cast<uintptr_t>(p->v) & 15)) return SV_ERR_UNSUPPORTED;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // the views' K/V base is where key 0 of kv head 0 starts; rows are row_stride apart
    CUtensorMap tk, tv;
    if (!make_decode_tmap(&tk, p->k, p->k_type, HD, NKV, row_stride, S) ||
        !make_decode_tmap(&tv, p->v, p->v_type, HD, NKV, row_stride, S))
        return SV_ERR_UNSUPPORTED;
    const int es = p->q_type == SV_TYPE_F32 ? 4 : 2;
    if (p->q_nb[0] != (size_t)es) return SV_ERR_UNSUPPORTED;
    AttnArgs a{};
    a.q = static_cast<const uint8_t*>(p->q);
    a.q_type = p->q_type;
    a.q_nb_t = (int64_t)p->q_nb[1];
    a.q_nb_h = (int64_t)p->q_nb[2];
    a.T = T;
    a.NH = NH;
    a.NKV = NKV;
    a.G = NH / NKV;
    a.S = S;
    a.mask_mode = p->mask ? SV_MASK_EXPLICIT : SV_MASK_NONE;
    a.mask = static_cast<const uint16_t*>(p->mask);
    a.mask_nb_t = (int64_t)(p->mask_nb1 / 2);
    a.mask_rows = (int)p->mask_ne1;
    a.scale_log2 = p->scale * 1.4426950408889634f;
    a.out = p->dst;
    a.out_nb_h = HD;
    a.out_nb_t = (int64_t)NH * HD;
    a.err = nullptr;
    // workspace: [partials][tickets]; tickets are zeroed here so any caller buffer works
    float* ws = nullptr;
    int* tickets = nullptr;
    size_t wsb = 0;
    int n_tk = 0;
    if (workspace && ws_bytes > 1024) {
        Plan pl = plan_decode(T, a.G, NKV, S, HD, false, (size_t)1 << 40, kMaxTickets, target_ctas_default());
        const size_t tiles = (size_t)NKV * pl.n_qtiles;
        const size_t tk_bytes = (tiles * sizeof(int) + 255) / 256 * 256;
        if (ws_bytes > tk_bytes + 256) {
            tickets = static_cast<int*>(workspace);
            n_tk = (int)tiles;
            ws = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + tk_bytes);
            wsb = ws_bytes - tk_bytes;
            cudaError_t e = cudaMemsetAsync(tickets, 0, tiles * sizeof(int), st);
            if (e != cudaSuccess) return cuda_status(e);
        }
    }
    return run_attention(nullptr, &tk, &tv, nullptr, nullptr, HD, p->k_type, a, S, false, ws, wsb, tickets, n_tk, st);
}

int sv_attn_append_at_peer(sv_kv* kv, int layer, const void* q, int q_type, const void* k_new, const void* v_new,
                           int T, int n_head, const int32_t* n_past_dev, int max_keys, float scale, sv_peer* peer,
                           int head_offset, int n_head_total, int slot, int wait_slot, const int32_t* epoch_dev,
                           void* stream) {
    if (!kv || layer < 0 || layer >= kv->n_layer || !q || !k_new || !v_new || T <= 0 || n_head <= 0 || !n_past_dev ||
        max_keys < T || !peer || !peer->imported || !epoch_dev || slot < 0 || slot >= peer->n_slots ||
        wait_slot >= peer->n_slots || head_offset < 0 || head_offset + n_head > n_head_total)
        return SV_ERR_INVALID;
    if (peer->device != kv->device) return SV_ERR_INVALID;
    if (kv->type != SV_TYPE_F16) return SV_ERR_UNSUPPORTED;   // the append is fused for f16 caches only
    if (n_head % kv->n_kv_head != 0) return SV_ERR_UNSUPPORTED;
    const int G = n_head / kv->n_kv_head;
    const int HD = kv->head_dim;
    // the fused gather lives in the grouped-query decode kernel
    if (!gqa_enabled() || !decode_gqa_applies(HD, kv->type, T, G, SV_MASK_CAUSAL)) return SV_ERR_UNSUPPORTED;
    if (q_type != SV_TYPE_F16 && q_type != SV_TYPE_F32) return SV_ERR_UNSUPPORTED;
    if ((size_t)T * n_head_total * HD * sizeof(float) > peer->slot_bytes) return SV_ERR_INVALID;
    if (max_keys > kv->n_ctx) return SV_ERR_OVERFLOW;
    if (kv->tm_dec.empty()) return SV_ERR_UNSUPPORTED;
    DeviceGuard g(kv->device);
    const int es = q_type == SV_TYPE_F32 ? 4 : 2;
    AttnArgs a{};
    a.q = static_cast<const uint8_t*>(q);
    a.q_type = q_type;
    a.q_nb_h = (int64_t)HD * es;
    a.q_nb_t = (int64_t)n_head * HD * es;
    a.T = T;
    a.NH = n_head;
    a.NKV = kv->n_kv_head;
    a.G = G;
    a.S = max_keys;
    a.mask_mode = SV_MASK_CAUSAL;
    a.causal_base_dev = n_past_dev;
    a.scale_log2 = scale * 1.4426950408889634f;
    a.out = nullptr;
    a.out_nb_h = HD;
    a.out_nb_t = (int64_t)n_head * HD;
    a.err = kv->err;
    a.n_new = T;
    a.knew = static_cast<const uint8_t*>(k_new);
    a.vnew = static_cast<const uint8_t*>(v_new);
    a.new_nb_t = (int64_t)kv->n_kv_head * HD * 2;
    a.kc_w = kv->tensor(layer, 0);
    a.vc_w = kv->tensor(layer, 1);
    a.cache_row_bytes = kv->row_bytes;
    a.peer_out = peer->d_out + (size_t)slot * peer->world;
    a.peer_ctr = peer->d_ctr + (size_t)slot * peer->world;
    a.n_peers = peer->world;
    a.head_offset = head_offset;
    a.peer_nb_t = (int64_t)n_head_total * HD;
    a.epoch_dev = epoch_dev;
    // each rank's output CTAs count once per kv head on every rank
    a.wait_per_epoch = (unsigned int)(kv->n_kv_head * peer->world);
    a.wait_ctr = wait_slot >= 0 ? peer->ctr(wait_slot) : nullptr;
    return run_attention(kv, &kv->tm_dec[2 * layer], &kv->tm_dec[2 * layer + 1], nullptr, nullptr, HD, kv->type, a,
                         max_keys, false, kv->ws, kv->ws_bytes, kv->tickets, kv->n_tickets,
                         static_cast<cudaStream_t>(stream), /*allow_cluster=*/true);
}

int sv_qk_norm_rope_append(sv_kv* kv, int layer, const float* q, const float* k, const float* v, int T, int n_head,
                           const float* q_norm, const float* k_norm, float eps, const sv_rope* rope,
                           const int32_t* pos, int slot_base, const int32_t* slot_base_dev, void* q_out,
                           int q_out_type, void* stream) {
    if (!kv || layer < 0 || layer >= kv->n_layer || !q || !k || !v || T <= 0 || n_head <= 0 || !q_out ||
        !(eps >= 0.0f))
        return SV_ERR_INVALID;
    if (n_head % kv->n_kv_head != 0) return SV_ERR_UNSUPPORTED;
    if (q_out_type != SV_TYPE_F16 && q_out_type != SV_TYPE_F32) return SV_ERR_UNSUPPORTED;
    const int mode = rope ? rope->mode : SV_ROPE_NONE;
    if (mode != SV_ROPE_NONE) {
        if (!pos || !(rope->freq_base > 0.0f)) return SV_ERR_INVALID;
        if (mode == SV_ROPE_IMROPE)
            for (int i = 0; i < 4; i++)
                if (rope->sections[i] < 0) return SV_ERR_INVALID;
    }
    if (!rope_supported(kv->head_dim, mode, mode == SV_ROPE_NONE ? kv->head_dim : rope->n_dims))
        return SV_ERR_UNSUPPORTED;
    if (!slot_base_dev && (slot_base < 0 || (int64_t)slot_base + T > kv->n_ctx)) return SV_ERR_OVERFLOW;
    DeviceGuard g(kv->device);
    RopeLaunch r{};
    r.q = q;
    r.k = k;
    r.v = v;
    r.T = T;
    r.NH = n_head;
    r.NKV = kv->n_kv_head;
    r.HD = kv->head_dim;
    r.qn = q_norm;
    r.kn = k_norm;
    r.eps = eps;
    r.mode = mode;
    r.n_dims = mode == SV_ROPE_NONE ? kv->head_dim : rope->n_dims;
    r.freq_base = mode == SV_ROPE_NONE ? 1.0f : rope->freq_base;
    for (int i = 0; i < 4; i++) r.sec[i] = mode == SV_ROPE_IMROPE ? rope->sections[i] : 0;
    r.pos = pos;
    r.slot_base = slot_base;
    r.slot_base_dev = slot_base_dev;
    r.kc = kv->tensor(layer, 0);
    r.vc = kv->tensor(layer, 1);
    r.row_bytes = kv->row_bytes;
    r.kv_type = kv->type;
    r.n_ctx = kv->n_ctx;
    r.q_out = q_out;
    r.q_out_type = q_out_type;
    r.err = kv->err;
    // the kernel lets the next launch start early, so that launch must not read cache rows before
    // its grid dependency resolves
    kv->rows_written_last = true;
    return cuda_status(launch_qk_norm_rope_append(r, static_cast<cudaStream_t>(stream)));
}

int sv_soft_max_ext(const float* x, int64_t ne0, int64_t n_rows, size_t x_nb1, const void* mask, int64_t mask_rows,
                    size_t mask_nb1, float scale, float* y, size_t y_nb1, void* stream) {
    if (!x || !y || ne0 <= 0 || n_rows < 0 || (mask && mask_rows <= 0)) return SV_ERR_INVALID;
    if (n_rows == 0) return SV_OK;
    return cuda_status(launch_soft_max(x, ne0, n_rows, x_nb1, static_cast<const uint16_t*>(mask), mask_rows, mask_nb1,
                                       scale, y, y_nb1, static_cast<cudaStream_t>(stream)));
}

// ------------------------------------------------------------------ eviction
int sv_kv_compact(sv_kv* kv, const sv_segment* segs, int n_segs, int dst_base, int* new_len, void* stream) {
    if (!kv || (!segs && n_segs > 0) || n_segs < 0 || dst_base < 0) return SV_ERR_INVALID;
    if (n_segs > 1024) return SV_ERR_UNSUPPORTED;
    if (kv->row_bytes % 16 != 0) return SV_ERR_UNSUPPORTED;   // rows move as 16-byte vectors
    int64_t kept = 0;
    int64_t prev_end = -1;
    for (int s = 0; s < n_segs; s++) {
        if (segs[s].n_rows < 0 || segs[s].src < 0 || (int64_t)segs[s].src + segs[s].n_rows > kv->n_ctx)
            return SV_ERR_INVALID;
        if (segs[s].src < prev_end) return SV_ERR_INVALID;       // segments ascend and do not overlap
        prev_end = (int64_t)segs[s].src + segs[s].n_rows;
        if (segs[s].keep) {
            if (segs[s].n_rows > 0 && (int64_t)segs[s].src < dst_base + kept) return SV_ERR_INVALID;   // front only
            kept += segs[s].n_rows;
        }
    }
    if (new_len) *new_len = (int)(dst_base + kept);
    DeviceGuard g(kv->device);
    kv->rows_written_last = false;   // compaction launches are never overlapped by the next launch
    return cuda_status(launch_compact(kv, nullptr, segs, n_segs, dst_base, static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
