// internal.hpp - library-internal types shared by the .cu/.cpp files.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <vector>

#include "../../include/svkv.h"

namespace svkv {

constexpr int kQK8_0 = 32;
constexpr int kQ8_0Bytes = 34;
constexpr int kNumSMs = 148;

inline size_t row_bytes_of(int type, int64_t ne0) {
    switch (type) {
        case SV_TYPE_F32: return (size_t)ne0 * 4;
        case SV_TYPE_F16: return (size_t)ne0 * 2;
        case SV_TYPE_Q8_0: return (size_t)(ne0 / kQK8_0) * kQ8_0Bytes;
        default: return 0;
    }
}

inline int ceil_div(int64_t a, int64_t b) { return (int)((a + b - 1) / b); }

// Runs init() once per device (the current one) and returns its cached status.  Kernel attributes
// (dynamic shared memory above 48 KB, non-portable cluster sizes) belong to a device's context, so a
// process that drives several GPUs must set them on each.
constexpr int kMaxDevices = 64;
template <class F>
cudaError_t once_per_device(std::once_flag (&once)[kMaxDevices], cudaError_t (&status)[kMaxDevices], F&& init) {
    int dev = 0;
    const cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::call_once(once[dev], [&] { status[dev] = init(); });
    return status[dev];
}

// SM count of the current device (cached per device); kNumSMs when the query fails
inline int device_sm_count() {
    static std::once_flag once[kMaxDevices];
    static int count[kMaxDevices];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return kNumSMs;
    std::call_once(once[dev], [&] {
        int n = 0;
        count[dev] = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0 ? n : kNumSMs;
    });
    return count[dev];
}

// ------------------------------------------------------------ attention args
// One attention launch: queries x one kv view.  All strides in bytes.
struct AttnArgs {
    const uint8_t* q;       // query element (t, h, e) at q + t*q_nb_t + h*q_nb_h + e*q_es
    int64_t q_nb_t, q_nb_h;
    int q_type;             // SV_TYPE_F16 / SV_TYPE_F32
    int T, NH, NKV, G;      // G = NH / NKV
    int qpt;                // queries per 16-row tile (decode kernel)
    int n_qtiles;
    int S;                  // keys in the view
    int row_base;           // tensor row of view key 0 (TMA y coordinate offset)
    int mask_mode;
    int causal_base;
    const int32_t* causal_base_dev;   // when set, the causal base is read on the device (graph-stable)
    const int32_t* lo;      // window mode, device [T]
    const int32_t* hi;
    const int32_t* own;
    const uint16_t* mask;   // explicit mode: f16 row t at mask + t*mask_nb_t (elements)
    int64_t mask_nb_t;
    int mask_rows;          // rows available in the mask (query t uses row t)
    float scale_log2;       // scale * log2(e)
    int chunk;              // keys per split
    int n_splits;
    int cluster_merge;      // 1: the n_splits CTAs of a tile form a cluster and merge through DSMEM
    float* out;             // (t, h, e) at out + t*out_nb_t + h*out_nb_h + e (floats)
    int64_t out_nb_t, out_nb_h;
    float* ws_o;            // split partials [tile][split][16][HD]
    float* ws_ml;           // [tile][split][16][2]
    int* tickets;           // [tile], zero between launches
    int merge_levels;       // GQA ticket merge: 2 = groups of 16 splits first (tickets[NKV + kvh*groups + g] too)
    int deep_ring;          // GQA f16 HD 128: one CTA per SM with a 6-stage ring (long splits, few kv heads)
    int* err;
    // fused append (f16 cache, decode kernel): rows [cbase, cbase + n_new) come from knew/vnew
    // (row stride new_nb_t bytes) and are written to kc_w/vc_w while being attended
    int n_new;
    const uint8_t* knew;
    const uint8_t* vnew;
    int64_t new_nb_t;
    uint8_t* kc_w;
    uint8_t* vc_w;
    size_t cache_row_bytes;
    int q_tma;              // prefill kernel: the query tiles arrive by TMA (f16 queries)
    // Head-sharded decode with the all-gather fused in (GQA decode kernel): every finished output
    // row is also stored into each rank's gathered buffer (peer_out[p], this slot's region, rows
    // laid out [T][n_head_total][HD] with this rank's heads at head_offset), and the CTA that
    // stored a kv head's rows then adds 1 to every rank's arrival counter peer_ctr[p].
    float* const* peer_out;
    unsigned int* const* peer_ctr;
    int n_peers;            // 0: plain output to out
    int head_offset;
    int64_t peer_nb_t;      // floats between queries in the gathered buffer
    // Before reading its query rows, wait (bounded) until *wait_ctr >= *epoch_dev * wait_per_epoch
    // (the previous layer's gather is complete); wait_ctr == nullptr: no wait.
    const unsigned int* wait_ctr;
    const int32_t* epoch_dev;
    unsigned int wait_per_epoch;
    // the fused append may fill its K/V ring before the grid dependency resolves: the launch before
    // it on the stream wrote no cache rows while letting it start early (host-tracked per handle)
    int ring_prefill;
};

struct PrefillArgs;  // attn_prefill.cu

// ------------------------------------------------------------ handle
struct KvHandle {
    int device = 0;
    int n_layer = 0, n_kv_head = 0, head_dim = 0, n_ctx = 0, type = SV_TYPE_F16;
    size_t row_bytes = 0, tensor_bytes = 0;
    uint8_t* buf = nullptr;              // 2*n_layer tensors, K then V per layer
    std::vector<CUtensorMap> tm_dec;     // decode-box tensor maps: [2*layer + is_v]
    std::vector<CUtensorMap> tm_pre;     // prefill-box tensor maps (f16 caches), same indexing
    // q8_0 caches: one layer's rows as f16 (hi, lo) planes for the tensor-core prefill (K hi, K lo,
    // V hi, V lo; n_ctx rows each), rebuilt by every prefill call, and their prefill-box tensor maps
    uint16_t* xbuf = nullptr;
    CUtensorMap tm_x[4];
    float* ws = nullptr;                 // split-K partials
    size_t ws_bytes = 0;
    int* tickets = nullptr;
    int n_tickets = 0;
    // the last launch this handle enqueued was an append that lets the next launch start early;
    // the next attention launch must then not read cache rows before its grid dependency resolves
    bool rows_written_last = false;
    int* err = nullptr;                  // device error word
    uint8_t* scratch = nullptr;          // one tensor's worth of rows for compaction fallback

    uint8_t* tensor(int layer, int is_v) const {
        return buf + (size_t)(2 * layer + is_v) * tensor_bytes;
    }
};

// ------------------------------------------------------------ host helpers
bool encode_tmap_2d(CUtensorMap* m, const void* base, CUtensorMapDataType dt, uint64_t dim0,
                    uint64_t dim1, uint64_t stride1_bytes, uint32_t box0, uint32_t box1,
                    CUtensorMapSwizzle swz);
bool encode_tmap_3d(CUtensorMap* m, const void* base, CUtensorMapDataType dt, const uint64_t dims[3],
                    const uint64_t strides_bytes[2], const uint32_t box[3], CUtensorMapSwizzle swz);

// decode kernel: can this (head_dim, kv type, row layout) run?
bool decode_supported(int head_dim, int kv_type, size_t row_bytes, int n_kv_head);
// build the decode tensor map of one cache view tensor
bool make_decode_tmap(CUtensorMap* m, const void* base, int kv_type, int head_dim, int n_kv_head,
                      size_t row_bytes, int64_t n_rows);
size_t decode_partial_floats(int head_dim);   // floats per (tile, split) partial incl. m/l
int decode_max_cluster(int head_dim, int kv_type);   // largest co-schedulable cluster (<= 16), 1 = none
// GQA decode kernel (attn_decode_gqa.cu): f16 cache HD 64/128 (T*G <= 8 rows) or q8_0 cache HD 256
// (T*G <= 4), causal or no mask
bool decode_gqa_applies(int head_dim, int kv_type, int T, int G, int mask_mode);
int decode_gqa_max_cluster(int head_dim, int kv_type);
int decode_gqa_ctas_per_sm(int kv_type);
cudaError_t launch_decode_gqa(const AttnArgs& a, int head_dim, int kv_type, const CUtensorMap* tk,
                              const CUtensorMap* tv, cudaStream_t st);
int decode_block_keys();                       // BK
cudaError_t launch_decode(const AttnArgs& a, int head_dim, int kv_type, const CUtensorMap* tk,
                          const CUtensorMap* tv, cudaStream_t st);

// prefill (tcgen05) kernel
bool prefill_supported(int head_dim, int kv_type, int G, size_t row_bytes);
bool make_prefill_tmap(CUtensorMap* m, const void* base, int head_dim, int n_kv_head, size_t row_bytes,
                       int64_t n_rows);
// tk_lo/tv_lo non-null: tk/tv map the hi parts and tk_lo/tv_lo the lo parts of a q8_0 cache's rows
// (q8_0_split_kernel), and every K/V tile goes through the tensor core as hi + lo
cudaError_t launch_prefill(const AttnArgs& a, int head_dim, const CUtensorMap* tk, const CUtensorMap* tv, float* ws,
                           size_t ws_floats, int* tickets, int n_tickets, cudaStream_t st,
                           const CUtensorMap* tk_lo = nullptr, const CUtensorMap* tv_lo = nullptr);
// rows [0, n_rows) of one layer's q8_0 K and V tensors -> f16 planes K hi, K lo, V hi, V lo
// (planes + i * plane_elems, each [row][ne0])
cudaError_t launch_q8_0_split(const uint8_t* kc, const uint8_t* vc, size_t row_bytes, int ne0, int n_rows,
                              uint16_t* planes, size_t plane_elems, cudaStream_t st);

cudaError_t launch_set_rows(void* dst, int dst_type, int64_t ne0, int64_t dst_rows, size_t dst_nb1,
                            const void* src, int src_type, size_t src_nb1, int64_t n_rows,
                            const int32_t* rows, int64_t base, int* err, int n_tensors,
                            size_t dst_tensor_stride, size_t src_tensor_stride, cudaStream_t st,
                            const int32_t* base_dev = nullptr, bool early_trigger = false);

cudaError_t launch_counter_add(int32_t* counter, int n, int delta, cudaStream_t st);

// q/k RMSNorm + rotary embedding + K/V append (rope.cu)
struct RopeLaunch {
    const float* q;
    const float* k;
    const float* v;
    int T, NH, NKV, HD;
    const float* qn;
    const float* kn;
    float eps;
    int mode, n_dims;
    float freq_base;
    int sec[4];
    const int32_t* pos;
    int slot_base;
    const int32_t* slot_base_dev;
    uint8_t* kc;
    uint8_t* vc;
    size_t row_bytes;
    int kv_type;
    int n_ctx;
    void* q_out;
    int q_out_type;
    int* err;
};
bool rope_supported(int head_dim, int mode, int n_dims);

// output projection of this rank's heads + sum over ranks through peer memory (out_proj.cu)
struct OutProjLaunch {
    const void* x;
    int x_type;
    int64_t x_nb_t;
    const uint16_t* w;
    int K_total, k_offset, K_local, D, T;
    float* const* peer_out;            // the slot's region on every rank [world]
    unsigned int* const* peer_bctr;    // the slot's band counters on every rank [world]
    int n_peers, rank;
    const unsigned int* my_bctr;       // this rank's band counters of the slot [kPeerBands]
    const float* my_slot;
    const int32_t* epoch_dev;
    float* out;
    int* err;
    int ll;                            // slots hold one 64-bit (value, epoch) word per partial
};
cudaError_t launch_out_proj_peer(const OutProjLaunch& r, cudaStream_t st);
int out_proj_max_t();
int out_proj_max_d();
cudaError_t launch_qk_norm_rope_append(const RopeLaunch& r, cudaStream_t st);

cudaError_t launch_compact(KvHandle* kv, const int32_t* seg_dev_unused, const sv_segment* segs, int n_segs,
                           int dst_base, cudaStream_t st);

cudaError_t launch_soft_max(const float* x, int64_t ne0, int64_t n_rows, size_t x_nb1, const uint16_t* mask,
                            int64_t mask_rows, size_t mask_nb1, float scale, float* y, size_t y_nb1,
                            cudaStream_t st);

}  // namespace svkv

struct sv_kv : svkv::KvHandle {};

namespace svkv {
// Gathered-output buffers of a head-sharded session, one per rank, mapped into every rank over
// CUDA IPC (peer memory over NVLink).  Local allocation: n_slots regions of slot_bytes, then one
// 32-bit arrival counter per slot.
// per slot, one arrival counter per output band of sv_out_proj_peer (its grid never exceeds this)
constexpr int kPeerBands = 512;
struct PeerGroup {
    int device = 0, rank = 0, world = 1, n_slots = 0;
    size_t slot_bytes = 0, ctr_off = 0, bctr_off = 0, buf_bytes = 0;
    uint8_t* buf = nullptr;
    uint8_t* base[8] = {nullptr};      // every rank's buffer in this process (base[rank] = buf)
    bool opened[8] = {false};
    float** d_out = nullptr;           // device [n_slots][world]: each rank's region of a slot
    unsigned int** d_ctr = nullptr;    // device [n_slots][world]: each rank's counter of a slot
    unsigned int** d_bctr = nullptr;   // device [n_slots][world]: each rank's band counters of a slot
    bool imported = false;
    unsigned int* ctr(int slot) const { return reinterpret_cast<unsigned int*>(buf + ctr_off) + slot; }
    unsigned int* bctr(int slot) const {
        return reinterpret_cast<unsigned int*>(buf + bctr_off) + (size_t)slot * kPeerBands;
    }
};
cudaError_t launch_peer_wait(const unsigned int* ctr, const int32_t* epoch_dev, unsigned int per_epoch, int* err,
                             cudaStream_t st);
}  // namespace svkv
struct sv_peer : svkv::PeerGroup {};
