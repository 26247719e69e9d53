// peer.cu - gathered-output buffers for head-sharded decode, shared between the ranks' processes
// over CUDA IPC, and the bounded wait on their arrival counters.
//
// One session too long for one GPU shards by kv head: rank g attends with its kv heads and must
// end each layer with every rank's [T, NH/G, HD] output in one [T, NH, HD] buffer (the all-gather
// of the reference-side design).  Instead of a collective call after the attention kernel, the
// attention kernel's output stores go straight into every rank's buffer (peer memory over
// NVLink) and count themselves on every rank's arrival counter; a later kernel (the next layer's
// attention, or sv_peer_wait) waits on the counter.
#include <cstring>

#include "common.cuh"
#include "internal.hpp"

namespace svkv {
namespace {

__global__ void peer_wait_kernel(const unsigned int* ctr, const int32_t* epoch_dev, unsigned int per_epoch, int* err) {
    pdl_wait();
    if (threadIdx.x == 0) {
        const unsigned int target = (unsigned int)(*reinterpret_cast<const volatile int*>(epoch_dev)) * per_epoch;
        const uint64_t t0 = globaltimer_ns();
        while (*reinterpret_cast<const volatile unsigned int*>(ctr) < target) {
            if (globaltimer_ns() - t0 > kWaitLimitNs) {
                if (err) atomicOr(err, ERRBIT_TIMEOUT);
                break;
            }
        }
        __threadfence_system();
    }
    pdl_trigger();
}

}  // namespace

cudaError_t launch_peer_wait(const unsigned int* ctr, const int32_t* epoch_dev, unsigned int per_epoch, int* err,
                             cudaStream_t st) {
    return launch_pdl(peer_wait_kernel, dim3(1), dim3(32), 0, st, ctr, epoch_dev, per_epoch, err);
}

}  // namespace svkv

extern "C" {

int sv_peer_create(int device, int rank, int world, int n_slots, size_t slot_bytes, sv_peer** out) {
    if (!out || world < 1 || world > 8 || rank < 0 || rank >= world || n_slots < 1 || slot_bytes == 0 ||
        (slot_bytes & 15))
        return SV_ERR_INVALID;
    *out = nullptr;
    int prev = 0;
    if (cudaGetDevice(&prev) != cudaSuccess) return SV_ERR_CUDA;
    if (cudaSetDevice(device) != cudaSuccess) return SV_ERR_CUDA;
    sv_peer* p = new sv_peer();
    p->device = device;
    p->rank = rank;
    p->world = world;
    p->n_slots = n_slots;
    p->slot_bytes = slot_bytes;
    p->ctr_off = ((size_t)n_slots * slot_bytes + 255) & ~(size_t)255;
    p->bctr_off = p->ctr_off + (((size_t)n_slots * sizeof(unsigned int) + 255) & ~(size_t)255);
    p->buf_bytes = p->bctr_off + (size_t)n_slots * svkv::kPeerBands * sizeof(unsigned int);
    bool ok = cudaMalloc(&p->buf, p->buf_bytes) == cudaSuccess;
    ok = ok && cudaMemset(p->buf, 0, p->buf_bytes) == cudaSuccess;
    ok = ok && cudaMalloc(&p->d_out, sizeof(float*) * n_slots * world) == cudaSuccess;
    ok = ok && cudaMalloc(&p->d_ctr, sizeof(unsigned int*) * n_slots * world) == cudaSuccess;
    ok = ok && cudaMalloc(&p->d_bctr, sizeof(unsigned int*) * n_slots * world) == cudaSuccess;
    ok = ok && cudaDeviceSynchronize() == cudaSuccess;
    cudaSetDevice(prev);
    if (!ok) {
        cudaGetLastError();
        if (p->buf) cudaFree(p->buf);
        if (p->d_out) cudaFree(p->d_out);
        if (p->d_ctr) cudaFree(p->d_ctr);
        if (p->d_bctr) cudaFree(p->d_bctr);
        delete p;
        return SV_ERR_NOMEM;
    }
    p->base[rank] = p->buf;
    *out = p;
    return SV_OK;
}

int sv_peer_export(const sv_peer* p, void* handle) {
    if (!p || !handle) return SV_ERR_INVALID;
    cudaIpcMemHandle_t h;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(p->device);
    const cudaError_t e = cudaIpcGetMemHandle(&h, p->buf);
    cudaSetDevice(prev);
    if (e != cudaSuccess) return SV_ERR_CUDA;
    static_assert(sizeof(cudaIpcMemHandle_t) == SV_PEER_HANDLE_BYTES, "IPC handle size");
    memcpy(handle, &h, sizeof(h));
    return SV_OK;
}

int sv_peer_import(sv_peer* p, const void* handles) {
    if (!p || !handles || p->imported) return SV_ERR_INVALID;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(p->device);
    int rc = SV_OK;
    for (int r = 0; r < p->world && rc == SV_OK; r++) {
        if (r == p->rank) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const uint8_t*>(handles) + (size_t)r * SV_PEER_HANDLE_BYTES, sizeof(h));
        void* ptr = nullptr;
        if (cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            rc = SV_ERR_CUDA;
            break;
        }
        p->base[r] = static_cast<uint8_t*>(ptr);
        p->opened[r] = true;
    }
    if (rc == SV_OK) {
        const int n = p->n_slots * p->world;
        float** h_out = new float*[n];
        unsigned int** h_ctr = new unsigned int*[n];
        unsigned int** h_bctr = new unsigned int*[n];
        for (int s = 0; s < p->n_slots; s++) {
            for (int r = 0; r < p->world; r++) {
                h_out[s * p->world + r] = reinterpret_cast<float*>(p->base[r] + (size_t)s * p->slot_bytes);
                h_ctr[s * p->world + r] = reinterpret_cast<unsigned int*>(p->base[r] + p->ctr_off) + s;
                h_bctr[s * p->world + r] =
                    reinterpret_cast<unsigned int*>(p->base[r] + p->bctr_off) + (size_t)s * svkv::kPeerBands;
            }
        }
        if (cudaMemcpy(p->d_out, h_out, sizeof(float*) * n, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(p->d_ctr, h_ctr, sizeof(unsigned int*) * n, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(p->d_bctr, h_bctr, sizeof(unsigned int*) * n, cudaMemcpyHostToDevice) != cudaSuccess)
            rc = SV_ERR_CUDA;
        delete[] h_out;
        delete[] h_ctr;
        delete[] h_bctr;
    }
    cudaSetDevice(prev);
    if (rc == SV_OK) p->imported = true;
    return rc;
}

int sv_peer_slot(const sv_peer* p, int slot, void** data) {
    if (!p || !data || slot < 0 || slot >= p->n_slots) return SV_ERR_INVALID;
    *data = p->buf + (size_t)slot * p->slot_bytes;
    return SV_OK;
}

int sv_peer_wait(sv_peer* p, int slot, const int32_t* epoch_dev, int per_epoch, int* err_dev, void* stream) {
    if (!p || slot < 0 || slot >= p->n_slots || !epoch_dev || per_epoch <= 0) return SV_ERR_INVALID;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(p->device);
    const cudaError_t e = svkv::launch_peer_wait(p->ctr(slot), epoch_dev, (unsigned int)per_epoch, err_dev,
                                                 static_cast<cudaStream_t>(stream));
    cudaSetDevice(prev);
    return e == cudaSuccess ? SV_OK : SV_ERR_CUDA;
}

int sv_out_proj_peer(sv_peer* p, const void* x, int x_type, int64_t x_nb_t, const void* w, int K_total, int k_offset,
                     int K_local, int D, int T, int slot, const int32_t* epoch_dev, float* out, int* err_dev,
                     void* stream) {
    if (!p || !p->imported || !x || !w || !out || !epoch_dev || slot < 0 || slot >= p->n_slots || T <= 0 || D <= 0 ||
        K_local <= 0 || k_offset < 0 || (int64_t)k_offset + K_local > K_total)
        return SV_ERR_INVALID;
    if (x_type != SV_TYPE_F16 && x_type != SV_TYPE_F32) return SV_ERR_UNSUPPORTED;
    // 16-byte weight loads: row starts and the column slice on 8-element boundaries; x staged in
    // shared memory (T x K_local f32 <= 128 KB)
    if (T > svkv::out_proj_max_t() || D > svkv::out_proj_max_d() || (K_total & 7) || (k_offset & 7) || (K_local & 7) || K_local > 4096 ||
        (reinterpret_cast<uintptr_t>(w) & 15))
        return SV_ERR_UNSUPPORTED;
    if ((size_t)p->world * T * D * sizeof(float) > p->slot_bytes) return SV_ERR_INVALID;
    if (x_nb_t < (int64_t)K_local * (x_type == SV_TYPE_F32 ? 4 : 2)) return SV_ERR_INVALID;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(p->device);
    svkv::OutProjLaunch r{};
    r.x = x;
    r.x_type = x_type;
    r.x_nb_t = x_nb_t;
    r.w = static_cast<const uint16_t*>(w);
    r.K_total = K_total;
    r.k_offset = k_offset;
    r.K_local = K_local;
    r.D = D;
    r.T = T;
    r.peer_out = p->d_out + (size_t)slot * p->world;
    r.peer_bctr = p->d_bctr + (size_t)slot * p->world;
    r.n_peers = p->world;
    r.rank = p->rank;
    r.my_bctr = p->bctr(slot);
    r.my_slot = reinterpret_cast<const float*>(p->buf + (size_t)slot * p->slot_bytes);
    r.epoch_dev = epoch_dev;
    r.out = out;
    r.err = err_dev;
    // slots with room for one 64-bit word per partial carry (value, epoch) words: no band counters
    r.ll = (size_t)p->world * T * D * sizeof(unsigned long long) <= p->slot_bytes ? 1 : 0;
    const cudaError_t e = svkv::launch_out_proj_peer(r, static_cast<cudaStream_t>(stream));
    cudaSetDevice(prev);
    return e == cudaSuccess ? SV_OK : SV_ERR_CUDA;
}

int sv_peer_destroy(sv_peer* p) {
    if (!p) return SV_OK;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(p->device);
    cudaDeviceSynchronize();
    for (int r = 0; r < p->world; r++)
        if (p->opened[r]) cudaIpcCloseMemHandle(p->base[r]);
    if (p->buf) cudaFree(p->buf);
    if (p->d_out) cudaFree(p->d_out);
    if (p->d_ctr) cudaFree(p->d_ctr);
    if (p->d_bctr) cudaFree(p->d_bctr);
    cudaSetDevice(prev);
    delete p;
    return SV_OK;
}

}  // extern "C"
