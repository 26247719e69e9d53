// noalloc.cu - sv_flash_attn_ext_static: flash attention whose scratch lives in
// a fixed device array of this library instead of memory the caller provides.
//
// Some callers cannot allocate device memory at the point where attention
// runs: an operator invoked inside a ggml backend graph gets only its input
// and output tensors (no workspace argument), and code running while a stream
// is being captured into a CUDA graph may not call cudaMalloc.  This entry
// point serves them: the split-K partials and merge tickets of the decode
// kernel live in kScratchBytes of static device memory, which every GPU that
// loads the library holds until the process exits.
//
// Set-up: the first call on a device looks the array's device address up with
// cudaGetSymbolAddress (host code cannot use the array's name as a device
// pointer) while that device is current, and caches it.  Make that first call
// before any stream capture.  Calls share the one array and it keeps the last
// call's contents; the merge tickets are cleared on every call.  Calls that
// overlap on the GPU (other streams, other threads) race on the array.
#include <cstdio>
#include <mutex>

#include "internal.hpp"

namespace {

constexpr size_t kScratchBytes = 4u << 20;   // 4 MiB

static __device__ __align__(256) unsigned char g_fa_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

}  // namespace

extern "C" int sv_flash_attn_ext_static(const sv_fa_params* p, void* stream) {
    if (!p) return SV_ERR_INVALID;
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return SV_ERR_CUDA;
    void* scratch = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_mu);
        if (!g_scratch_ptr[dev]) {
            void* ptr = nullptr;
            const cudaError_t e = cudaGetSymbolAddress(&ptr, g_fa_scratch);
            if (e != cudaSuccess || !ptr) {
                fprintf(stderr, "sv_flash_attn_ext_static: cudaGetSymbolAddress failed on device %d: %s\n", dev,
                        cudaGetErrorString(e));
                return SV_ERR_CUDA;
            }
            g_scratch_ptr[dev] = ptr;
        }
        scratch = g_scratch_ptr[dev];
    }
    const size_t need = sv_flash_attn_ext_workspace(p);
    if (need > kScratchBytes) {
        fprintf(stderr,
                "sv_flash_attn_ext_static: this shape needs %zu bytes of scratch, more than the %zu-byte static "
                "array; use sv_flash_attn_ext with a workspace\n",
                need, kScratchBytes);
        return SV_ERR_WORKSPACE;
    }
    // sv_flash_attn_ext zeroes the ticket words at the start of the workspace on every call
    return sv_flash_attn_ext(p, scratch, kScratchBytes, stream);
}
