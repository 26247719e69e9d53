// attn_prefill.cu - chunked-prefill attention on tcgen05 / TMEM (sm_100a).
// (placeholder: the decode kernel serves every query count until this lands)
#include "common.cuh"
#include "internal.hpp"

namespace svkv {

bool prefill_supported(int, int, int, size_t) { return false; }

bool make_prefill_tmap(CUtensorMap*, const void*, int, int, size_t, int64_t) { return false; }

cudaError_t launch_prefill(const AttnArgs&, int, const CUtensorMap*, const CUtensorMap*, cudaStream_t) {
    return cudaErrorNotSupported;
}

}  // namespace svkv
