// IQ2_XXS prefill GEMM (m > 16) on the sm_100a tensor cores. Until the tcgen05 kernel is in
// place, m > 16 is served by the generic GEMV kernel (gemm_path_ok returns false).
#include "iq2xxs_common.cuh"
#include "iq2xxs_internal.h"

namespace iq2 {

bool gemm_path_ok(uint32_t, uint32_t, uint32_t, const void*, int, const uint8_t*, const uint8_t*,
                  const float*) {
    return false;
}

size_t gemm_workspace_size(uint32_t, uint32_t, uint32_t, int) { return 0; }

cudaError_t launch_gemm(const void*, int, uint32_t, const uint8_t*, const uint8_t*, uint32_t, uint32_t,
                        float*, void*, int, cudaStream_t) {
    return cudaErrorNotSupported;
}

}  // namespace iq2
