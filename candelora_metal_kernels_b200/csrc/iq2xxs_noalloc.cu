// iq2_matmul_noalloc: the decode GEMV (m <= 16) with its scratch space in a fixed array of this
// library instead of a caller-provided workspace.
//
// Who needs it: callers that cannot allocate device memory at the call site -- a host engine
// whose memory pool already owns the whole GPU (a cudaMalloc would fail or fragment it), a
// latency-critical decode loop that must not pay for cudaMalloc's implicit synchronisation, or a
// plain C binding that is handed tensor pointers and has no allocator to get a workspace from.
//
// The scratch is a file-scope __device__ array of IQ2_NOALLOC_SCRATCH_BYTES (8 MiB): every GPU
// that loads this library holds that much for the life of the process. In host code the array's
// name is only a host-side stand-in, so its device address is obtained with cudaGetSymbolAddress
// (with that device current) during the first call on the device -- and again after the device's
// context was replaced (cudaDeviceReset) -- and cached; make that first call outside any stream
// capture. All calls share the one array and it
// keeps the previous call's contents. Nothing in it needs to start at zero: the x-limb prep
// kernel writes every limb and scale before the GEMV reads them, and the GEMV keeps its partial
// sums in shared memory. Calls whose kernels overlap on the GPU (different streams, or different
// host threads without ordering) race on the array.
#include <cstdio>
#include <mutex>

#include "../../include/candelora_iq2.h"
#include "iq2xxs_internal.h"

namespace {

static __device__ __align__(256) uint8_t g_noalloc_scratch[IQ2_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
struct ScratchSlot {
    void* ctx = nullptr;  // the context the address belongs to
    void* ptr = nullptr;
};
ScratchSlot g_scratch[kMaxDevices];

// Device address of g_noalloc_scratch on the current device. It is looked up once per device
// and context: after cudaDeviceReset the device's next primary context holds a new copy of the
// array, and the first call in that context looks its address up again.
cudaError_t scratch_for_current_device(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    void* const ctx = iq2::current_context_handle();
    std::lock_guard<std::mutex> lock(g_setup_mu);
    ScratchSlot& slot = g_scratch[dev];
    if (slot.ptr == nullptr || slot.ctx != ctx) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return e;
        slot.ptr = p;
        slot.ctx = ctx;
    }
    *out = slot.ptr;
    return cudaSuccess;
}

}  // namespace

extern "C" int iq2_matmul_noalloc(const void* x, int x_dtype, uint32_t m, const uint8_t* weight_bytes,
                                  size_t weight_bytes_len, const uint8_t* weight_scales,
                                  size_t weight_scales_len, uint32_t out_dim, uint32_t in_dim, float* out,
                                  iq2_stream_t stream) {
    if (m > 16) {
        return iq2::capi_fail(IQ2_ERR_UNSUPPORTED,
                              "iq2_matmul_noalloc: m = %u, only the decode path (m <= 16) has a "
                              "no-allocation form",
                              m);
    }
    // Argument, device and buffer checks: exactly those of iq2_matmul (with no workspace, so the
    // caller-workspace check is skipped).
    int rc = iq2::capi_validate_matmul("iq2_matmul_noalloc", x, x_dtype, m, weight_bytes, weight_bytes_len,
                                       weight_scales, weight_scales_len, out_dim, in_dim, out);
    if (rc != IQ2_OK || m == 0) return rc;
    const int sms = iq2::capi_num_sms();
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e;
    if (iq2::gemv_fast_path_ok(m, in_dim, weight_bytes, weight_scales)) {
        const size_t need = iq2::gemv_workspace_size(m, out_dim, in_dim, sms);
        if (need > (size_t)IQ2_NOALLOC_SCRATCH_BYTES) {
            return iq2::capi_fail(IQ2_ERR_WORKSPACE,
                                  "iq2_matmul_noalloc: this problem needs %zu bytes of scratch, more than "
                                  "the library's fixed %zu",
                                  need, (size_t)IQ2_NOALLOC_SCRATCH_BYTES);
        }
        void* scratch = nullptr;
        e = scratch_for_current_device(&scratch);
        if (e != cudaSuccess) return iq2::capi_cuda_fail("iq2_matmul_noalloc: cudaGetSymbolAddress", e);
        e = iq2::launch_gemv(x, x_dtype, m, weight_bytes, weight_scales, out_dim, in_dim, out, scratch, sms, s);
    } else {
        // unaligned buffers take the generic kernel, which needs no scratch at all
        e = iq2::launch_gemv_generic(x, x_dtype, m, weight_bytes, weight_scales, out_dim, in_dim, out, sms, s);
    }
    if (e != cudaSuccess) return iq2::capi_cuda_fail("iq2_matmul_noalloc", e);
    return IQ2_OK;
}
