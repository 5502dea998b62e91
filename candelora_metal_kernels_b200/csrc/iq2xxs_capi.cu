// C ABI of the IQ2_XXS matmul (declared in include/candelora_iq2.h).
//
// Validation follows the reference's host dispatch iq2_matmul_metal (src/iq2_matmul.rs:197-365)
// and iq2_dequantize_to_f16_metal (:367-505): the same conditions fail, in the same order, with
// the same messages where the reference has one ("Metal" reads "CUDA"). Shape parsing of x
// (rank 1 / rank 2, src/iq2_matmul.rs:170-195) belongs to the tensor-level host bindings; here
// x is already [m, in_dim].
#include <atomic>
#include <cinttypes>
#include <cstdarg>
#include <cstdio>
#include <algorithm>
#include <string>
#include <vector>

#include "../../include/candelora_iq2.h"
#include "../../include/candelora_iq2_testing.h"
#include "iq2xxs_internal.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int cuda_fail(const char* what, cudaError_t e) {
    return fail(IQ2_ERR_CUDA, "%s: CUDA error %d (%s)", what, (int)e, cudaGetErrorString(e));
}

// Per-device SM count, read once per device.
std::atomic<int> g_num_sms[64];

int num_sms_for_current_device() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return 148;
    if (dev >= 64) {
        int v = 0;
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        return v > 0 ? v : 148;
    }
    int v = g_num_sms[dev].load(std::memory_order_relaxed);
    if (v <= 0) {
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
        g_num_sms[dev].store(v, std::memory_order_relaxed);
    }
    return v;
}

// Where a pointer lives: -1 = not device memory, otherwise the device ordinal.
int pointer_device(const void* p) {
    cudaPointerAttributes a;
    cudaError_t e = cudaPointerGetAttributes(&a, p);
    if (e != cudaSuccess) {
        cudaGetLastError();  // clear the sticky-free error state of this query
        return -1;
    }
    if (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) return a.device;
    return -1;
}

std::string where(int dev) {
    if (dev < 0) return "Cpu";
    char b[32];
    snprintf(b, sizeof(b), "Cuda(%d)", dev);
    return b;
}

// Common validation of the weight buffers (src/iq2_matmul.rs:210-259 / :380-424).
int check_weights(const char* op, const uint8_t* weight_bytes, size_t weight_bytes_len,
                  const uint8_t* weight_scales, size_t weight_scales_len, uint32_t out_dim,
                  uint32_t in_dim, int variant, int dev_expected, const void* x) {
    if (weight_bytes == nullptr || weight_scales == nullptr)
        return fail(IQ2_ERR_INVALID_ARGUMENT, "%s: NULL weight pointer", op);
    const int db = pointer_device(weight_bytes), ds = pointer_device(weight_scales);
    const int dx = x ? pointer_device(x) : db;
    if ((x ? dx : db) < 0) return fail(IQ2_ERR_DEVICE, "%s requires a CUDA device", op);
    if (dx != db || dx != ds || dx != dev_expected) {
        if (x)
            return fail(IQ2_ERR_DEVICE, "%s device mismatch: x=%s, bytes=%s, scales=%s", op,
                        where(dx).c_str(), where(db).c_str(), where(ds).c_str());
        return fail(IQ2_ERR_DEVICE, "%s device mismatch: bytes=%s, scales=%s", op,
                    where(db).c_str(), where(ds).c_str());
    }
    const uint64_t blocks_per_row = ((uint64_t)in_dim + 255u) / 256u;
    // bytes / scale bytes per block (src/iq2_matmul.rs:14-29)
    static const uint64_t kBytes[4] = {64, 64, 72, 104}, kScales[4] = {2, 10, 10, 6};
    const uint64_t per_block_bytes = kBytes[variant], per_block_scales = kScales[variant];
    const uint64_t nblocks = (uint64_t)out_dim * blocks_per_row;  // < 2^56, cannot overflow
    const uint64_t expected_bytes = nblocks * per_block_bytes;
    const uint64_t expected_scales = nblocks * per_block_scales;
    if (expected_bytes > (uint64_t)SIZE_MAX) return fail(IQ2_ERR_OVERFLOW, "%s bytes size overflow", op);
    if (weight_bytes_len < expected_bytes)
        return fail(IQ2_ERR_TOO_SMALL, "%s weight_bytes too small: got %zu expected at least %" PRIu64, op,
                    weight_bytes_len, expected_bytes);
    if (weight_scales_len < expected_scales)
        return fail(IQ2_ERR_TOO_SMALL, "%s weight_scales too small: got %zu expected at least %" PRIu64, op,
                    weight_scales_len, expected_scales);
    return IQ2_OK;
}

// Checks that need no CUDA call, in the reference's order (zero dims first, :210-212).
int check_args(const char* op, uint32_t out_dim, uint32_t in_dim, int variant) {
    if (out_dim == 0 || in_dim == 0) return fail(IQ2_ERR_ZERO_DIM, "%s expects non-zero dimensions", op);
    if (variant < IQ2_VARIANT_IQ2_XXS || variant > IQ2_VARIANT_IQ3_S)
        return fail(IQ2_ERR_INVALID_ARGUMENT, "%s: unknown variant %d", op, variant);
    return IQ2_OK;
}

// The current device, or IQ2_ERR_DEVICE when there is none (the reference's "requires a Metal
// device", :213-215).
int current_device(const char* op, int* dev) {
    cudaError_t e = cudaGetDevice(dev);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(IQ2_ERR_DEVICE, "%s requires a CUDA device (%s)", op, cudaGetErrorString(e));
    }
    return IQ2_OK;
}

size_t workspace_for(uint32_t m, uint32_t out_dim, uint32_t in_dim, int x_dtype, int num_sms) {
    if (m == 0 || out_dim == 0 || in_dim == 0) return 0;
    if (m <= iq2::kGemvMaxM) return iq2::gemv_workspace_size(m, out_dim, in_dim, num_sms);
    return iq2::gemm_workspace_size(m, out_dim, in_dim, x_dtype, num_sms);
}

int matmul_impl(const char* op, const void* x, int x_dtype, uint32_t m, const uint8_t* weight_bytes,
                size_t weight_bytes_len, const uint8_t* weight_scales, size_t weight_scales_len,
                uint32_t out_dim, uint32_t in_dim, int variant, float* out, void* workspace,
                size_t workspace_bytes, iq2_stream_t stream) {
    int rc = check_args(op, out_dim, in_dim, variant);
    if (rc != IQ2_OK) return rc;
    int dev = 0;
    if ((rc = current_device(op, &dev)) != IQ2_OK) return rc;
    cudaError_t e = cudaSuccess;
    if (m > 0 && x == nullptr) return fail(IQ2_ERR_INVALID_ARGUMENT, "%s: NULL x", op);
    rc = check_weights(op, weight_bytes, weight_bytes_len, weight_scales, weight_scales_len,
                           out_dim, in_dim, variant, dev, m > 0 ? x : nullptr);
    if (rc != IQ2_OK) return rc;
    if (x_dtype < IQ2_DTYPE_F32 || x_dtype > IQ2_DTYPE_BF16)
        return fail(IQ2_ERR_DTYPE, "%s unsupported x dtype: %d", op, x_dtype);
    if (m == 0) return IQ2_OK;  // empty [0, out_dim] output: nothing to launch (:261-268)
    if (out == nullptr) return fail(IQ2_ERR_INVALID_ARGUMENT, "%s: NULL out", op);
    if (pointer_device(out) != dev) return fail(IQ2_ERR_DEVICE, "%s: out is not memory of Cuda(%d)", op, dev);
    const size_t esize = x_dtype == IQ2_DTYPE_F32 ? 4 : 2;
    if (reinterpret_cast<uintptr_t>(x) % esize != 0 || reinterpret_cast<uintptr_t>(out) % 4 != 0)
        return fail(IQ2_ERR_INVALID_ARGUMENT, "%s: x/out not aligned to their element size", op);
    const int sms = num_sms_for_current_device();
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (variant != IQ2_VARIANT_IQ2_XXS) {
        // the other formats: the tensor-core GEMM for m > kGemvMaxM when the caller gives the
        // workspace iq2_matmul_workspace_size asks for; else the f32 CUDA-core kernel (no workspace)
        const bool gemm = m > iq2::kGemvMaxM &&
                          iq2::gemm_path_ok(m, out_dim, in_dim, x, x_dtype, weight_bytes, weight_scales, out) &&
                          workspace != nullptr &&
                          workspace_bytes >= iq2::gemm_workspace_size(m, out_dim, in_dim, x_dtype, sms);
        // IQ2_XS, IQ2_S and IQ3_S with m <= kGemvMaxM: the IQ2_XXS decode GEMV's int8 tensor-core
        // decode, likewise when the call has its workspace
        const bool gemv = iq2::gemv_variant_ok(variant) && m <= iq2::kGemvMaxM &&
                          iq2::gemv_fast_path_ok(m, in_dim, weight_bytes, weight_scales) && workspace != nullptr &&
                          workspace_bytes >= iq2::gemv_variant_workspace_size(variant, m, out_dim, in_dim);
        if (gemm)
            e = iq2::launch_gemm(x, x_dtype, m, weight_bytes, weight_scales, out_dim, in_dim, out, workspace, sms, s,
                                 variant);
        else if (gemv)
            e = iq2::launch_gemv_variant(variant, x, x_dtype, m, weight_bytes, weight_scales, out_dim, in_dim, out,
                                         workspace, sms, s);
        else
            e = iq2::launch_variant_matmul(variant, x, x_dtype, m, weight_bytes, weight_scales, out_dim, in_dim, out,
                                           sms, s);
    } else if (m <= iq2::kGemvMaxM) {
        if (iq2::gemv_fast_path_ok(m, in_dim, weight_bytes, weight_scales)) {
            const size_t need = iq2::gemv_workspace_size(m, out_dim, in_dim, sms);
            if (need > 0 && (workspace == nullptr || workspace_bytes < need))
                return fail(IQ2_ERR_WORKSPACE, "%s: workspace of %zu bytes needed, got %zu", op, need,
                            workspace ? workspace_bytes : (size_t)0);
            e = iq2::launch_gemv(x, x_dtype, m, weight_bytes, weight_scales, out_dim, in_dim, out,
                                 workspace, sms, s);
        } else {
            e = iq2::launch_gemv_generic(x, x_dtype, m, weight_bytes, weight_scales, out_dim, in_dim,
                                         out, sms, s);
        }
    } else if (iq2::gemm_path_ok(m, out_dim, in_dim, x, x_dtype, weight_bytes, weight_scales, out)) {
        const size_t need = iq2::gemm_workspace_size(m, out_dim, in_dim, x_dtype, sms);
        if (need > 0 && (workspace == nullptr || workspace_bytes < need))
            return fail(IQ2_ERR_WORKSPACE, "%s: workspace of %zu bytes needed, got %zu", op, need,
                        workspace ? workspace_bytes : (size_t)0);
        e = iq2::launch_gemm(x, x_dtype, m, weight_bytes, weight_scales, out_dim, in_dim, out,
                             workspace, sms, s);
    } else {
        e = iq2::launch_gemv_generic(x, x_dtype, m, weight_bytes, weight_scales, out_dim, in_dim,
                                     out, sms, s);
    }
    if (e != cudaSuccess) return cuda_fail(op, e);
    return IQ2_OK;
}

// Splits a grouped call into launches: fast-path problems in chunks of gemv_max_group() when
// m <= kGemvMaxM; everything else one by one. With `ws` NULL only sizes the workspace.
int grouped_impl(const iq2_matmul_problem* probs, uint32_t count, uint32_t m, int x_dtype, void* ws,
                 size_t ws_bytes, iq2_stream_t stream, size_t* need_out) {
    const char* op = "iq2_matmul_grouped";
    const int sms = num_sms_for_current_device();
    size_t need = 0;
    std::vector<iq2::GemvProblemHost> fast;
    std::vector<uint32_t> slow;
    for (uint32_t i = 0; i < count; ++i) {
        const iq2_matmul_problem& p = probs[i];
        if (iq2::gemv_fast_path_ok(m, p.in_dim, p.weight_bytes, p.weight_scales)) {
            fast.push_back({p.x, p.weight_bytes, p.weight_scales, p.out_dim, p.in_dim, p.out});
        } else {
            slow.push_back(i);
            need = std::max(need, workspace_for(m, p.out_dim, p.in_dim, x_dtype, sms));
        }
    }
    const uint32_t chunk = iq2::gemv_max_group();
    for (size_t c0 = 0; c0 < fast.size(); c0 += chunk) {
        const uint32_t n = (uint32_t)std::min<size_t>(chunk, fast.size() - c0);
        need = std::max(need, iq2::gemv_group_workspace_size(fast.data() + c0, n, m, sms));
    }
    if (need_out) *need_out = need;
    if (ws == nullptr && need_out) return IQ2_OK;
    if (need > 0 && (ws == nullptr || ws_bytes < need))
        return fail(IQ2_ERR_WORKSPACE, "%s: workspace of %zu bytes needed, got %zu", op, need,
                    ws ? ws_bytes : (size_t)0);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    for (size_t c0 = 0; c0 < fast.size(); c0 += chunk) {
        const uint32_t n = (uint32_t)std::min<size_t>(chunk, fast.size() - c0);
        cudaError_t e = iq2::launch_gemv_group(fast.data() + c0, n, m, x_dtype, ws, sms, s);
        if (e != cudaSuccess) return cuda_fail(op, e);
    }
    for (uint32_t i : slow) {
        const iq2_matmul_problem& p = probs[i];
        int rc = matmul_impl(op, p.x, x_dtype, m, p.weight_bytes, p.weight_bytes_len, p.weight_scales,
                             p.weight_scales_len, p.out_dim, p.in_dim, IQ2_VARIANT_IQ2_XXS, p.out, ws,
                             ws_bytes, stream);
        if (rc != IQ2_OK) return rc;
    }
    return IQ2_OK;
}

}  // namespace

// Helpers shared with iq2xxs_noalloc.cu (declared in iq2xxs_internal.h).
namespace iq2 {

void* current_context_handle() {
    using CtxGetCurrentFn = int (*)(void**);  // CUresult cuCtxGetCurrent(CUcontext*)
    static const CtxGetCurrentFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<CtxGetCurrentFn>(p);
    }();
    void* ctx = nullptr;
    if (fn == nullptr || fn(&ctx) != 0) return nullptr;
    return ctx;
}

int capi_fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int capi_cuda_fail(const char* what, cudaError_t e) { return cuda_fail(what, e); }

int capi_ok() {
    g_last_error.clear();
    return IQ2_OK;
}

int capi_num_sms() { return num_sms_for_current_device(); }

// The checks iq2_matmul makes before choosing a kernel (clears the thread's error message first).
int capi_validate_matmul(const char* op, const void* x, int x_dtype, uint32_t m, const uint8_t* weight_bytes,
                         size_t weight_bytes_len, const uint8_t* weight_scales, size_t weight_scales_len,
                         uint32_t out_dim, uint32_t in_dim, const float* out, int variant) {
    g_last_error.clear();
    int rc = check_args(op, out_dim, in_dim, variant);
    if (rc != IQ2_OK) return rc;
    int dev = 0;
    if ((rc = current_device(op, &dev)) != IQ2_OK) return rc;
    if (m > 0 && x == nullptr) return fail(IQ2_ERR_INVALID_ARGUMENT, "%s: NULL x", op);
    rc = check_weights(op, weight_bytes, weight_bytes_len, weight_scales, weight_scales_len, out_dim, in_dim,
                       variant, dev, m > 0 ? x : nullptr);
    if (rc != IQ2_OK) return rc;
    if (x_dtype < IQ2_DTYPE_F32 || x_dtype > IQ2_DTYPE_BF16)
        return fail(IQ2_ERR_DTYPE, "%s unsupported x dtype: %d", op, x_dtype);
    if (m == 0) return IQ2_OK;
    if (out == nullptr) return fail(IQ2_ERR_INVALID_ARGUMENT, "%s: NULL out", op);
    if (pointer_device(out) != dev) return fail(IQ2_ERR_DEVICE, "%s: out is not memory of Cuda(%d)", op, dev);
    const size_t esize = x_dtype == IQ2_DTYPE_F32 ? 4 : 2;
    if (reinterpret_cast<uintptr_t>(x) % esize != 0 || reinterpret_cast<uintptr_t>(out) % 4 != 0)
        return fail(IQ2_ERR_INVALID_ARGUMENT, "%s: x/out not aligned to their element size", op);
    return IQ2_OK;
}

}  // namespace iq2

extern "C" {

const char* iq2_last_error(void) { return g_last_error.c_str(); }

int iq2_abi_version(void) { return IQ2_ABI_VERSION; }

int iq2_device_check(void) {
    g_last_error.clear();
    unsigned int status = 0;
    const cudaError_t e = (cudaError_t)iq2::gemm_take_status(&status);
    if (e != cudaSuccess) return cuda_fail("iq2_device_check", e);
    if (status != 0u)
        return fail(IQ2_ERR_TIMEOUT,
                    "iq2_device_check: a prefill GEMM gave up on a pipeline wait (status 0x%x:%s%s%s%s%s%s); the "
                    "outputs of that call are incomplete",
                    status, (status & 1u) ? " x producer" : "", (status & 2u) ? " x tile" : "",
                    (status & 4u) ? " decoded weights" : "", (status & 8u) ? " stage release" : "",
                    (status & 16u) ? " accumulator" : "", (status & 32u) ? " x tile after abort" : "");
    return IQ2_OK;
}

int iq2_testing_set_gemm_stall(uint64_t wait_limit_ns, uint32_t stall_stage) {
    g_last_error.clear();
    iq2::gemm_testing_set_stall(wait_limit_ns, stall_stage);
    return IQ2_OK;
}

size_t iq2_matmul_workspace_size(uint32_t m, uint32_t out_dim, uint32_t in_dim, int x_dtype,
                                 int variant) {
    if (variant < IQ2_VARIANT_IQ2_XXS || variant > IQ2_VARIANT_IQ3_S) return 0;
    if (variant != IQ2_VARIANT_IQ2_XXS && m <= iq2::kGemvMaxM)  // the other formats: their decode GEMV's x limbs
        return iq2::gemv_variant_ok(variant) && m > 0 && out_dim > 0 && in_dim > 0
                   ? iq2::gemv_variant_workspace_size(variant, m, out_dim, in_dim)
                   : 0;
    return workspace_for(m, out_dim, in_dim, x_dtype, num_sms_for_current_device());
}

int iq2_matmul(const void* x, int x_dtype, uint32_t m, const uint8_t* weight_bytes,
               size_t weight_bytes_len, const uint8_t* weight_scales, size_t weight_scales_len,
               uint32_t out_dim, uint32_t in_dim, int variant, float* out, void* workspace,
               size_t workspace_bytes, iq2_stream_t stream) {
    g_last_error.clear();
    return matmul_impl("iq2_matmul", x, x_dtype, m, weight_bytes, weight_bytes_len, weight_scales,
                       weight_scales_len, out_dim, in_dim, variant, out, workspace, workspace_bytes,
                       stream);
}

int iq2_matmul_with_activation_quant(const void* x, int x_dtype, uint32_t m,
                                     const uint8_t* weight_bytes, size_t weight_bytes_len,
                                     const uint8_t* weight_scales, size_t weight_scales_len,
                                     uint32_t out_dim, uint32_t in_dim, int variant, int act_mode,
                                     int strict, float* out, void* workspace,
                                     size_t workspace_bytes, iq2_stream_t stream) {
    g_last_error.clear();
    switch (act_mode) {
        case IQ2_ACT_QUANT_OFF:
            break;
        case IQ2_ACT_QUANT_W8A8: {
            // the reference's W8A8 kernels (src/iq2_matmul.rs:572-580 -> iq2_matmul.metal:437-499):
            // each x row quantised to int8 and back, then the float matmul of those values
            const char* op = "iq2_matmul";
            int rc = check_args(op, out_dim, in_dim, variant);
            if (rc != IQ2_OK) return rc;
            rc = iq2::capi_validate_matmul(op, x, x_dtype, m, weight_bytes, weight_bytes_len, weight_scales,
                                           weight_scales_len, out_dim, in_dim, out, variant);
            if (rc != IQ2_OK || m == 0) return rc;
            if (variant == IQ2_VARIANT_IQ2_XXS && m <= iq2::kGemvW8A8MaxM &&
                iq2::gemv_fast_path_ok(m, in_dim, weight_bytes, weight_scales)) {
                // decode: the int8 activations go straight into the GEMV as its single limb
                const size_t need = iq2::gemv_w8a8_workspace_size(m, out_dim, in_dim);
                if (need > 0 && (workspace == nullptr || workspace_bytes < need))
                    return fail(IQ2_ERR_WORKSPACE, "%s: workspace of %zu bytes needed, got %zu", op, need,
                                workspace ? workspace_bytes : (size_t)0);
                const cudaError_t e = iq2::launch_gemv_w8a8(x, x_dtype, m, weight_bytes, weight_scales, out_dim, in_dim,
                                                            out, workspace, num_sms_for_current_device(),
                                                            reinterpret_cast<cudaStream_t>(stream));
                if (e != cudaSuccess) return cuda_fail(op, e);
                return IQ2_OK;
            }
            const size_t xq_bytes = ((size_t)m * in_dim * sizeof(float) + 255) / 256 * 256;
            const size_t need = xq_bytes + (variant == IQ2_VARIANT_IQ2_XXS
                                                ? workspace_for(m, out_dim, in_dim, IQ2_DTYPE_F32, num_sms_for_current_device())
                                                : 0);
            if (workspace == nullptr || workspace_bytes < need)
                return fail(IQ2_ERR_WORKSPACE, "%s: workspace of %zu bytes needed, got %zu", op, need,
                            workspace ? workspace_bytes : (size_t)0);
            float* xq = static_cast<float*>(workspace);
            const cudaError_t e = iq2::launch_qdq_w8a8(x, x_dtype, m, in_dim, xq, reinterpret_cast<cudaStream_t>(stream));
            if (e != cudaSuccess) return cuda_fail(op, e);
            return matmul_impl(op, xq, IQ2_DTYPE_F32, m, weight_bytes, weight_bytes_len, weight_scales,
                               weight_scales_len, out_dim, in_dim, variant, out,
                               static_cast<uint8_t*>(workspace) + xq_bytes, workspace_bytes - xq_bytes, stream);
        }
        case IQ2_ACT_QUANT_W4A8:
            if (strict)
                return fail(IQ2_ERR_UNSUPPORTED,
                            "activation quant mode W4A8 requested in strict mode, but W4A8 kernel "
                            "path is not implemented yet");
            break;  // non-strict W4A8 falls back to the float path (src/iq2_matmul.rs:581-589)
        default:
            return fail(IQ2_ERR_INVALID_ARGUMENT, "unknown activation quant mode %d", act_mode);
    }
    return matmul_impl("iq2_matmul", x, x_dtype, m, weight_bytes, weight_bytes_len, weight_scales,
                       weight_scales_len, out_dim, in_dim, variant, out, workspace, workspace_bytes,
                       stream);
}

size_t iq2_matmul_with_activation_quant_workspace_size(uint32_t m, uint32_t out_dim, uint32_t in_dim,
                                                      int x_dtype, int variant, int act_mode) {
    if (act_mode != IQ2_ACT_QUANT_W8A8) return iq2_matmul_workspace_size(m, out_dim, in_dim, x_dtype, variant);
    if (m == 0 || out_dim == 0 || in_dim == 0 || variant < IQ2_VARIANT_IQ2_XXS || variant > IQ2_VARIANT_IQ3_S) return 0;
    // (the other formats: their GEMM's workspace after the int8-rounded x, which selects the
    // tensor-core path for m > kGemvMaxM; the call itself only requires the x part)
    const size_t qdq = ((size_t)m * in_dim * sizeof(float) + 255) / 256 * 256 +
                       iq2_matmul_workspace_size(m, out_dim, in_dim, IQ2_DTYPE_F32, variant);
    // the decode path (int8 activations into the GEMV) needs less; the larger of the two is asked
    // for so that either path can run with it
    const size_t gemv = (variant == IQ2_VARIANT_IQ2_XXS && m <= iq2::kGemvW8A8MaxM)
                            ? iq2::gemv_w8a8_workspace_size(m, out_dim, in_dim)
                            : 0;
    return std::max(qdq, gemv);
}

size_t iq2_matmul_grouped_workspace_size(const iq2_matmul_problem* problems, uint32_t count,
                                         uint32_t m, int x_dtype) {
    if (problems == nullptr || count == 0 || m == 0) return 0;
    size_t need = 0;
    grouped_impl(problems, count, m, x_dtype, nullptr, 0, nullptr, &need);
    return need;
}

int iq2_matmul_grouped(const iq2_matmul_problem* problems, uint32_t count, uint32_t m, int x_dtype,
                       void* workspace, size_t workspace_bytes, iq2_stream_t stream) {
    g_last_error.clear();
    const char* op = "iq2_matmul_grouped";
    if (count == 0) return IQ2_OK;
    if (problems == nullptr) return fail(IQ2_ERR_INVALID_ARGUMENT, "%s: NULL problems", op);
    if (x_dtype < IQ2_DTYPE_F32 || x_dtype > IQ2_DTYPE_BF16)
        return fail(IQ2_ERR_DTYPE, "%s unsupported x dtype: %d", op, x_dtype);
    int dev = 0;
    int rc = current_device(op, &dev);
    if (rc != IQ2_OK) return rc;
    // every problem is validated like a single iq2_matmul call before anything is launched
    for (uint32_t i = 0; i < count; ++i) {
        const iq2_matmul_problem& p = problems[i];
        if ((rc = check_args(op, p.out_dim, p.in_dim, IQ2_VARIANT_IQ2_XXS)) != IQ2_OK) return rc;
        if (m > 0 && p.x == nullptr) return fail(IQ2_ERR_INVALID_ARGUMENT, "%s: problem %u: NULL x", op, i);
        rc = check_weights(op, p.weight_bytes, p.weight_bytes_len, p.weight_scales, p.weight_scales_len,
                           p.out_dim, p.in_dim, IQ2_VARIANT_IQ2_XXS, dev, m > 0 ? p.x : nullptr);
        if (rc != IQ2_OK) return rc;
        if (m == 0) continue;
        if (p.out == nullptr || pointer_device(p.out) != dev)
            return fail(IQ2_ERR_DEVICE, "%s: problem %u: out is not memory of Cuda(%d)", op, i, dev);
        const size_t esize = x_dtype == IQ2_DTYPE_F32 ? 4 : 2;
        if (reinterpret_cast<uintptr_t>(p.x) % esize != 0 || reinterpret_cast<uintptr_t>(p.out) % 4 != 0)
            return fail(IQ2_ERR_INVALID_ARGUMENT, "%s: problem %u: x/out not aligned to their element size", op, i);
    }
    if (m == 0) return IQ2_OK;
    return grouped_impl(problems, count, m, x_dtype, workspace, workspace_bytes, stream, nullptr);
}

int iq2_dequantize(const uint8_t* weight_bytes, size_t weight_bytes_len,
                   const uint8_t* weight_scales, size_t weight_scales_len, uint32_t out_dim,
                   uint32_t in_dim, int variant, void* out, int out_dtype, iq2_stream_t stream) {
    g_last_error.clear();
    const char* op = "iq2_dequantize_to_f16";
    int rc = check_args(op, out_dim, in_dim, variant);
    if (rc != IQ2_OK) return rc;
    int dev = 0;
    if ((rc = current_device(op, &dev)) != IQ2_OK) return rc;
    cudaError_t e = cudaSuccess;
    rc = check_weights(op, weight_bytes, weight_bytes_len, weight_scales, weight_scales_len,
                           out_dim, in_dim, variant, dev, nullptr);
    if (rc != IQ2_OK) return rc;
    if (out_dtype < IQ2_DTYPE_F32 || out_dtype > IQ2_DTYPE_BF16)
        return fail(IQ2_ERR_DTYPE, "%s unsupported out dtype: %d", op, out_dtype);
    if (out == nullptr) return fail(IQ2_ERR_INVALID_ARGUMENT, "%s: NULL out", op);
    if (pointer_device(out) != dev) return fail(IQ2_ERR_DEVICE, "%s: out is not memory of Cuda(%d)", op, dev);
    const size_t esize = out_dtype == IQ2_DTYPE_F32 ? 4 : 2;
    if (reinterpret_cast<uintptr_t>(out) % esize != 0)
        return fail(IQ2_ERR_INVALID_ARGUMENT, "%s: out not aligned to its element size", op);
    if (variant == IQ2_VARIANT_IQ2_XXS)
        e = iq2::launch_dequant(weight_bytes, weight_scales, out_dim, in_dim, out, out_dtype,
                                num_sms_for_current_device(), reinterpret_cast<cudaStream_t>(stream));
    else
        e = iq2::launch_variant_dequant(variant, weight_bytes, weight_scales, out_dim, in_dim, out, out_dtype,
                                        num_sms_for_current_device(), reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(op, e);
    return IQ2_OK;
}

int iq2_split_interleaved(const uint8_t* blocks, size_t blocks_len, uint64_t nblocks, int variant,
                          uint8_t* weight_bytes, uint8_t* weight_scales, iq2_stream_t stream) {
    g_last_error.clear();
    const char* op = "iq2_split_interleaved";
    if (variant < IQ2_VARIANT_IQ2_XXS || variant > IQ2_VARIANT_IQ3_S)
        return fail(IQ2_ERR_INVALID_ARGUMENT, "%s: unknown variant %d", op, variant);
    if (nblocks == 0) return IQ2_OK;
    static const uint32_t kBytes[4] = {64, 64, 72, 104}, kScales[4] = {2, 10, 10, 6};
    const uint64_t need = nblocks * (uint64_t)(kBytes[variant] + kScales[variant]);
    if (blocks == nullptr || weight_bytes == nullptr || weight_scales == nullptr)
        return fail(IQ2_ERR_INVALID_ARGUMENT, "%s: NULL pointer", op);
    if (blocks_len < need)
        return fail(IQ2_ERR_TOO_SMALL, "%s: blocks too small: got %zu expected at least %" PRIu64, op, blocks_len, need);
    int dev = 0;
    int rc = current_device(op, &dev);
    if (rc != IQ2_OK) return rc;
    if (pointer_device(blocks) != dev || pointer_device(weight_bytes) != dev || pointer_device(weight_scales) != dev)
        return fail(IQ2_ERR_DEVICE, "%s: buffers are not memory of Cuda(%d)", op, dev);
    const cudaError_t e = iq2::launch_split_interleaved(blocks, nblocks, kBytes[variant], kScales[variant], weight_bytes,
                                                        weight_scales, num_sms_for_current_device(),
                                                        reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(op, e);
    return IQ2_OK;
}

int iq2_gather_columns(const float* gathered, uint32_t shards, uint32_t m, uint32_t shard_cols,
                       float* out, iq2_stream_t stream) {
    g_last_error.clear();
    if (shards == 0 || m == 0 || shard_cols == 0) return IQ2_OK;
    if (gathered == nullptr || out == nullptr)
        return fail(IQ2_ERR_INVALID_ARGUMENT, "iq2_gather_columns: NULL pointer");
    int dev = 0;
    cudaGetDevice(&dev);
    if (pointer_device(gathered) != dev || pointer_device(out) != dev)
        return fail(IQ2_ERR_DEVICE, "iq2_gather_columns: buffers are not memory of Cuda(%d)", dev);
    cudaError_t e = iq2::launch_gather_columns(gathered, shards, m, shard_cols, out,
                                               num_sms_for_current_device(),
                                               reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail("iq2_gather_columns", e);
    return IQ2_OK;
}

}  // extern "C"
