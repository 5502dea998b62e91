// TEST INFRASTRUCTURE ONLY (parity checker and timed CPU baseline) -- never linked into the
// shipped library.
//
// Runs the reference's OWN Metal kernels on host cores. The two reference sources are
// included in place from the reference checkout (paths passed by oracle/Makefile as
// REF_TABLES_METAL / REF_MATMUL_METAL; nothing is copied into this repository), compiled as
// C++17 through the Metal stand-in header oracle/metal_shim/metal_stdlib, exactly in the
// order the reference concatenates them (src/iq2_matmul.rs:1316-1321: tables, then kernels).
//
// Each exported function plays the role of the Metal dispatch in the reference host code
// (src/iq2_matmul.rs:343-357 for the matmul, :487-501 for the dequant): one invocation of
// the kernel function per thread_position_in_grid value gid in [0, m*out_dim) (matmul) or
// [0, out_dim*in_dim) (dequant). Invocations are independent, so they are spread over host
// threads with OpenMP; each still executes the reference's own per-thread loop unchanged.
#include <metal_stdlib>
#include REF_TABLES_METAL
#include REF_MATMUL_METAL

#include <cstddef>
#include <cstdint>
#include <omp.h>

namespace {

template <typename T, typename K>
void run_matmul(K kernel, uint32_t m, uint32_t out_dim, uint32_t in_dim, const void* x,
                const uint8_t* w_bytes, const uint8_t* w_scales, float* out, int threads) {
    const uint m_ = m, out_ = out_dim, in_ = in_dim;
    const uint blocks = (in_dim + 255u) / 256u;
    const T* xt = static_cast<const T*>(x);
    const long long total = (long long)m * (long long)out_dim;
    if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel for schedule(dynamic, 16) num_threads(threads)
    for (long long gid = 0; gid < total; ++gid) {
        kernel(m_, out_, in_, blocks, xt, w_bytes, w_scales, out, (uint)gid);
    }
}

template <typename K>
void run_dequant(K kernel, uint32_t out_dim, uint32_t in_dim, const uint8_t* w_bytes,
                 const uint8_t* w_scales, uint16_t* out, int threads) {
    const uint out_ = out_dim, in_ = in_dim;
    const uint blocks = (in_dim + 255u) / 256u;
    half* o = reinterpret_cast<half*>(out);
    const long long total = (long long)out_dim * (long long)in_dim;
    if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel for schedule(static) num_threads(threads)
    for (long long gid = 0; gid < total; ++gid) {
        kernel(out_, in_, blocks, w_bytes, w_scales, o, (uint)gid);
    }
}

}  // namespace

static_assert(sizeof(half) == 2 && sizeof(bfloat) == 2, "16-bit stand-ins");

extern "C" {

// dtype: 0 = f32, 1 = f16, 2 = bf16 (x is raw 16-bit patterns for 1 and 2).
// variant: 0 = IQ2_XXS, 1 = IQ2_XS, 2 = IQ2_S, 3 = IQ3_S (src/iq2_matmul.rs:31-37).
// w8a8: 0 = ActivationQuantMode::Off kernels, 1 = the *_w8a8_* kernels.
int iq2ref_matmul(int variant, int w8a8, int dtype, uint32_t m, uint32_t out_dim, uint32_t in_dim,
                  const void* x, const uint8_t* w_bytes, const uint8_t* w_scales, float* out,
                  int threads) {
#define IQ2REF_DISPATCH(KERNEL)                                                                  \
    switch (dtype) {                                                                             \
        case 0: run_matmul<float>(KERNEL<float>, m, out_dim, in_dim, x, w_bytes, w_scales, out, \
                                  threads); return 0;                                           \
        case 1: run_matmul<half>(KERNEL<half>, m, out_dim, in_dim, x, w_bytes, w_scales, out,   \
                                 threads); return 0;                                            \
        case 2: run_matmul<bfloat>(KERNEL<bfloat>, m, out_dim, in_dim, x, w_bytes, w_scales,    \
                                   out, threads); return 0;                                     \
        default: return -1;                                                                      \
    }
    if (!w8a8) {
        switch (variant) {
            case 0: IQ2REF_DISPATCH(iq2_xxs_matmul_kernel)
            case 1: IQ2REF_DISPATCH(iq2_xs_matmul_kernel)
            case 2: IQ2REF_DISPATCH(iq2_s_matmul_kernel)
            case 3: IQ2REF_DISPATCH(iq3_s_matmul_kernel)
            default: return -2;
        }
    } else {
        switch (variant) {
            case 0: IQ2REF_DISPATCH(iq2_xxs_matmul_w8a8_kernel)
            case 1: IQ2REF_DISPATCH(iq2_xs_matmul_w8a8_kernel)
            case 2: IQ2REF_DISPATCH(iq2_s_matmul_w8a8_kernel)
            case 3: IQ2REF_DISPATCH(iq3_s_matmul_w8a8_kernel)
            default: return -2;
        }
    }
#undef IQ2REF_DISPATCH
}

// Dense f16 [out_dim, in_dim] (raw binary16 patterns), the reference's *_dequantize_f16 kernels.
int iq2ref_dequantize_f16(int variant, uint32_t out_dim, uint32_t in_dim, const uint8_t* w_bytes,
                          const uint8_t* w_scales, uint16_t* out, int threads) {
    switch (variant) {
        case 0: run_dequant(iq2_xxs_dequantize_f16_kernel, out_dim, in_dim, w_bytes, w_scales, out, threads); return 0;
        case 1: run_dequant(iq2_xs_dequantize_f16_kernel, out_dim, in_dim, w_bytes, w_scales, out, threads); return 0;
        case 2: run_dequant(iq2_s_dequantize_f16_kernel, out_dim, in_dim, w_bytes, w_scales, out, threads); return 0;
        case 3: run_dequant(iq3_s_dequantize_f16_kernel, out_dim, in_dim, w_bytes, w_scales, out, threads); return 0;
        default: return -2;
    }
}

int iq2ref_max_threads(void) { return omp_get_max_threads(); }

}  // extern "C"
