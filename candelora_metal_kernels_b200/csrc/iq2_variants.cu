// The other IQ formats of the reference's dispatcher (Iq2MatmulVariant, src/iq2_matmul.rs:31-75):
// IQ2_XS, IQ2_S and IQ3_S matmul and dense dequantisation on sm_100a.
//
// Block geometry per 256 weights (src/iq2_matmul.rs:15-29) and value formulas
// (decode_iq2_xs_value / decode_iq2_s_value / decode_iq3_s_value, src/metal_src/iq2_matmul.metal:736-866):
//   IQ2_XS  64 B + 10 B: u16 word per 8 weights = grid index (9 bits) | sign index (7 bits) << 9;
//           scale byte per 32 weights, low nibble for words 0-1, high for 2-3; dl = d(0.5+s)/4.
//   IQ2_S   72 B + 10 B: qs[0..31] grid low bytes, qs[32..63] sign bytes, qh[8] two high bits of
//           the grid index per 8 weights; scale nibble per 16 weights; dl = d(0.5+s)/4.
//   IQ3_S  104 B + 6 B:  qs[64] grid low bytes (4 weights each), qh[8] ninth index bits,
//           signs[32] one byte per 8 weights; scale nibble per 32 weights; dl = d(1+2s).
// Every weight dl * grid_byte * sign is exact in f32 (at most 22 significant bits), so the f16
// and bf16 dequantisations are the round-to-nearest-even of the exact value, as the reference's.
//
// These formats are outside the benchmarked IQ2_XXS path: one warp per (weight row, 8 tokens)
// decodes each 8-weight group to f32 once and applies it to the warp's tokens (f32 FMA); the
// lanes split the row's groups and reduce at the end.
#include "iq2xxs_common.cuh"
#include "iq2xxs_codebook.h"
#include "iq2_variant_grids.h"
#include "iq2xxs_internal.h"

namespace iq2 {

namespace {

enum : int { V_XS = 1, V_S = 2, V_3S = 3 };  // IQ2_VARIANT_* of the C ABI

template <int V>
struct Geom {
    static constexpr uint32_t BYTES = V == V_XS ? 64 : (V == V_S ? 72 : 104);
    static constexpr uint32_t SCALES = V == V_3S ? 6 : 10;
};

// The 8 f32 weights of group gi (0..31, weights 8*gi .. 8*gi+7) of one block.
template <int V>
__device__ __forceinline__ void decode8(const uint8_t* __restrict__ q, const uint8_t* __restrict__ s, uint32_t gi,
                                        float (&w)[8]) {
    const float d = half_bits_to_float((uint32_t)s[0] | ((uint32_t)s[1] << 8));
    const uint32_t ib32 = gi >> 2, sub = gi & 3;
    if (V == V_XS) {
        const uint32_t word = (uint32_t)q[ib32 * 8 + 2 * sub] | ((uint32_t)q[ib32 * 8 + 2 * sub + 1] << 8);
        const uint32_t sb = s[2 + ib32];
        const float dl = d * (0.5f + (float)(sub < 2 ? (sb & 15u) : (sb >> 4))) * 0.25f;
        const uint64_t grid = __ldg(IQ2XS_GRID + (word & 0x1FFu));
        const uint32_t sg = IQ2_KSIGNS[(word >> 9) & 0x7Fu];
#pragma unroll
        for (int j = 0; j < 8; ++j)
            w[j] = dl * (float)((grid >> (8 * j)) & 0xFF) * (((sg >> j) & 1u) ? -1.0f : 1.0f);
    } else if (V == V_S) {
        const uint32_t il = sub >> 1, h = sub & 1, off = 4 * ib32 + 2 * il;
        const uint32_t nib = (uint32_t)q[64 + ib32] >> (4 * il);
        const uint32_t idx = (uint32_t)q[off + h] | ((nib << (h ? 6 : 8)) & 0x300u);
        const uint32_t sg = q[32 + off + h];
        const float dl = d * (0.5f + (float)(((uint32_t)s[2 + ib32] >> (4 * il)) & 15u)) * 0.25f;
        const uint64_t grid = __ldg(IQ2S_GRID + idx);
#pragma unroll
        for (int j = 0; j < 8; ++j)
            w[j] = dl * (float)((grid >> (8 * j)) & 0xFF) * (((sg >> j) & 1u) ? -1.0f : 1.0f);
    } else {
        const uint32_t l = sub, qh = q[64 + ib32];
        const uint32_t nib = ((uint32_t)s[2 + ib32 / 2] >> (4 * (ib32 & 1))) & 15u;
        const float dl = d * (1.0f + 2.0f * (float)nib);
        const uint32_t i1 = (uint32_t)q[8 * ib32 + 2 * l] | (((qh >> (2 * l)) & 1u) << 8);
        const uint32_t i2 = (uint32_t)q[8 * ib32 + 2 * l + 1] | (((qh >> (2 * l + 1)) & 1u) << 8);
        const uint32_t sg = q[72 + 4 * ib32 + l];
        const uint32_t g1 = __ldg(IQ3S_GRID + i1), g2 = __ldg(IQ3S_GRID + i2);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            w[j] = dl * (float)((g1 >> (8 * j)) & 0xFF) * (((sg >> j) & 1u) ? -1.0f : 1.0f);
            w[4 + j] = dl * (float)((g2 >> (8 * j)) & 0xFF) * (((sg >> (4 + j)) & 1u) ? -1.0f : 1.0f);
        }
    }
}

template <int V, typename XT>
__global__ void __launch_bounds__(256) variant_matmul_kernel(const XT* __restrict__ x, const uint8_t* __restrict__ qs,
                                                             const uint8_t* __restrict__ sc, float* __restrict__ out,
                                                             uint32_t M, uint32_t N, uint32_t K, uint32_t nb) {
    const int lane = threadIdx.x & 31;
    const uint32_t mchunks = (M + 7) / 8;
    const size_t total = (size_t)N * mchunks;
    for (size_t wi = (blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5; wi < total;
         wi += (size_t)gridDim.x * blockDim.x / 32) {
        const uint32_t n = (uint32_t)(wi / mchunks), mc = (uint32_t)(wi % mchunks) * 8;
        float acc[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
        for (uint32_t g = lane; g < nb * 32; g += 32) {
            const uint32_t blk = g >> 5;
            const size_t bi = (size_t)n * nb + blk;
            float w[8];
            decode8<V>(qs + bi * Geom<V>::BYTES, sc + bi * Geom<V>::SCALES, g & 31, w);
            const size_t k0 = (size_t)g * 8;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const size_t k = k0 + j;
                if (k >= K) break;
#pragma unroll
                for (int mm = 0; mm < 8; ++mm)
                    if (mc + mm < M) acc[mm] = fmaf(to_f32(x[(size_t)(mc + mm) * K + k]), w[j], acc[mm]);
            }
        }
#pragma unroll
        for (int mm = 0; mm < 8; ++mm) {
            float v = acc[mm];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
            if (lane == 0 && mc + mm < M) out[(size_t)(mc + mm) * N + n] = v;
        }
    }
}

// One thread per 8-weight group; OUT_DTYPE 0 f32, 1 f16, 2 bf16 (round to nearest even).
template <int V, int OUT_DTYPE>
__global__ void __launch_bounds__(256) variant_dequant_kernel(const uint8_t* __restrict__ qs,
                                                              const uint8_t* __restrict__ sc, void* __restrict__ out,
                                                              uint32_t N, uint32_t K, uint32_t nb) {
    const size_t groups_per_row = (size_t)nb * 32, total = (size_t)N * groups_per_row;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const size_t n = i / groups_per_row, g = i % groups_per_row;
        const size_t bi = n * nb + g / 32;
        float w[8];
        decode8<V>(qs + bi * Geom<V>::BYTES, sc + bi * Geom<V>::SCALES, (uint32_t)(g & 31), w);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const size_t k = g * 8 + j;
            if (k >= K) break;
            const size_t o = n * K + k;
            if (OUT_DTYPE == 0) static_cast<float*>(out)[o] = w[j];
            else if (OUT_DTYPE == 1) static_cast<__half*>(out)[o] = __float2half_rn(w[j]);
            else static_cast<__nv_bfloat16*>(out)[o] = __float2bfloat16_rn(w[j]);
        }
    }
}

unsigned grid_for(size_t items, size_t per_block, int num_sms) {
    size_t blocks = (items + per_block - 1) / per_block;
    const size_t cap = (size_t)(num_sms > 0 ? num_sms : 148) * 16;
    if (blocks > cap) blocks = cap;
    return (unsigned)(blocks ? blocks : 1);
}

template <int V>
cudaError_t launch_matmul_v(const void* x, int x_dtype, uint32_t m, const uint8_t* qs, const uint8_t* sc, uint32_t n,
                            uint32_t k, float* out, int num_sms, cudaStream_t s) {
    const uint32_t nb = (k + QK - 1) / QK;
    const unsigned blocks = grid_for((size_t)n * ((m + 7) / 8), 8, num_sms);
    switch (x_dtype) {
        case 0: variant_matmul_kernel<V, float><<<blocks, 256, 0, s>>>(static_cast<const float*>(x), qs, sc, out, m, n, k, nb); break;
        case 1: variant_matmul_kernel<V, __half><<<blocks, 256, 0, s>>>(static_cast<const __half*>(x), qs, sc, out, m, n, k, nb); break;
        default: variant_matmul_kernel<V, __nv_bfloat16><<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), qs, sc, out, m, n, k, nb); break;
    }
    return cudaGetLastError();
}

template <int V>
cudaError_t launch_dequant_v(const uint8_t* qs, const uint8_t* sc, uint32_t n, uint32_t k, void* out, int out_dtype,
                             int num_sms, cudaStream_t s) {
    const uint32_t nb = (k + QK - 1) / QK;
    const unsigned blocks = grid_for((size_t)n * nb * 32, 256, num_sms);
    switch (out_dtype) {
        case 0: variant_dequant_kernel<V, 0><<<blocks, 256, 0, s>>>(qs, sc, out, n, k, nb); break;
        case 1: variant_dequant_kernel<V, 1><<<blocks, 256, 0, s>>>(qs, sc, out, n, k, nb); break;
        default: variant_dequant_kernel<V, 2><<<blocks, 256, 0, s>>>(qs, sc, out, n, k, nb); break;
    }
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_variant_matmul(int variant, const void* x, int x_dtype, uint32_t m, const uint8_t* qs,
                                  const uint8_t* sc, uint32_t n, uint32_t k, float* out, int num_sms,
                                  cudaStream_t stream) {
    if (m == 0) return cudaSuccess;
    switch (variant) {
        case V_XS: return launch_matmul_v<V_XS>(x, x_dtype, m, qs, sc, n, k, out, num_sms, stream);
        case V_S: return launch_matmul_v<V_S>(x, x_dtype, m, qs, sc, n, k, out, num_sms, stream);
        case V_3S: return launch_matmul_v<V_3S>(x, x_dtype, m, qs, sc, n, k, out, num_sms, stream);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_variant_dequant(int variant, const uint8_t* qs, const uint8_t* sc, uint32_t n, uint32_t k,
                                   void* out, int out_dtype, int num_sms, cudaStream_t stream) {
    switch (variant) {
        case V_XS: return launch_dequant_v<V_XS>(qs, sc, n, k, out, out_dtype, num_sms, stream);
        case V_S: return launch_dequant_v<V_S>(qs, sc, n, k, out, out_dtype, num_sms, stream);
        case V_3S: return launch_dequant_v<V_3S>(qs, sc, n, k, out, out_dtype, num_sms, stream);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace iq2
