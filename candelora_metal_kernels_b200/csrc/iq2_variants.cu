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
// These formats are outside the benchmarked IQ2_XXS path: one warp per (weight row, up to 8
// tokens) walks the row two blocks at a time, lane l decoding group l of each block (8 weights)
// to f32 from decode tables staged in shared memory and applying it to the warp's tokens with
// f32 FMAs on x read as 16-byte vectors; the lanes reduce at the end.
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
                                        float (&w)[8], const uint64_t* __restrict__ g64,
                                        const uint32_t* __restrict__ g32, const uint8_t* __restrict__ ks) {
    const float d = half_bits_to_float((uint32_t)s[0] | ((uint32_t)s[1] << 8));
    const uint32_t ib32 = gi >> 2, sub = gi & 3;
    if (V == V_XS) {
        const uint32_t word = (uint32_t)q[ib32 * 8 + 2 * sub] | ((uint32_t)q[ib32 * 8 + 2 * sub + 1] << 8);
        const uint32_t sb = s[2 + ib32];
        const float dl = d * (0.5f + (float)(sub < 2 ? (sb & 15u) : (sb >> 4))) * 0.25f;
        const uint64_t grid = g64[word & 0x1FFu];
        const uint32_t sg = ks[(word >> 9) & 0x7Fu];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float p = dl * (float)((grid >> (8 * j)) & 0xFF);
            w[j] = ((sg >> j) & 1u) ? -p : p;
        }
    } else if (V == V_S) {
        const uint32_t il = sub >> 1, h = sub & 1, off = 4 * ib32 + 2 * il;
        const uint32_t nib = (uint32_t)q[64 + ib32] >> (4 * il);
        const uint32_t idx = (uint32_t)q[off + h] | ((nib << (h ? 6 : 8)) & 0x300u);
        const uint32_t sg = q[32 + off + h];
        const float dl = d * (0.5f + (float)(((uint32_t)s[2 + ib32] >> (4 * il)) & 15u)) * 0.25f;
        const uint64_t grid = g64[idx];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float p = dl * (float)((grid >> (8 * j)) & 0xFF);
            w[j] = ((sg >> j) & 1u) ? -p : p;
        }
    } else {
        const uint32_t l = sub, qh = q[64 + ib32];
        const uint32_t nib = ((uint32_t)s[2 + ib32 / 2] >> (4 * (ib32 & 1))) & 15u;
        const float dl = d * (1.0f + 2.0f * (float)nib);
        const uint32_t i1 = (uint32_t)q[8 * ib32 + 2 * l] | (((qh >> (2 * l)) & 1u) << 8);
        const uint32_t i2 = (uint32_t)q[8 * ib32 + 2 * l + 1] | (((qh >> (2 * l + 1)) & 1u) << 8);
        const uint32_t sg = q[72 + 4 * ib32 + l];
        const uint32_t g1 = g32[i1], g2 = g32[i2];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float p = dl * (float)((g1 >> (8 * j)) & 0xFF), p4 = dl * (float)((g2 >> (8 * j)) & 0xFF);
            w[j] = ((sg >> j) & 1u) ? -p : p;
            w[4 + j] = ((sg >> (4 + j)) & 1u) ? -p4 : p4;
        }
    }
}

// x[k0 .. k0+7] of one token as f32; VEC: 16-byte aligned and the eight values inside K.
template <typename XT>
__device__ __forceinline__ void load_x8(const XT* __restrict__ xr, size_t k0, uint32_t K, bool vec, float (&v)[8]) {
    if (vec && k0 + 8 <= K) {
        if constexpr (sizeof(XT) == 4) {
            const float4 a = __ldg(reinterpret_cast<const float4*>(xr + k0));
            const float4 b = __ldg(reinterpret_cast<const float4*>(xr + k0) + 1);
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        } else {
            const uint4 a = __ldg(reinterpret_cast<const uint4*>(xr + k0));
            const uint32_t u[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                XT lo, hi;
                const uint16_t l16 = (uint16_t)(u[j] & 0xFFFFu), h16 = (uint16_t)(u[j] >> 16);
                memcpy(&lo, &l16, 2);
                memcpy(&hi, &h16, 2);
                v[2 * j] = to_f32(lo);
                v[2 * j + 1] = to_f32(hi);
            }
        }
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = k0 + j < K ? to_f32(xr[k0 + j]) : 0.0f;
    }
}

// IQ2_XS / IQ2_S grids hold the IQ2_XXS magnitudes {8, 25, 43}: group `lane` of a block becomes
// eight signed int8 weights with one grid-selector lookup (nibble j: which magnitude byte j
// holds), one sign-selector lookup (nibble j: 4 when weight j is negative) and two `prmt`s of the
// magnitude words; w = dl * int8 is the exact value dl * grid * sign.
template <int V>
__device__ __forceinline__ void decode8_sel(const uint8_t* __restrict__ q, const uint8_t* __restrict__ s,
                                            uint32_t lane, float (&w)[8], const uint32_t* gsel,
                                            const uint32_t* ssel, const uint8_t* ks) {
    const float d = half_bits_to_float((uint32_t)s[0] | ((uint32_t)s[1] << 8));
    const uint32_t ib32 = lane >> 2, sub = lane & 3;
    uint32_t sel;
    float dl;
    if (V == V_XS) {
        const uint32_t word = (uint32_t)q[2 * lane] | ((uint32_t)q[2 * lane + 1] << 8);
        const uint32_t sb = s[2 + ib32];
        dl = d * (0.5f + (float)(sub < 2 ? (sb & 15u) : (sb >> 4))) * 0.25f;
        sel = gsel[word & 0x1FFu] | ssel[ks[(word >> 9) & 0x7Fu]];
    } else {
        const uint32_t il = sub >> 1, h = sub & 1;
        const uint32_t nib = (uint32_t)q[64 + ib32] >> (4 * il);
        const uint32_t idx = (uint32_t)q[lane] | ((nib << (h ? 6 : 8)) & 0x300u);
        dl = d * (0.5f + (float)(((uint32_t)s[2 + ib32] >> (4 * il)) & 15u)) * 0.25f;
        sel = gsel[idx] | ssel[q[32 + lane]];
    }
    const uint32_t lo = prmt(KPOS, KNEG, sel), hi = prmt(KPOS, KNEG, sel >> 16);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        w[j] = dl * (float)(int8_t)(lo >> (8 * j));
        w[4 + j] = dl * (float)(int8_t)(hi >> (8 * j));
    }
}

// MT tokens per warp pass (1 for m = 1, else 8 with the last pass masked).
template <int V, typename XT, int MT>
__global__ void __launch_bounds__(256) variant_matmul_kernel(const XT* __restrict__ x, const uint8_t* __restrict__ qs,
                                                             const uint8_t* __restrict__ sc, float* __restrict__ out,
                                                             uint32_t M, uint32_t N, uint32_t K, uint32_t nb,
                                                             bool xvec) {
    __shared__ uint32_t gsel_s[V == V_S ? 1024 : (V == V_XS ? 512 : 1)];  // grid selectors (IQ2_XS / IQ2_S)
    __shared__ uint32_t ssel_s[V == V_3S ? 1 : 256];                       // sign selectors by sign byte
    __shared__ uint32_t g32_s[V == V_3S ? 512 : 1];
    __shared__ uint8_t ks_s[128];
    if (V != V_3S) {
        const uint32_t entries = V == V_S ? 1024u : 512u;
        for (uint32_t i = threadIdx.x; i < entries; i += blockDim.x) {
            const uint64_t gw = V == V_S ? IQ2S_GRID[i] : IQ2XS_GRID[i];
            uint32_t sel = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const uint32_t b = (uint32_t)(gw >> (8 * j)) & 0xFFu;
                sel |= (b == 8u ? 0u : (b == 25u ? 1u : 2u)) << (4 * j);
            }
            gsel_s[i] = sel;
        }
        for (uint32_t i = threadIdx.x; i < 256; i += blockDim.x) {
            uint32_t sel = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) sel |= ((i >> j) & 1u) << (4 * j + 2);
            ssel_s[i] = sel;
        }
    }
    if (V == V_3S)
        for (int i = threadIdx.x; i < 512; i += blockDim.x) g32_s[i] = IQ3S_GRID[i];
    for (int i = threadIdx.x; i < 128; i += blockDim.x) ks_s[i] = IQ2_KSIGNS[i];
    __syncthreads();
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t mchunks = (M + MT - 1) / MT;
    const size_t total = (size_t)N * mchunks;
    for (size_t wi = (blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5; wi < total;
         wi += (size_t)gridDim.x * blockDim.x / 32) {
        const uint32_t n = (uint32_t)(wi / mchunks), mc = (uint32_t)(wi % mchunks) * MT;
        const uint8_t* qrow = qs + (size_t)n * nb * Geom<V>::BYTES;
        const uint8_t* srow = sc + (size_t)n * nb * Geom<V>::SCALES;
        float acc[MT];
#pragma unroll
        for (int i = 0; i < MT; ++i) acc[i] = 0.0f;
        // lane l takes group l of every block, in block order (the FMA order of each lane's sum)
        for (uint32_t b0 = 0; b0 < nb; b0 += 2) {
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const uint32_t blk = b0 + u;
                if (blk >= nb) break;
                const size_t k0 = (size_t)blk * QK + lane * 8;
                if (k0 >= K) continue;
                float w[8];
                if constexpr (V == V_3S)
                    decode8<V>(qrow + (size_t)blk * Geom<V>::BYTES, srow + (size_t)blk * Geom<V>::SCALES, lane, w,
                               nullptr, g32_s, ks_s);
                else
                    decode8_sel<V>(qrow + (size_t)blk * Geom<V>::BYTES, srow + (size_t)blk * Geom<V>::SCALES, lane, w,
                                   gsel_s, ssel_s, ks_s);
                const bool full = k0 + 8 <= K;  // only the last group of a ragged K is not
#pragma unroll
                for (int mm = 0; mm < MT; ++mm) {
                    if (MT > 1 && mc + mm >= M) break;
                    float xv[8];
                    load_x8<XT>(x + (size_t)(mc + mm) * K, k0, K, xvec, xv);
                    if (full) {
#pragma unroll
                        for (int j = 0; j < 8; ++j) acc[mm] = fmaf(xv[j], w[j], acc[mm]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 8; ++j)
                            if (k0 + j < K) acc[mm] = fmaf(xv[j], w[j], acc[mm]);
                    }
                }
            }
        }
#pragma unroll
        for (int mm = 0; mm < MT; ++mm) {
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
        decode8<V>(qs + bi * Geom<V>::BYTES, sc + bi * Geom<V>::SCALES, (uint32_t)(g & 31), w, V == V_S ? IQ2S_GRID : IQ2XS_GRID,
                   IQ3S_GRID, IQ2_KSIGNS);
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
    const uint32_t mt = m == 1 ? 1u : 8u;
    const unsigned blocks = grid_for((size_t)n * ((m + mt - 1) / mt), 8, num_sms);
    const uintptr_t xa = reinterpret_cast<uintptr_t>(x);
    const bool xvec = x_dtype == 0 ? (xa % 16 == 0 && k % 4 == 0) : (xa % 16 == 0 && k % 8 == 0);
    const uint8_t* q = qs;
    if (mt == 1) {
        switch (x_dtype) {
            case 0: variant_matmul_kernel<V, float, 1><<<blocks, 256, 0, s>>>(static_cast<const float*>(x), q, sc, out, m, n, k, nb, xvec); break;
            case 1: variant_matmul_kernel<V, __half, 1><<<blocks, 256, 0, s>>>(static_cast<const __half*>(x), q, sc, out, m, n, k, nb, xvec); break;
            default: variant_matmul_kernel<V, __nv_bfloat16, 1><<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), q, sc, out, m, n, k, nb, xvec); break;
        }
    } else {
        switch (x_dtype) {
            case 0: variant_matmul_kernel<V, float, 8><<<blocks, 256, 0, s>>>(static_cast<const float*>(x), q, sc, out, m, n, k, nb, xvec); break;
            case 1: variant_matmul_kernel<V, __half, 8><<<blocks, 256, 0, s>>>(static_cast<const __half*>(x), q, sc, out, m, n, k, nb, xvec); break;
            default: variant_matmul_kernel<V, __nv_bfloat16, 8><<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), q, sc, out, m, n, k, nb, xvec); break;
        }
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
