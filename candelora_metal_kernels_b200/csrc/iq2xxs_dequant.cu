// IQ2_XXS dense dequantisation (sm_100a) and the column-gather used after a sharded all-gather.
//
// Dequant follows the reference kernel iq2_xxs_dequantize_f16 (src/metal_src/iq2_matmul.metal:
// 868-887) and its decode_iq2_xxs_value (:701-734): value = d * (0.5 + s) * 0.25 * grid * sign in
// f32, then narrowed. Every factor is exact in f32 (d is an fp16 value with an 11-bit
// significand, 0.5+s has 5 significant bits, grid bytes at most 6), so the f32 value is exact
// whatever the evaluation order, and f16/bf16 outputs are its round-to-nearest-even: the f16
// output is bit-identical to the reference's.
//
// One thread produces one 8-weight group (one 16-byte f16/bf16 store or two f32 stores); the
// kernel is bound by the output write stream (2 bytes per weight vs 0.26 read).
#include "iq2xxs_common.cuh"
#include "iq2xxs_codebook.h"
#include "iq2xxs_internal.h"

namespace iq2 {

namespace {

template <int OUT_DTYPE>  // 0 f32, 1 f16, 2 bf16
__global__ void __launch_bounds__(256) dequant_kernel(const uint8_t* __restrict__ qs,
                                                      const uint8_t* __restrict__ sc,
                                                      void* __restrict__ out, uint32_t N,
                                                      uint32_t K, uint32_t nb, bool aligned) {
    __shared__ uint64_t grid_s[256];
    __shared__ uint8_t ksigns_s[128];
    for (int i = threadIdx.x; i < 256; i += blockDim.x) grid_s[i] = IQ2XXS_GRID[i];
    for (int i = threadIdx.x; i < 128; i += blockDim.x) ksigns_s[i] = IQ2_KSIGNS[i];
    __syncthreads();
    const size_t groups_per_row = (size_t)nb * 32;
    const size_t total = (size_t)N * groups_per_row;
    for (size_t gid = (size_t)blockIdx.x * blockDim.x + threadIdx.x; gid < total;
         gid += (size_t)gridDim.x * blockDim.x) {
        const uint32_t n = (uint32_t)(gid / groups_per_row);
        const uint32_t q = (uint32_t)(gid % groups_per_row);
        const uint32_t sbk = q >> 2, gi = q & 3, blk = sbk >> 3;
        const size_t k0 = (size_t)sbk * 32 + gi * 8;
        if (k0 >= K) continue;
        const uint8_t* pq = qs + (size_t)n * nb * QS_BYTES + (size_t)sbk * 8;
        uint32_t aux_g, aux_s, dbits;
        if (aligned) {
            const uint2 w = *reinterpret_cast<const uint2*>(pq);
            aux_g = w.x;
            aux_s = w.y;
            dbits = *reinterpret_cast<const uint16_t*>(sc + ((size_t)n * nb + blk) * SC_BYTES);
        } else {
            aux_g = ld_u32_le_unaligned(pq);
            aux_s = ld_u32_le_unaligned(pq + 4);
            dbits = ld_u16_le_unaligned(sc + ((size_t)n * nb + blk) * SC_BYTES);
        }
        const float d = half_bits_to_float(dbits);
        const float dl = d * (0.5f + (float)(aux_s >> 28)) * 0.25f;
        const uint64_t gw = grid_s[(aux_g >> (8 * gi)) & 0xFF];
        const uint32_t signs = ksigns_s[(aux_s >> (7 * gi)) & 0x7F];
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            v[j] = dl * (float)((gw >> (8 * j)) & 0xFF) * (((signs >> j) & 1u) ? -1.0f : 1.0f);
        }
        const size_t base = (size_t)n * K + k0;
        const bool full = k0 + 8 <= K;
        if (OUT_DTYPE == 0) {
            float* o = static_cast<float*>(out) + base;
            if (full && aligned && (base % 4) == 0) {
                reinterpret_cast<float4*>(o)[0] = make_float4(v[0], v[1], v[2], v[3]);
                reinterpret_cast<float4*>(o)[1] = make_float4(v[4], v[5], v[6], v[7]);
            } else {
                for (int j = 0; j < 8 && k0 + j < K; ++j) o[j] = v[j];
            }
        } else {
            uint16_t h[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                h[j] = OUT_DTYPE == 1 ? __half_as_ushort(__float2half_rn(v[j]))
                                      : __bfloat16_as_ushort(__float2bfloat16_rn(v[j]));
            }
            uint16_t* o = static_cast<uint16_t*>(out) + base;
            if (full && aligned && (base % 8) == 0) {
                uint4 pk;
                pk.x = (uint32_t)h[0] | ((uint32_t)h[1] << 16);
                pk.y = (uint32_t)h[2] | ((uint32_t)h[3] << 16);
                pk.z = (uint32_t)h[4] | ((uint32_t)h[5] << 16);
                pk.w = (uint32_t)h[6] | ((uint32_t)h[7] << 16);
                *reinterpret_cast<uint4*>(o) = pk;
            } else {
                for (int j = 0; j < 8 && k0 + j < K; ++j) o[j] = h[j];
            }
        }
    }
}

__global__ void gather_columns_kernel(const float* __restrict__ gathered, uint32_t shards,
                                      uint32_t m, uint32_t shard_cols, float* __restrict__ out) {
    const size_t total = (size_t)shards * m * shard_cols;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (size_t)gridDim.x * blockDim.x) {
        const size_t c = i % shard_cols;
        const size_t r = (i / shard_cols) % m;
        const size_t s = i / ((size_t)shard_cols * m);
        out[r * ((size_t)shards * shard_cols) + s * shard_cols + c] = gathered[i];
    }
}

// W8A8 activation quant-dequant of one token (row) per CTA, as the reference's W8A8 kernels do it
// (row_inv_scale_w8a8 / qdq_w8a8, src/metal_src/iq2_matmul.metal:85-102): inv = 127 / max|x| over
// the row (1 when max|x| < 1e-8), xq = clamp(round(x * inv), -127, 127) / inv, round half away
// from zero, f32 multiply and IEEE division.
template <typename XT>
__global__ void __launch_bounds__(256) qdq_w8a8_kernel(const XT* __restrict__ x, uint32_t K, float* __restrict__ xq) {
    __shared__ float red[8];
    const XT* xr = x + (size_t)blockIdx.x * K;
    float* qr = xq + (size_t)blockIdx.x * K;
    float mx = 0.0f;
    for (uint32_t k = threadIdx.x; k < K; k += blockDim.x) mx = fmaxf(mx, fabsf(to_f32(xr[k])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = red[0];
#pragma unroll
    for (int w = 1; w < 8; ++w) mx = fmaxf(mx, red[w]);
    const float inv = mx < 1e-8f ? 1.0f : 127.0f / mx;
    for (uint32_t k = threadIdx.x; k < K; k += blockDim.x) {
        const float q = fminf(fmaxf(roundf(__fmul_rn(to_f32(xr[k]), inv)), -127.0f), 127.0f);
        qr[k] = __fdiv_rn(q, inv);
    }
}

// ggml's interleaved blocks (d, then the packed weights, then the format's extra scale bytes) ->
// the reference's split tensors (weight_bytes: the packed weights; weight_scales: d, then the
// extra scale bytes). One thread per interleaved byte: coalesced reads, near-coalesced writes.
__global__ void __launch_bounds__(256) split_interleaved_kernel(const uint8_t* __restrict__ blocks, uint64_t total,
                                                                uint32_t ib, uint32_t bpb, uint32_t spb,
                                                                uint8_t* __restrict__ wb, uint8_t* __restrict__ ws) {
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t blk = i / ib;
        const uint32_t off = (uint32_t)(i % ib);
        const uint8_t v = blocks[i];
        if (off < 2) ws[blk * spb + off] = v;
        else if (off < 2 + bpb) wb[blk * bpb + off - 2] = v;
        else ws[blk * spb + 2 + (off - 2 - bpb)] = v;
    }
}

}  // namespace

cudaError_t launch_split_interleaved(const uint8_t* blocks, uint64_t nblocks, uint32_t bytes_per_block,
                                     uint32_t scales_per_block, uint8_t* wb, uint8_t* ws, int num_sms,
                                     cudaStream_t stream) {
    const uint32_t ib = bytes_per_block + scales_per_block;
    const uint64_t total = nblocks * ib;
    if (total == 0) return cudaSuccess;
    uint64_t grid = (total + 255) / 256;
    const uint64_t cap = (uint64_t)(num_sms > 0 ? num_sms : 148) * 16;
    if (grid > cap) grid = cap;
    split_interleaved_kernel<<<(unsigned)grid, 256, 0, stream>>>(blocks, total, ib, bytes_per_block, scales_per_block,
                                                                 wb, ws);
    return cudaGetLastError();
}

cudaError_t launch_qdq_w8a8(const void* x, int x_dtype, uint32_t m, uint32_t k, float* xq, cudaStream_t stream) {
    if (m == 0 || k == 0) return cudaSuccess;
    switch (x_dtype) {
        case 0: qdq_w8a8_kernel<float><<<m, 256, 0, stream>>>(static_cast<const float*>(x), k, xq); break;
        case 1: qdq_w8a8_kernel<__half><<<m, 256, 0, stream>>>(static_cast<const __half*>(x), k, xq); break;
        default:
            qdq_w8a8_kernel<__nv_bfloat16><<<m, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(x), k, xq);
            break;
    }
    return cudaGetLastError();
}

cudaError_t launch_dequant(const uint8_t* qs, const uint8_t* sc, uint32_t n, uint32_t k, void* out,
                           int out_dtype, int num_sms, cudaStream_t stream) {
    const uint32_t nb = (k + QK - 1) / QK;
    const bool aligned = (reinterpret_cast<uintptr_t>(qs) % 8) == 0 &&
                         (reinterpret_cast<uintptr_t>(sc) % 2) == 0 &&
                         (reinterpret_cast<uintptr_t>(out) % 16) == 0;
    const size_t total = (size_t)n * nb * 32;
    size_t blocks = (total + 255) / 256;
    const size_t cap = (size_t)num_sms * 16;
    if (blocks > cap) blocks = cap;
    switch (out_dtype) {
        case 0: dequant_kernel<0><<<(unsigned)blocks, 256, 0, stream>>>(qs, sc, out, n, k, nb, aligned); break;
        case 1: dequant_kernel<1><<<(unsigned)blocks, 256, 0, stream>>>(qs, sc, out, n, k, nb, aligned); break;
        default: dequant_kernel<2><<<(unsigned)blocks, 256, 0, stream>>>(qs, sc, out, n, k, nb, aligned); break;
    }
    return cudaGetLastError();
}

cudaError_t launch_gather_columns(const float* gathered, uint32_t shards, uint32_t m,
                                  uint32_t shard_cols, float* out, int num_sms, cudaStream_t stream) {
    const size_t total = (size_t)shards * m * shard_cols;
    size_t blocks = (total + 255) / 256;
    const size_t cap = (size_t)num_sms * 8;
    if (blocks > cap) blocks = cap;
    if (blocks == 0) return cudaSuccess;
    gather_columns_kernel<<<(unsigned)blocks, 256, 0, stream>>>(gathered, shards, m, shard_cols, out);
    return cudaGetLastError();
}

}  // namespace iq2
