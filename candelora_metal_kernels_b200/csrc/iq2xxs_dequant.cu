// IQ2_XXS dense dequantisation (sm_100a) and the column-gather used after a sharded all-gather.
//
// Dequant follows the reference kernel iq2_xxs_dequantize_f16 (src/metal_src/iq2_matmul.metal:
// 868-887) and its decode_iq2_xxs_value (:701-734): value = d * (0.5 + s) * 0.25 * grid * sign in
// f32, then narrowed. Every factor is exact in f32 (d is an fp16 value with an 11-bit
// significand, 0.5+s has 5 significant bits, grid bytes at most 6), so the f32 value is exact
// whatever the evaluation order, and f16/bf16 outputs are its round-to-nearest-even: the f16
// output is bit-identical to the reference's.
//
// One warp per weight row: lane (sub-block sb, group gi) of each 256-weight block turns its 8-byte
// sub-block word into the group's eight signed int8 grid values with one selector lookup and two
// `prmt`s (the decode of the GEMV), scales them by the exact block factor in f32 and writes one
// 16-byte f16/bf16 store (or two f32 stores): a warp writes 512 contiguous bytes per block and
// four blocks' words are loaded before any is decoded. No index division: the kernel is meant to
// run at the output write stream's speed (2 bytes per weight written vs 0.26 read).
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
    constexpr int U = 4;  // blocks whose words are in flight together
    __shared__ uint32_t sel_s[384];  // grid selectors (256), then sign selectors (128)
    for (int i = threadIdx.x; i < 384; i += blockDim.x) sel_s[i] = IQ2XXS_SEL_COMPACT[i];
    __syncthreads();
    const uint32_t lane = threadIdx.x & 31, gi = lane & 3, sb = lane >> 2;
    const uint32_t wpb = blockDim.x >> 5;
    const uint32_t warps = gridDim.x * wpb;
    for (uint32_t n = blockIdx.x * wpb + (threadIdx.x >> 5); n < N; n += warps) {
        const uint8_t* qrow = qs + (size_t)n * nb * QS_BYTES + sb * 8;
        const uint8_t* srow = sc + (size_t)n * nb * SC_BYTES;
        for (uint32_t b0 = 0; b0 < nb; b0 += U) {
            uint32_t ag[U], as[U], db[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const uint32_t blk = b0 + u;
                ag[u] = as[u] = db[u] = 0u;
                if (blk < nb) {
                    const uint8_t* pq = qrow + (size_t)blk * QS_BYTES;
                    if (aligned) {
                        const uint2 w = *reinterpret_cast<const uint2*>(pq);
                        ag[u] = w.x;
                        as[u] = w.y;
                        db[u] = *reinterpret_cast<const uint16_t*>(srow + (size_t)blk * SC_BYTES);
                    } else {
                        ag[u] = ld_u32_le_unaligned(pq);
                        as[u] = ld_u32_le_unaligned(pq + 4);
                        db[u] = ld_u16_le_unaligned(srow + (size_t)blk * SC_BYTES);
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const uint32_t blk = b0 + u;
                const uint32_t k0 = blk * QK + sb * 32 + gi * 8;
                if (blk >= nb || k0 >= K) continue;
                // every factor is exact in f32, so dl * (signed grid byte) is the exact value
                const float dl = half_bits_to_float(db[u]) * (0.5f + (float)(as[u] >> 28)) * 0.25f;
                const uint32_t sel = sel_s[(ag[u] >> (8 * gi)) & 0xFFu] | sel_s[256 + ((as[u] >> (7 * gi)) & 0x7Fu)];
                const uint32_t lo = prmt(KPOS, KNEG, sel), hi = prmt(KPOS, KNEG, sel >> 16);
                float v[8];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    v[j] = dl * (float)(int8_t)(lo >> (8 * j));
                    v[4 + j] = dl * (float)(int8_t)(hi >> (8 * j));
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
                    uint32_t h2[4];  // round to nearest even, two values per conversion
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        if (OUT_DTYPE == 1) {
                            const __half2 t = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
                            h2[j] = *reinterpret_cast<const uint32_t*>(&t);
                        } else {
                            const __nv_bfloat162 t = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
                            h2[j] = *reinterpret_cast<const uint32_t*>(&t);
                        }
                    }
                    uint16_t* o = static_cast<uint16_t*>(out) + base;
                    if (full && aligned && (base % 8) == 0) {
                        *reinterpret_cast<uint4*>(o) = make_uint4(h2[0], h2[1], h2[2], h2[3]);
                    } else {
                        for (int j = 0; j < 8 && k0 + j < K; ++j) o[j] = (uint16_t)(h2[j >> 1] >> (16 * (j & 1)));
                    }
                }
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

// The same repack for whole chunks of SPLIT_CHUNK blocks, one chunk per CTA pass: the chunk's
// interleaved bytes (a multiple of 16: every format's block size is even) come in as 16-byte loads
// to shared memory, the packed weights leave as 8-byte stores (every format's weight bytes per
// block are a multiple of 8, so no store straddles two blocks) and the scale bytes as 2-byte
// stores (every field is 2-byte aligned). Needs 16-byte aligned blocks and 8-byte aligned wb.
constexpr uint32_t SPLIT_CHUNK = 64;
constexpr uint32_t SPLIT_MAX_BLOCK = 112;  // >= the largest block (IQ3_S: 110 bytes)

__global__ void __launch_bounds__(256) split_chunks_kernel(const uint8_t* __restrict__ blocks, uint64_t nchunks,
                                                           uint32_t ib, uint32_t bpb, uint32_t spb,
                                                           uint8_t* __restrict__ wb, uint8_t* __restrict__ ws) {
    __shared__ __align__(16) uint8_t buf[SPLIT_CHUNK * SPLIT_MAX_BLOCK];
    const uint32_t in16 = SPLIT_CHUNK * ib / 16, out8 = SPLIT_CHUNK * bpb / 8, out2 = SPLIT_CHUNK * spb / 2;
    for (uint64_t ch = blockIdx.x; ch < nchunks; ch += gridDim.x) {
        const uint4* src = reinterpret_cast<const uint4*>(blocks + ch * SPLIT_CHUNK * ib);
        for (uint32_t i = threadIdx.x; i < in16; i += blockDim.x) reinterpret_cast<uint4*>(buf)[i] = src[i];
        __syncthreads();
        uint2* dw = reinterpret_cast<uint2*>(wb + ch * SPLIT_CHUNK * bpb);
        for (uint32_t c = threadIdx.x; c < out8; c += blockDim.x) {
            const uint32_t o = c * 8, blk = o / bpb;
            const uint16_t* p = reinterpret_cast<const uint16_t*>(buf + blk * ib + 2 + (o - blk * bpb));
            dw[c] = make_uint2((uint32_t)p[0] | ((uint32_t)p[1] << 16), (uint32_t)p[2] | ((uint32_t)p[3] << 16));
        }
        uint16_t* dsc = reinterpret_cast<uint16_t*>(ws + ch * SPLIT_CHUNK * spb);
        for (uint32_t j = threadIdx.x; j < out2; j += blockDim.x) {
            const uint32_t o = j * 2, blk = o / spb, off = o - blk * spb;  // d at 0..1, the rest after the weights
            dsc[j] = *reinterpret_cast<const uint16_t*>(buf + blk * ib + (off < 2 ? off : bpb + off));
        }
        __syncthreads();
    }
}

}  // namespace

cudaError_t launch_split_interleaved(const uint8_t* blocks, uint64_t nblocks, uint32_t bytes_per_block,
                                     uint32_t scales_per_block, uint8_t* wb, uint8_t* ws, int num_sms,
                                     cudaStream_t stream) {
    const uint32_t ib = bytes_per_block + scales_per_block;
    if (nblocks == 0 || ib == 0) return cudaSuccess;
    const uint64_t nchunks = nblocks / SPLIT_CHUNK;
    if (nchunks > 0 && ib % 2 == 0 && ib <= SPLIT_MAX_BLOCK && bytes_per_block % 8 == 0 &&
        scales_per_block % 2 == 0 && (reinterpret_cast<uintptr_t>(blocks) % 16) == 0 &&
        (reinterpret_cast<uintptr_t>(wb) % 8) == 0 && (reinterpret_cast<uintptr_t>(ws) % 2) == 0) {
        uint64_t g = nchunks;
        const uint64_t gcap = (uint64_t)(num_sms > 0 ? num_sms : 148) * 8;
        if (g > gcap) g = gcap;
        split_chunks_kernel<<<(unsigned)g, 256, 0, stream>>>(blocks, nchunks, ib, bytes_per_block, scales_per_block,
                                                             wb, ws);
        const uint64_t done = nchunks * SPLIT_CHUNK;
        blocks += done * ib;
        wb += done * bytes_per_block;
        ws += done * scales_per_block;
        nblocks -= done;
        if (nblocks == 0) return cudaGetLastError();
    }
    const uint64_t total = nblocks * ib;
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
    // one warp per row, eight per CTA; at most 16 CTAs per SM, the rows dealt round-robin
    size_t blocks = ((size_t)n + 7) / 8;
    const size_t cap = (size_t)(num_sms > 0 ? num_sms : 148) * 16;
    if (blocks > cap) blocks = cap;
    if (blocks == 0) return cudaSuccess;
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
