/*
 * TEST INFRASTRUCTURE ONLY -- the CPU oracle for the IQ2_XXS matmul path. Only the tests,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg load this; the shipped library
 * never links or calls it.
 *
 * A plain-C restatement of the reference's scalar CPU implementation of the path:
 *   iq2_matmul_reference, IQ2_XXS arm ........ src/iq2_matmul.rs:833-883
 *   accum_word_grid ........................... src/iq2_matmul.rs:789-809
 *   read_u16_le ............................... src/iq2_matmul.rs:761-763
 *   f16 -> f32 of the block scale `d` ......... half::f16::to_f32 (exact IEEE widening)
 * and of the reference's dequantisation:
 *   decode_iq2_xxs_value ...................... src/metal_src/iq2_matmul.metal:701-734
 *   iq2_xxs_dequantize_f16_kernel ............. src/metal_src/iq2_matmul.metal:868-887
 *     (f32 value, then narrowed to f16 with round-to-nearest-even)
 *   rowwise_quant_dequant_w8a8 ................ src/iq2_matmul.rs:1025-1044
 * and of the reference's test fixtures:
 *   lcg_fill / deterministic_x / force_f16_one_per_block  src/iq2_matmul.rs:765-787
 *
 * Parity pinning: every function here is checked against the reference's own Metal
 * kernels compiled from their source as C++ (oracle/_ref, see oracle/ref_harness.cpp) and
 * against the golden vectors in tests/golden/ that those kernels produced.
 *
 * Build with -ffp-contract=off (oracle/Makefile): the Rust reference never fuses a*b+c, so
 * neither may this file; the summation order below is the reference's (blk -> ib32 -> g -> j).
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

#include "iq2_tables_ref.h"

#define QK 256
#define XXS_BYTES_PER_BLOCK 64
#define XXS_SCALES_PER_BLOCK 2

static float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* IEEE binary16 -> binary32, exact (half::f16::to_f32). */
float oracle_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu;
    if (exp == 0x1Fu) return bits_f32(sign | 0x7F800000u | (man << 13));
    if (exp == 0) {
        float v = (float)man * 5.9604644775390625e-08f; /* man * 2^-24, exact */
        return sign ? -v : v;
    }
    return bits_f32(sign | ((exp + 112u) << 23) | (man << 13));
}

/* binary32 -> binary16, round to nearest, ties to even; overflow -> inf. */
uint16_t oracle_f32_to_f16(float f) {
    uint32_t u = f32_bits(f);
    uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
    uint32_t a = u & 0x7FFFFFFFu;
    if (a >= 0x7F800000u) return (uint16_t)(sign | (a > 0x7F800000u ? 0x7E00u : 0x7C00u));
    if (a >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);
    if (a < 0x38800000u) { /* subnormal result: round(value * 2^24) to even */
        float v = bits_f32(a) * 16777216.0f;
        return (uint16_t)(sign | (uint16_t)nearbyintf(v));
    }
    uint32_t h = (((a >> 23) - 112u) << 10) | ((a & 0x7FFFFFu) >> 13);
    uint32_t rem = a & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1u;
    return (uint16_t)(sign | h);
}

float oracle_bf16_to_f32(uint16_t b) { return bits_f32((uint32_t)b << 16); }

uint16_t oracle_f32_to_bf16(float f) {
    uint32_t u = f32_bits(f);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x40u);
    return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

static uint16_t read_u16_le(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* accum_word_grid (src/iq2_matmul.rs:789-809): 8 weights of one grid word, f32 accumulate,
 * stopping at the first column >= in_dim. */
static void accum_word_grid(uint64_t grid_pack, uint8_t signs, float dl, size_t base_col,
                            size_t in_dim, const float* x_row, float* acc) {
    for (int j = 0; j < 8; ++j) {
        size_t col = base_col + (size_t)j;
        if (col >= in_dim) break;
        float gv = (float)(uint8_t)((grid_pack >> (8 * j)) & 0xFF);
        float sign = (signs & ref_kmask_iq2xs[j]) ? -1.0f : 1.0f;
        *acc += x_row[col] * (dl * gv * sign);
    }
}

/* One output element of iq2_matmul_reference, IQ2_XXS arm (src/iq2_matmul.rs:853-883). */
static float xxs_dot(const float* x_row, size_t in_dim, size_t out_idx, size_t blocks_per_row,
                     const uint8_t* w_bytes, const uint8_t* w_scales) {
    float acc = 0.0f;
    for (size_t blk = 0; blk < blocks_per_row; ++blk) {
        size_t block_idx = out_idx * blocks_per_row + blk;
        size_t byte_base = block_idx * XXS_BYTES_PER_BLOCK;
        size_t scale_base = block_idx * XXS_SCALES_PER_BLOCK;
        float d = oracle_f16_to_f32(read_u16_le(w_scales + scale_base));
        for (size_t ib32 = 0; ib32 < 8; ++ib32) {
            const uint8_t* q2 = w_bytes + byte_base + ib32 * 8;
            uint32_t aux_g = (uint32_t)read_u16_le(q2) | ((uint32_t)read_u16_le(q2 + 2) << 16);
            uint32_t aux_s = (uint32_t)read_u16_le(q2 + 4) | ((uint32_t)read_u16_le(q2 + 6) << 16);
            float dl = d * (0.5f + (float)((aux_s >> 28) & 0xF)) * 0.25f;
            for (size_t g = 0; g < 4; ++g) {
                size_t grid_idx = (aux_g >> (8 * g)) & 0xFF;
                size_t signs_idx = (aux_s >> (7 * g)) & 0x7F;
                size_t base_col = blk * QK + ib32 * 32 + g * 8;
                accum_word_grid(ref_iq2xxs_grid[grid_idx], ref_ksigns_iq2xs[signs_idx], dl,
                                base_col, in_dim, x_row, &acc);
            }
        }
    }
    return acc;
}

/*
 * out[row * out_dim + n] = reference matmul, for rows [0, m) and output columns n in
 * `cols` (all columns when cols == NULL, ncols ignored). x is f32 [m, in_dim] row-major.
 * With cols given, out is [m, ncols]: the oracle can check sampled columns of a large matrix.
 */
void oracle_iq2xxs_matmul_f32(const float* x, size_t m, size_t out_dim, size_t in_dim,
                              const uint8_t* w_bytes, const uint8_t* w_scales,
                              const int64_t* cols, size_t ncols, float* out, int threads) {
    size_t blocks_per_row = (in_dim + QK - 1) / QK;
    size_t nc = cols ? ncols : out_dim;
    long long total = (long long)(m * nc);
    if (threads <= 0) threads = 1;
#pragma omp parallel for schedule(dynamic, 8) num_threads(threads)
    for (long long i = 0; i < total; ++i) {
        size_t row = (size_t)i / nc, c = (size_t)i % nc;
        size_t n = cols ? (size_t)cols[c] : c;
        out[row * nc + c] = xxs_dot(x + row * in_dim, in_dim, n, blocks_per_row, w_bytes, w_scales);
    }
}

/* The Metal kernels read x as f16/bf16 and widen each element with float(x): exact, so the
 * matmul of a 16-bit x is the f32 matmul of its widened copy. dtype: 1 = f16, 2 = bf16. */
void oracle_widen_x(const uint16_t* x16, int dtype, size_t count, float* out) {
    for (size_t i = 0; i < count; ++i)
        out[i] = dtype == 1 ? oracle_f16_to_f32(x16[i]) : oracle_bf16_to_f32(x16[i]);
}

/* decode_iq2_xxs_value (src/metal_src/iq2_matmul.metal:701-734): the f32 weight. */
static float xxs_value(const uint8_t* w_bytes, const uint8_t* w_scales, size_t block_idx,
                       size_t local_col) {
    float d = oracle_f16_to_f32(read_u16_le(w_scales + block_idx * 2));
    size_t ib32 = local_col / 32, within = local_col % 32, g = within / 8, j = within % 8;
    const uint8_t* q2 = w_bytes + block_idx * 64 + ib32 * 8;
    uint32_t aux_g = (uint32_t)read_u16_le(q2) | ((uint32_t)read_u16_le(q2 + 2) << 16);
    uint32_t aux_s = (uint32_t)read_u16_le(q2 + 4) | ((uint32_t)read_u16_le(q2 + 6) << 16);
    float dl = d * (0.5f + (float)((aux_s >> 28) & 0xF)) * 0.25f;
    uint64_t grid = ref_iq2xxs_grid[(aux_g >> (8 * g)) & 0xFF];
    uint8_t gv = (uint8_t)((grid >> (8 * j)) & 0xFF);
    uint8_t signs = ref_ksigns_iq2xs[(aux_s >> (7 * g)) & 0x7F];
    float sgn = (signs & ref_kmask_iq2xs[j]) ? -1.0f : 1.0f;
    return dl * (float)gv * sgn;
}

/* Dense [out_dim, in_dim] dequantisation. out_dtype: 0 = f32 (the exact value), 1 = f16 RNE
 * (iq2_xxs_dequantize_f16_kernel), 2 = bf16 RNE. `out` holds float or raw 16-bit patterns. */
void oracle_iq2xxs_dequantize(const uint8_t* w_bytes, const uint8_t* w_scales, size_t out_dim,
                              size_t in_dim, int out_dtype, void* out, int threads) {
    size_t blocks_per_row = (in_dim + QK - 1) / QK;
    long long total = (long long)(out_dim * in_dim);
    if (threads <= 0) threads = 1;
#pragma omp parallel for schedule(static) num_threads(threads)
    for (long long gid = 0; gid < total; ++gid) {
        size_t n = (size_t)gid / in_dim, col = (size_t)gid % in_dim;
        float v = xxs_value(w_bytes, w_scales, n * blocks_per_row + col / QK, col % QK);
        if (out_dtype == 0) ((float*)out)[gid] = v;
        else if (out_dtype == 1) ((uint16_t*)out)[gid] = oracle_f32_to_f16(v);
        else ((uint16_t*)out)[gid] = oracle_f32_to_bf16(v);
    }
}

/* rowwise_quant_dequant_w8a8 (src/iq2_matmul.rs:1025-1044), in place into `out`. */
void oracle_rowwise_qdq_w8a8(const float* x, size_t m, size_t in_dim, float* out) {
    for (size_t row = 0; row < m; ++row) {
        const float* xr = x + row * in_dim;
        float max_abs = 0.0f;
        for (size_t c = 0; c < in_dim; ++c) max_abs = fmaxf(max_abs, fabsf(xr[c]));
        float inv_scale = max_abs < 1e-8f ? 1.0f : 127.0f / max_abs;
        for (size_t c = 0; c < in_dim; ++c) {
            float q = roundf(xr[c] * inv_scale);
            q = fminf(fmaxf(q, -127.0f), 127.0f);
            out[row * in_dim + c] = q / inv_scale;
        }
    }
}

/* Reference test fixtures (src/iq2_matmul.rs:765-787). */
void oracle_lcg_fill(uint8_t* out, size_t len, uint32_t seed) {
    uint32_t state = seed;
    for (size_t i = 0; i < len; ++i) {
        state = state * 1664525u + 1013904223u;
        out[i] = (uint8_t)(state >> 24);
    }
}

void oracle_deterministic_x(float* out, size_t len) {
    for (size_t i = 0; i < len; ++i) out[i] = ((float)((i * 17) % 41) - 20.0f) / 13.0f;
}

void oracle_force_f16_one_per_block(uint8_t* scales, size_t len, size_t scales_per_block) {
    for (size_t b = 0; b + scales_per_block <= len; b += scales_per_block) {
        scales[b] = 0x00;
        scales[b + 1] = 0x3c;
    }
}
