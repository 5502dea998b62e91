/*
 * TEST INFRASTRUCTURE ONLY -- the CPU oracle for the other IQ variants of the matmul (IQ2_XS,
 * IQ2_S, IQ3_S). Only the tests load this; the shipped library never links or calls it.
 *
 * A plain-C restatement of the reference's scalar CPU implementation:
 *   iq2_matmul_reference, Iq2Xs / Iq2S / Iq3S arms ..... src/iq2_matmul.rs:884-1016
 *   accum_word_grid / accum_word_grid_u32 ............. src/iq2_matmul.rs:789-831
 * and of the reference's dequantisation:
 *   decode_iq2_xs_value / decode_iq2_s_value / decode_iq3_s_value
 *                                                   ... src/metal_src/iq2_matmul.metal:736-866
 *   iq2_{xs,s}/iq3_s_dequantize_f16_kernel ........... src/metal_src/iq2_matmul.metal:889-950
 * Block geometry (src/iq2_matmul.rs:15-29): bytes / scale bytes per 256-weight block are
 * 64 / 10 (IQ2_XS), 72 / 10 (IQ2_S), 104 / 6 (IQ3_S); scales start with the fp16 d.
 *
 * Pinned like the IQ2_XXS oracle: checked against the reference's own Metal kernels compiled as
 * C++ (oracle/_ref). Build with -ffp-contract=off; the summation order is the reference's.
 */
#include <stddef.h>
#include <stdint.h>
#include <string.h>

#include "iq2_tables_ref.h"

#define QK 256

float oracle_f16_to_f32(uint16_t h);
uint16_t oracle_f32_to_f16(float f);
uint16_t oracle_f32_to_bf16(float f);
void oracle_iq2xxs_matmul_f32(const float* x, size_t m, size_t out_dim, size_t in_dim, const uint8_t* w_bytes,
                              const uint8_t* w_scales, const int64_t* cols, size_t ncols, float* out, int threads);
void oracle_iq2xxs_dequantize(const uint8_t* w_bytes, const uint8_t* w_scales, size_t out_dim, size_t in_dim,
                              int out_dtype, void* out, int threads);

enum { V_XXS = 0, V_XS = 1, V_S = 2, V_3S = 3 };
static const size_t BYTES[4] = {64, 64, 72, 104};
static const size_t SCALES[4] = {2, 10, 10, 6};

static uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* accum_word_grid (src/iq2_matmul.rs:789-809) */
static void acc8(uint64_t grid, uint8_t signs, float dl, size_t base_col, size_t in_dim, const float* x,
                 float* acc) {
    for (int j = 0; j < 8; ++j) {
        size_t col = base_col + (size_t)j;
        if (col >= in_dim) break;
        float gv = (float)(uint8_t)((grid >> (8 * j)) & 0xFF);
        float sign = (signs & ref_kmask_iq2xs[j]) ? -1.0f : 1.0f;
        *acc += x[col] * (dl * gv * sign);
    }
}

/* accum_word_grid_u32 (src/iq2_matmul.rs:811-831): 4 weights, masks from `kmask`. */
static void acc4(uint32_t grid, uint8_t signs, float dl, size_t base_col, size_t in_dim, const float* x,
                 const uint8_t* kmask, float* acc) {
    for (int j = 0; j < 4; ++j) {
        size_t col = base_col + (size_t)j;
        if (col >= in_dim) break;
        float gv = (float)(uint8_t)((grid >> (8 * j)) & 0xFF);
        float sign = (signs & kmask[j]) ? -1.0f : 1.0f;
        *acc += x[col] * (dl * gv * sign);
    }
}

/* One output element of iq2_matmul_reference for the IQ2_XS / IQ2_S / IQ3_S arms. */
static float dot(int v, const float* x, size_t in_dim, size_t out_idx, size_t nb, const uint8_t* wb,
                 const uint8_t* ws) {
    float acc = 0.0f;
    for (size_t blk = 0; blk < nb; ++blk) {
        size_t bi = out_idx * nb + blk;
        const uint8_t* q = wb + bi * BYTES[v];
        const uint8_t* s = ws + bi * SCALES[v];
        float d = oracle_f16_to_f32(rd16(s));
        for (size_t ib32 = 0; ib32 < 8; ++ib32) {
            size_t base = blk * QK + ib32 * 32;
            if (v == V_XS) {
                uint8_t sb = s[2 + ib32];
                float dl0 = d * (0.5f + (float)(sb & 0x0F)) * 0.25f;
                float dl1 = d * (0.5f + (float)((sb >> 4) & 0x0F)) * 0.25f;
                for (int w = 0; w < 4; ++w) {
                    uint16_t word = rd16(q + ib32 * 8 + 2 * w);
                    acc8(ref_iq2xs_grid[word & 0x1FF], ref_ksigns_iq2xs[(word >> 9) & 0x7F], w < 2 ? dl0 : dl1,
                         base + 8 * (size_t)w, in_dim, x, &acc);
                }
            } else if (v == V_S) {
                const uint8_t* qs = q;
                const uint8_t* qh = q + 64;
                uint8_t sb = s[2 + ib32];
                for (size_t il = 0; il < 2; ++il) {
                    size_t off = 4 * ib32 + 2 * il;
                    uint8_t nib = (uint8_t)(qh[ib32] >> (4 * il));
                    float dl = d * (0.5f + (float)((sb >> (4 * il)) & 0x0F)) * 0.25f;
                    size_t g0 = (size_t)qs[off] | (((size_t)nib << 8) & 0x300);
                    size_t g1 = (size_t)qs[off + 1] | (((size_t)nib << 6) & 0x300);
                    acc8(ref_iq2s_grid[g0], qs[32 + off], dl, base + il * 16, in_dim, x, &acc);
                    acc8(ref_iq2s_grid[g1], qs[32 + off + 1], dl, base + il * 16 + 8, in_dim, x, &acc);
                }
            } else { /* IQ3_S */
                const uint8_t* qs = q;
                const uint8_t* qh = q + 64;
                const uint8_t* sg = q + 72;
                uint8_t nib = (uint8_t)((s[2 + ib32 / 2] >> (4 * (ib32 % 2))) & 0x0F);
                float dl = d * (1.0f + 2.0f * (float)nib);
                for (size_t l = 0; l < 4; ++l) {
                    size_t i1 = (size_t)qs[8 * ib32 + 2 * l] | ((qh[ib32] & ref_kmask_iq2xs[2 * l]) ? 256u : 0u);
                    size_t i2 = (size_t)qs[8 * ib32 + 2 * l + 1] | ((qh[ib32] & ref_kmask_iq2xs[2 * l + 1]) ? 256u : 0u);
                    uint8_t sb = sg[4 * ib32 + l];
                    acc4(ref_iq3s_grid[i1], sb, dl, base + l * 8, in_dim, x, ref_kmask_iq2xs, &acc);
                    acc4(ref_iq3s_grid[i2], sb, dl, base + l * 8 + 4, in_dim, x, ref_kmask_iq2xs + 4, &acc);
                }
            }
        }
    }
    return acc;
}

/* As oracle_iq2xxs_matmul_f32, for variant 0..3 (0 = IQ2_XXS). */
void oracle_iq2_matmul_f32(int v, const float* x, size_t m, size_t out_dim, size_t in_dim, const uint8_t* wb,
                           const uint8_t* ws, const int64_t* cols, size_t ncols, float* out, int threads) {
    if (v == V_XXS) {
        oracle_iq2xxs_matmul_f32(x, m, out_dim, in_dim, wb, ws, cols, ncols, out, threads);
        return;
    }
    size_t nb = (in_dim + QK - 1) / QK;
    size_t nc = cols ? ncols : out_dim;
    long long total = (long long)(m * nc);
    if (threads <= 0) threads = 1;
#pragma omp parallel for schedule(dynamic, 8) num_threads(threads)
    for (long long i = 0; i < total; ++i) {
        size_t row = (size_t)i / nc, c = (size_t)i % nc;
        size_t n = cols ? (size_t)cols[c] : c;
        out[row * nc + c] = dot(v, x + row * in_dim, in_dim, n, nb, wb, ws);
    }
}

/* decode_iq2_xs_value / decode_iq2_s_value / decode_iq3_s_value (iq2_matmul.metal:736-866). */
static float value(int v, const uint8_t* wb, const uint8_t* ws, size_t bi, size_t col) {
    const uint8_t* q = wb + bi * BYTES[v];
    const uint8_t* s = ws + bi * SCALES[v];
    float d = oracle_f16_to_f32(rd16(s));
    size_t ib32 = col / 32, w32 = col % 32;
    if (v == V_XS) {
        size_t word = w32 / 8, j = w32 % 8;
        uint16_t qw = rd16(q + ib32 * 8 + 2 * word);
        uint8_t sb = s[2 + ib32];
        float dl = word < 2 ? d * (0.5f + (float)(sb & 0x0F)) * 0.25f : d * (0.5f + (float)((sb >> 4) & 0x0F)) * 0.25f;
        uint8_t gv = (uint8_t)((ref_iq2xs_grid[qw & 0x1FF] >> (8 * j)) & 0xFF);
        float sgn = (ref_ksigns_iq2xs[(qw >> 9) & 0x7F] & ref_kmask_iq2xs[j]) ? -1.0f : 1.0f;
        return dl * (float)gv * sgn;
    }
    if (v == V_S) {
        size_t il = w32 / 16, w16 = w32 % 16, j = w16 % 8;
        uint8_t nib = (uint8_t)(q[64 + ib32] >> (4 * il));
        float dl = d * (0.5f + (float)((s[2 + ib32] >> (4 * il)) & 0x0F)) * 0.25f;
        size_t off = 4 * ib32 + 2 * il;
        size_t gi;
        uint8_t sign;
        if (w16 < 8) {
            gi = (size_t)q[off] | (((size_t)nib << 8) & 0x300);
            sign = q[32 + off];
        } else {
            gi = (size_t)q[off + 1] | (((size_t)nib << 6) & 0x300);
            sign = q[32 + off + 1];
        }
        uint8_t gv = (uint8_t)((ref_iq2s_grid[gi] >> (8 * j)) & 0xFF);
        float sgn = (sign & ref_kmask_iq2xs[j]) ? -1.0f : 1.0f;
        return dl * (float)gv * sgn;
    }
    /* IQ3_S */
    size_t l = w32 / 8, w8 = w32 % 8;
    uint8_t qh = q[64 + ib32];
    uint8_t nib = (uint8_t)((s[2 + ib32 / 2] >> (4 * (ib32 % 2))) & 0x0F);
    float dl = d * (1.0f + 2.0f * (float)nib);
    size_t i1 = (size_t)q[8 * ib32 + 2 * l] | ((qh & ref_kmask_iq2xs[2 * l]) ? 256u : 0u);
    size_t i2 = (size_t)q[8 * ib32 + 2 * l + 1] | ((qh & ref_kmask_iq2xs[2 * l + 1]) ? 256u : 0u);
    uint8_t sign = q[72 + 4 * ib32 + l];
    if (w8 < 4) {
        uint8_t gv = (uint8_t)((ref_iq3s_grid[i1] >> (8 * w8)) & 0xFF);
        return dl * (float)gv * ((sign & ref_kmask_iq2xs[w8]) ? -1.0f : 1.0f);
    }
    uint8_t gv = (uint8_t)((ref_iq3s_grid[i2] >> (8 * (w8 - 4))) & 0xFF);
    return dl * (float)gv * ((sign & ref_kmask_iq2xs[w8]) ? -1.0f : 1.0f);
}

/* As oracle_iq2xxs_dequantize, for variant 0..3. */
void oracle_iq2_dequantize(int v, const uint8_t* wb, const uint8_t* ws, size_t out_dim, size_t in_dim,
                           int out_dtype, void* out, int threads) {
    if (v == V_XXS) {
        oracle_iq2xxs_dequantize(wb, ws, out_dim, in_dim, out_dtype, out, threads);
        return;
    }
    size_t nb = (in_dim + QK - 1) / QK;
    long long total = (long long)(out_dim * in_dim);
    if (threads <= 0) threads = 1;
#pragma omp parallel for schedule(static) num_threads(threads)
    for (long long gid = 0; gid < total; ++gid) {
        size_t n = (size_t)gid / in_dim, col = (size_t)gid % in_dim;
        float val = value(v, wb, ws, n * nb + col / QK, col % QK);
        if (out_dtype == 0) ((float*)out)[gid] = val;
        else if (out_dtype == 1) ((uint16_t*)out)[gid] = oracle_f32_to_f16(val);
        else ((uint16_t*)out)[gid] = oracle_f32_to_bf16(val);
    }
}
