// IQ2_XXS decode GEMV for small m (m <= 32) on sm_100a, single or grouped projections.
//
// Computes out[m, n] = sum_k x[m, k] * W[n, k] with W the IQ2_XXS weights in the reference's
// split layout (reference: iq2_xxs_matmul_kernel, src/metal_src/iq2_matmul.metal:188-240;
// weight formula decode_iq2_xxs_value :701-734):
//   W[n, blk*256 + ib32*32 + g*8 + j] = d * (0.5 + s) * 0.25 * grid[aux_g.byte g].byte j * sign
// with, per 32-weight sub-block ib32 of block blk (8 bytes at qs + (n*nb + blk)*64 + ib32*8):
//   aux_g = bytes 0..3 (four 8-bit grid indices), aux_s = bytes 4..7 (four 7-bit sign indices
//   at bits 7g..7g+6, 4-bit scale s at bits 28..31), d = fp16 block scale.
//
// B200 design. At m = 1 every weight is used once, so what matters is the work per weight
// between HBM and an accumulator; the weights never become floats:
//   * d*(0.5+s)*0.25 = d*(2s+1)/8 and every signed grid value is an int8 in {+-8,+-25,+-43}. One
//     `prmt` turns a 16-bit selector (grid code | sign, from two lane-replicated shared-memory
//     tables that each CTA builds, so a warp's random lookups never share a bank) into four
//     signed int8 weights.
//   * x is turned per (token, 256-block) into fixed point: for m <= 4 four 7-bit signed limbs of
//     a 28-bit value (two tokens fill the eight columns of one n8 tile); for 5 <= m <= 32 a
//     16-bit value split into a signed high byte and an unsigned low byte (eight tokens per pair
//     of n8 tiles: high bytes in the first half of the tiles, low bytes in the second, multiplied
//     with mma .s8.u8). x @ W^T becomes mma.m16n8k32 per 32-weight sub-block, scaled by the odd
//     integer 2s+1 in s32 (exact, |sum| < 2^31) and turned into f32 once per 256-block with d and
//     the limb scale. The only roundings are the quantisation of x (2^-28 or 2^-16 of the
//     block's largest |x|) and f32 rounding of per-block partial sums (rel. error ~1e-6 for
//     m <= 4, ~4e-5 above).
//   * Weights stream through a per-warp cp.async ring in shared memory (one 256-weight block of
//     ROWS rows per stage), 16-byte chunks XOR-swizzled so the rows a warp reads together sit in
//     different banks; one 16-byte read feeds two sub-blocks.
//   * Work split: the launch's row tiles (ROWS rows x all of K of one projection) are dealt to
//     pairs of CTAs (2-CTA clusters) in contiguous ranges of about equal work; inside a pair the
//     32 warps split the range's (tile, block, sub-block) steps into equal contiguous pieces
//     (stream-K). A tile cut between warps is finished after a cluster barrier by its first warp,
//     which sums the partials of its warps in warp order, reading the other CTA's through
//     distributed shared memory: deterministic, and nothing goes through global memory.
//   * x limbs: a single projection whose limbs fit in shared memory gets them computed by every
//     CTA from x directly (one kernel per call); otherwise gemv_prep_kernel writes them to the
//     workspace once per distinct x and the GEMV reads them from L2.
//   * Grouped launches serve up to 256 projections (e.g. q/k/v or gate/up sharing x) with one
//     prep and one GEMV launch. Kernels use programmatic dependent launch: before its wait a
//     GEMV only builds its constant table and prefetches its first weights into L2.
//   * The other formats (template parameter FMT, single projections, x limbs from the prep
//     kernel; reference decode_iq2_xs_value / decode_iq2_s_value / decode_iq3_s_value,
//     iq2_matmul.metal:736-866): IQ2_XS and IQ2_S keep the selector decode with their larger grids
//     and run two MMAs per sub-block for their 16-weight scales; IQ3_S's grid holds the int8
//     magnitudes themselves and its signs are applied with a byte mask. Their blocks that are not
//     16-byte aligned (IQ2_S 72 bytes, IQ3_S 104) are staged as aligned windows around them.
#include "iq2xxs_common.cuh"
#include "iq2xxs_codebook.h"
#include "iq2_variant_grids.h"
#include "iq2xxs_internal.h"

#include <cstring>
#include <type_traits>
#include <vector>

namespace iq2 {

namespace {

constexpr int GEMV_WARPS = 16;            // per CTA; a cluster (2 CTAs) has 32
constexpr int CLUSTER = 2;
constexpr int LUT_BYTES = 256 * 256;      // 256 rows x (32 lanes grid selectors | 32 lanes sign)
// IQ2_XS: 512 grid rows x 32 lanes (64 KB), then 128 sign rows x 32 lanes
constexpr int LUT_BYTES_XS = 512 * 128 + 128 * 128;
// IQ2_S: 1024 grid rows x 16 lane copies (64 KB), then 256 sign rows x 16 lane copies
constexpr int LUT_BYTES_S = 1024 * 64 + 256 * 64;
// IQ3_S: 512 grid rows x 32 lane copies (64 KB, row `low * 2 + hb` of 128 bytes), then the 16
// sign-nibble rows x 16 lane copies of {byte mask, its low bits} (8 bytes each)
constexpr int LUT_BYTES_3S = 512 * 128 + 16 * 128;
constexpr int MAX_PROBLEMS = 256;         // per grouped launch
constexpr int MAX_CLUSTERS = 96;          // >= SMs / 2 of the device (74 on B200)
constexpr int SMEM_LIMIT = 227 * 1024;

// LB: the x encoding. 4: four 7-bit limbs per token (28 bits, m <= 4, two tokens per n8 tile);
// 16: the 16-bit split (5 <= m <= 32; tiles [0, NT/2) hold eight tokens' signed high bytes,
// tiles [NT/2, NT) the same tokens' unsigned low bytes); 1: the int8 activations of the W8A8
// mode, eight tokens per n8 tile.
// FMT: the weight format, 0 IQ2_XXS, 1 IQ2_XS (its 512-entry grid needs an 80 KB table, its
// scales a 16-byte slot per row and stage), 2 IQ2_S (1024-entry grid and its 256-entry sign table
// at 16 copies, 80 KB; per row and stage the 16-byte aligned 80-byte window around the row's
// 72-byte block, then a 12-byte scale slot), 3 IQ3_S (512-entry grid of int8 magnitudes at 32
// copies and a 16-entry sign-nibble table, 66 KB; the 112-byte window around the 104-byte block,
// then an 8-byte scale slot).
template <int NT, int LB = 4, int FMT = 0>
struct GemvShape {
    static constexpr bool SPLIT = LB == 16;
    static constexpr int LUT = FMT == 3 ? LUT_BYTES_3S : (FMT == 2 ? LUT_BYTES_S : (FMT == 1 ? LUT_BYTES_XS : LUT_BYTES));
    static constexpr int SLOT = FMT == 0 ? 4 : (FMT == 1 ? 16 : (FMT == 2 ? 12 : 8));  // per row: the scales
    static constexpr int QROW = FMT == 2 ? 80 : (FMT == 3 ? 112 : 64);                 // per row: the packed bytes
    static constexpr int T = ((NT <= 2 && LB != 1) || (NT == 1 && LB == 1)) ? 2 : 1;  // 16-row mma tiles per warp
    static constexpr int ROWS = 16 * T;                // rows of a tile
    static constexpr int TPN = SPLIT ? 8 : 8 / LB;     // tokens per n8 tile (SPLIT: per high-byte tile)
    static constexpr int TOK = SPLIT ? 4 * NT : TPN * NT;  // tokens incl. the zero padding
    static constexpr int STAGE_QS = ROWS * QROW;       // one block of qs per row
    // + per row the aligned scale word (IQ2_XS, IQ2_S: the 12 aligned bytes holding d and the 8
    // scale bytes)
    static constexpr int STAGE_BYTES = STAGE_QS + ROWS * SLOT;
    // fewer stages where the partials (TOK x ROWS per warp slot) are large
    static constexpr int NSTAGES0 = T == 2 ? 3 : ((LB == 4 || (LB == 1 && NT <= 2) || (SPLIT && NT <= 4)) ? 6 : 4);
    static constexpr int PART_BYTES = GEMV_WARPS * 2 * TOK * ROWS * 4;  // [warp][first|last][token][row]
    // IQ2_XS, IQ2_S, IQ3_S: as many as fit beside the larger table (2..5)
    static constexpr int NS_FIT = (SMEM_LIMIT - LUT - PART_BYTES) / ((GEMV_WARPS + 1) * STAGE_BYTES);
    static constexpr int NSTAGES = FMT != 0 ? (NS_FIT < NSTAGES0 ? NS_FIT : NSTAGES0) : NSTAGES0;
    static_assert(NSTAGES >= 2, "stages");
    static constexpr int RING_BYTES = NSTAGES * STAGE_BYTES;  // per warp
    // The table sits at the first 64 KB-aligned shared address of the block's window and the
    // warps' rings fill the space around it; whatever the window's base, this suffices:
    static constexpr int SMEM = LUT + (GEMV_WARPS + 1) * RING_BYTES + PART_BYTES;
};

int nt_for(uint32_t m) { return m <= 2 ? 1 : (m <= 8 ? 2 : (m <= 16 ? 4 : 8)); }
int rows_for(uint32_t m) { return nt_for(m) <= 2 ? 32 : 16; }
int limbs_for(uint32_t m) { return m <= 4 ? 4 : 16; }  // the LB of GemvShape
int nt_w8a8(uint32_t m) { return m <= 8 ? 1 : (m <= 16 ? 2 : 4); }  // one limb: 8 tokens per n8 tile

// x limbs of one block (256 k) of one x, for the kernel-side layout
__host__ __device__ inline size_t xs_bytes(uint32_t nb, int nt) { return (size_t)nb * 8 * nt * 256; }
__host__ __device__ inline size_t cs_bytes(uint32_t nb, int nt) { return (size_t)nb * nt * 8 * sizeof(float); }

// ---------------------------------------------------------------------------------------------
// x -> int8 limb fragments of one (token m, block b). Lane = (sub-block sbi, group t) owns the 8
// activations k = b*256 + sbi*32 + t*8 + [0, 8). With amax = max |x| over the block,
// amax = f * 2^E (f in [0.5, 1)) and B = 7*LB - 1 bits (27 for four limbs, 13 for two):
//   q = rint(x * 2^(B-E)) (|q| <= 2^B), |q| = sum of 7-bit limbs L_l * 2^(7l) (the last one at
//   most 2^6), each limb carrying the sign of q; column scale of limb l = 2^(E - B + 7l) / 8 (the
//   /8 is the weight scale's (2s+1)/8). Non-finite blocks get NaN scales, so the output is NaN.
//   Tokens m >= M (the padding of the last n8 tile) get zero limbs and scales.
// Fragment layout (mma B operand, m16n8k32 "col"), sub-block sb, n8 tile nt = m / (8/LB):
//   xb[((sb*NT + nt)*32 + col*4 + t)*8 + i] = limb of group t, element i; col = (m % (8/LB))*LB + l.
template <typename XT, int NT, int LB = 4>
__device__ __forceinline__ void limb_job(const XT* __restrict__ x, uint32_t M, uint32_t K, uint32_t m,
                                         uint32_t b, uint8_t* xb, float* colscale, int lane) {
    const int sbi = lane >> 2, t = lane & 3;
    if (m >= M) {
        // a padding token (warp-uniform): zero limbs and zero column scales, nothing to read
        const size_t sb = (size_t)b * 8 + sbi;
        if constexpr (LB == 16) {
            const uint32_t ntile = m >> 3, col = m & 7u;
            *reinterpret_cast<uint2*>(xb + ((sb * NT + ntile) * 32 + col * 4 + t) * 8) = make_uint2(0u, 0u);
            *reinterpret_cast<uint2*>(xb + ((sb * NT + NT / 2 + ntile) * 32 + col * 4 + t) * 8) = make_uint2(0u, 0u);
            if (lane < 2) colscale[(size_t)b * (NT * 8) + (lane == 0 ? ntile : NT / 2 + ntile) * 8 + col] = 0.0f;
        } else {
            constexpr uint32_t TPN = 8 / LB;
            const uint32_t nt = m / TPN, colbase = (m % TPN) * LB;
#pragma unroll
            for (int l = 0; l < LB; ++l)
                *reinterpret_cast<uint2*>(xb + ((sb * NT + nt) * 32 + (colbase + l) * 4 + t) * 8) = make_uint2(0u, 0u);
            if (lane < LB) colscale[(size_t)b * (NT * 8) + nt * 8 + colbase + lane] = 0.0f;
        }
        return;
    }
    const size_t k0 = (size_t)b * QK + sbi * 32 + t * 8;
    const XT* xr = x + (size_t)min(m, M - 1u) * K;
    float v[8];
    float amax = 0.0f;
    bool bad = false;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const size_t k = k0 + i;
        v[i] = (m < M && k < K) ? to_f32(xr[k]) : 0.0f;
        bad |= !isfinite(v[i]);
        amax = fmaxf(amax, fabsf(v[i]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
    bad = __any_sync(0xFFFFFFFFu, bad);

    // E from the exponent field (amax normal); 2^(B-E) is then a normal float for E >= -100,
    // and x * 2^(B-E) is exact. Tiny or subnormal blocks take the library path.
    const uint32_t abits = __float_as_uint(amax);
    constexpr int B = LB == 16 ? 15 : 7 * LB - 1;
    const bool fast = (abits >> 23) >= 27u;  // amax >= 2^-100
    int E = (int)(abits >> 23) - 126;
    if (!fast && !bad && amax > 0.0f) frexpf(amax, &E);
    const float sc = __uint_as_float((uint32_t)(127 + B - E) << 23);
    if constexpr (LB == 16) {
        // q = rint(x * 2^(15-E)) in [-32768, 32767] (|x| < 2^E; the clamp only touches a value
        // that rounds up to 2^15), q = 256 * hi + lo with hi = q >> 8 signed, lo = q & 255 unsigned
        uint32_t hw[2] = {0u, 0u}, lw[2] = {0u, 0u};
        if (!bad && amax > 0.0f) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float f = rintf(fast ? v[i] * sc : ldexpf(v[i], B - E));
                const int q = (int)fminf(fmaxf(f, -32768.0f), 32767.0f);
                hw[i >> 2] |= ((uint32_t)(q >> 8) & 255u) << (8 * (i & 3));
                lw[i >> 2] |= ((uint32_t)q & 255u) << (8 * (i & 3));
            }
        }
        const uint32_t ntile = m >> 3, col = m & 7u;
        const size_t sb = (size_t)b * 8 + sbi;
        *reinterpret_cast<uint2*>(xb + ((sb * NT + ntile) * 32 + col * 4 + t) * 8) = make_uint2(hw[0], hw[1]);
        *reinterpret_cast<uint2*>(xb + ((sb * NT + NT / 2 + ntile) * 32 + col * 4 + t) * 8) =
            make_uint2(lw[0], lw[1]);
        if (lane < 2) {
            // column scale of the high byte 2^(E-15+8)/8, of the low byte 2^(E-15)/8
            float s;
            if (bad) s = __int_as_float(0x7FC00000);
            else if (amax == 0.0f) s = 0.0f;
            else s = ldexpf(1.0f, E - B - 3 + (lane == 0 ? 8 : 0));
            colscale[(size_t)b * (NT * 8) + (lane == 0 ? ntile : NT / 2 + ntile) * 8 + col] = s;
        }
    } else {
        uint32_t lo[LB], hi[LB];
#pragma unroll
        for (int l = 0; l < LB; ++l) lo[l] = hi[l] = 0u;
        if (!bad && amax > 0.0f) {
            if constexpr (LB == 4) {
                // element i -> one word whose byte l is its signed limb l: |q| < 2^27 spread into
                // four 7-bit bytes, negated bytewise for q < 0 ((0x80 - v) ^ 0x80 is -v mod 256 for
                // every byte v <= 127, with no borrow between bytes); then a 4x4 byte transpose per
                // half gives the words of limb l over elements 0..3 (lo) and 4..7 (hi)
                uint32_t w[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int q = (int)rintf(fast ? v[i] * sc : ldexpf(v[i], B - E));
                    const uint32_t mag = (uint32_t)(q < 0 ? -q : q);
                    const uint32_t sp = (mag & 0x7Fu) | ((mag << 1) & 0x7F00u) | ((mag << 2) & 0x7F0000u) |
                                        ((mag << 3) & 0x7F000000u);
                    w[i] = q < 0 ? ((0x80808080u - sp) ^ 0x80808080u) : sp;
                }
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    uint32_t* dst = h ? hi : lo;
                    const uint32_t a0 = prmt(w[4 * h], w[4 * h + 1], 0x5140u);  // {e0.b0, e1.b0, e0.b1, e1.b1}
                    const uint32_t a1 = prmt(w[4 * h], w[4 * h + 1], 0x7362u);  // {e0.b2, e1.b2, e0.b3, e1.b3}
                    const uint32_t b0 = prmt(w[4 * h + 2], w[4 * h + 3], 0x5140u);
                    const uint32_t b1 = prmt(w[4 * h + 2], w[4 * h + 3], 0x7362u);
                    dst[0] = prmt(a0, b0, 0x5410u);
                    dst[1] = prmt(a0, b0, 0x7632u);
                    dst[2] = prmt(a1, b1, 0x5410u);
                    dst[3] = prmt(a1, b1, 0x7632u);
                }
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int q = (int)rintf(fast ? v[i] * sc : ldexpf(v[i], B - E));
                    const uint32_t mag = (uint32_t)(q < 0 ? -q : q);
#pragma unroll
                    for (int l = 0; l < LB; ++l) {
                        const int limb =
                            (l < LB - 1) ? (int)((mag >> (7 * l)) & 127u) : (int)(mag >> (7 * (LB - 1)));
                        const uint32_t byte = (uint32_t)(uint8_t)(int8_t)(q < 0 ? -limb : limb);
                        if (i < 4) lo[l] |= byte << (8 * i);
                        else hi[l] |= byte << (8 * (i - 4));
                    }
                }
            }
        }
        constexpr uint32_t TPN = 8 / LB;
        const uint32_t nt = m / TPN, colbase = (m % TPN) * LB;
        const size_t sb = (size_t)b * 8 + sbi;
#pragma unroll
        for (int l = 0; l < LB; ++l) {
            uint2* dst = reinterpret_cast<uint2*>(xb + ((sb * NT + nt) * 32 + (colbase + l) * 4 + t) * 8);
            *dst = make_uint2(lo[l], hi[l]);
        }
        if (lane < LB) {
            float s;
            if (bad) s = __int_as_float(0x7FC00000);
            else if (amax == 0.0f) s = 0.0f;
            else s = ldexpf(1.0f, E - B - 3 + 7 * lane);
            colscale[(size_t)b * (NT * 8) + nt * 8 + colbase + lane] = s;
        }
    }
}

struct PrepItem {
    const void* x;
    uint8_t* xb;
    float* colscale;
    uint32_t K, nb, warp_begin, pad;
};

template <int CAP>
struct PrepLaunch {
    PrepItem item[CAP];
    uint32_t count, M;
};

// One warp per (x item, token m < TOK, block b).
template <typename XT, int NT, int CAP, int LB = 4>
__global__ void __launch_bounds__(256) gemv_prep_kernel(const __grid_constant__ PrepLaunch<CAP> L) {
    // The GEMV may be scheduled at once: before its own wait it only copies weights and builds
    // its constant table. x may be written by the previous kernel and the workspace may still be
    // read by the previous GEMV, so wait for both before touching memory.
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t wid = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    uint32_t it = 0;
    while (it + 1 < L.count && L.item[it + 1].warp_begin <= wid) ++it;
    const PrepItem& P = L.item[it];
    const uint32_t local = wid - P.warp_begin;
    if (local >= (uint32_t)GemvShape<NT, LB>::TOK * P.nb) return;
    limb_job<XT, NT, LB>(static_cast<const XT*>(P.x), L.M, P.K, local / P.nb, local % P.nb, P.xb, P.colscale,
                         lane);
}

// W8A8 activations (the reference's per-row int8 quantisation, src/metal_src/iq2_matmul.metal:
// 85-102): inv = 127 / max|x| over the row (1 when that is below 1e-8), q = clamp(round(x * inv),
// -127, 127). The int8 q is the GEMV's single limb (col = m % 8, n8 tile m / 8); the column scale
// (1/inv)/8 is the same for every block of the row (the /8 is the weight scale's (2s+1)/8), so
// x' = q / inv times the weights is computed with one rounding of 1/inv instead of one per
// element. A row with a non-finite value gets NaN scales (its outputs are NaN). One warp per
// (x item, token m < 8*NT, block b), each reading its whole row for the maximum (from L2);
// tokens m >= M get zeros.
template <typename XT, int NT, int CAP>
__global__ void __launch_bounds__(256) gemv_prep_w8a8_kernel(const __grid_constant__ PrepLaunch<CAP> L) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t wid = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    uint32_t it = 0;
    while (it + 1 < L.count && L.item[it + 1].warp_begin <= wid) ++it;
    const PrepItem& P = L.item[it];
    const uint32_t local = wid - P.warp_begin;
    if (local >= 8u * NT * P.nb) return;
    const uint32_t m = local / P.nb, b = local % P.nb;
    const XT* xr = static_cast<const XT*>(P.x) + (size_t)min(m, L.M - 1u) * P.K;
    const bool live = m < L.M;
    float amax = 0.0f;
    if (live)
        for (uint32_t k = lane; k < P.K; k += 32) amax = fmaxf(amax, fabsf(to_f32(xr[k])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
    const bool bad = !isfinite(amax);
    const float inv = amax < 1e-8f ? 1.0f : 127.0f / amax;
    const float scale = bad ? __int_as_float(0x7FC00000) : (live ? __fdiv_rn(1.0f, inv) * 0.125f : 0.0f);
    const int sbi = lane >> 2, t = lane & 3;
    const uint32_t nt = m >> 3, col = m & 7u;
    {
        const size_t k0 = (size_t)b * QK + sbi * 32 + t * 8;
        uint32_t lo = 0, hi = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const size_t k = k0 + i;
            float q = 0.0f;
            if (live && !bad && k < P.K)
                q = fminf(fmaxf(roundf(__fmul_rn(to_f32(xr[k]), inv)), -127.0f), 127.0f);
            const uint32_t byte = (uint32_t)(uint8_t)(int8_t)(int)q;
            if (i < 4) lo |= byte << (8 * i);
            else hi |= byte << (8 * (i - 4));
        }
        const size_t sb = (size_t)b * 8 + sbi;
        *reinterpret_cast<uint2*>(P.xb + ((sb * NT + nt) * 32 + col * 4 + t) * 8) = make_uint2(lo, hi);
        if (lane == 0) P.colscale[(size_t)b * (NT * 8) + nt * 8 + col] = scale;
    }
}

// ---------------------------------------------------------------------------------------------
struct GemvProblem {  // 64 bytes
    const uint8_t* qs;
    const uint8_t* sc;
    const uint8_t* xb;        // x fragments from the prep kernel (unused when fused)
    const float* colscale;    // their column scales
    float* out;
    uint32_t N, nb, tiles, tb_begin;  // tiles = ceil(N / ROWS); tb_begin: first tile-block (ROWS rows x 1 block)
    uint32_t ldo;                     // elements between output rows
    uint32_t pad;
};

template <int CAP>
struct GemvLaunch {
    GemvProblem prob[CAP];
    uint32_t count, M;
    const void* x;                          // fused: the activations [M, K] of the single projection
    uint32_t K, clusters;
    uint32_t cl_tb[MAX_CLUSTERS + 1];       // cluster c owns tile-blocks [cl_tb[c], cl_tb[c+1]) (whole tiles)
    uint16_t cl_p[MAX_CLUSTERS];            // problem of the cluster's first tile
    // 2, as a value the compiler cannot see: the decode forms each weight scale 2s+1 as one
    // multiply-add on the FMA pipe instead of a shift and an OR on the integer ALU pipe that
    // bounds the kernel (3 % on the grouped M=1 launch)
    uint32_t two;
    GemvPeers peers;                        // peer-memory outputs (P2P launches only)
};

constexpr unsigned long long PEER_WAIT_NS = 1000000000ull;  // 1 s: a rank that never arrives

__device__ __forceinline__ SymmHeader* peer_header(const GemvPeers& pe, int r) {
    return reinterpret_cast<SymmHeader*>(reinterpret_cast<char*>(pe.hdr) + pe.delta[r]);
}

// Stream-K partition of [base, base + 32q + r) over a cluster's 32 warps: the first r get q+1 steps.
struct Partition {
    uint32_t q, r, base;
    __device__ __forceinline__ uint32_t begin(uint32_t w) const { return base + w * q + min(w, r); }
    __device__ __forceinline__ uint32_t owner(uint32_t s) const {
        const uint32_t ls = s - base, big = r * (q + 1);
        return ls < big ? ls / (q + 1) : r + (ls - big) / q;
    }
};

// Cursor over the tile-blocks (problem p, tile rg, block blk) of a launch, in order.
struct TbCursor {
    uint32_t tb, p, rg, blk;
};

template <int CAP>
__device__ __forceinline__ void cursor_seek(const GemvLaunch<CAP>& L, uint32_t p, uint32_t tb, TbCursor& c) {
    while (p + 1 < L.count && L.prob[p + 1].tb_begin <= tb) ++p;
    const uint32_t local = tb - L.prob[p].tb_begin;
    c.tb = tb;
    c.p = p;
    c.rg = local / L.prob[p].nb;
    c.blk = local % L.prob[p].nb;
}

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of the same shared-memory byte in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_shared(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}

// Per-lane decode constants. The table base is 64 KB-aligned, so every table address is
// assembled by one byte permute (grid: base | idx<<8 | lane*4) or one LOP3 (sign: base | 128 |
// sidx<<8 | lane*4), with no add.
struct DecodeK {
    uint32_t gsrc;  // bytes {lane*4, 0, base.b2, base.b3}
    uint32_t gsel;  // prmt selector {gsrc.b0, aux_g.byte t, gsrc.b2, gsrc.b3}
    uint32_t rot;   // rotate that brings sign index t (bits 7t..7t+6) to bits 8..14
    uint32_t soff;  // base | 128 | lane*4
    // IQ2_XS: prmt selector taking this lane's u16 word t of a sub-block to bits 0..15, and the
    // grid / sign tables' bases | lane*4 (both 64 KB-aligned, rows of 128 bytes).
    // IQ2_S: xsel = {byte t, 0, 0, 0}; sbase = sign table | (lane % 16) * 4 (rows of 64 bytes);
    // gsel2 = {qa.b0, low byte t, qa.b2, qa.b3} for the grid address word (+1: qa.b1); qsh the
    // shift taking qh bits 2t, 2t+1 of every byte to bits 6, 7; qfill = (lane % 16) * 4 in
    // every byte; lutw the table base (its bytes 2, 3)
    uint32_t xsel, gbase, sbase;
    uint32_t gsel2, qsh, qfill, lutw;
    uint32_t two;  // GemvLaunch::two
    // IQ3_S: xsel = {byte 2t, byte 2t+1} of a sub-block's 8 grid low bytes; qsh = 2t; qfill =
    // (lane * 4) in bytes 0 and 1 and the table base in bytes 2, 3; sbase = sign table | (lane %
    // 16) * 8; st8 = 8t
    uint32_t st8;
};

// Four signed int8 weights of one 8-weight group (sub-block word {aux_g, aux_s}) for this
// lane's group t: lo = weights 0..3, hi = weights 4..7.
__device__ __forceinline__ void decode_group(const DecodeK& k, uint32_t aux_g, uint32_t aux_s,
                                             uint32_t& lo, uint32_t& hi) {
    const uint32_t ga = prmt(aux_g, k.gsrc, k.gsel);
    const uint32_t sa = (__funnelshift_r(aux_s, aux_s, k.rot) & 0x7F00u) | k.soff;
    const uint32_t sel = ld_shared_const(ga) | ld_shared_const(sa);
    lo = prmt(KPOS, KNEG, sel);
    hi = prmt(KPOS, KNEG, sel >> 16);
}

// IQ2_XS: four signed int8 weights of one 8-weight group for this lane's word t of the sub-block
// {lo32 = words 0, 1; hi32 = words 2, 3} (grid index bits 0..8, sign index bits 9..15).
__device__ __forceinline__ void decode_group_xs(const DecodeK& k, uint32_t lo32, uint32_t hi32, uint32_t& lo,
                                                uint32_t& hi) {
    const uint32_t word = prmt(lo32, hi32, k.xsel);  // (bits 16..31: don't care)
    const uint32_t ga = ((word << 7) & 0xFF80u) | k.gbase;
    const uint32_t sa = ((word >> 2) & 0x3F80u) | k.sbase;
    const uint32_t sel = ld_shared_const(ga) | ld_shared_const(sa);
    lo = prmt(KPOS, KNEG, sel);
    hi = prmt(KPOS, KNEG, sel >> 16);
}

// IQ2_S: four signed int8 weights of one 8-weight group for this lane's group t of a sub-block
// (lows: its 4 grid low bytes, signs: its 4 sign bytes). The grid row of entry low | qh2 << 8
// sits at low * 256 + qh2 * 64 of the table, so its address is one permute of the low byte
// and qa = {(qh2 of sub-blocks 2j, 2j+1) << 6 | (lane % 16) * 4, same, table base bytes 2, 3};
// h picks the sub-block (qa.b0 or qa.b1; a constant after unrolling).
__device__ __forceinline__ void decode_group_s(const DecodeK& k, uint32_t lows, uint32_t signs, uint32_t qa,
                                               uint32_t h, uint32_t& lo, uint32_t& hi) {
    const uint32_t ga = prmt(lows, qa, k.gsel2 + h);
    const uint32_t sa = prmt(signs, 0u, k.xsel) * 64u + k.sbase;
    const uint32_t sel = ld_shared_const(ga) | ld_shared_const(sa);
    lo = prmt(KPOS, KNEG, sel);
    hi = prmt(KPOS, KNEG, sel >> 16);
}

// IQ3_S: eight signed int8 weights of one 8-weight group (lane t of a sub-block): lows = the
// sub-block's 8 grid low bytes, qw = its qh byte shifted right by 2t (bits j*8 + 0, 1 for
// j = sb % 4 are the high bits of the group's two grid indices), sw = its 4 sign bytes. The grid
// row of index low | hb << 8 sits at low * 256 + hb * 128 of the table, so its address is one
// permute of the low byte and {copy | hb << 7, copy | hb' << 7, base}; a sign nibble's table entry
// is {0xFF in each negative weight's byte, 0x01 in the same bytes}, and (g ^ mask) + low bits
// negates those bytes (the magnitudes are 1..15: no carry between bytes).
__device__ __forceinline__ void decode_group_3s(const DecodeK& k, uint2 lows, uint32_t qw, uint32_t j, uint32_t sw,
                                                uint32_t& lo, uint32_t& hi) {
    const uint32_t lw = prmt(lows.x, lows.y, k.xsel);
    const uint32_t v = (qw >> (8u * j)) & 3u;
    const uint32_t qa = ((v * 0x4080u) & 0x8080u) | k.qfill;
    const uint32_t g1 = ld_shared_const(prmt(lw, qa, 0x7604u));
    const uint32_t g2 = ld_shared_const(prmt(lw, qa, 0x7615u));
    const uint32_t t1 = sw >> k.st8;
    const uint2 m1 = ld_shared_v2_const((t1 & 15u) * 128u + k.sbase);
    const uint2 m2 = ld_shared_v2_const(((t1 >> 4) & 15u) * 128u + k.sbase);
    lo = (g1 ^ m1.x) + m1.y;
    hi = (g2 ^ m2.x) + m2.y;
}

__device__ __forceinline__ uint32_t ld_shared_u8_volatile(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.u8 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}

// IQ2_XS / IQ2_S stage: as stage_compute, but the scale changes every 16 weights (groups 0-1:
// the low nibble of the sub-block's scale byte, groups 2-3: the high one). Lane t holds group t's
// weights, i.e. MMA k-chunks 4t.. and 16+4t.., so two MMAs whose x fragments are zero on lanes
// t >= 2 (resp. t < 2) give the two halves' sums, each scaled by its 2s+1. slot_s: this stage's
// slot of row g (row r at + (r - g) * SLOT); so: the offset of the first scale byte in it.
// IQ2_S: rowbase is row g's block in the stage (its 80-byte window + 0 or 8; row r at
// + (r - g) * 80): grid low bytes of sub-block sb at + 4 sb, sign bytes at + 32 + 4 sb, qh at + 64.
template <int NT, int T, bool PARTIAL, bool SPLIT, int FMT, int SLOT>
__device__ __forceinline__ void stage_compute_xs(const DecodeK& dk, uint32_t st_s, const uint8_t* xbp, uint32_t s_lo,
                                                 uint32_t s_hi, uint32_t rowbase, uint32_t swz, uint32_t slot_s,
                                                 uint32_t so, bool low_lane, int (&I)[T][NT][4]) {
    const uint32_t sc_s = slot_s + so;
    // IQ2_S: per row (tt, half) the qh words of sub-blocks 0-3 / 4-7, this lane's two bits of
    // every byte at bits 6, 7 and (lane % 16) * 4 below them
    uint32_t qx[T][2], qy[T][2];
    if constexpr (FMT == 2) {
#pragma unroll
        for (int tt = 0; tt < T; ++tt)
#pragma unroll
            for (int hr = 0; hr < 2; ++hr) {
                const uint2 q = ld_shared_v2_volatile(st_s + rowbase + (uint32_t)((tt * 16 + hr * 8) * 80) + 64u);
                qx[tt][hr] = ((q.x << dk.qsh) & 0xC0C0C0C0u) | dk.qfill;
                qy[tt][hr] = ((q.y << dk.qsh) & 0xC0C0C0C0u) | dk.qfill;
            }
    }
#pragma unroll
    for (int pair = 0; pair < 4; ++pair) {
        // qw[tt][half]: IQ2_XS: the 16-byte chunk of sub-blocks 2 pair, 2 pair + 1; IQ2_S: their
        // {lows, lows, signs, signs}
        uint4 qw[T][2];
        if constexpr (FMT == 2) {
#pragma unroll
            for (int tt = 0; tt < T; ++tt)
#pragma unroll
                for (int hr = 0; hr < 2; ++hr) {
                    const uint32_t ra = st_s + rowbase + (uint32_t)((tt * 16 + hr * 8) * 80 + 8 * pair);
                    const uint2 l = ld_shared_v2_volatile(ra), sg = ld_shared_v2_volatile(ra + 32u);
                    qw[tt][hr] = make_uint4(l.x, l.y, sg.x, sg.y);
                }
        } else {
            const uint32_t a0 = st_s + rowbase + (((uint32_t)pair ^ swz) << 4);
            qw[0][0] = ld_shared_v4<0>(a0);
            qw[0][1] = ld_shared_v4<512>(a0);
            if (T == 2) {
                qw[T - 1][0] = ld_shared_v4<1024>(a0);
                qw[T - 1][1] = ld_shared_v4<1536>(a0);
            }
        }
        uint32_t qa[T][2];  // IQ2_S: the grid address words of this pair's sub-blocks
        if constexpr (FMT == 2) {
#pragma unroll
            for (int tt = 0; tt < T; ++tt)
#pragma unroll
                for (int hr = 0; hr < 2; ++hr)
                    qa[tt][hr] = prmt(pair < 2 ? qx[tt][hr] : qy[tt][hr], dk.lutw, (pair & 1) ? 0x7632u : 0x7610u);
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t sb = pair * 2 + h;
            uint32_t bfa[NT][2], bfb[NT][2];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                uint2 v = __ldg(reinterpret_cast<const uint2*>(xbp + (sb * NT + nt) * 256));
                if (PARTIAL && (sb < s_lo || sb >= s_hi)) v = make_uint2(0u, 0u);
                bfa[nt][0] = low_lane ? v.x : 0u;
                bfa[nt][1] = low_lane ? v.y : 0u;
                bfb[nt][0] = low_lane ? 0u : v.x;
                bfb[nt][1] = low_lane ? 0u : v.y;
            }
#pragma unroll
            for (int tt = 0; tt < T; ++tt) {
                uint32_t w0, w1, w2, w3;
                if constexpr (FMT == 2) {
                    const uint32_t l0 = h ? qw[tt][0].y : qw[tt][0].x, s0 = h ? qw[tt][0].w : qw[tt][0].z;
                    const uint32_t l1 = h ? qw[tt][1].y : qw[tt][1].x, s1 = h ? qw[tt][1].w : qw[tt][1].z;
                    decode_group_s(dk, l0, s0, qa[tt][0], (uint32_t)h, w0, w2);
                    decode_group_s(dk, l1, s1, qa[tt][1], (uint32_t)h, w1, w3);
                } else {
                    const uint32_t l0 = h ? qw[tt][0].z : qw[tt][0].x, h0 = h ? qw[tt][0].w : qw[tt][0].y;
                    const uint32_t l1 = h ? qw[tt][1].z : qw[tt][1].x, h1 = h ? qw[tt][1].w : qw[tt][1].y;
                    decode_group_xs(dk, l0, h0, w0, w2);
                    decode_group_xs(dk, l1, h1, w1, w3);
                }
                const uint32_t b0 = ld_shared_u8_volatile(sc_s + (uint32_t)(tt * 16 * SLOT) + sb);
                const uint32_t b1 = ld_shared_u8_volatile(sc_s + (uint32_t)((tt * 16 + 8) * SLOT) + sb);
                const int ca0 = (int)((b0 & 15u) * dk.two + 1u), cb0 = (int)((b0 >> 4) * dk.two + 1u);
                const int ca1 = (int)((b1 & 15u) * dk.two + 1u), cb1 = (int)((b1 >> 4) * dk.two + 1u);
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    int d1[4], d2[4];
                    if (SPLIT && nt >= NT / 2) {
                        mma_s8u8_16832(d1, w0, w1, w2, w3, bfa[nt][0], bfa[nt][1]);
                        mma_s8u8_16832(d2, w0, w1, w2, w3, bfb[nt][0], bfb[nt][1]);
                    } else {
                        mma_s8_16832(d1, w0, w1, w2, w3, bfa[nt][0], bfa[nt][1]);
                        mma_s8_16832(d2, w0, w1, w2, w3, bfb[nt][0], bfb[nt][1]);
                    }
                    const int v0 = ca0 * d1[0] + cb0 * d2[0], v1 = ca0 * d1[1] + cb0 * d2[1];
                    const int v2 = ca1 * d1[2] + cb1 * d2[2], v3 = ca1 * d1[3] + cb1 * d2[3];
                    if (sb == 0) {
                        I[tt][nt][0] = v0;
                        I[tt][nt][1] = v1;
                        I[tt][nt][2] = v2;
                        I[tt][nt][3] = v3;
                    } else {
                        I[tt][nt][0] += v0;
                        I[tt][nt][1] += v1;
                        I[tt][nt][2] += v2;
                        I[tt][nt][3] += v3;
                    }
                }
            }
        }
    }
}

// IQ3_S stage: as stage_compute (one scale per 32-weight sub-block, one MMA), with the row's
// 112-byte window at rowbase (+ (r - g) * 112): grid low bytes of sub-block sb at + 8 sb, qh at
// + 64, sign bytes at + 72 + 4 sb; the scale nibbles at sc_s (row r at + (r - g) * SLOT), two
// sub-blocks per byte.
template <int NT, int T, bool PARTIAL, bool SPLIT, int SLOT>
__device__ __forceinline__ void stage_compute_3s(const DecodeK& dk, uint32_t st_s, const uint8_t* xbp, uint32_t s_lo,
                                                 uint32_t s_hi, uint32_t rowbase, uint32_t sc_s, int (&I)[T][NT][4]) {
    uint32_t qx[T][2], qy[T][2];
#pragma unroll
    for (int tt = 0; tt < T; ++tt)
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
            const uint2 q = ld_shared_v2_volatile(st_s + rowbase + (uint32_t)((tt * 16 + hr * 8) * 112) + 64u);
            qx[tt][hr] = q.x >> dk.qsh;
            qy[tt][hr] = q.y >> dk.qsh;
        }
#pragma unroll
    for (int pair = 0; pair < 4; ++pair) {
        uint32_t cb[T][2];  // the scale byte of sub-blocks 2 pair, 2 pair + 1 of rows g (+ 8)
#pragma unroll
        for (int tt = 0; tt < T; ++tt) {
            cb[tt][0] = ld_shared_u8_volatile(sc_s + (uint32_t)(tt * 16 * SLOT + pair));
            cb[tt][1] = ld_shared_u8_volatile(sc_s + (uint32_t)((tt * 16 + 8) * SLOT + pair));
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t sb = pair * 2 + h;
            uint32_t bf[NT][2];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const uint2 v = __ldg(reinterpret_cast<const uint2*>(xbp + (sb * NT + nt) * 256));
                bf[nt][0] = v.x;
                bf[nt][1] = v.y;
                if (PARTIAL && (sb < s_lo || sb >= s_hi)) bf[nt][0] = bf[nt][1] = 0u;
            }
#pragma unroll
            for (int tt = 0; tt < T; ++tt) {
                uint32_t w[4];
#pragma unroll
                for (int hr = 0; hr < 2; ++hr) {
                    const uint32_t ra = st_s + rowbase + (uint32_t)((tt * 16 + hr * 8) * 112);
                    const uint2 lows = ld_shared_v2_volatile(ra + 8u * sb);
                    const uint32_t sw = ld_shared_u32_volatile(ra + 72u + 4u * sb);
                    decode_group_3s(dk, lows, sb < 4 ? qx[tt][hr] : qy[tt][hr], sb & 3u, sw, w[hr], w[2 + hr]);
                }
                const int c0 = (int)(((cb[tt][0] >> (4 * h)) & 15u) * dk.two + 1u);
                const int c1 = (int)(((cb[tt][1] >> (4 * h)) & 15u) * dk.two + 1u);
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    int d[4];
                    if (SPLIT && nt >= NT / 2) mma_s8u8_16832(d, w[0], w[1], w[2], w[3], bf[nt][0], bf[nt][1]);
                    else mma_s8_16832(d, w[0], w[1], w[2], w[3], bf[nt][0], bf[nt][1]);
                    if (sb == 0) {
                        I[tt][nt][0] = c0 * d[0];
                        I[tt][nt][1] = c0 * d[1];
                        I[tt][nt][2] = c1 * d[2];
                        I[tt][nt][3] = c1 * d[3];
                    } else {
                        I[tt][nt][0] += c0 * d[0];
                        I[tt][nt][1] += c0 * d[1];
                        I[tt][nt][2] += c1 * d[2];
                        I[tt][nt][3] += c1 * d[3];
                    }
                }
            }
        }
    }
}

// One stage (a block of ROWS rows) of the decode: s32 sums per 256-block in I. The first
// sub-block initialises I, so I needs no clearing. PARTIAL: only sub-blocks [s_lo, s_hi) count
// (the first/last stage of a warp's range); the others see zero x fragments. FUSED: fragments
// from shared memory (xsp: shared address), else from global memory (xbp).
template <int NT, int T, bool PARTIAL, bool FUSED, bool SPLIT>
__device__ __forceinline__ void stage_compute(const DecodeK& dk, uint32_t st_s, const uint8_t* xbp, uint32_t xsp,
                                              uint32_t s_lo, uint32_t s_hi, uint32_t rowbase, uint32_t swz,
                                              int (&I)[T][NT][4]) {
#pragma unroll
    for (int pair = 0; pair < 4; ++pair) {
        // one 16-byte chunk = sub-blocks 2*pair and 2*pair+1 of a row
        const uint32_t a0 = st_s + rowbase + (((uint32_t)pair ^ swz) << 4);
        uint4 qw[T][2];
        qw[0][0] = ld_shared_v4<0>(a0);
        qw[0][1] = ld_shared_v4<512>(a0);
        if (T == 2) {
            qw[T - 1][0] = ld_shared_v4<1024>(a0);
            qw[T - 1][1] = ld_shared_v4<1536>(a0);
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t sb = pair * 2 + h;
            uint32_t bf[NT][2];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                uint2 v;
                if (FUSED) v = ld_shared_v2_const(xsp + (sb * NT + nt) * 256);
                else v = __ldg(reinterpret_cast<const uint2*>(xbp + (sb * NT + nt) * 256));
                bf[nt][0] = v.x;
                bf[nt][1] = v.y;
                if (PARTIAL && (sb < s_lo || sb >= s_hi)) bf[nt][0] = bf[nt][1] = 0u;
            }
#pragma unroll
            for (int tt = 0; tt < T; ++tt) {
                const uint32_t g0 = h ? qw[tt][0].z : qw[tt][0].x, s0 = h ? qw[tt][0].w : qw[tt][0].y;
                const uint32_t g1 = h ? qw[tt][1].z : qw[tt][1].x, s1 = h ? qw[tt][1].w : qw[tt][1].y;
                uint32_t w0, w1, w2, w3;
                decode_group(dk, g0, s0, w0, w2);
                decode_group(dk, g1, s1, w1, w3);
                const int c0 = (int)((s0 >> 28) * dk.two + 1u), c1 = (int)((s1 >> 28) * dk.two + 1u);
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    int d[4];
                    if (SPLIT && nt >= NT / 2) mma_s8u8_16832(d, w0, w1, w2, w3, bf[nt][0], bf[nt][1]);
                    else mma_s8_16832(d, w0, w1, w2, w3, bf[nt][0], bf[nt][1]);
                    if (sb == 0) {
                        I[tt][nt][0] = c0 * d[0];
                        I[tt][nt][1] = c0 * d[1];
                        I[tt][nt][2] = c1 * d[2];
                        I[tt][nt][3] = c1 * d[3];
                    } else {
                        I[tt][nt][0] += c0 * d[0];
                        I[tt][nt][1] += c0 * d[1];
                        I[tt][nt][2] += c1 * d[2];
                        I[tt][nt][3] += c1 * d[3];
                    }
                }
            }
        }
    }
}

// XDT < 0: x fragments come from gemv_prep_kernel (workspace); XDT = 0/1/2: a single projection
// whose f32/f16/bf16 x this kernel turns into limbs itself (kernel-side layout in shared memory).
// P2P: every output is stored at the same offset of every rank's symmetric region (the
// column-sharded call's all-gather done by the epilogue), ordered by the header words.
template <int NT, int CAP, int XDT, bool P2P = false, int LB = 4, int FMT = 0>
__global__ void __launch_bounds__(GEMV_WARPS * 32, 1) gemv_kernel(const __grid_constant__ GemvLaunch<CAP> L) {
    using S_ = GemvShape<NT, LB, FMT>;
    static_assert(FMT == 0 || (!P2P && (LB == 4 || LB == 16)), "IQ2_XS, IQ2_S, IQ3_S: the plain decode GEMV only");
    constexpr uint32_t SC_B = FMT == 3 ? 6u : (FMT != 0 ? 10u : (uint32_t)SC_BYTES);  // scale bytes per block
    constexpr uint32_t QB = FMT == 3 ? 104u : (FMT == 2 ? 72u : (uint32_t)QS_BYTES);   // packed bytes per block
    // IQ2_S, IQ3_S: the row's block in 16-byte copies of its aligned window (the last one reads
    // only the block's 8 bytes when the block starts the window); the aligned scale words
    constexpr int NCH = FMT == 3 ? 7 : 5;
    constexpr int WIN = (int)S_::QROW;
    constexpr uint32_t NSW = FMT == 3 ? 2u : 3u;
    constexpr uint32_t SLOT = (uint32_t)S_::SLOT;
    constexpr bool FUSED = XDT >= 0;
    constexpr int T = S_::T, ROWS = S_::ROWS, TOK = S_::TOK, STAGE_QS = S_::STAGE_QS;
    constexpr int STAGE_BYTES = S_::STAGE_BYTES, NSTAGES = S_::NSTAGES, RING_BYTES = S_::RING_BYTES;
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    // The next call's kernels may be scheduled now; each waits for this grid to finish before
    // it touches memory this one uses.
    pdl_launch_dependents();

    // ---- shared layout: table at the first 64 KB-aligned address, rings around it, then the
    // ---- partial slots and (fused) the x limbs and their scales
    const uint32_t base_s = smem_u32(smem);
    const uint32_t lut_s = (base_s + 0xFFFFu) & ~0xFFFFu;
    const uint32_t gap = lut_s - base_s;
    const uint32_t gap_warps = min(gap / RING_BYTES, (uint32_t)GEMV_WARPS);
    const uint32_t ring_off = (uint32_t)warp < gap_warps
                                  ? (uint32_t)warp * RING_BYTES
                                  : gap + S_::LUT + ((uint32_t)warp - gap_warps) * RING_BYTES;
    uint8_t* ring = smem + ring_off;
    const uint32_t ring_s = base_s + ring_off;
    const uint32_t part_off = gap + S_::LUT + (GEMV_WARPS - gap_warps) * RING_BYTES;
    float* part = reinterpret_cast<float*>(smem + part_off);
    const uint32_t part_s = base_s + part_off;
    const uint32_t xs_off = part_off + S_::PART_BYTES;
    const uint32_t xs_s = base_s + xs_off;
    const uint32_t nbx = FUSED ? L.prob[0].nb : 0u;
    const uint32_t cs_off = xs_off + (uint32_t)xs_bytes(nbx, NT);
    (void)ring;

    // This warp's step range [a, b) of its cluster and the tile-blocks it touches [tb0, tb1).
    const uint32_t rank = cluster_rank();
    const uint32_t cl = blockIdx.x / CLUSTER;
    const uint32_t TB0 = L.cl_tb[cl], TB1 = L.cl_tb[cl + 1];
    const uint32_t S = (TB1 - TB0) * 8;
    const Partition part_{S / (CLUSTER * GEMV_WARPS), S % (CLUSTER * GEMV_WARPS), TB0 * 8};
    const uint32_t wg = rank * GEMV_WARPS + warp;  // warp index within the cluster
    const uint32_t a = part_.begin(wg), b = part_.begin(wg + 1);
    const uint32_t tb0 = a >> 3, tb1 = (b + 7) >> 3;
    const uint32_t p0 = L.cl_p[cl];

    // ---- issue side: cp.async stages of one tile-block each, NSTAGES ahead ----
    // State of the issue cursor: this lane's 16-byte chunk t of row g (iq; rows g+8c at
    // iq + c*i_rstep; IQ2_S: the block of row lane % ROWS) and the scale of row `lane` (isp). With up to four n8 tiles it is set up
    // once per tile (iss_tile) and advanced by one block per stage, so that a stage costs no
    // 64-bit index arithmetic (+4..7 % at m <= 8); the eight-tile kernels have no registers to
    // keep it across the loop and recompute it per stage.
    constexpr bool LEAN = NT <= 4;
    TbCursor ic;
    ic.tb = tb1;
    if (a < b) cursor_seek(L, p0, tb0, ic);
    const uint32_t tbf_lo = (a + 7) >> 3, tbf_hi = b >> 3;  // tile-blocks whose 8 sub-blocks are all this warp's
    const uint32_t lane_off = (uint32_t)g * 64u + ((((uint32_t)t) ^ (((uint32_t)g >> 1) & 3u)) << 4);
    const uint8_t* iq = nullptr;
    const uint8_t* isp = nullptr;
    const uint8_t* i_scend = nullptr;
    uint32_t i_rstep = 0, i_nb = 1, i_tiles = 1;
    bool i_full = false;
    auto iss_tile = [&]() {
        const GemvProblem& P = L.prob[ic.p];
        const uint32_t row0 = ic.rg * ROWS;
        i_nb = P.nb;
        i_tiles = P.tiles;
        i_full = row0 + ROWS <= P.N;
        i_rstep = P.nb * QB * 8u;
        // (IQ2_S, IQ3_S: the block of row lane % ROWS)
        iq = FMT >= 2 ? P.qs + ((size_t)(row0 + ((uint32_t)lane & (ROWS - 1))) * P.nb + ic.blk) * QB
                      : P.qs + ((size_t)(row0 + g) * P.nb + ic.blk) * QB + t * 16;
        isp = P.sc + ((size_t)(row0 + lane) * P.nb + ic.blk) * SC_B;
        i_scend = P.sc + (size_t)P.N * P.nb * SC_B;
    };
    if (LEAN && ic.tb < tb1) iss_tile();
    int islot = 0;
    auto issue = [&]() {
        if (ic.tb < tb1) {
            if (!LEAN) iss_tile();
            const uint32_t st_s = ring_s + islot * STAGE_BYTES;
            if (ic.tb >= tbf_lo && ic.tb < tbf_hi && i_full) {
                // the common case: every sub-block and every row of the stage is needed; chunk t
                // of row r = 8c + g goes to chunk t ^ ((r >> 1) & 3) of the row's 64 bytes
                if constexpr (FMT >= 2) {
                    // the 16-byte aligned window around the row's block (which starts at byte 0
                    // or 8 of it) in 16-byte copies; the last one reads only bytes of the block
                    const uint32_t odd = (uint32_t)reinterpret_cast<uintptr_t>(iq) & 8u;
                    const uint8_t* win = iq - odd;
                    const uint32_t r = (uint32_t)lane & (ROWS - 1);
#pragma unroll
                    for (int i = 0; i < (ROWS * NCH + 31) / 32; ++i) {
                        const uint32_t idx = (uint32_t)lane + 32u * i;
                        if ((ROWS * NCH) % 32 != 0 && idx >= (uint32_t)(ROWS * NCH)) break;
                        const uint32_t ch = idx / ROWS;
                        cp_async_16(st_s + r * WIN + ch * 16, win + ch * 16, (ch == NCH - 1 && !odd) ? 8u : 16u);
                    }
                } else {
#pragma unroll
                    for (int c = 0; c < ROWS * 4 / 32; ++c)
                        cp_async_16(st_s + c * 512 + lane_off, iq + (size_t)((uint32_t)c * i_rstep), 16u);
                }
                if (lane < ROWS) {
                    // the 4-byte aligned word holding this row's d (the buffer is 4-byte aligned;
                    // IQ2_XS: the three words holding d and the 8 scale bytes); at the end of the
                    // buffer only the bytes that exist are read
                    const uint8_t* ea = reinterpret_cast<const uint8_t*>(reinterpret_cast<uintptr_t>(isp) & ~(uintptr_t)3);
                    const size_t rem = (size_t)(i_scend - ea);
                    if constexpr (FMT != 0) {
#pragma unroll
                        for (uint32_t w = 0; w < NSW; ++w) {
                            const size_t r4 = rem > 4 * w ? rem - 4 * w : 0;
                            cp_async_4(st_s + STAGE_QS + lane * SLOT + 4 * w, r4 ? ea + 4 * w : ea,
                                       r4 < 4 ? (uint32_t)r4 : 4u);
                        }
                    } else {
                        cp_async_4(st_s + STAGE_QS + lane * 4, ea, rem < 4 ? (uint32_t)rem : 4u);
                    }
                }
            } else {
                const GemvProblem& P = L.prob[ic.p];
                const uint32_t row0 = ic.rg * ROWS;
                const uint32_t s_lo = ic.tb * 8 < a ? a - ic.tb * 8 : 0u;        // first sub-block needed
                const uint32_t s_hi = min(8u, b - ic.tb * 8);                     // one past the last
                const uint32_t ch_lo = s_lo >> 1, ch_hi = (s_hi + 1) >> 1;        // 16-byte chunks needed
                const uint8_t* qrow = P.qs + ((size_t)row0 * P.nb + ic.blk) * QB;
                const size_t row_bytes = (size_t)P.nb * QB;
                if constexpr (FMT >= 2) {
                    // rows that exist: their whole window, as in the common case; others: zeros
                    const uint32_t r = (uint32_t)lane & (ROWS - 1);
                    const bool ok = row0 + r < P.N;
                    const uint8_t* blkp = ok ? qrow + (size_t)r * row_bytes : P.qs;
                    const uint32_t odd = (uint32_t)reinterpret_cast<uintptr_t>(blkp) & 8u;
                    const uint8_t* win = blkp - odd;
#pragma unroll
                    for (int i = 0; i < (ROWS * NCH + 31) / 32; ++i) {
                        const uint32_t idx = (uint32_t)lane + 32u * i;
                        if ((ROWS * NCH) % 32 != 0 && idx >= (uint32_t)(ROWS * NCH)) break;
                        const uint32_t ch = idx / ROWS;
                        cp_async_16(st_s + r * WIN + ch * 16, ok ? win + ch * 16 : P.qs,
                                    ok ? ((ch == NCH - 1 && !odd) ? 8u : 16u) : 0u);
                    }
                } else {
#pragma unroll
                    for (int c = 0; c < ROWS * 4 / 32; ++c) {
                        const int idx = c * 32 + lane;
                        const int r = idx >> 2, ch = idx & 3;
                        const bool ok = row0 + r < P.N && (uint32_t)ch >= ch_lo && (uint32_t)ch < ch_hi;
                        const uint8_t* src = ok ? qrow + (size_t)r * row_bytes + ch * 16 : P.qs;
                        // swizzle: chunk ch of row r goes to chunk ch ^ ((r >> 1) & 3)
                        cp_async_16(st_s + r * 64 + ((ch ^ ((r >> 1) & 3)) << 4), src, ok ? 16u : 0u);
                    }
                }
                if (lane < ROWS) {
                    const uint32_t row = row0 + lane;
                    const bool ok = row < P.N;
                    const size_t e = ((size_t)row * P.nb + ic.blk) * SC_B;
                    const size_t ea = e & ~(size_t)3, total = (size_t)P.N * P.nb * SC_B;
                    if constexpr (FMT != 0) {
#pragma unroll
                        for (uint32_t w = 0; w < NSW; ++w) {
                            const size_t at = ea + 4 * w;
                            const uint32_t nbytes = ok && at < total ? (uint32_t)min((size_t)4, total - at) : 0u;
                            cp_async_4(st_s + STAGE_QS + lane * SLOT + 4 * w, P.sc + (nbytes ? at : 0), nbytes);
                        }
                    } else {
                        const uint32_t nbytes = ok ? (uint32_t)min((size_t)4, total - ea) : 0u;
                        cp_async_4(st_s + STAGE_QS + lane * 4, P.sc + (ok ? ea : 0), nbytes);
                    }
                }
            }
            ++ic.tb;
            iq += QB;
            isp += SC_B;
            if (++ic.blk == i_nb) {
                ic.blk = 0;
                if (++ic.rg == i_tiles) {
                    ic.rg = 0;
                    ++ic.p;
                }
                if (LEAN && ic.tb < tb1) iss_tile();
            }
        }
        cp_async_commit();
        islot = (islot + 1 == NSTAGES) ? 0 : islot + 1;
    };

    // The weights are only ever written by kernels that do not release their dependents early
    // (only this library's GEMV and prep kernels do, and they never write weights), so the first
    // stages can be copied before the wait: their DRAM latency overlaps the table build and the
    // previous kernel's tail.
#pragma unroll
    for (int i = 0; i < NSTAGES; ++i) issue();

    // ---- the decode table, built from the 1.5 KB compact copy: row e = 32 copies (one per lane)
    // ---- of the grid selector of code e, then (e < 128) 32 copies of the sign selector of index e
    if constexpr (FMT == 3) {
        // IQ3_S: grid index low | hb << 8 at low * 256 + hb * 128: 32 copies of its four magnitude
        // bytes; then row n (64 KB + n * 128) = 16 copies of {0xFF in byte j for bit j of n set,
        // the same bytes' low bits}
        for (int c = threadIdx.x; c < LUT_BYTES_3S / 16; c += blockDim.x) {
            uint4 v;
            if (c < 4096) {
                const uint32_t gv = IQ3S_GRID[(c >> 4) | (((c >> 3) & 1) << 8)];
                v = make_uint4(gv, gv, gv, gv);
            } else {
                const uint32_t n = (uint32_t)(c - 4096) >> 3;
                uint32_t mask = 0;
#pragma unroll
                for (int j = 0; j < 4; ++j) mask |= ((n >> j) & 1u) * (0xFFu << (8 * j));
                v = make_uint4(mask, mask & 0x01010101u, mask, mask & 0x01010101u);
            }
            *reinterpret_cast<uint4*>(smem + gap + c * 16) = v;
        }
    } else if constexpr (FMT == 2) {
        // IQ2_S: 64-byte rows of 16 copies: row 4 * low + qh2 (< 1024) = the grid selector of
        // grid entry low | qh2 << 8 (nibble j: the magnitude code of weight j); then sign row s =
        // the sign selector of sign byte s (nibble j: 4 when bit j is set)
        constexpr int PER_THREAD = LUT_BYTES_S / 16 / (GEMV_WARPS * 32);
        static_assert(LUT_BYTES_S % (16 * GEMV_WARPS * 32) == 0, "table chunks per thread");
        uint32_t v[PER_THREAD];
#pragma unroll
        for (int i = 0; i < PER_THREAD; ++i) {
            const int c = threadIdx.x + i * GEMV_WARPS * 32;
            const int row = c >> 2;
            uint32_t sel = 0;
            if (row < 1024) {
                const uint64_t gw = IQ2S_GRID[(row >> 2) | ((row & 3) << 8)];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const uint32_t b = (uint32_t)(gw >> (8 * j)) & 0xFFu;
                    sel |= (b == 8u ? 0u : (b == 25u ? 1u : 2u)) << (4 * j);
                }
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) sel |= (((uint32_t)(row - 1024) >> j) & 1u) << (4 * j + 2);
            }
            v[i] = sel;
        }
#pragma unroll
        for (int i = 0; i < PER_THREAD; ++i) {
            const int c = threadIdx.x + i * GEMV_WARPS * 32;
            *reinterpret_cast<uint4*>(smem + gap + c * 16) = make_uint4(v[i], v[i], v[i], v[i]);
        }
    } else if constexpr (FMT == 1) {
        // IQ2_XS: row e < 512 = 32 copies of the grid selector of grid entry e (nibble j: the
        // magnitude code of weight j), then row 512 + e (e < 128) = 32 copies of the sign selector
        // of sign index e (IQ2_XS uses IQ2_XXS's sign table)
        constexpr int PER_THREAD = LUT_BYTES_XS / 16 / (GEMV_WARPS * 32);
        uint32_t v[PER_THREAD];
#pragma unroll
        for (int i = 0; i < PER_THREAD; ++i) {
            const int row = (threadIdx.x + i * GEMV_WARPS * 32) >> 3;  // 8 x 16 bytes per row
            if (row < 512) {
                const uint64_t gw = IQ2XS_GRID[row];
                uint32_t sel = 0;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const uint32_t b = (uint32_t)(gw >> (8 * j)) & 0xFFu;
                    sel |= (b == 8u ? 0u : (b == 25u ? 1u : 2u)) << (4 * j);
                }
                v[i] = sel;
            } else {
                v[i] = __ldg(IQ2XXS_SEL_COMPACT + 256 + (row - 512));
            }
        }
#pragma unroll
        for (int i = 0; i < PER_THREAD; ++i) {
            const int c = threadIdx.x + i * GEMV_WARPS * 32;
            *reinterpret_cast<uint4*>(smem + gap + c * 16) = make_uint4(v[i], v[i], v[i], v[i]);
        }
    } else {
        constexpr int PER_THREAD = LUT_BYTES / 16 / (GEMV_WARPS * 32);
        uint32_t v[PER_THREAD];  // all loads first: one latency, not one per store
#pragma unroll
        for (int i = 0; i < PER_THREAD; ++i) {
            const int c = threadIdx.x + i * GEMV_WARPS * 32;
            const int row = c >> 4, half = (c >> 3) & 1;
            v[i] = half == 0 ? __ldg(IQ2XXS_SEL_COMPACT + row)
                             : (row < 128 ? __ldg(IQ2XXS_SEL_COMPACT + 256 + row) : 0u);
        }
#pragma unroll
        for (int i = 0; i < PER_THREAD; ++i) {
            const int c = threadIdx.x + i * GEMV_WARPS * 32;
            *reinterpret_cast<uint4*>(smem + gap + c * 16) = make_uint4(v[i], v[i], v[i], v[i]);
        }
    }

    if constexpr (FUSED) {
        constexpr uint32_t XB = XDT == 0 ? 4u : 2u;
        const uint8_t* xp = static_cast<const uint8_t*>(L.x);
        for (uint32_t o = threadIdx.x * 128u; o < L.M * L.K * XB; o += blockDim.x * 128u) prefetch_l2(xp + o);
    }
    // x (fused) or its fragments (prep kernel), and the outputs, may belong to earlier kernels.
    pdl_wait();
    // P2P entry: this rank has started call `epoch` (everything before it on this stream is
    // done, so no earlier kernel still reads the outputs); block 0 tells every rank at once. The
    // wait for the others is off the compute path: the first warp that is about to store takes
    // it on (go_owner), waits until every rank has entered, and opens `go` for the rest.
    // Once an exchange of this communicator has failed (the sticky error word is set, by a timed-out
    // wait or a rank-local failure of an earlier call) the ranks' call numbers can no longer be
    // trusted to match, so the call runs local-only: no entry, no waits, no peer stores; its
    // outputs hold this rank's columns only and iq2_comm_check keeps reporting the error until
    // the communicator is destroyed.
    unsigned long long epoch = 0;
    bool dead = false;
    if constexpr (P2P) {
        const GemvPeers& pe = L.peers;
        epoch = *reinterpret_cast<volatile unsigned long long*>(&pe.hdr->epoch) + 1ull;
        dead = *reinterpret_cast<volatile unsigned*>(&pe.hdr->err) != 0u;
        if (!dead && blockIdx.x == 0 && threadIdx.x == 0)
            for (int r = 0; r < pe.world; ++r) st_relaxed_sys_u64(peer_header(pe, r)->entry + pe.rank, epoch);
    }
    // Before its first store a warp sees `go` (one lane waits, bounded); if it never opens the
    // outputs stay local and the error bit is set.
    bool go_seen = !P2P || dead, peers_ok = P2P && !dead;
    auto wait_go = [&]() {
        if constexpr (P2P) {
            if (go_seen) return;
            int ok = 1;
            if (lane == 0) {
                const GemvPeers& pe = L.peers;
                const unsigned long long t0 = gtimer_ns();
                if (ld_acquire_gpu_u64(&pe.hdr->go) < epoch &&
                    atomicCAS(&pe.hdr->go_owner, epoch - 1ull, epoch) == epoch - 1ull) {
                    for (int r = 0; r < pe.world && ok; ++r)
                        while (ld_acquire_sys_u64(pe.hdr->entry + r) < epoch) {
                            if (gtimer_ns() - t0 > PEER_WAIT_NS) {
                                ok = 0;
                                break;
                            }
                            __nanosleep(32);
                        }
                    if (ok) st_release_gpu_u64(&pe.hdr->go, epoch);
                    else atomicOr(&pe.hdr->err, 1u);
                } else {
                    while (ld_acquire_gpu_u64(&pe.hdr->go) < epoch) {
                        if (gtimer_ns() - t0 > 2 * PEER_WAIT_NS) {
                            ok = 0;
                            break;
                        }
                        __nanosleep(32);
                    }
                }
            }
            ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
            __syncwarp();
            go_seen = true;
            peers_ok = ok != 0;
        }
    };
    auto put = [&](float* o, float v) {
        if constexpr (P2P) {
            if (peers_ok) {
                for (int r = 0; r < L.peers.world; ++r)
                    *reinterpret_cast<float*>(reinterpret_cast<char*>(o) + L.peers.delta[r]) = v;
                return;
            }
        }
        *o = v;
    };
    if constexpr (FUSED) {
        using XT = typename std::conditional<XDT == 0, float, typename std::conditional<XDT == 1, __half, __nv_bfloat16>::type>::type;
        for (uint32_t job = warp; job < TOK * nbx; job += GEMV_WARPS)
            limb_job<XT, NT, LB>(static_cast<const XT*>(L.x), L.M, L.K, job / nbx, job % nbx, smem + xs_off,
                             reinterpret_cast<float*>(smem + cs_off), lane);
    }
    __syncthreads();  // the table (and the fused limbs) are complete

    DecodeK dk;
    dk.two = L.two;
    dk.gsrc = (lut_s & 0xFFFF0000u) | ((uint32_t)lane * 4u);
    dk.gsel = 0x7604u | ((uint32_t)t << 4);
    dk.rot = (7u * t + 24u) & 31u;
    dk.soff = lut_s | 128u | ((uint32_t)lane * 4u);
    dk.xsel = (2u * t) | ((2u * t + 1u) << 4) | ((2u * t) << 8) | ((2u * t + 1u) << 12);
    dk.gbase = lut_s | ((uint32_t)lane * 4u);
    dk.sbase = (lut_s + 65536u) | ((uint32_t)lane * 4u);
    if constexpr (FMT == 2) {
        const uint32_t l16 = ((uint32_t)lane & 15u) * 4u;
        dk.xsel = (uint32_t)t | 0x4440u;
        dk.sbase = (lut_s + 65536u) | l16;
        dk.gsel2 = 4u | ((uint32_t)t << 4) | 0x7600u;
        dk.qsh = 6u - 2u * (uint32_t)t;
        dk.qfill = l16 * 0x01010101u;
        dk.lutw = lut_s;
    }
    if constexpr (FMT == 3) {
        dk.xsel = (2u * t) | ((2u * t + 1u) << 4);
        dk.qsh = 2u * (uint32_t)t;
        dk.qfill = ((uint32_t)lane * 4u) * 0x0101u | (lut_s & 0xFFFF0000u);
        dk.sbase = (lut_s + 65536u) | (((uint32_t)lane & 15u) * 8u);
        dk.st8 = 8u * (uint32_t)t;
    }
    const uint32_t swz = (uint32_t)((g >> 1) & 3);  // rows g, g+8, g+16, g+24 share it
    const uint32_t rowbase = (uint32_t)g * 64u;     // rows tt*16+g (+8): rowbase + tt*1024 (+512)

    float F[T][NT][4];
#pragma unroll
    for (int i = 0; i < T; ++i)
#pragma unroll
        for (int j = 0; j < NT; ++j)
#pragma unroll
            for (int k = 0; k < 4; ++k) F[i][j][k] = 0.0f;

    // Consumer cursor; per tile it keeps the problem's x fragments, column scales and block count.
    TbCursor cc;
    cc.tb = tb1;
    if (a < b) cursor_seek(L, p0, tb0, cc);
    const uint8_t* c_xb = nullptr;
    const float* c_cs = nullptr;
    uint32_t c_nb = 1, c_tiles = 1, c_dpar = 0;
    auto cons_tile = [&]() {
        const GemvProblem& P = L.prob[cc.p];
        c_nb = P.nb;
        c_tiles = P.tiles;
        c_xb = FUSED ? nullptr : P.xb + lane * 8;
        c_cs = FUSED ? nullptr : P.colscale + 2 * t;
        // d sits in the high half of its aligned word when row*nb + blk is odd; this lane's rows
        // all have the parity of g (tiles start at multiples of 16 rows)
        c_dpar = (uint32_t)g & P.nb & 1u;
    };
    if (cc.tb < tb1) cons_tile();
    int slot = 0;
    for (; cc.tb < tb1;) {
        cp_async_wait<NSTAGES - 1>();
        __syncwarp();
        const uint32_t st_s = ring_s + slot * STAGE_BYTES;
        const uint32_t s_lo = cc.tb * 8 < a ? a - cc.tb * 8 : 0u;
        const uint32_t s_hi = min(8u, b - cc.tb * 8);

        int I[T][NT][4];
        const uint8_t* xbp = FUSED ? nullptr : c_xb + (size_t)(cc.blk * (8u * NT * 256u));
        const uint32_t xsp = xs_s + cc.blk * 8 * NT * 256 + lane * 8;
        if constexpr (FMT != 0) {
            // the row's 12 scale bytes start at its slot; d is at byte 2 * parity, the sub-block
            // scale bytes after it (the parity of row * nb + blk, as for the d word)
            // (IQ2_S: the row's block sits at byte 8 * parity of its window)
            const uint32_t odd = (cc.blk & 1u) ^ c_dpar;
            const uint32_t so = odd ? 4u : 2u;
            const uint32_t slot_s = st_s + STAGE_QS + (uint32_t)g * SLOT;
            const uint32_t rb = FMT >= 2 ? (uint32_t)g * (uint32_t)WIN + odd * 8u : rowbase;
            if constexpr (FMT == 3) {
                // (IQ3_S: one scale per sub-block, one MMA)
                if (s_lo == 0 && s_hi == 8)
                    stage_compute_3s<NT, T, false, S_::SPLIT, SLOT>(dk, st_s, xbp, s_lo, s_hi, rb, slot_s + so, I);
                else
                    stage_compute_3s<NT, T, true, S_::SPLIT, SLOT>(dk, st_s, xbp, s_lo, s_hi, rb, slot_s + so, I);
            } else if (s_lo == 0 && s_hi == 8) {
                stage_compute_xs<NT, T, false, S_::SPLIT, FMT, SLOT>(dk, st_s, xbp, s_lo, s_hi, rb, swz, slot_s, so,
                                                                     t < 2, I);
            } else {
                stage_compute_xs<NT, T, true, S_::SPLIT, FMT, SLOT>(dk, st_s, xbp, s_lo, s_hi, rb, swz, slot_s, so,
                                                                    t < 2, I);
            }
        } else if (s_lo == 0 && s_hi == 8) {
            stage_compute<NT, T, false, FUSED, S_::SPLIT>(dk, st_s, xbp, xsp, s_lo, s_hi, rowbase, swz, I);
        } else {
            stage_compute<NT, T, true, FUSED, S_::SPLIT>(dk, st_s, xbp, xsp, s_lo, s_hi, rowbase, swz, I);
        }

        // Block epilogue: s32 -> f32 with d (per row) and the limb scale (per column).
        {
            float2 cs[NT];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const uint32_t ci = cc.blk * (NT * 8) + nt * 8;
                if (FUSED) cs[nt] = *reinterpret_cast<const float2*>(smem + cs_off + (ci + 2 * t) * 4);
                else cs[nt] = __ldg(reinterpret_cast<const float2*>(c_cs + ci));
            }
            const uint32_t dsel = ((cc.blk & 1u) ^ c_dpar) ? 0x3232u : 0x1010u;
#pragma unroll
            for (int tt = 0; tt < T; ++tt) {
                const uint32_t r0 = tt * 16 + g, r1 = r0 + 8;
                const uint32_t w0 = ld_shared_u32_volatile(st_s + STAGE_QS + r0 * SLOT);
                const uint32_t w1 = ld_shared_u32_volatile(st_s + STAGE_QS + r1 * SLOT);
                // (IQ3_S: its scale d (1 + 2s) has no /8, which the column scales carry)
                const float d0 = half_bits_to_float(prmt(w0, 0u, dsel)) * (FMT == 3 ? 8.0f : 1.0f);
                const float d1 = half_bits_to_float(prmt(w1, 0u, dsel)) * (FMT == 3 ? 8.0f : 1.0f);
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    F[tt][nt][0] = fmaf((float)I[tt][nt][0], d0 * cs[nt].x, F[tt][nt][0]);
                    F[tt][nt][1] = fmaf((float)I[tt][nt][1], d0 * cs[nt].y, F[tt][nt][1]);
                    F[tt][nt][2] = fmaf((float)I[tt][nt][2], d1 * cs[nt].x, F[tt][nt][2]);
                    F[tt][nt][3] = fmaf((float)I[tt][nt][3], d1 * cs[nt].y, F[tt][nt][3]);
                }
            }
        }

        const uint32_t rg = cc.rg, pdone = cc.p;
        const bool rg_done = (cc.blk + 1 == c_nb) || (cc.tb + 1 == tb1);
        ++cc.tb;
        if (++cc.blk == c_nb) {
            cc.blk = 0;
            if (++cc.rg == c_tiles) {
                cc.rg = 0;
                ++cc.p;
            }
            if (cc.tb < tb1) cons_tile();
        }
        __syncwarp();
        issue();  // refill the slot just consumed
        slot = (slot + 1 == NSTAGES) ? 0 : slot + 1;
        if (!rg_done) continue;
        const GemvProblem& P = L.prob[pdone];

        // ---- tile epilogue: reduce limb columns to tokens; write out, or a partial for the
        // ---- tile's first warp to finish after the cluster barrier
        const uint32_t rg_first = (P.tb_begin + rg * P.nb) * 8, rg_end = rg_first + P.nb * 8;
        const bool complete = a <= rg_first && b >= rg_end;
        const uint32_t row0 = rg * ROWS;
        const uint32_t j = a >= rg_first ? 0u : 1u;  // this tile is my first (0) or last (1)
        float* pslot = part + ((size_t)warp * 2 + j) * TOK * ROWS;
        if (complete) wait_go();
#pragma unroll
        for (int tt = 0; tt < T; ++tt) {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const uint32_t r0 = tt * 16 + g, r1 = r0 + 8;
                if (LB == 1 || LB == 16) {
                    // one value per token and column: the lane's four values are four outputs
                    // (tokens nt*8 + 2t and nt*8 + 2t + 1, rows r0 and r1); with the 16-bit split
                    // the high-byte tile nt and the low-byte tile nt + NT/2 add up to them
                    if (LB == 16 && nt >= NT / 2) {
                        F[tt][nt][0] = F[tt][nt][1] = F[tt][nt][2] = F[tt][nt][3] = 0.0f;
                        continue;
                    }
                    constexpr int LO = LB == 16 ? NT / 2 : 0;
                    if (LB == 16) {
#pragma unroll
                        for (int q = 0; q < 4; ++q) F[tt][nt][q] += F[tt][nt + LO][q];
                    }
                    const uint32_t m0 = nt * 8 + 2 * t, m1 = m0 + 1;
                    if (complete) {
                        if (m0 < L.M) {
                            float* o = P.out + (size_t)m0 * P.ldo;
                            if (row0 + r0 < P.N) put(o + row0 + r0, F[tt][nt][0]);
                            if (row0 + r1 < P.N) put(o + row0 + r1, F[tt][nt][2]);
                        }
                        if (m1 < L.M) {
                            float* o = P.out + (size_t)m1 * P.ldo;
                            if (row0 + r0 < P.N) put(o + row0 + r0, F[tt][nt][1]);
                            if (row0 + r1 < P.N) put(o + row0 + r1, F[tt][nt][3]);
                        }
                    } else {
                        pslot[m0 * ROWS + r0] = F[tt][nt][0];
                        pslot[m1 * ROWS + r0] = F[tt][nt][1];
                        pslot[m0 * ROWS + r1] = F[tt][nt][2];
                        pslot[m1 * ROWS + r1] = F[tt][nt][3];
                    }
                    F[tt][nt][0] = F[tt][nt][1] = F[tt][nt][2] = F[tt][nt][3] = 0.0f;
                    continue;
                }
                // four limbs: this lane's columns 2t, 2t+1 are half of a token's (the other half
                // in lane t^1)
                float v0 = F[tt][nt][0] + F[tt][nt][1];
                float v1 = F[tt][nt][2] + F[tt][nt][3];
                v0 += __shfl_xor_sync(0xFFFFFFFFu, v0, 1);
                v1 += __shfl_xor_sync(0xFFFFFFFFu, v1, 1);
                const uint32_t m = nt * 2 + (t >> 1);
                if ((t & 1) == 0) {
                    if (complete) {
                        if (m < L.M) {
                            float* o = P.out + (size_t)m * P.ldo;
                            if (row0 + r0 < P.N) put(o + row0 + r0, v0);
                            if (row0 + r1 < P.N) put(o + row0 + r1, v1);
                        }
                    } else {
                        pslot[m * ROWS + r0] = v0;
                        pslot[m * ROWS + r1] = v1;
                    }
                }
                F[tt][nt][0] = F[tt][nt][1] = F[tt][nt][2] = F[tt][nt][3] = 0.0f;
            }
        }
    }
    cp_async_wait<0>();

    // ---- tiles cut between warps: every partial is in shared memory after the barrier; the
    // ---- tile's first warp adds them in warp order (the other CTA's through DSMEM)
    cluster_sync();
    if (a < b) {
        TbCursor lc;
        cursor_seek(L, p0, tb1 - 1, lc);  // this warp's last tile
        const GemvProblem& P = L.prob[lc.p];
        const uint32_t rg_first = (P.tb_begin + lc.rg * P.nb) * 8, rg_end = rg_first + P.nb * 8;
        if (rg_end > b && rg_first >= a) {
            wait_go();
            const uint32_t w_last = part_.owner(rg_end - 1);
            const uint32_t row0 = lc.rg * ROWS;
            for (uint32_t idx = lane; idx < (uint32_t)ROWS * L.M; idx += 32) {
                const uint32_t m = idx / ROWS, r = idx % ROWS;
                if (row0 + r >= P.N) continue;
                float acc = 0.0f;
#pragma unroll 4
                for (uint32_t ww = wg; ww <= w_last; ++ww) {
                    const uint32_t jj = part_.begin(ww) >= rg_first ? 0u : 1u;
                    const uint32_t off = (((ww % GEMV_WARPS) * 2 + jj) * TOK + m) * ROWS + r;
                    const uint32_t addr = part_s + off * 4;
                    acc += ld_cluster_f32(map_shared(addr, ww / GEMV_WARPS));
                }
                put(P.out + (size_t)m * P.ldo + row0 + r, acc);
            }
        }
    }
    // keep this CTA's partials alive until the other CTA has read them (no data to publish)
    asm volatile("barrier.cluster.arrive.relaxed.aligned;\n\tbarrier.cluster.wait.aligned;" ::: "memory");

    // P2P exit: the last CTA to finish tells every rank that this rank's outputs are stored,
    // waits (bounded) until every rank has said so, then closes the call. The CTAs count in with
    // GPU-scope release; the last one's system-scope fence is cumulative, so one fence orders
    // every CTA's peer stores before the flags.
    if constexpr (P2P) {
        __syncthreads();
        if (threadIdx.x == 0) {
            const GemvPeers& pe = L.peers;
            __threadfence();
            const unsigned prev = atomicAdd(&pe.hdr->done, 1u);
            if (prev == gridDim.x - 1) {
                __threadfence();
                if (!dead && ld_acquire_gpu_u64(&pe.hdr->go) >= epoch) {
                    fence_acq_rel_sys();
                    for (int r = 0; r < pe.world; ++r) st_relaxed_sys_u64(peer_header(pe, r)->data + pe.rank, epoch);
                    bool ok = true;
                    const unsigned long long t0 = gtimer_ns();
                    for (int r = 0; r < pe.world && ok; ++r)
                        while (ld_acquire_sys_u64(pe.hdr->data + r) < epoch) {
                            if (gtimer_ns() - t0 > PEER_WAIT_NS) {
                                ok = false;
                                break;
                            }
                            __nanosleep(64);
                        }
                    if (!ok) atomicOr(&pe.hdr->err, 2u);
                }
                *reinterpret_cast<volatile unsigned*>(&pe.hdr->done) = 0u;
                st_release_gpu_u64(&pe.hdr->epoch, epoch);
            }
        }
    }
}

// ---------------------------------------------------------------------------------------------
// Generic fallback: any alignment, any K, any m (8 tokens per warp pass). One warp per output
// row n; f32 weights and accumulation as in the reference kernel, lanes split the row's
// 8-weight groups and reduce at the end.
template <typename XT>
__global__ void __launch_bounds__(256) gemv_generic_kernel(const XT* __restrict__ x,
                                                           const uint8_t* __restrict__ qs,
                                                           const uint8_t* __restrict__ sc,
                                                           float* __restrict__ out, uint32_t M,
                                                           uint32_t N, uint32_t K, uint32_t nb) {
    __shared__ uint64_t grid_s[256];
    __shared__ uint8_t ksigns_s[128];
    for (int i = threadIdx.x; i < 256; i += blockDim.x) grid_s[i] = IQ2XXS_GRID[i];
    for (int i = threadIdx.x; i < 128; i += blockDim.x) ksigns_s[i] = IQ2_KSIGNS[i];
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const uint32_t mchunks = (M + 7) / 8;
    const size_t total = (size_t)N * mchunks;
    for (size_t wi = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; wi < total;
         wi += (size_t)gridDim.x * blockDim.x / 32) {
        const uint32_t n = (uint32_t)(wi / mchunks), mc = (uint32_t)(wi % mchunks) * 8;
        float acc[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
        const uint32_t ngroups = nb * 32;
        for (uint32_t q = lane; q < ngroups; q += 32) {
            const uint32_t sbk = q >> 2, gi = q & 3, blk = sbk >> 3;
            const uint8_t* pq = qs + ((size_t)n * nb) * QS_BYTES + (size_t)sbk * 8;
            const uint32_t aux_g = ld_u32_le_unaligned(pq), aux_s = ld_u32_le_unaligned(pq + 4);
            const float d = half_bits_to_float(ld_u16_le_unaligned(sc + ((size_t)n * nb + blk) * SC_BYTES));
            const float dl = d * (0.5f + (float)(aux_s >> 28)) * 0.25f;
            const uint64_t gw = grid_s[(aux_g >> (8 * gi)) & 0xFF];
            const uint32_t signs = ksigns_s[(aux_s >> (7 * gi)) & 0x7F];
            const size_t k0 = (size_t)sbk * 32 + gi * 8;
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) {
                const size_t k = k0 + jj;
                if (k >= K) break;
                const float wv = dl * (float)((gw >> (8 * jj)) & 0xFF) * (((signs >> jj) & 1u) ? -1.0f : 1.0f);
#pragma unroll
                for (int mm = 0; mm < 8; ++mm) {
                    if (mc + mm < M) acc[mm] = fmaf(to_f32(x[(size_t)(mc + mm) * K + k]), wv, acc[mm]);
                }
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

// ---------------------------------------------------------------------------------------------
// Host-side planning of a grouped launch: workspace layout and launch parameters.
size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

struct GroupPlan {
    int nt, rows, limbs;
    bool fused;
    uint32_t clusters;
    std::vector<uint32_t> cl_tb;      // clusters + 1 tile-block boundaries (whole tiles)
    std::vector<uint16_t> cl_p;       // problem of each cluster's first tile
    std::vector<uint32_t> tb_begin, tiles, nb;
    size_t total;
    std::vector<uint32_t> x_of;       // problem -> unique x index
    std::vector<const void*> xs;      // unique x pointers
    std::vector<uint32_t> xk;         // their K
    std::vector<size_t> off_xb, off_cs;
    size_t smem;
};

template <int NT, int LB = 4, int FMT = 0>
size_t smem_for(bool fused, uint32_t nb) {
    return GemvShape<NT, LB, FMT>::SMEM + (fused ? xs_bytes(nb, NT) + cs_bytes(nb, NT) : 0);
}

template <int FMT>
size_t smem_for_variant(int nt, int limbs, uint32_t nb) {
    switch (nt) {  // x limbs always from the prep kernel
        case 1: return smem_for<1, 4, FMT>(false, nb);
        case 2: return limbs == 4 ? smem_for<2, 4, FMT>(false, nb) : smem_for<2, 16, FMT>(false, nb);
        case 4: return smem_for<4, 16, FMT>(false, nb);
        default: return smem_for<8, 16, FMT>(false, nb);
    }
}

size_t smem_for_nt(int nt, int limbs, bool fused, uint32_t nb, int fmt = 0) {
    if (fmt == 1) return smem_for_variant<1>(nt, limbs, nb);  // IQ2_XS
    if (fmt == 2) return smem_for_variant<2>(nt, limbs, nb);  // IQ2_S
    if (fmt == 3) return smem_for_variant<3>(nt, limbs, nb);  // IQ3_S
    if (limbs == 1) {
        switch (nt) {
            case 1: return smem_for<1, 1>(fused, nb);
            case 2: return smem_for<2, 1>(fused, nb);
            default: return smem_for<4, 1>(fused, nb);
        }
    }
    if (limbs == 16) {
        switch (nt) {
            case 2: return smem_for<2, 16>(fused, nb);
            case 4: return smem_for<4, 16>(fused, nb);
            default: return smem_for<8, 16>(fused, nb);
        }
    }
    return nt == 1 ? smem_for<1>(fused, nb) : smem_for<2>(fused, nb);  // four limbs: m <= 4
}

// How many 2-CTA clusters of the GEMV (one CTA per SM) the current device runs at once; launching
// more would make the surplus wait for a second wave. Asked once per device.
int max_active_clusters(int num_sms) {
    static int cached[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return num_sms / CLUSTER;
    if (cached[dev] > 0) return cached[dev];
    int n = 0;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = CLUSTER;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(num_sms);
    cfg.blockDim = dim3(GEMV_WARPS * 32);
    cfg.dynamicSmemBytes = SMEM_LIMIT;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaFuncSetAttribute(gemv_kernel<1, 1, -1>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_LIMIT) !=
            cudaSuccess ||
        cudaOccupancyMaxActiveClusters(&n, gemv_kernel<1, 1, -1>, &cfg) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        n = num_sms / CLUSTER;
    }
    if (n > num_sms / CLUSTER) n = num_sms / CLUSTER;
    cached[dev] = n > 0 ? n : 1;
    return cached[dev];
}

// max_cl: clusters the device can run at once (0 when only the workspace size is wanted).
// w8a8: the activations as the W8A8 mode's int8 (one limb, m <= 32).
// fmt: the weight format (0 IQ2_XXS, 1 IQ2_XS, 2 IQ2_S, 3 IQ3_S; only IQ2_XXS makes its x limbs in
// the GEMV).
GroupPlan plan_group(const GemvProblemHost* probs, uint32_t count, uint32_t m, int max_cl, bool w8a8 = false,
                     int fmt = 0) {
    GroupPlan pl;
    pl.nt = w8a8 ? nt_w8a8(m) : nt_for(m);
    pl.rows = w8a8 ? (pl.nt == 1 ? 32 : 16) : rows_for(m);
    pl.limbs = w8a8 ? 1 : limbs_for(m);
    uint64_t tbs = 0, total_tiles = 0;
    for (uint32_t i = 0; i < count; ++i) {
        const uint32_t nb = (probs[i].k + QK - 1) / QK;
        const uint32_t tiles = (probs[i].n + pl.rows - 1) / pl.rows;
        pl.nb.push_back(nb);
        pl.tiles.push_back(tiles);
        pl.tb_begin.push_back((uint32_t)tbs);
        tbs += (uint64_t)tiles * nb;
        total_tiles += tiles;
        uint32_t xi = 0;
        while (xi < pl.xs.size() && !(pl.xs[xi] == probs[i].x && pl.xk[xi] == probs[i].k)) ++xi;
        if (xi == pl.xs.size()) {
            pl.xs.push_back(probs[i].x);
            pl.xk.push_back(probs[i].k);
        }
        pl.x_of.push_back(xi);
    }
    // one projection whose limbs fit in shared memory: the GEMV makes them itself
    pl.fused = fmt == 0 && !w8a8 && count == 1 && pl.nt <= 2 &&
               smem_for_nt(pl.nt, pl.limbs, true, pl.nb[0]) <= (size_t)SMEM_LIMIT;
    pl.smem = smem_for_nt(pl.nt, pl.limbs, pl.fused, count ? pl.nb[0] : 0, fmt);
    // clusters: whole tiles, about equal numbers of tile-blocks each
    uint64_t cl = (uint64_t)(max_cl > 0 ? max_cl : 1);
    if (cl > MAX_CLUSTERS) cl = MAX_CLUSTERS;
    if (cl > total_tiles) cl = total_tiles;
    if (cl < 1) cl = 1;
    pl.cl_tb.push_back(0);
    pl.cl_p.push_back(0);
    {
        uint32_t p = 0, rg = 0;
        uint64_t done = 0;
        for (uint64_t c = 1; c < cl; ++c) {
            const uint64_t target = tbs * c / cl;
            // advance whole tiles while the boundary gets closer to the target
            while (p < count) {
                const uint64_t w = pl.nb[p];
                if (done >= target || (done + w > target && done + w - target > target - done)) break;
                done += w;
                if (++rg == pl.tiles[p]) { rg = 0; ++p; }
            }
            if (done <= pl.cl_tb.back()) continue;  // empty cluster: merge
            pl.cl_tb.push_back((uint32_t)done);
            uint32_t pp = p;
            while (pp < count && pl.tiles[pp] == 0) ++pp;
            pl.cl_p.push_back((uint16_t)(pp < count ? pp : count - 1));
        }
        pl.cl_tb.push_back((uint32_t)tbs);
    }
    pl.clusters = (uint32_t)pl.cl_tb.size() - 1;
    size_t off = 0;
    if (!pl.fused) {
        for (size_t xi = 0; xi < pl.xs.size(); ++xi) {
            const uint32_t nb = (pl.xk[xi] + QK - 1) / QK;
            pl.off_xb.push_back(off);
            off = align_up(off + xs_bytes(nb, pl.nt), 256);
            pl.off_cs.push_back(off);
            off = align_up(off + cs_bytes(nb, pl.nt), 256);
        }
    }
    pl.total = off;
    return pl;
}

template <int NT, int CAP, int XDT, bool P2P, int LB, int FMT = 0>
cudaError_t launch_gemv_kernel(const GemvLaunch<CAP>& L, const GroupPlan& pl, cudaStream_t stream) {
    static bool attr_set[64] = {};  // per device; an idempotent attribute, so a race is benign
    int dev = 0;
    cudaGetDevice(&dev);
    cudaError_t e;
    if (dev >= 64 || !attr_set[dev]) {
        e = cudaFuncSetAttribute(gemv_kernel<NT, CAP, XDT, P2P, LB, FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 SMEM_LIMIT);
        if (e != cudaSuccess) return e;
        if (dev < 64) attr_set[dev] = true;
    }
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = CLUSTER;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(pl.clusters * CLUSTER);
    cfg.blockDim = dim3(GEMV_WARPS * 32);
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, gemv_kernel<NT, CAP, XDT, P2P, LB, FMT>, L);
}

template <int NT, int CAP, int XDT, int LB = 4, int FMT = 0>
cudaError_t launch_gemv_kernel_p(const GemvLaunch<CAP>& L, const GroupPlan& pl, bool p2p, cudaStream_t stream) {
    if constexpr (FMT != 0) {
        (void)p2p;  // (the sharded calls are IQ2_XXS only)
        return launch_gemv_kernel<NT, CAP, XDT, false, LB, FMT>(L, pl, stream);
    } else {
        return p2p ? launch_gemv_kernel<NT, CAP, XDT, true, LB>(L, pl, stream)
                   : launch_gemv_kernel<NT, CAP, XDT, false, LB>(L, pl, stream);
    }
}

template <int NT, int CAP, int LB = 4, int FMT = 0>
cudaError_t launch_group_cap(const GemvProblemHost* probs, uint32_t count, uint32_t m, int x_dtype,
                             uint8_t* ws, const GroupPlan& pl, cudaStream_t stream, const GemvPeers* peers) {
    cudaError_t e;
    if (!pl.fused) {
        // ---- prep launch (unique x's) ----
        PrepLaunch<CAP> pre;
        pre.count = (uint32_t)pl.xs.size();
        pre.M = m;
        uint32_t warps = 0;
        for (uint32_t xi = 0; xi < pre.count; ++xi) {
            PrepItem& it = pre.item[xi];
            it.x = pl.xs[xi];
            it.xb = ws + pl.off_xb[xi];
            it.colscale = reinterpret_cast<float*>(ws + pl.off_cs[xi]);
            it.K = pl.xk[xi];
            it.nb = (pl.xk[xi] + QK - 1) / QK;
            it.warp_begin = warps;
            it.pad = 0;
            warps += (uint32_t)GemvShape<NT, LB>::TOK * it.nb;  // one warp per (token, block)
        }
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((warps * 32 + 255) / 256);
        cfg.blockDim = dim3(256);
        cfg.dynamicSmemBytes = 0;
        cfg.stream = stream;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if constexpr (LB == 1) {
            switch (x_dtype) {
                case 0: e = cudaLaunchKernelEx(&cfg, gemv_prep_w8a8_kernel<float, NT, CAP>, pre); break;
                case 1: e = cudaLaunchKernelEx(&cfg, gemv_prep_w8a8_kernel<__half, NT, CAP>, pre); break;
                default: e = cudaLaunchKernelEx(&cfg, gemv_prep_w8a8_kernel<__nv_bfloat16, NT, CAP>, pre); break;
            }
        } else {
            switch (x_dtype) {
                case 0: e = cudaLaunchKernelEx(&cfg, gemv_prep_kernel<float, NT, CAP, LB>, pre); break;
                case 1: e = cudaLaunchKernelEx(&cfg, gemv_prep_kernel<__half, NT, CAP, LB>, pre); break;
                default: e = cudaLaunchKernelEx(&cfg, gemv_prep_kernel<__nv_bfloat16, NT, CAP, LB>, pre); break;
            }
        }
        if (e != cudaSuccess) return e;
    }

    // ---- GEMV launch ----
    GemvLaunch<CAP> L;
    memset(&L, 0, sizeof(L));
    L.count = count;
    L.M = m;
    L.x = probs[0].x;
    L.K = probs[0].k;
    L.clusters = pl.clusters;
    L.two = 2u;
    for (uint32_t c = 0; c <= pl.clusters; ++c) L.cl_tb[c] = pl.cl_tb[c];
    for (uint32_t c = 0; c < pl.clusters; ++c) L.cl_p[c] = pl.cl_p[c];
    for (uint32_t i = 0; i < count; ++i) {
        GemvProblem& P = L.prob[i];
        P.qs = probs[i].qs;
        P.sc = probs[i].sc;
        P.xb = pl.fused ? nullptr : ws + pl.off_xb[pl.x_of[i]];
        P.colscale = pl.fused ? nullptr : reinterpret_cast<const float*>(ws + pl.off_cs[pl.x_of[i]]);
        P.out = probs[i].out;
        P.N = probs[i].n;
        P.nb = pl.nb[i];
        P.tiles = pl.tiles[i];
        P.tb_begin = pl.tb_begin[i];
        P.ldo = probs[i].ldo ? probs[i].ldo : probs[i].n;
    }
    const bool p2p = peers != nullptr;
    if (p2p) L.peers = *peers;
    if (!pl.fused) e = launch_gemv_kernel_p<NT, CAP, -1, LB, FMT>(L, pl, p2p, stream);
    else if constexpr (FMT == 0 && NT <= 2 && CAP == 1 && (LB == 4 || LB == 16)) {
        switch (x_dtype) {
            case 0: e = launch_gemv_kernel_p<NT, CAP, 0, LB>(L, pl, p2p, stream); break;
            case 1: e = launch_gemv_kernel_p<NT, CAP, 1, LB>(L, pl, p2p, stream); break;
            default: e = launch_gemv_kernel_p<NT, CAP, 2, LB>(L, pl, p2p, stream); break;
        }
    } else {
        e = cudaErrorInvalidValue;  // the planner never fuses these
    }
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

template <int NT>
cudaError_t launch_group_nt(const GemvProblemHost* probs, uint32_t count, uint32_t m, int x_dtype,
                            uint8_t* ws, const GroupPlan& pl, cudaStream_t stream, const GemvPeers* peers) {
    // four limbs for one n8 tile (m <= 2), the 16-bit split for more; parameter capacity: a single
    // projection ships ~1 KB of launch parameters, not 16 KB
    if constexpr (NT <= 2) {
        if (pl.limbs == 4) {  // m <= 4
            if (count <= 1) return launch_group_cap<NT, 1, 4>(probs, count, m, x_dtype, ws, pl, stream, peers);
            if (count <= 16) return launch_group_cap<NT, 16, 4>(probs, count, m, x_dtype, ws, pl, stream, peers);
            return launch_group_cap<NT, MAX_PROBLEMS, 4>(probs, count, m, x_dtype, ws, pl, stream, peers);
        }
    }
    if constexpr (NT >= 2) {
        if (count <= 1) return launch_group_cap<NT, 1, 16>(probs, count, m, x_dtype, ws, pl, stream, peers);
        if (count <= 16) return launch_group_cap<NT, 16, 16>(probs, count, m, x_dtype, ws, pl, stream, peers);
        return launch_group_cap<NT, MAX_PROBLEMS, 16>(probs, count, m, x_dtype, ws, pl, stream, peers);
    }
    return cudaErrorInvalidValue;  // (NT = 1 always has four limbs)
}

}  // namespace

bool gemv_fast_path_ok(uint32_t m, uint32_t k, const uint8_t* qs, const uint8_t* sc) {
    return m >= 1 && m <= kGemvMaxM && k >= 1 && (reinterpret_cast<uintptr_t>(qs) % 16) == 0 &&
           (reinterpret_cast<uintptr_t>(sc) % 4) == 0;
}

uint32_t gemv_max_group() { return MAX_PROBLEMS; }

size_t gemv_group_workspace_size(const GemvProblemHost* probs, uint32_t count, uint32_t m, int num_sms) {
    (void)num_sms;
    if (count == 0) return 0;
    return plan_group(probs, count, m, 0).total;
}

size_t gemv_workspace_size(uint32_t m, uint32_t n, uint32_t k, int num_sms) {
    GemvProblemHost p{nullptr, nullptr, nullptr, n, k, nullptr};
    return gemv_group_workspace_size(&p, 1, m, num_sms);
}

cudaError_t launch_gemv_group(const GemvProblemHost* probs, uint32_t count, uint32_t m, int x_dtype,
                              void* workspace, int num_sms, cudaStream_t stream, const GemvPeers* peers) {
    if (count == 0) return cudaSuccess;
    const GroupPlan pl = plan_group(probs, count, m, max_active_clusters(num_sms));
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    switch (pl.nt) {
        case 1: return launch_group_nt<1>(probs, count, m, x_dtype, ws, pl, stream, peers);
        case 2: return launch_group_nt<2>(probs, count, m, x_dtype, ws, pl, stream, peers);
        case 4: return launch_group_nt<4>(probs, count, m, x_dtype, ws, pl, stream, peers);
        default: return launch_group_nt<8>(probs, count, m, x_dtype, ws, pl, stream, peers);
    }
}

size_t gemv_w8a8_workspace_size(uint32_t m, uint32_t n, uint32_t k) {
    GemvProblemHost p{nullptr, nullptr, nullptr, n, k, nullptr};
    return plan_group(&p, 1, m, 0, true).total;
}

cudaError_t launch_gemv_w8a8(const void* x, int x_dtype, uint32_t m, const uint8_t* qs, const uint8_t* sc,
                             uint32_t n, uint32_t k, float* out, void* workspace, int num_sms, cudaStream_t stream) {
    GemvProblemHost p{x, qs, sc, n, k, out};
    const GroupPlan pl = plan_group(&p, 1, m, max_active_clusters(num_sms), true);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    switch (pl.nt) {
        case 1: return launch_group_cap<1, 1, 1>(&p, 1, m, x_dtype, ws, pl, stream, nullptr);
        case 2: return launch_group_cap<2, 1, 1>(&p, 1, m, x_dtype, ws, pl, stream, nullptr);
        default: return launch_group_cap<4, 1, 1>(&p, 1, m, x_dtype, ws, pl, stream, nullptr);
    }
}

cudaError_t launch_gemv(const void* x, int x_dtype, uint32_t m, const uint8_t* qs, const uint8_t* sc,
                        uint32_t n, uint32_t k, float* out, void* workspace, int num_sms,
                        cudaStream_t stream) {
    GemvProblemHost p{x, qs, sc, n, k, out};
    return launch_gemv_group(&p, 1, m, x_dtype, workspace, num_sms, stream);
}

bool gemv_variant_ok(int variant) { return variant >= 1 && variant <= 3; }

size_t gemv_variant_workspace_size(int variant, uint32_t m, uint32_t n, uint32_t k) {
    if (!gemv_variant_ok(variant)) return 0;
    GemvProblemHost p{nullptr, nullptr, nullptr, n, k, nullptr};
    return plan_group(&p, 1, m, 0, false, variant).total;
}

namespace {
template <int FMT>
cudaError_t launch_gemv_fmt(const GemvProblemHost& p, uint32_t m, int x_dtype, uint8_t* ws, const GroupPlan& pl,
                            cudaStream_t stream) {
    switch (pl.nt) {
        case 1: return launch_group_cap<1, 1, 4, FMT>(&p, 1, m, x_dtype, ws, pl, stream, nullptr);
        case 2:
            return pl.limbs == 4 ? launch_group_cap<2, 1, 4, FMT>(&p, 1, m, x_dtype, ws, pl, stream, nullptr)
                                 : launch_group_cap<2, 1, 16, FMT>(&p, 1, m, x_dtype, ws, pl, stream, nullptr);
        case 4: return launch_group_cap<4, 1, 16, FMT>(&p, 1, m, x_dtype, ws, pl, stream, nullptr);
        default: return launch_group_cap<8, 1, 16, FMT>(&p, 1, m, x_dtype, ws, pl, stream, nullptr);
    }
}
}  // namespace

cudaError_t launch_gemv_variant(int variant, const void* x, int x_dtype, uint32_t m, const uint8_t* qs,
                                const uint8_t* sc, uint32_t n, uint32_t k, float* out, void* workspace, int num_sms,
                                cudaStream_t stream) {
    if (!gemv_variant_ok(variant)) return cudaErrorInvalidValue;
    GemvProblemHost p{x, qs, sc, n, k, out};
    const GroupPlan pl = plan_group(&p, 1, m, max_active_clusters(num_sms), false, variant);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    switch (variant) {
        case 1: return launch_gemv_fmt<1>(p, m, x_dtype, ws, pl, stream);
        case 2: return launch_gemv_fmt<2>(p, m, x_dtype, ws, pl, stream);
        default: return launch_gemv_fmt<3>(p, m, x_dtype, ws, pl, stream);
    }
}

cudaError_t launch_gemv_generic(const void* x, int x_dtype, uint32_t m, const uint8_t* qs,
                                const uint8_t* sc, uint32_t n, uint32_t k, float* out,
                                int num_sms, cudaStream_t stream) {
    const uint32_t nb = (k + QK - 1) / QK;
    const size_t warps = (size_t)n * ((m + 7) / 8);
    size_t blocks = (warps + 7) / 8;
    const size_t cap = (size_t)num_sms * 8;
    if (blocks > cap) blocks = cap;
    switch (x_dtype) {
        case 0: gemv_generic_kernel<float><<<(unsigned)blocks, 256, 0, stream>>>(
                    static_cast<const float*>(x), qs, sc, out, m, n, k, nb); break;
        case 1: gemv_generic_kernel<__half><<<(unsigned)blocks, 256, 0, stream>>>(
                    static_cast<const __half*>(x), qs, sc, out, m, n, k, nb); break;
        default: gemv_generic_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, stream>>>(
                    static_cast<const __nv_bfloat16*>(x), qs, sc, out, m, n, k, nb); break;
    }
    return cudaGetLastError();
}

}  // namespace iq2
