// IQ2_XXS decode GEMV for small m (m <= 16) on sm_100a, single or grouped projections.
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
//     tables, so a warp's random lookups never share a bank) into four signed int8 weights.
//   * x is split per (token, 256-block) into four 7-bit signed limbs of a 28-bit fixed-point
//     value (gemv_prep_kernel): x @ W^T becomes mma.m16n8k32 s8 x s8 -> s32 per 32-weight
//     sub-block, scaled by the odd integer 2s+1 in s32 (exact, |sum| < 2^31) and turned into f32
//     once per 256-block with d and the limb scale. The only rounding is the 2^-28-relative
//     quantisation of x and f32 rounding of per-block partial sums (rel. error ~1e-6).
//   * Weights stream through a per-warp cp.async ring in shared memory (one 256-weight block of
//     ROWS rows per stage, ~140 KB in flight per SM), 16-byte chunks XOR-swizzled so the rows a
//     warp reads together sit in different banks; one 16-byte read feeds two sub-blocks.
//   * Stream-K: the (projection, row group, sub-block) steps of a launch are split into equal
//     contiguous ranges, one per warp, so every warp finishes at the same time whatever the
//     shapes. A row group cut by a range boundary is finished by the last of its (at most a few)
//     warps, which sums the others' partials in warp order: results are deterministic.
//   * Grouped launches: one prep launch and one GEMV launch serve up to 256 projections (e.g.
//     q/k/v or gate/up sharing x), amortising launch and table-fill costs; projections that share
//     an x share its limbs. Both kernels use programmatic dependent launch: the GEMV fills its
//     tables and starts streaming weights while the prep runs.
#include "iq2xxs_common.cuh"
#include "iq2xxs_codebook.h"
#include "iq2xxs_internal.h"

#include <vector>

namespace iq2 {

namespace {

constexpr int GEMV_WARPS = 16;
constexpr int LUT_BYTES = 256 * 256;  // 256 rows x (32 lanes grid selectors | 32 lanes sign)
constexpr int MAX_PROBLEMS = 256;     // per grouped launch

template <int NT>
struct GemvShape {
    static constexpr int T = NT <= 2 ? 2 : 1;          // 16-row mma tiles per warp
    static constexpr int ROWS = 16 * T;                // rows of a row group
    static constexpr int STAGE_QS = ROWS * 64;         // one block of qs per row
    static constexpr int STAGE_BYTES = STAGE_QS + ROWS * 4;  // + the aligned scale word per row
    static constexpr int NSTAGES = T == 2 ? 4 : 8;
    static constexpr int RING_BYTES = NSTAGES * STAGE_BYTES;  // per warp
    // The table sits at the first 64 KB-aligned shared address of the block's window and the
    // warps' rings fill the space around it; whatever the window's base, this suffices:
    static constexpr int SMEM = LUT_BYTES + (GEMV_WARPS + 1) * RING_BYTES;
};

int nt_for(uint32_t m) { return m <= 2 ? 1 : (m <= 4 ? 2 : (m <= 8 ? 4 : 8)); }
int rows_for(uint32_t m) { return nt_for(m) <= 2 ? 32 : 16; }

// ---------------------------------------------------------------------------------------------
// x -> int8 limb fragments. One warp per (x item, token m, block b); lane = (sub-block sbi,
// group t) owns the 8 activations k = b*256 + sbi*32 + t*8 + [0, 8).
// With amax = max |x| over the block and amax = f * 2^E (f in [0.5, 1)):
//   q = rint(x * 2^(27-E)) (|q| <= 2^27), |q| = L3*2^21 + L2*2^14 + L1*2^7 + L0 (7-bit limbs),
//   each limb carrying the sign of q; column scale of limb l = 2^(E - 27 + 7l) / 8 (the /8 is
//   the weight scale's (2s+1)/8). Non-finite blocks get NaN scales, so the output is NaN.
// Fragment layout (mma B operand, m16n8k32 "col"), sub-block sb, n8 tile nt:
//   xb[((sb*NT + nt)*32 + col*4 + t)*8 + i] = limb of group t, element i; col = (m%2)*4 + l.
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
    uint32_t* counters;
    uint32_t ncounters;
};

template <typename XT, int NT, int CAP>
__global__ void __launch_bounds__(256) gemv_prep_kernel(const __grid_constant__ PrepLaunch<CAP> L) {
    // x may be written by the previous kernel and the workspace may still be read by the
    // previous GEMV: wait for both before touching memory. Only then let the GEMV launch, so
    // its early weight prefetch also runs after every earlier kernel has finished.
    pdl_wait();
    pdl_launch_dependents();
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < L.ncounters; i += gridDim.x * blockDim.x)
        L.counters[i] = 0u;
    const uint32_t wid = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    uint32_t it = 0;
    while (it + 1 < L.count && L.item[it + 1].warp_begin <= wid) ++it;
    const PrepItem& P = L.item[it];
    const uint32_t local = wid - P.warp_begin;
    if (local >= L.M * P.nb) return;
    const uint32_t m = local / P.nb, b = local % P.nb;
    const int sbi = lane >> 2, t = lane & 3;
    const size_t k0 = (size_t)b * QK + sbi * 32 + t * 8;
    const XT* xr = static_cast<const XT*>(P.x) + (size_t)m * P.K;

    float v[8];
    float amax = 0.0f;
    bool bad = false;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const size_t k = k0 + i;
        v[i] = k < P.K ? to_f32(xr[k]) : 0.0f;
        bad |= !isfinite(v[i]);
        amax = fmaxf(amax, fabsf(v[i]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
    bad = __any_sync(0xFFFFFFFFu, bad);

    int E = 0;
    if (!bad && amax > 0.0f) frexpf(amax, &E);
    uint32_t lo[4] = {0, 0, 0, 0}, hi[4] = {0, 0, 0, 0};
    if (!bad && amax > 0.0f) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int q = (int)rintf(ldexpf(v[i], 27 - E));
            const uint32_t mag = (uint32_t)(q < 0 ? -q : q);
#pragma unroll
            for (int l = 0; l < 4; ++l) {
                const int limb = (l < 3) ? (int)((mag >> (7 * l)) & 127u) : (int)(mag >> 21);
                const uint32_t byte = (uint32_t)(uint8_t)(int8_t)(q < 0 ? -limb : limb);
                if (i < 4) lo[l] |= byte << (8 * i);
                else hi[l] |= byte << (8 * (i - 4));
            }
        }
    }
    const uint32_t nt = m >> 1, colbase = (m & 1u) * 4u;
    const size_t sb = (size_t)b * 8 + sbi;
#pragma unroll
    for (int l = 0; l < 4; ++l) {
        uint2* dst = reinterpret_cast<uint2*>(P.xb + ((sb * NT + nt) * 32 + (colbase + l) * 4 + t) * 8);
        *dst = make_uint2(lo[l], hi[l]);
    }
    if (lane < 4) {
        float s;
        if (bad) s = __int_as_float(0x7FC00000);
        else if (amax == 0.0f) s = 0.0f;
        else s = ldexpf(1.0f, E - 30 + 7 * lane);
        P.colscale[(size_t)b * (NT * 8) + nt * 8 + colbase + lane] = s;
    }
}

// ---------------------------------------------------------------------------------------------
struct GemvProblem {  // 64 bytes
    const uint8_t* qs;
    const uint8_t* sc;
    const uint8_t* xb;
    const float* colscale;
    float* out;
    uint32_t N, nb, row_groups, tb_begin;  // tb_begin: first tile-block (ROWS rows x 1 block)
    uint32_t counter_base, pad;
};

template <int CAP>
struct GemvLaunch {
    GemvProblem prob[CAP];
    uint32_t count, M;
    uint32_t total_steps;  // 8 sub-block steps per tile-block
    uint32_t pad;
    float* partial;        // [warps][2][ROWS * M]
    uint32_t* counters;
};

// Stream-K partition of [0, total) over W warps: the first r warps get q+1 steps, the rest q.
struct Partition {
    uint32_t q, r;
    __device__ __forceinline__ uint32_t begin(uint32_t w) const { return w * q + min(w, r); }
    __device__ __forceinline__ uint32_t owner(uint32_t s) const {
        const uint32_t big = r * (q + 1);
        return s < big ? s / (q + 1) : r + (s - big) / q;
    }
};

// Cursor over the tile-blocks (problem p, row group rg, block blk) of a launch, in order.
struct TbCursor {
    uint32_t tb, p, rg, blk;
};

template <int CAP>
__device__ __forceinline__ void cursor_seek(const GemvLaunch<CAP>& L, uint32_t tb, TbCursor& c) {
    uint32_t p = 0;
    while (p + 1 < L.count && L.prob[p + 1].tb_begin <= tb) ++p;
    const uint32_t local = tb - L.prob[p].tb_begin;
    c.tb = tb;
    c.p = p;
    c.rg = local / L.prob[p].nb;
    c.blk = local % L.prob[p].nb;
}

template <int CAP>
__device__ __forceinline__ void cursor_next(const GemvLaunch<CAP>& L, TbCursor& c) {
    ++c.tb;
    if (++c.blk == L.prob[c.p].nb) {
        c.blk = 0;
        if (++c.rg == L.prob[c.p].row_groups) {
            c.rg = 0;
            ++c.p;
        }
    }
}

// Per-lane decode constants. The table base is 64 KB-aligned, so every table address is
// assembled by one byte permute (grid: base | idx<<8 | lane*4) or one LOP3 (sign: base | 128 |
// sidx<<8 | lane*4), with no add.
struct DecodeK {
    uint32_t gsrc;  // bytes {lane*4, 0, base.b2, base.b3}
    uint32_t gsel;  // prmt selector {gsrc.b0, aux_g.byte t, gsrc.b2, gsrc.b3}
    uint32_t rot;   // rotate that brings sign index t (bits 7t..7t+6) to bits 8..14
    uint32_t soff;  // base | 128 | lane*4
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

// One stage (a block of ROWS rows) of the decode: accumulate s32 sums per 256-block in I.
// PARTIAL: only sub-blocks [s_lo, s_hi) count (the first/last stage of a warp's range).
template <int NT, bool PARTIAL>
__device__ __forceinline__ void stage_compute(const DecodeK& dk, uint32_t st_s, const uint8_t* xbp,
                                              const bool (&bact)[NT], uint32_t s_lo, uint32_t s_hi,
                                              uint32_t rowbase, uint32_t swz,
                                              int (&I)[GemvShape<NT>::T][NT][4]) {
    constexpr int T = GemvShape<NT>::T;
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
                bool on = bact[nt];
                if (PARTIAL) on = on && sb >= s_lo && sb < s_hi;  // other sub-blocks add 0
                uint2 v = make_uint2(0u, 0u);
                if (on) v = __ldg(reinterpret_cast<const uint2*>(xbp + (sb * NT + nt) * 256));
                bf[nt][0] = v.x;
                bf[nt][1] = v.y;
            }
#pragma unroll
            for (int tt = 0; tt < T; ++tt) {
                const uint32_t g0 = h ? qw[tt][0].z : qw[tt][0].x, s0 = h ? qw[tt][0].w : qw[tt][0].y;
                const uint32_t g1 = h ? qw[tt][1].z : qw[tt][1].x, s1 = h ? qw[tt][1].w : qw[tt][1].y;
                uint32_t w0, w1, w2, w3;
                decode_group(dk, g0, s0, w0, w2);
                decode_group(dk, g1, s1, w1, w3);
                const int c0 = (int)((s0 >> 27) | 1u), c1 = (int)((s1 >> 27) | 1u);
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    int d[4];
                    mma_s8_16832(d, w0, w1, w2, w3, bf[nt][0], bf[nt][1]);
                    I[tt][nt][0] += c0 * d[0];
                    I[tt][nt][1] += c0 * d[1];
                    I[tt][nt][2] += c1 * d[2];
                    I[tt][nt][3] += c1 * d[3];
                }
            }
        }
    }
}

template <int NT, int CAP>
__global__ void __launch_bounds__(GEMV_WARPS * 32, 1) gemv_kernel(const __grid_constant__ GemvLaunch<CAP> L) {
    using S_ = GemvShape<NT>;
    constexpr int T = S_::T, ROWS = S_::ROWS, STAGE_QS = S_::STAGE_QS;
    constexpr int STAGE_BYTES = S_::STAGE_BYTES, NSTAGES = S_::NSTAGES, RING_BYTES = S_::RING_BYTES;
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;

    // ---- shared layout: table at the first 64 KB-aligned address, rings around it ----
    const uint32_t base_s = smem_u32(smem);
    const uint32_t lut_s = (base_s + 0xFFFFu) & ~0xFFFFu;
    const uint32_t gap = lut_s - base_s;
    const uint32_t gap_warps = gap / RING_BYTES;
    const uint32_t ring_off = (uint32_t)warp < gap_warps
                                  ? (uint32_t)warp * RING_BYTES
                                  : gap + LUT_BYTES + ((uint32_t)warp - gap_warps) * RING_BYTES;
    uint8_t* ring = smem + ring_off;
    const uint32_t ring_s = base_s + ring_off;

    // This warp's step range [a, b) and the tile-blocks it touches [tb0, tb1).
    const uint32_t W = gridDim.x * GEMV_WARPS;
    const uint32_t w = blockIdx.x * GEMV_WARPS + warp;
    const Partition part{L.total_steps / W, L.total_steps % W};
    const uint32_t a = part.begin(w), b = part.begin(w + 1);
    const uint32_t tb0 = a >> 3, tb1 = (b + 7) >> 3;

    // ---- the decode table: 64 KB image from global memory (one cp.async group) ----
    {
        const uint8_t* src = reinterpret_cast<const uint8_t*>(&IQ2XXS_LUT_IMAGE);
        for (int i = threadIdx.x; i < LUT_BYTES / 16; i += blockDim.x)
            cp_async_16(lut_s + i * 16, src + i * 16, 16u);
        cp_async_commit();
    }

    // ---- issue side: cp.async stages of one tile-block each, NSTAGES ahead ----
    TbCursor ic;
    if (a < b) cursor_seek(L, tb0, ic);
    int islot = 0;
    auto issue = [&]() {
        if (a < b && ic.tb < tb1) {
            const GemvProblem& P = L.prob[ic.p];
            const uint32_t st_s = ring_s + islot * STAGE_BYTES;
            const uint32_t s_lo = ic.tb * 8 < a ? a - ic.tb * 8 : 0u;        // first sub-block needed
            const uint32_t s_hi = min(8u, b - ic.tb * 8);                     // one past the last
            const uint32_t ch_lo = s_lo >> 1, ch_hi = (s_hi + 1) >> 1;        // 16-byte chunks needed
            const uint32_t row0 = ic.rg * ROWS;
            const uint8_t* qrow = P.qs + ((size_t)row0 * P.nb + ic.blk) * QS_BYTES;
            const size_t row_bytes = (size_t)P.nb * QS_BYTES;
#pragma unroll
            for (int c = 0; c < ROWS * 4 / 32; ++c) {
                const int idx = c * 32 + lane;
                const int r = idx >> 2, ch = idx & 3;
                const bool ok = row0 + r < P.N && (uint32_t)ch >= ch_lo && (uint32_t)ch < ch_hi;
                const uint8_t* src = ok ? qrow + (size_t)r * row_bytes + ch * 16 : P.qs;
                // swizzle: chunk ch of row r goes to chunk ch ^ ((r >> 1) & 3)
                cp_async_16(st_s + r * 64 + ((ch ^ ((r >> 1) & 3)) << 4), src, ok ? 16u : 0u);
            }
            if (lane < ROWS) {
                // the 4-byte aligned word holding this row's d; near the end of the buffer only
                // the bytes that exist are read (the rest of the word is zero-filled)
                const uint32_t row = row0 + lane;
                const bool ok = row < P.N;
                const size_t e = ((size_t)row * P.nb + ic.blk) * SC_BYTES;
                const size_t ea = e & ~(size_t)3, total = (size_t)P.N * P.nb * SC_BYTES;
                const uint32_t nbytes = ok ? (uint32_t)min((size_t)4, total - ea) : 0u;
                cp_async_4(st_s + STAGE_QS + lane * 4, P.sc + (ok ? ea : 0), nbytes);
            }
            cursor_next(L, ic);
        }
        cp_async_commit();
        islot = (islot + 1 == NSTAGES) ? 0 : islot + 1;
    };

    // The first stages only read weights: start them before waiting for anything.
#pragma unroll
    for (int i = 0; i < NSTAGES; ++i) issue();
    cp_async_wait<NSTAGES>();  // the table group (issued first) has landed
    __syncthreads();
    // x fragments, column scales, counters and outputs are produced by / shared with the prep
    // kernel: wait for it here.
    pdl_wait();
    if (a >= b) {
        cp_async_wait<0>();
        pdl_launch_dependents();
        return;
    }

    DecodeK dk;
    dk.gsrc = (lut_s & 0xFFFF0000u) | ((uint32_t)lane * 4u);
    dk.gsel = 0x7604u | ((uint32_t)t << 4);
    dk.rot = (7u * t + 24u) & 31u;
    dk.soff = lut_s | 128u | ((uint32_t)lane * 4u);
    const uint32_t swz = (uint32_t)((g >> 1) & 3);  // rows g, g+8, g+16, g+24 share it
    const uint32_t rowbase = (uint32_t)g * 64u;     // rows tt*16+g (+8): rowbase + tt*1024 (+512)

    bool bact[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) bact[nt] = (uint32_t)(nt * 2 + (g >> 2)) < L.M;

    float F[T][NT][4];
#pragma unroll
    for (int i = 0; i < T; ++i)
#pragma unroll
        for (int j = 0; j < NT; ++j)
#pragma unroll
            for (int k = 0; k < 4; ++k) F[i][j][k] = 0.0f;

    TbCursor cc;
    cursor_seek(L, tb0, cc);
    int slot = 0;
    for (; cc.tb < tb1;) {
        const GemvProblem& P = L.prob[cc.p];
        cp_async_wait<NSTAGES - 1>();
        __syncwarp();
        const uint32_t st_s = ring_s + slot * STAGE_BYTES;
        const uint8_t* st = ring + slot * STAGE_BYTES;
        const uint32_t s_lo = cc.tb * 8 < a ? a - cc.tb * 8 : 0u;
        const uint32_t s_hi = min(8u, b - cc.tb * 8);

        int I[T][NT][4];
#pragma unroll
        for (int i = 0; i < T; ++i)
#pragma unroll
            for (int j = 0; j < NT; ++j)
#pragma unroll
                for (int k = 0; k < 4; ++k) I[i][j][k] = 0;

        const uint8_t* xbp = P.xb + (size_t)cc.blk * 8 * NT * 256 + lane * 8;
        if (s_lo == 0 && s_hi == 8)
            stage_compute<NT, false>(dk, st_s, xbp, bact, s_lo, s_hi, rowbase, swz, I);
        else
            stage_compute<NT, true>(dk, st_s, xbp, bact, s_lo, s_hi, rowbase, swz, I);

        // Block epilogue: s32 -> f32 with d (per row) and the limb scale (per column).
        {
            float2 cs[NT];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
                cs[nt] = __ldg(reinterpret_cast<const float2*>(P.colscale + (size_t)cc.blk * (NT * 8) + nt * 8 + 2 * t));
            const uint32_t row0 = cc.rg * ROWS;
#pragma unroll
            for (int tt = 0; tt < T; ++tt) {
                const uint32_t r0 = tt * 16 + g, r1 = r0 + 8;
                const uint32_t w0 = ld_shared_u32_volatile(st_s + STAGE_QS + r0 * 4);
                const uint32_t w1 = ld_shared_u32_volatile(st_s + STAGE_QS + r1 * 4);
                const uint32_t o0 = ((row0 + r0) * P.nb + cc.blk) & 1u, o1 = ((row0 + r1) * P.nb + cc.blk) & 1u;
                const float d0 = half_bits_to_float(o0 ? (w0 >> 16) : w0);
                const float d1 = half_bits_to_float(o1 ? (w1 >> 16) : w1);
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    F[tt][nt][0] = fmaf((float)I[tt][nt][0], d0 * cs[nt].x, F[tt][nt][0]);
                    F[tt][nt][1] = fmaf((float)I[tt][nt][1], d0 * cs[nt].y, F[tt][nt][1]);
                    F[tt][nt][2] = fmaf((float)I[tt][nt][2], d1 * cs[nt].x, F[tt][nt][2]);
                    F[tt][nt][3] = fmaf((float)I[tt][nt][3], d1 * cs[nt].y, F[tt][nt][3]);
                }
            }
        }
        (void)st;

        const uint32_t rg = cc.rg;
        const bool rg_done = (cc.blk + 1 == P.nb) || (cc.tb + 1 == tb1);
        cursor_next(L, cc);
        __syncwarp();
        issue();  // refill the slot just consumed
        slot = (slot + 1 == NSTAGES) ? 0 : slot + 1;
        if (!rg_done) continue;

        // ---- row group epilogue: reduce limb columns to tokens; write out or a partial ----
        const uint32_t rg_first = (P.tb_begin + rg * P.nb) * 8, rg_end = rg_first + P.nb * 8;
        const bool complete = a <= rg_first && b >= rg_end;
        const uint32_t row0 = rg * ROWS;
        const uint32_t j = a >= rg_first ? 0u : 1u;  // this row group is my first (0) or last (1)
        float* pslot = L.partial + ((size_t)w * 2 + j) * ROWS * L.M;
#pragma unroll
        for (int tt = 0; tt < T; ++tt) {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                float v0 = F[tt][nt][0] + F[tt][nt][1];
                float v1 = F[tt][nt][2] + F[tt][nt][3];
                v0 += __shfl_xor_sync(0xFFFFFFFFu, v0, 1);
                v1 += __shfl_xor_sync(0xFFFFFFFFu, v1, 1);
                const uint32_t m = nt * 2 + (t >> 1);
                const uint32_t r0 = tt * 16 + g, r1 = r0 + 8;
                if ((t & 1) == 0 && m < L.M) {
                    if (complete) {
                        float* o = P.out + (size_t)m * P.N;
                        if (row0 + r0 < P.N) o[row0 + r0] = v0;
                        if (row0 + r1 < P.N) o[row0 + r1] = v1;
                    } else {
                        pslot[m * ROWS + r0] = v0;
                        pslot[m * ROWS + r1] = v1;
                    }
                }
                F[tt][nt][0] = F[tt][nt][1] = F[tt][nt][2] = F[tt][nt][3] = 0.0f;
            }
        }
        if (!complete) {
            const uint32_t w_first = part.owner(rg_first), w_last = part.owner(rg_end - 1);
            const uint32_t count = w_last - w_first + 1;
            __threadfence();
            __syncwarp();
            uint32_t prev = 0;
            if (lane == 0) prev = atomicAdd(L.counters + P.counter_base + rg, 1u);
            prev = __shfl_sync(0xFFFFFFFFu, prev, 0);
            if (prev == count - 1) {
                __threadfence();
                for (uint32_t idx = lane; idx < (uint32_t)ROWS * L.M; idx += 32) {
                    const uint32_t m = idx / ROWS, r = idx % ROWS;
                    if (row0 + r >= P.N) continue;
                    float acc = 0.0f;
                    for (uint32_t ww = w_first; ww <= w_last; ++ww) {
                        const uint32_t jj = part.begin(ww) >= rg_first ? 0u : 1u;
                        acc += __ldcg(L.partial + ((size_t)ww * 2 + jj) * ROWS * L.M + m * ROWS + r);
                    }
                    P.out[(size_t)m * P.N + row0 + r] = acc;
                }
                if (lane == 0) L.counters[P.counter_base + rg] = 0u;
            }
        }
    }
    cp_async_wait<0>();
    pdl_launch_dependents();
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
    int nt, rows;
    uint32_t warps;          // W = grid * GEMV_WARPS
    uint32_t grid;
    uint32_t total_steps;
    size_t off_counters, off_partial, off_x, total;
    std::vector<uint32_t> x_of;       // problem -> unique x index
    std::vector<const void*> xs;      // unique x pointers
    std::vector<uint32_t> xk;         // their K
    std::vector<size_t> off_xb, off_cs;
    std::vector<uint32_t> counter_base;
};

GroupPlan plan_group(const GemvProblemHost* probs, uint32_t count, uint32_t m, int num_sms) {
    GroupPlan pl;
    pl.nt = nt_for(m);
    pl.rows = rows_for(m);
    uint64_t steps = 0;
    uint32_t counters = 0;
    pl.counter_base.resize(count);
    for (uint32_t i = 0; i < count; ++i) {
        const uint32_t nb = (probs[i].k + QK - 1) / QK;
        const uint32_t rgs = (probs[i].n + pl.rows - 1) / pl.rows;
        pl.counter_base[i] = counters;
        counters += rgs;
        steps += (uint64_t)rgs * nb * 8;
        uint32_t xi = 0;
        while (xi < pl.xs.size() && !(pl.xs[xi] == probs[i].x && pl.xk[xi] == probs[i].k)) ++xi;
        if (xi == pl.xs.size()) {
            pl.xs.push_back(probs[i].x);
            pl.xk.push_back(probs[i].k);
        }
        pl.x_of.push_back(xi);
    }
    pl.total_steps = (uint32_t)steps;
    // at least ~16 steps per warp, at most one CTA per SM
    uint64_t ctas = (steps + (uint64_t)GEMV_WARPS * 16 - 1) / ((uint64_t)GEMV_WARPS * 16);
    if (ctas < 1) ctas = 1;
    if (ctas > (uint64_t)num_sms) ctas = num_sms;
    pl.grid = (uint32_t)ctas;
    pl.warps = pl.grid * GEMV_WARPS;
    size_t off = 0;
    pl.off_counters = off;
    off = align_up(off + (size_t)counters * sizeof(uint32_t), 256);
    pl.off_partial = off;
    off = align_up(off + (size_t)pl.warps * 2 * pl.rows * m * sizeof(float), 256);
    pl.off_x = off;
    for (size_t xi = 0; xi < pl.xs.size(); ++xi) {
        const uint32_t nb = (pl.xk[xi] + QK - 1) / QK;
        pl.off_xb.push_back(off);
        off = align_up(off + (size_t)nb * 8 * pl.nt * 256, 256);
        pl.off_cs.push_back(off);
        off = align_up(off + (size_t)nb * pl.nt * 8 * sizeof(float), 256);
    }
    pl.total = off;
    return pl;
}

template <int NT, int CAP>
cudaError_t launch_group_cap(const GemvProblemHost* probs, uint32_t count, uint32_t m, int x_dtype,
                             uint8_t* ws, const GroupPlan& pl, cudaStream_t stream) {
    using S_ = GemvShape<NT>;
    // ---- prep launch (unique x's) ----
    PrepLaunch<CAP> pre;
    pre.count = (uint32_t)pl.xs.size();
    pre.M = m;
    pre.counters = reinterpret_cast<uint32_t*>(ws + pl.off_counters);
    pre.ncounters = pl.counter_base.empty() ? 0u
                                            : pl.counter_base.back() + (probs[count - 1].n + pl.rows - 1) / pl.rows;
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
        warps += m * it.nb;
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
    cudaError_t e;
    switch (x_dtype) {
        case 0: e = cudaLaunchKernelEx(&cfg, gemv_prep_kernel<float, NT, CAP>, pre); break;
        case 1: e = cudaLaunchKernelEx(&cfg, gemv_prep_kernel<__half, NT, CAP>, pre); break;
        default: e = cudaLaunchKernelEx(&cfg, gemv_prep_kernel<__nv_bfloat16, NT, CAP>, pre); break;
    }
    if (e != cudaSuccess) return e;

    // ---- GEMV launch ----
    static bool attr_set[64] = {};  // per device; an idempotent attribute, so a race is benign
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 64 || !attr_set[dev]) {
        e = cudaFuncSetAttribute(gemv_kernel<NT, CAP>, cudaFuncAttributeMaxDynamicSharedMemorySize, S_::SMEM);
        if (e != cudaSuccess) return e;
        if (dev < 64) attr_set[dev] = true;
    }
    GemvLaunch<CAP> L;
    L.count = count;
    L.M = m;
    L.total_steps = pl.total_steps;
    L.pad = 0;
    L.partial = reinterpret_cast<float*>(ws + pl.off_partial);
    L.counters = reinterpret_cast<uint32_t*>(ws + pl.off_counters);
    uint32_t tb = 0;
    for (uint32_t i = 0; i < count; ++i) {
        GemvProblem& P = L.prob[i];
        const uint32_t nb = (probs[i].k + QK - 1) / QK;
        P.qs = probs[i].qs;
        P.sc = probs[i].sc;
        P.xb = ws + pl.off_xb[pl.x_of[i]];
        P.colscale = reinterpret_cast<const float*>(ws + pl.off_cs[pl.x_of[i]]);
        P.out = probs[i].out;
        P.N = probs[i].n;
        P.nb = nb;
        P.row_groups = (probs[i].n + pl.rows - 1) / pl.rows;
        P.tb_begin = tb;
        P.counter_base = pl.counter_base[i];
        P.pad = 0;
        tb += P.row_groups * nb;
    }
    cfg.gridDim = dim3(pl.grid);
    cfg.blockDim = dim3(GEMV_WARPS * 32);
    cfg.dynamicSmemBytes = S_::SMEM;
    e = cudaLaunchKernelEx(&cfg, gemv_kernel<NT, CAP>, L);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

template <int NT>
cudaError_t launch_group_nt(const GemvProblemHost* probs, uint32_t count, uint32_t m, int x_dtype,
                            uint8_t* ws, const GroupPlan& pl, cudaStream_t stream) {
    // parameter capacity: a single projection ships ~100 bytes of launch parameters, not 16 KB
    if (count <= 1) return launch_group_cap<NT, 1>(probs, count, m, x_dtype, ws, pl, stream);
    if (count <= 16) return launch_group_cap<NT, 16>(probs, count, m, x_dtype, ws, pl, stream);
    return launch_group_cap<NT, MAX_PROBLEMS>(probs, count, m, x_dtype, ws, pl, stream);
}

}  // namespace

bool gemv_fast_path_ok(uint32_t m, uint32_t k, const uint8_t* qs, const uint8_t* sc) {
    return m >= 1 && m <= 16 && k >= 1 && (reinterpret_cast<uintptr_t>(qs) % 16) == 0 &&
           (reinterpret_cast<uintptr_t>(sc) % 4) == 0;
}

uint32_t gemv_max_group() { return MAX_PROBLEMS; }

size_t gemv_group_workspace_size(const GemvProblemHost* probs, uint32_t count, uint32_t m, int num_sms) {
    if (count == 0) return 0;
    return plan_group(probs, count, m, num_sms).total;
}

size_t gemv_workspace_size(uint32_t m, uint32_t n, uint32_t k, int num_sms) {
    GemvProblemHost p{nullptr, nullptr, nullptr, n, k, nullptr};
    return gemv_group_workspace_size(&p, 1, m, num_sms);
}

cudaError_t launch_gemv_group(const GemvProblemHost* probs, uint32_t count, uint32_t m, int x_dtype,
                              void* workspace, int num_sms, cudaStream_t stream) {
    if (count == 0) return cudaSuccess;
    const GroupPlan pl = plan_group(probs, count, m, num_sms);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    switch (pl.nt) {
        case 1: return launch_group_nt<1>(probs, count, m, x_dtype, ws, pl, stream);
        case 2: return launch_group_nt<2>(probs, count, m, x_dtype, ws, pl, stream);
        case 4: return launch_group_nt<4>(probs, count, m, x_dtype, ws, pl, stream);
        default: return launch_group_nt<8>(probs, count, m, x_dtype, ws, pl, stream);
    }
}

cudaError_t launch_gemv(const void* x, int x_dtype, uint32_t m, const uint8_t* qs, const uint8_t* sc,
                        uint32_t n, uint32_t k, float* out, void* workspace, int num_sms,
                        cudaStream_t stream) {
    GemvProblemHost p{x, qs, sc, n, k, out};
    return launch_gemv_group(&p, 1, m, x_dtype, workspace, num_sms, stream);
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
