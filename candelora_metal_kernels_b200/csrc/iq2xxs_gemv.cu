// IQ2_XXS decode GEMV for small m (m <= 16) on sm_100a.
//
// Computes out[m, n] = sum_k x[m, k] * W[n, k] with W the IQ2_XXS weights in the reference's
// split layout (reference: iq2_xxs_matmul_kernel, src/metal_src/iq2_matmul.metal:188-240;
// weight formula decode_iq2_xxs_value :701-734):
//   W[n, blk*256 + ib32*32 + g*8 + j] = d * (0.5 + s) * 0.25 * grid[aux_g.byte g].byte j * sign
// with, per 32-weight sub-block ib32 of block blk (8 bytes at qs + (n*nb + blk)*64 + ib32*8):
//   aux_g = bytes 0..3 (four 8-bit grid indices), aux_s = bytes 4..7 (four 7-bit sign indices
//   at bits 7g..7g+6, 4-bit scale s at bits 28..31), d = fp16 block scale.
//
// B200 design. Every weight is used once at m = 1, so the cost that matters is the work per
// weight on the way from HBM to an accumulator. The weights never become floats:
//   * d*(0.5+s)*0.25 = d * (2s+1) / 8, and every signed grid value is an int8 in
//     {+-8, +-25, +-43}. One `prmt` turns a 16-bit selector (grid code | sign, from two
//     lane-replicated shared-memory tables) into four signed int8 weights.
//   * x is split per (token, 256-block) into four 7-bit signed limbs of a 28-bit fixed-point
//     value (gemv_prep_kernel), so x @ W^T becomes integer tensor-core work:
//     mma.m16n8k32 s8 x s8 -> s32 per 32-weight sub-block, scaled by the odd integer (2s+1)
//     in s32 (exact: |sum| < 2^31), and turned into f32 once per 256-block with d and the
//     limb/token scale. The only rounding is the 2^-28-relative quantisation of x and f32
//     rounding of the per-block partial sums, far inside the 1e-4 relative L2 bound.
//   * The weight stream is staged with cp.async into a per-warp shared-memory ring (no
//     register staging, several KB in flight per warp); 16-byte chunks are XOR-swizzled so the
//     8 rows a warp reads per step hit 8 different banks.
//   * Work units are (32 or 16 rows) x (a few 256-blocks of K): split-K keeps every SM busy
//     for k/v-sized projections. Split-K partials are summed in a fixed order by the last
//     warp to finish a row group (an atomic ticket per group), so results are deterministic.
#include "iq2xxs_common.cuh"
#include "iq2xxs_codebook.h"
#include "iq2xxs_internal.h"

namespace iq2 {

namespace {

constexpr int GEMV_WARPS = 16;
constexpr int LUT_BYTES = 256 * 256;  // 256 rows x (32 lanes grid selectors | 32 lanes sign)

template <int NT>
struct GemvShape {
    static constexpr int T = NT <= 2 ? 2 : 1;           // 16-row mma tiles per warp
    static constexpr int ROWS = 16 * T;                 // rows per work unit
    static constexpr int STAGE_QS = ROWS * 128;         // 2 blocks of qs per row
    static constexpr int STAGE_BYTES = STAGE_QS + ROWS * 4;  // + 2 fp16 scales per row
    static constexpr int NSTAGES = T == 2 ? 2 : 4;
    static constexpr int SMEM = LUT_BYTES + GEMV_WARPS * NSTAGES * STAGE_BYTES;
};

// ---------------------------------------------------------------------------------------------
// x -> int8 limb fragments. One warp per (token m, block b); lane = (sub-block sbi, group t)
// owns the 8 activations k = b*256 + sbi*32 + t*8 + [0, 8).
// With amax = max |x| over the block and amax = f * 2^E (f in [0.5, 1)):
//   q = rint(x * 2^(27-E)) (|q| <= 2^27), |q| = L3*2^21 + L2*2^14 + L1*2^7 + L0 (7-bit limbs),
//   each limb carrying the sign of q; column scale of limb l = 2^(E - 27 + 7l) / 8 (the /8 is
//   the weight scale's (2s+1)/8). Non-finite blocks get NaN scales, so the output is NaN.
// Output fragment layout (mma B operand, m16n8k32 "col"): for sub-block sb and n8 tile nt,
//   xb[((sb*NT + nt)*32 + col*4 + t)*8 + i] = limb of activation group t, element i, where
//   col = (m % 2)*4 + l and nt = m / 2.
template <typename XT, int NT>
__global__ void __launch_bounds__(256) gemv_prep_kernel(const XT* __restrict__ x, uint32_t M,
                                                        uint32_t K, uint32_t nb,
                                                        uint8_t* __restrict__ xb,
                                                        float* __restrict__ colscale,
                                                        uint32_t* __restrict__ counters,
                                                        uint32_t ncounters) {
    // x may be written by the previous kernel and the workspace may still be read by the
    // previous GEMV: wait for both before touching memory. Only then let the GEMV launch, so
    // its early weight prefetch also runs after every earlier kernel has finished.
    pdl_wait();
    pdl_launch_dependents();
    if (blockIdx.x == 0) {
        for (uint32_t i = threadIdx.x; i < ncounters; i += blockDim.x) counters[i] = 0u;
    }
    const uint32_t wid = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (wid >= M * nb) return;
    const uint32_t m = wid / nb, b = wid % nb;
    const int sbi = lane >> 2, t = lane & 3;
    const size_t k0 = (size_t)b * QK + sbi * 32 + t * 8;
    const XT* xr = x + (size_t)m * K;

    float v[8];
    float amax = 0.0f;
    bool bad = false;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const size_t k = k0 + i;
        v[i] = k < K ? to_f32(xr[k]) : 0.0f;
        bad |= !isfinite(v[i]);
        amax = fmaxf(amax, fabsf(v[i]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
    }
    bad = __any_sync(0xFFFFFFFFu, bad);

    int E = 0;
    if (!bad && amax > 0.0f) frexpf(amax, &E);
    uint32_t lo[4] = {0, 0, 0, 0}, hi[4] = {0, 0, 0, 0};
    if (!bad && amax > 0.0f) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float qf = rintf(ldexpf(v[i], 27 - E));
            const int q = (int)qf;
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
        uint2* dst = reinterpret_cast<uint2*>(xb + ((sb * NT + nt) * 32 + (colbase + l) * 4 + t) * 8);
        *dst = make_uint2(lo[l], hi[l]);
    }
    if (lane < 4) {
        float s;
        if (bad) s = __int_as_float(0x7FC00000);
        else if (amax == 0.0f) s = 0.0f;
        else s = ldexpf(1.0f, E - 30 + 7 * lane);
        colscale[(size_t)b * (NT * 8) + nt * 8 + colbase + lane] = s;
    }
}

// ---------------------------------------------------------------------------------------------
struct GemvParams {
    const uint8_t* qs;
    const uint8_t* sc;
    const uint8_t* xb;
    const float* colscale;
    float* out;
    float* partial;
    uint32_t* counters;
    size_t row_bytes;  // nb * 64
    uint32_t M, N, nb;
    uint32_t S, kb;    // K splits per row group, blocks per split
    uint32_t total_units;
};

// Four signed int8 weights of one 8-weight group (row's sub-block word q), for this lane's
// group t: lo = weights 0..3, hi = weights 4..7.
__device__ __forceinline__ void decode_group(const uint8_t* lut, uint2 q, uint32_t selg,
                                             uint32_t laneoff, uint32_t rot, uint32_t soff,
                                             uint32_t& lo, uint32_t& hi) {
    const uint32_t ga = prmt(q.x, laneoff, selg);               // grid_idx*256 + lane*4
    const uint32_t sa = (__funnelshift_r(q.y, q.y, rot) & 0x7F00u) | soff;  // sign_idx*256+128+lane*4
    const uint32_t sel = lds32(lut, ga) | lds32(lut, sa);
    lo = prmt(KPOS, KNEG, sel);
    hi = prmt(KPOS, KNEG, sel >> 16);
}

template <int NT>
__global__ void __launch_bounds__(GEMV_WARPS * 32, 1) gemv_kernel(const GemvParams p) {
    using S_ = GemvShape<NT>;
    constexpr int T = S_::T, ROWS = S_::ROWS, STAGE_QS = S_::STAGE_QS;
    constexpr int STAGE_BYTES = S_::STAGE_BYTES, NSTAGES = S_::NSTAGES;
    extern __shared__ __align__(128) uint8_t smem[];
    const uint8_t* lut = smem;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    uint8_t* ring = smem + LUT_BYTES + warp * (NSTAGES * STAGE_BYTES);

    // Lane-replicated selector tables: row e holds IQ2XXS_GRID_SEL[e] in bytes [0,128) (one
    // copy per lane) and IQ2XXS_SIGN_SEL[e] in [128,256) for e < 128. A lane only ever reads
    // its own copy, so the random table lookups of a warp never conflict on a bank.
    {
        uint32_t* lw = reinterpret_cast<uint32_t*>(smem);
        for (int i = threadIdx.x; i < 256 * 64; i += blockDim.x) {
            const int e = i >> 6, w = i & 63;
            lw[i] = (w < 32) ? IQ2XXS_GRID_SEL[e] : (e < 128 ? IQ2XXS_SIGN_SEL[e] : 0u);
        }
    }
    __syncthreads();

    const uint32_t W = gridDim.x * GEMV_WARPS;
    const uint32_t gw = blockIdx.x * GEMV_WARPS + warp;
    const uint32_t laneoff = (uint32_t)lane * 4u;
    const uint32_t selg = 0x5504u | ((uint32_t)t << 4);
    const uint32_t rot = (7u * t + 24u) & 31u;
    const uint32_t soff = 128u + laneoff;

    // ---- producer side: issue cursor over (unit, stage) ----
    uint32_t iu = gw, ist = 0;
    int islot = 0;
    auto issue = [&]() {
        if (iu < p.total_units) {
            const uint32_t rg = iu / p.S, s = iu % p.S;
            const uint32_t blk = s * p.kb + 2u * ist;
            const uint32_t row0 = rg * ROWS;
            uint8_t* st = ring + islot * STAGE_BYTES;
#pragma unroll
            for (int c = 0; c < ROWS * 8 / 32; ++c) {
                const int idx = c * 32 + lane;
                const int r = idx >> 3, ch = idx & 7;
                const uint32_t row = row0 + r;
                const bool ok = row < p.N;
                const uint8_t* src = p.qs + (ok ? (size_t)row * p.row_bytes + (size_t)blk * QS_BYTES + ch * 16 : 0);
                cp_async_16(smem_u32(st + r * 128 + ((ch ^ (r & 7)) << 4)), src, ok ? 16u : 0u);
            }
            if (lane < ROWS) {
                const uint32_t row = row0 + lane;
                const bool ok = row < p.N;
                const uint8_t* src = p.sc + (ok ? ((size_t)row * p.nb + blk) * SC_BYTES : 0);
                cp_async_4(smem_u32(st + STAGE_QS + lane * 4), src, ok ? 4u : 0u);
            }
            const uint32_t nblk = min(p.kb, p.nb - s * p.kb);
            if ((++ist) * 2u >= nblk) {
                ist = 0;
                iu += W;
            }
        }
        cp_async_commit();
        islot = (islot + 1 == NSTAGES) ? 0 : islot + 1;
    };

#pragma unroll
    for (int i = 0; i < NSTAGES; ++i) issue();

    // Everything above (table fill, first weight stages) reads only constants and weights; the
    // x fragments, scales table, counters and outputs come from / are shared with the prep
    // kernel, so wait for it here.
    pdl_wait();

    bool bact[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) bact[nt] = (uint32_t)(nt * 2 + (g >> 2)) < p.M;

    float F[T][NT][4];
#pragma unroll
    for (int a = 0; a < T; ++a)
#pragma unroll
        for (int b = 0; b < NT; ++b)
#pragma unroll
            for (int c = 0; c < 4; ++c) F[a][b][c] = 0.0f;

    uint32_t cu = gw, cst = 0;
    int slot = 0;
    while (cu < p.total_units) {
        cp_async_wait<NSTAGES - 1>();
        __syncwarp();
        const uint8_t* st = ring + slot * STAGE_BYTES;
        const uint32_t rg = cu / p.S, s = cu % p.S;
        const uint32_t nblk_u = min(p.kb, p.nb - s * p.kb);
        const uint32_t blk0 = s * p.kb + 2u * cst;

#pragma unroll 1
        for (int bi = 0; bi < 2; ++bi) {
            const uint32_t gblk = blk0 + bi;
            int I[T][NT][4];
#pragma unroll
            for (int a = 0; a < T; ++a)
#pragma unroll
                for (int b = 0; b < NT; ++b)
#pragma unroll
                    for (int c = 0; c < 4; ++c) I[a][b][c] = 0;

#pragma unroll
            for (int sbi = 0; sbi < 8; ++sbi) {
                const int sb = bi * 8 + sbi;
                uint32_t bf[NT][2];
                const uint8_t* bsrc = p.xb + ((size_t)(gblk * 8 + sbi) * NT) * 256 + lane * 8;
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    uint2 v = make_uint2(0u, 0u);
                    if (bact[nt]) v = __ldg(reinterpret_cast<const uint2*>(bsrc + nt * 256));
                    bf[nt][0] = v.x;
                    bf[nt][1] = v.y;
                }
                const uint32_t off = ((((uint32_t)sb >> 1) ^ (uint32_t)g) << 4) | (((uint32_t)sb & 1u) << 3);
#pragma unroll
                for (int tt = 0; tt < T; ++tt) {
                    const uint2 q0 = lds64(st, (tt * 16 + g) * 128 + off);
                    const uint2 q1 = lds64(st, (tt * 16 + g + 8) * 128 + off);
                    uint32_t a0, a1, a2, a3;
                    decode_group(lut, q0, selg, laneoff, rot, soff, a0, a2);
                    decode_group(lut, q1, selg, laneoff, rot, soff, a1, a3);
                    const int c0 = (int)((q0.y >> 27) | 1u), c1 = (int)((q1.y >> 27) | 1u);
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        int d[4];
                        mma_s8_16832(d, a0, a1, a2, a3, bf[nt][0], bf[nt][1]);
                        I[tt][nt][0] += c0 * d[0];
                        I[tt][nt][1] += c0 * d[1];
                        I[tt][nt][2] += c1 * d[2];
                        I[tt][nt][3] += c1 * d[3];
                    }
                }
            }
            // Block epilogue: s32 -> f32 with d (per row) and the limb/token scale (per column).
            float2 cs[NT];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
                cs[nt] = __ldg(reinterpret_cast<const float2*>(p.colscale + (size_t)gblk * (NT * 8) + nt * 8 + 2 * t));
#pragma unroll
            for (int tt = 0; tt < T; ++tt) {
                const float d0 = half_bits_to_float(*reinterpret_cast<const uint16_t*>(st + STAGE_QS + (tt * 16 + g) * 4 + bi * 2));
                const float d1 = half_bits_to_float(*reinterpret_cast<const uint16_t*>(st + STAGE_QS + (tt * 16 + g + 8) * 4 + bi * 2));
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    F[tt][nt][0] = fmaf((float)I[tt][nt][0], d0 * cs[nt].x, F[tt][nt][0]);
                    F[tt][nt][1] = fmaf((float)I[tt][nt][1], d0 * cs[nt].y, F[tt][nt][1]);
                    F[tt][nt][2] = fmaf((float)I[tt][nt][2], d1 * cs[nt].x, F[tt][nt][2]);
                    F[tt][nt][3] = fmaf((float)I[tt][nt][3], d1 * cs[nt].y, F[tt][nt][3]);
                }
            }
        }

        const bool last = (cst + 1u) * 2u >= nblk_u;
        __syncwarp();
        issue();  // refill the slot just consumed
        slot = (slot + 1 == NSTAGES) ? 0 : slot + 1;
        if (!last) {
            ++cst;
            continue;
        }

        // ---- unit epilogue: reduce limb columns to tokens, write out or a split-K partial ----
        const uint32_t row0 = rg * ROWS;
        float* dst_base = p.S == 1 ? p.out : p.partial + (size_t)s * p.M * p.N;
#pragma unroll
        for (int tt = 0; tt < T; ++tt) {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                float v0 = F[tt][nt][0] + F[tt][nt][1];
                float v1 = F[tt][nt][2] + F[tt][nt][3];
                v0 += __shfl_xor_sync(0xFFFFFFFFu, v0, 1);
                v1 += __shfl_xor_sync(0xFFFFFFFFu, v1, 1);
                const uint32_t m = nt * 2 + (t >> 1);
                const uint32_t r0 = row0 + tt * 16 + g, r1 = r0 + 8;
                if ((t & 1) == 0 && m < p.M) {
                    float* dst = dst_base + (size_t)m * p.N;
                    if (r0 < p.N) dst[r0] = v0;
                    if (r1 < p.N) dst[r1] = v1;
                }
                F[tt][nt][0] = F[tt][nt][1] = F[tt][nt][2] = F[tt][nt][3] = 0.0f;
            }
        }
        if (p.S > 1) {
            __threadfence();
            __syncwarp();
            uint32_t prev = 0;
            if (lane == 0) prev = atomicAdd(p.counters + rg, 1u);
            prev = __shfl_sync(0xFFFFFFFFu, prev, 0);
            if (prev == p.S - 1) {
                __threadfence();
                for (uint32_t idx = lane; idx < (uint32_t)ROWS * p.M; idx += 32) {
                    const uint32_t m = idx / ROWS, row = row0 + idx % ROWS;
                    if (row >= p.N) continue;
                    float acc = 0.0f;
                    for (uint32_t ss = 0; ss < p.S; ++ss)
                        acc += __ldcg(p.partial + ((size_t)ss * p.M + m) * p.N + row);
                    p.out[(size_t)m * p.N + row] = acc;
                }
                if (lane == 0) p.counters[rg] = 0u;
            }
        }
        cst = 0;
        cu += W;
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
    for (size_t w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; w < total;
         w += (size_t)gridDim.x * blockDim.x / 32) {
        const uint32_t n = (uint32_t)(w / mchunks), mc = (uint32_t)(w % mchunks) * 8;
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
            for (int j = 0; j < 8; ++j) {
                const size_t k = k0 + j;
                if (k >= K) break;
                const float wv = dl * (float)((gw >> (8 * j)) & 0xFF) * (((signs >> j) & 1u) ? -1.0f : 1.0f);
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
template <int NT>
int nt_of() { return NT; }

struct Plan {
    int nt;
    uint32_t rows, row_groups, S, kb, units, grid;
    size_t off_xb, off_cs, off_partial, off_counters, total;
};

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

Plan make_plan(uint32_t m, uint32_t n, uint32_t k, int num_sms) {
    Plan pl{};
    pl.nt = m <= 2 ? 1 : (m <= 4 ? 2 : (m <= 8 ? 4 : 8));
    pl.rows = pl.nt <= 2 ? 32u : 16u;
    const uint32_t nb = (k + QK - 1) / QK;
    pl.row_groups = (n + pl.rows - 1) / pl.rows;
    const uint64_t warps = (uint64_t)num_sms * GEMV_WARPS;
    uint32_t kb = 2;
    while (kb * 2 <= nb && (uint64_t)pl.row_groups * ((nb + kb * 2 - 1) / (kb * 2)) >= 6 * warps) kb *= 2;
    pl.kb = kb;
    pl.S = (nb + kb - 1) / kb;
    pl.units = pl.row_groups * pl.S;
    const uint64_t ctas = (pl.units + GEMV_WARPS - 1) / GEMV_WARPS;
    pl.grid = (uint32_t)(ctas < (uint64_t)num_sms ? ctas : (uint64_t)num_sms);
    size_t off = 0;
    pl.off_xb = off;
    off = align_up(off + (size_t)nb * 8 * pl.nt * 256, 256);
    pl.off_cs = off;
    off = align_up(off + (size_t)nb * pl.nt * 8 * sizeof(float), 256);
    pl.off_partial = off;
    if (pl.S > 1) off = align_up(off + (size_t)pl.S * m * n * sizeof(float), 256);
    pl.off_counters = off;
    if (pl.S > 1) off = align_up(off + (size_t)pl.row_groups * sizeof(uint32_t), 256);
    pl.total = off;
    return pl;
}

template <int NT>
cudaError_t launch_gemv_nt(const void* x, int x_dtype, uint32_t m, const uint8_t* qs, const uint8_t* sc,
                           uint32_t n, uint32_t k, float* out, uint8_t* ws, const Plan& pl,
                           cudaStream_t stream) {
    const uint32_t nb = (k + QK - 1) / QK;
    uint8_t* xb = ws + pl.off_xb;
    float* cs = reinterpret_cast<float*>(ws + pl.off_cs);
    float* partial = reinterpret_cast<float*>(ws + pl.off_partial);
    uint32_t* counters = reinterpret_cast<uint32_t*>(ws + pl.off_counters);
    const uint32_t ncounters = pl.S > 1 ? pl.row_groups : 0u;
    const uint32_t prep_blocks = (m * nb * 32 + 255) / 256;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(prep_blocks);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e;
    switch (x_dtype) {
        case 0: e = cudaLaunchKernelEx(&cfg, gemv_prep_kernel<float, NT>, static_cast<const float*>(x), m, k,
                                       nb, xb, cs, counters, ncounters); break;
        case 1: e = cudaLaunchKernelEx(&cfg, gemv_prep_kernel<__half, NT>, static_cast<const __half*>(x), m,
                                       k, nb, xb, cs, counters, ncounters); break;
        default: e = cudaLaunchKernelEx(&cfg, gemv_prep_kernel<__nv_bfloat16, NT>,
                                        static_cast<const __nv_bfloat16*>(x), m, k, nb, xb, cs, counters,
                                        ncounters); break;
    }
    if (e != cudaSuccess) return e;
    using S_ = GemvShape<NT>;
    static bool attr_set[64] = {};  // per device; benign race (idempotent attribute set)
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr_set[dev]) {
        e = cudaFuncSetAttribute(gemv_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, S_::SMEM);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    GemvParams p;
    p.qs = qs;
    p.sc = sc;
    p.xb = xb;
    p.colscale = cs;
    p.out = out;
    p.partial = partial;
    p.counters = counters;
    p.row_bytes = (size_t)nb * QS_BYTES;
    p.M = m;
    p.N = n;
    p.nb = nb;
    p.S = pl.S;
    p.kb = pl.kb;
    p.total_units = pl.units;
    cfg.gridDim = dim3(pl.grid);
    cfg.blockDim = dim3(GEMV_WARPS * 32);
    cfg.dynamicSmemBytes = S_::SMEM;
    e = cudaLaunchKernelEx(&cfg, gemv_kernel<NT>, p);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

}  // namespace

bool gemv_fast_path_ok(uint32_t m, uint32_t k, const uint8_t* qs, const uint8_t* sc) {
    const uint32_t nb = (k + QK - 1) / QK;
    return m >= 1 && m <= 16 && nb >= 2 && (nb % 2) == 0 &&
           (reinterpret_cast<uintptr_t>(qs) % 16) == 0 && (reinterpret_cast<uintptr_t>(sc) % 4) == 0;
}

size_t gemv_workspace_size(uint32_t m, uint32_t n, uint32_t k, int num_sms) {
    return make_plan(m, n, k, num_sms).total;
}

cudaError_t launch_gemv(const void* x, int x_dtype, uint32_t m, const uint8_t* qs, const uint8_t* sc,
                        uint32_t n, uint32_t k, float* out, void* workspace, int num_sms,
                        cudaStream_t stream) {
    const Plan pl = make_plan(m, n, k, num_sms);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    switch (pl.nt) {
        case 1: return launch_gemv_nt<1>(x, x_dtype, m, qs, sc, n, k, out, ws, pl, stream);
        case 2: return launch_gemv_nt<2>(x, x_dtype, m, qs, sc, n, k, out, ws, pl, stream);
        case 4: return launch_gemv_nt<4>(x, x_dtype, m, qs, sc, n, k, out, ws, pl, stream);
        default: return launch_gemv_nt<8>(x, x_dtype, m, qs, sc, n, k, out, ws, pl, stream);
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
