// IQ2_XXS prefill GEMM (m > 32) on the sm_100a tensor cores: tcgen05.mma with TMEM accumulators.
//
// out[m, n] = sum_k x[m, k] * W[n, k] (reference: iq2_xxs_matmul_kernel,
// src/metal_src/iq2_matmul.metal:188-240, which recomputes the weights per output element) as a
// dense bf16 x bf16 -> f32 contraction:
//   * A = x, bf16 [M, K] (f32/f16 x is first narrowed to bf16 into the workspace), loaded by TMA
//     as 128-row x 64-k boxes with the 128-byte swizzle;
//   * B = W, dequantised to bf16 in shared memory by 16 decode warps, directly in the canonical
//     SW128 K-major layout the MMA reads. Each weight is bf16(d*(2s+1)/8 * g) for g in {8,25,43}:
//     the three products of a 32-weight sub-block are rounded once and a `prmt` picks the bf16
//     pairs by grid code (IQ2XXS_BF16_SEL), an XOR applies the signs (the 7 stored sign bits and
//     their parity spread to the bf16 sign bits by one multiply per pair). This is bit-identical to
//     rounding every weight's exact f32 value (the dequant kernel's bf16). The table is kept small
//     (2 KB, held in 16 interleaved copies so that the 16 lanes of a half-warp, each reading its
//     own copy, never share a bank) because the tensor core reads its operands through the same
//     shared memory.
//   * D: two 128 x BN f32 accumulators in TMEM (512 columns allocated): one CTA computes a tile of
//     256 tokens x BN weight rows (BN = 256 or 224, from the cost model of gemm_plan), issuing per
//     64-k stage 2 x 4 tcgen05.mma (M=128, N=BN, K=16) from one thread; tcgen05.commit frees each
//     stage when the tensor core has read it. The tiles of the last, part-full wave of CTAs are
//     split over K (partial tiles, summed in order by splitk_tile_sum_kernel).
//   * Pipeline: 3 stages of 64 KB, mbarriers for "x landed" (TMA transaction bytes), "weights
//     written" (decode warps) and "stage free" (MMA commit). Every wait is bounded: on timeout
//     the kernel records an error code, stops issuing work and still frees its TMEM.
//   * Epilogue: TMEM -> registers -> a 32 x 32 tile in the idle stage ring -> TMA store.
// No TMA multicast is used anywhere (this library also runs on multi-GPU jobs).
#include "iq2xxs_common.cuh"
#include "iq2xxs_codebook.h"
#include "iq2xxs_internal.h"

#include <cuda.h>

#include <algorithm>
#include <cstring>
#include <mutex>

namespace iq2 {

namespace {

constexpr int G_BM = 256;                       // tokens per CTA (two M=128 MMAs)
constexpr int G_BN = 256;                       // weight rows per CTA (MMA N), at most; BN = 224 also used
constexpr int G_BK = 64;                        // k per stage (one 128-byte swizzle row of bf16)
constexpr int G_STAGES = 3;
constexpr int G_DEC_WARPS = 16;                 // decode warps = epilogue warps
constexpr int G_TMA_WARP = G_DEC_WARPS;         // warp 16
constexpr int G_MMA_WARP = G_DEC_WARPS + 1;     // warp 17
constexpr int G_THREADS = (G_DEC_WARPS + 2) * 32;
constexpr int G_A_HALF = 128 * G_BK * 2;        // 16 KB: one 128-token box
constexpr int G_A_BYTES = 2 * G_A_HALF;         // 32 KB
constexpr int G_B_BYTES = G_BN * G_BK * 2;      // 32 KB
constexpr int G_STAGE_BYTES = G_A_BYTES + G_B_BYTES;
constexpr int G_SEL_COPIES = 16;                 // the decode table, once per lane of a half-warp
constexpr int G_SEL_BYTES = 256 * G_SEL_COPIES * 8;  // selector pairs per grid code, interleaved copies
constexpr int G_SMEM = 1024 /*align*/ + G_STAGES * G_STAGE_BYTES + G_SEL_BYTES + 256 /*barriers*/;
constexpr uint32_t G_TMEM_COLS = 512;
constexpr uint64_t WAIT_LIMIT_NS = 2000000000ull;  // 2 s: only a broken pipeline waits that long

// Per-device sticky status of the GEMM's bounded waits (the bits of the waits that ran out since
// the last iq2_device_check; 0 = none). Every GPU that loads the library has its own copy.
__device__ unsigned int g_gemm_status;

// Test knobs (iq2_testing_set_gemm_stall): the wait bound, and a stage whose "weights written"
// arrival the decode warps withhold, so that the MMA thread's wait on it runs out.
uint64_t g_wait_limit_ns = WAIT_LIMIT_NS;
uint32_t g_stall_stage = 0;  // 0: none; s > 0: stage s - 1 of every CTA

// Instruction descriptor, kind::f16: F32 accumulate, BF16 A and B, both K-major, M=128, N=BN.
template <int BN>
constexpr uint32_t idesc_for() {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

// The launch's work units (blockIdx.x): tiles t = (m-tile t / nt, n-tile t % nt). The first `full`
// tiles are computed whole, one unit each; each of the R tiles after them is split into `s`
// ranges of whole 256-blocks of K (units full + (t - full) * s + z), whose partial sums go to
// part[(t - full) * s + z][row][col] and are added up in z order by splitk_tile_sum_kernel. The
// split fills the last wave of CTAs (or the only one, when there are fewer tiles than SMs).
struct GemmParams {
    const uint8_t* qs;
    const uint8_t* sc;
    float* out;     // [M, N]
    float* part;    // [R * s][PR][BN] partial sums of the split tiles (null when none is split)
    unsigned int* err;  // the device's sticky status word (g_gemm_status); set on a pipeline timeout
    uint64_t wait_ns;   // bound of every mbarrier wait
    uint32_t stall;     // test hook: see g_stall_stage
    uint32_t M, N, K, nb;
    uint32_t nt, full, s;
    uint32_t PR;    // rows of a partial tile: 256, or M rounded up to 32 below that
    uint32_t tma;   // the epilogue stores through the tensor maps (else per thread)
    uint32_t vec;   // per-thread stores may be 16 bytes wide (N % 4 == 0 and out 16-byte aligned)
};

// ---- mbarrier / tcgen05 / TMA wrappers (inline PTX) ----
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(bar),
                 "r"(bytes)
                 : "memory");
}
// One test of the phase; a thread may be suspended for at most ~10 us (the hint) inside it.
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(10000u)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Bounded wait: false (and the error code recorded) if the phase does not complete within
// `limit` ns of wall time.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, unsigned int* err, uint32_t code,
                                          uint64_t limit) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (;;) {
        for (int i = 0; i < 32; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (global_ns() - t0 > limit) {
            atomicOr(err, code);
            return false;
        }
    }
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            dst),
        "l"(map), "r"(bar), "r"(x), "r"(y)
        : "memory");
}

// TMA store of a 32 x 32 f32 tile (128-byte swizzled rows in shared memory) to a 3-D f32 tensor
// (the output [1][M][N] or the partial tiles [R*s][PR][BN]); what lies outside it is not written.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t src, int x, int y, int z) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(map),
                 "r"(src), "r"(x), "r"(y), "r"(z)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// SW128 K-major shared-memory matrix descriptor: start address, LBO = 16 B (unused for swizzled
// K-major), SBO = 1024 B between 8-row groups, version 1, layout SWIZZLE_128B.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
    d |= (uint64_t)1u << 16;
    d |= (uint64_t)(1024u >> 4) << 32;
    d |= (uint64_t)1u << 46;
    d |= (uint64_t)2u << 61;
    return d;
}

__device__ __forceinline__ uint32_t cvt_bf16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint4 v) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

// One 32-weight sub-block (8 bytes: aux_g, aux_s) of one row -> 32 bf16 weights, written as four
// 16-byte chunks at dst ^ (t << 4) (dst: the row's first chunk of the sub-block in the SW128 tile,
// its low 7 bits the swizzled chunk; t < 4 only flips bits 4-5). Each weight is
// bf16(d*(2s+1)/8 * g) with g in {8, 25, 43}: the three products are rounded once and a `prmt`
// picks the bf16 pairs by grid code (sel_l: this lane's copy of IQ2XXS_BF16_SEL, two words per
// entry, entries 128 bytes apart); an XOR applies the signs. TAIL: zero the weights at k >= K
// (k_lo = the sub-block's first k).
template <bool TAIL>
__device__ __forceinline__ void decode_sub(uint2 q, float d, uint32_t sel_l, uint32_t dst, uint32_t k_lo,
                                           uint32_t K) {
    const uint32_t aux_g = q.x, aux_s = q.y;
    const float dl = d * (float)((aux_s >> 27) | 1u) * 0.125f;  // d*(2s+1)/8, exact
    const uint32_t qlo = cvt_bf16x2(dl * 8.0f, dl * 25.0f);     // {bf16(8dl), bf16(25dl)}
    const uint32_t qhi = cvt_bf16x2(dl * 43.0f, 0.0f);          // {bf16(43dl), 0}
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        const uint32_t gi = (aux_g >> (8 * t)) & 0xFFu, si = (aux_s >> (7 * t)) & 0x7Fu;
        const uint2 sel = ld_shared_v2_const(sel_l + gi * (G_SEL_COPIES * 8));
        // the 8 sign bits (bit j: weight j negative): 7 stored, the 8th makes their parity even
        const uint32_t S = si | ((__popc(si) & 1u) << 7);
        // (S * K_i) & 0x80008000 puts sign bits 2i and 2i+1 at bits 15 and 31 (the two bf16 sign
        // bits of pair i): the shifted copies of S never overlap, no carries.
        uint4 w;
        w.x = prmt(qlo, qhi, sel.x) ^ ((S * 0x40008000u) & 0x80008000u);
        w.y = prmt(qlo, qhi, sel.x >> 16) ^ ((S * 0x10002000u) & 0x80008000u);
        w.z = prmt(qlo, qhi, sel.y) ^ ((S * 0x04000800u) & 0x80008000u);
        w.w = prmt(qlo, qhi, sel.y >> 16) ^ ((S * 0x01000200u) & 0x80008000u);
        if (TAIL && k_lo + t * 8 + 8 > K) {  // weights past in_dim contribute 0
            const uint32_t k0 = k_lo + t * 8;
            const uint32_t keep = k0 >= K ? 0u : K - k0;  // 0..7 weights kept
            w.x = keep >= 2 ? w.x : (keep == 1 ? (w.x & 0xFFFFu) : 0u);
            w.y = keep >= 4 ? w.y : (keep == 3 ? (w.y & 0xFFFFu) : 0u);
            w.z = keep >= 6 ? w.z : (keep == 5 ? (w.z & 0xFFFFu) : 0u);
            w.w = keep >= 8 ? w.w : (keep == 7 ? (w.w & 0xFFFFu) : 0u);
        }
        st_shared_v4(dst ^ ((uint32_t)t << 4), w);
    }
}

// ---- the kernel ----
// BN: weight rows per CTA (256, or 224 where that fills the last wave better); the stage
// layout is always sized for 256 rows.
template <int BN>
__global__ void __launch_bounds__(G_THREADS, 1) gemm_kernel(const __grid_constant__ CUtensorMap tmap_x,
                                                            const __grid_constant__ CUtensorMap tmap_out,
                                                            const __grid_constant__ CUtensorMap tmap_part,
                                                            const GemmParams p) {
    static_assert(BN % 32 == 0 && BN <= G_BN, "BN");
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_s = smem_u32(smem_raw);
    const uint32_t base_s = (raw_s + 1023u) & ~1023u;  // SW128 tiles need 1024-byte alignment
    uint8_t* base = smem_raw + (base_s - raw_s);
    const uint32_t sel_s = base_s + G_STAGES * G_STAGE_BYTES;
    const uint32_t bar_s = sel_s + G_SEL_BYTES;
    // barriers: full_a[S], full_b[S], empty[S], acc_full; then the TMEM address word; abort flag
    auto full_a = [&](int s) { return bar_s + 8u * s; };
    auto full_b = [&](int s) { return bar_s + 8u * (G_STAGES + s); };
    auto empty = [&](int s) { return bar_s + 8u * (2 * G_STAGES + s); };
    const uint32_t acc_full = bar_s + 8u * (3 * G_STAGES);
    uint32_t* tmem_addr_word = reinterpret_cast<uint32_t*>(base + (bar_s - base_s) + 8 * (3 * G_STAGES + 1));
    volatile uint32_t* abort_flag = tmem_addr_word + 1;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // this CTA's unit: tile t, K range z of nz; pu = its partial tile (-1: the tile is whole)
    uint32_t t, z, nz;
    int pu;
    if (blockIdx.x < p.full) {
        t = blockIdx.x;
        z = 0;
        nz = 1;
        pu = -1;
    } else {
        const uint32_t v = blockIdx.x - p.full;
        t = p.full + v / p.s;
        z = v % p.s;
        nz = p.s;
        pu = (int)v;
    }
    const uint32_t n0 = (t % p.nt) * BN, m0 = (t / p.nt) * G_BM;
    // this CTA's share of K: the 256-blocks [b0, b1) of range z, i.e. the 64-k stages
    // [kt0, kt0 + NKT) (at least one: the host never makes more ranges than blocks)
    const uint32_t b0 = (uint32_t)((uint64_t)z * p.nb / nz);
    const uint32_t b1 = (uint32_t)((uint64_t)(z + 1) * p.nb / nz);
    const uint32_t kt0 = b0 * (QK / G_BK);
    const uint32_t NKT = min(b1 * (QK / G_BK), (p.K + G_BK - 1) / G_BK) - kt0;
    const bool upper = m0 + 128 < p.M;  // the tile's second 128-token half holds tokens

    // decode table -> shared memory: per grid entry the four 16-bit prmt selectors packed in two
    // words, G_SEL_COPIES times (copy c of entry e at (e * G_SEL_COPIES + c) * 8)
    for (int i = threadIdx.x; i < 256 * G_SEL_COPIES; i += blockDim.x) {
        const uint32_t* e = IQ2XXS_BF16_SEL[i / G_SEL_COPIES];
        reinterpret_cast<uint2*>(base + (sel_s - base_s))[i] = make_uint2(e[0] | (e[1] << 16), e[2] | (e[3] << 16));
    }
    if (threadIdx.x == 0) {
        for (int s = 0; s < G_STAGES; ++s) {
            mbar_init(full_a(s), 1);
            mbar_init(full_b(s), G_DEC_WARPS);
            mbar_init(empty(s), 1);
        }
        mbar_init(acc_full, 1);
        *abort_flag = 0u;
        fence_barrier_init();
    }
    if (warp == G_MMA_WARP) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_addr_word)),
                     "r"(G_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_addr_word;

    if (warp == G_TMA_WARP) {
        // ---------------- x producer ----------------
        if (lane == 0) {
            uint32_t issued = 0;
            bool aborted = false;
            for (uint32_t i = 0; i < NKT; ++i) {
                const int s = i % G_STAGES;
                if (i >= G_STAGES && !mbar_wait(empty(s), ((i / G_STAGES) - 1) & 1, p.err, 1u, p.wait_ns)) {
                    *abort_flag = 1u;
                    aborted = true;
                    break;
                }
                if (*abort_flag) {
                    aborted = true;
                    break;
                }
                const uint32_t a_s = base_s + s * G_STAGE_BYTES;
                const int kx = (int)((kt0 + i) * G_BK);
                mbar_expect_tx(full_a(s), upper ? G_A_BYTES : G_A_HALF);
                tma_load_2d(a_s, &tmap_x, full_a(s), kx, (int)m0);
                if (upper) tma_load_2d(a_s + G_A_HALF, &tmap_x, full_a(s), kx, (int)(m0 + 128));
                ++issued;
            }
            // after an abort, the loads already issued (at most one per stage slot, each the last
            // use of its slot) land before the CTA's shared memory goes away (bounded as well)
            if (aborted)
                for (uint32_t j = issued > G_STAGES ? issued - G_STAGES : 0u; j < issued; ++j)
                    mbar_wait(full_a(j % G_STAGES), (j / G_STAGES) & 1u, p.err, 32u, p.wait_ns);
        }
    } else if (warp == G_MMA_WARP) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            bool ok = true;
            for (uint32_t i = 0; i < NKT && ok; ++i) {
                const int s = i % G_STAGES;
                const uint32_t ph = (i / G_STAGES) & 1;
                ok = mbar_wait(full_a(s), ph, p.err, 2u, p.wait_ns) && mbar_wait(full_b(s), ph, p.err, 4u, p.wait_ns);
                if (!ok || *abort_flag) {
                    *abort_flag = 1u;
                    break;
                }
                tc_fence_after();
                const uint32_t a_s = base_s + s * G_STAGE_BYTES, b_s = a_s + G_A_BYTES;
#pragma unroll
                for (int ks = 0; ks < G_BK / 16; ++ks) {
                    const uint64_t bd = sw128_desc(b_s + ks * 32);
                    const uint32_t acc = (i | ks) ? 1u : 0u;
                    tc_mma(tmem, sw128_desc(a_s + ks * 32), bd, idesc_for<BN>(), acc);
                    if (upper) tc_mma(tmem + 256, sw128_desc(a_s + G_A_HALF + ks * 32), bd, idesc_for<BN>(), acc);
                }
                tc_commit(empty(s));  // the stage is free once these MMAs have read it
            }
            tc_commit(acc_full);      // fires when every MMA issued above has completed
        }
    } else {
        // ---------------- weight decode (warps 0..15), then epilogue ----------------
        // thread = (tile row r, sub-block hh of the stage's two). Warps whose 32 rows all lie past
        // BN skip the decode (the MMA never reads those rows); a row past N decodes row N - 1
        // instead (it only reaches accumulator columns the epilogue skips), so the loop carries no
        // per-thread condition.
        const uint32_t r = threadIdx.x & 255u, hh = threadIdx.x >> 8;
        const bool live = (r & ~31u) < (uint32_t)BN;  // warp-uniform: BN is a multiple of 32
        const uint32_t row = min(n0 + r, p.N - 1u);
        const uint8_t* qrow = p.qs + (size_t)row * p.nb * QS_BYTES + hh * 8;
        const uint8_t* srow = p.sc + (size_t)row * p.nb * SC_BYTES;
        // this thread's 16-byte chunks of a stage: row r of the SW128 tile, chunk (hh*4 + t) ^ (r%8)
        const uint32_t brow = base_s + G_A_BYTES + (r >> 3) * 1024u + (r & 7u) * 128u +
                              ((((hh * 4u) ^ (r & 7u))) << 4);
        const uint32_t kt_full = p.K / G_BK;  // stages below this one have no K tail
        const uint32_t sel_l = sel_s + (lane & (G_SEL_COPIES - 1)) * 8u;  // this lane's table copy
        // loads run ahead of the decode (the sub-block two stages on, the block scale one block
        // on), clamped to this CTA's last stage and block
        const uint32_t kt_last = kt0 + NKT - 1u, b_last = b1 - 1u;
        auto ld_q = [&](uint32_t kt) {
            return __ldg(reinterpret_cast<const uint2*>(qrow + (size_t)min(kt, kt_last) * 16));
        };
        auto ld_d = [&](uint32_t blk) {
            const uint8_t* e = srow + (size_t)min(blk, b_last) * 2;
            return (uint32_t)e[0] | ((uint32_t)e[1] << 8);
        };
        uint2 q1 = ld_q(kt0), q2 = ld_q(kt0 + 1);
        uint32_t dbits = ld_d(b0), dnext = ld_d(b0 + 1);
        uint32_t s = 0, ph = 0;  // stage slot and the parity of its current use
        for (uint32_t i = 0; i < NKT; ++i) {
            const uint32_t kt = kt0 + i;
            const uint2 q = q1;
            q1 = q2;
            q2 = ld_q(kt + 2);
            if ((kt & 3) == 0 && i > 0) {
                dbits = dnext;
                dnext = ld_d((kt >> 2) + 1);
            }
            if (i >= G_STAGES) {
                // a wait that runs out (only a broken pipeline) stops this warp; the MMA thread
                // then runs out of its own waits and stops too
                bool go = true;
                if (lane == 0) go = mbar_wait(empty(s), ph ^ 1u, p.err, 8u, p.wait_ns);
                go = __shfl_sync(0xFFFFFFFFu, go ? 1 : 0, 0) != 0;  // one decision for the whole warp
                if (!go) {
                    *abort_flag = 1u;
                    break;
                }
            }
            if (live) {
                const float d = half_bits_to_float(dbits);
                const uint32_t dst = brow + s * G_STAGE_BYTES;
                if (kt < kt_full) decode_sub<false>(q, d, sel_l, dst, 0, p.K);
                else decode_sub<true>(q, d, sel_l, dst, kt * G_BK + hh * 32, p.K);
            }
            fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
            __syncwarp();
            if (lane == 0 && i + 1 != p.stall) mbar_arrive(full_b(s));
            if (++s == G_STAGES) {
                s = 0;
                ph ^= 1u;
            }
        }

        // ---------------- epilogue: TMEM -> registers -> global ----------------
        bool ok = true;
        if (lane == 0) ok = mbar_wait(acc_full, 0, p.err, 16u, p.wait_ns) && !*abort_flag;
        ok = __shfl_sync(0xFFFFFFFFu, ok ? 1 : 0, 0) != 0;  // the TMEM loads below are warp-wide
        // accumulator, TMEM lane quadrant (fixed by the warp's rank in its group of 4), column half
        const uint32_t acc = (warp >> 2) & 1, quad = warp & 3, chalf = warp >> 3;
        if (ok && (acc == 0 || upper) && p.tma) {
            // each warp's 32 x 32 tiles leave through TMA stores, staged in two 4 KB buffers of
            // the (now idle) stage ring: row `lane` of a tile in the 128-byte swizzle the tensor
            // map expects (16-byte chunk j at j ^ (lane % 8)), so the stores are whole lines and
            // overlap the next tile's TMEM load
            tc_fence_after();
            const uint32_t lrow0 = acc * 128 + quad * 32, token0 = m0 + lrow0;
            const uint32_t buf0 = base_s + (uint32_t)warp * 8192u;
            int it = 0;
#pragma unroll 1
            for (int c = (int)chalf; c < BN / 32; c += 2, ++it) {
                uint32_t v[32];
                tmem_ld32(tmem + ((quad * 32u) << 16) + acc * 256u + c * 32u, v);
                const uint32_t buf = buf0 + (uint32_t)(it & 1) * 4096u;
                if (it >= 2) {  // the store two tiles back has finished reading this buffer
                    if (lane == 0) bulk_wait_read_1();
                    __syncwarp();
                }
                const uint32_t row = buf + (uint32_t)lane * 128u;
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    st_shared_v4(row + (((uint32_t)j ^ ((uint32_t)lane & 7u)) << 4),
                                 make_uint4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]));
                fence_proxy_async_smem();  // generic-proxy writes -> visible to the TMA engine
                __syncwarp();
                if (lane == 0) {
                    // a tile wholly outside the output stores nothing, but still closes a (then
                    // empty) group, so that "one group back" is always the other buffer's store
                    if (n0 + c * 32 < p.N && token0 < p.M) {
                        if (pu < 0) tma_store_3d(&tmap_out, buf, (int)(n0 + c * 32), (int)token0, 0);
                        else tma_store_3d(&tmap_part, buf, c * 32, (int)lrow0, pu);
                    }
                    bulk_commit();
                }
            }
            if (lane == 0) bulk_wait_all();  // the stores are done before the CTA's memory goes
            __syncwarp();
        } else if (ok && (acc == 0 || upper)) {
            tc_fence_after();
            const uint32_t lrow = acc * 128 + quad * 32 + lane, token = m0 + lrow;
            // the output row, or this unit's partial tile row (columns relative to n0)
            float* orow = pu < 0 ? p.out + (size_t)token * p.N
                                 : p.part + ((size_t)pu * p.PR + lrow) * BN;
            const bool vec = pu >= 0 || p.vec;
#pragma unroll 1
            for (int c = (int)chalf; c < BN / 32; c += 2) {
                uint32_t v[32];
                tmem_ld32(tmem + ((quad * 32u) << 16) + acc * 256u + c * 32u, v);
                if (token < p.M) {
                    const uint32_t nc = n0 + c * 32, oc = pu < 0 ? nc : c * 32u;
                    if (vec && nc + 32 <= p.N) {
#pragma unroll
                        for (int j = 0; j < 32; j += 4)
                            *reinterpret_cast<float4*>(orow + oc + j) =
                                make_float4(__uint_as_float(v[j]), __uint_as_float(v[j + 1]),
                                            __uint_as_float(v[j + 2]), __uint_as_float(v[j + 3]));
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (nc + j < p.N) orow[oc + j] = __uint_as_float(v[j]);
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == G_MMA_WARP) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(G_TMEM_COLS)
                     : "memory");
    }
}

// x (f32 / f16) -> bf16, row-major [M, K] (round to nearest even).
template <typename XT>
__global__ void __launch_bounds__(256) to_bf16_kernel(const XT* __restrict__ x, __nv_bfloat16* __restrict__ y,
                                                      size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        y[i] = __float2bfloat16_rn(to_f32(x[i]));
}

// The split tiles' outputs: out = the sum of each tile's K ranges, in range order (deterministic).
// One thread per 4 columns of a partial tile row.
__global__ void __launch_bounds__(256) splitk_tile_sum_kernel(const float* __restrict__ part, float* __restrict__ out,
                                                              uint32_t M, uint32_t N, uint32_t nt, uint32_t full,
                                                              uint32_t R, uint32_t s, uint32_t BN, uint32_t PR) {
    const uint32_t q = BN / 4;  // column quads per row
    const size_t total = (size_t)R * PR * q;
    for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
        const uint32_t i = (uint32_t)(e / ((size_t)PR * q));
        const uint32_t rem = (uint32_t)(e % ((size_t)PR * q));
        const uint32_t row = rem / q, c4 = (rem % q) * 4;
        const uint32_t t = full + i;
        const uint32_t token = (t / nt) * G_BM + row, n = (t % nt) * BN + c4;
        if (token >= M || n >= N) continue;
        const float4* src = reinterpret_cast<const float4*>(part + (((size_t)i * s) * PR + row) * BN + c4);
        float4 a = src[0];
        for (uint32_t z = 1; z < s; ++z) {
            const float4 b = src[(size_t)z * PR * BN / 4];
            a.x += b.x;
            a.y += b.y;
            a.z += b.z;
            a.w += b.w;
        }
        float* o = out + (size_t)token * N + n;
        o[0] = a.x;
        if (n + 1 < N) o[1] = a.y;
        if (n + 2 < N) o[2] = a.z;
        if (n + 3 < N) o[3] = a.w;
    }
}

// Driver entry point for cuTensorMapEncodeTiled (no link-time dependency on libcuda).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

size_t align256(size_t v) { return (v + 255) / 256 * 256; }

struct GemmPlan {
    uint32_t bn;          // weight rows per tile: 256 or 224
    uint32_t nt, tiles;   // tiles along N, all tiles
    uint32_t full, R, s;  // whole tiles; the split ones after them, and their K ranges
    uint32_t PR;          // rows of a partial tile
};

// Tile width and split. The CTAs (one per SM) run in waves of `sms`; the tiles of the full waves
// are computed whole, and the tiles of the last, part-full wave (all of them when there are
// fewer tiles than SMs) are split into ranges of whole 256-blocks of K, at least two blocks per
// range, so that the last wave fills the SMs and ends after 1/s of a tile's time (plus a fixed
// cost of about 1/20 of one: set-up, the partial tiles' stores, the sum). Of the two tile widths
// the cheaper is taken; a tile's time is nearly independent of its width (the decode of a stage
// takes its warps the same time whether 224 or 256 rows are live), measured on B200 as
// 0.7 + 0.3 * BN / 256 of a 256-wide tile's.
GemmPlan gemm_plan(uint32_t m, uint32_t n, uint32_t k, int num_sms) {
    const uint64_t sms = num_sms > 0 ? (uint64_t)num_sms : 148u;
    const uint64_t mt = (m + G_BM - 1) / G_BM, nb = (k + QK - 1) / QK;
    GemmPlan best{};
    double best_cost = 1e300;
    for (uint32_t bn : {(uint32_t)G_BN, 224u}) {
        GemmPlan pl{};
        pl.bn = bn;
        pl.nt = (n + bn - 1) / bn;
        pl.tiles = (uint32_t)(pl.nt * mt);
        pl.PR = m >= (uint32_t)G_BM ? (uint32_t)G_BM : (m + 31) / 32 * 32;
        const uint64_t T = pl.tiles;
        uint64_t R = T <= sms ? T : T - ((T + sms - 1) / sms - 1) * sms;
        if (R == sms) R = 0;
        uint64_t sp = R ? std::max<uint64_t>(1, std::min<uint64_t>(sms / R, nb / 2)) : 1;
        if (sp <= 1) {
            R = 0;
            sp = 1;
        }
        pl.R = (uint32_t)R;
        pl.s = (uint32_t)sp;
        pl.full = (uint32_t)(T - R);
        const double waves = (double)((pl.full + sms - 1) / sms) + (R ? 1.0 / (double)sp + 0.05 : 0.0);
        const double cost = waves * (0.7 + 0.3 * (double)bn / (double)G_BN);
        if (cost < best_cost - 1e-9) {
            best_cost = cost;
            best = pl;
        }
    }
    return best;
}

// Device address of g_gemm_status on the current device, looked up with cudaGetSymbolAddress once
// per device and context (a new primary context, e.g. after cudaDeviceReset, is looked up again).
std::mutex g_status_mu;
struct StatusSlot {
    void* ctx = nullptr;
    unsigned int* ptr = nullptr;
};
StatusSlot g_status_slot[64];

cudaError_t status_word_for_current_device(unsigned int** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    void* const ctx = current_context_handle();
    std::lock_guard<std::mutex> lock(g_status_mu);
    StatusSlot& slot = g_status_slot[dev];
    if (slot.ptr == nullptr || slot.ctx != ctx) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_gemm_status);
        if (e != cudaSuccess) return e;
        slot.ptr = static_cast<unsigned int*>(p);
        slot.ctx = ctx;
    }
    *out = slot.ptr;
    return cudaSuccess;
}

}  // namespace

int gemm_take_status(unsigned int* status) {
    unsigned int* word = nullptr;
    cudaError_t e = status_word_for_current_device(&word);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(status, word, sizeof(unsigned int), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && *status != 0u) e = cudaMemset(word, 0, sizeof(unsigned int));
    return (int)e;
}

void gemm_testing_set_stall(uint64_t wait_limit_ns, uint32_t stall_stage) {
    g_wait_limit_ns = wait_limit_ns ? wait_limit_ns : WAIT_LIMIT_NS;
    g_stall_stage = stall_stage;
}

bool gemm_path_ok(uint32_t m, uint32_t n, uint32_t k, const void* x, int x_dtype, const uint8_t* qs,
                  const uint8_t* sc, const float* out) {
    (void)sc;
    (void)out;
    (void)n;
    (void)x_dtype;
    // TMA rows must be 16-byte aligned: bf16 x (or its bf16 copy) needs k % 8 == 0
    return m > 16 && k % 8 == 0 && (x_dtype != kDtypeBf16 || reinterpret_cast<uintptr_t>(x) % 16 == 0) &&
           reinterpret_cast<uintptr_t>(qs) % 16 == 0 && encode_fn() != nullptr;
}

size_t gemm_workspace_size(uint32_t m, uint32_t n, uint32_t k, int x_dtype, int num_sms) {
    size_t ws = 256;  // (reserved)
    if (x_dtype != kDtypeBf16) ws += align256((size_t)m * k * 2);  // bf16 copy of x
    const GemmPlan pl = gemm_plan(m, n, k, num_sms);
    if (pl.R) ws += align256((size_t)pl.R * pl.s * pl.PR * pl.bn * sizeof(float));  // partial tiles
    return ws;
}

cudaError_t launch_gemm(const void* x, int x_dtype, uint32_t m, const uint8_t* qs, const uint8_t* sc, uint32_t n,
                        uint32_t k, float* out, void* workspace, int num_sms, cudaStream_t stream) {
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    unsigned int* err = nullptr;
    cudaError_t e = status_word_for_current_device(&err);
    if (e != cudaSuccess) return e;
    const void* xb = x;
    size_t ws_off = 256;
    if (x_dtype != kDtypeBf16) {
        __nv_bfloat16* y = reinterpret_cast<__nv_bfloat16*>(ws + ws_off);
        ws_off += align256((size_t)m * k * 2);
        const size_t total = (size_t)m * k;
        const unsigned blocks = (unsigned)std::min<size_t>((total + 255) / 256, 148 * 16);
        if (x_dtype == 0) to_bf16_kernel<float><<<blocks, 256, 0, stream>>>(static_cast<const float*>(x), y, total);
        else to_bf16_kernel<__half><<<blocks, 256, 0, stream>>>(static_cast<const __half*>(x), y, total);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        xb = y;
    }
    CUtensorMap map;
    const cuuint64_t dims[2] = {k, m};
    const cuuint64_t strides[1] = {(cuuint64_t)k * 2};
    const cuuint32_t box[2] = {G_BK, 128};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(xb), dims, strides, box,
                             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 64 || !attr_set[dev]) {
        e = cudaFuncSetAttribute(gemm_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, G_SMEM);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(gemm_kernel<224>, cudaFuncAttributeMaxDynamicSharedMemorySize, G_SMEM);
        if (e != cudaSuccess) return e;
        if (dev < 64) attr_set[dev] = true;
    }
    GemmParams p;
    p.qs = qs;
    p.sc = sc;
    p.out = out;
    p.err = err;
    p.wait_ns = g_wait_limit_ns;
    p.stall = g_stall_stage;
    p.M = m;
    p.N = n;
    p.K = k;
    p.nb = (k + QK - 1) / QK;
    const GemmPlan pl = gemm_plan(m, n, k, num_sms);
    p.nt = pl.nt;
    p.full = pl.full;
    p.s = pl.s;
    p.PR = pl.PR;
    p.part = pl.R ? reinterpret_cast<float*>(ws + ws_off) : nullptr;
    p.vec = n % 4 == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0;
    // tensor maps of the TMA-store epilogue: the output [1][M][N] and the partial tiles
    // [R*s][PR][BN] (f32, 32x32 boxes, 128-byte swizzle)
    auto encode_out = [&](CUtensorMap* map, void* base, cuuint64_t d0, cuuint64_t d1, cuuint64_t d2) {
        const cuuint64_t dims[3] = {d0, d1, d2};
        const cuuint64_t str[2] = {d0 * 4, d0 * d1 * 4};
        const cuuint32_t box[3] = {32, 32, 1};
        const cuuint32_t es[3] = {1, 1, 1};
        return encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base, dims, str, box, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    };
    CUtensorMap omap, pmap;
    std::memset(&omap, 0, sizeof(omap));
    std::memset(&pmap, 0, sizeof(pmap));
    bool tma = p.vec && encode_out(&omap, out, n, m, 1);
    if (tma && pl.R) tma = encode_out(&pmap, p.part, pl.bn, pl.PR, (cuuint64_t)pl.R * pl.s);
    p.tma = tma ? 1u : 0u;
    const unsigned units = pl.full + pl.R * pl.s;
    if (pl.bn == 224) gemm_kernel<224><<<units, G_THREADS, G_SMEM, stream>>>(map, omap, pmap, p);
    else gemm_kernel<256><<<units, G_THREADS, G_SMEM, stream>>>(map, omap, pmap, p);
    e = cudaGetLastError();
    if (e != cudaSuccess || pl.R == 0) return e;
    const size_t quads = (size_t)pl.R * pl.PR * (pl.bn / 4);
    const int sms = num_sms > 0 ? num_sms : 148;
    const unsigned blocks = (unsigned)std::max<size_t>(1, std::min<size_t>((quads + 255) / 256, (size_t)sms * 8));
    splitk_tile_sum_kernel<<<blocks, 256, 0, stream>>>(p.part, out, m, n, pl.nt, pl.full, pl.R, pl.s, pl.bn, pl.PR);
    return cudaGetLastError();
}

}  // namespace iq2
