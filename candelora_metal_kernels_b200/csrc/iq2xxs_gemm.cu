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
//   * Paired CTAs (m > 256): 2-CTA clusters share one 256-row weight tile across two 256-token
//     tiles with the paired MMA (tcgen05.mma.cta_group::2, M=256): each CTA decodes only its 128
//     rows of the weights, so the decode per MMA is halved (the decode, not the tensor core or
//     the x loads, is what bounds the unpaired kernel).
//   * Pipeline: 3 stages of 64 KB (paired: 4 of 48 KB), mbarriers for "x landed" (TMA transaction
//     bytes), "weights written" (decode warps) and "stage free" (MMA commit). Every wait is
//     bounded: on timeout the kernel records an error code, stops issuing work and still frees its
//     TMEM.
//   * Epilogue: TMEM -> registers -> a 32 x 32 tile in the idle stage ring -> TMA store.
// No TMA multicast is used anywhere (this library also runs on multi-GPU jobs).
#include "iq2xxs_common.cuh"
#include "iq2xxs_codebook.h"
#include "iq2_variant_grids.h"
#include "iq2xxs_internal.h"

#include <cuda.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <type_traits>

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
// Paired CTAs hold half of the weight tile each (128 rows): 48 KB stages, four of them in the same
// shared memory.
constexpr int G_STAGES_PAIR = 4;
constexpr int G_STAGE_BYTES_PAIR = G_A_BYTES + (G_BN / 2) * G_BK * 2;
static_assert(G_STAGES_PAIR * G_STAGE_BYTES_PAIR <= G_STAGES * G_STAGE_BYTES, "paired stages fit the ring");
constexpr uint32_t G_TMEM_COLS = 512;
constexpr uint64_t WAIT_LIMIT_NS = 2000000000ull;  // 2 s: only a broken pipeline waits that long

// Paired CTAs (see gemm_kernel) for m > 256 (0: always unpaired).
#ifndef IQ2_GEMM_PAIR
#define IQ2_GEMM_PAIR 1
#endif
constexpr bool g_pair_enabled = IQ2_GEMM_PAIR != 0;

// Per-device sticky status of the GEMM's bounded waits (the bits of the waits that ran out since
// the last iq2_device_check; 0 = none). Every GPU that loads the library has its own copy.
__device__ unsigned int g_gemm_status;

// Test knobs (iq2_testing_set_gemm_stall): the wait bound, and a stage whose "weights written"
// arrival the decode warps withhold, so that the MMA thread's wait on it runs out.
uint64_t g_wait_limit_ns = WAIT_LIMIT_NS;
uint32_t g_stall_stage = 0;  // 0: none; s > 0: stage s - 1 of every CTA

// Instruction descriptor, kind::f16: F32 accumulate, BF16 A and B, both K-major, M=128, N=BN.
// (MM = 256: the paired form, cta_group::2, each CTA holding 128 of the rows.)
template <int BN, int MM = 128>
constexpr uint32_t idesc_for() {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(MM >> 4) << 24);
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

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t map_peer(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
// An arrival on a barrier of either CTA of the pair (a shared::cluster address), with the default
// (CTA-scope release) semantics: a cluster-scope release would also wait for the thread's loads in
// flight.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void cluster_barrier() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
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
// The paired forms (cta_group::2, issued by the even CTA of a 2-CTA cluster): one MMA of M = 256
// whose A rows (128 per CTA) and B rows (N/2 per CTA) are read from both CTAs' shared memory at the
// same offsets, each CTA's 128 rows of D landing in its own TMEM; a commit that arrives on the
// barrier at this offset in both CTAs (mask 3).
__device__ __forceinline__ void tc_mma_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void tc_commit_pair(uint32_t bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
        "h"((uint16_t)3u)
        : "memory");
}
// TMEM allocation: the whole warp, in both CTAs of a pair for the paired form.
template <bool PAIR>
__device__ __forceinline__ void tmem_alloc(uint32_t dst_word, uint32_t cols) {
    if (PAIR) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_word), "r"(cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    } else {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_word), "r"(cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
}
template <bool PAIR>
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
    if (PAIR)
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
    else
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
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

// Half of decode_sub for the paired kernel: groups 2*half and 2*half + 1 of the sub-block (the
// chunks at dst ^ (t << 4), t = 2*half + tt).
template <bool TAIL>
__device__ __forceinline__ void decode_half(uint2 q, float d, uint32_t sel_l, uint32_t dst, uint32_t half,
                                            uint32_t k_lo, uint32_t K) {
    const uint32_t aux_g = q.x, aux_s = q.y;
    const float dl = d * (float)((aux_s >> 27) | 1u) * 0.125f;  // d*(2s+1)/8, exact
    const uint32_t qlo = cvt_bf16x2(dl * 8.0f, dl * 25.0f);
    const uint32_t qhi = cvt_bf16x2(dl * 43.0f, 0.0f);
#pragma unroll
    for (int tt = 0; tt < 2; ++tt) {
        const uint32_t t = 2 * half + tt;
        const uint32_t gi = (aux_g >> (8 * t)) & 0xFFu, si = (aux_s >> (7 * t)) & 0x7Fu;
        const uint2 sel = ld_shared_v2_const(sel_l + gi * (G_SEL_COPIES * 8));
        const uint32_t S = si | ((__popc(si) & 1u) << 7);
        uint4 w;
        w.x = prmt(qlo, qhi, sel.x) ^ ((S * 0x40008000u) & 0x80008000u);
        w.y = prmt(qlo, qhi, sel.x >> 16) ^ ((S * 0x10002000u) & 0x80008000u);
        w.z = prmt(qlo, qhi, sel.y) ^ ((S * 0x04000800u) & 0x80008000u);
        w.w = prmt(qlo, qhi, sel.y >> 16) ^ ((S * 0x01000200u) & 0x80008000u);
        if (TAIL && k_lo + t * 8 + 8 > K) {
            const uint32_t k0 = k_lo + t * 8;
            const uint32_t keep = k0 >= K ? 0u : K - k0;
            w.x = keep >= 2 ? w.x : (keep == 1 ? (w.x & 0xFFFFu) : 0u);
            w.y = keep >= 4 ? w.y : (keep == 3 ? (w.y & 0xFFFFu) : 0u);
            w.z = keep >= 6 ? w.z : (keep == 5 ? (w.z & 0xFFFFu) : 0u);
            w.w = keep >= 8 ? w.w : (keep == 7 ? (w.w & 0xFFFFu) : 0u);
        }
        st_shared_v4(dst ^ (t << 4), w);
    }
}

// ---- the other formats (IQ2_XS, IQ2_S, IQ3_S) ----
// Split-layout geometry per 256-weight block (weight bytes QB, scale bytes SB; reference
// src/iq2_matmul.rs:15-29) and the decode table: E entries of ENT bytes, C interleaved copies
// (E * ENT * C = the table's TBL bytes), copy `lane % C` for each lane. The paired kernel of the
// other formats has three 48 KB stages and a 64 KB table (16 / 8 / 8 copies: the lookups of a
// half-warp bank-conflict less); everything else four paired or three unpaired stages and 32 KB.
template <int V, bool PAIR = false>
struct GFmt {
    static constexpr uint32_t TBL = (PAIR && V != 0) ? 2u * (uint32_t)G_SEL_BYTES : (uint32_t)G_SEL_BYTES;
    static constexpr int STAGES = PAIR ? (V == 0 ? G_STAGES_PAIR : 3) : G_STAGES;
    static constexpr uint32_t QB = V == 2 ? 72u : (V == 3 ? 104u : 64u);
    static constexpr uint32_t SB = V == 0 ? 2u : (V == 3 ? 6u : 10u);
    static constexpr uint32_t ENT = V == 3 ? 16u : 8u;
    static constexpr uint32_t E = V == 0 ? 256u : (V == 2 ? 1024u : 512u);
    static constexpr uint32_t C = TBL / (E * ENT);
    static_assert(C >= 1 && (C & (C - 1)) == 0, "copies");
};

// Table entry of a {8, 25, 43} grid word (IQ2_XS, IQ2_S): per pair p of weights (2p, 2p+1) the
// 16-bit prmt selector picking bf16(g * dl) out of {qlo, qhi} (magnitude code c: bytes 2c, 2c+1),
// the same layout as IQ2XXS_BF16_SEL.
__device__ __forceinline__ uint2 sel_from_grid8(uint64_t g) {
    uint32_t w[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        const uint32_t b0 = (uint32_t)(g >> (16 * p)) & 0xFFu, b1 = (uint32_t)(g >> (16 * p + 8)) & 0xFFu;
        const uint32_t c0 = b0 == 8u ? 0u : (b0 == 25u ? 1u : 2u), c1 = b1 == 8u ? 0u : (b1 == 25u ? 1u : 2u);
        w[p] = (2u * c0) | ((2u * c0 + 1u) << 4) | ((2u * c1) << 8) | ((2u * c1 + 1u) << 12);
    }
    return make_uint2(w[0] | (w[1] << 16), w[2] | (w[3] << 16));
}

// IQ3_S table entry of a grid word (four magnitudes v in {1, 3, ..., 15}, code k = (v - 1) / 2):
// x = the prmt selectors of pairs (0,1) and (2,3) into {c0, c1} or {c2, c3} (code k & 3: bytes
// 2(k & 3), 2(k & 3) + 1), y / z = the halves of pairs (0,1) / (2,3) that take the high set (k >= 4).
__device__ __forceinline__ uint4 sel_from_grid3s(uint32_t g) {
    uint32_t sel = 0, m[2] = {0u, 0u};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t k = ((g >> (8 * j)) & 0xFFu) >> 1, kk = k & 3u;
        sel |= ((2u * kk) | ((2u * kk + 1u) << 4)) << (8 * j);
        if (k >= 4u) m[j >> 1] |= 0xFFFFu << (16 * (j & 1));
    }
    return make_uint4(sel, m[0], m[1], 0u);
}

// The raw bytes of one 32-weight sub-block ib of one row (qblk / sblk: the row's block), loaded
// two stages ahead of their decode:
//   IQ2_XS: x, y = the four u16 words (9-bit grid index | 7-bit sign index << 9); w = scale byte
//   IQ2_S:  x = the four grid low bytes, y = the four sign bytes; w = qh byte | scale byte << 8
//   IQ3_S:  x, y = the eight grid low bytes (two per 8 weights), z = the four sign bytes;
//           w = qh byte | this sub-block's scale nibble << 8
template <int V>
__device__ __forceinline__ uint4 ld_raw(const uint8_t* qblk, const uint8_t* sblk, uint32_t ib) {
    if (V == 1) {
        const uint2 q = __ldg(reinterpret_cast<const uint2*>(qblk + ib * 8));
        return make_uint4(q.x, q.y, 0u, (uint32_t)__ldg(sblk + 2 + ib));
    } else if (V == 2) {
        const uint32_t lo = __ldg(reinterpret_cast<const uint32_t*>(qblk + ib * 4));
        const uint32_t sg = __ldg(reinterpret_cast<const uint32_t*>(qblk + 32 + ib * 4));
        return make_uint4(lo, sg, 0u, (uint32_t)__ldg(qblk + 64 + ib) | ((uint32_t)__ldg(sblk + 2 + ib) << 8));
    } else {
        const uint2 lo = __ldg(reinterpret_cast<const uint2*>(qblk + ib * 8));
        const uint32_t sg = __ldg(reinterpret_cast<const uint32_t*>(qblk + 72 + ib * 4));
        const uint32_t nib = ((uint32_t)__ldg(sblk + 2 + ib / 2) >> (4 * (ib & 1))) & 15u;
        return make_uint4(lo.x, lo.y, sg, (uint32_t)__ldg(qblk + 64 + ib) | (nib << 8));
    }
}

// Groups t0 .. t0 + NG - 1 (8 weights each) of a sub-block of format V to bf16, stored as 16-byte
// chunks at dst ^ (t << 4) like decode_sub. Each weight is bf16 of its exact value dl * g * sign
// (dl * g has at most 22 significant bits): the candidate products are rounded once and `prmt`
// picks them by grid code; an XOR applies the signs. TAIL: zero the weights at k >= K.
template <int V, int NG, bool TAIL, bool PAIR>
__device__ __forceinline__ void decode_v(uint4 raw, float d, uint32_t sel_l, uint32_t dst, uint32_t t0,
                                         uint32_t k_lo, uint32_t K) {
    constexpr uint32_t STRIDE = GFmt<V, PAIR>::C * GFmt<V, PAIR>::ENT;  // bytes between table entries
    uint32_t ca = 0, cb = 0, cc = 0, cdd = 0;  // the rounded candidates (IQ3_S: all four; else qlo, qhi)
    uint32_t cur_nib = 0xFFFFFFFFu;
#pragma unroll
    for (int tt = 0; tt < NG; ++tt) {
        const uint32_t t = t0 + tt;
        uint32_t S;  // the 8 sign bits of the group (bit j: weight j negative)
        uint4 w;
        if (V == 3) {
            if (tt == 0) {
                const float dl = d * (float)(1u + 2u * (raw.w >> 8));  // d(1+2s), exact
                ca = cvt_bf16x2(dl * 1.0f, dl * 3.0f);
                cb = cvt_bf16x2(dl * 5.0f, dl * 7.0f);
                cc = cvt_bf16x2(dl * 9.0f, dl * 11.0f);
                cdd = cvt_bf16x2(dl * 13.0f, dl * 15.0f);
            }
            const uint32_t lo = ((t < 2 ? raw.x : raw.y) >> (16 * (t & 1))) & 0xFFFFu;
            const uint32_t i1 = (lo & 0xFFu) | (((raw.w >> (2 * t)) & 1u) << 8);
            const uint32_t i2 = (lo >> 8) | (((raw.w >> (2 * t + 1)) & 1u) << 8);
            const uint4 e1 = ld_shared_v4_const(sel_l + i1 * STRIDE);
            const uint4 e2 = ld_shared_v4_const(sel_l + i2 * STRIDE);
            S = (raw.z >> (8 * t)) & 0xFFu;
            auto pick = [&](uint32_t sel, uint32_t m) {
                const uint32_t a = prmt(ca, cb, sel), b = prmt(cc, cdd, sel);
                return (a & ~m) | (b & m);
            };
            w.x = pick(e1.x, e1.y);
            w.y = pick(e1.x >> 16, e1.z);
            w.z = pick(e2.x, e2.y);
            w.w = pick(e2.x >> 16, e2.z);
        } else {
            uint32_t gi, nib;
            if (V == 1) {
                const uint32_t word = ((t < 2 ? raw.x : raw.y) >> (16 * (t & 1))) & 0xFFFFu;
                gi = word & 0x1FFu;
                const uint32_t si = word >> 9;
                S = si | ((__popc(si) & 1u) << 7);  // ksigns: the 8th sign makes the parity even
                nib = (raw.w >> (4 * (t >> 1))) & 15u;
            } else {
                gi = ((raw.x >> (8 * t)) & 0xFFu) | (((raw.w >> (2 * t)) & 3u) << 8);
                S = (raw.y >> (8 * t)) & 0xFFu;
                nib = (raw.w >> (8 + 4 * (t >> 1))) & 15u;
            }
            if (nib != cur_nib) {  // (uniform per pair of groups: the scale nibble covers 16 weights)
                cur_nib = nib;
                const float dl = d * (float)(2u * nib + 1u) * 0.125f;  // d(0.5+s)/4, exact
                ca = cvt_bf16x2(dl * 8.0f, dl * 25.0f);
                cb = cvt_bf16x2(dl * 43.0f, 0.0f);
            }
            const uint2 sel = ld_shared_v2_const(sel_l + gi * STRIDE);
            w.x = prmt(ca, cb, sel.x);
            w.y = prmt(ca, cb, sel.x >> 16);
            w.z = prmt(ca, cb, sel.y);
            w.w = prmt(ca, cb, sel.y >> 16);
        }
        w.x ^= (S * 0x40008000u) & 0x80008000u;
        w.y ^= (S * 0x10002000u) & 0x80008000u;
        w.z ^= (S * 0x04000800u) & 0x80008000u;
        w.w ^= (S * 0x01000200u) & 0x80008000u;
        if (TAIL && k_lo + t * 8 + 8 > K) {
            const uint32_t k0 = k_lo + t * 8;
            const uint32_t keep = k0 >= K ? 0u : K - k0;
            w.x = keep >= 2 ? w.x : (keep == 1 ? (w.x & 0xFFFFu) : 0u);
            w.y = keep >= 4 ? w.y : (keep == 3 ? (w.y & 0xFFFFu) : 0u);
            w.z = keep >= 6 ? w.z : (keep == 5 ? (w.z & 0xFFFFu) : 0u);
            w.w = keep >= 8 ? w.w : (keep == 7 ? (w.w & 0xFFFFu) : 0u);
        }
        st_shared_v4(dst ^ (t << 4), w);
    }
}

// ---- the kernel ----
// BN: weight rows per CTA (256, or 224 where that fills the last wave better); the stage
// layout is always sized for 256 rows.
// PAIR: 2-CTA clusters on one 256-row weight tile and two consecutive 256-token tiles (CTA rank r
// takes token tile 2j + r), with the paired tensor-core form (cta_group::2): CTA r decodes weight
// rows [128r, 128r + 128) of the tile into its own stage, and the even CTA's MMAs (M = 256: its
// own 128 tokens of a half and the odd CTA's) read both halves of the weights from the two CTAs'
// shared memory. Every weight is decoded once per 512 tokens instead of once per 256, with no
// shared-memory traffic between the CTAs. The even CTA's `full_b` counts the decode warps of both
// CTAs plus one arrival from the odd CTA's idle MMA warp, which relays that the odd CTA's x tile
// has landed (each CTA's x loads complete on its own `full_a`, so that an aborted CTA can still
// wait for its own loads). The even CTA's commits arrive on both CTAs' `empty` and `acc_full`. No
// TMA multicast.
// V: the weight format (0 IQ2_XXS, 1 IQ2_XS, 2 IQ2_S, 3 IQ3_S); only the decode table and the
// decode differ.
template <int BN, bool PAIR, int V = 0>
__global__ void __launch_bounds__(G_THREADS, 1) gemm_kernel(const __grid_constant__ CUtensorMap tmap_x,
                                                            const __grid_constant__ CUtensorMap tmap_out,
                                                            const __grid_constant__ CUtensorMap tmap_part,
                                                            const GemmParams p) {
    static_assert(BN % 32 == 0 && BN <= G_BN, "BN");
    static_assert(!PAIR || BN == G_BN, "paired CTAs split a 256-row tile");
    using F = GFmt<V, PAIR>;
    constexpr int S = F::STAGES;                                        // stages in the ring
    constexpr uint32_t SB = PAIR ? G_STAGE_BYTES_PAIR : G_STAGE_BYTES;  // bytes per stage
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_s = smem_u32(smem_raw);
    const uint32_t base_s = (raw_s + 1023u) & ~1023u;  // SW128 tiles need 1024-byte alignment
    uint8_t* base = smem_raw + (base_s - raw_s);
    const uint32_t sel_s = base_s + S * SB;
    const uint32_t bar_s = sel_s + F::TBL;
    static_assert(1024 + S * SB + F::TBL + 256 <= (uint32_t)G_SMEM, "shared memory");
    // barriers: full_a[S], full_b[S], empty[S], acc_full; then the TMEM address word; abort flag
    auto full_a = [&](int s) { return bar_s + 8u * s; };
    auto full_b = [&](int s) { return bar_s + 8u * (S + s); };
    auto empty = [&](int s) { return bar_s + 8u * (2 * S + s); };
    const uint32_t acc_full = bar_s + 8u * (3 * S);
    uint32_t* tmem_addr_word = reinterpret_cast<uint32_t*>(base + (bar_s - base_s) + 8 * (3 * S + 1));
    volatile uint32_t* abort_flag = tmem_addr_word + 1;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // The split tiles' sum kernel (launched as a programmatic dependent) may be scheduled now: it
    // waits for this grid to complete before it reads anything. (Kernels of this library that
    // read before their own wait only read weights, which this kernel never writes.)
    pdl_launch_dependents();
    // this CTA's unit: tile t, K range z of nz; pu = its partial tile (-1: the tile is whole).
    // PAIR: units are pairs (cluster = blockIdx.x / 2, rank = the CTA's rank in it); tile t is a
    // pair tile (n-tile t % nt, token tiles 2 * (t / nt) + rank), partial tile (2 * (t - full) +
    // rank) * s + z.
    const uint32_t rank = PAIR ? cluster_ctarank() : 0u, unit = PAIR ? blockIdx.x >> 1 : blockIdx.x;
    const bool leader = rank == 0;  // (always, unpaired)
    uint32_t t, z, nz;
    int pu;
    if (unit < p.full) {
        t = unit;
        z = 0;
        nz = 1;
        pu = -1;
    } else {
        const uint32_t v = unit - p.full;
        t = p.full + v / p.s;
        z = v % p.s;
        nz = p.s;
        pu = PAIR ? (int)((2 * (v / p.s) + rank) * p.s + z) : (int)v;
    }
    const uint32_t n0 = (t % p.nt) * BN, m0 = (PAIR ? 2 * (t / p.nt) + rank : t / p.nt) * G_BM;
    // this CTA's share of K: the 256-blocks [b0, b1) of range z, i.e. the 64-k stages
    // [kt0, kt0 + NKT) (at least one: the host never makes more ranges than blocks)
    const uint32_t b0 = (uint32_t)((uint64_t)z * p.nb / nz);
    const uint32_t b1 = (uint32_t)((uint64_t)(z + 1) * p.nb / nz);
    const uint32_t kt0 = b0 * (QK / G_BK);
    const uint32_t NKT = min(b1 * (QK / G_BK), (p.K + G_BK - 1) / G_BK) - kt0;
    const bool upper = m0 + 128 < p.M;  // this CTA's second 128-token half holds tokens
    // the second MMA (second halves) runs when the first token tile's second half holds tokens
    // (PAIR: the even CTA's; the odd CTA then loads its second half too, zeros past M)
    const bool upper_mma = (PAIR ? m0 - rank * G_BM : m0) + 128 < p.M;

    // decode table -> shared memory: per grid entry the four 16-bit prmt selectors packed in two
    // words (IQ3_S: GFmt<3>'s 16-byte entries), C times (copy c of entry e at (e * C + c) * ENT)
    for (int i = threadIdx.x; i < (int)(F::E * F::C); i += blockDim.x) {
        const uint32_t e = (uint32_t)i / F::C;
        if constexpr (V == 0) {
            const uint32_t* w = IQ2XXS_BF16_SEL[e];
            reinterpret_cast<uint2*>(base + (sel_s - base_s))[i] = make_uint2(w[0] | (w[1] << 16), w[2] | (w[3] << 16));
        } else if constexpr (V == 3) {
            reinterpret_cast<uint4*>(base + (sel_s - base_s))[i] = sel_from_grid3s(IQ3S_GRID[e]);
        } else {
            reinterpret_cast<uint2*>(base + (sel_s - base_s))[i] = sel_from_grid8(V == 1 ? IQ2XS_GRID[e] : IQ2S_GRID[e]);
        }
    }
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(full_a(s), 1);
            // the decode warps (PAIR: both CTAs', plus the odd CTA's relay; only the even CTA's is used)
            mbar_init(full_b(s), PAIR ? 2 * G_DEC_WARPS + 1 : G_DEC_WARPS);
            mbar_init(empty(s), 1);
        }
        mbar_init(acc_full, 1);
        *abort_flag = 0u;
        fence_barrier_init();
    }
    if (warp == G_MMA_WARP) tmem_alloc<PAIR>(smem_u32(tmem_addr_word), G_TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    if (PAIR) cluster_barrier();  // the peer's barriers are initialised before anything reaches them
    tc_fence_after();
    const uint32_t tmem = *tmem_addr_word;
    // the even CTA's `full_b` (shared::cluster addresses), where the odd CTA's arrivals go
    const uint32_t full_b_lead0 = PAIR ? map_peer(full_b(0), 0u) : 0u;

    if (warp == G_TMA_WARP) {
        // ---------------- x producer ----------------
        if (lane == 0) {
            uint32_t issued = 0;
            bool aborted = false;
            for (uint32_t i = 0; i < NKT; ++i) {
                const int s = i % S;
                if (i >= (uint32_t)S && !mbar_wait(empty(s), ((i / S) - 1) & 1, p.err, 1u, p.wait_ns)) {
                    *abort_flag = 1u;
                    aborted = true;
                    break;
                }
                if (*abort_flag) {
                    aborted = true;
                    break;
                }
                const uint32_t a_s = base_s + s * SB;
                const int kx = (int)((kt0 + i) * G_BK);
                mbar_expect_tx(full_a(s), upper_mma ? G_A_BYTES : G_A_HALF);
                tma_load_2d(a_s, &tmap_x, full_a(s), kx, (int)m0);
                if (upper_mma) tma_load_2d(a_s + G_A_HALF, &tmap_x, full_a(s), kx, (int)(m0 + 128));
                ++issued;
            }
            // after an abort, the loads already issued (at most one per stage slot, each the last
            // use of its slot) land before the CTA's shared memory goes away (bounded as well)
            if (aborted)
                for (uint32_t j = issued > (uint32_t)S ? issued - S : 0u; j < issued; ++j)
                    mbar_wait(full_a(j % S), (j / S) & 1u, p.err, 32u, p.wait_ns);
        }
    } else if (warp == G_MMA_WARP) {
        if (lane == 0 && leader) {
            // ---------------- MMA issuer ----------------
            bool ok = true;
            for (uint32_t i = 0; i < NKT && ok; ++i) {
                const int s = i % S;
                const uint32_t ph = (i / S) & 1;
                ok = mbar_wait(full_a(s), ph, p.err, 2u, p.wait_ns) && mbar_wait(full_b(s), ph, p.err, 4u, p.wait_ns);
                if (!ok || *abort_flag) {
                    *abort_flag = 1u;
                    break;
                }
                tc_fence_after();
                const uint32_t a_s = base_s + s * SB, b_s = a_s + G_A_BYTES;
#pragma unroll
                for (int ks = 0; ks < G_BK / 16; ++ks) {
                    const uint64_t bd = sw128_desc(b_s + ks * 32);
                    const uint32_t acc = (i | ks) ? 1u : 0u;
                    if (PAIR) {
                        tc_mma_pair(tmem, sw128_desc(a_s + ks * 32), bd, idesc_for<BN, 256>(), acc);
                        if (upper_mma)
                            tc_mma_pair(tmem + 256, sw128_desc(a_s + G_A_HALF + ks * 32), bd, idesc_for<BN, 256>(),
                                        acc);
                    } else {
                        tc_mma(tmem, sw128_desc(a_s + ks * 32), bd, idesc_for<BN>(), acc);
                        if (upper_mma)
                            tc_mma(tmem + 256, sw128_desc(a_s + G_A_HALF + ks * 32), bd, idesc_for<BN>(), acc);
                    }
                }
                // the stage is free once these MMAs have read it (PAIR: in both CTAs)
                if (PAIR) tc_commit_pair(empty(s));
                else tc_commit(empty(s));
            }
            // fires when every MMA issued above has completed
            if (PAIR) tc_commit_pair(acc_full);
            else tc_commit(acc_full);
        } else if (lane == 0 && PAIR) {
            // ---------------- the odd CTA: relay "x landed" to the even CTA ----------------
            for (uint32_t i = 0; i < NKT; ++i) {
                const int s = i % S;
                if (!mbar_wait(full_a(s), (i / S) & 1, p.err, 2u, p.wait_ns) || *abort_flag) {
                    *abort_flag = 1u;
                    break;
                }
                mbar_arrive_cluster(full_b_lead0 + 8u * s);
            }
        }
    } else {
        // ---------------- weight decode (warps 0..15), then epilogue ----------------
        // thread = (tile row r, sub-block hh of the stage's two). Warps whose 32 rows all lie past
        // BN skip the decode (the MMA never reads those rows); a row past N decodes row N - 1
        // instead (it only reaches accumulator columns the epilogue skips), so the loop carries no
        // per-thread condition.
        // PAIR: thread = (row r of this CTA's 128, sub-block hh, half `ghalf` of its four groups);
        // the weight row is n0 + 128 * rank + r.
        const uint32_t r = PAIR ? (threadIdx.x & 127u) : threadIdx.x & 255u;
        const uint32_t hh = PAIR ? (threadIdx.x >> 8) & 1u : threadIdx.x >> 8;
        const uint32_t ghalf = (threadIdx.x >> 7) & 1u;  // (PAIR only)
        const bool live = (r & ~31u) < (uint32_t)BN;  // warp-uniform: BN is a multiple of 32
        const uint32_t row = min(n0 + (PAIR ? 128u * rank : 0u) + r, p.N - 1u);
        // (IQ2_XXS: the row's sub-block hh of each stage; the others: the row's first block)
        const uint8_t* qrow = p.qs + (size_t)row * p.nb * GFmt<V>::QB + (V == 0 ? hh * 8 : 0u);
        const uint8_t* srow = p.sc + (size_t)row * p.nb * GFmt<V>::SB;
        // this thread's 16-byte chunks of a stage: row r of the SW128 tile, chunk (hh*4 + t) ^ (r%8)
        const uint32_t brow = base_s + G_A_BYTES + (r >> 3) * 1024u + (r & 7u) * 128u +
                              ((((hh * 4u) ^ (r & 7u))) << 4);
        const uint32_t kt_full = p.K / G_BK;  // stages below this one have no K tail
        const uint32_t sel_l = sel_s + (lane & (F::C - 1)) * F::ENT;  // this lane's table copy
        // loads run ahead of the decode (the sub-block two stages on, the block scale one block
        // on), clamped to this CTA's last stage and block
        const uint32_t kt_last = kt0 + NKT - 1u, b_last = b1 - 1u;
        using Raw = typename std::conditional<V == 0, uint2, uint4>::type;
        auto ld_q = [&](uint32_t kt) -> Raw {
            const uint32_t kc = min(kt, kt_last);
            if constexpr (V == 0) return __ldg(reinterpret_cast<const uint2*>(qrow + (size_t)kc * 16));
            else
                return ld_raw<V>(qrow + (size_t)(kc >> 2) * GFmt<V>::QB, srow + (size_t)(kc >> 2) * GFmt<V>::SB,
                                 (kc & 3u) * 2u + hh);
        };
        auto ld_d = [&](uint32_t blk) {
            const uint8_t* e = srow + (size_t)min(blk, b_last) * GFmt<V>::SB;
            return (uint32_t)e[0] | ((uint32_t)e[1] << 8);
        };
        Raw q1 = ld_q(kt0), q2 = ld_q(kt0 + 1);
        uint32_t dbits = ld_d(b0), dnext = ld_d(b0 + 1);
        uint32_t s = 0, ph = 0;  // stage slot and the parity of its current use
        for (uint32_t i = 0; i < NKT; ++i) {
            const uint32_t kt = kt0 + i;
            const Raw q = q1;
            q1 = q2;
            q2 = ld_q(kt + 2);
            if ((kt & 3) == 0 && i > 0) {
                dbits = dnext;
                dnext = ld_d((kt >> 2) + 1);
            }
            if (i >= (uint32_t)S) {
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
            const float d = half_bits_to_float(dbits);
            const uint32_t dst = brow + s * SB;
            if constexpr (V != 0) {
                constexpr int NG = PAIR ? 2 : 4;  // groups per thread
                const uint32_t t0 = PAIR ? 2u * ghalf : 0u;
                if (PAIR || live) {
                    if (kt < kt_full) decode_v<V, NG, false, PAIR>(q, d, sel_l, dst, t0, 0, p.K);
                    else decode_v<V, NG, true, PAIR>(q, d, sel_l, dst, t0, kt * G_BK + hh * 32, p.K);
                }
            } else if (PAIR) {
                if (kt < kt_full) decode_half<false>(q, d, sel_l, dst, ghalf, 0, p.K);
                else decode_half<true>(q, d, sel_l, dst, ghalf, kt * G_BK + hh * 32, p.K);
            } else if (live) {
                if (kt < kt_full) decode_sub<false>(q, d, sel_l, dst, 0, p.K);
                else decode_sub<true>(q, d, sel_l, dst, kt * G_BK + hh * 32, p.K);
            }
            fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
            __syncwarp();
            if (lane == 0 && i + 1 != p.stall) {
                if (PAIR) mbar_arrive_cluster(full_b_lead0 + 8u * s);  // (the even CTA's barrier)
                else mbar_arrive(full_b(s));
            }
            if (++s == (uint32_t)S) {
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
    // PAIR: neither CTA frees its TMEM (a pair allocation) or leaves while the other may still
    // arrive on its barriers or have MMAs reading its shared memory
    if (PAIR) cluster_barrier();
    if (warp == G_MMA_WARP) tmem_dealloc<PAIR>(tmem, G_TMEM_COLS);
}

// x (f32 / f16) -> bf16, row-major [M, K] (round to nearest even).
template <typename XT>
__global__ void __launch_bounds__(256) to_bf16_kernel(const XT* __restrict__ x, __nv_bfloat16* __restrict__ y,
                                                      size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        y[i] = __float2bfloat16_rn(to_f32(x[i]));
}

// The split tiles' outputs: out = the sum of each tile's K ranges, in range order (deterministic).
// One thread per 4 columns of a partial tile row; the ranges' loads are issued four at a time.
// R: split tiles (PAIR: split pair tiles, 2R partial tiles, tile i = pair i / 2, rank i % 2).
// Launched as a programmatic dependent of the GEMM: its blocks may become resident while the GEMM
// runs and wait here until it has completed and its partial tiles are visible.
__global__ void __launch_bounds__(256) splitk_tile_sum_kernel(const float* __restrict__ part, float* __restrict__ out,
                                                              uint32_t M, uint32_t N, uint32_t nt, uint32_t full,
                                                              uint32_t R, uint32_t s, uint32_t BN, uint32_t PR,
                                                              uint32_t pair) {
    pdl_wait();
    const uint32_t q = BN / 4;  // column quads per row
    const size_t total = (size_t)(pair ? 2 * R : R) * PR * q;
    for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
        const uint32_t i = (uint32_t)(e / ((size_t)PR * q));
        const uint32_t rem = (uint32_t)(e % ((size_t)PR * q));
        const uint32_t row = rem / q, c4 = (rem % q) * 4;
        const uint32_t t = full + (pair ? i >> 1 : i);
        const uint32_t mtile = pair ? 2 * (t / nt) + (i & 1u) : t / nt;
        const uint32_t token = mtile * G_BM + row, n = (t % nt) * BN + c4;
        if (token >= M || n >= N) continue;
        const float4* src = reinterpret_cast<const float4*>(part + (((size_t)i * s) * PR + row) * BN + c4);
        const size_t zs = (size_t)PR * BN / 4;  // float4s between ranges
        float4 a = src[0];
        for (uint32_t z0 = 1; z0 < s; z0 += 4) {
            float4 b[4];
#pragma unroll
            for (uint32_t j = 0; j < 4; ++j)
                if (z0 + j < s) b[j] = src[(z0 + j) * zs];
#pragma unroll
            for (uint32_t j = 0; j < 4; ++j)
                if (z0 + j < s) {
                    a.x += b[j].x;
                    a.y += b[j].y;
                    a.z += b[j].z;
                    a.w += b[j].w;
                }
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
    bool pair;            // 2-CTA clusters sharing each weight tile (units and R count pairs)
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
    if (mt >= 2 && g_pair_enabled) {
        // two token tiles per weight tile, one decode for both: units are pair tiles, a wave is
        // sms / 2 of them; the split of the last wave as below
        GemmPlan pl{};
        pl.pair = true;
        pl.bn = G_BN;
        pl.nt = (n + G_BN - 1) / G_BN;
        pl.tiles = (uint32_t)(pl.nt * ((mt + 1) / 2));
        pl.PR = G_BM;
        const uint64_t slots = std::max<uint64_t>(1, sms / 2), T = pl.tiles;
        uint64_t R = T <= slots ? T : T - ((T + slots - 1) / slots - 1) * slots;
        if (R == slots) R = 0;
        uint64_t sp = R ? std::max<uint64_t>(1, std::min<uint64_t>(slots / R, nb / 2)) : 1;
        if (sp <= 1) {
            R = 0;
            sp = 1;
        }
        pl.R = (uint32_t)R;
        pl.s = (uint32_t)sp;
        pl.full = (uint32_t)(T - R);
        return pl;
    }
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
    if (pl.R) ws += align256((size_t)(pl.pair ? 2 : 1) * pl.R * pl.s * pl.PR * pl.bn * sizeof(float));  // partial tiles
    return ws;
}

namespace {
// The three launch forms of format V: paired (one 2-CTA cluster per unit), or one CTA per unit
// with 256- or 224-row tiles.
template <int V>
cudaError_t set_attributes_v() {
    cudaError_t e = cudaFuncSetAttribute(gemm_kernel<256, false, V>, cudaFuncAttributeMaxDynamicSharedMemorySize, G_SMEM);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(gemm_kernel<224, false, V>, cudaFuncAttributeMaxDynamicSharedMemorySize, G_SMEM);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(gemm_kernel<256, true, V>, cudaFuncAttributeMaxDynamicSharedMemorySize, G_SMEM);
    return e;
}

template <int V>
cudaError_t launch_forms(const GemmPlan& pl, unsigned units, const CUtensorMap& map, const CUtensorMap& omap,
                         const CUtensorMap& pmap, const GemmParams& p, cudaStream_t stream) {
    if (pl.pair) {
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * units);
        cfg.blockDim = dim3(G_THREADS);
        cfg.dynamicSmemBytes = G_SMEM;
        cfg.stream = stream;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        return cudaLaunchKernelEx(&cfg, gemm_kernel<256, true, V>, map, omap, pmap, p);
    }
    if (pl.bn == 224) gemm_kernel<224, false, V><<<units, G_THREADS, G_SMEM, stream>>>(map, omap, pmap, p);
    else gemm_kernel<256, false, V><<<units, G_THREADS, G_SMEM, stream>>>(map, omap, pmap, p);
    return cudaGetLastError();
}
}  // namespace

cudaError_t launch_gemm(const void* x, int x_dtype, uint32_t m, const uint8_t* qs, const uint8_t* sc, uint32_t n,
                        uint32_t k, float* out, void* workspace, int num_sms, cudaStream_t stream, int variant) {
    if (variant < 0 || variant > 3) return cudaErrorInvalidValue;
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
        e = set_attributes_v<0>();
        if (e == cudaSuccess) e = set_attributes_v<1>();
        if (e == cudaSuccess) e = set_attributes_v<2>();
        if (e == cudaSuccess) e = set_attributes_v<3>();
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
    const uint32_t ptiles = (pl.pair ? 2u : 1u) * pl.R;  // partial tiles (each split s ways)
    if (tma && pl.R) tma = encode_out(&pmap, p.part, pl.bn, pl.PR, (cuuint64_t)ptiles * pl.s);
    p.tma = tma ? 1u : 0u;
    const unsigned units = pl.full + pl.R * pl.s;
    switch (variant) {
        case 0: e = launch_forms<0>(pl, units, map, omap, pmap, p, stream); break;
        case 1: e = launch_forms<1>(pl, units, map, omap, pmap, p, stream); break;
        case 2: e = launch_forms<2>(pl, units, map, omap, pmap, p, stream); break;
        default: e = launch_forms<3>(pl, units, map, omap, pmap, p, stream); break;
    }
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess || pl.R == 0) return e;
    const size_t quads = (size_t)ptiles * pl.PR * (pl.bn / 4);
    const int sms = num_sms > 0 ? num_sms : 148;
    const unsigned blocks = (unsigned)std::max<size_t>(1, std::min<size_t>((quads + 255) / 256, (size_t)sms * 8));
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(blocks);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, splitk_tile_sum_kernel, static_cast<const float*>(p.part), out, m, n, pl.nt,
                           pl.full, pl.R, pl.s, pl.bn, pl.PR, pl.pair ? 1u : 0u);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

}  // namespace iq2
