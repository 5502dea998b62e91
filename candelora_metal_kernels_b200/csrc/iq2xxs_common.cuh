// Shared device helpers for the IQ2_XXS kernels (sm_100a).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

namespace iq2 {

// IQ2_XXS geometry (reference src/iq2_matmul.rs:12-17): 256 weights per block, 64 bytes of
// `qs` (8 sub-blocks of 32 weights, 8 bytes each) and a 2-byte fp16 `d` per block.
constexpr int QK = 256;
constexpr int QS_BYTES = 64;
constexpr int SC_BYTES = 2;

// Signed int8 weight magnitudes {+8, +25, +43, 0} and {-8, -25, -43, 0}: the byte pair a
// `prmt` with IQ2XXS_GRID_SEL | IQ2XXS_SIGN_SEL selectors picks weights from.
constexpr uint32_t KPOS = 0x002B1908u;
constexpr uint32_t KNEG = 0x00D5E7F8u;

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Shared/global loads are plain C++ accesses so the compiler orders them with barriers and
// is free to schedule them.
__device__ __forceinline__ uint32_t lds32(const uint8_t* base, uint32_t off) {
    return *reinterpret_cast<const uint32_t*>(base + off);
}

__device__ __forceinline__ uint2 lds64(const uint8_t* base, uint32_t off) {
    return *reinterpret_cast<const uint2*>(base + off);
}

// Shared-memory loads from 32-bit shared-window addresses (PTX .shared state space).
// ld_shared_const: for tables that are read-only once filled (after a barrier that the load
// depends on through its address), so the compiler may schedule it freely.
__device__ __forceinline__ uint32_t ld_shared_const(uint32_t addr) {
    uint32_t v;
    asm("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}

// ld_shared_v2_const: 8 bytes of such a read-only table.
__device__ __forceinline__ uint2 ld_shared_v2_const(uint32_t addr) {
    uint2 v;
    asm("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
    return v;
}

// ld_shared_v4_const: 16 bytes of such a read-only table.
__device__ __forceinline__ uint4 ld_shared_v4_const(uint32_t addr) {
    uint4 v;
    asm("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}

// ld_shared_v4: 16 bytes at addr + OFF, kept in program order with the other volatile asm
// (the cp.async waits that make the data valid).
template <int OFF>
__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4+%5];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(addr), "n"(OFF));
    return v;
}

__device__ __forceinline__ uint2 ld_shared_v2_volatile(uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
    return v;
}

__device__ __forceinline__ uint32_t ld_shared_u32_volatile(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}

// 16-byte (or `bytes`-wide) asynchronous global->shared copy; src_bytes = 0 writes zeros and
// reads nothing.
__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes)
                 : "memory");
}

__device__ __forceinline__ void cp_async_4(uint32_t dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(src_bytes)
                 : "memory");
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// D = A (16x32 s8, row) * B (32x8 s8, col), s32 accumulate from zero.
__device__ __forceinline__ void mma_s8_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                             uint32_t a3, uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// D = A (16x32 s8, row) * B (32x8 u8, col), s32 accumulate from zero.
__device__ __forceinline__ void mma_s8u8_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// Programmatic dependent launch (PTX griddepcontrol). `pdl_wait` blocks until every grid this
// one depends on has completed and its memory is visible (a no-op for a normal launch);
// `pdl_launch_dependents` lets the next PDL-launched kernel in the stream start early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// L2 prefetch: no data reaches the SM, so they may run before a griddepcontrol.wait.
__device__ __forceinline__ void prefetch_l2(const void* p) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// Global-memory flag words with system-scope ordering (peer GPUs' memory mapped into this
// process is global memory too) and the wall clock that bounds every wait on them.
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void st_release_gpu_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_gpu_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned long long gtimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ float half_bits_to_float(uint32_t h) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(h & 0xFFFFu)));
}

// Little-endian loads that need no alignment (byte reads; for the generic paths).
__device__ __forceinline__ uint32_t ld_u32_le_unaligned(const uint8_t* p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

__device__ __forceinline__ uint32_t ld_u16_le_unaligned(const uint8_t* p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8);
}

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

}  // namespace iq2
