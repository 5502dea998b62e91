/*
 * candelora_iq2.h -- C ABI of the B200 (sm_100a) IQ2_XXS quantised matmul.
 *
 * This is the boundary a host binding (the Rust candle op, a ctypes/cgo stub, the C++ mirror
 * in this repository) calls. It replaces the Metal dispatch of the reference crate
 * candelora-metal-kernels: every entry point below names the reference function it stands in
 * for (file:line in that crate).
 *
 * Conventions
 *  - All tensors are DEVICE pointers on the caller's current CUDA device, contiguous, with the
 *    reference's layouts:
 *      x              [m, in_dim]   row-major, f32 / f16 / bf16 (x_dtype)
 *      weight_bytes   u8 [out_dim * ceil(in_dim/256) * 64]   the 64-byte `qs` of every 256-weight
 *                     block, row n's blocks contiguous (block index n*blocks_per_row + blk)
 *      weight_scales  u8 [out_dim * ceil(in_dim/256) * 2]    little-endian fp16 `d` per block
 *      out            f32 [m, out_dim] row-major (always f32, whatever x_dtype is)
 *  - Every call is stream-ordered on `stream` and never synchronises the host. No entry point
 *    allocates device memory: scratch space is the caller's `workspace` (size from the
 *    matching *_workspace_size query). The workspace may be reused by later calls on the same
 *    stream; concurrent calls need separate workspaces.
 *  - Return value 0 = success; otherwise an IQ2_ERR_* code, and iq2_last_error() returns a
 *    message for the calling thread (the reference's bail! strings where one exists).
 *  - Thread-safe and re-entrant: there is no global mutable state apart from the per-thread
 *    error message and a per-device cache of device attributes.
 */
#ifndef CANDELORA_IQ2_H
#define CANDELORA_IQ2_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* cudaStream_t without the CUDA headers (same type: struct CUstream_st*). NULL = legacy stream. */
typedef struct CUstream_st* iq2_stream_t;

#define IQ2_ABI_VERSION 2

/* Status codes. The reference bails with a message in each of these situations. */
enum iq2_status {
    IQ2_OK = 0,
    IQ2_ERR_INVALID_ARGUMENT = 1, /* NULL pointer, unknown enum value                               */
    IQ2_ERR_ZERO_DIM = 2,         /* "expects non-zero dimensions"      src/iq2_matmul.rs:210-212   */
    IQ2_ERR_DEVICE = 3,           /* pointer not device memory of the current device  :213-225      */
    IQ2_ERR_DTYPE = 4,            /* "unsupported x dtype"               :73-74                      */
    IQ2_ERR_OVERFLOW = 5,         /* "size overflow" / "too large"       :238-245, :305-311          */
    IQ2_ERR_TOO_SMALL = 6,        /* "weight_bytes too small" / "weight_scales too small" :246-259  */
    IQ2_ERR_UNSUPPORTED = 7,      /* W4A8 in strict mode :300-302, :581-589; variant not built      */
    IQ2_ERR_WORKSPACE = 8,        /* workspace NULL or smaller than the *_workspace_size query      */
    IQ2_ERR_CUDA = 9,             /* a CUDA runtime call failed                                     */
    IQ2_ERR_COMM = 10,            /* an NCCL call of the sharded path failed, or a wait on the
                                     other ranks ran out (the communicator is then unusable)         */
    IQ2_ERR_TIMEOUT = 11          /* a kernel of this library gave up on a bounded in-kernel wait   */
};

/* Activation dtypes (the reference dispatches on x.dtype(), src/iq2_matmul.rs:59-75). */
enum iq2_dtype { IQ2_DTYPE_F32 = 0, IQ2_DTYPE_F16 = 1, IQ2_DTYPE_BF16 = 2 };

/* Iq2MatmulVariant (src/iq2_matmul.rs:31-37). Every variant has a matmul and a dequantisation
 * kernel; the grouped, sharded and no-allocation entry points take IQ2_XXS only. */
enum iq2_variant {
    IQ2_VARIANT_IQ2_XXS = 0,
    IQ2_VARIANT_IQ2_XS = 1,
    IQ2_VARIANT_IQ2_S = 2,
    IQ2_VARIANT_IQ3_S = 3
};

/* ActivationQuantMode (src/activation_quant.rs:7-15). */
enum iq2_act_quant_mode { IQ2_ACT_QUANT_OFF = 0, IQ2_ACT_QUANT_W8A8 = 1, IQ2_ACT_QUANT_W4A8 = 2 };

/* Message for the last failed call on this thread ("" if none). Valid until the next call. */
const char* iq2_last_error(void);

/* IQ2_ABI_VERSION of the loaded library. */
int iq2_abi_version(void);

/*
 * Status of this library's bounded in-kernel waits on the current device. No reference
 * counterpart: the reference's Metal dispatch has no in-kernel waits. The prefill GEMM's pipeline
 * waits give up after 2 s (only a broken pipeline waits that long); a call whose kernel gave up
 * has incomplete outputs although the call itself returned IQ2_OK (it was asynchronous). This
 * synchronises the device and returns IQ2_ERR_TIMEOUT (with a message naming the waits) when any
 * kernel gave up since the previous iq2_device_check, else IQ2_OK; the status is then cleared.
 */
int iq2_device_check(void);

/* Bytes of device scratch iq2_matmul needs for this problem. 0 means none: workspace may then be NULL.
 * IQ2_XS, IQ2_S and IQ3_S report the workspace of their
 * tensor-core path (the GEMM; the decode GEMV's x limbs); a call of theirs without it is still
 * valid and runs the f32 CUDA-core kernel instead. */
size_t iq2_matmul_workspace_size(uint32_t m, uint32_t out_dim, uint32_t in_dim, int x_dtype,
                                 int variant);

/*
 * out = x @ dequant(W)^T, f32 accumulate, f32 output [m, out_dim].
 * Replaces iq2_matmul (src/iq2_matmul.rs:535-553) -> iq2_matmul_metal (:197-365) with
 * ActivationQuantMode::Off, and through it iq2_xxs_matmul (:604-619).
 * m == 0 is valid and launches nothing (the reference returns an empty [0, out_dim] tensor).
 * weight_*_len are the element counts of the caller's buffers (checked like :246-259).
 * Routing (not part of the contract): IQ2_XXS with m <= 32 runs the decode GEMV (int8 tensor-core
 * decode; x in 28-bit fixed point for m <= 4, rel. error ~1e-6, and 16-bit above, ~4e-5), larger
 * m the tcgen05 GEMM (bf16 operands, f32 accumulate). IQ2_XS, IQ2_S and IQ3_S with m > 32 and a
 * workspace of iq2_matmul_workspace_size bytes run the same tcgen05 GEMM (weights decoded to
 * bf16), with m <= 32 and that workspace the decode GEMV (as IQ2_XXS); otherwise an f32
 * CUDA-core kernel (src/iq2_matmul.rs:884-1016 numerics, FMA accumulate).
 */
int iq2_matmul(const void* x, int x_dtype, uint32_t m, const uint8_t* weight_bytes,
               size_t weight_bytes_len, const uint8_t* weight_scales, size_t weight_scales_len,
               uint32_t out_dim, uint32_t in_dim, int variant, float* out, void* workspace,
               size_t workspace_bytes, iq2_stream_t stream);

/*
 * iq2_matmul with an activation-quant contract. Replaces iq2_matmul_with_activation_quant
 * (src/iq2_matmul.rs:555-591): OFF -> iq2_matmul; W4A8 -> IQ2_ERR_UNSUPPORTED when strict,
 * else iq2_matmul; W8A8 -> the reference's W8A8 numerics (src/metal_src/iq2_matmul.metal:85-102,
 * :437-499): every x row quantised to int8 with inv = 127/max|x| and back, then the matmul of
 * those values. W8A8 needs the workspace of iq2_matmul_with_activation_quant_workspace_size.
 */
int iq2_matmul_with_activation_quant(const void* x, int x_dtype, uint32_t m,
                                     const uint8_t* weight_bytes, size_t weight_bytes_len,
                                     const uint8_t* weight_scales, size_t weight_scales_len,
                                     uint32_t out_dim, uint32_t in_dim, int variant, int act_mode,
                                     int strict, float* out, void* workspace,
                                     size_t workspace_bytes, iq2_stream_t stream);

/* Workspace for iq2_matmul_with_activation_quant with this act_mode (W8A8 adds m*in_dim floats). */
size_t iq2_matmul_with_activation_quant_workspace_size(uint32_t m, uint32_t out_dim, uint32_t in_dim,
                                                      int x_dtype, int variant, int act_mode);

/* One projection of a grouped call (see iq2_matmul_grouped). */
typedef struct iq2_matmul_problem {
    const void* x;                 /* [m, in_dim] in the call's x_dtype                      */
    const uint8_t* weight_bytes;   /* IQ2_XXS qs, layout as for iq2_matmul                   */
    size_t weight_bytes_len;
    const uint8_t* weight_scales;  /* fp16 d per block                                       */
    size_t weight_scales_len;
    uint32_t out_dim, in_dim;
    float* out;                    /* [m, out_dim] f32                                       */
} iq2_matmul_problem;

/* Bytes of device scratch iq2_matmul_grouped needs for these problems. */
size_t iq2_matmul_grouped_workspace_size(const iq2_matmul_problem* problems, uint32_t count,
                                         uint32_t m, int x_dtype);

/*
 * `count` independent IQ2_XXS projections with the same m and x dtype, e.g. the q/k/v or
 * gate/up projections of a layer, in as few launches as possible (one x-prep and one GEMV
 * launch per 256 projections when m <= 32; projections that share an x pointer share its
 * preparation). Each problem's result equals iq2_matmul on it. No reference counterpart: the
 * reference issues one dispatch per projection (src/iq2_matmul.rs:316-357); this is the batched
 * form of that call.
 */
int iq2_matmul_grouped(const iq2_matmul_problem* problems, uint32_t count, uint32_t m, int x_dtype,
                       void* workspace, size_t workspace_bytes, iq2_stream_t stream);

/* Size of the fixed scratch array behind iq2_matmul_noalloc (8 MiB per GPU that loads the library). */
#define IQ2_NOALLOC_SCRATCH_BYTES (8u * 1024u * 1024u)

/*
 * iq2_matmul for the decode path (m <= 16) that allocates nothing and takes no workspace.
 * No counterpart in the reference (which allocates its output and needs no scratch); it exists
 * for callers that cannot allocate device memory where they call this: an engine whose memory
 * pool owns the whole GPU, a decode loop that must not pay cudaMalloc's synchronisation, a C
 * binding handed only tensor pointers. The caller still provides x and out.
 * Scratch comes from one library-owned device array of IQ2_NOALLOC_SCRATCH_BYTES, shared by all
 * calls on a device: problems that would need more (large out_dim x m) fail with
 * IQ2_ERR_WORKSPACE, and calls whose kernels overlap on the GPU race on it. The first call on a
 * device looks up the array's device address (cudaGetSymbolAddress); make it outside any stream
 * capture. The address is looked up again after the device's context was replaced
 * (cudaDeviceReset). m > 16 returns IQ2_ERR_UNSUPPORTED. Same checks as iq2_matmul otherwise, and
 * the same kernels, so the same results bit for bit.
 */
int iq2_matmul_noalloc(const void* x, int x_dtype, uint32_t m, const uint8_t* weight_bytes,
                       size_t weight_bytes_len, const uint8_t* weight_scales, size_t weight_scales_len,
                       uint32_t out_dim, uint32_t in_dim, float* out, iq2_stream_t stream);

/*
 * Dense dequantisation to out [out_dim, in_dim] in out_dtype (f16 / bf16 / f32).
 * Replaces iq2_dequantize_to_f16 (src/iq2_matmul.rs:593-602, :367-505) when out_dtype is
 * IQ2_DTYPE_F16: bit-identical to the reference kernel iq2_xxs_dequantize_f16
 * (src/metal_src/iq2_matmul.metal:868-887). f32 gives the exact weight value; bf16 its RNE.
 */
int iq2_dequantize(const uint8_t* weight_bytes, size_t weight_bytes_len,
                   const uint8_t* weight_scales, size_t weight_scales_len, uint32_t out_dim,
                   uint32_t in_dim, int variant, void* out, int out_dtype, iq2_stream_t stream);

/*
 * Column-sharding helper for multi-GPU runs: out [m, shards*shard_cols] <- gathered
 * [shards, m, shard_cols] (the layout an all-gather of per-rank f32 outputs produces).
 * No reference counterpart (the reference is single-device).
 */
int iq2_gather_columns(const float* gathered, uint32_t shards, uint32_t m, uint32_t shard_cols,
                       float* out, iq2_stream_t stream);

/*
 * ggml / GGUF block layout -> the split tensors this library (and the reference) take. No
 * reference counterpart: the reference only reads split tensors; this is the ingest of the
 * on-disk format they come from. `blocks` holds nblocks interleaved ggml blocks of `variant`
 * (block_iq2_xxs 66 B: d, qs[64]; block_iq2_xs 74 B: d, qs[64], scales[8]; block_iq2_s 82 B:
 * d, qs[64], qh[8], scales[8]; block_iq3_s 110 B: d, qs[64], qh[8], signs[32], scales[4]);
 * weight_bytes receives nblocks * {64, 64, 72, 104} bytes, weight_scales nblocks * {2, 10, 10, 6}
 * (d, then the block's scale bytes). Device pointers, stream-ordered.
 */
int iq2_split_interleaved(const uint8_t* blocks, size_t blocks_len, uint64_t nblocks, int variant,
                          uint8_t* weight_bytes, uint8_t* weight_scales, iq2_stream_t stream);

/*
 * Column sharding over the GPUs of one node (no reference counterpart: the reference is
 * single-device; this is the multi-GPU layout the benchmark specification asks for). Rank r of a
 * world of g holds rows [r*N/g, (r+1)*N/g) of each projection's weights, a contiguous slice of
 * both weight tensors (weight_bytes from byte r*(N/g)*ceil(K/256)*64, weight_scales from byte
 * r*(N/g)*ceil(K/256)*2); every rank gets the full [m, N] output through one NCCL all-gather.
 * One process per GPU: rank 0 makes the id, every rank passes the same id to iq2_comm_init with
 * its own device current.
 */
#define IQ2_COMM_ID_BYTES 128
typedef struct iq2_comm_s* iq2_comm_t;
int iq2_comm_unique_id(uint8_t* id /* IQ2_COMM_ID_BYTES */);
/* The communicator is a non-blocking NCCL communicator: every wait of this library on the other
 * ranks (joining, NCCL calls, the barriers of iq2_comm_symmetric_alloc / iq2_comm_destroy) is
 * polled and bounded by timeout_ms of wall time (iq2_comm_init: 120 s). A wait that runs out, or
 * an asynchronous NCCL error, aborts the communicator and returns IQ2_ERR_COMM; every later call
 * on it returns IQ2_ERR_COMM (iq2_comm_destroy still frees it). A rank that never calls
 * iq2_comm_init makes the others' iq2_comm_init return IQ2_ERR_COMM after timeout_ms. */
int iq2_comm_init_with_timeout(const uint8_t* id, int world, int rank, uint32_t timeout_ms, iq2_comm_t* comm);
int iq2_comm_init(const uint8_t* id, int world, int rank, iq2_comm_t* comm);
int iq2_comm_destroy(iq2_comm_t comm);  /* collective when a symmetric region exists */

/*
 * Symmetric output region (no reference counterpart; it is the fused all-gather epilogue of the
 * sharded decode). Collective: every rank asks for the same `bytes`; each gets a device buffer of
 * that size whose storage every other rank of the communicator has mapped (CUDA IPC over NVLink).
 * One region per communicator, freed by iq2_comm_destroy. When every `out` of an
 * iq2_matmul_grouped_sharded call lies in the region (at the same offsets on all ranks) and
 * m <= 32, the decode GEMV stores each output straight into every rank's region: no NCCL call, no
 * gather buffer, one kernel launch. Its waits for the other ranks are bounded (about a second).
 * A wait that runs out, or a call that fails on one rank after the ranks chose this path (e.g. a
 * misaligned weight slice), sets a sticky error: that call's outputs, and those of every later
 * fused call of the communicator, hold only this rank's columns (the calls run local-only, with
 * no waits), and iq2_comm_check reports IQ2_ERR_COMM on every rank until the communicator is
 * destroyed.
 */
int iq2_comm_symmetric_alloc(iq2_comm_t comm, size_t bytes, void** ptr);
/* IQ2_OK, or IQ2_ERR_COMM if a fused exchange of this communicator failed (synchronising), if
 * NCCL reported an asynchronous error, or if the communicator was aborted. */
int iq2_comm_check(iq2_comm_t comm);

/* Workspace for iq2_matmul_grouped_sharded: the problems describe the rank's slices, with
 * out_dim the full N (a multiple of world) and out the full [m, N] output. */
size_t iq2_matmul_grouped_sharded_workspace_size(const iq2_matmul_problem* problems, uint32_t count,
                                                 uint32_t m, int x_dtype, int world);
/* Up to 256 projections: their slices through one grouped call, one ncclAllGather of all of them
 * on `stream`, one scatter kernel into the outputs (or, with every output in the symmetric
 * region and m <= 32, the fused exchange above; its weight slices must then be 16-byte (bytes)
 * and 4-byte (scales) aligned on every rank). For m > 32 with at most 64 projections the exchange
 * is pipelined: each projection (split along m when its gathered output passes 256 MB) is
 * computed on `stream` while the previous one's all-gather and scatter run on two streams of the
 * communicator, which `stream` waits for before the call's later work. Stream-ordered, collective:
 * every rank makes the same call with the same shapes; a communicator serves one such call at a
 * time. */
int iq2_matmul_grouped_sharded(iq2_comm_t comm, const iq2_matmul_problem* problems, uint32_t count,
                               uint32_t m, int x_dtype, void* workspace, size_t workspace_bytes,
                               iq2_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* CANDELORA_IQ2_H */
