// Internal launch interface between the C ABI (iq2xxs_capi.cu) and the kernel files.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace iq2 {

constexpr int kDtypeBf16 = 2;  // IQ2_DTYPE_BF16 of the C ABI

// Decode GEMV (iq2xxs_gemv.cu), m <= kGemvMaxM (x in four 7-bit limbs for m <= 4, as a 16-bit
// value split into a signed and an unsigned byte for 4 < m <= 32). A group is up to gemv_max_group() projections with the same m and x dtype,
// computed by one prep launch and one GEMV launch.
constexpr uint32_t kGemvMaxM = 32;
struct GemvProblemHost {
    const void* x;
    const uint8_t* qs;
    const uint8_t* sc;
    uint32_t n, k;
    float* out;
    uint32_t ldo = 0;  // elements between output rows (0: n)
};

// Peer-memory outputs of a sharded decode GEMV. Every rank of a communicator owns a symmetric
// region (same size, mapped into every other rank's process); it starts with this header. A GEMV
// launched with peers stores each output at the same offset of every rank's region, and the
// header words order the exchange (all written and read with system-scope release/acquire):
//   entry[r]  the last call rank r has started (a rank stores into peers only after all entered:
//             entering proves the peer's earlier stream work, which may still read the previous
//             call's outputs, is done);
//   data[r]   the last call whose outputs rank r has finished storing into this region;
//   go        this rank's last call whose entry barrier completed (go_owner: the call whose
//             barrier a warp has taken on: the first warp that needs it waits for the entries);
//   epoch     this rank's last finished call (the next one is epoch + 1; kept on the device so that
//             captured CUDA graphs replay correctly);
//   done      CTAs of the running call that finished storing; err: sticky error bits.
struct SymmHeader {
    unsigned long long entry[8];
    unsigned long long data[8];
    unsigned long long go;
    unsigned long long go_owner;
    unsigned long long epoch;
    unsigned int done;
    unsigned int err;  // bit 0: entry barrier timed out; bit 1: data barrier timed out;
                       // bit 2: a call failed on this rank before its launch (sticky until destroy)
};
constexpr size_t kSymmHeaderBytes = 4096;
constexpr int kMaxRanks = 8;
struct GemvPeers {
    SymmHeader* hdr;             // this rank's header (device address)
    long long delta[kMaxRanks];  // rank r's region minus this rank's, in bytes (0 for this rank)
    int world, rank;
};
bool gemv_fast_path_ok(uint32_t m, uint32_t k, const uint8_t* qs, const uint8_t* sc);
uint32_t gemv_max_group();
size_t gemv_group_workspace_size(const GemvProblemHost* probs, uint32_t count, uint32_t m, int num_sms);
cudaError_t launch_gemv_group(const GemvProblemHost* probs, uint32_t count, uint32_t m, int x_dtype,
                              void* workspace, int num_sms, cudaStream_t stream, const GemvPeers* peers = nullptr);
size_t gemv_workspace_size(uint32_t m, uint32_t n, uint32_t k, int num_sms);
// The W8A8 mode's decode (m <= kGemvW8A8MaxM): x quantised per row to int8 (the reference's
// numerics), the int8 values fed to the GEMV as its only limb.
constexpr uint32_t kGemvW8A8MaxM = 32;
size_t gemv_w8a8_workspace_size(uint32_t m, uint32_t n, uint32_t k);
cudaError_t launch_gemv_w8a8(const void* x, int x_dtype, uint32_t m, const uint8_t* qs, const uint8_t* sc,
                             uint32_t n, uint32_t k, float* out, void* workspace, int num_sms, cudaStream_t stream);
cudaError_t launch_gemv(const void* x, int x_dtype, uint32_t m, const uint8_t* qs, const uint8_t* sc,
                        uint32_t n, uint32_t k, float* out, void* workspace, int num_sms,
                        cudaStream_t stream);
// The same decode GEMV for IQ2_XS, IQ2_S and IQ3_S weights (variant 1, 2 or 3 as IQ2_VARIANT_*;
// m <= kGemvMaxM; qs 16-byte and sc 4-byte aligned). gemv_variant_ok: the formats it takes.
bool gemv_variant_ok(int variant);
size_t gemv_variant_workspace_size(int variant, uint32_t m, uint32_t n, uint32_t k);
cudaError_t launch_gemv_variant(int variant, const void* x, int x_dtype, uint32_t m, const uint8_t* qs,
                                const uint8_t* sc, uint32_t n, uint32_t k, float* out, void* workspace, int num_sms,
                                cudaStream_t stream);
cudaError_t launch_gemv_generic(const void* x, int x_dtype, uint32_t m, const uint8_t* qs,
                                const uint8_t* sc, uint32_t n, uint32_t k, float* out,
                                int num_sms, cudaStream_t stream);

// Tensor-core GEMM (iq2xxs_gemm.cu), m > 16. variant: the weight format (IQ2_VARIANT_*: 0
// IQ2_XXS, 1 IQ2_XS, 2 IQ2_S, 3 IQ3_S; the workspace size does not depend on it).
bool gemm_path_ok(uint32_t m, uint32_t n, uint32_t k, const void* x, int x_dtype, const uint8_t* qs,
                  const uint8_t* sc, const float* out);
size_t gemm_workspace_size(uint32_t m, uint32_t n, uint32_t k, int x_dtype, int num_sms);
cudaError_t launch_gemm(const void* x, int x_dtype, uint32_t m, const uint8_t* qs, const uint8_t* sc,
                        uint32_t n, uint32_t k, float* out, void* workspace, int num_sms,
                        cudaStream_t stream, int variant = 0);

// The prefill GEMM's per-device sticky status (iq2xxs_gemm.cu): synchronises the current device,
// stores the status bits in *status and clears them; returns a cudaError_t.
int gemm_take_status(unsigned int* status);
// Test hook of the GEMM's bounded waits (process-wide): wait bound (0: the default 2 s) and a stage
// whose "weights written" arrival is withheld (0: none).
void gemm_testing_set_stall(uint64_t wait_limit_ns, uint32_t stall_stage);

// The current CUDA context of the calling thread (a CUcontext, as an opaque handle; nullptr when
// none): caches of device addresses are keyed on it so that a new primary context (after
// cudaDeviceReset) is looked up again.
void* current_context_handle();

// C ABI helpers (iq2xxs_capi.cu) used by iq2xxs_noalloc.cu and iq2xxs_sharded.cu.
int capi_fail(int code, const char* fmt, ...);
int capi_cuda_fail(const char* what, cudaError_t e);
int capi_ok();  // clears the thread's error message
int capi_num_sms();
int capi_validate_matmul(const char* op, const void* x, int x_dtype, uint32_t m, const uint8_t* weight_bytes,
                         size_t weight_bytes_len, const uint8_t* weight_scales, size_t weight_scales_len,
                         uint32_t out_dim, uint32_t in_dim, const float* out, int variant = 0);

// Dequantisation and the sharding gather (iq2xxs_dequant.cu).
cudaError_t launch_dequant(const uint8_t* qs, const uint8_t* sc, uint32_t n, uint32_t k, void* out,
                           int out_dtype, int num_sms, cudaStream_t stream);
// The IQ2_XS / IQ2_S / IQ3_S formats (iq2_variants.cu); variant = IQ2_VARIANT_* of the C ABI.
cudaError_t launch_variant_matmul(int variant, const void* x, int x_dtype, uint32_t m, const uint8_t* qs,
                                  const uint8_t* sc, uint32_t n, uint32_t k, float* out, int num_sms,
                                  cudaStream_t stream);
cudaError_t launch_variant_dequant(int variant, const uint8_t* qs, const uint8_t* sc, uint32_t n, uint32_t k,
                                   void* out, int out_dtype, int num_sms, cudaStream_t stream);
cudaError_t launch_split_interleaved(const uint8_t* blocks, uint64_t nblocks, uint32_t bytes_per_block,
                                     uint32_t scales_per_block, uint8_t* wb, uint8_t* ws, int num_sms,
                                     cudaStream_t stream);
cudaError_t launch_qdq_w8a8(const void* x, int x_dtype, uint32_t m, uint32_t k, float* xq, cudaStream_t stream);
cudaError_t launch_gather_columns(const float* gathered, uint32_t shards, uint32_t m,
                                  uint32_t shard_cols, float* out, int num_sms, cudaStream_t stream);

}  // namespace iq2
