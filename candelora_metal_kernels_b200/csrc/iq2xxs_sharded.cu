// Column-sharded IQ2_XXS matmul across the GPUs of one node: rank r of a world of g holds the weight
// rows [r*N/g, (r+1)*N/g) of every projection (a contiguous slice of both weight tensors, so no
// repacking), computes its [m, N/g] output slice with the single-GPU kernels, and one NCCL
// all-gather over NVLink gives every rank the full [m, N] output. The reference is single-device;
// this is the sharding the benchmark specification asks for (large projections over 2/4/8 B200).
//
// Per call: one grouped matmul of all local slices into a packed buffer of the workspace, one
// ncclAllGather of that buffer (rank-major), then one kernel that scatters the gathered slices
// into each projection's [m, N] output. A single projection at m = 1 is all-gathered straight
// into its output (rank-major slices of one row are already the row).
//
// Pipelined exchange (m above the decode GEMV's range, the tensor-core GEMM): the call is cut into
// chunks (each projection, split along m into parts of at most ~256 MB of gathered output), each
// chunk's slice is computed on the caller's stream, and its all-gather and scatter run on two
// side streams while the next chunk computes, so that the exchange (the larger part at 4-8
// ranks: the f32 outputs cross NVLink) overlaps the GEMMs.
//
// Fused exchange: when every output lies in the communicator's symmetric region (allocated by
// iq2_comm_symmetric_alloc: one device allocation per rank, mapped into every other rank's process
// with CUDA IPC) and m <= 32, the decode GEMV stores each output value straight into all ranks'
// regions over NVLink (plain peer stores) and synchronises through flag words at the head of each
// region: no NCCL call, no gather buffer, no scatter kernel, one launch per call.
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "../../include/candelora_iq2.h"
#include "iq2xxs_common.cuh"
#include "iq2xxs_internal.h"

struct iq2_comm_s {
    ncclComm_t nccl;
    int world, rank, device;
    uint32_t timeout_ms = 0;     // bound of every wait on the other ranks (NCCL calls, barriers)
    bool aborted = false;        // a wait ran out or NCCL failed: the NCCL communicator was aborted
    uint8_t* symm = nullptr;     // this rank's symmetric region (header + user area)
    size_t symm_bytes = 0;       // user area bytes
    void* peer[iq2::kMaxRanks] = {};  // the other ranks' regions mapped here (IPC); peer[rank] = symm
    // The pipelined exchange (m above the decode GEMV's range): a stream for the all-gathers, one for
    // the scatters, and events that fork them from and join them to the caller's stream; created on
    // the first such call.
    cudaStream_t xs[2] = {};
    cudaEvent_t ev[2 * 64 + 2] = {};
};

namespace iq2 {
namespace {

constexpr uint32_t SCATTER_CAP = 256;
constexpr uint32_t kDefaultCommTimeoutMs = 120000;  // iq2_comm_init: two minutes

double elapsed_ms(std::chrono::steady_clock::time_point t0) {
    return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
}

// The communicators are non-blocking (ncclConfig_t.blocking = 0): an NCCL call may return
// ncclInProgress, and the communicator's state is then polled with ncclCommGetAsyncError until it
// leaves that state or `timeout_ms` of wall time pass. Returns the final state; ncclInProgress
// means the wait ran out (the caller aborts the communicator).
ncclResult_t nccl_settle(ncclComm_t c, ncclResult_t r, uint32_t timeout_ms) {
    if (r != ncclInProgress) return r;
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        ncclResult_t st = ncclInProgress;
        const ncclResult_t q = ncclCommGetAsyncError(c, &st);
        if (q != ncclSuccess) return q;
        if (st != ncclInProgress) return st;
        if (elapsed_ms(t0) > timeout_ms) return ncclInProgress;
        std::this_thread::sleep_for(std::chrono::microseconds(100));
    }
}

// Waits for the work queued on `s` (which may hold NCCL kernels waiting for other ranks) while
// polling the communicator for asynchronous errors, for at most the communicator's timeout.
ncclResult_t stream_settle(iq2_comm_t comm, cudaStream_t s) {
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        const cudaError_t e = cudaStreamQuery(s);
        if (e == cudaSuccess) return ncclSuccess;
        if (e != cudaErrorNotReady) return ncclUnhandledCudaError;
        ncclResult_t st = ncclSuccess;
        if (ncclCommGetAsyncError(comm->nccl, &st) != ncclSuccess) return ncclInternalError;
        if (st != ncclSuccess && st != ncclInProgress) return st;
        if (elapsed_ms(t0) > comm->timeout_ms) return ncclInProgress;
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

// A wait on the other ranks ran out or NCCL reported an error: abort the communicator (this
// ends its pending work and frees its resources) so that the process stays usable.
int comm_failed(iq2_comm_t comm, const char* op, const char* what, ncclResult_t r) {
    if (!comm->aborted) {
        ncclCommAbort(comm->nccl);
        comm->aborted = true;
    }
    if (r == ncclInProgress)
        return capi_fail(IQ2_ERR_COMM, "%s: %s: no answer from the other ranks within %u ms; communicator aborted", op,
                         what, comm->timeout_ms);
    return capi_fail(IQ2_ERR_COMM, "%s: %s: %s; communicator aborted", op, what, ncclGetErrorString(r));
}

struct ScatterItem {
    float* out;
    uint64_t off;    // element offset of this projection's slice in a rank's packed buffer
    uint32_t n_loc;  // columns per rank
    uint32_t pad;
};

struct ScatterLaunch {
    const float* gathered;
    uint64_t per_rank;  // packed elements per rank
    uint32_t world, m;
    ScatterItem item[SCATTER_CAP];
};

// blockIdx.y = projection; each block copies whole segments (rank r's n_loc columns of one row,
// contiguous in both the gathered slices and the output), 16 bytes per thread and step where the
// columns per rank are a multiple of 4 and the output is 16-byte aligned: a memory-bound copy with
// no per-element index arithmetic, so that it takes little from GEMMs running beside it.
__global__ void __launch_bounds__(256) scatter_slices_kernel(const __grid_constant__ ScatterLaunch L) {
    const ScatterItem& it = L.item[blockIdx.y];
    const uint32_t nl = it.n_loc, segs = L.m * L.world;
    const uint64_t n = (uint64_t)nl * L.world;
    const bool vec = nl % 4 == 0 && L.per_rank % 4 == 0 && it.off % 4 == 0 &&
                     (reinterpret_cast<uintptr_t>(it.out) & 15u) == 0 && (reinterpret_cast<uintptr_t>(L.gathered) & 15u) == 0;
    for (uint32_t sg = blockIdx.x; sg < segs; sg += gridDim.x) {
        const uint32_t row = sg / L.world, r = sg % L.world;
        const float* src = L.gathered + r * L.per_rank + it.off + (uint64_t)row * nl;
        float* dst = it.out + row * n + (uint64_t)r * nl;
        if (vec) {
            for (uint32_t j = threadIdx.x * 4u; j < nl; j += blockDim.x * 4u)
                *reinterpret_cast<float4*>(dst + j) = __ldcs(reinterpret_cast<const float4*>(src + j));
        } else {
            for (uint32_t j = threadIdx.x; j < nl; j += blockDim.x) dst[j] = src[j];
        }
    }
}

size_t align256(size_t v) { return (v + 255) / 256 * 256; }

// Sets bits of the sticky error word of this rank's symmetric-region header (stream-ordered).
__global__ void mark_comm_error_kernel(unsigned* err, unsigned bits) { atomicOr(err, bits); }

struct ShardPlan {
    std::vector<uint64_t> off;  // packed offsets (elements)
    uint64_t per_rank = 0;
    size_t packed_bytes = 0, gathered_bytes = 0, inner_off = 0;
    bool direct = false;  // one projection, m == 1: all-gather into out
};

ShardPlan plan_shards(const iq2_matmul_problem* probs, uint32_t count, uint32_t m, int world) {
    ShardPlan pl;
    for (uint32_t i = 0; i < count; ++i) {
        pl.off.push_back(pl.per_rank);
        pl.per_rank += (uint64_t)m * (probs[i].out_dim / (uint32_t)world);
    }
    pl.direct = count == 1 && m == 1;
    pl.packed_bytes = align256(pl.per_rank * sizeof(float));
    pl.gathered_bytes = pl.direct ? 0 : align256(pl.per_rank * world * sizeof(float));
    pl.inner_off = pl.packed_bytes + pl.gathered_bytes;
    return pl;
}

// The local problems: each projection's rank slice, written into the packed buffer.
std::vector<iq2_matmul_problem> local_problems(const iq2_matmul_problem* probs, uint32_t count, uint32_t m,
                                               int world, const ShardPlan& pl, float* packed) {
    std::vector<iq2_matmul_problem> loc(probs, probs + count);
    for (uint32_t i = 0; i < count; ++i) {
        loc[i].out_dim = probs[i].out_dim / (uint32_t)world;
        loc[i].out = packed + pl.off[i];
    }
    (void)m;
    return loc;
}


// Pipelined exchange: chunk c is rows [m0, m0 + mlen) of projection i; its slice sits at `off`
// (elements) of the packed buffer and, gathered, at world * off ([rank][mlen][n_loc]).
struct Chunk {
    uint32_t i, m0, mlen;
    uint64_t off;
};
constexpr uint32_t kMaxChunks = 64;
constexpr uint64_t kChunkGatherBytes = 256ull << 20;

bool use_pipeline(uint32_t m, uint32_t count, int world) { return world > 1 && m > kGemvMaxM && count <= kMaxChunks; }

std::vector<Chunk> plan_chunks(const iq2_matmul_problem* probs, uint32_t count, uint32_t m, int world) {
    std::vector<Chunk> ch;
    uint64_t off = 0;
    // parts per projection: at most ~kChunkGatherBytes gathered, a multiple of 256 rows (the GEMM's
    // token tile) each, at most kMaxChunks in all
    const uint32_t budget = std::max<uint32_t>(1, kMaxChunks / std::max<uint32_t>(1, count));
    for (uint32_t i = 0; i < count; ++i) {
        const uint64_t bytes = (uint64_t)m * probs[i].out_dim * sizeof(float);
        uint32_t parts = (uint32_t)std::min<uint64_t>((bytes + kChunkGatherBytes - 1) / kChunkGatherBytes, budget);
        uint32_t mlen = (m + parts - 1) / parts;
        mlen = std::min(m, (mlen + 255) / 256 * 256);
        const uint32_t n_loc = probs[i].out_dim / (uint32_t)world;
        for (uint32_t m0 = 0; m0 < m; m0 += mlen) {
            const uint32_t len = std::min(mlen, m - m0);
            ch.push_back({i, m0, len, off});
            off += (uint64_t)len * n_loc;
        }
    }
    return ch;
}

// The chunk's local problem: its x rows, this rank's weight slice, its packed output.
iq2_matmul_problem chunk_problem(const iq2_matmul_problem& p, const Chunk& c, int x_dtype, int world,
                                 float* packed) {
    iq2_matmul_problem q = p;
    const size_t esize = x_dtype == IQ2_DTYPE_F32 ? 4 : 2;
    q.x = static_cast<const uint8_t*>(p.x) + (size_t)c.m0 * p.in_dim * esize;
    q.out_dim = p.out_dim / (uint32_t)world;
    q.out = packed ? packed + c.off : nullptr;
    return q;
}

}  // namespace

// The fused-exchange path is taken when every output lies in the symmetric region and m <= 32.
// Every input to this decision is the same on all ranks (the region is allocated collectively and
// carved identically), so all ranks take the same path.
bool use_peer_path(iq2_comm_t comm, const iq2_matmul_problem* probs, uint32_t count, uint32_t m) {
    if (comm->symm == nullptr || m > kGemvMaxM || count > gemv_max_group()) return false;
    const uintptr_t lo = reinterpret_cast<uintptr_t>(comm->symm) + kSymmHeaderBytes;
    const uintptr_t hi = lo + comm->symm_bytes;
    for (uint32_t i = 0; i < count; ++i) {
        const uintptr_t o = reinterpret_cast<uintptr_t>(probs[i].out);
        if (o < lo || o > hi || (uint64_t)m * probs[i].out_dim * sizeof(float) > hi - o) return false;
    }
    return true;
}

// A call that fails on this rank after every rank has chosen the fused exchange never launches
// here, so this rank's call count falls behind the others'. The failure is therefore recorded in
// the sticky error word (bit 2): every later fused call of the communicator on this rank runs
// local-only, the other ranks' bounded waits for this call run out and set their own error words,
// and iq2_comm_check reports the failure on every rank.
int peer_local_failure(iq2_comm_t comm, iq2_stream_t stream, int rc) {
    auto* hdr = reinterpret_cast<SymmHeader*>(comm->symm);
    mark_comm_error_kernel<<<1, 1, 0, reinterpret_cast<cudaStream_t>(stream)>>>(&hdr->err, 4u);
    (void)cudaGetLastError();  // the call's own error is the one reported
    return rc;
}

int sharded_peer(iq2_comm_t comm, const iq2_matmul_problem* probs, uint32_t count, uint32_t m, int x_dtype,
                 void* workspace, size_t workspace_bytes, iq2_stream_t stream) {
    const char* op = "iq2_matmul_grouped_sharded";
    std::vector<GemvProblemHost> loc(count);
    for (uint32_t i = 0; i < count; ++i) {
        const iq2_matmul_problem& p = probs[i];
        const uint32_t n_loc = p.out_dim / (uint32_t)comm->world;
        float* out = p.out + (size_t)comm->rank * n_loc;  // this rank's columns of the full [m, out_dim]
        int rc = capi_validate_matmul(op, p.x, x_dtype, m, p.weight_bytes, p.weight_bytes_len, p.weight_scales,
                                      p.weight_scales_len, n_loc, p.in_dim, out, IQ2_VARIANT_IQ2_XXS);
        if (rc != IQ2_OK) return peer_local_failure(comm, stream, rc);
        // no fallback here: the other ranks are already committed to the fused exchange (their
        // bounded waits end in an error that iq2_comm_check reports)
        if (!gemv_fast_path_ok(m, p.in_dim, p.weight_bytes, p.weight_scales))
            return peer_local_failure(
                comm, stream,
                capi_fail(IQ2_ERR_UNSUPPORTED,
                          "%s: problem %u: with outputs in the symmetric region the weight slices must be 16-byte "
                          "(bytes) and 4-byte (scales) aligned",
                          op, i));
        loc[i] = GemvProblemHost{p.x, p.weight_bytes, p.weight_scales, n_loc, p.in_dim, out, p.out_dim};
    }
    const int sms = capi_num_sms();
    const size_t need = gemv_group_workspace_size(loc.data(), count, m, sms);
    if (need > 0 && (workspace == nullptr || workspace_bytes < need))
        return peer_local_failure(comm, stream,
                                  capi_fail(IQ2_ERR_WORKSPACE, "%s: workspace of %zu bytes needed, got %zu", op, need,
                                            workspace ? workspace_bytes : (size_t)0));
    GemvPeers pe;
    pe.hdr = reinterpret_cast<SymmHeader*>(comm->symm);
    pe.world = comm->world;
    pe.rank = comm->rank;
    for (int r = 0; r < kMaxRanks; ++r)
        pe.delta[r] = r < comm->world ? (long long)(static_cast<uint8_t*>(comm->peer[r]) - comm->symm) : 0;
    const cudaError_t e = launch_gemv_group(loc.data(), count, m, x_dtype, workspace, sms,
                                            reinterpret_cast<cudaStream_t>(stream), &pe);
    if (e != cudaSuccess) return peer_local_failure(comm, stream, capi_cuda_fail(op, e));
    return capi_ok();
}

namespace {

// Side streams and events of the pipelined exchange, created once per communicator.
int pipeline_resources(iq2_comm_t comm, const char* op) {
    if (comm->xs[0] != nullptr) return IQ2_OK;
    int lo = 0, hi = 0;
    cudaDeviceGetStreamPriorityRange(&lo, &hi);
    for (int i = 0; i < 2; ++i) {
        // the all-gathers first (the GEMMs fill every SM, and a late all-gather stalls the chain);
        // the scatters at the GEMMs' priority
        const cudaError_t e = cudaStreamCreateWithPriority(&comm->xs[i], cudaStreamNonBlocking, i == 0 ? hi : lo);
        if (e != cudaSuccess) return capi_cuda_fail(op, e);
    }
    for (cudaEvent_t& ev : comm->ev) {
        const cudaError_t e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
        if (e != cudaSuccess) return capi_cuda_fail(op, e);
    }
    return IQ2_OK;
}

}  // namespace

// The pipelined exchange (see the top of this file). Chunk c: its slice on the caller's stream,
// then on xs[0] (after the slice) its all-gather, then on xs[1] (after the gather) its scatter;
// at the end the caller's stream waits for both side streams. Works under stream capture (the side
// streams fork from and join the caller's stream through events).
int sharded_pipelined(iq2_comm_t comm, const iq2_matmul_problem* probs, uint32_t count, uint32_t m, int x_dtype,
                      uint8_t* ws, size_t ws_bytes, iq2_stream_t stream) {
    const char* op = "iq2_matmul_grouped_sharded";
    int rc = pipeline_resources(comm, op);
    if (rc != IQ2_OK) return rc;
    const int world = comm->world;
    const ShardPlan pl = plan_shards(probs, count, m, world);
    const std::vector<Chunk> chunks = plan_chunks(probs, count, m, world);
    float* packed = reinterpret_cast<float*>(ws);
    float* gathered = reinterpret_cast<float*>(ws + pl.packed_bytes);
    const size_t inner_off = pl.packed_bytes + align256(pl.per_rank * world * sizeof(float));
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream), g = comm->xs[0], sc = comm->xs[1];
    cudaEvent_t* ev_slice = comm->ev;              // [kMaxChunks]
    cudaEvent_t* ev_gath = comm->ev + kMaxChunks;  // [kMaxChunks]
    cudaEvent_t ev_g_end = comm->ev[2 * kMaxChunks], ev_s_end = comm->ev[2 * kMaxChunks + 1];
    cudaError_t e = cudaSuccess;
    // On a failure after the first fork the side streams may still hold this call's gathers and
    // scatters: the caller's stream waits for them all the same, so that nothing it runs next
    // overwrites buffers they still read.
    auto join = [&]() {
        cudaEventRecord(ev_g_end, g);
        cudaEventRecord(ev_s_end, sc);
        cudaStreamWaitEvent(s, ev_g_end, 0);
        cudaStreamWaitEvent(s, ev_s_end, 0);
    };
    // every chunk's problem passes the argument checks before anything is launched (as in the
    // single grouped call): the first chunk of each projection is checked without a launch
    for (uint32_t i = 0; i < count; ++i) {
        const Chunk* first = nullptr;
        for (const Chunk& c : chunks)
            if (c.i == i) {
                first = &c;
                break;
            }
        const iq2_matmul_problem q = chunk_problem(probs[i], *first, x_dtype, world, packed);
        rc = capi_validate_matmul(op, q.x, x_dtype, first->mlen, q.weight_bytes, q.weight_bytes_len, q.weight_scales,
                                  q.weight_scales_len, q.out_dim, q.in_dim, q.out, IQ2_VARIANT_IQ2_XXS);
        if (rc != IQ2_OK) return rc;
    }
    for (size_t ci = 0; ci < chunks.size(); ++ci) {
        const Chunk& c = chunks[ci];
        const iq2_matmul_problem q = chunk_problem(probs[c.i], c, x_dtype, world, packed);
        // 1. this rank's slice of the chunk (validated like iq2_matmul)
        rc = iq2_matmul_grouped(&q, 1, c.mlen, x_dtype, ws + inner_off, ws_bytes - inner_off, stream);
        if (rc != IQ2_OK) {
            if (ci > 0) join();
            return rc;
        }
        // 2. every rank's slices of it, rank-major, while the next chunk computes
        if ((e = cudaEventRecord(ev_slice[ci], s)) != cudaSuccess ||
            (e = cudaStreamWaitEvent(g, ev_slice[ci], 0)) != cudaSuccess)
            return capi_cuda_fail(op, e);
        const uint64_t count_c = (uint64_t)c.mlen * q.out_dim;
        const ncclResult_t r = nccl_settle(
            comm->nccl,
            ncclAllGather(packed + c.off, gathered + (uint64_t)world * c.off, count_c, ncclFloat, comm->nccl, g),
            comm->timeout_ms);
        if (r != ncclSuccess) return comm_failed(comm, op, "ncclAllGather", r);
        // 3. its rows of the projection's [m, out_dim] output
        if ((e = cudaEventRecord(ev_gath[ci], g)) != cudaSuccess ||
            (e = cudaStreamWaitEvent(sc, ev_gath[ci], 0)) != cudaSuccess)
            return capi_cuda_fail(op, e);
        ScatterLaunch L;
        std::memset(&L, 0, sizeof(L));
        L.gathered = gathered + (uint64_t)world * c.off;
        L.per_rank = count_c;
        L.world = (uint32_t)world;
        L.m = c.mlen;
        L.item[0].out = probs[c.i].out + (size_t)c.m0 * probs[c.i].out_dim;
        L.item[0].off = 0;
        L.item[0].n_loc = q.out_dim;
        const unsigned bx = (unsigned)std::min<uint64_t>((uint64_t)c.mlen * world, 1184);
        scatter_slices_kernel<<<dim3(bx, 1), 256, 0, sc>>>(L);
        if ((e = cudaGetLastError()) != cudaSuccess) return capi_cuda_fail(op, e);
    }
    // the caller's stream goes on once every chunk is gathered and scattered
    if ((e = cudaEventRecord(ev_g_end, g)) != cudaSuccess || (e = cudaEventRecord(ev_s_end, sc)) != cudaSuccess ||
        (e = cudaStreamWaitEvent(s, ev_g_end, 0)) != cudaSuccess ||
        (e = cudaStreamWaitEvent(s, ev_s_end, 0)) != cudaSuccess)
        return capi_cuda_fail(op, e);
    return capi_ok();
}

}  // namespace iq2

using iq2::capi_fail;

extern "C" {

int iq2_comm_unique_id(uint8_t* id) {
    if (id == nullptr) return capi_fail(IQ2_ERR_INVALID_ARGUMENT, "iq2_comm_unique_id: NULL id");
    ncclUniqueId uid;
    const ncclResult_t r = ncclGetUniqueId(&uid);
    if (r != ncclSuccess) return capi_fail(IQ2_ERR_COMM, "iq2_comm_unique_id: %s", ncclGetErrorString(r));
    static_assert(sizeof(uid.internal) == IQ2_COMM_ID_BYTES, "NCCL unique id size");
    std::memcpy(id, uid.internal, IQ2_COMM_ID_BYTES);
    return iq2::capi_ok();
}

int iq2_comm_init_with_timeout(const uint8_t* id, int world, int rank, uint32_t timeout_ms, iq2_comm_t* comm) {
    const char* op = "iq2_comm_init";
    if (id == nullptr || comm == nullptr) return capi_fail(IQ2_ERR_INVALID_ARGUMENT, "%s: NULL id or comm", op);
    *comm = nullptr;
    if (world < 1 || rank < 0 || rank >= world)
        return capi_fail(IQ2_ERR_INVALID_ARGUMENT, "%s: rank %d of world %d", op, rank, world);
    if (timeout_ms == 0) return capi_fail(IQ2_ERR_INVALID_ARGUMENT, "%s: zero timeout", op);
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return capi_fail(IQ2_ERR_DEVICE, "%s requires a CUDA device", op);
    ncclUniqueId uid;
    std::memcpy(uid.internal, id, IQ2_COMM_ID_BYTES);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;  // every NCCL call returns at once; the waits are polled and bounded here
    ncclComm_t c = nullptr;
    ncclResult_t r = ncclCommInitRankConfig(&c, world, uid, rank, &cfg);
    if (c != nullptr) r = iq2::nccl_settle(c, r, timeout_ms);
    if (r != ncclSuccess) {
        if (c != nullptr) ncclCommAbort(c);
        if (r == ncclInProgress)
            return capi_fail(IQ2_ERR_COMM, "%s: rank %d of %d: not every rank joined within %u ms; aborted", op, rank,
                             world, timeout_ms);
        return capi_fail(IQ2_ERR_COMM, "%s: %s", op, ncclGetErrorString(r));
    }
    auto* h = new iq2_comm_s{c, world, rank, dev};
    h->timeout_ms = timeout_ms;
    *comm = h;
    return iq2::capi_ok();
}

int iq2_comm_init(const uint8_t* id, int world, int rank, iq2_comm_t* comm) {
    return iq2_comm_init_with_timeout(id, world, rank, iq2::kDefaultCommTimeoutMs, comm);
}

namespace {

// Every rank reaches this point before any goes on (a one-element all-reduce), so that no rank
// unmaps or frees a region a peer may still store into.
// Bounded: ncclInProgress when the other ranks did not all arrive within the communicator's timeout.
ncclResult_t comm_barrier(iq2_comm_t comm, cudaStream_t s) {
    if (comm->aborted) return ncclInvalidUsage;
    float* one = nullptr;
    if (cudaMalloc(&one, sizeof(float)) != cudaSuccess) return ncclUnhandledCudaError;
    ncclResult_t r = iq2::nccl_settle(comm->nccl, ncclAllReduce(one, one, 1, ncclFloat, ncclSum, comm->nccl, s),
                                      comm->timeout_ms);
    if (r == ncclSuccess) r = iq2::stream_settle(comm, s);
    if (r == ncclSuccess) cudaFree(one);  // (while NCCL may still use it, the 4 bytes are left)
    return r;
}

void release_symmetric(iq2_comm_t comm) {
    for (int r = 0; r < comm->world && r < iq2::kMaxRanks; ++r)
        if (r != comm->rank && comm->peer[r] != nullptr) cudaIpcCloseMemHandle(comm->peer[r]);
    if (comm->symm != nullptr) cudaFree(comm->symm);
    comm->symm = nullptr;
    comm->symm_bytes = 0;
    for (auto& p : comm->peer) p = nullptr;
}

}  // namespace

int iq2_comm_destroy(iq2_comm_t comm) {
    if (comm == nullptr) return iq2::capi_ok();
    const char* op = "iq2_comm_destroy";
    ncclResult_t r = ncclSuccess;
    if (comm->symm != nullptr && !comm->aborted) {
        // no rank unmaps its region while a peer may still store into it
        cudaStream_t s = nullptr;
        cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
        r = comm_barrier(comm, s);
        if (r == ncclSuccess) cudaStreamDestroy(s);
    }
    int rc = IQ2_OK;
    if (!comm->aborted) {
        if (r == ncclSuccess) r = iq2::nccl_settle(comm->nccl, ncclCommFinalize(comm->nccl), comm->timeout_ms);
        if (r == ncclSuccess) ncclCommDestroy(comm->nccl);
        else rc = iq2::comm_failed(comm, op, "the final barrier", r);
    }
    // after an abort a peer may still hold this rank's region mapped: it is then left allocated
    if (comm->symm != nullptr && r == ncclSuccess) release_symmetric(comm);
    for (cudaStream_t x : comm->xs)
        if (x != nullptr) cudaStreamDestroy(x);
    for (cudaEvent_t e : comm->ev)
        if (e != nullptr) cudaEventDestroy(e);
    delete comm;
    return rc == IQ2_OK ? iq2::capi_ok() : rc;
}

int iq2_comm_symmetric_alloc(iq2_comm_t comm, size_t bytes, void** ptr) {
    const char* op = "iq2_comm_symmetric_alloc";
    if (comm == nullptr || ptr == nullptr) return capi_fail(IQ2_ERR_INVALID_ARGUMENT, "%s: NULL comm or ptr", op);
    *ptr = nullptr;
    if (bytes == 0) return capi_fail(IQ2_ERR_INVALID_ARGUMENT, "%s: zero bytes", op);
    if (comm->aborted) return capi_fail(IQ2_ERR_COMM, "%s: the communicator was aborted", op);
    if (comm->symm != nullptr) return capi_fail(IQ2_ERR_INVALID_ARGUMENT, "%s: the communicator already has one", op);
    if (comm->world > iq2::kMaxRanks)
        return capi_fail(IQ2_ERR_UNSUPPORTED, "%s: at most %d ranks, got %d", op, iq2::kMaxRanks, comm->world);
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev != comm->device)
        return capi_fail(IQ2_ERR_DEVICE, "%s: the current device is not the communicator's Cuda(%d)", op, comm->device);
    const size_t total = iq2::kSymmHeaderBytes + (bytes + 255) / 256 * 256;
    cudaStream_t s = nullptr;
    cudaError_t e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
    if (e != cudaSuccess) return iq2::capi_cuda_fail(op, e);
    // what every rank publishes: its IPC handle and its size (all sizes must agree, since a rank
    // stores into the others' regions at its own offsets)
    struct Entry {
        cudaIpcMemHandle_t handle;
        unsigned long long total;
    };
    uint8_t* base = nullptr;
    uint8_t* entries = nullptr;  // world entries, gathered on the device
    ncclResult_t nr = ncclSuccess;
    std::vector<Entry> h(comm->world);
    std::memset(h.data(), 0, sizeof(Entry) * h.size());
    e = cudaMalloc(&entries, sizeof(Entry) * comm->world);
    if (e != cudaSuccess) {
        cudaStreamDestroy(s);
        return iq2::capi_cuda_fail(op, e);
    }
    // a rank that fails here still takes part in the exchange (publishing size 0), so that all
    // ranks see the failure instead of waiting for it
    cudaError_t le = cudaMalloc(&base, total);
    if (le == cudaSuccess) le = cudaMemset(base, 0, total);  // zero header: no call entered yet
    if (le == cudaSuccess) le = cudaIpcGetMemHandle(&h[comm->rank].handle, base);
    h[comm->rank].total = le == cudaSuccess ? total : 0ull;
    e = cudaMemcpy(entries + sizeof(Entry) * comm->rank, &h[comm->rank], sizeof(Entry), cudaMemcpyHostToDevice);
    nr = iq2::nccl_settle(comm->nccl,
                          ncclAllGather(entries + sizeof(Entry) * comm->rank, entries, sizeof(Entry), ncclUint8,
                                        comm->nccl, s),
                          comm->timeout_ms);
    if (nr == ncclSuccess) nr = iq2::stream_settle(comm, s);
    if (nr != ncclSuccess) {
        // the other ranks did not all take part: nothing was mapped; give up on the communicator
        const int rc = iq2::comm_failed(comm, op, "the handle exchange", nr);
        if (base != nullptr) cudaFree(base);
        return rc;
    }
    if (e == cudaSuccess && nr == ncclSuccess)
        e = cudaMemcpy(h.data(), entries, sizeof(Entry) * comm->world, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = le;
    bool same_size = true;
    for (int r = 0; r < comm->world; ++r) same_size = same_size && h[r].total == total;
    comm->symm = base;
    comm->peer[comm->rank] = base;
    for (int r = 0; r < comm->world && same_size && e == cudaSuccess && nr == ncclSuccess; ++r)
        if (r != comm->rank) e = cudaIpcOpenMemHandle(&comm->peer[r], h[r].handle, cudaIpcMemLazyEnablePeerAccess);
    // every rank takes part in this barrier whatever happened above, so none is left waiting
    const ncclResult_t br = comm_barrier(comm, s);  // every rank has mapped every region
    if (br != ncclSuccess) {
        const int rc = iq2::comm_failed(comm, op, "the mapping barrier", br);
        comm->symm = nullptr;  // a peer may have mapped it: left allocated
        for (auto& q : comm->peer) q = nullptr;
        return rc;
    }
    if (entries != nullptr) cudaFree(entries);
    cudaStreamDestroy(s);
    if (e != cudaSuccess || nr != ncclSuccess || !same_size) {
        release_symmetric(comm);
        if (e != cudaSuccess) return iq2::capi_cuda_fail(op, e);
        if (nr != ncclSuccess) return capi_fail(IQ2_ERR_COMM, "%s: %s", op, ncclGetErrorString(nr));
        return capi_fail(IQ2_ERR_INVALID_ARGUMENT, "%s: the ranks asked for different sizes", op);
    }
    comm->symm_bytes = total - iq2::kSymmHeaderBytes;
    *ptr = base + iq2::kSymmHeaderBytes;
    return iq2::capi_ok();
}

int iq2_comm_check(iq2_comm_t comm) {
    if (comm == nullptr) return capi_fail(IQ2_ERR_INVALID_ARGUMENT, "iq2_comm_check: NULL comm");
    if (comm->aborted)
        return capi_fail(IQ2_ERR_COMM, "iq2_comm_check: the communicator was aborted after a wait on the other "
                                       "ranks ran out or NCCL failed");
    ncclResult_t st = ncclSuccess;
    if (ncclCommGetAsyncError(comm->nccl, &st) == ncclSuccess && st != ncclSuccess && st != ncclInProgress)
        return iq2::comm_failed(comm, "iq2_comm_check", "NCCL", st);
    if (comm->symm == nullptr) return iq2::capi_ok();
    unsigned err = 0;
    const cudaError_t e = cudaMemcpy(&err, &reinterpret_cast<iq2::SymmHeader*>(comm->symm)->err, sizeof(err),
                                     cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return iq2::capi_cuda_fail("iq2_comm_check", e);
    if (err != 0) {
        std::string why;
        if (err & 1u) why += "a rank never entered a call";
        if (err & 2u) why += std::string(why.empty() ? "" : ", ") + "a rank never finished a call";
        if (err & 4u) why += std::string(why.empty() ? "" : ", ") + "a call failed on this rank before its launch";
        return capi_fail(IQ2_ERR_COMM,
                         "iq2_comm_check: a peer exchange failed (%s); the outputs of that call and of every later "
                         "fused call of this communicator hold this rank's columns only (destroy the communicator "
                         "to recover)",
                         why.c_str());
    }
    return iq2::capi_ok();
}

size_t iq2_matmul_grouped_sharded_workspace_size(const iq2_matmul_problem* problems, uint32_t count, uint32_t m,
                                                 int x_dtype, int world) {
    if (problems == nullptr || count == 0 || m == 0 || world < 1) return 0;
    const iq2::ShardPlan pl = iq2::plan_shards(problems, count, m, world);
    if (iq2::use_pipeline(m, count, world)) {
        // the chunks' GEMMs run one after another on the caller's stream and share the scratch
        size_t inner = 0;
        for (const iq2::Chunk& c : iq2::plan_chunks(problems, count, m, world)) {
            const iq2_matmul_problem q = iq2::chunk_problem(problems[c.i], c, x_dtype, world, nullptr);
            inner = std::max(inner, iq2_matmul_grouped_workspace_size(&q, 1, c.mlen, x_dtype));
        }
        return pl.packed_bytes + iq2::align256(pl.per_rank * world * sizeof(float)) + inner;
    }
    std::vector<iq2_matmul_problem> loc = iq2::local_problems(problems, count, m, world, pl, nullptr);
    return pl.inner_off + iq2_matmul_grouped_workspace_size(loc.data(), count, m, x_dtype);
}

int iq2_matmul_grouped_sharded(iq2_comm_t comm, const iq2_matmul_problem* problems, uint32_t count, uint32_t m,
                               int x_dtype, void* workspace, size_t workspace_bytes, iq2_stream_t stream) {
    const char* op = "iq2_matmul_grouped_sharded";
    if (comm == nullptr) return capi_fail(IQ2_ERR_INVALID_ARGUMENT, "%s: NULL comm", op);
    if (count == 0 || m == 0) return iq2::capi_ok();
    if (problems == nullptr) return capi_fail(IQ2_ERR_INVALID_ARGUMENT, "%s: NULL problems", op);
    if (count > iq2::SCATTER_CAP)
        return capi_fail(IQ2_ERR_UNSUPPORTED, "%s: at most %u projections per call, got %u", op, iq2::SCATTER_CAP,
                         count);
    if (comm->aborted) return capi_fail(IQ2_ERR_COMM, "%s: the communicator was aborted", op);
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev != comm->device)
        return capi_fail(IQ2_ERR_DEVICE, "%s: the current device is not the communicator's Cuda(%d)", op,
                         comm->device);
    for (uint32_t i = 0; i < count; ++i) {
        if (problems[i].out_dim == 0 || problems[i].in_dim == 0)
            return capi_fail(IQ2_ERR_ZERO_DIM, "iq2_matmul expects non-zero dimensions");
        if (problems[i].out_dim % (uint32_t)comm->world != 0)
            return capi_fail(IQ2_ERR_INVALID_ARGUMENT, "%s: problem %u: out_dim %u is not a multiple of the world size %d",
                             op, i, problems[i].out_dim, comm->world);
        if (problems[i].out == nullptr) return capi_fail(IQ2_ERR_INVALID_ARGUMENT, "%s: problem %u: NULL out", op, i);
    }
    if (iq2::use_peer_path(comm, problems, count, m))
        return iq2::sharded_peer(comm, problems, count, m, x_dtype, workspace, workspace_bytes, stream);
    const iq2::ShardPlan pl = iq2::plan_shards(problems, count, m, comm->world);
    const size_t need = iq2_matmul_grouped_sharded_workspace_size(problems, count, m, x_dtype, comm->world);
    if (workspace == nullptr || workspace_bytes < need)
        return capi_fail(IQ2_ERR_WORKSPACE, "%s: workspace of %zu bytes needed, got %zu", op, need,
                         workspace ? workspace_bytes : (size_t)0);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    if (iq2::use_pipeline(m, count, comm->world))
        return iq2::sharded_pipelined(comm, problems, count, m, x_dtype, ws, workspace_bytes, stream);
    float* packed = reinterpret_cast<float*>(ws);
    std::vector<iq2_matmul_problem> loc = iq2::local_problems(problems, count, m, comm->world, pl, packed);
    // 1. this rank's slices (the grouped call validates every slice like iq2_matmul does)
    int rc = iq2_matmul_grouped(loc.data(), count, m, x_dtype, ws + pl.inner_off, workspace_bytes - pl.inner_off,
                                stream);
    if (rc != IQ2_OK) return rc;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    // 2. every rank's slices, rank-major
    float* gathered = pl.direct ? problems[0].out : reinterpret_cast<float*>(ws + pl.packed_bytes);
    // (enqueued on the stream; a non-blocking communicator may still be connecting: bounded)
    const ncclResult_t r =
        iq2::nccl_settle(comm->nccl, ncclAllGather(packed, gathered, pl.per_rank, ncclFloat, comm->nccl, s),
                         comm->timeout_ms);
    if (r != ncclSuccess) return iq2::comm_failed(comm, op, "ncclAllGather", r);
    if (pl.direct) return iq2::capi_ok();
    // 3. slices -> each projection's [m, out_dim]
    iq2::ScatterLaunch L;
    std::memset(&L, 0, sizeof(L));
    L.gathered = gathered;
    L.per_rank = pl.per_rank;
    L.world = (uint32_t)comm->world;
    L.m = m;
    for (uint32_t i = 0; i < count; ++i) {
        L.item[i].out = problems[i].out;
        L.item[i].off = pl.off[i];
        L.item[i].n_loc = problems[i].out_dim / (uint32_t)comm->world;
    }
    const unsigned bx = (unsigned)std::min<uint64_t>((uint64_t)m * comm->world, 1184);
    iq2::scatter_slices_kernel<<<dim3(bx, count), 256, 0, s>>>(L);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return iq2::capi_cuda_fail(op, e);
    return iq2::capi_ok();
}

}  // extern "C"
