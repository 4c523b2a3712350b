// Peer access to a row-sharded pool (one process per GPU on one node): CUDA
// IPC handles of each rank's shard, and the gather of pool rows by global index
// from whichever rank holds them (plain 16-byte loads; over NVLink when the row
// is a peer's).  This is how the assembly of a rank's sequences reads winning
// rows that live on other ranks (replaces _distributed_gather's masked psum,
// src/dwa/model.py:16-47, which all-reduces B*k*D values over the model axis).

#include <atomic>
#include <cstring>
#include <mutex>

#include <cuda.h>

#include "dwa_common.cuh"

namespace dwa {

extern std::atomic<uint64_t> g_launches_total;

constexpr int kMaxShards = 16;

struct GatherShards {
    int world;
    int64_t row_bytes;
    const char* base[kMaxShards];
    int64_t row_lo[kMaxShards + 1];
};

using PFN_addr_range = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

static PFN_addr_range addr_range_fn() {
    static PFN_addr_range fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_addr_range>(p);
    });
    return fn;
}

// One CTA per (16 KB chunk, gathered row): the owner is the last shard whose
// first row is <= the global row; 16-byte loads, four in flight per thread,
// so each CTA makes one round trip (over NVLink for a peer's row) and the
// chunks of a row are fetched at once.
constexpr int kGatherThreads = 256, kGatherUnroll = 4;
constexpr int64_t kGatherChunkVecs = kGatherThreads * kGatherUnroll;

__global__ void __launch_bounds__(kGatherThreads) gather_rows_kernel(GatherShards sh, const int32_t* __restrict__ idx,
                                                                     char* __restrict__ out, uint32_t* status) {
    pdl_enter();
    const int i = blockIdx.y;
    const int64_t r = idx[i];
    const int64_t nvec = sh.row_bytes / 16;
    const int64_t v0 = static_cast<int64_t>(blockIdx.x) * kGatherChunkVecs + threadIdx.x;
    uint4* dst = reinterpret_cast<uint4*>(out + static_cast<int64_t>(i) * sh.row_bytes);
    int p = -1;
    if (r >= sh.row_lo[0] && r < sh.row_lo[sh.world])
        for (int q = 0; q < sh.world; ++q)
            if (r >= sh.row_lo[q] && r < sh.row_lo[q + 1]) p = q;
    if (p < 0) {
        if (threadIdx.x == 0 && blockIdx.x == 0) raise_status(status, DWA_STATUS_BAD_ROW_INDEX);
#pragma unroll
        for (int u = 0; u < kGatherUnroll; ++u) {
            const int64_t v = v0 + u * kGatherThreads;
            if (v < nvec) dst[v] = make_uint4(0, 0, 0, 0);
        }
        return;
    }
    const uint4* src = reinterpret_cast<const uint4*>(sh.base[p] + (r - sh.row_lo[p]) * sh.row_bytes);
    uint4 t[kGatherUnroll];
#pragma unroll
    for (int u = 0; u < kGatherUnroll; ++u) {
        const int64_t v = v0 + u * kGatherThreads;
        if (v < nvec) t[u] = src[v];
    }
#pragma unroll
    for (int u = 0; u < kGatherUnroll; ++u) {
        const int64_t v = v0 + u * kGatherThreads;
        if (v < nvec) dst[v] = t[u];
    }
}

}  // namespace dwa

using namespace dwa;

extern "C" size_t dwa_ipc_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

extern "C" int dwa_ipc_handle(const void* ptr, void* handle, int64_t* offset) {
    if (!ptr || !handle || !offset) return fail(DWA_ERR_INVALID_ARG, "a required pointer is NULL");
    PFN_addr_range range = addr_range_fn();
    if (!range) return fail(DWA_ERR_CUDA, "cuMemGetAddressRange is not available");
    CUdeviceptr base = 0;
    size_t size = 0;
    if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
        return fail(DWA_ERR_INVALID_ARG, "ptr is not inside a device allocation");
    cudaIpcMemHandle_t h;
    DWA_CUDA_TRY(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
    std::memcpy(handle, &h, sizeof h);
    *offset = static_cast<int64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
    return DWA_OK;
}

extern "C" int dwa_ipc_open(const void* handle, int64_t offset, void** ptr) {
    if (!handle || !ptr || offset < 0) return fail(DWA_ERR_INVALID_ARG, "bad handle, offset or ptr");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof h);
    void* base = nullptr;
    DWA_CUDA_TRY(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess));
    *ptr = static_cast<char*>(base) + offset;
    return DWA_OK;
}

extern "C" int dwa_ipc_close(void* ptr, int64_t offset) {
    if (!ptr || offset < 0) return fail(DWA_ERR_INVALID_ARG, "bad ptr or offset");
    DWA_CUDA_TRY(cudaIpcCloseMemHandle(static_cast<char*>(ptr) - offset));
    return DWA_OK;
}

extern "C" size_t dwa_gather_rows_workspace_bytes(void) { return 256; }

extern "C" int dwa_gather_rows(void* stream, int n, int64_t D, int dtype, const int32_t* indices,
                               const DwaPoolShards* shards, void* out, void* workspace,
                               size_t workspace_bytes) {
    if (n < 0 || D <= 0) return fail(DWA_ERR_INVALID_ARG, "n must be >= 0 and D > 0");
    if (dtype != DWA_F32 && dtype != DWA_BF16) return fail(DWA_ERR_INVALID_ARG, "dtype must be DWA_F32 or DWA_BF16");
    if (!shards || shards->world <= 0 || shards->world > kMaxShards || !shards->bases || !shards->row_lo)
        return fail(DWA_ERR_INVALID_ARG, "shards: 1..16 ranks with bases and row_lo");
    if (n > 0 && (!indices || !out)) return fail(DWA_ERR_INVALID_ARG, "a required pointer is NULL");
    if (!workspace || reinterpret_cast<uintptr_t>(workspace) % 256 != 0 || workspace_bytes < 256)
        return fail(DWA_ERR_WORKSPACE, "workspace: 256 bytes, 256-byte aligned");
    GatherShards sh{};
    sh.world = shards->world;
    sh.row_bytes = D * static_cast<int64_t>(dtype_bytes(dtype));
    if (sh.row_bytes % 16 != 0 || reinterpret_cast<uintptr_t>(out) % 16 != 0)
        return fail(DWA_ERR_UNSUPPORTED, "rows and out must be 16-byte multiples / aligned");
    for (int p = 0; p <= sh.world; ++p) sh.row_lo[p] = shards->row_lo[p];
    for (int p = 0; p < sh.world; ++p) {
        if (sh.row_lo[p + 1] < sh.row_lo[p]) return fail(DWA_ERR_INVALID_ARG, "row_lo must be non-decreasing");
        sh.base[p] = static_cast<const char*>(shards->bases[p]);
        if (sh.row_lo[p + 1] > sh.row_lo[p] && (!sh.base[p] || reinterpret_cast<uintptr_t>(sh.base[p]) % 16 != 0))
            return fail(DWA_ERR_INVALID_ARG, "a non-empty shard needs a 16-byte aligned base");
    }
    if (n == 0) return DWA_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (n > 65535) return fail(DWA_ERR_UNSUPPORTED, "dwa_gather_rows: at most 65535 rows per call");
    const int64_t chunks = (sh.row_bytes / 16 + kGatherChunkVecs - 1) / kGatherChunkVecs;
    DWA_TIMED("gather_rows", st, launch_pdl(gather_rows_kernel, dim3(static_cast<unsigned>(chunks), n),
                                            kGatherThreads, 0, st, sh, indices, static_cast<char*>(out),
                                            static_cast<uint32_t*>(workspace)));
    DWA_LAUNCH_CHECK("gather_rows_kernel");
    ++g_launches_total;
    return DWA_OK;
}

// ---------------------------------------------------------------------------
// All-gather among the ranks of one node through exchange buffers every rank
// has mapped (dwa_peer_allgather).  Layout of a rank's exchange buffer:
//   [0, 4096)        flags: word 32*q holds the last call rank q has finished
//                    writing into this buffer (one 128-byte line per source)
//   [4096, 4100)     this rank's call counter (never written by peers)
//   [4100, 4104)     this rank's status bits (DWA_STATUS_WAIT_TIMEOUT)
//   [8192, ...)      two halves of world slots of `bytes`; call e writes half
//                    e % 2, so a rank one call ahead never overwrites a slot
//                    its owner is still reading
// One CTA per call: it copies the input into slot `rank` of every rank's
// half (16-byte stores, over NVLink for peers), fences at system scope,
// stores its flag into every peer with release semantics, waits (bounded,
// kWaitLimitNs) for every peer's flag of this call, and copies the gathered
// half to `out`.  Replaces an NCCL all-gather of a few kilobytes per rank,
// whose fixed cost is tens of microseconds per call.
// ---------------------------------------------------------------------------
namespace dwa {

constexpr int kMaxGatherRanks = 16;
constexpr int64_t kGatherFlagBytes = 4096, kGatherCounter = 4096, kGatherStatus = 4100, kGatherData = 8192;

struct GatherPeers {
    char* buf[kMaxGatherRanks];
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __launch_bounds__(512) peer_allgather_kernel(GatherPeers peers, int rank, int world,
                                                             const uint4* __restrict__ src, int64_t n16,
                                                             uint4* __restrict__ out) {
    __shared__ uint32_t s_call;
    __shared__ int s_fail;
    char* mine = peers.buf[rank];
    uint32_t* counter = reinterpret_cast<uint32_t*>(mine + kGatherCounter);
    uint32_t* status = reinterpret_cast<uint32_t*>(mine + kGatherStatus);
    pdl_enter();
    if (threadIdx.x == 0) {
        s_call = *counter + 1u;
        s_fail = 0;
    }
    __syncthreads();
    const uint32_t e = s_call;
    const int64_t half = static_cast<int64_t>(e & 1u) * world * n16;
    for (int d = 0; d < world; ++d) {
        uint4* dst = reinterpret_cast<uint4*>(peers.buf[d] + kGatherData) + half + static_cast<int64_t>(rank) * n16;
        for (int64_t i = threadIdx.x; i < n16; i += blockDim.x) dst[i] = src[i];
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        for (int d = 0; d < world; ++d)
            if (d != rank) st_release_sys(reinterpret_cast<uint32_t*>(peers.buf[d]) + 32 * rank, e);
    }
    if (threadIdx.x < world && static_cast<int>(threadIdx.x) != rank) {
        const uint32_t* flag = reinterpret_cast<const uint32_t*>(mine) + 32 * threadIdx.x;
        if (static_cast<int32_t>(ld_acquire_sys(flag) - e) < 0) {
            const uint64_t t0 = global_timer_ns();
            while (static_cast<int32_t>(ld_acquire_sys(flag) - e) < 0) {
                if (global_timer_ns() - t0 > kWaitLimitNs) {
                    atomicOr(status, DWA_STATUS_WAIT_TIMEOUT);
                    s_fail = 1;
                    break;
                }
            }
        }
    }
    __syncthreads();
    const uint4* got = reinterpret_cast<const uint4*>(mine + kGatherData) + half;
    for (int64_t i = threadIdx.x; i < world * n16; i += blockDim.x) out[i] = got[i];
    if (threadIdx.x == 0 && !s_fail) *counter = e;
}

}  // namespace dwa

extern "C" size_t dwa_peer_allgather_buffer_bytes(int world, size_t bytes) {
    if (world <= 0 || world > dwa::kMaxGatherRanks) return 0;
    return static_cast<size_t>(dwa::kGatherData) + 2 * static_cast<size_t>(world) * bytes;
}

extern "C" int dwa_peer_allgather(void* stream, int rank, int world, const void* src, size_t bytes,
                                  void* const* peer_buffers, void* out) {
    using namespace dwa;
    if (world <= 0 || world > kMaxGatherRanks || rank < 0 || rank >= world)
        return fail(DWA_ERR_INVALID_ARG, "peer all-gather: 1..16 ranks and 0 <= rank < world");
    if (!src || !out || !peer_buffers) return fail(DWA_ERR_INVALID_ARG, "a required pointer is NULL");
    if (bytes == 0 || bytes % 16 != 0 || reinterpret_cast<uintptr_t>(src) % 16 != 0 ||
        reinterpret_cast<uintptr_t>(out) % 16 != 0)
        return fail(DWA_ERR_UNSUPPORTED, "peer all-gather: bytes a non-zero multiple of 16, 16-byte aligned src/out");
    GatherPeers pe{};
    for (int r = 0; r < world; ++r) {
        pe.buf[r] = static_cast<char*>(peer_buffers[r]);
        if (!pe.buf[r] || reinterpret_cast<uintptr_t>(pe.buf[r]) % 256 != 0)
            return fail(DWA_ERR_INVALID_ARG, "peer all-gather: every exchange buffer 256-byte aligned");
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    DWA_TIMED("peer_allgather", st,
              launch_pdl(peer_allgather_kernel, 1, 512, 0, st, pe, rank, world, static_cast<const uint4*>(src),
                         static_cast<int64_t>(bytes / 16), static_cast<uint4*>(out)));
    DWA_LAUNCH_CHECK("peer_allgather_kernel");
    ++g_launches_total;
    return DWA_OK;
}

extern "C" int dwa_peer_allgather_status(void* stream, const void* buffer, uint32_t* status, int clear) {
    using namespace dwa;
    if (!buffer || !status) return fail(DWA_ERR_INVALID_ARG, "a required pointer is NULL");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    char* p = static_cast<char*>(const_cast<void*>(buffer)) + kGatherStatus;
    DWA_CUDA_TRY(cudaMemcpyAsync(status, p, sizeof(uint32_t), cudaMemcpyDeviceToHost, st));
    DWA_CUDA_TRY(cudaStreamSynchronize(st));
    if (clear) DWA_CUDA_TRY(cudaMemsetAsync(p, 0, sizeof(uint32_t), st));
    return DWA_OK;
}
