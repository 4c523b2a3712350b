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

// One CTA per gathered row: the owner is the last shard whose first row is
// <= the global row; 16-byte loads, four in flight per thread.
__global__ void __launch_bounds__(256) gather_rows_kernel(GatherShards sh, const int32_t* __restrict__ idx,
                                                          char* __restrict__ out, uint32_t* status) {
    pdl_enter();
    const int i = blockIdx.x;
    const int64_t r = idx[i];
    const int64_t nvec = sh.row_bytes / 16;
    uint4* dst = reinterpret_cast<uint4*>(out + static_cast<int64_t>(i) * sh.row_bytes);
    int p = -1;
    if (r >= sh.row_lo[0] && r < sh.row_lo[sh.world])
        for (int q = 0; q < sh.world; ++q)
            if (r >= sh.row_lo[q] && r < sh.row_lo[q + 1]) p = q;
    if (p < 0) {
        if (threadIdx.x == 0) raise_status(status, DWA_STATUS_BAD_ROW_INDEX);
        for (int64_t v = threadIdx.x; v < nvec; v += blockDim.x) dst[v] = make_uint4(0, 0, 0, 0);
        return;
    }
    const uint4* src = reinterpret_cast<const uint4*>(sh.base[p] + (r - sh.row_lo[p]) * sh.row_bytes);
    for (int64_t v0 = threadIdx.x; v0 < nvec; v0 += 4 * blockDim.x) {
        uint4 t[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int64_t v = v0 + u * blockDim.x;
            if (v < nvec) t[u] = src[v];
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int64_t v = v0 + u * blockDim.x;
            if (v < nvec) dst[v] = t[u];
        }
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
    DWA_TIMED("gather_rows", st, launch_pdl(gather_rows_kernel, n, 256, 0, st, sh, indices, static_cast<char*>(out),
                                            static_cast<uint32_t*>(workspace)));
    DWA_LAUNCH_CHECK("gather_rows_kernel");
    ++g_launches_total;
    return DWA_OK;
}
