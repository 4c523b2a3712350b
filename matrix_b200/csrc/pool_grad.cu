// Pool-row gradient scatter: the VJP of the gather pool[indices]
// (src/dwa/model.py:193-195, and of _distributed_gather, model.py:16-47).
//   g_pool[row - row_lo, :] += sum of g_rows[i, :] over the i with indices[i] == row
// for the rows inside this call's window [row_lo, row_hi) (the whole pool, or
// one rank's rows).  Deterministic: one CTA sorts the (row, i) pairs (bitonic,
// in shared memory), then one CTA per (unique row, column chunk) adds that row's
// contributions in ascending i in fp32 and updates the gradient row once (f32,
// or bf16 rounded once).  Rows outside [0, n_global) raise
// DWA_STATUS_BAD_ROW_INDEX and are skipped.

#include <atomic>

#include "dwa_common.cuh"

namespace dwa {

extern std::atomic<uint64_t> g_launches_total;

constexpr int kScatterMaxN = 8192;   // contributions per call (one CTA sorts them)
constexpr int kScatterCols = 1024;   // columns per CTA of the add

// order[j] = i of the j-th (row, i) in ascending order; seg[0..nseg] = segment
// starts over order; nseg stored at seg[kScatterMaxN + 1].
__global__ void __launch_bounds__(1024) scatter_sort_kernel(const int32_t* __restrict__ idx, int n,
                                                           int64_t n_global, int64_t row_lo, int64_t row_hi,
                                                           int32_t* __restrict__ order, int32_t* __restrict__ seg,
                                                           uint32_t* status) {
    pdl_enter();
    extern __shared__ uint64_t key[];   // [np2]
    int np2 = 1;
    while (np2 < n) np2 <<= 1;
    for (int i = threadIdx.x; i < np2; i += blockDim.x) {
        uint64_t k = ~0ull;   // padding and rows outside the window sort last
        if (i < n) {
            const int64_t r = idx[i];
            if (r == DWA_PAD_INDEX) {
                // a padding slot: no contribution
            } else if (r < 0 || r >= n_global) raise_status(status, DWA_STATUS_BAD_ROW_INDEX);
            else if (r >= row_lo && r < row_hi) k = (static_cast<uint64_t>(r - row_lo) << 32) | static_cast<uint32_t>(i);
        }
        key[i] = k;
    }
    __syncthreads();
    for (int size = 2; size <= np2; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < np2; i += blockDim.x) {
                const int j = i ^ stride;
                if (j > i) {
                    const bool up = (i & size) == 0;
                    const uint64_t a = key[i], b = key[j];
                    if ((a > b) == up) { key[i] = b; key[j] = a; }
                }
            }
            __syncthreads();
        }
    }
    // order, then the segment starts (j where the row changes) compacted in
    // order by one warp's ballots; the valid keys come first after the sort
    for (int j = threadIdx.x; j < n; j += blockDim.x)
        order[j] = key[j] == ~0ull ? -1 : static_cast<int32_t>(key[j] & 0xffffffffu);
    if (threadIdx.x < 32) {
        int base = 0, valid = 0;
        for (int j0 = 0; j0 < n; j0 += 32) {
            const int j = j0 + threadIdx.x;
            const uint64_t k = j < n ? key[j] : ~0ull;
            const bool start = k != ~0ull && (j == 0 || (key[j - 1] >> 32) != (k >> 32));
            const unsigned m = __ballot_sync(0xffffffffu, start);
            if (start) seg[base + __popc(m & ((1u << threadIdx.x) - 1))] = j;
            base += __popc(m);
            valid += __popc(__ballot_sync(0xffffffffu, k != ~0ull));
        }
        if (threadIdx.x == 0) {
            seg[base] = valid;                 // end of the last segment
            seg[kScatterMaxN + 1] = base;      // number of segments
        }
    }
}

template <class TG, class TR>
__global__ void __launch_bounds__(256) scatter_add_kernel(const int32_t* __restrict__ idx,
                                                          const TR* __restrict__ g_rows, int D,
                                                          const int32_t* __restrict__ order,
                                                          const int32_t* __restrict__ seg, int64_t row_lo,
                                                          TG* __restrict__ g_pool) {
    pdl_enter();
    const int s = blockIdx.x;
    if (s >= seg[kScatterMaxN + 1]) return;
    const int j0 = seg[s], j1 = seg[s + 1];
    const int64_t row = static_cast<int64_t>(idx[order[j0]]) - row_lo;
    for (int c = blockIdx.y * kScatterCols + threadIdx.x; c < D && c < (blockIdx.y + 1) * kScatterCols;
         c += blockDim.x) {
        float acc = 0.f;
        for (int j = j0; j < j1; ++j) acc += Elem<TR>::to_f(g_rows[static_cast<int64_t>(order[j]) * D + c]);
        TG* p = g_pool + row * D + c;
        *p = Elem<TG>::from_f(Elem<TG>::to_f(*p) + acc);
    }
}

// Returning row gradients to the ranks that own the rows: CTA i takes
// contribution i of this rank (slot rank*slot + i of every owner's receive
// area).  The owner of indices[i] gets the row, converted to the receive
// dtype with 16-byte stores, and the index; every other owner gets the pad
// index in that slot, so that each area holds exactly this call's rows.
constexpr int kMaxOwners = 16;
struct RecvAreas {
    int world;
    int slot;
    int64_t D;
    char* base[kMaxOwners];            // each owner's area: idx [world*slot] int32, then rows
    int64_t row_lo[kMaxOwners + 1];
    int64_t rows_off;                  // byte offset of the rows in an area
};

template <class TO>
__global__ void __launch_bounds__(256) grad_send_kernel(RecvAreas ra, int rank, int n,
                                                        const int32_t* __restrict__ indices,
                                                        const float* __restrict__ g_rows, uint32_t* status) {
    pdl_enter();
    const int i = blockIdx.x;
    const int64_t slot = static_cast<int64_t>(rank) * ra.slot + i;
    int o = -1;
    int32_t r = DWA_PAD_INDEX;
    if (i < n) {
        r = indices[i];
        for (int q = 0; q < ra.world; ++q)
            if (r >= ra.row_lo[q] && r < ra.row_lo[q + 1]) o = q;
        if (o < 0) {
            if (threadIdx.x == 0) raise_status(status, DWA_STATUS_BAD_ROW_INDEX);
            r = DWA_PAD_INDEX;
        }
    }
    if (threadIdx.x < ra.world)
        reinterpret_cast<int32_t*>(ra.base[threadIdx.x])[slot] = threadIdx.x == o ? r : DWA_PAD_INDEX;
    if (o >= 0) {
        const float* src = g_rows + static_cast<int64_t>(i) * ra.D;
        TO* dst = reinterpret_cast<TO*>(ra.base[o] + ra.rows_off) + slot * ra.D;
        if constexpr (sizeof(TO) == 2) {
            // 8 elements per thread and step: two float4 loads, one 16-byte store
            for (int64_t c = static_cast<int64_t>(threadIdx.x) * 8; c + 8 <= ra.D; c += 8 * blockDim.x) {
                const float4 a = *reinterpret_cast<const float4*>(src + c);
                const float4 b = *reinterpret_cast<const float4*>(src + c + 4);
                __nv_bfloat162 h[4] = {__floats2bfloat162_rn(a.x, a.y), __floats2bfloat162_rn(a.z, a.w),
                                       __floats2bfloat162_rn(b.x, b.y), __floats2bfloat162_rn(b.z, b.w)};
                *reinterpret_cast<uint4*>(dst + c) = *reinterpret_cast<const uint4*>(h);
            }
        } else {
            for (int64_t c = static_cast<int64_t>(threadIdx.x) * 4; c + 4 <= ra.D; c += 4 * blockDim.x)
                *reinterpret_cast<float4*>(dst + c) = *reinterpret_cast<const float4*>(src + c);
        }
    }
    // the owner reads the area after a collective that follows this kernel
    __threadfence_system();
}

}  // namespace dwa

using namespace dwa;

extern "C" size_t dwa_pool_grad_scatter_workspace_bytes(int n) {
    if (n <= 0 || n > kScatterMaxN) return 0;
    return 256 + align_up(static_cast<size_t>(n) * 4, 256) + align_up((kScatterMaxN + 2) * 4, 256);
}

extern "C" int dwa_pool_grad_scatter(void* stream, int n, int D, const int32_t* indices, const float* g_rows,
                                     int64_t n_global, int64_t row_lo, int64_t row_hi, int g_dtype,
                                     void* g_pool, void* workspace, size_t workspace_bytes) {
    return dwa_pool_grad_scatter_typed(stream, n, D, indices, DWA_F32, g_rows, n_global, row_lo, row_hi, g_dtype,
                                       g_pool, workspace, workspace_bytes);
}

extern "C" int dwa_pool_grad_scatter_typed(void* stream, int n, int D, const int32_t* indices, int rows_dtype,
                                           const void* g_rows, int64_t n_global, int64_t row_lo, int64_t row_hi,
                                           int g_dtype, void* g_pool, void* workspace, size_t workspace_bytes) {
    if (rows_dtype != DWA_F32 && rows_dtype != DWA_BF16)
        return fail(DWA_ERR_INVALID_ARG, "rows_dtype must be DWA_F32 or DWA_BF16");
    if (n <= 0 || D <= 0) return fail(DWA_ERR_INVALID_ARG, "n and D must be positive");
    if (n > kScatterMaxN) return fail(DWA_ERR_UNSUPPORTED, "more than 8192 contributions per call");
    if (n_global <= 0 || n_global >= (int64_t(1) << 31) || row_lo < 0 || row_hi < row_lo || row_hi > n_global)
        return fail(DWA_ERR_INVALID_ARG, "need 0 <= row_lo <= row_hi <= n_global < 2^31");
    if (g_dtype != DWA_F32 && g_dtype != DWA_BF16) return fail(DWA_ERR_INVALID_ARG, "g_dtype must be DWA_F32 or DWA_BF16");
    if (!indices || !g_rows || (!g_pool && row_hi > row_lo)) return fail(DWA_ERR_INVALID_ARG, "a required pointer is NULL");
    if (!workspace || reinterpret_cast<uintptr_t>(workspace) % 256 != 0)
        return fail(DWA_ERR_WORKSPACE, "workspace must be non-NULL and 256-byte aligned");
    if (workspace_bytes < dwa_pool_grad_scatter_workspace_bytes(n)) return fail(DWA_ERR_WORKSPACE, "workspace too small");
    if (row_hi == row_lo) return DWA_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    char* w = static_cast<char*>(workspace);
    uint32_t* status = reinterpret_cast<uint32_t*>(w);
    int32_t* order = reinterpret_cast<int32_t*>(w + 256);
    int32_t* seg = reinterpret_cast<int32_t*>(w + 256 + align_up(static_cast<size_t>(n) * 4, 256));
    int np2 = 1;
    while (np2 < n) np2 <<= 1;
    const size_t sh = static_cast<size_t>(np2) * 8;
    if (sh > 48 * 1024) {
        int dev = 0;
        DWA_CUDA_TRY(cudaGetDevice(&dev));
        static bool attr_set[64] = {};
        if (dev < 0 || dev >= 64 || !attr_set[dev]) {
            DWA_CUDA_TRY(cudaFuncSetAttribute(scatter_sort_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              kScatterMaxN * 8));
            if (dev >= 0 && dev < 64) attr_set[dev] = true;
        }
    }
    DWA_TIMED("scatter_sort", st, launch_pdl(scatter_sort_kernel, 1, 1024, sh, st, indices, n, n_global, row_lo, row_hi,
                                                                         order, seg, status));
    DWA_LAUNCH_CHECK("scatter_sort_kernel");
    const dim3 g(static_cast<unsigned>(n), static_cast<unsigned>((D + kScatterCols - 1) / kScatterCols));
    using bf = __nv_bfloat16;
    const bool rb = rows_dtype == DWA_BF16;
    if (g_dtype == DWA_BF16 && rb)
        DWA_TIMED("scatter_add", st, launch_pdl(scatter_add_kernel<bf, bf>, g, 256, 0, st, indices,
                                                static_cast<const bf*>(g_rows), D, order, seg, row_lo, static_cast<bf*>(g_pool)));
    else if (g_dtype == DWA_BF16)
        DWA_TIMED("scatter_add", st, launch_pdl(scatter_add_kernel<bf, float>, g, 256, 0, st, indices,
                                                static_cast<const float*>(g_rows), D, order, seg, row_lo, static_cast<bf*>(g_pool)));
    else if (rb)
        DWA_TIMED("scatter_add", st, launch_pdl(scatter_add_kernel<float, bf>, g, 256, 0, st, indices,
                                                static_cast<const bf*>(g_rows), D, order, seg, row_lo, static_cast<float*>(g_pool)));
    else
        DWA_TIMED("scatter_add", st, launch_pdl(scatter_add_kernel<float, float>, g, 256, 0, st, indices,
                                                static_cast<const float*>(g_rows), D, order, seg, row_lo, static_cast<float*>(g_pool)));
    DWA_LAUNCH_CHECK("scatter_add_kernel");
    g_launches_total += 2;
    return DWA_OK;
}

extern "C" size_t dwa_pool_grad_recv_bytes(int world, int slot, int64_t D, int rows_dtype) {
    if (world <= 0 || world > kMaxOwners || slot <= 0 || D <= 0 || (rows_dtype != DWA_F32 && rows_dtype != DWA_BF16))
        return 0;
    const size_t slots = static_cast<size_t>(world) * slot;
    return align_up(slots * 4, 256) + slots * static_cast<size_t>(D) * dtype_bytes(rows_dtype);
}

extern "C" int dwa_pool_grad_send(void* stream, int rank, int n, int slot, int64_t D, const int32_t* indices,
                                  const float* g_rows, int rows_dtype, const DwaPoolShards* recv, void* workspace,
                                  size_t workspace_bytes) {
    if (!recv || recv->world <= 0 || recv->world > kMaxOwners || !recv->bases || !recv->row_lo)
        return fail(DWA_ERR_INVALID_ARG, "recv: 1..16 owners with bases and row_lo");
    if (rank < 0 || rank >= recv->world) return fail(DWA_ERR_INVALID_ARG, "rank outside [0, world)");
    if (slot <= 0 || n < 0 || n > slot) return fail(DWA_ERR_INVALID_ARG, "need 0 <= n <= slot and slot > 0");
    if (static_cast<int64_t>(recv->world) * slot > kScatterMaxN)
        return fail(DWA_ERR_UNSUPPORTED, "world * slot above 8192 (one scatter call per area)");
    if (rows_dtype != DWA_F32 && rows_dtype != DWA_BF16)
        return fail(DWA_ERR_INVALID_ARG, "rows_dtype must be DWA_F32 or DWA_BF16");
    if (D <= 0 || D % 8 != 0) return fail(DWA_ERR_UNSUPPORTED, "D must be a positive multiple of 8");
    if (n > 0 && (!indices || !g_rows || reinterpret_cast<uintptr_t>(g_rows) % 16 != 0))
        return fail(DWA_ERR_INVALID_ARG, "indices and a 16-byte aligned g_rows are required");
    if (!workspace || reinterpret_cast<uintptr_t>(workspace) % 256 != 0 || workspace_bytes < 256)
        return fail(DWA_ERR_WORKSPACE, "workspace: 256 bytes, 256-byte aligned");
    RecvAreas ra{};
    ra.world = recv->world;
    ra.slot = slot;
    ra.D = D;
    ra.rows_off = static_cast<int64_t>(align_up(static_cast<size_t>(recv->world) * slot * 4, 256));
    for (int q = 0; q <= ra.world; ++q) ra.row_lo[q] = recv->row_lo[q];
    for (int q = 0; q < ra.world; ++q) {
        if (ra.row_lo[q + 1] < ra.row_lo[q]) return fail(DWA_ERR_INVALID_ARG, "row_lo must be non-decreasing");
        ra.base[q] = static_cast<char*>(const_cast<void*>(recv->bases[q]));
        if (!ra.base[q] || reinterpret_cast<uintptr_t>(ra.base[q]) % 256 != 0)
            return fail(DWA_ERR_INVALID_ARG, "every receive area needs a 256-byte aligned base");
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    uint32_t* status = static_cast<uint32_t*>(workspace);
    if (rows_dtype == DWA_BF16)
        DWA_TIMED("grad_send", st, launch_pdl(grad_send_kernel<__nv_bfloat16>, slot, 256, 0, st, ra, rank, n,
                                              indices, g_rows, status));
    else
        DWA_TIMED("grad_send", st, launch_pdl(grad_send_kernel<float>, slot, 256, 0, st, ra, rank, n, indices,
                                              g_rows, status));
    DWA_LAUNCH_CHECK("grad_send_kernel");
    ++g_launches_total;
    return DWA_OK;
}
