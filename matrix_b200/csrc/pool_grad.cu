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
            if (r < 0 || r >= n_global) raise_status(status, DWA_STATUS_BAD_ROW_INDEX);
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

template <class TG>
__global__ void __launch_bounds__(256) scatter_add_kernel(const int32_t* __restrict__ idx,
                                                          const float* __restrict__ g_rows, int D,
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
        for (int j = j0; j < j1; ++j) acc += g_rows[static_cast<int64_t>(order[j]) * D + c];
        TG* p = g_pool + row * D + c;
        *p = Elem<TG>::from_f(Elem<TG>::to_f(*p) + acc);
    }
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
    if (g_dtype == DWA_BF16)
        DWA_TIMED("scatter_add", st, launch_pdl(scatter_add_kernel<__nv_bfloat16>, g, 256, 0, st, 
                                         indices, g_rows, D, order, seg, row_lo, static_cast<__nv_bfloat16*>(g_pool)));
    else
        DWA_TIMED("scatter_add", st, launch_pdl(scatter_add_kernel<float>, g, 256, 0, st, 
                                         indices, g_rows, D, order, seg, row_lo, static_cast<float*>(g_pool)));
    DWA_LAUNCH_CHECK("scatter_add_kernel");
    g_launches_total += 2;
    return DWA_OK;
}
