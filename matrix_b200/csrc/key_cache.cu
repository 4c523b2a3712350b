// Key cache of the pool and the centroid EMA.
//
// dwa_key_cache replaces compute_key_cache (src/dwa/assembly_pallas.py:392-400)
// and VectorPool.compute_keys (src/dwa/pool.py:37-44):
//   keys[s, n, :] = pool[n, :] @ key_proj[s]   (einsum "nd,sda->sna", fp32),
// computed once per training window (train.py:253-256).  All S aspects are one
// GEMM with N_gemm = S*d_k (256 for the reference's S = 4, d_k = 64):
// A = the pool rows (K-major, lda = D), B = the projections re-laid out once into
// [S*d_k, D] (K-major) in the workspace, fp32 accumulation; the epilogue writes
// fp32 keys straight into the [S, N, d_k] layout the retrieval reads.  bf16 pool
// and projections: tcgen05 GEMM (products of bf16 values are exact in fp32, so
// the keys equal the reference's fp32 einsum up to summation order); f32: the
// CUDA-core FMA GEMM (tf32 tensor cores would not keep fp32 accuracy).
// Roofline at N = 262144, D = 17408 (bf16): 9.1 GB of pool read once, 1.40 ms at
// 6.54 TB/s, and 2.34 TFLOP, 1.40 ms at 1.67 PFLOP/s: the two bounds coincide.
//
// dwa_centroid_ema replaces the centroid update of train.py:318-328:
//   centroids[s, c] = decay * centroids[s, c] + (1 - decay) * mean(keys[s, list c])
// with the reference's decay 0.9; lists are CSR ranges (equal lists are
// off[c] = c*N/C, the reference's reshape).  HBM-bound: one read of the keys.

#include <atomic>
#include <cstdlib>

#include <cstring>

#include "dwa_common.cuh"
#include "epilogue.cuh"
#include "simt_gemm.cuh"
#include "tc_gemm.cuh"

namespace dwa {

extern std::atomic<uint64_t> g_launches_total, g_launches_tc, g_launches_simt;

// bt[s*d_k + a, d] = kp[s, d, a]: 32 x 32 tiles through shared memory.
template <class T>
__global__ void proj_relayout_kernel(const T* __restrict__ kp, T* __restrict__ bt, int S, int D, int d_k) {
    pdl_enter();
    __shared__ T tile[32][33];
    const int s = blockIdx.z, d0 = blockIdx.x * 32, a0 = blockIdx.y * 32;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int d = d0 + i, a = a0 + threadIdx.x;
        if (d < D && a < d_k) tile[i][threadIdx.x] = kp[(static_cast<int64_t>(s) * D + d) * d_k + a];
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int a = a0 + i, d = d0 + threadIdx.x;
        if (a < d_k && d < D) bt[(static_cast<int64_t>(s) * d_k + a) * D + d] = tile[threadIdx.x][i];
    }
}

// keys[s, row, a] = acc(row, s*d_k + a)
struct EpiKeys : NoReduce {
    float* keys; int64_t N; int d_k;
    struct Frag {};
    __device__ void load(int, int, int, int, Frag&) const {}
    __device__ float finish(int, int row, int col0, const float* v, int cnt, const Frag&) const {
        if (cnt == 8 && d_k % 8 == 0) {
            // eight columns inside one aspect (col0 is a multiple of 8)
            store8_stream(keys + (static_cast<int64_t>(col0 / d_k) * N + row) * d_k + col0 % d_k, v);
        } else {
            for (int c = 0; c < cnt; ++c) {
                const int j = col0 + c;
                keys[(static_cast<int64_t>(j / d_k) * N + row) * d_k + j % d_k] = v[c];
            }
        }
        return 0.f;
    }
    DWA_EPI_CALL
};

// One block per (list c, aspect s): the mean of the list's key rows, then the EMA.
__global__ void centroid_ema_kernel(const float* __restrict__ keys, const int64_t* __restrict__ off,
                                    int64_t N, int C, int d_k, float decay, float* __restrict__ cent,
                                    uint32_t* status) {
    pdl_enter();
    extern __shared__ float part[];   // [blockDim.y][d_k]
    const int c = blockIdx.x, s = blockIdx.y;
    const int64_t lo = off[c], hi = off[c + 1];
    if (lo < 0 || hi < lo || hi > N) {
        if (threadIdx.x == 0 && threadIdx.y == 0) raise_status(status, DWA_STATUS_BAD_LIST);
        return;
    }
    const float* base = keys + static_cast<int64_t>(s) * N * d_k;
    for (int a = threadIdx.x; a < d_k; a += blockDim.x) {
        float acc = 0.f;
        for (int64_t r = lo + threadIdx.y; r < hi; r += blockDim.y) acc += base[r * d_k + a];
        part[threadIdx.y * d_k + a] = acc;
    }
    __syncthreads();
    if (threadIdx.y == 0) {
        for (int a = threadIdx.x; a < d_k; a += blockDim.x) {
            float sum = 0.f;
            for (int y = 0; y < blockDim.y; ++y) sum += part[y * d_k + a];
            float* o = cent + (static_cast<int64_t>(s) * C + c) * d_k + a;
            // an empty list keeps its centroid
            if (hi > lo) *o = decay * *o + (1.f - decay) * (sum / static_cast<float>(hi - lo));
        }
    }
}

static int check_kc(const DwaKeyCacheDims* d) {
    if (!d) return fail(DWA_ERR_INVALID_ARG, "dims is NULL");
    if (d->N <= 0 || d->D <= 0 || d->S <= 0 || d->d_k <= 0)
        return fail(DWA_ERR_INVALID_ARG, "N, D, S, d_k must be positive");
    if (d->N >= (int64_t(1) << 31)) return fail(DWA_ERR_UNSUPPORTED, "N >= 2^31");
    if (static_cast<int64_t>(d->S) * d->d_k > 4096) return fail(DWA_ERR_UNSUPPORTED, "S * d_k > 4096");
    if (d->dtype != DWA_F32 && d->dtype != DWA_BF16)
        return fail(DWA_ERR_INVALID_ARG, "dtype must be DWA_F32 or DWA_BF16");
    return DWA_OK;
}

}  // namespace dwa

using namespace dwa;

extern "C" size_t dwa_key_cache_workspace_bytes(const DwaKeyCacheDims* dims) {
    if (check_kc(dims)) return 0;
    const size_t es = dims->dtype == DWA_BF16 ? 2 : 4;
    return 256 + align_up(static_cast<size_t>(dims->S) * dims->d_k * dims->D * es, 256);
}

extern "C" int dwa_key_cache(void* stream, const DwaKeyCacheDims* dims, const void* pool_vectors,
                             const void* key_proj, float* keys, void* workspace, size_t workspace_bytes) {
    int rc = check_kc(dims);
    if (rc) return rc;
    const DwaKeyCacheDims& d = *dims;
    if (!pool_vectors || !key_proj || !keys) return fail(DWA_ERR_INVALID_ARG, "a required pointer is NULL");
    if (!workspace || reinterpret_cast<uintptr_t>(workspace) % 256 != 0)
        return fail(DWA_ERR_WORKSPACE, "workspace must be non-NULL and 256-byte aligned");
    if (workspace_bytes < dwa_key_cache_workspace_bytes(dims))
        return fail(DWA_ERR_WORKSPACE, "workspace too small");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    uint32_t* status = static_cast<uint32_t*>(workspace);
    void* bt = static_cast<char*>(workspace) + 256;
    const dim3 gr((d.D + 31) / 32, (d.d_k + 31) / 32, d.S), br(32, 8);
    if (d.dtype == DWA_BF16)
        launch_pdl(proj_relayout_kernel<__nv_bfloat16>, gr, br, 0, st, static_cast<const __nv_bfloat16*>(key_proj),
                                                              static_cast<__nv_bfloat16*>(bt), d.S, d.D, d.d_k);
    else
        launch_pdl(proj_relayout_kernel<float>, gr, br, 0, st, static_cast<const float*>(key_proj),
                                                      static_cast<float*>(bt), d.S, d.D, d.d_k);
    DWA_LAUNCH_CHECK("proj_relayout_kernel");
    ++g_launches_total;

    const int M = static_cast<int>(d.N), Ng = d.S * d.d_k, K = d.D;
    EpiKeys epi;
    epi.keys = keys;
    epi.N = d.N;
    epi.d_k = d.d_k;
    const char* gsel = std::getenv("DWA_GEMM");
    if (d.dtype == DWA_BF16 && !(gsel && std::strcmp(gsel, "simt") == 0)) {
        const bool pers = tc::persistent_gemm();
        const tc::Operand A{pool_vectors, false, K, 0}, B{bt, false, K, 0};
        const int64_t ctas256 = static_cast<int64_t>((M + 127) / 128) * ((Ng + 255) / 256);
        if (Ng >= 256 && ctas256 >= 120 && tc::tc_operand_ok(A, M, K, 128) && tc::tc_operand_ok(B, Ng, K, 256)) {
            ++g_launches_tc;
            prof_begin("key_cache", st);
            rc = pers ? tc::launch_gemm_bf16_persistent<256, 4, false, false>(A, B, M, Ng, K, 1, epi, status, st)
                      : tc::launch_gemm_bf16<256, 4, false, false>(A, B, M, Ng, K, 1, epi, status, st);
            prof_end("key_cache", st);
            ++g_launches_total;
            return rc;
        }
        if (Ng >= 128 && tc::tc_operand_ok(A, M, K, 128) && tc::tc_operand_ok(B, Ng, K, 128)) {
            ++g_launches_tc;
            prof_begin("key_cache", st);
            rc = pers ? tc::launch_gemm_bf16_persistent<128, 6, false, false>(A, B, M, Ng, K, 1, epi, status, st)
                      : tc::launch_gemm_bf16<128, 6, false, false>(A, B, M, Ng, K, 1, epi, status, st);
            prof_end("key_cache", st);
            ++g_launches_total;
            return rc;
        }
    }
    const simt::Operand A{pool_vectors, false, K, 0}, B{bt, false, K, 0};
    ++g_launches_simt;
    prof_begin("key_cache", st);
    if (d.dtype == DWA_BF16)
        rc = simt::launch_gemm<__nv_bfloat16, __nv_bfloat16>(A, B, M, Ng, K, 1, epi, st);
    else
        rc = simt::launch_gemm<float, float>(A, B, M, Ng, K, 1, epi, st);
    prof_end("key_cache", st);
    ++g_launches_total;
    return rc;
}

extern "C" int dwa_centroid_ema(void* stream, int S, int C, int d_k, int64_t N, const float* keys,
                                const int64_t* list_offsets, float decay, float* centroids,
                                void* workspace, size_t workspace_bytes) {
    if (S <= 0 || C <= 0 || d_k <= 0 || N <= 0) return fail(DWA_ERR_INVALID_ARG, "S, C, d_k, N must be positive");
    if (d_k > 1024) return fail(DWA_ERR_UNSUPPORTED, "d_k > 1024");
    if (!keys || !list_offsets || !centroids) return fail(DWA_ERR_INVALID_ARG, "a required pointer is NULL");
    if (!(decay >= 0.f && decay <= 1.f)) return fail(DWA_ERR_INVALID_ARG, "decay must be in [0, 1]");
    if (!workspace || reinterpret_cast<uintptr_t>(workspace) % 256 != 0 || workspace_bytes < 256)
        return fail(DWA_ERR_WORKSPACE, "workspace: 256 bytes, 256-byte aligned (status word)");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int tx = d_k < 64 ? d_k : 64;
    const int ty = 1024 / tx < 16 ? 1024 / tx : 16;
    const size_t sh = static_cast<size_t>(ty) * d_k * sizeof(float);
    if (sh > 48 * 1024) return fail(DWA_ERR_UNSUPPORTED, "d_k too large for the EMA reduction");
    DWA_TIMED("centroid_ema", st, launch_pdl(centroid_ema_kernel, dim3(C, S), dim3(tx, ty), sh, st, 
                                      keys, list_offsets, N, C, d_k, decay, centroids,
                                      static_cast<uint32_t*>(workspace)));
    DWA_LAUNCH_CHECK("centroid_ema_kernel");
    ++g_launches_total;
    return DWA_OK;
}
