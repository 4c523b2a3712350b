// RMSNorm of the assembly output (the assembler's layer_norm,
// src/dwa/assembly.py:29, applied at src/dwa/model.py:207-219):
//   y[r, j] = x[r, j] * (rsqrt(mean_j x[r, j]^2 + eps) * scale[j])
// as flax's nnx.RMSNorm computes it (statistics in fp32, epsilon 1e-6 by
// default, output promoted to the scale's fp32 or kept in the input type), and
// its VJP:
//   g_x[r, j]  = rstd_r * scale_j * g_j - rstd_r^3 / d * x[r, j] * sum_i g_i scale_i x[r, i]
//   g_scale[j] = sum_r g[r, j] * x[r, j] * rstd_r
// Both directions are HBM-bound row passes (one CTA per group of rows, 16-byte
// vector accesses); g_scale is reduced deterministically: per-CTA partials,
// then a column sum in a fixed order.

#include <atomic>

#include "dwa_common.cuh"
#include "epilogue.cuh"

namespace dwa {

extern std::atomic<uint64_t> g_launches_total;

constexpr int kNormThreads = 256;
constexpr int kNormRowsPerBlock = 8;   // rows per CTA in the backward (g_scale partials)

__device__ __forceinline__ float block_sum(float v, float* red) {
    v = warp_sum(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    float t = 0.f;
    if (threadIdx.x < 32) {
        t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
        t = warp_sum(t);
        if (threadIdx.x == 0) red[32] = t;
    }
    __syncthreads();
    return red[32];
}

__device__ __forceinline__ void ld8(const float* p, float* v) { load8(p, v); }
__device__ __forceinline__ void ld8(const __nv_bfloat16* p, float* v) { load8(p, v); }

// One CTA per row; d % 8 == 0 and 16-byte aligned rows (checked on the host).
template <class TI, class TO>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_fwd_kernel(const TI* __restrict__ x,
                                                                  const float* __restrict__ scale, int d,
                                                                  float eps, TO* __restrict__ y,
                                                                  float* __restrict__ rstd) {
    pdl_enter();
    __shared__ float red[33];
    const int64_t r = blockIdx.x;
    const TI* xr = x + r * d;
    float ss = 0.f;
    for (int c = threadIdx.x * 8; c < d; c += blockDim.x * 8) {
        float v[8];
        ld8(xr + c, v);
#pragma unroll
        for (int i = 0; i < 8; ++i) ss = fmaf(v[i], v[i], ss);
    }
    const float inv = rsqrtf(block_sum(ss, red) / static_cast<float>(d) + eps);
    if (threadIdx.x == 0) rstd[r] = inv;
    for (int c = threadIdx.x * 8; c < d; c += blockDim.x * 8) {
        float v[8], s[8], o[8];
        ld8(xr + c, v);
        load8(scale + c, s);
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = v[i] * (inv * s[i]);
        store8(y + r * d + c, o);
    }
}

// kNormRowsPerBlock rows per CTA: g_x per row, and this CTA's partial of
// g_scale over its rows into part[blockIdx.x, :].
template <class TI, class TG>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_bwd_kernel(const TI* __restrict__ x,
                                                                  const float* __restrict__ scale,
                                                                  const float* __restrict__ rstd,
                                                                  const TG* __restrict__ gy, int64_t rows,
                                                                  int d, TI* __restrict__ gx,
                                                                  float* __restrict__ part) {
    pdl_enter();
    __shared__ float red[33];
    extern __shared__ float gs[];   // [d] partial g_scale of this CTA
    for (int c = threadIdx.x; c < d; c += blockDim.x) gs[c] = 0.f;
    __syncthreads();
    const int64_t r0 = static_cast<int64_t>(blockIdx.x) * kNormRowsPerBlock;
    for (int64_t r = r0; r < r0 + kNormRowsPerBlock && r < rows; ++r) {
        const TI* xr = x + r * d;
        const TG* gr = gy + r * d;
        const float inv = rstd[r];
        float dot = 0.f;
        for (int c = threadIdx.x * 8; c < d; c += blockDim.x * 8) {
            float v[8], g[8], s[8];
            ld8(xr + c, v);
            ld8(gr + c, g);
            load8(scale + c, s);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                dot = fmaf(g[i] * s[i], v[i], dot);
                gs[c + i] = fmaf(g[i], v[i] * inv, gs[c + i]);
            }
        }
        const float k = block_sum(dot, red) * inv * inv * inv / static_cast<float>(d);
        for (int c = threadIdx.x * 8; c < d; c += blockDim.x * 8) {
            float v[8], g[8], s[8], o[8];
            ld8(xr + c, v);
            ld8(gr + c, g);
            load8(scale + c, s);
#pragma unroll
            for (int i = 0; i < 8; ++i) o[i] = inv * s[i] * g[i] - k * v[i];
            store8(gx + r * d + c, o);
        }
    }
    __syncthreads();
    for (int c = threadIdx.x; c < d; c += blockDim.x) part[static_cast<int64_t>(blockIdx.x) * d + c] = gs[c];
}

static int check_norm(int64_t rows, int d, int a, int b) {
    if (rows <= 0 || d <= 0) return fail(DWA_ERR_INVALID_ARG, "rows and d must be positive");
    if (d % 8 != 0) return fail(DWA_ERR_UNSUPPORTED, "d must be a multiple of 8");
    if (static_cast<size_t>(d) * sizeof(float) > 48 * 1024) return fail(DWA_ERR_UNSUPPORTED, "d > 12288");
    if ((a != DWA_F32 && a != DWA_BF16) || (b != DWA_F32 && b != DWA_BF16))
        return fail(DWA_ERR_INVALID_ARG, "dtypes must be DWA_F32 or DWA_BF16");
    if (rows >= (int64_t(1) << 31)) return fail(DWA_ERR_UNSUPPORTED, "rows >= 2^31");
    return DWA_OK;
}

static bool aligned16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

}  // namespace dwa

using namespace dwa;

extern "C" int dwa_rmsnorm_fwd(void* stream, int64_t rows, int d, int x_dtype, int y_dtype, const void* x,
                               const float* scale, float eps, void* y, float* rstd) {
    int rc = check_norm(rows, d, x_dtype, y_dtype);
    if (rc) return rc;
    if (!x || !scale || !y || !rstd) return fail(DWA_ERR_INVALID_ARG, "a required pointer is NULL");
    if (!aligned16(x) || !aligned16(scale) || !aligned16(y))
        return fail(DWA_ERR_INVALID_ARG, "x, scale and y must be 16-byte aligned");
    if (!(eps >= 0.f)) return fail(DWA_ERR_INVALID_ARG, "eps must be >= 0");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const unsigned g = static_cast<unsigned>(rows);
#define DWA_NORM_FWD(TI, TO)                                                                             \
    DWA_TIMED("rmsnorm_fwd", st, (launch_pdl(rmsnorm_fwd_kernel<TI, TO>, g, kNormThreads, 0, st,                  \
                                      static_cast<const TI*>(x), scale, d, eps, static_cast<TO*>(y), rstd)))
    if (x_dtype == DWA_BF16 && y_dtype == DWA_BF16) DWA_NORM_FWD(__nv_bfloat16, __nv_bfloat16);
    else if (x_dtype == DWA_BF16) DWA_NORM_FWD(__nv_bfloat16, float);
    else if (y_dtype == DWA_BF16) DWA_NORM_FWD(float, __nv_bfloat16);
    else DWA_NORM_FWD(float, float);
#undef DWA_NORM_FWD
    DWA_LAUNCH_CHECK("rmsnorm_fwd_kernel");
    ++g_launches_total;
    return DWA_OK;
}

extern "C" size_t dwa_rmsnorm_bwd_workspace_bytes(int64_t rows, int d) {
    if (rows <= 0 || d <= 0) return 0;
    const int64_t nblk = (rows + kNormRowsPerBlock - 1) / kNormRowsPerBlock;
    return 256 + align_up(static_cast<size_t>(nblk) * d * sizeof(float), 256);
}

extern "C" int dwa_rmsnorm_bwd(void* stream, int64_t rows, int d, int x_dtype, int g_dtype, const void* x,
                               const float* scale, const float* rstd, const void* g_y, void* g_x,
                               float* g_scale, void* workspace, size_t workspace_bytes) {
    int rc = check_norm(rows, d, x_dtype, g_dtype);
    if (rc) return rc;
    if (!x || !scale || !rstd || !g_y || !g_x || !g_scale) return fail(DWA_ERR_INVALID_ARG, "a required pointer is NULL");
    if (!aligned16(x) || !aligned16(scale) || !aligned16(g_y) || !aligned16(g_x))
        return fail(DWA_ERR_INVALID_ARG, "x, scale, g_y and g_x must be 16-byte aligned");
    if (!workspace || reinterpret_cast<uintptr_t>(workspace) % 256 != 0)
        return fail(DWA_ERR_WORKSPACE, "workspace must be non-NULL and 256-byte aligned");
    if (workspace_bytes < dwa_rmsnorm_bwd_workspace_bytes(rows, d)) return fail(DWA_ERR_WORKSPACE, "workspace too small");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    float* part = reinterpret_cast<float*>(static_cast<char*>(workspace) + 256);
    const int nblk = static_cast<int>((rows + kNormRowsPerBlock - 1) / kNormRowsPerBlock);
    const size_t sh = static_cast<size_t>(d) * sizeof(float);
#define DWA_NORM_BWD(TI, TG)                                                                              \
    DWA_TIMED("rmsnorm_bwd", st, (launch_pdl(rmsnorm_bwd_kernel<TI, TG>, nblk, kNormThreads, sh, st,               \
                                      static_cast<const TI*>(x), scale, rstd, static_cast<const TG*>(g_y),  \
                                      rows, d, static_cast<TI*>(g_x), part)))
    if (x_dtype == DWA_BF16 && g_dtype == DWA_BF16) DWA_NORM_BWD(__nv_bfloat16, __nv_bfloat16);
    else if (x_dtype == DWA_BF16) DWA_NORM_BWD(__nv_bfloat16, float);
    else if (g_dtype == DWA_BF16) DWA_NORM_BWD(float, __nv_bfloat16);
    else DWA_NORM_BWD(float, float);
#undef DWA_NORM_BWD
    DWA_LAUNCH_CHECK("rmsnorm_bwd_kernel");
    launch_pdl(column_sum_kernel<float>, dim3((d + 63) / 64, 1), 1024, 0, st, part, nblk, d, 0, g_scale);
    DWA_LAUNCH_CHECK("column_sum_kernel");
    g_launches_total += 2;
    return DWA_OK;
}
