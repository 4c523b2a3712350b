// Batched GEMM on the CUDA cores with fp32 FMA, any shape and layout.
//
// Same contract and epilogue protocol as tc_gemm.cuh.  It serves the float32
// activation dtype (the tensor cores would round fp32 operands to tf32, which
// cannot meet a 1e-5 relative tolerance) and bf16 shapes the TMA rules exclude
// (row strides that are not a multiple of 16 bytes, extents below one tile).
#pragma once

#include "dwa_common.cuh"

namespace dwa {
namespace simt {

struct Operand {
    const void* ptr;
    bool mn_major;
    int64_t ld;
    int64_t bstride;
};

constexpr int TM = 64, TN = 64, TK = 16;

template <class T>
__device__ __forceinline__ float ld_op(const Operand& op, int b, int mn, int k) {
    const T* p = static_cast<const T*>(op.ptr) + op.bstride * b;
    const int64_t i = op.mn_major ? static_cast<int64_t>(k) * op.ld + mn
                                  : static_cast<int64_t>(mn) * op.ld + k;
    return Elem<T>::to_f(p[i]);
}

template <class TA, class TB, class Epi>
__global__ void __launch_bounds__(256)
    gemm_kernel(Operand A, Operand B, int M, int N, int K, Epi epi) {
    pdl_enter();
    __shared__ float As[TK][TM + 4];
    __shared__ float Bs[TK][TN + 4];
    __shared__ float s_red[8];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int m0 = blockIdx.y * TM, n0 = blockIdx.x * TN, bz = blockIdx.z;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

    for (int k0 = 0; k0 < K; k0 += TK) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int e = threadIdx.x + 256 * i;
            int mm, kk;
            if (A.mn_major) { kk = e / TM; mm = e % TM; } else { mm = e / TK; kk = e % TK; }
            const int gm = m0 + mm, gk = k0 + kk;
            As[kk][mm] = (gm < M && gk < K) ? ld_op<TA>(A, bz, gm, gk) : 0.f;
            int nn;
            if (B.mn_major) { kk = e / TN; nn = e % TN; } else { nn = e / TK; kk = e % TK; }
            const int gn = n0 + nn, gk2 = k0 + kk;
            Bs[kk][nn] = (gn < N && gk2 < K) ? ld_op<TB>(B, bz, gn, gk2) : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < TK; ++kk) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }

    float cta_acc = 0.f;
    const int col0 = n0 + tx * 4;
    const int cnt = min(4, N - col0);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int row = m0 + ty * 4 + i;
        float part = 0.f;
        if (row < M && cnt > 0) part = epi(bz, row, col0, acc[i], cnt);
        if (Epi::kReduce == 1) {
            if (row < M && cnt > 0) epi.row_done(bz, row, part);
        } else {
            cta_acc += part;
        }
    }
    if (Epi::kReduce == 2) {
        cta_acc = warp_sum(cta_acc);
        if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = cta_acc;
        __syncthreads();
        if (threadIdx.x == 0) {
            float t = 0.f;
            for (int w = 0; w < 8; ++w) t += s_red[w];
            epi.cta_done(bz, t);
        }
    }
}

template <class TA, class TB, class Epi>
int launch_gemm(const Operand& A, const Operand& B, int M, int N, int K, int batch, const Epi& epi,
                cudaStream_t stream) {
    dim3 grid((N + TN - 1) / TN, (M + TM - 1) / TM, batch);
    launch_pdl(gemm_kernel<TA, TB, Epi>, grid, 256, 0, stream, A, B, M, N, K, epi);
    DWA_LAUNCH_CHECK("simt::gemm_kernel");
    return DWA_OK;
}

}  // namespace simt
}  // namespace dwa
