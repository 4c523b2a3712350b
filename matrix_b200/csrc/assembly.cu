// DWA assembly forward and backward on B200.
//
// Forward (replaces src/dwa/assembly_pallas.py:139-222):
//   prep    gather each (b,k) pool row (or read the gathered row), split it into
//           U [d_B,r] | V [r,d_A] | b [d_B] (config.py:159-165) and write
//             Ug[b] [d_B, k*r]   Ug[b][j][k*r+rho] = U_k[j][rho]     (K-major A)
//             Vs[b] [k*r, d_A]   Vs[b][k*r+rho][i] = alpha_k V_k[rho][i]
//             pb[b] [d_B]        b_base + sum_k alpha_k b_k
//   GEMM W  W[b] = W_base + Ug[b] Vs[b]          M=d_B N=d_A K=k*r  (fp32 + act copy)
//   GEMM y  h_mid[b] = h_A[b] + gamma h_A[b] W[b]^T + pb[b]     M=T N=d_B K=d_A
// W is the primal's second output, so forming it costs no extra pass: the
// apply is one GEMM against the assembled W instead of the reference's three
// (assembly_pallas.py:113-117), and the [B,k,d_B,d_A] product of :212-221 is
// never materialised.
//
// Backward (replaces assembly_pallas.py:246-329), with G[b] = g[b]^T h_A[b]:
//   GEMM G    gW[b] = gamma G[b] + g_W_out[b]          -> act copy, += g_W_base,
//             g_gamma += <G[b], W[b]>  (= sum g * h_A W^T, :275)
//   GEMM gh   g_hA[b] = g[b] + gamma g[b] W[b]         (:283-285)
//   GEMM P    g_U[b] = gW[b] Vs[b]^T   (alpha folded into Vs; :303-305)
//   GEMM Q    Q[b] = Ug[b]^T gW[b]: g_V = alpha Q (:310-312), and
//             g_alpha += <V_k, Q_k> = <U_k V_k, gW> (:298) without forming U_k V_k
//   colsum    g_bias[b] = sum_t g[b];  finalize: g_alpha += <b_k, g_bias>,
//             g_b = alpha g_bias, pad columns zero, g_b_base, g_gamma.
#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <type_traits>

#include "dwa_common.cuh"
#include "epilogue.cuh"
#include "simt_gemm.cuh"
#include "tc_gemm.cuh"
#include "tc_gemm_pair.cuh"
#include "tc_gemm_w.cuh"

namespace dwa {

extern std::atomic<uint64_t> g_launches_total, g_launches_tc, g_launches_simt;

// ------------------------------------------------------------ row source ---
struct RowSrc {
    const void* rows;
    const int32_t* row_index;
    int64_t n_rows;
    int64_t D;
    int k;
    int dtype;
    // Element offset of row (b, kk), or -1 when its index is outside the pool.
    __device__ __forceinline__ int64_t offset(int b, int kk) const {
        int64_t r = static_cast<int64_t>(b) * k + kk;
        if (row_index) {
            const int64_t i = row_index[r];
            if (i < 0 || i >= n_rows) return -1;
            r = i;
        }
        return r * D;
    }
};

// ------------------------------------------------------- vector helpers ----
// 8 consecutive elements through 16-byte accesses (the pointer must be 16-byte
// aligned for bf16, 16-byte aligned for fp32 pairs of float4).
// W[b](j,i) = W_base(j,i) + acc   -> fp32 W_out and/or act-typed W_act
template <class ACT>
struct EpiW : NoReduce {
    const float* W_base; float* W_out; ACT* W_act; int d_B, d_A; bool vec;
    struct Frag { float wb[8]; };
    __device__ void load(int, int row, int col0, int cnt, Frag& f) const {
        if (vec && cnt == 8) load8(W_base + static_cast<int64_t>(row) * d_A + col0, f.wb);
    }
    __device__ float finish(int b, int row, int col0, const float* v, int cnt, const Frag& f) const {
        const int64_t o = (static_cast<int64_t>(b) * d_B + row) * d_A + col0;
        if (vec && cnt == 8) {
            float w[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) w[i] = f.wb[i] + v[i];
            if (W_out) store8_stream(W_out + o, w);     // the API's W: not read again in this call
            if (W_act) store8(W_act + o, w);            // the apply GEMM's operand, read next
        } else {
            const float* wb = W_base + static_cast<int64_t>(row) * d_A + col0;
            for (int c = 0; c < cnt; ++c) {
                const float w = wb[c] + v[c];
                if (W_out) W_out[o + c] = w;
                if (W_act) W_act[o + c] = Elem<ACT>::from_f(w);
            }
        }
        return 0.f;
    }
    DWA_EPI_CALL
};

// h_mid[b](t,j) = h_A[b](t,j) + gamma acc + pb[b](j)
template <class ACT>
struct EpiApply : NoReduce {
    const ACT* hA; const float* pb; const float* gamma; ACT* out; int T, d; bool vec;
    struct Frag { float h[8], q[8]; };
    __device__ void load(int b, int row, int col0, int cnt, Frag& f) const {
        if (vec && cnt == 8) {
            load8(hA + (static_cast<int64_t>(b) * T + row) * d + col0, f.h);
            load8(pb + static_cast<int64_t>(b) * d + col0, f.q);
        }
    }
    __device__ float finish(int b, int row, int col0, const float* v, int cnt, const Frag& f) const {
        const int64_t o = (static_cast<int64_t>(b) * T + row) * d + col0;
        const float g = __ldg(gamma);
        if (vec && cnt == 8) {
            float h[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) h[i] = f.h[i] + g * v[i] + f.q[i];
            store8(out + o, h);
        } else {
            const float* p = pb + static_cast<int64_t>(b) * d + col0;
            for (int c = 0; c < cnt; ++c)
                out[o + c] = Elem<ACT>::from_f(Elem<ACT>::to_f(hA[o + c]) + g * v[c] + p[c]);
        }
        return 0.f;
    }
    DWA_EPI_CALL
};

// gW[b](j,i) = gamma G + g_W_out; g_W_base += gW; g_gamma += G * W
template <class ACT>
struct EpiG {
    static constexpr int kReduce = 2;
    const float* gamma; const float* gWo; ACT* gW; float* gWbase; const ACT* Wact;
    float* gamma_acc; int d_B, d_A; bool vec;
    struct Frag { float w[8], x[8]; };
    __device__ void load(int b, int row, int col0, int cnt, Frag& f) const {
        if (vec && cnt == 8) {
            const int64_t o = (static_cast<int64_t>(b) * d_B + row) * d_A + col0;
            load8(Wact + o, f.w);
            if (gWo) load8(gWo + o, f.x);
        }
    }
    __device__ float finish(int b, int row, int col0, const float* v, int cnt, const Frag& f) const {
        const int64_t o = (static_cast<int64_t>(b) * d_B + row) * d_A + col0;
        const int64_t ob = static_cast<int64_t>(row) * d_A + col0;
        const float g = __ldg(gamma);
        float part = 0.f;
        if (vec && cnt == 8) {
            float x[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                part = fmaf(v[i], f.w[i], part);
                x[i] = gWo ? fmaf(g, v[i], f.x[i]) : g * v[i];
            }
            store8(gW + o, x);
            red_add4(gWbase + ob, x[0], x[1], x[2], x[3]);
            red_add4(gWbase + ob + 4, x[4], x[5], x[6], x[7]);
        } else {
            for (int c = 0; c < cnt; ++c) {
                part = fmaf(v[c], Elem<ACT>::to_f(Wact[o + c]), part);
                const float x = gWo ? fmaf(g, v[c], gWo[o + c]) : g * v[c];
                gW[o + c] = Elem<ACT>::from_f(x);
                atomicAdd(gWbase + ob + c, x);
            }
        }
        return part;
    }
    DWA_EPI_CALL
    __device__ void row_done(int, int, float) const {}
    __device__ void cta_done(int, float acc) const { atomicAdd(gamma_acc, acc); }
};

// g_hA[b](t,i) = g[b](t,i) + gamma acc
template <class ACT>
struct EpiGhA : NoReduce {
    const ACT* g; const float* gamma; ACT* out; int T, d; bool vec;
    struct Frag { float x[8]; };
    __device__ void load(int b, int row, int col0, int cnt, Frag& f) const {
        if (vec && cnt == 8) load8(g + (static_cast<int64_t>(b) * T + row) * d + col0, f.x);
    }
    __device__ float finish(int b, int row, int col0, const float* v, int cnt, const Frag& f) const {
        const int64_t o = (static_cast<int64_t>(b) * T + row) * d + col0;
        const float gm = __ldg(gamma);
        if (vec && cnt == 8) {
            float x[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) x[i] = fmaf(gm, v[i], f.x[i]);
            store8(out + o, x);
        } else {
            for (int c = 0; c < cnt; ++c)
                out[o + c] = Elem<ACT>::from_f(fmaf(gm, v[c], Elem<ACT>::to_f(g[o + c])));
        }
        return 0.f;
    }
    DWA_EPI_CALL
};

// g_U: g_rows[b][kk][j*r + rho] = acc(j, kk*r + rho)
struct EpiP : NoReduce {
    float* g_rows; int64_t D; int k, r; bool vec;
    struct Frag {};
    __device__ void load(int, int, int, int, Frag&) const {}
    __device__ float finish(int b, int row, int col0, const float* v, int cnt, const Frag&) const {
        if (vec && cnt == 8 && r == 8) {   // the 8 columns are the 8 factors of one pool row
            store8(g_rows + (static_cast<int64_t>(b) * k + col0 / 8) * D + static_cast<int64_t>(row) * 8, v);
            return 0.f;
        }
        for (int c = 0; c < cnt; ++c) {
            const int n = col0 + c;
            const int kk = n / r, rho = n - kk * r;
            g_rows[(static_cast<int64_t>(b) * k + kk) * D + static_cast<int64_t>(row) * r + rho] = v[c];
        }
        return 0.f;
    }
    DWA_EPI_CALL
};

// g_V: g_rows[b][kk][s1 + rho*d_A + i] = alpha[b,kk] acc(kk*r+rho, i);
// g_alpha[b,kk] += sum_i V_kk[rho][i] acc(kk*r+rho, i)
template <class RT>
struct EpiQ {
    static constexpr int kReduce = 1;
    RowSrc src; const float* alphas; float* g_rows; float* dW_acc; int64_t s1; int d_A, r; bool vec;
    struct Frag { float vv[8]; float a; bool has; };
    __device__ void load(int b, int row, int col0, int cnt, Frag& f) const {
        const int kk = row / r, rho = row - kk * r;
        f.a = __ldg(alphas + static_cast<int64_t>(b) * src.k + kk);
        const int64_t ro = src.offset(b, kk);
        f.has = ro >= 0;
        if (vec && cnt == 8 && f.has)
            load8(static_cast<const RT*>(src.rows) + ro + s1 + static_cast<int64_t>(rho) * d_A + col0, f.vv);
    }
    __device__ float finish(int b, int row, int col0, const float* v, int cnt, const Frag& f) const {
        const int kk = row / r, rho = row - kk * r;
        const int64_t go = (static_cast<int64_t>(b) * src.k + kk) * src.D + s1 +
                           static_cast<int64_t>(rho) * d_A + col0;
        float part = 0.f;
        if (vec && cnt == 8) {
            float x[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                x[i] = f.a * v[i];
                if (f.has) part = fmaf(f.vv[i], v[i], part);
            }
            store8(g_rows + go, x);
        } else {
            const int64_t ro = src.offset(b, kk);
            const RT* V = ro < 0 ? nullptr
                                 : static_cast<const RT*>(src.rows) + ro + s1 +
                                       static_cast<int64_t>(rho) * d_A + col0;
            for (int c = 0; c < cnt; ++c) {
                g_rows[go + c] = f.a * v[c];
                if (V) part = fmaf(Elem<RT>::to_f(V[c]), v[c], part);
            }
        }
        return part;
    }
    DWA_EPI_CALL
    __device__ void row_done(int b, int row, float acc) const {
        atomicAdd(dW_acc + static_cast<int64_t>(b) * src.k + row / r, acc);
    }
    __device__ void cta_done(int, float) const {}
};

// --------------------------------------------------------------- kernels ---
template <class ACT, class RT>
__global__ void prep_factors_kernel(RowSrc src, const float* __restrict__ alphas, int d_A, int d_B,
                                    int r, int64_t ldu, ACT* __restrict__ Ug, ACT* __restrict__ Vs,
                                    uint32_t* status) {
    pdl_enter();
    const int kk = blockIdx.x, b = blockIdx.y, k = src.k;
    const int64_t off = src.offset(b, kk);
    if (off < 0 && threadIdx.x == 0) raise_status(status, DWA_STATUS_BAD_ROW_INDEX);
    const RT* row = off < 0 ? nullptr : static_cast<const RT*>(src.rows) + off;
    const float a = alphas[static_cast<int64_t>(b) * k + kk];
    ACT* ug = Ug + static_cast<int64_t>(b) * d_B * ldu + static_cast<int64_t>(kk) * r;
    const int nU = d_B * r;
    for (int e = threadIdx.x; e < nU; e += blockDim.x) {
        const int j = e / r, rho = e - j * r;
        const float u = row ? Elem<RT>::to_f(row[e]) : 0.f;
        ug[static_cast<int64_t>(j) * ldu + rho] = Elem<ACT>::from_f(u);
    }
    const int64_t kr = static_cast<int64_t>(k) * r;
    ACT* vs = Vs + (static_cast<int64_t>(b) * kr + static_cast<int64_t>(kk) * r) * d_A;
    const int nV = r * d_A;
    for (int e = threadIdx.x; e < nV; e += blockDim.x) {
        const float x = row ? Elem<RT>::to_f(row[nU + e]) : 0.f;
        vs[e] = Elem<ACT>::from_f(a * x);
    }
}

// bf16 rows, bf16 activations, r == 8: one 16-byte vector per (row j, k) of U
// (its 8 factors) and per 8 elements of V.
__global__ void __launch_bounds__(256) prep_factors_bf16_r8_kernel(
    RowSrc src, const float* __restrict__ alphas, int d_A, int d_B, int64_t ldu,
    __nv_bfloat16* __restrict__ Ug, __nv_bfloat16* __restrict__ Vs, uint32_t* status) {
    pdl_enter();
    const int kk = blockIdx.x, b = blockIdx.y, k = src.k;
    const int64_t off = src.offset(b, kk);
    if (off < 0 && threadIdx.x == 0) raise_status(status, DWA_STATUS_BAD_ROW_INDEX);
    const uint4* row = off < 0 ? nullptr
                               : reinterpret_cast<const uint4*>(
                                     static_cast<const __nv_bfloat16*>(src.rows) + off);
    const float a = alphas[static_cast<int64_t>(b) * k + kk];
    const uint4 zero = make_uint4(0, 0, 0, 0);
    __nv_bfloat16* ug = Ug + static_cast<int64_t>(b) * d_B * ldu + static_cast<int64_t>(kk) * 8;
    const int64_t kr = static_cast<int64_t>(k) * 8;
    uint4* vs = reinterpret_cast<uint4*>(Vs + (static_cast<int64_t>(b) * kr + static_cast<int64_t>(kk) * 8) * d_A);
    // U: d_B vectors, V: d_A vectors (8 rows of d_A); up to 8 of each in flight
    for (int j0 = threadIdx.x; j0 < d_B || j0 < d_A; j0 += blockDim.x * 8) {
        uint4 u[8], v[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) {
            const int j = j0 + t * blockDim.x;
            u[t] = (row && j < d_B) ? __ldg(row + j) : zero;
            v[t] = (row && j < d_A) ? __ldg(row + d_B + j) : zero;
        }
#pragma unroll
        for (int t = 0; t < 8; ++t) {
            const int j = j0 + t * blockDim.x;
            if (j < d_B) *reinterpret_cast<uint4*>(ug + static_cast<int64_t>(j) * ldu) = u[t];
            if (j < d_A) {
                __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&v[t]);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float2 f = __bfloat1622float2(h[i]);
                    h[i] = __floats2bfloat162_rn(a * f.x, a * f.y);
                }
                vs[j] = v[t];
            }
        }
    }
}

// pb[b][j] = b_base[j] + sum_k alpha[b,k] b_k[j].  A CTA owns 8*32 = 256
// columns of one sequence: the k row offsets and weights are staged in shared
// memory first, then each of its 4 warps (8 columns per lane, one 16-byte
// load per row for bf16 rows) takes a quarter of the k rows with all loads
// independent, and the quarters' partial sums are added in order.
template <class RT>
__global__ void __launch_bounds__(128) prep_bias_kernel(RowSrc src, const float* __restrict__ alphas,
                                                        const float* __restrict__ b_base, int64_t s2,
                                                        int d_B, float* __restrict__ pb) {
    pdl_enter();
    __shared__ float part[4][256];
    extern __shared__ int64_t offs[];                 // [k] row offsets, then [k] weights (as float)
    float* wts = reinterpret_cast<float*>(offs + src.k);
    const int b = blockIdx.y, q = threadIdx.x >> 5, t = threadIdx.x & 31;
    for (int kk = threadIdx.x; kk < src.k; kk += blockDim.x) {
        offs[kk] = src.offset(b, kk);
        wts[kk] = alphas[static_cast<int64_t>(b) * src.k + kk];
    }
    __syncthreads();
    const int j0 = blockIdx.x * 256 + t * 8;
    const RT* rows = static_cast<const RT*>(src.rows);
    const int kq = (src.k + 3) / 4, k_lo = q * kq, k_hi = min(src.k, k_lo + kq);
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    const bool vec = (s2 % 8 == 0) && (src.D % 8 == 0) && j0 + 8 <= d_B &&
                     reinterpret_cast<uintptr_t>(rows) % 16 == 0;
#pragma unroll 8
    for (int kk = k_lo; kk < k_hi; ++kk) {
        const int64_t off = offs[kk];
        if (off < 0) continue;
        const float w = wts[kk];
        if (vec) {
            float x[8];
            load8(rows + off + s2 + j0, x);
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] = fmaf(w, x[i], acc[i]);
        } else {
            for (int i = 0; i < 8 && j0 + i < d_B; ++i)
                acc[i] = fmaf(w, Elem<RT>::to_f(rows[off + s2 + j0 + i]), acc[i]);
        }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) part[q][t * 8 + i] = acc[i];
    __syncthreads();
    for (int c = threadIdx.x; c < 256; c += blockDim.x) {
        const int j = blockIdx.x * 256 + c;
        if (j < d_B) pb[static_cast<int64_t>(b) * d_B + j] = b_base[j] + (((part[0][c] + part[1][c]) + part[2][c]) + part[3][c]);
    }
}

template <class RT>
__global__ void finalize_kernel(RowSrc src, const float* __restrict__ alphas,
                                const float* __restrict__ gbias, const float* __restrict__ dW_acc,
                                const float* __restrict__ gamma_acc, int64_t s2, int d_B,
                                float* __restrict__ g_rows, float* __restrict__ g_alpha,
                                float* __restrict__ g_gamma) {
    pdl_enter();
    const int kk = blockIdx.x, b = blockIdx.y, k = src.k;
    __shared__ float s_red[32];
    const int64_t off = src.offset(b, kk);
    const RT* bv = off < 0 ? nullptr : static_cast<const RT*>(src.rows) + off + s2;
    const float a = alphas[static_cast<int64_t>(b) * k + kk];
    const float* gb = gbias + static_cast<int64_t>(b) * d_B;
    float* gr = g_rows + (static_cast<int64_t>(b) * k + kk) * src.D;
    float dot = 0.f;
    for (int j = threadIdx.x; j < d_B; j += blockDim.x) {
        const float x = gb[j];
        if (bv) dot = fmaf(Elem<RT>::to_f(bv[j]), x, dot);
        gr[s2 + j] = a * x;
    }
    for (int64_t c = s2 + d_B + threadIdx.x; c < src.D; c += blockDim.x) gr[c] = 0.f;
    dot = warp_sum(dot);
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = dot;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.f;
        for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t += s_red[w];
        g_alpha[static_cast<int64_t>(b) * k + kk] = dW_acc[static_cast<int64_t>(b) * k + kk] + t;
        if (kk == 0 && b == 0) *g_gamma = *gamma_acc;
    }
}

__global__ void bias_grad_kernel(const float* __restrict__ gbias, int B, int d,
                                 float* __restrict__ g_b_base) {
    pdl_enter();
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= d) return;
    float acc = 0.f;
    for (int b = 0; b < B; ++b) acc += gbias[static_cast<int64_t>(b) * d + j];
    g_b_base[j] = acc;
}

// -------------------------------------------------------- factored apply ---
// h_mid without W: the Pallas kernel's own factored form
// (assembly_pallas.py:109-117), h_mid = h_A + gamma (h_A W_base^T + (h_A V_s^T) U_f) + pb,
// for sequences of a few rows (decode, T <= kFactoredMaxT).  Each gathered row
// is read once (its V part by factored_hv_kernel, its U and b parts by
// factored_out_kernel) and the d_B x d_A x k*r product that forming W costs is
// skipped: at T = 1 that product is ~700x the flops of the apply itself.
constexpr int kFactoredMaxT = 16;

// hv[b][t][kk*r + rho] = alpha[b,kk] <V_kk[rho], h_A[b][t]>: one warp per (kk, rho),
// eight per CTA; the warp streams the d_A elements of its V row with 16-byte loads.
// TMAX: compile-time bound on T (accumulators per lane).
template <class ACT, class RT, int TMAX>
__global__ void __launch_bounds__(256) factored_hv_kernel(RowSrc src, const float* __restrict__ alphas,
                                                          const ACT* __restrict__ hA, int T, int d_A,
                                                          int64_t s1, int r, bool vec,
                                                          float* __restrict__ hv, uint32_t* status) {
    pdl_enter();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b = blockIdx.y, k = src.k;
    const int kr = k * r;
    const int p = blockIdx.x * 8 + warp;
    if (p >= kr) return;
    const int kk = p / r, rho = p - kk * r;
    const int64_t off = src.offset(b, kk);
    float acc[TMAX];
#pragma unroll
    for (int t = 0; t < TMAX; ++t) acc[t] = 0.f;
    if (off < 0) {
        if (lane == 0 && rho == 0) raise_status(status, DWA_STATUS_BAD_ROW_INDEX);
    } else {
        const RT* V = static_cast<const RT*>(src.rows) + off + s1 + static_cast<int64_t>(rho) * d_A;
        const ACT* h = hA + static_cast<int64_t>(b) * T * d_A;
        if (vec) {
#pragma unroll 4
            for (int i0 = lane * 8; i0 < d_A; i0 += 256) {
                float v[8];
                load8(V + i0, v);
#pragma unroll
                for (int t = 0; t < TMAX; ++t) {
                    if (t < T) {
                        float x[8];
                        load8(h + static_cast<int64_t>(t) * d_A + i0, x);
#pragma unroll
                        for (int e = 0; e < 8; ++e) acc[t] = fmaf(v[e], x[e], acc[t]);
                    }
                }
            }
        } else {
            for (int i = lane; i < d_A; i += 32) {
                const float v = Elem<RT>::to_f(V[i]);
#pragma unroll
                for (int t = 0; t < TMAX; ++t)
                    if (t < T) acc[t] = fmaf(v, Elem<ACT>::to_f(h[static_cast<int64_t>(t) * d_A + i]), acc[t]);
            }
        }
    }
    const float a = off < 0 ? 0.f : __ldg(alphas + static_cast<int64_t>(b) * k + kk);
#pragma unroll
    for (int t = 0; t < TMAX; ++t) {
        if (t < T) {
            float s = acc[t];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            if (lane == 0) hv[(static_cast<int64_t>(b) * T + t) * kr + p] = a * s;
        }
    }
}

// h_mid[b][t][j] = h_A[b][t][j] + gamma (base[b*T+t][j] + sum_{kk,rho} U_kk[j][rho] hv[b][t][kk*r+rho])
//                  + b_base[j] + sum_kk alpha[b,kk] b_kk[j]
// One thread per output column j, 128 per CTA; hv[b], the k row offsets and
// alphas sit in shared memory; the U factors of (row kk, column j) are r
// consecutive elements, so a warp reads 32*r contiguous elements per row.
template <class ACT, class RT, int TMAX>
__global__ void __launch_bounds__(128) factored_out_kernel(RowSrc src, const float* __restrict__ alphas,
                                                           const ACT* __restrict__ hA,
                                                           const float* __restrict__ base,
                                                           const float* __restrict__ hv,
                                                           const float* __restrict__ b_base,
                                                           const float* __restrict__ gamma, int T, int d_B,
                                                           int r, int64_t s2, bool vec_u, int kchunk,
                                                           float* __restrict__ part, float* __restrict__ pbias,
                                                           ACT* __restrict__ h_mid) {
    pdl_enter();
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int b = blockIdx.y, k = src.k, kr = k * r;
    const int kk0 = blockIdx.z * kchunk, kk1 = min(k, kk0 + kchunk);
    float* s_hv = reinterpret_cast<float*>(smem_raw);                                // [T][kr]
    int64_t* s_off = reinterpret_cast<int64_t*>(s_hv + ((T * kr + 1) & ~1));          // [k]
    float* s_a = reinterpret_cast<float*>(s_off + k);                                // [k]
    for (int e = threadIdx.x; e < T * kr; e += blockDim.x)
        s_hv[e] = hv[static_cast<int64_t>(b) * T * kr + e];
    for (int kk = threadIdx.x; kk < k; kk += blockDim.x) {
        s_off[kk] = src.offset(b, kk);
        s_a[kk] = alphas[static_cast<int64_t>(b) * k + kk];
    }
    __syncthreads();
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= d_B) return;
    const RT* rows = static_cast<const RT*>(src.rows);
    float acc[TMAX];
#pragma unroll
    for (int t = 0; t < TMAX; ++t) acc[t] = 0.f;
    float bias = 0.f;
#pragma unroll 4
    for (int kk = kk0; kk < kk1; ++kk) {
        const int64_t off = s_off[kk];
        if (off < 0) continue;
        const RT* U = rows + off + static_cast<int64_t>(j) * r;
        bias = fmaf(s_a[kk], Elem<RT>::to_f(rows[off + s2 + j]), bias);
        const float* h = s_hv + kk * r;
        if (vec_u) {    // r == 8
            float u[8];
            load8(U, u);
#pragma unroll
            for (int t = 0; t < TMAX; ++t) {
                if (t < T) {
#pragma unroll
                    for (int e = 0; e < 8; ++e) acc[t] = fmaf(u[e], h[t * kr + e], acc[t]);
                }
            }
        } else {
            for (int rho = 0; rho < r; ++rho) {
                const float u = Elem<RT>::to_f(U[rho]);
#pragma unroll
                for (int t = 0; t < TMAX; ++t)
                    if (t < T) acc[t] = fmaf(u, h[t * kr + rho], acc[t]);
            }
        }
    }
    if (gridDim.z > 1) {   // row-split partial sums: factored_combine_kernel finishes
        const int64_t BT = static_cast<int64_t>(gridDim.y) * T;
#pragma unroll
        for (int t = 0; t < TMAX; ++t)
            if (t < T) part[(blockIdx.z * BT + static_cast<int64_t>(b) * T + t) * d_B + j] = acc[t];
        pbias[(static_cast<int64_t>(blockIdx.z) * gridDim.y + b) * d_B + j] = bias;
        return;
    }
    const float g = __ldg(gamma);
    const float pbj = b_base[j] + bias;
#pragma unroll
    for (int t = 0; t < TMAX; ++t) {
        if (t < T) {
            const int64_t o = (static_cast<int64_t>(b) * T + t) * d_B + j;
            h_mid[o] = Elem<ACT>::from_f(Elem<ACT>::to_f(hA[o]) + g * (base[o] + acc[t]) + pbj);
        }
    }
}

// h_mid from the row-split partial sums of factored_out_kernel, added in split order.
template <class ACT>
__global__ void __launch_bounds__(256) factored_combine_kernel(const float* __restrict__ part,
                                                               const float* __restrict__ pbias, int nsplit,
                                                               const ACT* __restrict__ hA,
                                                               const float* __restrict__ base,
                                                               const float* __restrict__ b_base,
                                                               const float* __restrict__ gamma, int B, int T,
                                                               int d_B, ACT* __restrict__ h_mid) {
    pdl_enter();
    const int64_t BT = static_cast<int64_t>(B) * T, n = BT * d_B;
    const int64_t o = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (o >= n) return;
    const int j = static_cast<int>(o % d_B);
    const int64_t bt = o / d_B;
    const int b = static_cast<int>(bt / T);
    float acc = 0.f, bias = 0.f;
    for (int z = 0; z < nsplit; ++z) {
        acc += part[z * n + o];
        bias += pbias[(static_cast<int64_t>(z) * B + b) * d_B + j];
    }
    const float g = __ldg(gamma);
    h_mid[o] = Elem<ACT>::from_f(Elem<ACT>::to_f(hA[o]) + g * (base[o] + acc) + (b_base[j] + bias));
}

// 4 consecutive elements as floats (8-byte bf16 / 16-byte f32 access).
__device__ __forceinline__ void load4(const float* p, float* v) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
}
__device__ __forceinline__ void load4(const __nv_bfloat16* p, float* v) {
    const uint2 t = *reinterpret_cast<const uint2*>(p);
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&t.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&t.y));
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}

// base[m][j] = <W_base[j], h[m]> for a few rows m (M <= MMAX): W_base is read
// once, in fp32, straight from the parameter (no cast, no tile padding).  A
// CTA owns 4 rows of W_base (every h load feeds 4 of them) and its 8 warps
// split the d_A columns, so that 8x more loads are in flight than with one
// warp per row group; the 8 partial sums are added in warp order.
template <class ACT, int MMAX>
__global__ void __launch_bounds__(256) base_rows_kernel(const float* __restrict__ W_base,
                                                        const ACT* __restrict__ hA, int M, int d_A, int d_B,
                                                        bool vec, float* __restrict__ base) {
    pdl_enter();
    __shared__ float s_part[8][4][MMAX];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int j0 = blockIdx.x * 4;
    const int nj = min(4, d_B - j0);
    float acc[4][MMAX];
#pragma unroll
    for (int jj = 0; jj < 4; ++jj)
#pragma unroll
        for (int m = 0; m < MMAX; ++m) acc[jj][m] = 0.f;
    if (vec) {
        const int span = (d_A / 4 + 7) / 8 * 4;          // columns per warp, a multiple of 4
        const int c0 = warp * span, c1 = min(d_A, c0 + span);
#pragma unroll 2
        for (int i0 = c0 + lane * 4; i0 < c1; i0 += 128) {
            float4 w[4];
#pragma unroll
            for (int jj = 0; jj < 4; ++jj)
                w[jj] = jj < nj ? __ldg(reinterpret_cast<const float4*>(W_base + static_cast<int64_t>(j0 + jj) * d_A + i0))
                                : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int m = 0; m < MMAX; ++m) {
                if (m < M) {
                    float x[4];
                    load4(hA + static_cast<int64_t>(m) * d_A + i0, x);
#pragma unroll
                    for (int jj = 0; jj < 4; ++jj)
                        acc[jj][m] = fmaf(w[jj].x, x[0], fmaf(w[jj].y, x[1], fmaf(w[jj].z, x[2],
                                     fmaf(w[jj].w, x[3], acc[jj][m]))));
                }
            }
        }
    } else {
        for (int i = threadIdx.x; i < d_A; i += 256) {
            float w[4];
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) w[jj] = jj < nj ? W_base[static_cast<int64_t>(j0 + jj) * d_A + i] : 0.f;
#pragma unroll
            for (int m = 0; m < MMAX; ++m) {
                if (m < M) {
                    const float x = Elem<ACT>::to_f(hA[static_cast<int64_t>(m) * d_A + i]);
#pragma unroll
                    for (int jj = 0; jj < 4; ++jj) acc[jj][m] = fmaf(w[jj], x, acc[jj][m]);
                }
            }
        }
    }
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
#pragma unroll
        for (int m = 0; m < MMAX; ++m) {
            if (m < M) {
                float v = acc[jj][m];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                if (lane == 0) s_part[warp][jj][m] = v;
            }
        }
    }
    __syncthreads();
    for (int t = threadIdx.x; t < 4 * MMAX; t += blockDim.x) {
        const int jj = t / MMAX, m = t - jj * MMAX;
        if (jj < nj && m < M) {
            float v = 0.f;
            for (int w = 0; w < 8; ++w) v += s_part[w][jj][m];
            base[static_cast<int64_t>(m) * d_B + j0 + jj] = v;
        }
    }
}

// W_base in the activation dtype (the B operand of the batched base GEMM).
__global__ void __launch_bounds__(256) cast_bf16_kernel(const float* __restrict__ x, int64_t n, bool vec,
                                                        __nv_bfloat16* __restrict__ y) {
    pdl_enter();
    const int64_t n8 = vec ? n / 8 : 0;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n8;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        float v[8];
        load8(x + i * 8, v);
        store8(y + i * 8, v);
    }
    for (int64_t i = n8 * 8 + blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        y[i] = __float2bfloat16_rn(x[i]);
}

// base[row][j] = acc (row = b*T + t of the batched h_A W_base^T)
struct EpiStore : NoReduce {
    float* out; int N; bool vec;
    struct Frag {};
    __device__ void load(int, int, int, int, Frag&) const {}
    __device__ float finish(int, int row, int col0, const float* v, int cnt, const Frag&) const {
        float* o = out + static_cast<int64_t>(row) * N + col0;
        if (vec && cnt == 8) {
            store8(o, v);
        } else {
            for (int c = 0; c < cnt; ++c) o[c] = v[c];
        }
        return 0.f;
    }
    DWA_EPI_CALL
};

// ------------------------------------------------------------------ host ---
static bool force_simt() {
    static const bool v = [] {
        const char* e = std::getenv("DWA_GEMM");
        return e && std::string(e) == "simt";
    }();
    return v;
}

// GEMMs (by name) that run two 128-column CTAs per SM (DWA_GEMM_PAIR: "all" or a
// comma-separated list of names).
static bool pair_config(const char* name) {
    const char* v = std::getenv("DWA_GEMM_PAIR");
    if (!v || !*v) return false;
    if (std::strcmp(v, "all") == 0) return true;
    const size_t n = std::strlen(name);
    for (const char* p = v; *p;) {
        const char* q = std::strchr(p, ',');
        const size_t len = q ? static_cast<size_t>(q - p) : std::strlen(p);
        if (len == n && std::strncmp(p, name, n) == 0) return true;
        if (!q) break;
        p = q + 1;
    }
    return false;
}

template <class ACT, bool A_MN, bool B_MN, class Epi>
static int gemm(const char* name, const void* a, int64_t lda, int64_t bsa, const void* b, int64_t ldb, int64_t bsb,
                int M, int N, int K, int batch, const Epi& epi, uint32_t* status, cudaStream_t st) {
    if constexpr (std::is_same<ACT, __nv_bfloat16>::value) {
      if (!force_simt()) {
        const tc::Operand A{a, A_MN, lda, bsa}, B{b, B_MN, ldb, bsb};
        if (pair_config(name) && N >= 128 && tc::tc_operand_ok(A, M, K, 128) && tc::tc_operand_ok(B, N, K, 128)) {
            ++g_launches_tc;
            prof_begin(name, st);
            const int rc = tc::launch_gemm_bf16<128, 3, A_MN, B_MN, Epi, 8>(A, B, M, N, K, batch, epi, status, st);
            prof_end(name, st);
            return rc;
        }
        const int64_t ctas256 = static_cast<int64_t>((M + 127) / 128) * ((N + 255) / 256) * batch;
        // persistent only when CTAs get several tiles (a single wave gains nothing
        // from it), and for short K (the store-heavy W epilogue) only from four
        // waves on: below that one tile per CTA is as fast
        const bool pers = tc::persistent_gemm() && ctas256 > tc::sm_count() &&
                          (K >= 1024 || ctas256 >= 4 * static_cast<int64_t>(tc::sm_count()));
        // long-K multi-wave GEMMs (the apply product) on CTA pairs: 256-row tiles
        // whose two CTAs stage half of B each
        if (pers && K >= 1024 && tc::pair_gemm() && N >= 256 && M >= 256 && tc::tc_operand_ok(A, M, K, 128) &&
            tc::tc_operand_ok(B, N, K, 128)) {
            ++g_launches_tc;
            prof_begin(name, st);
            const int rc = tc::launch_gemm_bf16_pair<256, 6, A_MN, B_MN>(A, B, M, N, K, batch, epi, status, st);
            prof_end(name, st);
            return rc;
        }
        if (N >= 256 && ctas256 >= 120 && tc::tc_operand_ok(A, M, K, 128) &&
            tc::tc_operand_ok(B, N, K, 256)) {
            ++g_launches_tc;
            prof_begin(name, st);
            const int rc = pers ? tc::launch_gemm_bf16_persistent<256, 4, A_MN, B_MN>(A, B, M, N, K, batch, epi, status, st)
                                : tc::launch_gemm_bf16<256, 4, A_MN, B_MN>(A, B, M, N, K, batch, epi, status, st);
            prof_end(name, st);
            return rc;
        }
        if (N >= 128 && tc::tc_operand_ok(A, M, K, 128) && tc::tc_operand_ok(B, N, K, 128)) {
            ++g_launches_tc;
            prof_begin(name, st);
            const int rc = pers ? tc::launch_gemm_bf16_persistent<128, 6, A_MN, B_MN>(A, B, M, N, K, batch, epi, status, st)
                                : tc::launch_gemm_bf16<128, 6, A_MN, B_MN>(A, B, M, N, K, batch, epi, status, st);
            prof_end(name, st);
            return rc;
        }
      }
    }
    const simt::Operand A{a, A_MN, lda, bsa}, B{b, B_MN, ldb, bsb};
    ++g_launches_simt;
    prof_begin(name, st);
    const int rc = simt::launch_gemm<ACT, ACT>(A, B, M, N, K, batch, epi, st);
    prof_end(name, st);
    return rc;
}

static int check_dims(const DwaAssembleDims* d) {
    if (!d) return fail(DWA_ERR_INVALID_ARG, "dims is NULL");
    if (d->B <= 0 || d->T <= 0 || d->k <= 0 || d->r <= 0 || d->d_A <= 0 || d->d_B <= 0)
        return fail(DWA_ERR_INVALID_ARG, "B, T, k, r, d_A, d_B must be positive");
    if (d->d_A != d->d_B)
        return fail(DWA_ERR_INVALID_ARG, "d_A must equal d_B for the residual (config.py:59)");
    const int64_t need = static_cast<int64_t>(d->d_B) * d->r + static_cast<int64_t>(d->r) * d->d_A + d->d_B;
    if (d->D < need)
        return fail(DWA_ERR_INVALID_ARG, "D < d_B*r + r*d_A + d_B (config.py:54-58)");
    if ((d->act_dtype != DWA_F32 && d->act_dtype != DWA_BF16) ||
        (d->rows_dtype != DWA_F32 && d->rows_dtype != DWA_BF16))
        return fail(DWA_ERR_INVALID_ARG, "dtype must be DWA_F32 or DWA_BF16");
    if (static_cast<int64_t>(d->k) * d->r > (1 << 30) || static_cast<int64_t>(d->T) > (1 << 30))
        return fail(DWA_ERR_INVALID_ARG, "size out of range");
    return DWA_OK;
}

struct AsmWorkspace {
    uint32_t* status;
    void* Ug;       // [B, d_B, ldu] act
    void* Vs;       // [B, kr, d_A]  act
    float* pb;      // [B, d_B]
    void* Wact;     // [B, d_B, d_A] act (forward, when the caller passes none)
    void* gW;       // [B, d_B, d_A] act (backward)
    float* gbias;   // [B, d_B]
    float* dW_acc;  // [B, k]
    float* gamma_acc;
    int64_t ldu;
    size_t bytes;
};

static AsmWorkspace carve(void* base, const DwaAssembleDims& d, bool bwd) {
    Carver c(base);
    AsmWorkspace w{};
    const size_t es = dtype_bytes(d.act_dtype);
    const int64_t kr = static_cast<int64_t>(d.k) * d.r;
    w.ldu = static_cast<int64_t>(align_up(static_cast<size_t>(kr), 8));
    w.status = static_cast<uint32_t*>(base);
    w.Ug = c.take<char>(static_cast<size_t>(d.B) * d.d_B * w.ldu * es);
    w.Vs = c.take<char>(static_cast<size_t>(d.B) * kr * d.d_A * es);
    w.pb = c.take<float>(static_cast<size_t>(d.B) * d.d_B);
    w.Wact = c.take<char>(static_cast<size_t>(d.B) * d.d_B * d.d_A * es);
    if (bwd) {
        w.gW = c.take<char>(static_cast<size_t>(d.B) * d.d_B * d.d_A * es);
        w.gbias = c.take<float>(static_cast<size_t>(d.B) * d.d_B);
        w.dW_acc = c.take<float>(static_cast<size_t>(d.B) * d.k);
        w.gamma_acc = c.take<float>(64);
    }
    w.bytes = c.bytes();
    return w;
}

// The W GEMM with the TMA epilogue (tc_gemm_w.cuh): bf16 activations, both
// W (fp32) and W_act (bf16) written, 16-byte aligned buffers and rows, and a
// grid of more than one wave (small workload, 1.7 waves: 28 -> 21 us);
// DWA_W_EPILOGUE=lsu keeps the per-thread epilogue.
template <class ACT>
static bool w_tma_epilogue(const DwaAssembleDims& d, const float* W_base, const float* W_out, const void* W_act,
                           const AsmWorkspace& w, int64_t kr) {
    if constexpr (!std::is_same<ACT, __nv_bfloat16>::value) {
        return false;
    } else {
        static const bool lsu = [] {
            const char* v = std::getenv("DWA_W_EPILOGUE");
            return v && std::strcmp(v, "lsu") == 0;
        }();
        if (lsu || force_simt() || !tc::persistent_gemm() || !W_base || !W_out || !W_act) return false;
        if (d.d_A % 8 != 0 || d.d_A < 256 || kr < 64) return false;
        const auto al16 = [](const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
        if (!al16(W_base) || !al16(W_out) || !al16(W_act)) return false;
        const int64_t ctas256 = static_cast<int64_t>((d.d_B + 127) / 128) * ((d.d_A + 255) / 256) * d.B;
        if (ctas256 <= static_cast<int64_t>(tc::sm_count())) return false;
        const tc::Operand A{w.Ug, false, w.ldu, static_cast<int64_t>(d.d_B) * w.ldu}, B{w.Vs, true, d.d_A, kr * d.d_A};
        return tc::tc_operand_ok(A, d.d_B, kr, 128) && tc::tc_operand_ok(B, d.d_A, kr, 256);
    }
}

static bool vec_ok(const void* p, int64_t ld, size_t es) {
    return p == nullptr ||
           ((reinterpret_cast<uintptr_t>(p) % 16 == 0) && ((ld * static_cast<int64_t>(es)) % 16 == 0));
}

template <class ACT, class RT>
static int prep(cudaStream_t st, const DwaAssembleDims& d, const RowSrc& src, const float* alphas,
                const float* b_base, const AsmWorkspace& w, bool with_factors, bool with_bias) {
    dim3 g1(d.k, d.B);
    const bool vec8 = std::is_same<ACT, __nv_bfloat16>::value && std::is_same<RT, __nv_bfloat16>::value &&
                      d.r == 8 && d.D % 8 == 0 && d.d_A % 8 == 0 && w.ldu % 8 == 0 &&
                      reinterpret_cast<uintptr_t>(src.rows) % 16 == 0;
    if (!with_factors) {
    } else if (vec8)
        DWA_TIMED("prep_factors", st,
                  launch_pdl(prep_factors_bf16_r8_kernel, g1, 256, 0, st, 
                      src, alphas, d.d_A, d.d_B, w.ldu, static_cast<__nv_bfloat16*>(w.Ug),
                      static_cast<__nv_bfloat16*>(w.Vs), w.status));
    else
        DWA_TIMED("prep_factors", st,
                  launch_pdl(prep_factors_kernel<ACT, RT>, g1, 256, 0, st, src, alphas, d.d_A, d.d_B, d.r,
                                                                   w.ldu, static_cast<ACT*>(w.Ug),
                                                                   static_cast<ACT*>(w.Vs), w.status));
    DWA_LAUNCH_CHECK("prep_factors_kernel");
    if (with_factors) ++g_launches_total;
    if (with_bias) {
        const int64_t s2 = static_cast<int64_t>(d.d_B) * d.r + static_cast<int64_t>(d.r) * d.d_A;
        dim3 g2((d.d_B + 255) / 256, d.B);
        DWA_TIMED("prep_bias", st,
                  launch_pdl(prep_bias_kernel<RT>, g2, 128, static_cast<size_t>(d.k) * 12, st, src, alphas, b_base,
                             s2, d.d_B, w.pb));
        DWA_LAUNCH_CHECK("prep_bias_kernel");
        ++g_launches_total;
    }
    return DWA_OK;
}

template <class ACT, class RT>
static int fwd_impl(cudaStream_t st, const DwaAssembleDims& d, const RowSrc& src,
                    const float* alphas, const ACT* hA, const float* W_base, const float* b_base,
                    const float* gamma, ACT* h_mid, float* W_out, ACT* W_act, const AsmWorkspace& w) {
    Lanes lanes(st);
    int rc = lanes.rc;
    if (rc) return rc;
    // aux0: the bias pb (needed only by the apply epilogue); main: factors + W
    if ((rc = prep<ACT, RT>(lanes.aux[0], d, src, alphas, b_base, w, false, true))) return rc;
    if ((rc = prep<ACT, RT>(st, d, src, alphas, b_base, w, true, false))) return rc;
    const int64_t kr = static_cast<int64_t>(d.k) * d.r;
    const size_t es = sizeof(ACT);
    if (std::is_same<ACT, float>::value && W_act == reinterpret_cast<ACT*>(W_out)) W_act = nullptr;
    ACT* Wop = W_act ? W_act
                     : (std::is_same<ACT, float>::value && W_out ? reinterpret_cast<ACT*>(W_out)
                                                                 : static_cast<ACT*>(w.Wact));
    ACT* Wact_store = (Wop == reinterpret_cast<ACT*>(W_out)) ? nullptr : Wop;
    const int64_t dd = static_cast<int64_t>(d.d_B) * d.d_A;

    EpiW<ACT> ew;
    ew.W_base = W_base; ew.W_out = W_out; ew.W_act = Wact_store; ew.d_B = d.d_B; ew.d_A = d.d_A;
    ew.vec = vec_ok(W_base, d.d_A, 4) && vec_ok(W_out, d.d_A, 4) && vec_ok(Wact_store, d.d_A, es);
    // A = Ug (M=d_B, K=kr, K-major); B = Vs (N=d_A, K=kr, MN-major)
    if (w_tma_epilogue<ACT>(d, W_base, W_out, Wact_store, w, kr)) {
        const tc::Operand A{w.Ug, false, w.ldu, static_cast<int64_t>(d.d_B) * w.ldu}, B{w.Vs, true, d.d_A, kr * d.d_A};
        ++g_launches_tc;
        prof_begin("gemm_W", st);
        rc = tc::launch_gemm_w_tma(A, B, d.d_B, d.d_A, static_cast<int>(kr), d.B, W_base, W_out, Wact_store, w.status,
                                   st);
        prof_end("gemm_W", st);
    } else {
        rc = gemm<ACT, false, true>("gemm_W", w.Ug, w.ldu, static_cast<int64_t>(d.d_B) * w.ldu, w.Vs, d.d_A,
                                    kr * d.d_A, d.d_B, d.d_A, static_cast<int>(kr), d.B, ew, w.status, st);
    }
    if (rc) return rc;
    ++g_launches_total;

    if ((rc = lanes.join())) return rc;
    EpiApply<ACT> ea;
    ea.hA = hA; ea.pb = w.pb; ea.gamma = gamma; ea.out = h_mid; ea.T = d.T; ea.d = d.d_B;
    ea.vec = vec_ok(hA, d.d_A, es) && vec_ok(h_mid, d.d_B, es) && vec_ok(w.pb, d.d_B, 4);
    // A = h_A (M=T, K=d_A, K-major); B = W (N=d_B, K=d_A, K-major)
    rc = gemm<ACT, false, false>("gemm_apply", hA, d.d_A, static_cast<int64_t>(d.T) * d.d_A, Wop, d.d_A, dd, d.T,
                                 d.d_B, d.d_A, d.B, ea, w.status, st);
    if (rc) return rc;
    ++g_launches_total;
    return DWA_OK;
}

template <class ACT, class RT>
static int bwd_impl(cudaStream_t st, const DwaAssembleDims& d, const RowSrc& src,
                    const float* alphas, const ACT* hA, const ACT* Wact, const float* gamma,
                    const ACT* g, const float* gWo, float* g_rows, float* g_alpha, ACT* g_hA,
                    float* g_W_base, float* g_b_base, float* g_gamma, const AsmWorkspace& w) {
    const int64_t kr = static_cast<int64_t>(d.k) * d.r;
    const int64_t dd = static_cast<int64_t>(d.d_B) * d.d_A;
    const int64_t s1 = static_cast<int64_t>(d.d_B) * d.r;
    const int64_t s2 = s1 + static_cast<int64_t>(d.r) * d.d_A;
    const size_t es = sizeof(ACT);
    DWA_CUDA_TRY(cudaMemsetAsync(g_W_base, 0, dd * sizeof(float), st));
    DWA_CUDA_TRY(cudaMemsetAsync(w.dW_acc, 0, static_cast<size_t>(d.B) * d.k * sizeof(float), st));
    DWA_CUDA_TRY(cudaMemsetAsync(w.gamma_acc, 0, sizeof(float), st));
    // Three lanes:  main: G -> P      aux0: prep -> gh -> Q      aux1: colsum
    Lanes lanes(st);
    int rc = lanes.rc;
    if (rc) return rc;
    cudaStream_t a0 = lanes.aux[0], a1 = lanes.aux[1];
    ACT* gW = static_cast<ACT*>(w.gW);

    EpiG<ACT> eg;
    eg.gamma = gamma; eg.gWo = gWo; eg.gW = gW; eg.gWbase = g_W_base; eg.Wact = Wact;
    eg.gamma_acc = w.gamma_acc; eg.d_B = d.d_B; eg.d_A = d.d_A;
    eg.vec = vec_ok(gWo, d.d_A, 4) && vec_ok(gW, d.d_A, es) && vec_ok(g_W_base, d.d_A, 4) &&
             vec_ok(Wact, d.d_A, es);
    // G = g^T h: A(m=j,k=t) = g[t][j] MN-major; B(n=i,k=t) = h[t][i] MN-major
    rc = gemm<ACT, true, true>("gemm_G", g, d.d_B, static_cast<int64_t>(d.T) * d.d_B, hA, d.d_A,
                               static_cast<int64_t>(d.T) * d.d_A, d.d_B, d.d_A, d.T, d.B, eg,
                               w.status, st);
    if (rc) return rc;
    ++g_launches_total;

    if (d.d_B % 8 == 0 && reinterpret_cast<uintptr_t>(g) % 16 == 0) {
        DWA_TIMED("colsum", a1, launch_column_sum8<ACT>(a1, g, d.B, d.T, d.d_B, 0, w.gbias));
    } else {
        dim3 gc((d.d_B + 63) / 64, d.B);
        DWA_TIMED("colsum", a1, launch_pdl(column_sum_kernel<ACT>, gc, 1024, 0, a1, g, d.T, d.d_B, 0, w.gbias));
    }
    DWA_LAUNCH_CHECK("colsum_kernel");
    DWA_TIMED("bias_grad", a1,
              launch_pdl(bias_grad_kernel, (d.d_B + 255) / 256, 256, 0, a1, w.gbias, d.B, d.d_B, g_b_base));
    DWA_LAUNCH_CHECK("bias_grad_kernel");
    g_launches_total += 2;

    if ((rc = prep<ACT, RT>(a0, d, src, alphas, nullptr, w, true, false))) return rc;
    EpiGhA<ACT> eh;
    eh.g = g; eh.gamma = gamma; eh.out = g_hA; eh.T = d.T; eh.d = d.d_A;
    eh.vec = vec_ok(g, d.d_A, es) && vec_ok(g_hA, d.d_A, es);
    // g W: A(m=t,k=j) = g[t][j] K-major; B(n=i,k=j) = W[j][i] MN-major
    rc = gemm<ACT, false, true>("gemm_gh", g, d.d_B, static_cast<int64_t>(d.T) * d.d_B, Wact, d.d_A, dd, d.T,
                                d.d_A, d.d_B, d.B, eh, w.status, a0);
    if (rc) return rc;
    ++g_launches_total;

    // main: P needs gW (main) and Vs (aux0's prep)
    if ((rc = lanes.depend(st, a0, 1))) return rc;
    EpiP ep;
    ep.g_rows = g_rows; ep.D = d.D; ep.k = d.k; ep.r = d.r;
    ep.vec = vec_ok(g_rows, d.D, 4);
    // g_U = gW Vs^T: A(m=j,k=i) = gW[j][i] K-major; B(n=kr,k=i) = Vs[n][i] K-major
    rc = gemm<ACT, false, false>("gemm_P", gW, d.d_A, dd, w.Vs, d.d_A, kr * d.d_A, d.d_B,
                                 static_cast<int>(kr), d.d_A, d.B, ep, w.status, st);
    if (rc) return rc;
    ++g_launches_total;

    // aux0: Q needs gW (main's G) and Ug (its own prep)
    if ((rc = lanes.depend(a0, st, 2))) return rc;
    EpiQ<RT> eq;
    eq.src = src; eq.alphas = alphas; eq.g_rows = g_rows; eq.dW_acc = w.dW_acc; eq.s1 = s1;
    eq.d_A = d.d_A; eq.r = d.r;
    eq.vec = vec_ok(g_rows, d.D, 4) && (s1 % 8 == 0) && (d.d_A % 8 == 0) &&
             vec_ok(src.rows, d.D, sizeof(RT));
    // Q = Ug^T gW: A(m=kr,k=j) = Ug[j][m] MN-major; B(n=i,k=j) = gW[j][i] MN-major
    rc = gemm<ACT, true, true>("gemm_Q", w.Ug, w.ldu, static_cast<int64_t>(d.d_B) * w.ldu, gW, d.d_A, dd,
                               static_cast<int>(kr), d.d_A, d.d_B, d.B, eq, w.status, a0);
    if (rc) return rc;
    ++g_launches_total;

    if ((rc = lanes.join())) return rc;
    dim3 gf(d.k, d.B);
    DWA_TIMED("finalize", st,
              launch_pdl(finalize_kernel<RT>, gf, 256, 0, st, src, alphas, w.gbias, w.dW_acc, w.gamma_acc, s2,
                                                      d.d_B, g_rows, g_alpha, g_gamma));
    DWA_LAUNCH_CHECK("finalize_kernel");
    ++g_launches_total;
    return DWA_OK;
}

static int check_ws(void* ws, size_t have, size_t need) {
    if (!ws) return fail(DWA_ERR_WORKSPACE, "workspace is NULL");
    if (reinterpret_cast<uintptr_t>(ws) % 256 != 0)
        return fail(DWA_ERR_WORKSPACE, "workspace must be 256-byte aligned");
    if (have < need)
        return fail(DWA_ERR_WORKSPACE, "workspace too small: need " + std::to_string(need) +
                                           " bytes, got " + std::to_string(have));
    return DWA_OK;
}

}  // namespace dwa

using namespace dwa;

extern "C" size_t dwa_assemble_workspace_bytes(const DwaAssembleDims* dims, int with_backward) {
    if (check_dims(dims)) return 0;
    return carve(nullptr, *dims, with_backward != 0).bytes;
}

extern "C" int dwa_assemble_fwd(void* stream, const DwaAssembleDims* dims, const void* rows,
                                const int32_t* row_index, const float* alphas, const void* h_A,
                                const float* W_base, const float* b_base, const float* gamma,
                                void* h_mid, float* W_out, void* W_act, void* workspace,
                                size_t workspace_bytes) {
    int rc = check_dims(dims);
    if (rc) return rc;
    const DwaAssembleDims& d = *dims;
    if (!rows || !alphas || !h_A || !W_base || !b_base || !gamma || !h_mid)
        return fail(DWA_ERR_INVALID_ARG, "a required pointer is NULL");
    const AsmWorkspace w = carve(workspace, d, false);
    if ((rc = check_ws(workspace, workspace_bytes, w.bytes))) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const RowSrc src{rows, row_index, row_index ? d.n_rows : static_cast<int64_t>(d.B) * d.k, d.D,
                     d.k, d.rows_dtype};
    if (d.act_dtype == DWA_BF16) {
        using A = __nv_bfloat16;
        if (d.rows_dtype == DWA_BF16)
            return fwd_impl<A, __nv_bfloat16>(st, d, src, alphas, static_cast<const A*>(h_A), W_base,
                                              b_base, gamma, static_cast<A*>(h_mid), W_out,
                                              static_cast<A*>(W_act), w);
        return fwd_impl<A, float>(st, d, src, alphas, static_cast<const A*>(h_A), W_base, b_base,
                                  gamma, static_cast<A*>(h_mid), W_out, static_cast<A*>(W_act), w);
    }
    if (d.rows_dtype == DWA_BF16)
        return fwd_impl<float, __nv_bfloat16>(st, d, src, alphas, static_cast<const float*>(h_A),
                                              W_base, b_base, gamma, static_cast<float*>(h_mid),
                                              W_out, static_cast<float*>(W_act), w);
    return fwd_impl<float, float>(st, d, src, alphas, static_cast<const float*>(h_A), W_base, b_base,
                                  gamma, static_cast<float*>(h_mid), W_out,
                                  static_cast<float*>(W_act), w);
}

extern "C" int dwa_assemble_bwd(void* stream, const DwaAssembleDims* dims, const void* rows,
                                const int32_t* row_index, const float* alphas, const void* h_A,
                                const void* W_act, const float* gamma, const void* g_hmid,
                                const float* g_W_out, float* g_rows, float* g_alpha, void* g_hA,
                                float* g_W_base, float* g_b_base, float* g_gamma, void* workspace,
                                size_t workspace_bytes) {
    int rc = check_dims(dims);
    if (rc) return rc;
    const DwaAssembleDims& d = *dims;
    if (!rows || !alphas || !h_A || !W_act || !gamma || !g_hmid || !g_rows || !g_alpha || !g_hA ||
        !g_W_base || !g_b_base || !g_gamma)
        return fail(DWA_ERR_INVALID_ARG, "a required pointer is NULL");
    const AsmWorkspace w = carve(workspace, d, true);
    if ((rc = check_ws(workspace, workspace_bytes, w.bytes))) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const RowSrc src{rows, row_index, row_index ? d.n_rows : static_cast<int64_t>(d.B) * d.k, d.D,
                     d.k, d.rows_dtype};
#define DWA_BWD_ARGS(A, R)                                                                       \
    st, d, src, alphas, static_cast<const A*>(h_A), static_cast<const A*>(W_act), gamma,         \
        static_cast<const A*>(g_hmid), g_W_out, g_rows, g_alpha, static_cast<A*>(g_hA), g_W_base, \
        g_b_base, g_gamma, w
    if (d.act_dtype == DWA_BF16) {
        if (d.rows_dtype == DWA_BF16)
            return bwd_impl<__nv_bfloat16, __nv_bfloat16>(DWA_BWD_ARGS(__nv_bfloat16, __nv_bfloat16));
        return bwd_impl<__nv_bfloat16, float>(DWA_BWD_ARGS(__nv_bfloat16, float));
    }
    if (d.rows_dtype == DWA_BF16)
        return bwd_impl<float, __nv_bfloat16>(DWA_BWD_ARGS(float, __nv_bfloat16));
    return bwd_impl<float, float>(DWA_BWD_ARGS(float, float));
#undef DWA_BWD_ARGS
}

// ------------------------------------------------- factored apply (host) ---
namespace dwa {

static size_t factored_smem(const DwaAssembleDims& d) {
    const size_t kr = static_cast<size_t>(d.k) * d.r;
    return align_up(static_cast<size_t>(d.T) * kr, 2) * sizeof(float) +
           static_cast<size_t>(d.k) * (sizeof(int64_t) + sizeof(float));
}

// The factored kernels hold T accumulators per thread and hv[b] in shared memory.
static bool factored_ok(const DwaAssembleDims& d) {
    return d.T <= kFactoredMaxT && factored_smem(d) <= 160 * 1024;
}

// Rows of the base product up to which base_rows_kernel runs; beyond, a GEMM
// (bf16: the tensor-core GEMM over h_A padded to whole 128-row tiles).
constexpr int kBaseRowsMax = 16;

static bool base_on_tensor_cores(const DwaAssembleDims& d) {
    return d.act_dtype == DWA_BF16 && static_cast<int64_t>(d.B) * d.T > kBaseRowsMax;
}

struct FactWorkspace {
    uint32_t* status;
    void* Wb;       // [d_B, d_A] W_base in the activation dtype (bf16 activations, B*T > 16)
    void* hpad;     // [Mp, d_A] h_A rows padded with zeros to a whole 128-row tile (same case)
    float* hv;      // [B, T, k*r]
    float* base;    // [Mp, d_B] h_A W_base^T
    float* part;    // [nsplit, B*T, d_B] row-split partial sums (nsplit > 1)
    float* pbias;   // [nsplit, B, d_B]
    int nsplit, kchunk;
    size_t bytes;
};

// Splits of the k rows of factored_out_kernel: enough CTAs for two per SM
// when the batch alone gives fewer, at least 4 rows per split.
static void factored_split(const DwaAssembleDims& d, int* nsplit, int* kchunk) {
    const int64_t ctas = static_cast<int64_t>((d.d_B + 127) / 128) * d.B;
    int ns = static_cast<int>(std::min<int64_t>((2 * 148 + ctas - 1) / ctas, std::max(1, d.k / 4)));
    ns = std::max(ns, 1);
    const int kc = (d.k + ns - 1) / ns;
    *kchunk = kc;
    *nsplit = (d.k + kc - 1) / kc;
}

static FactWorkspace carve_factored(void* base, const DwaAssembleDims& d) {
    Carver c(base);
    FactWorkspace w{};
    w.status = static_cast<uint32_t*>(base);
    const size_t bt = static_cast<size_t>(d.B) * d.T, kr = static_cast<size_t>(d.k) * d.r;
    const bool tc = base_on_tensor_cores(d);
    const size_t mp = tc ? align_up(bt, 128) : bt;
    w.Wb = c.take<char>(tc ? static_cast<size_t>(d.d_B) * d.d_A * 2 : 0);
    w.hpad = c.take<char>(tc ? mp * d.d_A * 2 : 0);
    w.hv = c.take<float>(bt * kr);
    w.base = c.take<float>(mp * d.d_B);
    factored_split(d, &w.nsplit, &w.kchunk);
    const size_t ns = w.nsplit > 1 ? static_cast<size_t>(w.nsplit) : 0;
    w.part = c.take<float>(ns * bt * d.d_B);
    w.pbias = c.take<float>(ns * d.B * d.d_B);
    w.bytes = c.bytes();
    return w;
}

static bool aligned16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

template <class ACT, class RT>
static int factored_impl(cudaStream_t st, const DwaAssembleDims& d, const RowSrc& src, const float* alphas,
                         const ACT* hA, const float* W_base, const float* b_base, const float* gamma,
                         ACT* h_mid, const FactWorkspace& w) {
    Lanes lanes(st);
    int rc = lanes.rc;
    if (rc) return rc;
    const int kr = d.k * d.r;
    const int BT = d.B * d.T;
    const int64_t s1 = static_cast<int64_t>(d.d_B) * d.r, s2 = s1 + static_cast<int64_t>(d.r) * d.d_A;
    // aux0: hv = alpha (V h_A), one warp per (row, factor)
    const bool vec_hv = d.d_A % 8 == 0 && d.D % 8 == 0 && s1 % 8 == 0 && aligned16(src.rows) && aligned16(hA);
    const dim3 g_hv((kr + 7) / 8, d.B);
    if (d.T == 1)
        DWA_TIMED("factored_hv", lanes.aux[0],
                  launch_pdl(factored_hv_kernel<ACT, RT, 1>, g_hv, 256, 0, lanes.aux[0], src, alphas, hA, d.T,
                             d.d_A, s1, d.r, vec_hv, w.hv, w.status));
    else if (d.T <= 4)
        DWA_TIMED("factored_hv", lanes.aux[0],
                  launch_pdl(factored_hv_kernel<ACT, RT, 4>, g_hv, 256, 0, lanes.aux[0], src, alphas, hA, d.T,
                             d.d_A, s1, d.r, vec_hv, w.hv, w.status));
    else
        DWA_TIMED("factored_hv", lanes.aux[0],
                  launch_pdl(factored_hv_kernel<ACT, RT, kFactoredMaxT>, g_hv, 256, 0, lanes.aux[0], src, alphas,
                             hA, d.T, d.d_A, s1, d.r, vec_hv, w.hv, w.status));
    DWA_LAUNCH_CHECK("factored_hv_kernel");
    ++g_launches_total;
    // main: base = h_A W_base^T over all B*T rows at once (W_base read once)
    if (BT <= kBaseRowsMax) {
        const bool vec_b = d.d_A % 4 == 0 && aligned16(W_base) && aligned16(hA);
        const dim3 g_b((d.d_B + 3) / 4);
        if (BT <= 4)
            DWA_TIMED("base_rows", st,
                      launch_pdl(base_rows_kernel<ACT, 4>, g_b, 256, 0, st, W_base, hA, BT, d.d_A, d.d_B, vec_b,
                                 w.base));
        else if (BT <= 8)
            DWA_TIMED("base_rows", st,
                      launch_pdl(base_rows_kernel<ACT, 8>, g_b, 256, 0, st, W_base, hA, BT, d.d_A, d.d_B, vec_b,
                                 w.base));
        else
            DWA_TIMED("base_rows", st,
                      launch_pdl(base_rows_kernel<ACT, kBaseRowsMax>, g_b, 256, 0, st, W_base, hA, BT, d.d_A,
                                 d.d_B, vec_b, w.base));
        DWA_LAUNCH_CHECK("base_rows_kernel");
        ++g_launches_total;
    } else if (!std::is_same<ACT, __nv_bfloat16>::value) {
        // float activations, more than 16 rows: the CUDA-core GEMM, fp32 throughout
        EpiStore es_;
        es_.out = w.base; es_.N = d.d_B; es_.vec = d.d_B % 8 == 0;
        rc = gemm<ACT, false, false>("gemm_base", hA, d.d_A, static_cast<int64_t>(BT) * d.d_A, W_base, d.d_A,
                                     static_cast<int64_t>(d.d_B) * d.d_A, BT, d.d_B, d.d_A, 1, es_, w.status, st);
        if (rc) return rc;
        ++g_launches_total;
    } else {
        const int64_t n = static_cast<int64_t>(d.d_B) * d.d_A;
        const int grid = static_cast<int>(std::min<int64_t>((n / 8 + 255) / 256 + 1, 148 * 8));
        DWA_TIMED("cast_w_base", st,
                  launch_pdl(cast_bf16_kernel, dim3(grid), 256, 0, st, W_base, n, aligned16(W_base),
                             static_cast<__nv_bfloat16*>(w.Wb)));
        DWA_LAUNCH_CHECK("cast_bf16_kernel");
        ++g_launches_total;
        const size_t es = sizeof(ACT);
        const int Mp = static_cast<int>(align_up(static_cast<size_t>(BT), 128));
        DWA_CUDA_TRY(cudaMemcpyAsync(w.hpad, hA, static_cast<size_t>(BT) * d.d_A * es, cudaMemcpyDeviceToDevice, st));
        if (Mp > BT)
            DWA_CUDA_TRY(cudaMemsetAsync(static_cast<char*>(w.hpad) + static_cast<size_t>(BT) * d.d_A * es, 0,
                                         static_cast<size_t>(Mp - BT) * d.d_A * es, st));
        EpiStore es_;
        es_.out = w.base; es_.N = d.d_B; es_.vec = d.d_B % 8 == 0;
        // A = h_A padded (M=Mp, K=d_A, K-major); B = W_base (N=d_B, K=d_A, K-major)
        rc = gemm<ACT, false, false>("gemm_base", w.hpad, d.d_A, static_cast<int64_t>(Mp) * d.d_A, w.Wb, d.d_A,
                                     static_cast<int64_t>(d.d_B) * d.d_A, Mp, d.d_B, d.d_A, 1, es_, w.status, st);
        if (rc) return rc;
        ++g_launches_total;
    }
    if ((rc = lanes.join())) return rc;
    const size_t smem = factored_smem(d);
    const bool vec_u = d.r == 8 && d.D % 8 == 0 && aligned16(src.rows);
    const dim3 g_out((d.d_B + 127) / 128, d.B, w.nsplit);
#define DWA_FACT_OUT(TM)                                                                                       \
    do {                                                                                                       \
        if (smem > 48 * 1024)                                                                                  \
            DWA_CUDA_TRY(cudaFuncSetAttribute(factored_out_kernel<ACT, RT, TM>,                                \
                                              cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem))); \
        DWA_TIMED("factored_out", st,                                                                          \
                  launch_pdl(factored_out_kernel<ACT, RT, TM>, g_out, 128, smem, st, src, alphas, hA,           \
                             static_cast<const float*>(w.base), static_cast<const float*>(w.hv), b_base, gamma, \
                             d.T, d.d_B, d.r, s2, vec_u, w.kchunk, w.part, w.pbias, h_mid));                   \
    } while (0)
    if (d.T == 1)
        DWA_FACT_OUT(1);
    else if (d.T <= 4)
        DWA_FACT_OUT(4);
    else
        DWA_FACT_OUT(kFactoredMaxT);
#undef DWA_FACT_OUT
    DWA_LAUNCH_CHECK("factored_out_kernel");
    ++g_launches_total;
    if (w.nsplit > 1) {
        const int64_t n = static_cast<int64_t>(BT) * d.d_B;
        DWA_TIMED("factored_combine", st,
                  launch_pdl(factored_combine_kernel<ACT>, dim3(static_cast<unsigned>((n + 255) / 256)), 256, 0, st,
                             static_cast<const float*>(w.part), static_cast<const float*>(w.pbias), w.nsplit, hA,
                             static_cast<const float*>(w.base), b_base, gamma, d.B, d.T, d.d_B, h_mid));
        DWA_LAUNCH_CHECK("factored_combine_kernel");
        ++g_launches_total;
    }
    return DWA_OK;
}

}  // namespace dwa

extern "C" size_t dwa_assemble_apply_workspace_bytes(const DwaAssembleDims* dims) {
    if (check_dims(dims)) return 0;
    return factored_ok(*dims) ? carve_factored(nullptr, *dims).bytes : carve(nullptr, *dims, false).bytes;
}

extern "C" int dwa_assemble_apply(void* stream, const DwaAssembleDims* dims, const void* rows,
                                  const int32_t* row_index, const float* alphas, const void* h_A,
                                  const float* W_base, const float* b_base, const float* gamma, void* h_mid,
                                  void* workspace, size_t workspace_bytes) {
    int rc = check_dims(dims);
    if (rc) return rc;
    const DwaAssembleDims& d = *dims;
    if (!factored_ok(d))   // long sequences: assembling W first is the cheaper order
        return dwa_assemble_fwd(stream, dims, rows, row_index, alphas, h_A, W_base, b_base, gamma, h_mid,
                                nullptr, nullptr, workspace, workspace_bytes);
    if (!rows || !alphas || !h_A || !W_base || !b_base || !gamma || !h_mid)
        return fail(DWA_ERR_INVALID_ARG, "a required pointer is NULL");
    const FactWorkspace w = carve_factored(workspace, d);
    if ((rc = check_ws(workspace, workspace_bytes, w.bytes))) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const RowSrc src{rows, row_index, row_index ? d.n_rows : static_cast<int64_t>(d.B) * d.k, d.D,
                     d.k, d.rows_dtype};
#define DWA_APPLY_ARGS(A)                                                                            \
    st, d, src, alphas, static_cast<const A*>(h_A), W_base, b_base, gamma, static_cast<A*>(h_mid), w
    if (d.act_dtype == DWA_BF16) {
        if (d.rows_dtype == DWA_BF16)
            return factored_impl<__nv_bfloat16, __nv_bfloat16>(DWA_APPLY_ARGS(__nv_bfloat16));
        return factored_impl<__nv_bfloat16, float>(DWA_APPLY_ARGS(__nv_bfloat16));
    }
    if (d.rows_dtype == DWA_BF16)
        return factored_impl<float, __nv_bfloat16>(DWA_APPLY_ARGS(float));
    return factored_impl<float, float>(DWA_APPLY_ARGS(float));
#undef DWA_APPLY_ARGS
}
