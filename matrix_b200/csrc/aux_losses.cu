// Auxiliary losses (src/dwa/losses.py:9-73) and their gradients, without
// dense passes where the algebra allows:
//   l_util   = N Σ_n f_n P_n = N / (B² k) Σ_(b',j) Σ_b soft[b, idx[b',j]]
//              (only the selected columns of soft_full are read);
//              g_soft[b, n] = λ_util N cnt_n / (B² k) (non-zero on selected columns)
//   l_div    = Σ_b Σ_{i<j} r̂_i·r̂_j / (B k(k-1)/2 + 1e-8), r = aspect mean of the
//              retrieved keys, r̂ = r / (|r| + 1e-8), summed pair by pair;
//              g_r̂_i = c (U - r̂_i) with U = Σ_i r̂_i, so no k x k matrix is
//              stored; the key
//              gradient goes to every aspect's row idx[b,i] (deterministic
//              sorted scatter, duplicates added in order)
//   l_norm   = mean_b |W_b - W_base|²_F; g_W = 2 λ_norm (W - W_base) / B,
//              g_W_base = -Σ_b g_W (one pass over W)
//   l_sparse = -mean_b Σ_i a log a, a = clip(α, 1e-8, 1); g_α = -λ_sparse
//              (log a + 1) / B times jnp.clip's gradient (1 inside, 1/2 on a
//              bound, 0 outside)
// Reductions run in a fixed order (per-query and per-CTA partials added in
// index order).

#include <atomic>

#include "dwa_common.cuh"

namespace dwa {

extern std::atomic<uint64_t> g_launches_total;

constexpr int kAuxThreads = 256;
constexpr int kNormChunk = 4096;     // elements of [d_B * d_A] per CTA of the l_norm pass

__device__ __forceinline__ float aux_block_sum(float v, float* red) {
    v = warp_sum(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    float t = 0.f;
    if (threadIdx.x < 32) {
        t = threadIdx.x < static_cast<int>(blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
        t = warp_sum(t);
        if (threadIdx.x == 0) red[32] = t;
    }
    __syncthreads();
    return red[32];
}

struct AuxQueryArgs {
    int B, k, S, d_k;
    int64_t N;
    float lam_div, lam_sparse;
    const float* alphas;       // [B, k]
    const int32_t* indices;    // [B, k]
    const float* keys;         // [S, N, d_k]
    const float* soft;         // [B, N]
    float* part;               // [B, 3]: util, div, sparse
    float* g_alphas;           // [B, k] or null
    float* g_rk;               // [B, k, d_k] (already / S) or null
    uint32_t* status;
    const float* rk_in;        // [B, k, d_k] aspect-mean keys given (a sharded pool's finish) or null
};

// One CTA per query: l_sparse and its gradient, the query's l_util share and
// l_div with the gradient of its aspect-mean keys.
__global__ void __launch_bounds__(kAuxThreads) aux_query_kernel(AuxQueryArgs a) {
    pdl_enter();
    __shared__ float red[33];
    extern __shared__ __align__(16) float aux_sm[];
    const int b = blockIdx.x, tid = threadIdx.x, k = a.k, d_k = a.d_k, S = a.S;
    float* rk = aux_sm;                 // [k][d_k] aspect-mean keys
    float* U = rk + k * d_k;            // [d_k]
    float* inv = U + d_k;               // [k] 1 / (|r_i| + eps)
    float* nrm = inv + k;               // [k] |r_i|
    const float* al = a.alphas + static_cast<int64_t>(b) * k;
    const int32_t* ix = a.indices + static_cast<int64_t>(b) * k;
    // l_sparse
    float sp = 0.f;
    for (int i = tid; i < k; i += blockDim.x) {
        const float x = al[i];
        const float v = fminf(fmaxf(x, 1e-8f), 1.f);
        const float lg = logf(v);
        sp -= v * lg;
        if (a.g_alphas) {
            const float cg = (x > 1e-8f && x < 1.f) ? 1.f : (x == 1e-8f || x == 1.f) ? 0.5f : 0.f;
            a.g_alphas[static_cast<int64_t>(b) * k + i] = -a.lam_sparse * (lg + 1.f) / static_cast<float>(a.B) * cg;
        }
    }
    sp = aux_block_sum(sp, red);
    // l_util share: Σ_j Σ_b' soft[b', idx[b, j]] (none without soft_full: a sharded finish)
    float ut = 0.f;
    for (int i = tid; i < k && a.soft; i += blockDim.x) {
        const int64_t n = ix[i];
        if (n < 0 || n >= a.N) { raise_status(a.status, DWA_STATUS_BAD_ROW_INDEX); continue; }
        float c = 0.f;
        for (int bb = 0; bb < a.B; ++bb) c += a.soft[static_cast<int64_t>(bb) * a.N + n];
        ut += c;
    }
    ut = aux_block_sum(ut, red);
    // aspect-mean keys of the k retrieved rows
    for (int e = tid; e < k * d_k; e += blockDim.x) {
        if (a.rk_in) {
            rk[e] = a.rk_in[static_cast<int64_t>(b) * k * d_k + e];
            continue;
        }
        const int i = e / d_k, d = e - i * d_k;
        int64_t n = ix[i];
        n = n < 0 ? 0 : n >= a.N ? a.N - 1 : n;
        float acc = 0.f;
        for (int s = 0; s < S; ++s) acc += a.keys[(static_cast<int64_t>(s) * a.N + n) * d_k + d];
        rk[e] = acc / static_cast<float>(S);
    }
    __syncthreads();
    const int warp = tid >> 5, lane = tid & 31, nwarps = blockDim.x >> 5;
    for (int i = warp; i < k; i += nwarps) {
        float ss = 0.f;
        for (int d = lane; d < d_k; d += 32) ss = fmaf(rk[i * d_k + d], rk[i * d_k + d], ss);
        ss = warp_sum(ss);
        if (lane == 0) {
            nrm[i] = sqrtf(ss);
            inv[i] = 1.f / (sqrtf(ss) + 1e-8f);
        }
    }
    __syncthreads();
    // r̂ values rounded once (__fmul_rn, no contraction into an FMA), so that
    // U - r̂_i below is exact when only r̂_i makes up U
    for (int d = tid; d < d_k; d += blockDim.x) {
        float u = 0.f;
        for (int i = 0; i < k; ++i) u = __fadd_rn(u, __fmul_rn(rk[i * d_k + d], inv[i]));
        U[d] = u;
    }
    __syncthreads();
    // Σ_{i<j} r̂_i·r̂_j pair by pair (the identity with |U|² cancels badly)
    float pairs = 0.f;
    for (int e = tid; e < k * k; e += blockDim.x) {
        const int i = e / k, j = e - i * k;
        if (i >= j) continue;
        float dt = 0.f;
        for (int d = 0; d < d_k; ++d) dt = fmaf(rk[i * d_k + d], rk[j * d_k + d], dt);
        pairs = fmaf(dt, inv[i] * inv[j], pairs);
    }
    pairs = aux_block_sum(pairs, red);
    if (tid == 0) {
        float* p = a.part + static_cast<int64_t>(b) * 3;
        p[0] = ut;
        p[1] = pairs;
        p[2] = sp;
    }
    if (a.g_rk) {
        // g_r̂_i = c (U - r̂_i); g_r_i = g_r̂_i inv - r_i (r_i·g_r̂_i) inv² / |r_i|; / S per aspect
        const float c = a.lam_div / (static_cast<float>(static_cast<int64_t>(k) * (k - 1) / 2 * a.B) + 1e-8f);
        for (int i = warp; i < k; i += nwarps) {
            float dt = 0.f;
            for (int d = lane; d < d_k; d += 32) {
                const float g = c * __fsub_rn(U[d], __fmul_rn(rk[i * d_k + d], inv[i]));
                dt = fmaf(rk[i * d_k + d], g, dt);
            }
            dt = warp_sum(dt);
            const float coef = nrm[i] > 0.f ? dt * inv[i] * inv[i] / nrm[i] : 0.f;
            for (int d = lane; d < d_k; d += 32) {
                const float g = c * __fsub_rn(U[d], __fmul_rn(rk[i * d_k + d], inv[i]));
                a.g_rk[(static_cast<int64_t>(b) * k + i) * d_k + d] =
                    (g * inv[i] - rk[i * d_k + d] * coef) / static_cast<float>(S);
            }
        }
    }
}

// l_norm partial sums of (W - W_base)² per CTA over elements
// [blockIdx.x * kNormChunk, +kNormChunk) of every W_b, and the gradients.
__global__ void __launch_bounds__(kAuxThreads) aux_norm_kernel(const float* __restrict__ W,
                                                               const float* __restrict__ W_base, int B,
                                                               int64_t E, float gscale, float* __restrict__ g_W,
                                                               float* __restrict__ g_W_base,
                                                               float* __restrict__ part) {
    pdl_enter();
    __shared__ float red[33];
    const int64_t e0 = static_cast<int64_t>(blockIdx.x) * kNormChunk;
    float acc = 0.f;
    for (int64_t e = e0 + threadIdx.x; e < E && e < e0 + kNormChunk; e += blockDim.x) {
        const float wb = W_base[e];
        float gb = 0.f, sq = 0.f;
        for (int b = 0; b < B; ++b) {
            const float diff = W[static_cast<int64_t>(b) * E + e] - wb;
            sq = fmaf(diff, diff, sq);
            if (g_W) g_W[static_cast<int64_t>(b) * E + e] = gscale * diff;
            gb -= gscale * diff;
        }
        if (g_W_base) g_W_base[e] = gb;
        acc += sq;
    }
    acc = aux_block_sum(acc, red);
    if (threadIdx.x == 0) part[blockIdx.x] = acc;
}

// Selection counts of the pool rows, then g_soft[b, n] = scale * cnt[n] on the
// selected columns (the rest of g_soft is zeroed before).
__global__ void aux_count_kernel(const int32_t* __restrict__ idx, int n, int64_t row_lo, int64_t N,
                                 int* __restrict__ cnt) {
    pdl_enter();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int64_t r = static_cast<int64_t>(idx[i]) - row_lo;
    if (r >= 0 && r < N) atomicAdd(&cnt[r], 1);
}

__global__ void aux_soft_grad_kernel(const int32_t* __restrict__ idx, int n, int B, int64_t row_lo, int64_t N,
                                     const int* __restrict__ cnt, float scale, float* __restrict__ g_soft) {
    pdl_enter();
    const int i = blockIdx.x;
    if (i >= n) return;
    const int64_t c = static_cast<int64_t>(idx[i]) - row_lo;
    if (c < 0 || c >= N) return;
    const float v = scale * static_cast<float>(cnt[c]);
    for (int b = threadIdx.x; b < B; b += blockDim.x) g_soft[static_cast<int64_t>(b) * N + c] = v;
}

// losses = {l_util, l_div, l_norm, l_sparse, total} from the partials, in order.
__global__ void aux_finish_kernel(const float* __restrict__ qpart, int B, int k, int64_t N,
                                  const float* __restrict__ npart, int nn, float lu, float ld, float ln,
                                  float ls, float* __restrict__ losses) {
    pdl_enter();
    if (threadIdx.x != 0) return;
    float u = 0.f, dv = 0.f, sp = 0.f, nm = 0.f;
    for (int b = 0; b < B; ++b) {
        u += qpart[3 * b];
        dv += qpart[3 * b + 1];
        sp += qpart[3 * b + 2];
    }
    for (int i = 0; i < nn; ++i) nm += npart[i];
    const float fB = static_cast<float>(B);
    const float l_util = static_cast<float>(N) / (fB * fB * static_cast<float>(k)) * u;
    const float l_div = dv / (static_cast<float>(static_cast<int64_t>(k) * (k - 1) / 2) * fB + 1e-8f);
    const float l_norm = nm / fB;
    const float l_sparse = sp / fB;
    losses[0] = l_util;
    losses[1] = l_div;
    losses[2] = l_norm;
    losses[3] = l_sparse;
    losses[4] = lu * l_util + ld * l_div + ln * l_norm + ls * l_sparse;
}

// A rank of a row-sharded pool, per query: its share of l_util's sum (the
// selected columns it holds) and the aspect-mean keys of the winners it holds
// (zeros for the others), so that a sum over the ranks gives every winner's.
__global__ void __launch_bounds__(kAuxThreads) aux_local_kernel(const int32_t* __restrict__ indices, int k,
                                                               int B, int S, int d_k, int64_t row_lo,
                                                               int64_t n_loc, const float* __restrict__ keys,
                                                               const float* __restrict__ soft,
                                                               float* __restrict__ ushare,
                                                               float* __restrict__ rk_out) {
    pdl_enter();
    __shared__ float red[33];
    const int b = blockIdx.x, tid = threadIdx.x;
    const int32_t* ix = indices + static_cast<int64_t>(b) * k;
    float ut = 0.f;
    for (int i = tid; i < k && soft; i += blockDim.x) {
        const int64_t n = static_cast<int64_t>(ix[i]) - row_lo;
        if (n < 0 || n >= n_loc) continue;
        float c = 0.f;
        for (int bb = 0; bb < B; ++bb) c += soft[static_cast<int64_t>(bb) * n_loc + n];
        ut += c;
    }
    ut = aux_block_sum(ut, red);
    if (tid == 0) ushare[b] = ut;
    for (int e = tid; e < k * d_k; e += blockDim.x) {
        const int i = e / d_k, d = e - i * d_k;
        const int64_t n = static_cast<int64_t>(ix[i]) - row_lo;
        float acc = 0.f;
        if (n >= 0 && n < n_loc) {
            for (int s = 0; s < S; ++s) acc += keys[(static_cast<int64_t>(s) * n_loc + n) * d_k + d];
            acc /= static_cast<float>(S);
        }
        rk_out[static_cast<int64_t>(b) * k * d_k + e] = acc;
    }
}

// part[0] = Σ_b ushare[b], part[1] = Σ of the l_norm partials, in order.
__global__ void aux_local_sums_kernel(const float* __restrict__ ushare, int B, const float* __restrict__ npart,
                                      int nn, float* __restrict__ part) {
    pdl_enter();
    if (threadIdx.x != 0) return;
    float u = 0.f, nm = 0.f;
    for (int b = 0; b < B; ++b) u += ushare[b];
    for (int i = 0; i < nn; ++i) nm += npart[i];
    part[0] = u;
    part[1] = nm;
}

// The losses of a sharded call from the summed part (l_util's sum, l_norm's
// sum) and the per-query l_div / l_sparse terms of the finish.
__global__ void aux_finish_sharded_kernel(const float* __restrict__ part_sum, const float* __restrict__ qpart, int B,
                                          int k, int64_t N, float lu, float ld, float ln, float ls,
                                          float* __restrict__ losses) {
    pdl_enter();
    if (threadIdx.x != 0) return;
    float dv = 0.f, sp = 0.f;
    for (int b = 0; b < B; ++b) {
        dv += qpart[3 * b + 1];
        sp += qpart[3 * b + 2];
    }
    const float fB = static_cast<float>(B);
    const float l_util = static_cast<float>(N) / (fB * fB * static_cast<float>(k)) * part_sum[0];
    const float l_div = dv / (static_cast<float>(static_cast<int64_t>(k) * (k - 1) / 2) * fB + 1e-8f);
    const float l_norm = part_sum[1] / fB;
    const float l_sparse = sp / fB;
    losses[0] = l_util;
    losses[1] = l_div;
    losses[2] = l_norm;
    losses[3] = l_sparse;
    losses[4] = lu * l_util + ld * l_div + ln * l_norm + ls * l_sparse;
}

struct AuxWorkspace {
    float* qpart;
    float* npart;
    int* cnt;
    float* g_rk;
    void* scatter_ws;
    size_t scatter_bytes;
    int nn;
    size_t bytes;
};

static AuxWorkspace carve_aux(void* base, const DwaAuxDims& d) {
    Carver c(base);
    AuxWorkspace w{};
    const int64_t E = static_cast<int64_t>(d.d_B) * d.d_A;
    w.nn = static_cast<int>((E + kNormChunk - 1) / kNormChunk);
    w.qpart = c.take<float>(static_cast<size_t>(d.B) * 3);
    w.npart = c.take<float>(static_cast<size_t>(w.nn));
    w.cnt = c.take<int>(static_cast<size_t>(d.N));
    w.g_rk = c.take<float>(static_cast<size_t>(d.B) * d.k * d.d_k);
    w.scatter_bytes = dwa_pool_grad_scatter_workspace_bytes(d.B * d.k);
    w.scatter_ws = c.take<char>(w.scatter_bytes);
    w.bytes = c.bytes();
    return w;
}

static int check_aux(const DwaAuxDims* d) {
    if (!d) return fail(DWA_ERR_INVALID_ARG, "dims is NULL");
    if (d->B <= 0 || d->k <= 0 || d->S <= 0 || d->d_k <= 0 || d->d_B <= 0 || d->d_A <= 0 || d->N <= 0)
        return fail(DWA_ERR_INVALID_ARG, "B, k, S, d_k, d_B, d_A, N must be positive");
    if (d->N >= (int64_t(1) << 31)) return fail(DWA_ERR_UNSUPPORTED, "N >= 2^31");
    if (static_cast<int64_t>(d->B) * d->k > 8192) return fail(DWA_ERR_UNSUPPORTED, "B * k > 8192");
    if ((static_cast<size_t>(d->k) * d->d_k + d->d_k + 2 * d->k) * sizeof(float) > 200 * 1024)
        return fail(DWA_ERR_UNSUPPORTED, "k * d_k too large for shared memory");
    return DWA_OK;
}

}  // namespace dwa

using namespace dwa;

extern "C" size_t dwa_aux_losses_workspace_bytes(const DwaAuxDims* dims) {
    if (check_aux(dims)) return 0;
    return carve_aux(nullptr, *dims).bytes;
}

extern "C" int dwa_aux_losses(void* stream, const DwaAuxDims* dims, const DwaAuxWeights* lambdas,
                              const float* alphas, const int32_t* indices, const float* pool_keys,
                              const float* W, const float* W_base, const float* soft_full, float* losses,
                              float* g_alphas, float* g_soft_full, float* g_W, float* g_W_base,
                              float* g_pool_keys, void* workspace, size_t workspace_bytes) {
    int rc = check_aux(dims);
    if (rc) return rc;
    if (!lambdas || !alphas || !indices || !pool_keys || !W || !W_base || !soft_full || !losses)
        return fail(DWA_ERR_INVALID_ARG, "a required pointer is NULL");
    const DwaAuxDims& d = *dims;
    const AuxWorkspace w = carve_aux(workspace, d);
    if (!workspace || reinterpret_cast<uintptr_t>(workspace) % 256 != 0)
        return fail(DWA_ERR_WORKSPACE, "workspace must be non-NULL and 256-byte aligned");
    if (workspace_bytes < w.bytes) return fail(DWA_ERR_WORKSPACE, "workspace too small");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    uint32_t* status = static_cast<uint32_t*>(workspace);
    // per-query terms
    AuxQueryArgs qa{};
    qa.B = d.B; qa.k = d.k; qa.S = d.S; qa.d_k = d.d_k; qa.N = d.N;
    qa.lam_div = lambdas->div; qa.lam_sparse = lambdas->sparse;
    qa.alphas = alphas; qa.indices = indices; qa.keys = pool_keys; qa.soft = soft_full;
    qa.part = w.qpart; qa.g_alphas = g_alphas; qa.g_rk = g_pool_keys ? w.g_rk : nullptr; qa.status = status;
    const size_t qsh = (static_cast<size_t>(d.k) * d.d_k + d.d_k + 2 * d.k) * sizeof(float);
    {
        int dv = 0;
        DWA_CUDA_TRY(cudaGetDevice(&dv));
        static bool attr[64] = {};
        if (dv < 0 || dv >= 64 || !attr[dv]) {
            DWA_CUDA_TRY(cudaFuncSetAttribute(aux_query_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
            if (dv >= 0 && dv < 64) attr[dv] = true;
        }
    }
    DWA_TIMED("aux_query", st, launch_pdl(aux_query_kernel, d.B, kAuxThreads, qsh, st, qa));
    DWA_LAUNCH_CHECK("aux_query_kernel");
    // l_norm and the W gradients
    const int64_t E = static_cast<int64_t>(d.d_B) * d.d_A;
    DWA_TIMED("aux_norm", st, launch_pdl(aux_norm_kernel, w.nn, kAuxThreads, 0, st, W, W_base, d.B, E,
                                         2.f * lambdas->norm / static_cast<float>(d.B), g_W, g_W_base, w.npart));
    DWA_LAUNCH_CHECK("aux_norm_kernel");
    g_launches_total += 2;
    // l_util's gradient on soft_full
    const int n = d.B * d.k;
    if (g_soft_full) {
        DWA_CUDA_TRY(cudaMemsetAsync(g_soft_full, 0, static_cast<size_t>(d.B) * d.N * sizeof(float), st));
        DWA_CUDA_TRY(cudaMemsetAsync(w.cnt, 0, static_cast<size_t>(d.N) * sizeof(int), st));
        launch_pdl(aux_count_kernel, (n + 255) / 256, 256, 0, st, indices, n, int64_t(0), d.N, w.cnt);
        DWA_LAUNCH_CHECK("aux_count_kernel");
        const float fB = static_cast<float>(d.B);
        launch_pdl(aux_soft_grad_kernel, n, 32, 0, st, indices, n, d.B, int64_t(0), d.N, w.cnt,
                   lambdas->util * static_cast<float>(d.N) / (fB * fB * static_cast<float>(d.k)), g_soft_full);
        DWA_LAUNCH_CHECK("aux_soft_grad_kernel");
        g_launches_total += 2;
    }
    launch_pdl(aux_finish_kernel, 1, 32, 0, st, w.qpart, d.B, d.k, d.N, w.npart, w.nn, lambdas->util, lambdas->div,
               lambdas->norm, lambdas->sparse, losses);
    DWA_LAUNCH_CHECK("aux_finish_kernel");
    ++g_launches_total;
    // l_div's key gradient into every aspect's rows
    if (g_pool_keys) {
        for (int s = 0; s < d.S; ++s) {
            rc = dwa_pool_grad_scatter(stream, n, d.d_k, indices, w.g_rk, d.N, 0, d.N, DWA_F32,
                                       g_pool_keys + static_cast<int64_t>(s) * d.N * d.d_k, w.scatter_ws,
                                       w.scatter_bytes);
            if (rc) return rc;
        }
    }
    return DWA_OK;
}

extern "C" int dwa_aux_losses_local(void* stream, const DwaAuxDims* dims, const DwaAuxShard* shard,
                                    const DwaAuxWeights* lambdas, const int32_t* indices, const float* local_keys,
                                    const float* W, const float* W_base, const float* soft_full, float* part,
                                    float* rk_part, float* g_soft_full, float* g_W, float* g_W_base_part,
                                    void* workspace, size_t workspace_bytes) {
    int rc = check_aux(dims);
    if (rc) return rc;
    const DwaAuxDims& d = *dims;
    if (!shard || shard->row_lo < 0 || shard->n_global < shard->row_lo + d.N || shard->w_batch < 0 ||
        shard->w_batch > d.B)
        return fail(DWA_ERR_INVALID_ARG, "shard: need row_lo + N <= n_global and 0 <= w_batch <= B");
    if (!lambdas || !indices || !local_keys || !W_base || !soft_full || !part || !rk_part || (shard->w_batch && !W))
        return fail(DWA_ERR_INVALID_ARG, "a required pointer is NULL");
    const AuxWorkspace w = carve_aux(workspace, d);
    if (!workspace || reinterpret_cast<uintptr_t>(workspace) % 256 != 0 || workspace_bytes < w.bytes)
        return fail(DWA_ERR_WORKSPACE, "workspace: dwa_aux_losses_workspace_bytes, 256-byte aligned");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    launch_pdl(aux_local_kernel, d.B, kAuxThreads, 0, st, indices, d.k, d.B, d.S, d.d_k, shard->row_lo, d.N,
               local_keys, soft_full, w.qpart, rk_part);
    DWA_LAUNCH_CHECK("aux_local_kernel");
    const int64_t E = static_cast<int64_t>(d.d_B) * d.d_A;
    if (shard->w_batch > 0) {
        launch_pdl(aux_norm_kernel, w.nn, kAuxThreads, 0, st, W, W_base, static_cast<int>(shard->w_batch), E,
                   2.f * lambdas->norm / static_cast<float>(d.B), g_W, g_W_base_part, w.npart);
        DWA_LAUNCH_CHECK("aux_norm_kernel");
    } else {
        DWA_CUDA_TRY(cudaMemsetAsync(w.npart, 0, static_cast<size_t>(w.nn) * sizeof(float), st));
        if (g_W_base_part) DWA_CUDA_TRY(cudaMemsetAsync(g_W_base_part, 0, static_cast<size_t>(E) * sizeof(float), st));
    }
    launch_pdl(aux_local_sums_kernel, 1, 32, 0, st, w.qpart, d.B, w.npart, w.nn, part);
    DWA_LAUNCH_CHECK("aux_local_sums_kernel");
    g_launches_total += 3;
    const int n = d.B * d.k;
    if (g_soft_full) {
        DWA_CUDA_TRY(cudaMemsetAsync(g_soft_full, 0, static_cast<size_t>(d.B) * d.N * sizeof(float), st));
        DWA_CUDA_TRY(cudaMemsetAsync(w.cnt, 0, static_cast<size_t>(d.N) * sizeof(int), st));
        launch_pdl(aux_count_kernel, (n + 255) / 256, 256, 0, st, indices, n, shard->row_lo, d.N, w.cnt);
        DWA_LAUNCH_CHECK("aux_count_kernel");
        const float fB = static_cast<float>(d.B);
        launch_pdl(aux_soft_grad_kernel, n, 32, 0, st, indices, n, d.B, shard->row_lo, d.N, w.cnt,
                   lambdas->util * static_cast<float>(shard->n_global) / (fB * fB * static_cast<float>(d.k)),
                   g_soft_full);
        DWA_LAUNCH_CHECK("aux_soft_grad_kernel");
        g_launches_total += 2;
    }
    return DWA_OK;
}

extern "C" int dwa_aux_losses_finish(void* stream, const DwaAuxDims* dims, const DwaAuxShard* shard,
                                     const DwaAuxWeights* lambdas, const float* alphas, const int32_t* indices,
                                     const float* part_sum, const float* rk_sum, float* losses, float* g_alphas,
                                     float* g_pool_keys, void* workspace, size_t workspace_bytes) {
    int rc = check_aux(dims);
    if (rc) return rc;
    const DwaAuxDims& d = *dims;
    if (!shard || shard->row_lo < 0 || shard->n_global < shard->row_lo + d.N)
        return fail(DWA_ERR_INVALID_ARG, "shard: need row_lo + N <= n_global");
    if (!lambdas || !alphas || !indices || !part_sum || !rk_sum || !losses)
        return fail(DWA_ERR_INVALID_ARG, "a required pointer is NULL");
    const AuxWorkspace w = carve_aux(workspace, d);
    if (!workspace || reinterpret_cast<uintptr_t>(workspace) % 256 != 0 || workspace_bytes < w.bytes)
        return fail(DWA_ERR_WORKSPACE, "workspace: dwa_aux_losses_workspace_bytes, 256-byte aligned");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    AuxQueryArgs qa{};
    qa.B = d.B; qa.k = d.k; qa.S = d.S; qa.d_k = d.d_k; qa.N = d.N;
    qa.lam_div = lambdas->div; qa.lam_sparse = lambdas->sparse;
    qa.alphas = alphas; qa.indices = indices; qa.keys = nullptr; qa.soft = nullptr; qa.rk_in = rk_sum;
    qa.part = w.qpart; qa.g_alphas = g_alphas; qa.g_rk = g_pool_keys ? w.g_rk : nullptr;
    qa.status = static_cast<uint32_t*>(workspace);
    const size_t qsh = (static_cast<size_t>(d.k) * d.d_k + d.d_k + 2 * d.k) * sizeof(float);
    DWA_CUDA_TRY(cudaFuncSetAttribute(aux_query_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    launch_pdl(aux_query_kernel, d.B, kAuxThreads, qsh, st, qa);
    DWA_LAUNCH_CHECK("aux_query_kernel");
    launch_pdl(aux_finish_sharded_kernel, 1, 32, 0, st, part_sum, w.qpart, d.B, d.k, shard->n_global, lambdas->util,
               lambdas->div, lambdas->norm, lambdas->sparse, losses);
    DWA_LAUNCH_CHECK("aux_finish_sharded_kernel");
    g_launches_total += 2;
    if (g_pool_keys) {
        const int n = d.B * d.k;
        for (int s = 0; s < d.S; ++s) {
            rc = dwa_pool_grad_scatter(stream, n, d.d_k, indices, w.g_rk, shard->n_global, shard->row_lo,
                                       shard->row_lo + d.N, DWA_F32, g_pool_keys + static_cast<int64_t>(s) * d.N * d.d_k,
                                       w.scatter_ws, w.scatter_bytes);
            if (rc) return rc;
        }
    }
    return DWA_OK;
}
