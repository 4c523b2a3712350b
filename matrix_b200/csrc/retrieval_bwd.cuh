// Retrieval VJP: the backward of MultiAspectRetrieval.__call__
// (src/dwa/retrieval.py:64-158) as jax.vjp gives it, from the cotangents of
// alphas [B,k] and soft_full [B,N] to z, W_Q, aspect_weights, tau and
// (optionally) the key cache.  Included by retrieval.cu (one translation unit
// with the forward, whose query, coarse top-m and scoring kernels it reuses).
//
//   recompute   q = W_Q z, the probed lists and, in gate mode, every
//               candidate's score s (the forward's kernels)
//   G [B,N]     dL/ds per (query, pool row):
//                 soft_full: soft (g_soft - Σ_n g_soft soft) / T on every row
//                 warmup:    α (g_α - Σ α g_α) / T on the winners' rows
//                 gate:      g_raw raw (λ(1-σ) + 1/T) on every candidate row,
//                            g_raw = g_rn/(Z+ε) - Σ g_rn raw/(Z+ε)², g_rn the
//                            top-k backward of α = top/(Σ top + ε)
//   key pass    A[b,s,:] = Σ_n G[b,n] k̂[s,n] over the rows where G may be
//               non-zero (every row, or the probed lists only); optionally
//               g_keys = normalize-VJP(w_s Σ_b G[b,n] q̂[b,s])
//   queries     g_q̂ = w_s A, g_w[s] = Σ_b q̂·A, g_q = normalize-VJP(g_q̂),
//               g_W_Q = Σ_b g_q ⊗ z, g_z = W_Qᵀ g_q, g_aw = softmax-VJP(g_w),
//               g_τ = -Σ g_raw raw λ(1-σ)
// Every reduction runs in a fixed order: bit-identical repeats.
#pragma once

namespace dwa {

constexpr int kKeyTile = 32;          // key rows per tile of the key pass
constexpr int kKeyThreads = 256;
constexpr int kBwdMaxQ = 32;          // queries per key pass (larger B: several passes)

struct KeyGradArgs {
    const float* keys;      // [S, N, d_k]
    int64_t N;
    int S, d_k, B;          // B: queries of the whole call
    int b0, nb;             // this pass: queries [b0, b0 + nb)
    const float* G;         // [B, N]
    const float* qh;        // [B, S, d_k] normalised queries (unweighted)
    const float* w;         // [S] softmax(aspect_weights)
    const uint8_t* tile_on; // [ntiles] or null (every tile)
    int64_t ntiles;
    float* partial;         // [gridDim.x, nb, S*d_k]
    float* g_keys;          // [S, N, d_k] or null
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(tc::smem_u32(dst)), "l"(src) : "memory");
}
// 4 bytes, or zeros when n == 0 (nothing is read then)
__device__ __forceinline__ void cp_async4(void* dst, const void* src, int n) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(tc::smem_u32(dst)), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// One persistent CTA walks the active key tiles t = blockIdx.x, +gridDim.x,
// ... with two shared-memory buffers: the next tile's keys (S x 32 rows) and G
// values ([row][QB], zero for queries past nb) stream in by cp.async while the
// current tile is reduced.  Per tile: the row norms (one thread per (row,
// aspect)), then A += G k̂ per (query, column) in registers: thread t owns
// columns t, t + 256, ..., reads G four queries at a time (broadcast float4)
// and issues QB FMAs per column and row.  With g_keys, also writes the key
// gradient of its rows.  Partial sums per CTA; added in CTA order afterwards.
// Needs d_k % 4 == 0 and d_k dividing 1024.
template <int CPT, int QB, bool FUSED = false>
__global__ void __launch_bounds__(kKeyThreads) key_grad_pass_kernel(KeyGradArgs a) {
    pdl_enter();
    extern __shared__ __align__(16) float kg_sm[];
    const int S = a.S, d_k = a.d_k, cols = S * d_k;
    float* ktb = kg_sm;                               // [2][kKeyTile][cols]
    float* gtb = ktb + 2 * kKeyTile * cols;           // [2][kKeyTile][QB]
    float* gk = gtb + 2 * QB * kKeyTile;              // [kKeyTile][cols] (g_keys only)
    float* nrm = gk + (a.g_keys ? kKeyTile * cols : 0);// [kKeyTile][S]
    float* inv = nrm + kKeyTile * S;                  // [kKeyTile][S]
    float* dotk = inv + kKeyTile * S;                 // [kKeyTile][S] (g_keys: the normalisation VJP's coefficient)
    const int tid = threadIdx.x;
    // Key gradient folded into the row loop (FUSED, launched with g_keys): a
    // thread keeps its columns' weighted queries in registers and forms g_k̂
    // from the G values the row loop already holds, into shared memory; then
    // one thread per (row, aspect) takes the normalisation VJP's dot k·g_k̂
    // and its coefficient, and the tile's gradient rows are written.
    float qsr[CPT][FUSED ? QB : 1];
    if constexpr (FUSED) {
#pragma unroll
        for (int c = 0; c < CPT; ++c) {
            const int col = tid + c * kKeyThreads;
#pragma unroll
            for (int b = 0; b < QB; ++b)
                qsr[c][b] = (col < cols && b < a.nb)
                                ? a.qh[static_cast<int64_t>(a.b0 + b) * cols + col] * a.w[col / d_k] : 0.f;
        }
    }
    // this thread's part of a tile load: float4 c4 of rows r0, r0 + rstep, ...
    const int q4 = d_k / 4;
    const int c4 = tid % q4, r0 = tid / q4, rstep = kKeyThreads / q4;
    int col_s[CPT];
#pragma unroll
    for (int c = 0; c < CPT; ++c) col_s[c] = (tid + c * kKeyThreads) / d_k;
    auto next_active = [&](int64_t t) {
        while (t < a.ntiles && a.tile_on && !a.tile_on[t]) t += gridDim.x;
        return t;
    };
    auto issue = [&](int64_t t, int buf) {
        const int64_t row0 = t * kKeyTile;
        const int rows = static_cast<int>(a.N - row0 < kKeyTile ? a.N - row0 : kKeyTile);
        float* kt = ktb + buf * kKeyTile * cols;
        for (int s = 0; s < S; ++s) {
            const float4* src = reinterpret_cast<const float4*>(a.keys + (static_cast<int64_t>(s) * a.N + row0) * d_k);
            for (int r = r0; r < rows; r += rstep) cp_async16(kt + r * cols + s * d_k + 4 * c4, src + r * q4 + c4);
        }
        float* gt = gtb + buf * QB * kKeyTile;
        for (int i = tid; i < QB * kKeyTile; i += blockDim.x) {
            const int b = i / kKeyTile, r = i - b * kKeyTile;
            const bool in = r < rows && b < a.nb;
            cp_async4(gt + r * QB + b, in ? a.G + static_cast<int64_t>(a.b0 + b) * a.N + row0 + r : a.G, in ? 4 : 0);
        }
    };
    float acc[CPT][QB];
#pragma unroll
    for (int c = 0; c < CPT; ++c)
#pragma unroll
        for (int b = 0; b < QB; ++b) acc[c][b] = 0.f;
    int64_t t = next_active(blockIdx.x);
    if (t < a.ntiles) issue(t, 0);
    cp_async_commit();
    int cur = 0;
    while (t < a.ntiles) {
        const int64_t tn = next_active(t + gridDim.x);
        if (tn < a.ntiles) issue(tn, cur ^ 1);
        cp_async_commit();
        cp_async_wait1();          // this thread's copies of tile t are done
        __syncthreads();           // everyone's are
        const int64_t row0 = t * kKeyTile;
        const int rows = static_cast<int>(a.N - row0 < kKeyTile ? a.N - row0 : kKeyTile);
        const float* kt = ktb + cur * kKeyTile * cols;
        const float* gt = gtb + cur * QB * kKeyTile;
        // norms: one thread per (row, aspect); each starts at a different float4
        // of the row so that the threads of a warp spread over the banks
        for (int p = tid; p < rows * S; p += blockDim.x) {
            const int r = p / S, s = p - r * S;
            const float4* kr = reinterpret_cast<const float4*>(kt + r * cols + s * d_k);
            float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
            for (int i = 0; i < q4; ++i) {
                const float4 v = kr[(i + p) % q4];
                s0 = fmaf(v.x, v.x, s0);
                s1 = fmaf(v.y, v.y, s1);
                s2 = fmaf(v.z, v.z, s2);
                s3 = fmaf(v.w, v.w, s3);
            }
            const float n = sqrtf((s0 + s1) + (s2 + s3));
            nrm[r * S + s] = n;
            inv[r * S + s] = 1.f / (n + 1e-8f);
        }
        __syncthreads();
#pragma unroll 4
        for (int r = 0; r < rows; ++r) {
            const float4* gr = reinterpret_cast<const float4*>(gt + r * QB);
#pragma unroll
            for (int c = 0; c < CPT; ++c) {
                const int col = tid + c * kKeyThreads;
                if (CPT == 1 || col < cols) {
                    const float kr = kt[r * cols + col];
                    const float kh = kr * inv[r * S + col_s[c]];
                    float gkv = 0.f;
#pragma unroll
                    for (int q = 0; q < QB / 4; ++q) {
                        const float4 g = gr[q];
                        acc[c][4 * q] = fmaf(g.x, kh, acc[c][4 * q]);
                        acc[c][4 * q + 1] = fmaf(g.y, kh, acc[c][4 * q + 1]);
                        acc[c][4 * q + 2] = fmaf(g.z, kh, acc[c][4 * q + 2]);
                        acc[c][4 * q + 3] = fmaf(g.w, kh, acc[c][4 * q + 3]);
                        if constexpr (FUSED) {
                            gkv = fmaf(g.x, qsr[c][4 * q], gkv);
                            gkv = fmaf(g.y, qsr[c][4 * q + 1], gkv);
                            gkv = fmaf(g.z, qsr[c][4 * q + 2], gkv);
                            gkv = fmaf(g.w, qsr[c][4 * q + 3], gkv);
                        }
                    }
                    if constexpr (FUSED) gk[r * cols + col] = gkv;
                }
            }
        }
        if constexpr (FUSED) {
            __syncthreads();   // the tile's g_k̂
            // coefficient of the normalisation VJP per (row, aspect):
            // (k·g_k̂) / (|k| (|k| + eps)^2); four partial chains over float4s,
            // each thread starting at a different float4 (spread over the banks)
            for (int p = tid; p < rows * S; p += blockDim.x) {
                const int r = p / S, s = p - r * S;
                const float4* kr4 = reinterpret_cast<const float4*>(kt + r * cols + s * d_k);
                const float4* gr4 = reinterpret_cast<const float4*>(gk + r * cols + s * d_k);
                float t0 = 0.f, t1 = 0.f, t2 = 0.f, t3 = 0.f;
                for (int i = 0; i < q4; ++i) {
                    const int j = (i + p) % q4;
                    const float4 u = kr4[j], v = gr4[j];
                    t0 = fmaf(u.x, v.x, t0);
                    t1 = fmaf(u.y, v.y, t1);
                    t2 = fmaf(u.z, v.z, t2);
                    t3 = fmaf(u.w, v.w, t3);
                }
                const float dt = (t0 + t1) + (t2 + t3), iv = inv[p], n = nrm[p];
                dotk[p] = n > 0.f ? dt * iv * iv / n : 0.f;
            }
            __syncthreads();
#pragma unroll
            for (int c = 0; c < CPT; ++c) {
                const int col = tid + c * kKeyThreads;
                if (CPT > 1 && col >= cols) continue;
                const int s = col_s[c], d = col - s * d_k;
                float* dst = a.g_keys + (static_cast<int64_t>(s) * a.N + row0) * d_k + d;
#pragma unroll 4
                for (int r = 0; r < rows; ++r)
                    dst[static_cast<int64_t>(r) * d_k] =
                        gk[r * cols + col] * inv[r * S + s] - kt[r * cols + col] * dotk[r * S + s];
            }
        }
        __syncthreads();           // buffer cur is free for the tile after next
        t = tn;
        cur ^= 1;
    }
    float* out = a.partial + static_cast<int64_t>(blockIdx.x) * a.nb * cols;
#pragma unroll
    for (int c = 0; c < CPT; ++c) {
        const int col = tid + c * kKeyThreads;
        if (col < cols)
#pragma unroll
            for (int b = 0; b < QB; ++b)
                if (b < a.nb) out[static_cast<int64_t>(b) * cols + col] = acc[c][b];
    }
}

__host__ inline size_t key_grad_smem(int S, int d_k, int QB, bool g_keys) {
    const size_t cols = static_cast<size_t>(S) * d_k;
    return (kKeyTile * cols * (g_keys ? 3 : 2) + 2 * static_cast<size_t>(QB) * kKeyTile + 3 * kKeyTile * S) *
           sizeof(float);
}

// Tiles of the key pass that hold a probed list's rows: tile_on[t] = 1 when
// rows [t*32, t*32+32) meet a list some query probes (top_clusters).
__global__ void key_tile_flags_kernel(const int32_t* __restrict__ topc, int B, int m,
                                      const int64_t* __restrict__ list_off, int64_t row_lo, int64_t N,
                                      uint8_t* __restrict__ tile_on) {
    pdl_enter();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= B * m) return;
    const int c = topc[i];
    int64_t lo = list_off[c] - row_lo, hi = list_off[c + 1] - row_lo;
    lo = lo < 0 ? 0 : lo;
    hi = hi > N ? N : hi;
    for (int64_t t = lo / kKeyTile; t * kKeyTile < hi; ++t) tile_on[t] = 1;
}

// soft_full part of G: dot[b] = Σ_n g_soft soft (per-CTA partials, then in
// CTA order), G[b, n] = soft (g_soft - dot[b]) / T.  Grid (chunks, B).
constexpr int kSoftChunk = 4096;
__global__ void __launch_bounds__(256) soft_dot_kernel(const float* __restrict__ soft,
                                                      const float* __restrict__ g_soft, int64_t N,
                                                      float* __restrict__ part) {
    pdl_enter();
    __shared__ float red[33];
    const int b = blockIdx.y;
    const int64_t n0 = static_cast<int64_t>(blockIdx.x) * kSoftChunk;
    const int64_t n1 = n0 + kSoftChunk < N ? n0 + kSoftChunk : N;
    float acc = 0.f;
    if ((N & 3) == 0) {
        // 16-byte rows (N % 4 == 0): float4 loads
        const float4* s4 = reinterpret_cast<const float4*>(soft + static_cast<int64_t>(b) * N);
        const float4* g4 = reinterpret_cast<const float4*>(g_soft + static_cast<int64_t>(b) * N);
        for (int64_t n = n0 / 4 + threadIdx.x; n < n1 / 4; n += blockDim.x) {
            const float4 sv = s4[n], gv = g4[n];
            acc = fmaf(gv.x, sv.x, acc);
            acc = fmaf(gv.y, sv.y, acc);
            acc = fmaf(gv.z, sv.z, acc);
            acc = fmaf(gv.w, sv.w, acc);
        }
    } else {
        for (int64_t n = n0 + threadIdx.x; n < n1; n += blockDim.x)
            acc = fmaf(g_soft[static_cast<int64_t>(b) * N + n], soft[static_cast<int64_t>(b) * N + n], acc);
    }
    acc = block_reduce(acc, false, red);
    if (threadIdx.x == 0) part[static_cast<int64_t>(b) * gridDim.x + blockIdx.x] = acc;
}

__global__ void __launch_bounds__(256) soft_grad_kernel(const float* __restrict__ soft,
                                                       const float* __restrict__ g_soft, int64_t N,
                                                       const float* __restrict__ part, int nchunks, int pstride,
                                                       float invT, float* __restrict__ G) {
    pdl_enter();
    __shared__ float s_dot;
    const int b = blockIdx.y;
    if (threadIdx.x == 0) {
        float d = 0.f;
        for (int i = 0; i < nchunks; ++i) d += part[static_cast<int64_t>(b) * pstride + i];
        s_dot = d;
    }
    __syncthreads();
    const float dot = s_dot;
    const int64_t n0 = static_cast<int64_t>(blockIdx.x) * kSoftChunk;
    const int64_t n1 = n0 + kSoftChunk < N ? n0 + kSoftChunk : N;
    if ((N & 3) == 0) {
        const float4* s4 = reinterpret_cast<const float4*>(soft + static_cast<int64_t>(b) * N);
        const float4* g4 = reinterpret_cast<const float4*>(g_soft + static_cast<int64_t>(b) * N);
        float4* G4 = reinterpret_cast<float4*>(G + static_cast<int64_t>(b) * N);
        for (int64_t n = n0 / 4 + threadIdx.x; n < n1 / 4; n += blockDim.x) {
            const float4 sv = s4[n], gv = g4[n];
            G4[n] = make_float4(sv.x * (gv.x - dot) * invT, sv.y * (gv.y - dot) * invT,
                                sv.z * (gv.z - dot) * invT, sv.w * (gv.w - dot) * invT);
        }
    } else {
        for (int64_t n = n0 + threadIdx.x; n < n1; n += blockDim.x) {
            const int64_t i = static_cast<int64_t>(b) * N + n;
            G[i] = soft[i] * (g_soft[i] - dot) * invT;
        }
    }
}

// Selection backward of one query (one CTA): adds dL/ds of the alphas'
// cotangent to G[b, rows] and writes this query's part of g_tau.
struct SelGradArgs {
    const float* scores;       // [B, K_cap] candidate scores (gate)
    const int64_t* probe_lo;   // [B, m+1]
    const int64_t* cand_base;
    int m;
    int64_t K_cap, N;
    int k;
    float T;
    int is_warmup;
    const float* lambda_val;
    const float* tau;
    const float* alphas;       // [B, k]
    const int32_t* indices;    // [B, k] global rows
    const float* g_alphas;     // [B, k]
    int64_t row_lo;
    float* G;                  // [B, N]
    float* gtau;               // [B]
    uint32_t* status;
};

__global__ void __launch_bounds__(1024) sel_grad_kernel(SelGradArgs a) {
    pdl_enter();
    __shared__ int64_t s_lo[kMaxK + 1], s_base[kMaxK + 1];
    __shared__ float red[33];
    __shared__ float w_raw[kMaxK], w_fac[kMaxK], w_gt[kMaxK];
    __shared__ int64_t w_row[kMaxK];
    const int b = blockIdx.x, tid = threadIdx.x;
    for (int j = tid; j <= a.m; j += blockDim.x) {
        s_lo[j] = a.probe_lo[static_cast<int64_t>(b) * (a.m + 1) + j];
        s_base[j] = a.cand_base[static_cast<int64_t>(b) * (a.m + 1) + j];
    }
    __syncthreads();
    const int64_t n = s_base[a.m];
    const int got = static_cast<int>(n < a.k ? n : a.k);
    const float* ga = a.g_alphas + static_cast<int64_t>(b) * a.k;
    const float* al = a.alphas + static_cast<int64_t>(b) * a.k;
    float* Gb = a.G + static_cast<int64_t>(b) * a.N;
    const float T = a.T, invT = 1.f / a.T;
    if (a.is_warmup) {
        // α = softmax(top / T): g_top = α (g_α - Σ α g_α) / T on the winners
        float d = 0.f;
        for (int i = tid; i < got; i += blockDim.x) d = fmaf(al[i], ga[i], d);
        d = block_reduce(d, false, red);
        for (int i = tid; i < got; i += blockDim.x) {
            const int64_t row = static_cast<int64_t>(a.indices[static_cast<int64_t>(b) * a.k + i]) - a.row_lo;
            if (row < 0 || row >= a.N) { raise_status(a.status, DWA_STATUS_BAD_ROW_INDEX); continue; }
            Gb[row] += al[i] * (ga[i] - d) * invT;
        }
        if (tid == 0) a.gtau[b] = 0.f;
        return;
    }
    const float lam = __ldg(a.lambda_val), tau = __ldg(a.tau);
    const float* sc = a.scores + static_cast<int64_t>(b) * a.K_cap;
    // Z = Σ raw over every candidate
    float z = 0.f;
    for (int j = 0; j < a.m; ++j) {
        const int64_t base = s_base[j], sz = s_base[j + 1] - s_base[j];
        for (int64_t r = tid; r < sz; r += blockDim.x) z += gate_raw(sc[base + r], lam, tau, T);
    }
    const float Zp = block_reduce(z, false, red) + 1e-8f;
    // the winners: raw, the derivative factor, their candidate rows
    for (int i = tid; i < got; i += blockDim.x) {
        const int64_t row = static_cast<int64_t>(a.indices[static_cast<int64_t>(b) * a.k + i]) - a.row_lo;
        int64_t pos = -1;
        for (int j = 0; j < a.m && pos < 0; ++j)
            if (row >= s_lo[j] && row < s_lo[j] + (s_base[j + 1] - s_base[j])) pos = s_base[j] + (row - s_lo[j]);
        float raw = 0.f, fac = 0.f;
        if (pos < 0) {
            raise_status(a.status, DWA_STATUS_BAD_ROW_INDEX);
        } else {
            const float s = sc[pos];
            const float g = 1.f / (1.f + expf(-(lam * (s - tau))));
            raw = g * expf(s / T);
            fac = lam * (1.f - g) + invT;
        }
        w_raw[i] = raw;
        w_fac[i] = fac;
        w_row[i] = pos < 0 ? -1 : row;
    }
    __syncthreads();
    // α = t / (Σ t + ε), t = raw / Z: g_t = g_α / St - Σ g_α t / St²
    float st = 0.f, gt_dot = 0.f;
    for (int i = tid; i < got; i += blockDim.x) {
        const float t = w_raw[i] / Zp;
        st += t;
        gt_dot = fmaf(ga[i], t, gt_dot);
    }
    const float St = block_reduce(st, false, red) + 1e-8f;
    const float GD = block_reduce(gt_dot, false, red);
    float graw_dot = 0.f;
    for (int i = tid; i < got; i += blockDim.x) {
        const float g_t = ga[i] / St - GD / (St * St);
        w_gt[i] = g_t;
        graw_dot = fmaf(g_t, w_raw[i], graw_dot);
    }
    // g_raw = g_rn / Z - Σ g_rn raw / Z²: a common term on every candidate ...
    const float cz = -block_reduce(graw_dot, false, red) / (Zp * Zp);
    float tacc = 0.f;
    for (int j = 0; j < a.m; ++j) {
        const int64_t lo = s_lo[j], base = s_base[j], sz = s_base[j + 1] - s_base[j];
        for (int64_t r = tid; r < sz; r += blockDim.x) {
            const float s = sc[base + r];
            const float g = 1.f / (1.f + expf(-(lam * (s - tau))));
            const float raw = g * expf(s / T);
            Gb[lo + r] += cz * raw * (lam * (1.f - g) + invT);
            tacc += cz * raw * (-lam * (1.f - g));
        }
    }
    __syncthreads();   // the common terms are in G before the winners' terms add to them
    // ... and the winners' own term g_t / Z
    for (int i = tid; i < got; i += blockDim.x) {
        if (w_row[i] < 0) continue;
        const float graw = w_gt[i] / Zp;
        Gb[w_row[i]] += graw * w_raw[i] * w_fac[i];
        tacc -= graw * w_raw[i] * (w_fac[i] - invT);   // w_fac - 1/T = λ(1-σ)
    }
    tacc = block_reduce(tacc, false, red);
    if (tid == 0) a.gtau[b] = tacc;
}

// For the key gradient: q̂[b,s,:] = q / (|q| + 1e-8) (one warp per aspect of
// query b) and, from CTA 0, ws = softmax(aspect_weights).
__global__ void unweighted_queries_kernel(const float* __restrict__ q, const float* __restrict__ aspect_w, int S,
                                          int d_k, float* __restrict__ qh, float* __restrict__ ws) {
    pdl_enter();
    const int b = blockIdx.x, s = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (s >= S) return;
    const float* qr = q + (static_cast<int64_t>(b) * S + s) * d_k;
    float ss = 0.f;
    for (int d = lane; d < d_k; d += 32) ss = fmaf(qr[d], qr[d], ss);
    const float dn = sqrtf(warp_sum(ss)) + 1e-8f;
    for (int d = lane; d < d_k; d += 32) qh[(static_cast<int64_t>(b) * S + s) * d_k + d] = qr[d] / dn;
    if (b == 0 && lane == 0) {
        float mx = -INFINITY;
        for (int t = 0; t < S; ++t) mx = fmaxf(mx, aspect_w[t]);
        float den = 0.f;
        for (int t = 0; t < S; ++t) den += expf(aspect_w[t] - mx);
        ws[s] = expf(aspect_w[s] - mx) / den;
    }
}

// First level of A = Σ_CTA partial: group g of kPartGroups adds the partials
// [P*g/G, P*(g+1)/G) of every (query, column) in CTA order, 4 loads in flight
// per thread.  Grid (ceil(nb*cols/256), kPartGroups).
constexpr int kPartGroups = 16;
__global__ void __launch_bounds__(256) partial_reduce_kernel(const float* __restrict__ partial, int nparts,
                                                            int64_t width, float* __restrict__ out) {
    pdl_enter();
    const int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (e >= width) return;
    const int g = blockIdx.y;
    const int p0 = static_cast<int>(static_cast<int64_t>(nparts) * g / kPartGroups);
    const int p1 = static_cast<int>(static_cast<int64_t>(nparts) * (g + 1) / kPartGroups);
    float acc = 0.f;
    int p = p0;
    for (; p + 4 <= p1; p += 4) {
        const float v0 = partial[static_cast<int64_t>(p) * width + e];
        const float v1 = partial[static_cast<int64_t>(p + 1) * width + e];
        const float v2 = partial[static_cast<int64_t>(p + 2) * width + e];
        const float v3 = partial[static_cast<int64_t>(p + 3) * width + e];
        acc = (((acc + v0) + v1) + v2) + v3;
    }
    for (; p < p1; ++p) acc += partial[static_cast<int64_t>(p) * width + e];
    out[static_cast<int64_t>(g) * width + e] = acc;
}

// A = Σ_CTA partial (in CTA order), then per (query, aspect): g_q̂ = w_s A,
// g_w partial q̂·A, and g_q = normalize-VJP(g_q̂) into gq [B, S*d_k].
// One CTA per (query, aspect), d_k threads rounded up to a warp multiple.
__global__ void query_grad_kernel(const float* __restrict__ partial, int nparts, int nb, int b0, int rstride,
                                  const float* __restrict__ q, const float* __restrict__ aspect_w, int S,
                                  int d_k, float* __restrict__ gq, float* __restrict__ gw_part) {
    pdl_enter();
    __shared__ float red[33];
    const int bl = blockIdx.x, s = blockIdx.y, b = b0 + bl, d = threadIdx.x;
    float A = 0.f, qv = 0.f;
    if (d < d_k) {
        for (int p = 0; p < nparts; ++p) A += partial[(static_cast<int64_t>(p) * nb + bl) * rstride + s * d_k + d];
        qv = q[(static_cast<int64_t>(b) * S + s) * d_k + d];
    }
    float mx = -INFINITY;
    for (int t = 0; t < S; ++t) mx = fmaxf(mx, aspect_w[t]);
    float den = 0.f;
    for (int t = 0; t < S; ++t) den += expf(aspect_w[t] - mx);
    const float ws = expf(aspect_w[s] - mx) / den;
    const float n = sqrtf(block_reduce(qv * qv, false, red));
    const float dn = n + 1e-8f;
    const float gqh = ws * A;
    const float qh_dot_A = block_reduce((qv / dn) * A, false, red);   // g_w[s] share of this query
    const float q_dot_g = block_reduce(qv * gqh, false, red);
    if (d < d_k) {
        const float coef = n > 0.f ? q_dot_g / (n * dn * dn) : 0.f;
        gq[(static_cast<int64_t>(b) * S + s) * d_k + d] = gqh / dn - qv * coef;
    }
    if (d == 0) gw_part[static_cast<int64_t>(b) * S + s] = qh_dot_A;
}

// g_W_Q[o, a] = Σ_b gq[b, o] z[b, a] and this chunk's part of g_z[b, a] =
// Σ_o gq[b, o] W_Q[o, a]; grid (ceil(d_A/128), ceil(O/32)), 128 threads.
constexpr int kGradRowsPerCta = 32;
template <class ZT>
__global__ void __launch_bounds__(128) wq_grad_kernel(const float* __restrict__ gq, const ZT* __restrict__ z,
                                                     const float* __restrict__ W_Q, int B, int O, int d_A,
                                                     float* __restrict__ g_W_Q, float* __restrict__ gz_part) {
    pdl_enter();
    extern __shared__ float gqs[];   // [B][kGradRowsPerCta]
    const int a = blockIdx.x * 128 + threadIdx.x, o0 = blockIdx.y * kGradRowsPerCta;
    const int no = min(kGradRowsPerCta, O - o0);
    for (int i = threadIdx.x; i < B * kGradRowsPerCta; i += blockDim.x) {
        const int b = i / kGradRowsPerCta, r = i - b * kGradRowsPerCta;
        gqs[i] = r < no ? gq[static_cast<int64_t>(b) * O + o0 + r] : 0.f;
    }
    __syncthreads();
    if (a >= d_A) return;
    for (int r = 0; r < no; ++r) {
        float g = 0.f;
        for (int b = 0; b < B; ++b) g = fmaf(gqs[b * kGradRowsPerCta + r], Elem<ZT>::to_f(z[static_cast<int64_t>(b) * d_A + a]), g);
        g_W_Q[static_cast<int64_t>(o0 + r) * d_A + a] = g;
    }
    for (int b = 0; b < B; ++b) {
        float g = 0.f;
        for (int r = 0; r < no; ++r) g = fmaf(gqs[b * kGradRowsPerCta + r], W_Q[static_cast<int64_t>(o0 + r) * d_A + a], g);
        gz_part[(static_cast<int64_t>(blockIdx.y) * B + b) * d_A + a] = g;
    }
}

// g_z = Σ_chunks gz_part (chunk order); CTA 0 also writes g_aspect_weights
// (softmax VJP of g_w = Σ_b gw_part) and g_tau = Σ_b gtau.
__global__ void query_grad_finish_kernel(const float* __restrict__ gz_part, int nchunks, int B, int d_A,
                                         const float* __restrict__ gw_part, const float* __restrict__ aspect_w,
                                         int S, const float* __restrict__ gtau, int gtau_stride, float* __restrict__ g_z,
                                         float* __restrict__ g_aw, float* __restrict__ g_tau) {
    pdl_enter();
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < static_cast<int64_t>(B) * d_A) {
        float g = 0.f;
        for (int c = 0; c < nchunks; ++c) g += gz_part[static_cast<int64_t>(c) * B * d_A + i];
        g_z[i] = g;
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        float mx = -INFINITY;
        for (int t = 0; t < S; ++t) mx = fmaxf(mx, aspect_w[t]);
        float den = 0.f;
        for (int t = 0; t < S; ++t) den += expf(aspect_w[t] - mx);
        float wg = 0.f;
        for (int t = 0; t < S; ++t) {
            float gw = 0.f;
            for (int b = 0; b < B; ++b) gw += gw_part[static_cast<int64_t>(b) * S + t];
            wg += (expf(aspect_w[t] - mx) / den) * gw;
        }
        for (int t = 0; t < S; ++t) {
            float gw = 0.f;
            for (int b = 0; b < B; ++b) gw += gw_part[static_cast<int64_t>(b) * S + t];
            g_aw[t] = (expf(aspect_w[t] - mx) / den) * (gw - wg);
        }
        float gt = 0.f;
        for (int b = 0; b < B; ++b) gt += gtau[static_cast<int64_t>(b) * gtau_stride];
        g_tau[0] = gt;
    }
}

struct BwdWorkspace {
    RetWorkspace f;      // the forward's query / probe / score buffers
    float* G;            // [B, N]
    float* partial;      // [grid, min(B, 32), S*d_k]
    float* gq;           // [B, S*d_k]
    float* part2;        // [kPartGroups, min(B, 32), S*d_k]
    float* qh;           // [B, S*d_k] normalised queries, unweighted (key gradient)
    float* ws;           // [S] softmax(aspect_weights) (key gradient)
    float* gw_part;      // [B, S]
    float* gtau;         // [B]
    float* gz_part;      // [ceil(S*d_k/32), B, d_A]
    float* soft_part;    // [B, ceil(N/4096)]
    uint8_t* tile_on;    // [ceil(N/32)]
    int grid;
    size_t bytes;
};

static int key_pass_grid() {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return 4 * sms;
}

static BwdWorkspace carve_bwd(void* base, const DwaRetrieveDims& d, bool ivf) {
    BwdWorkspace w{};
    // the forward's buffers first (with fine scores, without soft_full's), then ours
    w.f = carve_ret(base, d, ivf, false);
    Carver c(base);
    c.off = w.f.bytes;
    const int cols = d.S * d.d_k;
    const int64_t ntiles = (d.N + kKeyTile - 1) / kKeyTile;
    w.grid = static_cast<int>(std::min<int64_t>(ntiles, key_pass_grid()));
    w.G = c.take<float>(static_cast<size_t>(d.B) * d.N);
    w.partial = c.take<float>(static_cast<size_t>(w.grid) * std::min(d.B, kBwdMaxQ) * cols);
    w.gq = c.take<float>(static_cast<size_t>(d.B) * cols);
    w.part2 = c.take<float>(static_cast<size_t>(kPartGroups) * std::min(d.B, kBwdMaxQ) * cols);
    w.qh = c.take<float>(static_cast<size_t>(d.B) * cols);
    w.ws = c.take<float>(static_cast<size_t>(d.S));
    w.gw_part = c.take<float>(static_cast<size_t>(d.B) * d.S);
    w.gtau = c.take<float>(static_cast<size_t>(d.B));
    w.gz_part = c.take<float>(static_cast<size_t>((cols + kGradRowsPerCta - 1) / kGradRowsPerCta) * d.B * d.d_A);
    w.soft_part = c.take<float>(static_cast<size_t>(d.B) * ((d.N + kSoftChunk - 1) / kSoftChunk));
    w.tile_on = c.take<uint8_t>(static_cast<size_t>(ntiles));
    w.bytes = c.bytes();
    return w;
}

static int check_bwd(const DwaRetrieveDims* d, int use_ivf) {
    int rc = check_ret(d, use_ivf);
    if (rc) return rc;
    if (d->d_k % 4 != 0 || 1024 % d->d_k != 0)
        return fail(DWA_ERR_UNSUPPORTED, "retrieval VJP needs d_k % 4 == 0 and d_k dividing 1024");
    if (d->S * d->d_k > 4 * kKeyThreads) return fail(DWA_ERR_UNSUPPORTED, "retrieval VJP needs S*d_k <= 1024");
    return DWA_OK;
}

// The key pass of a VJP call over the key rows [0, d.N) of `keys`: the probed
// lists' tiles only when `probed_only`, the key gradient when g_pool_keys is
// non-NULL; `per_pass(b0, nb, grid)` runs after each pass of <= kBwdMaxQ
// queries on its per-CTA partials.
template <class PerPass>
static int run_key_pass(cudaStream_t st, const DwaRetrieveDims& d, const BwdWorkspace& w, const float* keys,
                        const float* aspect_weights, const int64_t* list_offsets, int64_t row_lo,
                        bool probed_only, float* g_pool_keys, const PerPass& per_pass) {
    const RetWorkspace& f = w.f;
    const int64_t ntiles = (d.N + kKeyTile - 1) / kKeyTile;
    if (probed_only) {
        DWA_CUDA_TRY(cudaMemsetAsync(w.tile_on, 0, static_cast<size_t>(ntiles), st));
        launch_pdl(key_tile_flags_kernel, (d.B * f.m_eff + 127) / 128, 128, 0, st, f.topc, d.B, f.m_eff,
                   list_offsets, row_lo, d.N, w.tile_on);
        DWA_LAUNCH_CHECK("key_tile_flags_kernel");
        ++g_launches_total;
    }
    const int cols = d.S * d.d_k;
    const int cpt = (cols + kKeyThreads - 1) / kKeyThreads;
    if (g_pool_keys) {
        // the key gradient needs the normalised queries unweighted and the aspect weights
        launch_pdl(unweighted_queries_kernel, d.B, 32 * d.S, 0, st, f.q, aspect_weights, d.S, d.d_k, w.qh, w.ws);
        DWA_LAUNCH_CHECK("unweighted_queries_kernel");
        ++g_launches_total;
    }
    for (int b0 = 0; b0 < d.B; b0 += kBwdMaxQ) {
        const int nb = std::min(kBwdMaxQ, d.B - b0);
        const int qb = nb <= 8 ? 8 : nb <= 16 ? 16 : 32;
        KeyGradArgs ka{};
        ka.keys = keys; ka.N = d.N; ka.S = d.S; ka.d_k = d.d_k; ka.B = d.B; ka.b0 = b0; ka.nb = nb;
        ka.G = w.G; ka.qh = w.qh; ka.w = w.ws; ka.tile_on = probed_only ? w.tile_on : nullptr;
        ka.ntiles = ntiles; ka.partial = w.partial; ka.g_keys = g_pool_keys;
        if (cpt > 2 && qb > 16) return fail(DWA_ERR_UNSUPPORTED, "retrieval VJP: S*d_k > 512 needs B <= 16 per pass");
        const size_t sm = key_grad_smem(d.S, d.d_k, qb, g_pool_keys != nullptr);
        if (sm > 200 * 1024) return fail(DWA_ERR_UNSUPPORTED, "retrieval VJP: S*d_k too large for the key tile");
        void (*fn)(KeyGradArgs) = nullptr;
        const bool fused = g_pool_keys != nullptr;   // the key gradient is always the fused pass
        if (fused) {
            if (cpt == 1) fn = qb == 8 ? key_grad_pass_kernel<1, 8, true> : qb == 16 ? key_grad_pass_kernel<1, 16, true> : key_grad_pass_kernel<1, 32, true>;
            else if (cpt == 2) fn = qb == 8 ? key_grad_pass_kernel<2, 8, true> : qb == 16 ? key_grad_pass_kernel<2, 16, true> : key_grad_pass_kernel<2, 32, true>;
            else fn = qb == 8 ? key_grad_pass_kernel<4, 8, true> : key_grad_pass_kernel<4, 16, true>;
        } else if (cpt == 1) fn = qb == 8 ? key_grad_pass_kernel<1, 8> : qb == 16 ? key_grad_pass_kernel<1, 16> : key_grad_pass_kernel<1, 32>;
        else if (cpt == 2) fn = qb == 8 ? key_grad_pass_kernel<2, 8> : qb == 16 ? key_grad_pass_kernel<2, 16> : key_grad_pass_kernel<2, 32>;
        else fn = qb == 8 ? key_grad_pass_kernel<4, 8> : key_grad_pass_kernel<4, 16>;
        DWA_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sm)));
        // one wave of persistent CTAs (at most the grid the partials were sized for)
        int occ = 1, dv = 0, sms = 148;
        DWA_CUDA_TRY(cudaGetDevice(&dv));
        DWA_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dv));
        DWA_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, kKeyThreads, sm));
        const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(
            {static_cast<int64_t>(w.grid), static_cast<int64_t>(std::max(occ, 1)) * sms, ntiles})));
        DWA_TIMED("key_grad", st, launch_pdl(fn, grid, kKeyThreads, sm, st, ka));
        DWA_LAUNCH_CHECK("key_grad_pass_kernel");
        const int64_t width = static_cast<int64_t>(nb) * cols;
        launch_pdl(partial_reduce_kernel, dim3(static_cast<unsigned>((width + 255) / 256), kPartGroups), 256, 0, st,
                   w.partial, grid, width, w.part2);
        DWA_LAUNCH_CHECK("partial_reduce_kernel");
        g_launches_total += 2;
        int rc = per_pass(b0, nb);
        if (rc) return rc;
    }
    return DWA_OK;
}

}  // namespace dwa

extern "C" size_t dwa_retrieve_bwd_workspace_bytes(const DwaRetrieveDims* dims, int use_ivf) {
    using namespace dwa;
    if (check_bwd(dims, use_ivf)) return 0;
    return carve_bwd(nullptr, *dims, use_ivf != 0).bytes;
}

extern "C" int dwa_retrieve_bwd(void* stream, const DwaRetrieveDims* dims, int use_ivf, int is_warmup,
                                const float* lambda_val, const void* z, const float* W_Q,
                                const float* aspect_weights, const float* tau, const float* centroids,
                                const int64_t* list_offsets, const float* pool_keys, const float* alphas,
                                const int32_t* indices, const float* soft_full, const float* g_alphas,
                                const float* g_soft_full, float* g_z, float* g_W_Q, float* g_aspect_weights,
                                float* g_tau, float* g_pool_keys, void* workspace, size_t workspace_bytes) {
    using namespace dwa;
    int rc = check_bwd(dims, use_ivf);
    if (rc) return rc;
    const DwaRetrieveDims& d = *dims;
    const bool ivf = use_ivf != 0;
    if (!lambda_val || !z || !W_Q || !aspect_weights || !tau || !pool_keys || !g_z || !g_W_Q ||
        !g_aspect_weights || !g_tau)
        return fail(DWA_ERR_INVALID_ARG, "a required pointer is NULL");
    if (g_alphas && (!alphas || !indices)) return fail(DWA_ERR_INVALID_ARG, "g_alphas needs alphas and indices");
    if (g_soft_full && !soft_full) return fail(DWA_ERR_INVALID_ARG, "g_soft_full needs soft_full");
    if (ivf && (!centroids || !list_offsets)) return fail(DWA_ERR_INVALID_ARG, "IVF needs centroids and list_offsets");
    if (reinterpret_cast<uintptr_t>(pool_keys) % 16 != 0) return fail(DWA_ERR_INVALID_ARG, "pool_keys must be 16-byte aligned");
    if (g_pool_keys && d.B > kBwdMaxQ) return fail(DWA_ERR_UNSUPPORTED, "retrieval VJP: the key gradient needs B <= 32");
    const BwdWorkspace w = carve_bwd(workspace, d, ivf);
    if (!workspace || reinterpret_cast<uintptr_t>(workspace) % 256 != 0)
        return fail(DWA_ERR_WORKSPACE, "workspace must be non-NULL and 256-byte aligned");
    if (workspace_bytes < w.bytes) return fail(DWA_ERR_WORKSPACE, "workspace too small: need " + std::to_string(w.bytes));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const bool dk64 = d.d_k == 64 && (!ivf || reinterpret_cast<uintptr_t>(centroids) % 16 == 0);
    const RetWorkspace& f = w.f;
    const size_t qsh = static_cast<size_t>(d.S) * d.d_k * sizeof(float);

    // 1. the forward's queries and probes
    if ((rc = launch_queries_and_probes(st, d, ivf, dk64, z, W_Q, aspect_weights, centroids, list_offsets, 0, d.N, f)))
        return rc;
    const bool gate = !is_warmup && g_alphas;
    // 2. gate mode: every candidate's score
    float* scores = ivf ? f.scores : f.sfull;   // [B, K_cap]; K_cap = N without IVF
    if (gate) {
        dim3 gf(static_cast<unsigned>(((ivf ? d.max_list : d.N) + 255) / 256), f.m_eff, d.B);
        if (dk64)
            launch_pdl(fine_kernel<64>, gf, 256, qsh, st, f.qw, pool_keys, d.N, d.S, d.d_k, f.m_eff, f.probe_lo,
                       f.cand_base, f.K_cap, scores);
        else
            launch_pdl(fine_kernel<0>, gf, 256, qsh, st, f.qw, pool_keys, d.N, d.S, d.d_k, f.m_eff, f.probe_lo,
                       f.cand_base, f.K_cap, scores);
        DWA_LAUNCH_CHECK("fine_kernel");
        ++g_launches_total;
    }
    // 3. G: the soft_full part (or zeros), then the selection part
    const int nchunks = static_cast<int>((d.N + kSoftChunk - 1) / kSoftChunk);
    if (g_soft_full) {
        launch_pdl(soft_dot_kernel, dim3(nchunks, d.B), 256, 0, st, soft_full, g_soft_full, d.N, w.soft_part);
        DWA_LAUNCH_CHECK("soft_dot_kernel");
        launch_pdl(soft_grad_kernel, dim3(nchunks, d.B), 256, 0, st, soft_full, g_soft_full, d.N, w.soft_part,
                   nchunks, nchunks, 1.f / d.T, w.G);
        DWA_LAUNCH_CHECK("soft_grad_kernel");
        g_launches_total += 2;
    } else {
        DWA_CUDA_TRY(cudaMemsetAsync(w.G, 0, static_cast<size_t>(d.B) * d.N * sizeof(float), st));
    }
    if (g_alphas) {
        SelGradArgs sa{};
        sa.scores = scores; sa.probe_lo = f.probe_lo; sa.cand_base = f.cand_base; sa.m = f.m_eff;
        sa.K_cap = f.K_cap; sa.N = d.N; sa.k = d.k; sa.T = d.T; sa.is_warmup = is_warmup;
        sa.lambda_val = lambda_val; sa.tau = tau; sa.alphas = alphas; sa.indices = indices;
        sa.g_alphas = g_alphas; sa.row_lo = 0; sa.G = w.G; sa.gtau = w.gtau; sa.status = f.status;
        DWA_TIMED("sel_grad", st, launch_pdl(sel_grad_kernel, d.B, 1024, 0, st, sa));
        DWA_LAUNCH_CHECK("sel_grad_kernel");
        ++g_launches_total;
    } else {
        DWA_CUDA_TRY(cudaMemsetAsync(w.gtau, 0, static_cast<size_t>(d.B) * sizeof(float), st));
    }
    // 4. key pass: every row, or the tiles of probed lists when only the
    //    selection has a cotangent and no key gradient is asked for;
    // 5. the queries' gradients of each pass
    const int cols = d.S * d.d_k;
    const int qthreads = (d.d_k + 31) / 32 * 32;
    rc = run_key_pass(st, d, w, pool_keys, aspect_weights, list_offsets, 0, ivf && !g_soft_full && !g_pool_keys,
                      g_pool_keys, [&](int b0, int nb) {
                          launch_pdl(query_grad_kernel, dim3(nb, d.S), qthreads, 0, st, w.part2, kPartGroups, nb, b0,
                                     cols, f.q, aspect_weights, d.S, d.d_k, w.gq, w.gw_part);
                          DWA_LAUNCH_CHECK("query_grad_kernel");
                          ++g_launches_total;
                          return DWA_OK;
                      });
    if (rc) return rc;
    const int nchunk_o = (cols + kGradRowsPerCta - 1) / kGradRowsPerCta;
    const size_t gsh = static_cast<size_t>(d.B) * kGradRowsPerCta * sizeof(float);
    if (gsh > 48 * 1024) return fail(DWA_ERR_UNSUPPORTED, "retrieval VJP: B too large for the W_Q gradient");
    const dim3 gw((d.d_A + 127) / 128, nchunk_o);
    if (d.z_dtype == DWA_BF16)
        launch_pdl(wq_grad_kernel<__nv_bfloat16>, gw, 128, gsh, st, w.gq, static_cast<const __nv_bfloat16*>(z), W_Q,
                   d.B, cols, d.d_A, g_W_Q, w.gz_part);
    else
        launch_pdl(wq_grad_kernel<float>, gw, 128, gsh, st, w.gq, static_cast<const float*>(z), W_Q, d.B, cols,
                   d.d_A, g_W_Q, w.gz_part);
    DWA_LAUNCH_CHECK("wq_grad_kernel");
    const int64_t nz = static_cast<int64_t>(d.B) * d.d_A;
    launch_pdl(query_grad_finish_kernel, static_cast<unsigned>((nz + 255) / 256), 256, 0, st, w.gz_part, nchunk_o, d.B,
               d.d_A, w.gw_part, aspect_weights, d.S, w.gtau, 1, g_z, g_aspect_weights, g_tau);
    DWA_LAUNCH_CHECK("query_grad_finish_kernel");
    g_launches_total += 2;
    return DWA_OK;
}

// ---------------------------------------------------------------------------
// The VJP over a row-sharded pool: every rank runs phase 1 on its rows, the
// caller sums the [B, k+3] partials over the ranks, every rank runs phase 2,
// the caller sums the [B, S*d_k+1] partials, and every rank runs phase 3.
// The same workspace goes to all three phases of one call.
// ---------------------------------------------------------------------------
namespace dwa {

// Phase-1 partials of query b, [k+3]: the scores of the winners this rank
// holds (0 for the others), Σ raw over this rank's candidates (gate mode),
// Σ g_soft·soft over its rows (added in chunk order), its candidate count.
struct Part1Args {
    const float* scores;       // [B, K_cap] (gate) or null
    const int64_t* probe_lo;
    const int64_t* cand_base;
    int m;
    int64_t K_cap, N, row_lo;
    int k;
    float T;
    int gate;
    const float* lambda_val;
    const float* tau;
    const int32_t* indices;    // [B, k] global rows
    const float* soft_part;    // [B, nchunks] or null
    int nchunks;
    float* part1;              // [B, k+3]
};

__global__ void __launch_bounds__(256) bwd_part1_kernel(Part1Args a) {
    pdl_enter();
    __shared__ int64_t s_lo[kMaxK + 1], s_base[kMaxK + 1];
    __shared__ float red[33];
    const int b = blockIdx.x, tid = threadIdx.x, W = a.k + 3;
    for (int j = tid; j <= a.m; j += blockDim.x) {
        s_lo[j] = a.probe_lo[static_cast<int64_t>(b) * (a.m + 1) + j];
        s_base[j] = a.cand_base[static_cast<int64_t>(b) * (a.m + 1) + j];
    }
    __syncthreads();
    float* out = a.part1 + static_cast<int64_t>(b) * W;
    const float* sc = a.gate ? a.scores + static_cast<int64_t>(b) * a.K_cap : nullptr;
    for (int i = tid; i < a.k; i += blockDim.x) {
        float v = 0.f;
        if (sc) {
            const int64_t row = static_cast<int64_t>(a.indices[static_cast<int64_t>(b) * a.k + i]) - a.row_lo;
            for (int j = 0; j < a.m; ++j)
                if (row >= s_lo[j] && row < s_lo[j] + (s_base[j + 1] - s_base[j])) v = sc[s_base[j] + (row - s_lo[j])];
        }
        out[i] = v;
    }
    float z = 0.f;
    if (sc) {
        const float lam = __ldg(a.lambda_val), tau = __ldg(a.tau);
        for (int j = 0; j < a.m; ++j) {
            const int64_t base = s_base[j], sz = s_base[j + 1] - s_base[j];
            for (int64_t r = tid; r < sz; r += blockDim.x) z += gate_raw(sc[base + r], lam, tau, a.T);
        }
    }
    z = block_reduce(z, false, red);
    if (tid == 0) {
        float dt = 0.f;
        if (a.soft_part)
            for (int c = 0; c < a.nchunks; ++c) dt += a.soft_part[static_cast<int64_t>(b) * a.nchunks + c];
        out[a.k] = z;
        out[a.k + 1] = dt;
        out[a.k + 2] = static_cast<float>(s_base[a.m]);
    }
}

// Selection backward of query b on this rank's rows from the summed phase-1
// values: the same quantities as sel_grad_kernel (the gate sum Z, the winners'
// gate terms, the top-k backward of α), added to G for this rank's candidates
// and winners only; this rank's share of g_tau.
struct SelGradGlobalArgs {
    SelGradArgs s;             // scores / probes / N / row_lo of this rank
    const float* part1;        // [B, k+3] summed over the ranks
};

__global__ void __launch_bounds__(1024) sel_grad_global_kernel(SelGradGlobalArgs g) {
    pdl_enter();
    const SelGradArgs& a = g.s;
    __shared__ int64_t s_lo[kMaxK + 1], s_base[kMaxK + 1];
    __shared__ float red[33];
    __shared__ float w_raw[kMaxK], w_fac[kMaxK], w_gt[kMaxK];
    const int b = blockIdx.x, tid = threadIdx.x, W = a.k + 3;
    for (int j = tid; j <= a.m; j += blockDim.x) {
        s_lo[j] = a.probe_lo[static_cast<int64_t>(b) * (a.m + 1) + j];
        s_base[j] = a.cand_base[static_cast<int64_t>(b) * (a.m + 1) + j];
    }
    __syncthreads();
    const float* p1 = g.part1 + static_cast<int64_t>(b) * W;
    const float n_all = p1[a.k + 2];
    const int got = n_all < static_cast<float>(a.k) ? static_cast<int>(n_all) : a.k;
    const float* ga = a.g_alphas + static_cast<int64_t>(b) * a.k;
    const float* al = a.alphas + static_cast<int64_t>(b) * a.k;
    float* Gb = a.G + static_cast<int64_t>(b) * a.N;
    const float T = a.T, invT = 1.f / a.T;
    auto local_row = [&](int i) {
        const int64_t row = static_cast<int64_t>(a.indices[static_cast<int64_t>(b) * a.k + i]) - a.row_lo;
        return (row >= 0 && row < a.N) ? row : int64_t(-1);
    };
    if (a.is_warmup) {
        float d = 0.f;
        for (int i = tid; i < got; i += blockDim.x) d = fmaf(al[i], ga[i], d);
        d = block_reduce(d, false, red);
        for (int i = tid; i < got; i += blockDim.x) {
            const int64_t row = local_row(i);
            if (row >= 0) Gb[row] += al[i] * (ga[i] - d) * invT;
        }
        if (tid == 0) a.gtau[b] = 0.f;
        return;
    }
    const float lam = __ldg(a.lambda_val), tau = __ldg(a.tau);
    const float Zp = p1[a.k] + 1e-8f;
    for (int i = tid; i < got; i += blockDim.x) {
        const float s = p1[i];
        const float sg = 1.f / (1.f + expf(-(lam * (s - tau))));
        w_raw[i] = sg * expf(s / T);
        w_fac[i] = lam * (1.f - sg) + invT;
    }
    __syncthreads();
    float st = 0.f, gt_dot = 0.f;
    for (int i = tid; i < got; i += blockDim.x) {
        const float t = w_raw[i] / Zp;
        st += t;
        gt_dot = fmaf(ga[i], t, gt_dot);
    }
    const float St = block_reduce(st, false, red) + 1e-8f;
    const float GD = block_reduce(gt_dot, false, red);
    float graw_dot = 0.f;
    for (int i = tid; i < got; i += blockDim.x) {
        const float g_t = ga[i] / St - GD / (St * St);
        w_gt[i] = g_t;
        graw_dot = fmaf(g_t, w_raw[i], graw_dot);
    }
    const float cz = -block_reduce(graw_dot, false, red) / (Zp * Zp);
    const float* sc = a.scores + static_cast<int64_t>(b) * a.K_cap;
    float tacc = 0.f;
    for (int j = 0; j < a.m; ++j) {
        const int64_t lo = s_lo[j], base = s_base[j], sz = s_base[j + 1] - s_base[j];
        for (int64_t r = tid; r < sz; r += blockDim.x) {
            const float s = sc[base + r];
            const float sg = 1.f / (1.f + expf(-(lam * (s - tau))));
            const float raw = sg * expf(s / T);
            Gb[lo + r] += cz * raw * (lam * (1.f - sg) + invT);
            tacc += cz * raw * (-lam * (1.f - sg));
        }
    }
    __syncthreads();
    for (int i = tid; i < got; i += blockDim.x) {
        const int64_t row = local_row(i);
        if (row < 0) continue;
        const float graw = w_gt[i] / Zp;
        Gb[row] += graw * w_raw[i] * w_fac[i];
        tacc -= graw * w_raw[i] * (w_fac[i] - invT);
    }
    tacc = block_reduce(tacc, false, red);
    if (tid == 0) a.gtau[b] = tacc;
}

// This rank's A of queries [b0, b0+nb) = Σ of the kPartGroups partial groups,
// into part2 [B, cols+1] (row stride cols+1), with its g_tau share in column cols.
__global__ void a_final_kernel(const float* __restrict__ part, int nb, int b0, int cols,
                               const float* __restrict__ gtau, float* __restrict__ part2) {
    pdl_enter();
    const int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t width = static_cast<int64_t>(nb) * cols;
    if (e < width) {
        float acc = 0.f;
        for (int g = 0; g < kPartGroups; ++g) acc += part[static_cast<int64_t>(g) * width + e];
        const int bl = static_cast<int>(e / cols), col = static_cast<int>(e % cols);
        part2[static_cast<int64_t>(b0 + bl) * (cols + 1) + col] = acc;
    } else if (e < width + nb) {
        const int bl = static_cast<int>(e - width);
        part2[static_cast<int64_t>(b0 + bl) * (cols + 1) + cols] = gtau[b0 + bl];
    }
}

}  // namespace dwa

extern "C" size_t dwa_retrieve_bwd_local_workspace_bytes(const DwaRetrieveDims* dims, int use_ivf) {
    return dwa_retrieve_bwd_workspace_bytes(dims, use_ivf);
}

extern "C" int dwa_retrieve_bwd_local1(void* stream, const DwaRetrieveDims* dims, const DwaShard* shard, int use_ivf,
                                       int is_warmup, const float* lambda_val, const void* z, const float* W_Q,
                                       const float* aspect_weights, const float* tau, const float* centroids,
                                       const int64_t* list_offsets, const float* local_keys, const int32_t* indices,
                                       const float* soft_full, const float* g_soft_full, float* part1,
                                       void* workspace, size_t workspace_bytes) {
    using namespace dwa;
    int rc = check_bwd(dims, use_ivf);
    if (rc) return rc;
    const DwaRetrieveDims& d = *dims;
    const bool ivf = use_ivf != 0;
    if (!shard || shard->row_lo < 0 || shard->n_global < shard->row_lo + d.N || shard->n_global >= (int64_t(1) << 31))
        return fail(DWA_ERR_INVALID_ARG, "shard: need 0 <= row_lo and row_lo + N <= n_global < 2^31");
    if (!lambda_val || !z || !W_Q || !aspect_weights || !tau || !local_keys || !indices || !part1)
        return fail(DWA_ERR_INVALID_ARG, "a required pointer is NULL");
    if (g_soft_full && !soft_full) return fail(DWA_ERR_INVALID_ARG, "g_soft_full needs soft_full");
    if (ivf && (!centroids || !list_offsets)) return fail(DWA_ERR_INVALID_ARG, "IVF needs centroids and list_offsets");
    const BwdWorkspace w = carve_bwd(workspace, d, ivf);
    if (!workspace || reinterpret_cast<uintptr_t>(workspace) % 256 != 0 || workspace_bytes < w.bytes)
        return fail(DWA_ERR_WORKSPACE, "workspace: dwa_retrieve_bwd_local_workspace_bytes, 256-byte aligned");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const bool dk64 = d.d_k == 64 && reinterpret_cast<uintptr_t>(local_keys) % 16 == 0 &&
                      (!ivf || reinterpret_cast<uintptr_t>(centroids) % 16 == 0);
    const RetWorkspace& f = w.f;
    const size_t qsh = static_cast<size_t>(d.S) * d.d_k * sizeof(float);
    if ((rc = launch_queries_and_probes(st, d, ivf, dk64, z, W_Q, aspect_weights, centroids, list_offsets,
                                        shard->row_lo, shard->n_global, f)))
        return rc;
    const bool gate = !is_warmup;
    float* scores = ivf ? f.scores : f.sfull;
    if (gate) {
        dim3 gf(static_cast<unsigned>(((ivf ? d.max_list : d.N) + 255) / 256), f.m_eff, d.B);
        if (dk64)
            launch_pdl(fine_kernel<64>, gf, 256, qsh, st, f.qw, local_keys, d.N, d.S, d.d_k, f.m_eff, f.probe_lo,
                       f.cand_base, f.K_cap, scores);
        else
            launch_pdl(fine_kernel<0>, gf, 256, qsh, st, f.qw, local_keys, d.N, d.S, d.d_k, f.m_eff, f.probe_lo,
                       f.cand_base, f.K_cap, scores);
        DWA_LAUNCH_CHECK("fine_kernel");
        ++g_launches_total;
    }
    const int nchunks = static_cast<int>((d.N + kSoftChunk - 1) / kSoftChunk);
    if (g_soft_full) {
        launch_pdl(soft_dot_kernel, dim3(nchunks, d.B), 256, 0, st, soft_full, g_soft_full, d.N, w.soft_part);
        DWA_LAUNCH_CHECK("soft_dot_kernel");
        ++g_launches_total;
    }
    Part1Args pa{};
    pa.scores = gate ? scores : nullptr; pa.probe_lo = f.probe_lo; pa.cand_base = f.cand_base; pa.m = f.m_eff;
    pa.K_cap = f.K_cap; pa.N = d.N; pa.row_lo = shard->row_lo; pa.k = d.k; pa.T = d.T; pa.gate = gate;
    pa.lambda_val = lambda_val; pa.tau = tau; pa.indices = indices;
    pa.soft_part = g_soft_full ? w.soft_part : nullptr; pa.nchunks = nchunks; pa.part1 = part1;
    launch_pdl(bwd_part1_kernel, d.B, 256, 0, st, pa);
    DWA_LAUNCH_CHECK("bwd_part1_kernel");
    ++g_launches_total;
    return DWA_OK;
}

extern "C" int dwa_retrieve_bwd_local2(void* stream, const DwaRetrieveDims* dims, const DwaShard* shard, int use_ivf,
                                       int is_warmup, const float* lambda_val, const float* tau,
                                       const float* aspect_weights, const int64_t* list_offsets,
                                       const float* local_keys, const float* alphas, const int32_t* indices,
                                       const float* soft_full, const float* g_alphas, const float* g_soft_full,
                                       const float* part1_sum, float* part2, float* g_pool_keys, void* workspace,
                                       size_t workspace_bytes) {
    using namespace dwa;
    int rc = check_bwd(dims, use_ivf);
    if (rc) return rc;
    const DwaRetrieveDims& d = *dims;
    const bool ivf = use_ivf != 0;
    if (!shard || shard->row_lo < 0) return fail(DWA_ERR_INVALID_ARG, "shard is NULL or row_lo < 0");
    if (!lambda_val || !tau || !aspect_weights || !local_keys || !part1_sum || !part2 || (ivf && !list_offsets))
        return fail(DWA_ERR_INVALID_ARG, "a required pointer is NULL");
    if (g_alphas && (!alphas || !indices)) return fail(DWA_ERR_INVALID_ARG, "g_alphas needs alphas and indices");
    if (g_soft_full && !soft_full) return fail(DWA_ERR_INVALID_ARG, "g_soft_full needs soft_full");
    if (reinterpret_cast<uintptr_t>(local_keys) % 16 != 0) return fail(DWA_ERR_INVALID_ARG, "keys must be 16-byte aligned");
    if (g_pool_keys && d.B > kBwdMaxQ) return fail(DWA_ERR_UNSUPPORTED, "retrieval VJP: the key gradient needs B <= 32");
    const BwdWorkspace w = carve_bwd(workspace, d, ivf);
    if (!workspace || reinterpret_cast<uintptr_t>(workspace) % 256 != 0 || workspace_bytes < w.bytes)
        return fail(DWA_ERR_WORKSPACE, "workspace: dwa_retrieve_bwd_local_workspace_bytes, 256-byte aligned");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const RetWorkspace& f = w.f;
    float* scores = ivf ? f.scores : f.sfull;
    if (g_soft_full) {
        const int nc = static_cast<int>((d.N + kSoftChunk - 1) / kSoftChunk);
        launch_pdl(soft_grad_kernel, dim3(nc, d.B), 256, 0, st, soft_full, g_soft_full, d.N, part1_sum + d.k + 1, 1,
                   d.k + 3, 1.f / d.T, w.G);
        DWA_LAUNCH_CHECK("soft_grad_kernel");
        ++g_launches_total;
    } else {
        DWA_CUDA_TRY(cudaMemsetAsync(w.G, 0, static_cast<size_t>(d.B) * d.N * sizeof(float), st));
    }
    if (g_alphas) {
        SelGradGlobalArgs ga{};
        SelGradArgs& sa = ga.s;
        sa.scores = scores; sa.probe_lo = f.probe_lo; sa.cand_base = f.cand_base; sa.m = f.m_eff;
        sa.K_cap = f.K_cap; sa.N = d.N; sa.k = d.k; sa.T = d.T; sa.is_warmup = is_warmup;
        sa.lambda_val = lambda_val; sa.tau = tau; sa.alphas = alphas; sa.indices = indices;
        sa.g_alphas = g_alphas; sa.row_lo = shard->row_lo; sa.G = w.G; sa.gtau = w.gtau; sa.status = f.status;
        ga.part1 = part1_sum;
        launch_pdl(sel_grad_global_kernel, d.B, 1024, 0, st, ga);
        DWA_LAUNCH_CHECK("sel_grad_global_kernel");
        ++g_launches_total;
    } else {
        DWA_CUDA_TRY(cudaMemsetAsync(w.gtau, 0, static_cast<size_t>(d.B) * sizeof(float), st));
    }
    const int cols = d.S * d.d_k;
    rc = run_key_pass(st, d, w, local_keys, aspect_weights, list_offsets, shard->row_lo,
                      ivf && !g_soft_full && !g_pool_keys, g_pool_keys, [&](int b0, int nb) {
                          const int64_t width = static_cast<int64_t>(nb) * cols;
                          launch_pdl(a_final_kernel, static_cast<unsigned>((width + nb + 255) / 256), 256, 0, st,
                                     w.part2, nb, b0, cols, w.gtau, part2);
                          DWA_LAUNCH_CHECK("a_final_kernel");
                          ++g_launches_total;
                          return DWA_OK;
                      });
    if (rc) return rc;
    return DWA_OK;
}

extern "C" int dwa_retrieve_bwd_finish(void* stream, const DwaRetrieveDims* dims, int use_ivf, const void* z,
                                       const float* W_Q, const float* aspect_weights, const float* part2_sum,
                                       float* g_z, float* g_W_Q, float* g_aspect_weights, float* g_tau,
                                       void* workspace, size_t workspace_bytes) {
    using namespace dwa;
    int rc = check_bwd(dims, use_ivf);
    if (rc) return rc;
    const DwaRetrieveDims& d = *dims;
    if (!z || !W_Q || !aspect_weights || !part2_sum || !g_z || !g_W_Q || !g_aspect_weights || !g_tau)
        return fail(DWA_ERR_INVALID_ARG, "a required pointer is NULL");
    const BwdWorkspace w = carve_bwd(workspace, d, use_ivf != 0);
    if (!workspace || reinterpret_cast<uintptr_t>(workspace) % 256 != 0 || workspace_bytes < w.bytes)
        return fail(DWA_ERR_WORKSPACE, "workspace: dwa_retrieve_bwd_local_workspace_bytes, 256-byte aligned");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int cols = d.S * d.d_k;
    // the raw queries again (this phase needs no rows, so an empty rank runs it too)
    const dim3 gq((cols + kProjRows - 1) / kProjRows, (d.B + kProjQ - 1) / kProjQ);
    if (d.z_dtype == DWA_BF16)
        launch_pdl(query_proj_kernel<__nv_bfloat16>, gq, kProjThreads, 0, st, static_cast<const __nv_bfloat16*>(z),
                   W_Q, d.B, cols, d.d_A, w.f.q);
    else
        launch_pdl(query_proj_kernel<float>, gq, kProjThreads, 0, st, static_cast<const float*>(z), W_Q, d.B, cols,
                   d.d_A, w.f.q);
    DWA_LAUNCH_CHECK("query_proj_kernel");
    ++g_launches_total;
    const int qthreads = (d.d_k + 31) / 32 * 32;
    launch_pdl(query_grad_kernel, dim3(d.B, d.S), qthreads, 0, st, part2_sum, 1, d.B, 0, cols + 1, w.f.q,
               aspect_weights, d.S, d.d_k, w.gq, w.gw_part);
    DWA_LAUNCH_CHECK("query_grad_kernel");
    const int nchunk_o = (cols + kGradRowsPerCta - 1) / kGradRowsPerCta;
    const size_t gsh = static_cast<size_t>(d.B) * kGradRowsPerCta * sizeof(float);
    if (gsh > 48 * 1024) return fail(DWA_ERR_UNSUPPORTED, "retrieval VJP: B too large for the W_Q gradient");
    const dim3 gw((d.d_A + 127) / 128, nchunk_o);
    if (d.z_dtype == DWA_BF16)
        launch_pdl(wq_grad_kernel<__nv_bfloat16>, gw, 128, gsh, st, w.gq, static_cast<const __nv_bfloat16*>(z), W_Q,
                   d.B, cols, d.d_A, g_W_Q, w.gz_part);
    else
        launch_pdl(wq_grad_kernel<float>, gw, 128, gsh, st, w.gq, static_cast<const float*>(z), W_Q, d.B, cols,
                   d.d_A, g_W_Q, w.gz_part);
    DWA_LAUNCH_CHECK("wq_grad_kernel");
    const int64_t nz = static_cast<int64_t>(d.B) * d.d_A;
    launch_pdl(query_grad_finish_kernel, static_cast<unsigned>((nz + 255) / 256), 256, 0, st, w.gz_part, nchunk_o, d.B,
               d.d_A, w.gw_part, aspect_weights, d.S, part2_sum + cols, cols + 1, g_z, g_aspect_weights, g_tau);
    DWA_LAUNCH_CHECK("query_grad_finish_kernel");
    g_launches_total += 3;
    return DWA_OK;
}
