// DWA multi-aspect IVF retrieval on B200 (replaces src/dwa/retrieval.py:48-159).
//
//   query    qw[b,s,:] = softmax(aspect_weights)_s * normalize(W_Q[s] z[b])   (:64-69)
//   coarse   c_score[b,c] = sum_s qw[b,s] . c[s,c] / (|c[s,c]| + 1e-8)       (:85-89)
//   top-m    the m best lists per query, ties to the lower list index          (:90-91)
//   fine     s_i over the rows of the probed lists, candidate order =
//            list rank, then row (:94-106); lists are CSR ranges so unequal
//            (Zipf) lists work; the reference's equal lists are one case.
//   soft     s_full over every row + softmax(s_full / T) (:114-119), two passes
//   select   radix top-k of s_i on (score desc, pool row asc) + warmup softmax
//            or sigmoid-gated weights (:143-156)
//
// Every score, fine or full, goes through row_scores(): the same operations in
// the same order, so a row's fine score and its full score are bit-identical
// and the selection may read them from the full pass when soft_full is on.
// All scoring is bound by HBM reads of the fp32 key cache.
#include <algorithm>
#include <atomic>
#include <mutex>

#include "dwa_common.cuh"

namespace dwa {

extern std::atomic<uint64_t> g_launches_total;

constexpr int kMaxK = 256;  // top-k / top-m capacity of the block selection

// ------------------------------------------------------------- scoring -----
// sc[q] = sum_s (qw[q][s] . key_s) / (sqrt(|key_s|^2) + 1e-8)   for one row.
template <int NB>
__device__ __forceinline__ void row_scores(const float* __restrict__ keys, int64_t N, int S,
                                           int d_k, int64_t row, const float* qw, int nb,
                                           float* sc) {
#pragma unroll
    for (int q = 0; q < NB; ++q) sc[q] = 0.f;
    for (int s = 0; s < S; ++s) {
        const float* kp = keys + (static_cast<int64_t>(s) * N + row) * d_k;
        float dot[NB];
#pragma unroll
        for (int q = 0; q < NB; ++q) dot[q] = 0.f;
        float nrm = 0.f;
        if ((d_k & 3) == 0) {
            for (int d = 0; d < d_k; d += 4) {
                const float4 kv = __ldg(reinterpret_cast<const float4*>(kp + d));
                nrm = fmaf(kv.x, kv.x, nrm);
                nrm = fmaf(kv.y, kv.y, nrm);
                nrm = fmaf(kv.z, kv.z, nrm);
                nrm = fmaf(kv.w, kv.w, nrm);
#pragma unroll
                for (int q = 0; q < NB; ++q) {
                    if (q < nb) {
                        const float* qq = qw + (q * S + s) * d_k + d;
                        dot[q] = fmaf(kv.x, qq[0], dot[q]);
                        dot[q] = fmaf(kv.y, qq[1], dot[q]);
                        dot[q] = fmaf(kv.z, qq[2], dot[q]);
                        dot[q] = fmaf(kv.w, qq[3], dot[q]);
                    }
                }
            }
        } else {
            for (int d = 0; d < d_k; ++d) {
                const float x = __ldg(kp + d);
                nrm = fmaf(x, x, nrm);
#pragma unroll
                for (int q = 0; q < NB; ++q)
                    if (q < nb) dot[q] = fmaf(x, qw[(q * S + s) * d_k + d], dot[q]);
            }
        }
        const float den = sqrtf(nrm) + 1e-8f;
#pragma unroll
        for (int q = 0; q < NB; ++q) sc[q] += dot[q] / den;
    }
}

__device__ __forceinline__ uint32_t float_ord(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
// Larger key = better: score descending, then tie (row / list index) ascending.
__device__ __forceinline__ uint64_t make_key(float score, uint32_t tie) {
    return (static_cast<uint64_t>(float_ord(score)) << 32) | (0xFFFFFFFFu - tie);
}

__device__ __forceinline__ float block_reduce(float v, bool is_max, float* sh) {
    v = is_max ? warp_max(v) : warp_sum(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (l == 0) sh[w] = v;
    __syncthreads();
    if (w == 0) {
        float x = l < nw ? sh[l] : (is_max ? -INFINITY : 0.f);
        x = is_max ? warp_max(x) : warp_sum(x);
        if (l == 0) sh[32] = x;
    }
    __syncthreads();
    return sh[32];
}

// Selects the min(k, n) largest keys of key_at(0..n) into sel_key/sel_pos,
// sorted descending.  MSB-first radix select (8 bits per pass) on the 64-bit
// keys, stopping as soon as the boundary bucket is taken whole, then a
// bitonic sort of the winners.  Keys must be distinct.
template <class KeyAt>
__device__ int block_topk(int64_t n, int k, const KeyAt& key_at, uint64_t* sel_key,
                          int64_t* sel_pos) {
    __shared__ unsigned hist[256];
    __shared__ uint64_t s_prefix;
    __shared__ int s_kleft, s_done, s_count;
    const int tid = threadIdx.x, nt = blockDim.x;
    const int kk = static_cast<int>(n < k ? n : k);
    if (kk <= 0) return 0;
    uint64_t prefix = 0, mask = 0;
    int kleft = kk;
    for (int pass = 0; pass < 8; ++pass) {
        const int shift = 56 - 8 * pass;
        for (int i = tid; i < 256; i += nt) hist[i] = 0;
        __syncthreads();
        for (int64_t i = tid; i < n; i += nt) {
            const uint64_t key = key_at(i);
            if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 0xFF], 1u);
        }
        __syncthreads();
        if (tid == 0) {
            int acc = 0, dsel = 0;
            for (int dg = 255; dg >= 0; --dg) {
                if (acc + static_cast<int>(hist[dg]) >= kleft) { dsel = dg; break; }
                acc += static_cast<int>(hist[dg]);
            }
            s_kleft = kleft - acc;
            s_done = (static_cast<int>(hist[dsel]) == kleft - acc);
            s_prefix = prefix | (static_cast<uint64_t>(dsel) << shift);
        }
        __syncthreads();
        prefix = s_prefix;
        mask |= 0xFFull << shift;
        kleft = s_kleft;
        const int done = s_done;
        __syncthreads();
        if (done) break;
    }
    if (tid == 0) s_count = 0;
    __syncthreads();
    for (int64_t i = tid; i < n; i += nt) {
        const uint64_t key = key_at(i);
        if ((key & mask) >= prefix) {
            const int slot = atomicAdd(&s_count, 1);
            if (slot < kMaxK) { sel_key[slot] = key; sel_pos[slot] = i; }
        }
    }
    __syncthreads();
    int P = 1;
    while (P < kk) P <<= 1;
    for (int i = kk + tid; i < P; i += nt) { sel_key[i] = 0; sel_pos[i] = -1; }
    __syncthreads();
    for (int size = 2; size <= P; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = tid; i < P; i += nt) {
                const int j = i ^ stride;
                if (j > i) {
                    const bool desc = (i & size) == 0;
                    const uint64_t a = sel_key[i], c = sel_key[j];
                    if ((a < c) == desc) {
                        sel_key[i] = c; sel_key[j] = a;
                        const int64_t t = sel_pos[i]; sel_pos[i] = sel_pos[j]; sel_pos[j] = t;
                    }
                }
            }
            __syncthreads();
        }
    }
    return kk;
}

// --------------------------------------------------------------- kernels ---
template <class ZT>
__global__ void query_kernel(const ZT* __restrict__ z, const float* __restrict__ W_Q,
                             const float* __restrict__ aspect_w, int S, int d_k, int d_A,
                             float* __restrict__ qw) {
    extern __shared__ float sh[];
    float* zs = sh;        // [d_A]
    float* q = sh + d_A;   // [S*d_k]
    const int b = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (int i = threadIdx.x; i < d_A; i += blockDim.x)
        zs[i] = Elem<ZT>::to_f(z[static_cast<int64_t>(b) * d_A + i]);
    __syncthreads();
    for (int o = warp; o < S * d_k; o += nw) {
        const float* w = W_Q + static_cast<int64_t>(o) * d_A;
        float acc = 0.f;
        for (int i = lane; i < d_A; i += 32) acc = fmaf(w[i], zs[i], acc);
        acc = warp_sum(acc);
        if (lane == 0) q[o] = acc;
    }
    __syncthreads();
    for (int s = warp; s < S; s += nw) {
        float ss = 0.f;
        for (int d = lane; d < d_k; d += 32) ss = fmaf(q[s * d_k + d], q[s * d_k + d], ss);
        ss = warp_sum(ss);
        const float inv_den = 1.f / (sqrtf(ss) + 1e-8f);
        float mx = -INFINITY;
        for (int t = 0; t < S; ++t) mx = fmaxf(mx, aspect_w[t]);
        float den = 0.f;
        for (int t = 0; t < S; ++t) den += expf(aspect_w[t] - mx);
        const float ws = expf(aspect_w[s] - mx) / den;
        for (int d = lane; d < d_k; d += 32)
            qw[(static_cast<int64_t>(b) * S + s) * d_k + d] = (q[s * d_k + d] * inv_den) * ws;
    }
}

__global__ void coarse_kernel(const float* __restrict__ qw, const float* __restrict__ centroids,
                              int S, int d_k, int C, float* __restrict__ c_score) {
    extern __shared__ float qs[];
    const int b = blockIdx.y;
    for (int i = threadIdx.x; i < S * d_k; i += blockDim.x)
        qs[i] = qw[static_cast<int64_t>(b) * S * d_k + i];
    __syncthreads();
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= C) return;
    float sc;
    row_scores<1>(centroids, C, S, d_k, c, qs, 1, &sc);
    c_score[static_cast<int64_t>(b) * C + c] = sc;
}

__global__ void topm_kernel(const float* __restrict__ c_score, int C, int m,
                            const int64_t* __restrict__ list_off, int64_t N, int max_list,
                            int32_t* __restrict__ top_clusters, int64_t* __restrict__ probe_lo,
                            int64_t* __restrict__ cand_base, uint32_t* status) {
    __shared__ uint64_t sel_key[kMaxK];
    __shared__ int64_t sel_pos[kMaxK];
    const int b = blockIdx.x;
    const float* cs = c_score + static_cast<int64_t>(b) * C;
    auto key_at = [&](int64_t i) { return make_key(cs[i], static_cast<uint32_t>(i)); };
    const int got = block_topk(C, m, key_at, sel_key, sel_pos);
    if (threadIdx.x == 0) {
        int64_t acc = 0;
        for (int j = 0; j < m; ++j) {
            const int c = j < got ? static_cast<int>(sel_pos[j]) : 0;
            int64_t lo = list_off[c], hi = list_off[c + 1];
            if (lo < 0 || hi < lo || hi > N) { raise_status(status, DWA_STATUS_BAD_LIST); lo = hi = 0; }
            int64_t sz = hi - lo;
            if (sz > max_list) { raise_status(status, DWA_STATUS_LIST_OVERFLOW); sz = max_list; }
            top_clusters[static_cast<int64_t>(b) * m + j] = c;
            probe_lo[static_cast<int64_t>(b) * (m + 1) + j] = lo;
            cand_base[static_cast<int64_t>(b) * (m + 1) + j] = acc;
            acc += sz;
        }
        probe_lo[static_cast<int64_t>(b) * (m + 1) + m] = 0;
        cand_base[static_cast<int64_t>(b) * (m + 1) + m] = acc;
    }
}

__global__ void fine_kernel(const float* __restrict__ qw, const float* __restrict__ keys, int64_t N,
                            int S, int d_k, int m, const int64_t* __restrict__ probe_lo,
                            const int64_t* __restrict__ cand_base, int64_t K_cap,
                            float* __restrict__ scores) {
    extern __shared__ float qs[];
    const int b = blockIdx.z, j = blockIdx.y;
    for (int i = threadIdx.x; i < S * d_k; i += blockDim.x)
        qs[i] = qw[static_cast<int64_t>(b) * S * d_k + i];
    __syncthreads();
    const int64_t* cb = cand_base + static_cast<int64_t>(b) * (m + 1);
    const int64_t base = cb[j], sz = cb[j + 1] - cb[j];
    const int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (r >= sz) return;
    const int64_t row = probe_lo[static_cast<int64_t>(b) * (m + 1) + j] + r;
    float sc;
    row_scores<1>(keys, N, S, d_k, row, qs, 1, &sc);
    scores[static_cast<int64_t>(b) * K_cap + base + r] = sc;
}

// Full-pool scores for up to NB queries at a time; writes raw s_full and per
// block (max, sum exp) of s/T for the softmax.
template <int NB>
__global__ void full_scores_kernel(const float* __restrict__ qw, const float* __restrict__ keys,
                                   int64_t N, int S, int d_k, int B, float T,
                                   float* __restrict__ sfull, float* __restrict__ partial) {
    extern __shared__ float qs[];  // [NB][S][d_k]
    __shared__ float red[33];
    const int64_t row = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int nblk = gridDim.x;
    for (int b0 = 0; b0 < B; b0 += NB) {
        const int nb = min(NB, B - b0);
        __syncthreads();
        for (int i = threadIdx.x; i < nb * S * d_k; i += blockDim.x)
            qs[i] = qw[static_cast<int64_t>(b0) * S * d_k + i];
        __syncthreads();
        float sc[NB];
        if (row < N) row_scores<NB>(keys, N, S, d_k, row, qs, nb, sc);
        for (int q = 0; q < nb; ++q) {
            float x = -INFINITY;
            if (row < N) {
                sfull[static_cast<int64_t>(b0 + q) * N + row] = sc[q];
                x = sc[q] / T;
            }
            const float mx = block_reduce(x, true, red);
            const float e = row < N ? expf(x - mx) : 0.f;
            const float zs = block_reduce(e, false, red);
            if (threadIdx.x == 0) {
                partial[(static_cast<int64_t>(b0 + q) * nblk + blockIdx.x) * 2] = mx;
                partial[(static_cast<int64_t>(b0 + q) * nblk + blockIdx.x) * 2 + 1] = zs;
            }
        }
    }
}

__global__ void softmax_stats_kernel(const float* __restrict__ partial, int nblk,
                                     float* __restrict__ stats) {
    __shared__ float red[33];
    const int b = blockIdx.x;
    const float* p = partial + static_cast<int64_t>(b) * nblk * 2;
    float mx = -INFINITY;
    for (int i = threadIdx.x; i < nblk; i += blockDim.x) mx = fmaxf(mx, p[2 * i]);
    mx = block_reduce(mx, true, red);
    float z = 0.f;
    for (int i = threadIdx.x; i < nblk; i += blockDim.x) z += p[2 * i + 1] * expf(p[2 * i] - mx);
    z = block_reduce(z, false, red);
    if (threadIdx.x == 0) { stats[2 * b] = mx; stats[2 * b + 1] = z; }
}

__global__ void softmax_apply_kernel(float* __restrict__ sfull, int64_t N, float T,
                                     const float* __restrict__ stats) {
    const int b = blockIdx.y;
    const float mx = stats[2 * b], z = stats[2 * b + 1];
    float* p = sfull + static_cast<int64_t>(b) * N;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < N;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        p[i] = expf(p[i] / T - mx) / z;
}

struct SelectArgs {
    const float* scores;     // [B, K_cap] fine scores by candidate position, or
    const float* sfull;      // [B, N] raw full scores by pool row (when non-null)
    const int64_t* probe_lo; // [B, m+1]
    const int64_t* cand_base;
    int m;
    int64_t K_cap, N;
    int k;
    float T;
    int is_warmup;
    const float* lambda_val;
    const float* tau;
    float* alphas;
    int32_t* indices;
    uint32_t* status;
};

__device__ __forceinline__ float gate_raw(float s, float lam, float tau, float T) {
    const float g = 1.f / (1.f + expf(-(lam * (s - tau))));
    return g * expf(s / T);
}

__global__ void select_kernel(SelectArgs a) {
    __shared__ uint64_t sel_key[kMaxK];
    __shared__ int64_t sel_pos[kMaxK];
    __shared__ int64_t s_lo[kMaxK + 1], s_base[kMaxK + 1];
    __shared__ float red[33];
    const int b = blockIdx.x;
    for (int j = threadIdx.x; j <= a.m; j += blockDim.x) {
        s_lo[j] = a.probe_lo[static_cast<int64_t>(b) * (a.m + 1) + j];
        s_base[j] = a.cand_base[static_cast<int64_t>(b) * (a.m + 1) + j];
    }
    __syncthreads();
    const int64_t n = s_base[a.m];
    const float lam = __ldg(a.lambda_val), tau = __ldg(a.tau), T = a.T;
    const bool gate = !a.is_warmup;
    const bool rank_raw = gate && lam < 0.f;  // raw is monotone in s only for lambda >= 0
    auto locate = [&](int64_t pos, int64_t* row) {
        int lo = 0, hi = a.m - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (s_base[mid] <= pos) lo = mid; else hi = mid - 1;
        }
        *row = s_lo[lo] + (pos - s_base[lo]);
        return a.sfull ? a.sfull[static_cast<int64_t>(b) * a.N + *row]
                       : a.scores[static_cast<int64_t>(b) * a.K_cap + pos];
    };
    auto key_at = [&](int64_t pos) {
        int64_t row;
        const float s = locate(pos, &row);
        return make_key(rank_raw ? gate_raw(s, lam, tau, T) : s, static_cast<uint32_t>(row));
    };
    float Z = 0.f;
    if (gate) {
        float acc = 0.f;
        for (int64_t p = threadIdx.x; p < n; p += blockDim.x) {
            int64_t row;
            acc += gate_raw(locate(p, &row), lam, tau, T);
        }
        Z = block_reduce(acc, false, red);
    }
    const int got = block_topk(n, a.k, key_at, sel_key, sel_pos);
    if (threadIdx.x == 0) {
        if (got < a.k) raise_status(a.status, DWA_STATUS_FEW_CANDIDATES);
        float sv[kMaxK];
        int64_t rows[kMaxK];
        for (int i = 0; i < got; ++i) sv[i] = locate(sel_pos[i], &rows[i]);
        float* al = a.alphas + static_cast<int64_t>(b) * a.k;
        int32_t* ix = a.indices + static_cast<int64_t>(b) * a.k;
        if (!gate) {
            const float mx = got > 0 ? sv[0] / T : 0.f;
            float den = 0.f;
            for (int i = 0; i < got; ++i) den += expf(sv[i] / T - mx);
            for (int i = 0; i < got; ++i) al[i] = expf(sv[i] / T - mx) / den;
        } else {
            float tot = 0.f;
            for (int i = 0; i < got; ++i) {
                sv[i] = gate_raw(sv[i], lam, tau, T) / (Z + 1e-8f);
                tot += sv[i];
            }
            for (int i = 0; i < got; ++i) al[i] = sv[i] / (tot + 1e-8f);
        }
        for (int i = 0; i < got; ++i) ix[i] = static_cast<int32_t>(rows[i]);
        for (int i = got; i < a.k; ++i) { al[i] = 0.f; ix[i] = got > 0 ? ix[0] : 0; }
    }
}

__global__ void full_probe_kernel(int B, int64_t N, int64_t* probe_lo, int64_t* cand_base) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    probe_lo[2 * b] = 0; probe_lo[2 * b + 1] = 0;
    cand_base[2 * b] = 0; cand_base[2 * b + 1] = N;
}

template <class T>
__global__ void seq_mean_kernel(const T* __restrict__ h, int T_, int d, float* __restrict__ z) {
    const int b = blockIdx.y;
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= d) return;
    const T* p = h + static_cast<int64_t>(b) * T_ * d + j;
    float acc = 0.f;
    for (int t = 0; t < T_; ++t) acc += Elem<T>::to_f(p[static_cast<int64_t>(t) * d]);
    z[static_cast<int64_t>(b) * d + j] = acc / static_cast<float>(T_);
}

// ------------------------------------------------------------------ host ---
struct RetWorkspace {
    uint32_t* status;
    float* qw;
    float* c_score;
    int32_t* topc;
    int64_t* probe_lo;
    int64_t* cand_base;
    float* scores;
    float* sfull;
    float* partial;
    float* stats;
    int m_eff;
    int64_t K_cap;
    int nblk;
    size_t bytes;
};

constexpr int kFullRows = 256;

static RetWorkspace carve_ret(void* base, const DwaRetrieveDims& d, bool ivf, bool want_sf) {
    Carver c(base);
    RetWorkspace w{};
    w.status = static_cast<uint32_t*>(base);
    w.m_eff = ivf ? (d.m < d.C ? d.m : d.C) : 1;
    w.K_cap = ivf ? static_cast<int64_t>(w.m_eff) * d.max_list : d.N;
    w.nblk = static_cast<int>((d.N + kFullRows - 1) / kFullRows);
    w.qw = c.take<float>(static_cast<size_t>(d.B) * d.S * d.d_k);
    w.probe_lo = c.take<int64_t>(static_cast<size_t>(d.B) * (w.m_eff + 1));
    w.cand_base = c.take<int64_t>(static_cast<size_t>(d.B) * (w.m_eff + 1));
    if (ivf) {
        w.c_score = c.take<float>(static_cast<size_t>(d.B) * d.C);
        w.topc = c.take<int32_t>(static_cast<size_t>(d.B) * w.m_eff);
        if (!want_sf) w.scores = c.take<float>(static_cast<size_t>(d.B) * w.K_cap);
    }
    const bool full_pass = !ivf || want_sf;
    if (!ivf && !want_sf) w.sfull = c.take<float>(static_cast<size_t>(d.B) * d.N);
    if (full_pass) {
        w.partial = c.take<float>(static_cast<size_t>(d.B) * w.nblk * 2);
        w.stats = c.take<float>(static_cast<size_t>(d.B) * 2);
    }
    w.bytes = c.bytes();
    return w;
}

static int check_ret(const DwaRetrieveDims* d, int use_ivf) {
    if (!d) return fail(DWA_ERR_INVALID_ARG, "dims is NULL");
    if (d->B <= 0 || d->S <= 0 || d->d_k <= 0 || d->d_A <= 0 || d->N <= 0 || d->k <= 0)
        return fail(DWA_ERR_INVALID_ARG, "B, S, d_k, d_A, N, k must be positive");
    if (d->k > kMaxK) return fail(DWA_ERR_UNSUPPORTED, "k > 256");
    if (d->N >= (int64_t(1) << 31)) return fail(DWA_ERR_UNSUPPORTED, "N >= 2^31");
    if (!(d->T > 0.f)) return fail(DWA_ERR_INVALID_ARG, "temperature T must be > 0");
    if (d->z_dtype != DWA_F32 && d->z_dtype != DWA_BF16)
        return fail(DWA_ERR_INVALID_ARG, "z_dtype must be DWA_F32 or DWA_BF16");
    if (use_ivf) {
        if (d->C <= 0 || d->m <= 0 || d->max_list <= 0)
            return fail(DWA_ERR_INVALID_ARG, "C, m, max_list must be positive with IVF");
        if ((d->m < d->C ? d->m : d->C) > kMaxK) return fail(DWA_ERR_UNSUPPORTED, "m > 256");
    }
    const size_t qbytes = static_cast<size_t>(d->S) * d->d_k * sizeof(float);
    if (qbytes * 8 > 48 * 1024 || (d->d_A + d->S * d->d_k) * sizeof(float) > 48 * 1024)
        return fail(DWA_ERR_UNSUPPORTED, "S*d_k or d_A too large for shared memory staging");
    return DWA_OK;
}

}  // namespace dwa

using namespace dwa;

extern "C" size_t dwa_retrieve_workspace_bytes(const DwaRetrieveDims* dims, int use_ivf,
                                               int want_soft_full) {
    if (check_ret(dims, use_ivf)) return 0;
    return carve_ret(nullptr, *dims, use_ivf != 0, want_soft_full != 0).bytes;
}

extern "C" int dwa_retrieve(void* stream, const DwaRetrieveDims* dims, int use_ivf, int is_warmup,
                            const float* lambda_val, const void* z, const float* W_Q,
                            const float* aspect_weights, const float* tau, const float* centroids,
                            const int64_t* list_offsets, const float* pool_keys, float* alphas,
                            int32_t* indices, float* soft_full, void* workspace,
                            size_t workspace_bytes) {
    int rc = check_ret(dims, use_ivf);
    if (rc) return rc;
    const DwaRetrieveDims& d = *dims;
    const bool ivf = use_ivf != 0, want_sf = soft_full != nullptr;
    if (!lambda_val || !z || !W_Q || !aspect_weights || !tau || !pool_keys || !alphas || !indices)
        return fail(DWA_ERR_INVALID_ARG, "a required pointer is NULL");
    if (ivf && (!centroids || !list_offsets))
        return fail(DWA_ERR_INVALID_ARG, "IVF needs centroids and list_offsets");
    const RetWorkspace w = carve_ret(workspace, d, ivf, want_sf);
    if (!workspace || reinterpret_cast<uintptr_t>(workspace) % 256 != 0)
        return fail(DWA_ERR_WORKSPACE, "workspace must be non-NULL and 256-byte aligned");
    if (workspace_bytes < w.bytes)
        return fail(DWA_ERR_WORKSPACE, "workspace too small: need " + std::to_string(w.bytes));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const size_t qsh = static_cast<size_t>(d.S) * d.d_k * sizeof(float);

    // 1. aspect queries
    const size_t zsh = (static_cast<size_t>(d.d_A) + static_cast<size_t>(d.S) * d.d_k) * sizeof(float);
    if (d.z_dtype == DWA_BF16)
        DWA_TIMED("query", st, query_kernel<__nv_bfloat16><<<d.B, 256, zsh, st>>>(
                                     static_cast<const __nv_bfloat16*>(z), W_Q, aspect_weights,
                                     d.S, d.d_k, d.d_A, w.qw));
    else
        DWA_TIMED("query", st, query_kernel<float><<<d.B, 256, zsh, st>>>(
                                     static_cast<const float*>(z), W_Q, aspect_weights, d.S,
                                     d.d_k, d.d_A, w.qw));
    DWA_LAUNCH_CHECK("query_kernel");
    ++g_launches_total;

    float* sfull = want_sf ? soft_full : w.sfull;
    if (ivf) {
        // 2. coarse scores + top-m lists + candidate ranges
        dim3 gc((d.C + 127) / 128, d.B);
        DWA_TIMED("coarse", st, coarse_kernel<<<gc, 128, qsh, st>>>(w.qw, centroids, d.S, d.d_k,
                                                                    d.C, w.c_score));
        DWA_LAUNCH_CHECK("coarse_kernel");
        DWA_TIMED("topm", st, topm_kernel<<<d.B, 256, 0, st>>>(w.c_score, d.C, w.m_eff, list_offsets,
                                                               d.N, d.max_list, w.topc,
                                                               w.probe_lo, w.cand_base, w.status));
        DWA_LAUNCH_CHECK("topm_kernel");
        g_launches_total += 2;
    } else {
        full_probe_kernel<<<(d.B + 127) / 128, 128, 0, st>>>(d.B, d.N, w.probe_lo, w.cand_base);
        DWA_LAUNCH_CHECK("full_probe_kernel");
        ++g_launches_total;
    }
    // 3. full-pool raw scores (soft_full or full search)
    if (!ivf || want_sf) {
        constexpr int NB = 8;
        DWA_TIMED("full_scores", st,
                  full_scores_kernel<NB><<<w.nblk, kFullRows, NB * qsh, st>>>(
                      w.qw, pool_keys, d.N, d.S, d.d_k, d.B, d.T, sfull, w.partial));
        DWA_LAUNCH_CHECK("full_scores_kernel");
        ++g_launches_total;
    }
    // 4. fine scores of the probed lists (read from the full pass when it ran)
    if (ivf && !want_sf) {
        dim3 gf(static_cast<unsigned>((d.max_list + 255) / 256), w.m_eff, d.B);
        DWA_TIMED("fine", st, fine_kernel<<<gf, 256, qsh, st>>>(w.qw, pool_keys, d.N, d.S, d.d_k,
                                                                w.m_eff, w.probe_lo, w.cand_base,
                                                                w.K_cap, w.scores));
        DWA_LAUNCH_CHECK("fine_kernel");
        ++g_launches_total;
    }
    // 5. selection
    SelectArgs sa;
    sa.scores = w.scores;
    sa.sfull = (ivf && !want_sf) ? nullptr : sfull;
    sa.probe_lo = w.probe_lo;
    sa.cand_base = w.cand_base;
    sa.m = w.m_eff;
    sa.K_cap = w.K_cap;
    sa.N = d.N;
    sa.k = d.k;
    sa.T = d.T;
    sa.is_warmup = is_warmup;
    sa.lambda_val = lambda_val;
    sa.tau = tau;
    sa.alphas = alphas;
    sa.indices = indices;
    sa.status = w.status;
    DWA_TIMED("select", st, select_kernel<<<d.B, 512, 0, st>>>(sa));
    DWA_LAUNCH_CHECK("select_kernel");
    ++g_launches_total;
    // 6. normalise soft_full in place
    if (want_sf) {
        DWA_TIMED("softmax_stats", st,
                  softmax_stats_kernel<<<d.B, 256, 0, st>>>(w.partial, w.nblk, w.stats));
        DWA_LAUNCH_CHECK("softmax_stats_kernel");
        dim3 ga(static_cast<unsigned>(std::min<int64_t>((d.N + 255) / 256, 1184)), d.B);
        DWA_TIMED("softmax_apply", st,
                  softmax_apply_kernel<<<ga, 256, 0, st>>>(soft_full, d.N, d.T, w.stats));
        DWA_LAUNCH_CHECK("softmax_apply_kernel");
        g_launches_total += 2;
    }
    return DWA_OK;
}

extern "C" int dwa_sequence_mean(void* stream, int B, int T, int d, int dtype, const void* h_A,
                                 float* z) {
    if (B <= 0 || T <= 0 || d <= 0 || !h_A || !z)
        return fail(DWA_ERR_INVALID_ARG, "dwa_sequence_mean: bad sizes or NULL pointer");
    if (dtype != DWA_F32 && dtype != DWA_BF16) return fail(DWA_ERR_INVALID_ARG, "bad dtype");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    dim3 g((d + 255) / 256, B);
    if (dtype == DWA_BF16)
        DWA_TIMED("seq_mean", st, seq_mean_kernel<__nv_bfloat16><<<g, 256, 0, st>>>(
                                      static_cast<const __nv_bfloat16*>(h_A), T, d, z));
    else
        DWA_TIMED("seq_mean", st,
                  seq_mean_kernel<float><<<g, 256, 0, st>>>(static_cast<const float*>(h_A), T, d, z));
    DWA_LAUNCH_CHECK("seq_mean_kernel");
    ++g_launches_total;
    return DWA_OK;
}

// ---------------------------------------------------- allocation-free ---
// dwa_retrieve_noalloc runs the retrieval above with its scratch taken from
// this file-scope device array instead of a caller workspace.  Every GPU that
// loads libdwa keeps these 8 MiB until the process exits.  In host code the
// name g_retrieve_scratch is only a stand-in for the symbol, not a device
// address: the address a kernel may use comes from cudaGetSymbolAddress, once
// per device, with that device current.
namespace dwa {
constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;
static __device__ __align__(256) unsigned char g_retrieve_scratch[kNoAllocScratchBytes];

static std::mutex g_scratch_mu;
static void* g_scratch_addr[64];

static int scratch_address(void** out) {
    int dev = 0;
    DWA_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(DWA_ERR_UNSUPPORTED, "device ordinal above 63");
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (!g_scratch_addr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_retrieve_scratch);
        if (e != cudaSuccess || p == nullptr)
            return fail(DWA_ERR_CUDA, std::string("cudaGetSymbolAddress(g_retrieve_scratch): ") +
                                          cudaGetErrorString(e));
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return DWA_OK;
}
}  // namespace dwa

extern "C" int dwa_retrieve_noalloc(void* stream, const DwaRetrieveDims* dims, int use_ivf,
                                    int is_warmup, const float* lambda_val, const void* z,
                                    const float* W_Q, const float* aspect_weights,
                                    const float* tau, const float* centroids,
                                    const int64_t* list_offsets, const float* pool_keys,
                                    float* alphas, int32_t* indices, float* soft_full) {
    int rc = check_ret(dims, use_ivf);
    if (rc) return rc;
    const size_t need = carve_ret(nullptr, *dims, use_ivf != 0, soft_full != nullptr).bytes;
    if (need > kNoAllocScratchBytes)
        return fail(DWA_ERR_UNSUPPORTED,
                    "dwa_retrieve_noalloc: this shape needs " + std::to_string(need) +
                        " bytes of scratch but the built-in scratch holds " +
                        std::to_string(kNoAllocScratchBytes) +
                        " bytes; call dwa_retrieve with a caller workspace");
    void* scratch = nullptr;
    if ((rc = scratch_address(&scratch))) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // The scratch keeps the previous call's bytes; only the status word must
    // start at zero (every other byte is written before it is read).
    DWA_CUDA_TRY(cudaMemsetAsync(scratch, 0, 256, st));
    return dwa_retrieve(stream, dims, use_ivf, is_warmup, lambda_val, z, W_Q, aspect_weights, tau,
                        centroids, list_offsets, pool_keys, alphas, indices, soft_full, scratch,
                        kNoAllocScratchBytes);
}
