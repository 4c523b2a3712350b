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
#include <cstdlib>
#include <cstring>
#include <atomic>
#include <memory>
#include <mutex>

#include <cuda.h>

#include "dwa_common.cuh"
#include "tc_gemm.cuh"
#include "scores_scan.cuh"
#include "scores_tc.cuh"

namespace dwa {

extern std::atomic<uint64_t> g_launches_total;

constexpr int kMaxK = 256;  // top-k / top-m capacity of the block selection

// Summary of one query on one rank of a sharded call, 2k+3 floats:
//   [0, k)    scores s of the rank's top-k candidates, best first (-inf: none)
//   [k, 2k)   their global pool rows as int32 bits (-1: none)
//   [2k]      sum of raw over the rank's candidates (gate mode; 0 in warmup)
//   [2k+1]    max of s/T over the rank's rows (soft_full), [2k+2] sum exp(s/T - max)
__host__ __device__ constexpr int summary_width(int k) { return 2 * k + 3; }


// ------------------------------------------------------------- scoring -----
// sc[q] = sum_s (qw[q][s] . key_s) / (sqrt(|key_s|^2) + 1e-8)   for one row.
// DK > 0: d_k is the compile-time DK (fully unrolled, all loads of an aspect in
// flight at once); DK == 0: runtime d_k.  For a given row and query the
// operations and their order do not depend on NB, so the fine pass (NB = 1)
// and the full pass (NB > 1) give bit-identical scores.
template <int NB, int DK>
__device__ __forceinline__ void row_scores(const float* __restrict__ keys, int64_t N, int S,
                                           int d_k, int64_t row, const float* qw, int nb,
                                           float* sc) {
#pragma unroll
    for (int q = 0; q < NB; ++q) sc[q] = 0.f;
    if constexpr (DK > 0) {
        for (int s = 0; s < S; ++s) {
            const float4* kp = reinterpret_cast<const float4*>(keys + (static_cast<int64_t>(s) * N + row) * DK);
            float4 kv[DK / 4];
#pragma unroll
            for (int c = 0; c < DK / 4; ++c) kv[c] = __ldg(kp + c);
            float nrm = 0.f;
#pragma unroll
            for (int c = 0; c < DK / 4; ++c) {
                nrm = fmaf(kv[c].x, kv[c].x, nrm);
                nrm = fmaf(kv[c].y, kv[c].y, nrm);
                nrm = fmaf(kv[c].z, kv[c].z, nrm);
                nrm = fmaf(kv[c].w, kv[c].w, nrm);
            }
            const float den = sqrtf(nrm) + 1e-8f;
#pragma unroll
            for (int q = 0; q < NB; ++q) {
                if (q < nb) {
                    const float4* qq = reinterpret_cast<const float4*>(qw + (q * S + s) * DK);
                    float dot = 0.f;
#pragma unroll
                    for (int c = 0; c < DK / 4; ++c) {
                        const float4 qv = qq[c];
                        dot = fmaf(kv[c].x, qv.x, dot);
                        dot = fmaf(kv[c].y, qv.y, dot);
                        dot = fmaf(kv[c].z, qv.z, dot);
                        dot = fmaf(kv[c].w, qv.w, dot);
                    }
                    sc[q] += dot / den;
                }
            }
        }
    } else {
        for (int s = 0; s < S; ++s) {
            const float* kp = keys + (static_cast<int64_t>(s) * N + row) * d_k;
            float dot[NB];
#pragma unroll
            for (int q = 0; q < NB; ++q) dot[q] = 0.f;
            float nrm = 0.f;
            for (int d = 0; d < d_k; ++d) {
                const float x = __ldg(kp + d);
                nrm = fmaf(x, x, nrm);
#pragma unroll
                for (int q = 0; q < NB; ++q)
                    if (q < nb) dot[q] = fmaf(x, qw[(q * S + s) * d_k + d], dot[q]);
            }
            const float den = sqrtf(nrm) + 1e-8f;
#pragma unroll
            for (int q = 0; q < NB; ++q) sc[q] += dot[q] / den;
        }
    }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* tm, uint64_t* bar, int c0,
                                            int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(tc::smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(tc::smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
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
// sorted descending; keys must be distinct.  A few block-wide steps, each
// short, since the cost here is the length of the dependent chain:
//   1. the bits every key shares (block OR / AND) are known, so the radix
//      passes start at the highest bit on which keys differ;
//   2. MSB-first radix passes of 8 bits histogram the keys that still match
//      the prefix (shared-memory atomics); warp 0 finds the bucket holding the
//      k-th key.  The passes stop as soon as at most cap = max(64, kk) keys lie
//      at or above that bucket (usually after one pass);
//   3. those keys are gathered and each one's rank among them (the number of
//      larger keys) puts the top kk in order.
// With n <= cap the passes are skipped.
template <class KeyAt>
__device__ int block_topk(int64_t n, int k, const KeyAt& key_at, uint64_t* sel_key,
                          int64_t* sel_pos) {
    __shared__ unsigned hist[2][256];
    __shared__ uint64_t s_or[32], s_and[32];
    __shared__ uint64_t s_prefix[2];
    __shared__ int s_kleft[2], s_stop[2], s_count;
    __shared__ uint64_t t_key[kMaxK];
    __shared__ int64_t t_pos[kMaxK];
    const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, warp = tid >> 5;
    const int kk = static_cast<int>(n < k ? n : k);
    if (kk <= 0) return 0;
    const int cap = kk > 64 ? kk : 64;
    uint64_t prefix = 0, mask = 0;
    if (n > cap) {
        // 1. common bits
        uint64_t o = 0, a = ~0ull;
        for (int64_t i = tid; i < n; i += nt) {
            const uint64_t key = key_at(i);
            o |= key;
            a &= key;
        }
        const uint32_t o_lo = __reduce_or_sync(0xffffffffu, static_cast<uint32_t>(o));
        const uint32_t o_hi = __reduce_or_sync(0xffffffffu, static_cast<uint32_t>(o >> 32));
        const uint32_t a_lo = __reduce_and_sync(0xffffffffu, static_cast<uint32_t>(a));
        const uint32_t a_hi = __reduce_and_sync(0xffffffffu, static_cast<uint32_t>(a >> 32));
        if (lane == 0) {
            s_or[warp] = (static_cast<uint64_t>(o_hi) << 32) | o_lo;
            s_and[warp] = (static_cast<uint64_t>(a_hi) << 32) | a_lo;
        }
        for (int i = tid; i < 512; i += nt) (&hist[0][0])[i] = 0;
        __syncthreads();
        o = 0;
        a = ~0ull;
        for (int w = 0; w < (nt >> 5); ++w) {
            o |= s_or[w];
            a &= s_and[w];
        }
        // distinct keys differ somewhere (o != a); equal keys leave nothing to resolve
        int hi = o == a ? -1 : 63 - __clzll(static_cast<long long>(o ^ a));
        mask = hi < 0 ? ~0ull : hi == 63 ? 0ull : ~((2ull << hi) - 1);
        prefix = a & mask;
        int kleft = kk;
        // 2. radix passes over bits [lo, hi]; keys above the prefix: kk - kleft
        for (int pass = 0; hi >= 0; ++pass) {
            const int buf = pass & 1;
            const int lo = hi >= 7 ? hi - 7 : 0;
            const unsigned dmask = (1u << (hi - lo + 1)) - 1;
            for (int64_t i = tid; i < n; i += nt) {
                const uint64_t key = key_at(i);
                if ((key & mask) == prefix) atomicAdd(&hist[buf][static_cast<unsigned>(key >> lo) & dmask], 1u);
            }
            __syncthreads();
            for (int i = tid; i < 256; i += nt) hist[buf ^ 1][i] = 0;
            if (tid < 32) {
                // warp 0 scans the 256 buckets from the top: 8 buckets per lane
                unsigned c8[8], tot = 0;
#pragma unroll
                for (int i = 0; i < 8; ++i) { c8[i] = hist[buf][255 - (tid * 8 + i)]; tot += c8[i]; }
                unsigned incl = tot;  // inclusive prefix over lanes (lane 0 = highest buckets)
#pragma unroll
                for (int o2 = 1; o2 < 32; o2 <<= 1) {
                    const unsigned v = __shfl_up_sync(0xffffffffu, incl, o2);
                    if (tid >= o2) incl += v;
                }
                const unsigned before = incl - tot;
                const bool mine = before < static_cast<unsigned>(kleft) && incl >= static_cast<unsigned>(kleft);
                if (mine) {
                    unsigned acc = before;
                    for (int i = 0; i < 8; ++i) {
                        if (acc + c8[i] >= static_cast<unsigned>(kleft)) {
                            const int dsel = 255 - (tid * 8 + i);
                            // keys at or above the boundary bucket: (kk - kleft) + acc + c8[i]
                            s_kleft[buf] = kleft - static_cast<int>(acc);
                            s_stop[buf] = (kk - kleft) + static_cast<int>(acc + c8[i]) <= cap;
                            s_prefix[buf] = prefix | (static_cast<uint64_t>(dsel) << lo);
                            break;
                        }
                        acc += c8[i];
                    }
                }
            }
            __syncthreads();
            prefix = s_prefix[buf];
            mask |= static_cast<uint64_t>(dmask) << lo;
            kleft = s_kleft[buf];
            if (s_stop[buf]) break;
            hi = lo - 1;
        }
    }
    // 3. gather the keys at or above the threshold (at most cap of them) ...
    if (tid == 0) s_count = 0;
    __syncthreads();
    for (int64_t i = tid; i < n; i += nt) {
        const uint64_t key = key_at(i);
        if ((key & mask) >= prefix) {
            const int slot = atomicAdd(&s_count, 1);
            if (slot < kMaxK) { t_key[slot] = key; t_pos[slot] = i; }
        }
    }
    __syncthreads();
    // ... and place each by its rank among them
    const int cnt = s_count < kMaxK ? s_count : kMaxK;
    for (int t = tid; t < cnt; t += nt) {
        const uint64_t key = t_key[t];
        int r0 = 0, r1 = 0, r2 = 0, r3 = 0;
        int j = 0;
        for (; j + 4 <= cnt; j += 4) {
            r0 += t_key[j] > key;
            r1 += t_key[j + 1] > key;
            r2 += t_key[j + 2] > key;
            r3 += t_key[j + 3] > key;
        }
        for (; j < cnt; ++j) r0 += t_key[j] > key;
        const int rank = r0 + r1 + r2 + r3;
        if (rank < kk) { sel_key[rank] = key; sel_pos[rank] = t_pos[t]; }
    }
    __syncthreads();
    return kk;
}

// --------------------------------------------------------------- kernels ---
// Raw aspect queries q[b, o] = W_Q[o, :] . z[b, :] for o = s*d_k + kk
// (retrieval.py:65).  CTA (x, y) computes the kProjRows rows o of W_Q from
// x * kProjRows for the kProjQ queries from y * kProjQ: thread t takes columns
// t, t + 256, ... (kProjCols of them per batch of loads in flight), the 256
// partial dot products of an output are added by warp shuffles, then over the
// 8 warps in warp order.
// Larger batches take PR = 8 rows x PQ = 16 queries per CTA (fewer L2 re-reads
// of z and W_Q); every thread still adds its columns in the same order, so the
// outputs are bit-identical whichever tile computed them.
constexpr int kProjRows = 2, kProjQ = 8, kProjThreads = 256, kProjCols = 4;
template <class ZT, int PR = kProjRows, int PQ = kProjQ, int PC = kProjCols>
__global__ void __launch_bounds__(kProjThreads) query_proj_kernel(const ZT* __restrict__ z,
                                                                  const float* __restrict__ W_Q, int B,
                                                                  int rows, int d_A, float* __restrict__ q) {
    pdl_enter();
    constexpr int NO = PR * PQ;
    __shared__ float red[kProjThreads / 32][NO];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int o0 = blockIdx.x * PR, b0 = blockIdx.y * PQ;
    const int nr = min(PR, rows - o0), nb = min(PQ, B - b0);
    float acc[PR][PQ];
#pragma unroll
    for (int r = 0; r < PR; ++r)
#pragma unroll
        for (int j = 0; j < PQ; ++j) acc[r][j] = 0.f;
    for (int c0 = threadIdx.x; c0 < d_A; c0 += kProjThreads * PC) {
        float wv[PC][PR], zv[PC][PQ];
#pragma unroll
        for (int u = 0; u < PC; ++u) {
            const int c = c0 + u * kProjThreads;
#pragma unroll
            for (int r = 0; r < PR; ++r)
                wv[u][r] = (c < d_A && r < nr) ? __ldg(W_Q + static_cast<int64_t>(o0 + r) * d_A + c) : 0.f;
#pragma unroll
            for (int j = 0; j < PQ; ++j)
                zv[u][j] = (c < d_A && j < nb) ? Elem<ZT>::to_f(z[static_cast<int64_t>(b0 + j) * d_A + c]) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < PC; ++u)
#pragma unroll
            for (int r = 0; r < PR; ++r)
#pragma unroll
                for (int j = 0; j < PQ; ++j) acc[r][j] = fmaf(wv[u][r], zv[u][j], acc[r][j]);
    }
#pragma unroll
    for (int r = 0; r < PR; ++r)
#pragma unroll
        for (int j = 0; j < PQ; ++j) {
            const float v = warp_sum(acc[r][j]);
            if (lane == 0) red[warp][r * PQ + j] = v;
        }
    __syncthreads();
    if (threadIdx.x < NO) {
        const int r = threadIdx.x / PQ, j = threadIdx.x % PQ;
        float v = 0.f;
#pragma unroll
        for (int i = 0; i < kProjThreads / 32; ++i) v += red[i][threadIdx.x];
        if (r < nr && j < nb) q[static_cast<int64_t>(b0 + j) * rows + o0 + r] = v;
    }
}

// One aspect of one query, in place, by one warp:
// q <- softmax(aspect_weights)_s * q / (|q| + 1e-8)   (retrieval.py:66, :69).
// Shared by query_norm_kernel and the coarse top-m kernel, so both give the
// same bits.
__device__ __forceinline__ void normalize_aspect(float* q, const float* __restrict__ aspect_w, int S, int s,
                                                 int d_k) {
    const int lane = threadIdx.x & 31;
    float ss = 0.f;
    for (int d = lane; d < d_k; d += 32) ss = fmaf(q[d], q[d], ss);
    ss = warp_sum(ss);
    const float inv_den = 1.f / (sqrtf(ss) + 1e-8f);
    // the S <= 16 weights: one load per lane, then the sequential max and sum
    const float wl = lane < S ? aspect_w[lane] : 0.f;
    float mx = -INFINITY;
    for (int t = 0; t < S; ++t) mx = fmaxf(mx, __shfl_sync(0xffffffffu, wl, t));
    float den = 0.f;
    for (int t = 0; t < S; ++t) den += expf(__shfl_sync(0xffffffffu, wl, t) - mx);
    const float ws = expf(__shfl_sync(0xffffffffu, wl, s) - mx) / den;
    for (int d = lane; d < d_k; d += 32) q[d] = (q[d] * inv_den) * ws;
}

// qw[b,s,:] from the raw q[b,s,:]: one warp per aspect.
__global__ void query_norm_kernel(const float* __restrict__ q, const float* __restrict__ aspect_w, int S,
                                  int d_k, float* __restrict__ qw) {
    pdl_enter();
    const int b = blockIdx.x, s = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (s >= S) return;
    const int64_t off = (static_cast<int64_t>(b) * S + s) * d_k;
    for (int d = lane; d < d_k; d += 32) qw[off + d] = q[off + d];
    __syncwarp();
    normalize_aspect(qw + off, aspect_w, S, s, d_k);
}

// One thread per (centroid, aspect): t = (qw[b,s] . c[s,c]) / (|c[s,c]| + 1e-8)
// with row_scores' operation order; the S terms of a centroid are then added
// in aspect order (the same sum row_scores forms).
template <int DK>
__global__ void __launch_bounds__(1024) coarse_kernel(const float* __restrict__ qw,
                                                      const float* __restrict__ centroids, int S,
                                                      int d_k, int C, float* __restrict__ c_score) {
    pdl_enter();
    extern __shared__ __align__(16) float qs[];   // [S*d_k] then terms [S][64]
    float* terms = qs + S * d_k;
    const int b = blockIdx.y;
    for (int i = threadIdx.x; i < S * d_k; i += blockDim.x)
        qs[i] = qw[static_cast<int64_t>(b) * S * d_k + i];
    __syncthreads();
    const int cl = threadIdx.x & 63, s = threadIdx.x >> 6;
    const int c = blockIdx.x * 64 + cl;
    if (c < C && s < S) {
        const float* kp = centroids + (static_cast<int64_t>(s) * C + c) * d_k;
        const float* qq = qs + s * d_k;
        float dot = 0.f, nrm = 0.f;
        if constexpr (DK > 0) {
            float4 kv[DK / 4];
#pragma unroll
            for (int i = 0; i < DK / 4; ++i) kv[i] = __ldg(reinterpret_cast<const float4*>(kp) + i);
#pragma unroll
            for (int i = 0; i < DK / 4; ++i) {
                nrm = fmaf(kv[i].x, kv[i].x, nrm);
                nrm = fmaf(kv[i].y, kv[i].y, nrm);
                nrm = fmaf(kv[i].z, kv[i].z, nrm);
                nrm = fmaf(kv[i].w, kv[i].w, nrm);
            }
#pragma unroll
            for (int i = 0; i < DK / 4; ++i) {
                const float4 qv = reinterpret_cast<const float4*>(qq)[i];
                dot = fmaf(kv[i].x, qv.x, dot);
                dot = fmaf(kv[i].y, qv.y, dot);
                dot = fmaf(kv[i].z, qv.z, dot);
                dot = fmaf(kv[i].w, qv.w, dot);
            }
        } else {
            for (int d = 0; d < d_k; ++d) {
                const float x = __ldg(kp + d);
                nrm = fmaf(x, x, nrm);
                dot = fmaf(x, qq[d], dot);
            }
        }
        terms[s * 64 + cl] = dot / (sqrtf(nrm) + 1e-8f);
    }
    __syncthreads();
    if (s == 0 && c < C) {
        float sc = 0.f;
        for (int t = 0; t < S; ++t) sc += terms[t * 64 + cl];
        c_score[static_cast<int64_t>(b) * C + c] = sc;
    }
}

// Candidate ranges of query b's m chosen lists (sel_pos[0..got), best first):
// each list clipped to the key rows [row_lo, row_hi) this call holds and to
// max_list rows, as local key rows, and the prefix sum of their sizes.
__device__ void select_list_ranges(int got, int m, int b, const int64_t* sel_pos,
                                   const int64_t* __restrict__ list_off, int64_t n_global, int64_t row_lo,
                                   int64_t row_hi, int max_list, int32_t* __restrict__ top_clusters,
                                   int64_t* __restrict__ probe_lo, int64_t* __restrict__ cand_base,
                                   uint32_t* status, int64_t* s_sz) {
    for (int j = threadIdx.x; j < m; j += blockDim.x) {
        const int c = j < got ? static_cast<int>(sel_pos[j]) : 0;
        int64_t lo = list_off[c], hi = list_off[c + 1];
        if (lo < 0 || hi < lo || hi > n_global) { raise_status(status, DWA_STATUS_BAD_LIST); lo = hi = 0; }
        if (hi - lo > max_list) raise_status(status, DWA_STATUS_LIST_OVERFLOW);
        lo = lo > row_lo ? lo : row_lo;
        hi = hi < row_hi ? hi : row_hi;
        int64_t sz = hi > lo ? hi - lo : 0;
        if (sz > max_list) sz = max_list;
        top_clusters[static_cast<int64_t>(b) * m + j] = c;
        probe_lo[static_cast<int64_t>(b) * (m + 1) + j] = sz > 0 ? lo - row_lo : 0;
        s_sz[j] = sz;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int64_t acc = 0;
        for (int j = 0; j < m; ++j) {
            cand_base[static_cast<int64_t>(b) * (m + 1) + j] = acc;
            acc += s_sz[j];
        }
        probe_lo[static_cast<int64_t>(b) * (m + 1) + m] = 0;
        cand_base[static_cast<int64_t>(b) * (m + 1) + m] = acc;
    }
}

constexpr int kStageKeys = 6144;  // candidates staged in shared memory (48 KB of keys)

// Top-m lists per query (ties to the lower list) and each probed list's
// candidate range.  [row_lo, row_hi) is the window of pool rows whose keys this
// call holds (the whole pool, or one rank's slice): a list's candidates are its
// rows inside the window, as local key rows; n_global bounds the list offsets.
__global__ void __launch_bounds__(512) topm_kernel(
    const float* __restrict__ c_score, int C, int m, const int64_t* __restrict__ list_off,
    int64_t n_global, int64_t row_lo, int64_t row_hi, int max_list, int32_t* __restrict__ top_clusters,
    int64_t* __restrict__ probe_lo, int64_t* __restrict__ cand_base, uint32_t* status) {
    pdl_enter();
    __shared__ uint64_t sel_key[kMaxK];
    __shared__ int64_t sel_pos[kMaxK];
    extern __shared__ uint64_t skeys[];
    const int b = blockIdx.x;
    const float* cs = c_score + static_cast<int64_t>(b) * C;
    int got;
    if (C <= kStageKeys) {
        for (int i = threadIdx.x; i < C; i += blockDim.x) skeys[i] = make_key(cs[i], static_cast<uint32_t>(i));
        __syncthreads();
        auto key_at = [&](int64_t i) { return skeys[i]; };
        got = block_topk(C, m, key_at, sel_key, sel_pos);
    } else {
        auto key_at = [&](int64_t i) { return make_key(cs[i], static_cast<uint32_t>(i)); };
        got = block_topk(C, m, key_at, sel_key, sel_pos);
    }
    __shared__ int64_t s_sz[kMaxK + 1];
    select_list_ranges(got, m, b, sel_pos, list_off, n_global, row_lo, row_hi, max_list, top_clusters,
                       probe_lo, cand_base, status, s_sz);
}

// Coarse scores and top-m lists of one query by one cluster of CL CTAs
// (grid (CL, B), clusters (CL, 1, 1), 64*S threads): every CTA normalises the
// query's raw aspects in shared memory (normalize_aspect), scores its chunk of
// ceil(C / CL) centroids with coarse_kernel's operations and order, and stores
// their selection keys straight into cluster rank 0's key array (distributed
// shared memory); after one cluster barrier rank 0 writes the normalised qw[b]
// and picks the lists as topm_kernel does.  Replaces query_norm + coarse + topm
// when the C keys fit in shared memory.
struct CoarseTopmArgs {
    const float* q;          // [B, S, d_k] raw aspect queries
    const float* aspect_w;   // [S]
    const float* centroids;  // [S, C, d_k]
    int S, d_k, C, m;
    const int64_t* list_off;
    int64_t n_global, row_lo, row_hi;
    int max_list;
    float* qw;               // [B, S, d_k] out: normalised queries
    int32_t* top_clusters;
    int64_t* probe_lo;
    int64_t* cand_base;
    uint32_t* status;
};

constexpr int kCoarseCluster = 8;

__host__ __device__ inline size_t coarse_topm_keys_bytes(int C) { return (static_cast<size_t>(C) * 8 + 15) / 16 * 16; }
__host__ __device__ inline int coarse_topm_chunk(int C, int CL) { return (C + CL - 1) / CL; }
// Centroids scored per pass by one CTA of the fused coarse kernel: its chunk of
// the lists, rounded up to a warp, as far as S * cpp threads fit in 1024.
__host__ __device__ inline int coarse_topm_cpp(int C, int CL, int S) {
    int cpp = (coarse_topm_chunk(C, CL) + 31) / 32 * 32;
    const int cap = (1024 / S) / 32 * 32;
    cpp = cpp > cap ? cap : cpp;
    return cpp < 32 ? 32 : cpp;
}
__host__ __device__ inline size_t coarse_topm_smem(int C, int S, int d_k, int cpp) {
    return coarse_topm_keys_bytes(C) + (static_cast<size_t>(S) * d_k + static_cast<size_t>(S) * cpp) * sizeof(float);
}

template <int DK>
__global__ void __launch_bounds__(1024) coarse_topm_kernel(CoarseTopmArgs a) {
    __shared__ uint64_t sel_key[kMaxK];
    __shared__ int64_t sel_pos[kMaxK];
    __shared__ int64_t s_sz[kMaxK + 1];
    extern __shared__ __align__(16) unsigned char ctm[];
    cooperative_groups::cluster_group cl = cooperative_groups::this_cluster();
    cluster_arrive_relaxed();
    const int S = a.S, d_k = a.d_k, C = a.C;
    const int CL = static_cast<int>(cl.num_blocks()), rank = static_cast<int>(cl.block_rank());
    const int b = blockIdx.y, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int cpc = coarse_topm_chunk(C, CL), c_lo = rank * cpc, c_hi = min(C, c_lo + cpc);
    const int cpp = blockDim.x / S;             // centroids per pass (coarse_topm_cpp)
    const int cl_i = threadIdx.x % cpp, s = threadIdx.x / cpp;
    // The preceding kernel (the query projection) does not write the
    // centroids: the first chunk's rows and their squared norms are read
    // before waiting for it.
    float4 kv0[DK > 0 ? DK / 4 : 1];
    float nrm0 = 0.f;
    if constexpr (DK > 0) {
        if (c_lo + cl_i < c_hi) {
            const float4* kp = reinterpret_cast<const float4*>(a.centroids + (static_cast<int64_t>(s) * C + c_lo + cl_i) * d_k);
#pragma unroll
            for (int i = 0; i < DK / 4; ++i) kv0[i] = __ldg(kp + i);
#pragma unroll
            for (int i = 0; i < DK / 4; ++i) {
                nrm0 = fmaf(kv0[i].x, kv0[i].x, nrm0);
                nrm0 = fmaf(kv0[i].y, kv0[i].y, nrm0);
                nrm0 = fmaf(kv0[i].z, kv0[i].z, nrm0);
                nrm0 = fmaf(kv0[i].w, kv0[i].w, nrm0);
            }
        }
    }
    pdl_enter();
    uint64_t* keys = reinterpret_cast<uint64_t*>(ctm);
    float* qs = reinterpret_cast<float*>(ctm + coarse_topm_keys_bytes(C));
    float* terms = qs + S * d_k;
    uint64_t* keys0 = cl.map_shared_rank(keys, 0);
    for (int i = threadIdx.x; i < S * d_k; i += blockDim.x) qs[i] = a.q[static_cast<int64_t>(b) * S * d_k + i];
    __syncthreads();
    for (int t = warp; t < S; t += nwarps) normalize_aspect(qs + t * d_k, a.aspect_w, S, t, d_k);
    __syncthreads();
    if (rank == 0 && a.qw)   // qw == nullptr: query_norm_kernel has written it already
        for (int i = threadIdx.x; i < S * d_k; i += blockDim.x) a.qw[static_cast<int64_t>(b) * S * d_k + i] = qs[i];
    cluster_wait();   // rank 0 is running: its key array takes remote stores
    for (int cb = c_lo; cb < c_hi; cb += cpp) {
        const int c = cb + cl_i;
        if (c < c_hi) {
            const float* kp = a.centroids + (static_cast<int64_t>(s) * C + c) * d_k;
            const float* qq = qs + s * d_k;
            float dot = 0.f, nrm = 0.f;
            if constexpr (DK > 0) {
                float4 kv[DK / 4];
                if (cb == c_lo) {
#pragma unroll
                    for (int i = 0; i < DK / 4; ++i) kv[i] = kv0[i];
                    nrm = nrm0;
                } else {
#pragma unroll
                    for (int i = 0; i < DK / 4; ++i) kv[i] = __ldg(reinterpret_cast<const float4*>(kp) + i);
#pragma unroll
                    for (int i = 0; i < DK / 4; ++i) {
                        nrm = fmaf(kv[i].x, kv[i].x, nrm);
                        nrm = fmaf(kv[i].y, kv[i].y, nrm);
                        nrm = fmaf(kv[i].z, kv[i].z, nrm);
                        nrm = fmaf(kv[i].w, kv[i].w, nrm);
                    }
                }
#pragma unroll
                for (int i = 0; i < DK / 4; ++i) {
                    const float4 qv = reinterpret_cast<const float4*>(qq)[i];
                    dot = fmaf(kv[i].x, qv.x, dot);
                    dot = fmaf(kv[i].y, qv.y, dot);
                    dot = fmaf(kv[i].z, qv.z, dot);
                    dot = fmaf(kv[i].w, qv.w, dot);
                }
            } else {
                for (int d = 0; d < d_k; ++d) {
                    const float x = __ldg(kp + d);
                    nrm = fmaf(x, x, nrm);
                    dot = fmaf(x, qq[d], dot);
                }
            }
            terms[s * cpp + cl_i] = dot / (sqrtf(nrm) + 1e-8f);
        }
        __syncthreads();
        if (s == 0 && c < c_hi) {
            float sc = 0.f;
            for (int t = 0; t < S; ++t) sc += terms[t * cpp + cl_i];
            keys0[c] = make_key(sc, static_cast<uint32_t>(c));
        }
        __syncthreads();
    }
    cl.sync();   // every rank's keys are in rank 0's shared memory
    if (rank != 0) return;
    auto key_at = [&](int64_t i) { return keys[i]; };
    const int got = block_topk(C, a.m, key_at, sel_key, sel_pos);
    select_list_ranges(got, a.m, b, sel_pos, a.list_off, a.n_global, a.row_lo, a.row_hi, a.max_list,
                       a.top_clusters, a.probe_lo, a.cand_base, a.status, s_sz);
}

template <int DK>
__global__ void fine_kernel(const float* __restrict__ qw, const float* __restrict__ keys, int64_t N,
                            int S, int d_k, int m, const int64_t* __restrict__ probe_lo,
                            const int64_t* __restrict__ cand_base, int64_t K_cap,
                            float* __restrict__ scores) {
    pdl_enter();
    extern __shared__ __align__(16) float qs[];
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
    row_scores<1, DK>(keys, N, S, d_k, row, qs, 1, &sc);
    scores[static_cast<int64_t>(b) * K_cap + base + r] = sc;
}

// List-inverted fine scores for batches the key scans do not take (B > 32,
// d_k = 64, S <= 4, no soft_full).  One CTA per (64 rows of a list, list):
// it takes the probes (b, j) of list c (from the probe CSR, or by scanning all
// probes when there are too many lists for it), reads its 64-row chunk of the
// list's keys once into registers (thread = (aspect, row)) and scores every
// probing query against it, instead of every query re-reading its probed
// lists.  Per (row, query) the operations and their order are those of
// row_scores(), so the scores are bit-identical to fine_kernel's.
constexpr int kFlRows = 64, kFlChunks = 1, kFlBatch = 16, kFlCap = 1024;
constexpr int kFlMaxLists = 16384;   // lists up to which probe_lists_kernel builds the CSR

// The probes (b*m + j, with rows) of every list as CSR: list_start [C+1],
// list_ent [B*m].  One CTA; counts and cursors in shared memory.  Within a list
// the order is arbitrary (each probe's scores are written independently).
__global__ void __launch_bounds__(1024) probe_lists_kernel(const int32_t* __restrict__ top_clusters,
                                                           const int64_t* __restrict__ cand_base, int B, int m,
                                                           int C, int32_t* __restrict__ list_start,
                                                           int32_t* __restrict__ list_ent) {
    pdl_enter();
    extern __shared__ int sh_lists[];
    int* cnt = sh_lists;          // [C]
    int* cur = sh_lists + C;      // [C]
    __shared__ int s_seg[1024];
    const int tid = threadIdx.x, BM = B * m;
    for (int c = tid; c < C; c += 1024) cnt[c] = 0;
    __syncthreads();
    for (int e = tid; e < BM; e += 1024) {
        const int64_t* cb = cand_base + static_cast<int64_t>(e / m) * (m + 1) + (e % m);
        const int c = top_clusters[e];
        if (cb[1] > cb[0] && c >= 0 && c < C) atomicAdd(&cnt[c], 1);
    }
    __syncthreads();
    const int seg = (C + 1023) / 1024, c0 = tid * seg, c1 = min(C, c0 + seg);
    int sum = 0;
    for (int c = c0; c < c1; ++c) sum += cnt[c];
    s_seg[tid] = sum;
    __syncthreads();
    for (int off = 1; off < 1024; off <<= 1) {
        const int v = tid >= off ? s_seg[tid - off] : 0;
        __syncthreads();
        s_seg[tid] += v;
        __syncthreads();
    }
    int run = s_seg[tid] - sum;
    for (int c = c0; c < c1; ++c) {
        list_start[c] = run;
        cur[c] = run;
        run += cnt[c];
    }
    if (tid == 1023) list_start[C] = s_seg[1023];
    __syncthreads();
    for (int e = tid; e < BM; e += 1024) {
        const int64_t* cb = cand_base + static_cast<int64_t>(e / m) * (m + 1) + (e % m);
        const int c = top_clusters[e];
        if (cb[1] > cb[0] && c >= 0 && c < C) list_ent[atomicAdd(&cur[c], 1)] = e;
    }
}

__global__ void __launch_bounds__(256) fine_lists_kernel(
    const float* __restrict__ qw, const float* __restrict__ keys, int64_t N, int S, int B, int m,
    const int32_t* __restrict__ top_clusters, const int64_t* __restrict__ probe_lo,
    const int64_t* __restrict__ cand_base, int64_t K_cap, const int32_t* __restrict__ list_start,
    const int32_t* __restrict__ list_ent, float* __restrict__ scores) {
    pdl_enter();
    __shared__ int s_ent[kFlCap];
    __shared__ int s_wcnt[8];
    __shared__ __align__(16) float s_q[kFlBatch][4 * 64];
    __shared__ float s_part[kFlBatch][4][kFlRows];
    __shared__ int64_t s_out[kFlBatch];     // scores offset of each probe of the batch
    const int c = blockIdx.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int s = tid >> 6, rl = tid & 63;
    const int BM = B * m;
    for (int start = 0;; start += kFlCap) {
        // the probes of list c with ordinal in [start, start + kFlCap): from the
        // CSR when it was built, else in (b, j) order from a scan of all probes
        int seen = 0;
        if (list_start) {
            const int a0 = list_start[c];
            seen = list_start[c + 1] - a0;
            const int nn = min(seen - start, kFlCap);
            for (int i = tid; i < nn; i += 256) s_ent[i] = list_ent[a0 + start + i];
            __syncthreads();
        }
        for (int w0 = 0; !list_start && w0 < BM; w0 += 256) {
            const int e = w0 + tid;
            bool hit = false;
            if (e < BM && top_clusters[e] == c) {
                const int64_t* cb = cand_base + static_cast<int64_t>(e / m) * (m + 1) + (e % m);
                hit = cb[1] > cb[0];
            }
            const unsigned bal = __ballot_sync(0xffffffffu, hit);
            if (lane == 0) s_wcnt[warp] = __popc(bal);
            __syncthreads();
            int before = 0, total = 0;
            for (int w = 0; w < 8; ++w) {
                const int v = s_wcnt[w];
                before += w < warp ? v : 0;
                total += v;
            }
            if (hit) {
                const int ord = seen + before + __popc(bal & ((1u << lane) - 1u));
                if (ord >= start && ord < start + kFlCap) s_ent[ord - start] = e;
            }
            seen += total;
            __syncthreads();
        }
        const int n = min(seen - start, kFlCap);
        if (n <= 0) return;                      // same in every thread
        const int e0 = s_ent[0];
        const int b0 = e0 / m, j0 = e0 - b0 * m;
        const int64_t lo = probe_lo[static_cast<int64_t>(b0) * (m + 1) + j0];
        const int64_t sz = cand_base[static_cast<int64_t>(b0) * (m + 1) + j0 + 1] -
                           cand_base[static_cast<int64_t>(b0) * (m + 1) + j0];
        for (int ch = 0; ch < kFlChunks; ++ch) {
            const int64_t r0 = (static_cast<int64_t>(blockIdx.x) * kFlChunks + ch) * kFlRows;
            if (r0 >= sz) break;                 // same in every thread
            const int64_t row = r0 + rl;
            const bool valid = s < S && row < sz;
            float4 kv[16];
            float den = 1.f;
            if (valid) {
                const float4* kp = reinterpret_cast<const float4*>(keys + (static_cast<int64_t>(s) * N + lo + row) * 64);
#pragma unroll
                for (int i = 0; i < 16; ++i) kv[i] = __ldg(kp + i);
                float nrm = 0.f;
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    nrm = fmaf(kv[i].x, kv[i].x, nrm);
                    nrm = fmaf(kv[i].y, kv[i].y, nrm);
                    nrm = fmaf(kv[i].z, kv[i].z, nrm);
                    nrm = fmaf(kv[i].w, kv[i].w, nrm);
                }
                den = sqrtf(nrm) + 1e-8f;
            }
            for (int i0 = 0; i0 < n; i0 += kFlBatch) {
                const int nb = min(kFlBatch, n - i0);
                for (int t = tid; t < nb * S * 16; t += 256) {
                    const int i = t / (S * 16), o = t - i * (S * 16);
                    const int b = s_ent[i0 + i] / m;
                    reinterpret_cast<float4*>(s_q[i])[o] =
                        __ldg(reinterpret_cast<const float4*>(qw + static_cast<int64_t>(b) * S * 64) + o);
                }
                if (tid < nb) {
                    const int e = s_ent[i0 + tid];
                    const int b = e / m, j = e - b * m;
                    s_out[tid] = static_cast<int64_t>(b) * K_cap + cand_base[static_cast<int64_t>(b) * (m + 1) + j];
                }
                __syncthreads();
                if (valid) {
                    for (int i = 0; i < nb; ++i) {
                        const float4* qq = reinterpret_cast<const float4*>(&s_q[i][s * 64]);
                        float dot = 0.f;
#pragma unroll
                        for (int c4 = 0; c4 < 16; ++c4) {
                            const float4 qv = qq[c4];
                            dot = fmaf(kv[c4].x, qv.x, dot);
                            dot = fmaf(kv[c4].y, qv.y, dot);
                            dot = fmaf(kv[c4].z, qv.z, dot);
                            dot = fmaf(kv[c4].w, qv.w, dot);
                        }
                        s_part[i][s][rl] = dot / den;
                    }
                }
                __syncthreads();
                for (int t = tid; t < nb * kFlRows; t += 256) {
                    const int i = t / kFlRows, r2 = t - i * kFlRows;
                    const int64_t row2 = r0 + r2;
                    if (row2 < sz) {
                        float sc = 0.f;
                        for (int s2 = 0; s2 < S; ++s2) sc += s_part[i][s2][r2];
                        scores[s_out[i] + row2] = sc;
                    }
                }
                __syncthreads();
            }
        }
        if (seen - start <= kFlCap) return;
    }
}

// Full-pool scores for up to NB queries at a time; writes raw s_full and per
// block (max, sum exp) of s*invT (invT = 1/T) for the softmax.
template <int NB, int DK>
__global__ void __launch_bounds__(256) full_scores_kernel(
    const float* __restrict__ qw, const float* __restrict__ keys, int64_t N, int S, int d_k, int B,
    float invT, float* __restrict__ sfull, float* __restrict__ partial) {
    pdl_enter();
    extern __shared__ __align__(16) float qs[];  // [NB][S][d_k]
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
        if (row < N) row_scores<NB, DK>(keys, N, S, d_k, row, qs, nb, sc);
        for (int q = 0; q < nb; ++q) {
            float x = -INFINITY;
            if (row < N) {
                sfull[static_cast<int64_t>(b0 + q) * N + row] = sc[q];
                x = sc[q] * invT;
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

// The summary of a rank that holds no rows: no candidates, no soft_full mass.
__global__ void empty_summary_kernel(float* summary, int k) {
    pdl_enter();
    float* sm = summary + static_cast<int64_t>(blockIdx.x) * summary_width(k);
    for (int i = threadIdx.x; i < k; i += blockDim.x) {
        sm[i] = -INFINITY;
        sm[k + i] = __int_as_float(-1);
    }
    if (threadIdx.x == 0) { sm[2 * k] = 0.f; sm[2 * k + 1] = -INFINITY; sm[2 * k + 2] = 0.f; }
}

// soft_full[b, n] = exp(s*invT - M_b) * (1 / Z_b) in place (invT = 1/T, the
// factor the full pass used for M and Z); 8 elements per thread with 16-byte
// accesses from the first 16-byte boundary of the row on (a rank's slice of
// a row-sharded pool can have any row count, so rows need not start aligned),
// and the at most 3 + 7 elements before and after that body one per thread.
__global__ void __launch_bounds__(256) softmax_apply_kernel(float* __restrict__ sfull, int64_t N,
                                                            float invT, const float* __restrict__ stats) {
    pdl_enter();
    const int b = blockIdx.y;
    const float mx = stats[2 * b], rz = 1.f / stats[2 * b + 1];
    float* p = sfull + static_cast<int64_t>(b) * N;
    const int64_t lead = ((16 - (reinterpret_cast<uintptr_t>(p) & 15)) & 15) >> 2;
    const int64_t head = lead < N ? lead : N;
    const int64_t body = (N - head) & ~static_cast<int64_t>(7);
    const int64_t i0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
    if (i0 < body) {
        float4* q = reinterpret_cast<float4*>(p + head + i0);
        float4 a = q[0];
        float4 c = q[1];
        a.x = expf(a.x * invT - mx) * rz; a.y = expf(a.y * invT - mx) * rz;
        a.z = expf(a.z * invT - mx) * rz; a.w = expf(a.w * invT - mx) * rz;
        c.x = expf(c.x * invT - mx) * rz; c.y = expf(c.y * invT - mx) * rz;
        c.z = expf(c.z * invT - mx) * rz; c.w = expf(c.w * invT - mx) * rz;
        q[0] = a;
        q[1] = c;
    }
    if (blockIdx.x == 0 && threadIdx.x < 16) {
        const int64_t t = threadIdx.x;
        const int64_t i = t < head ? t : head + body + (t - head);
        if (i < N) p[i] = expf(p[i] * invT - mx) * rz;
    }
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
    int64_t row_lo;     // global pool row of local key row 0
    float* summary;     // non-null: a rank's part of a sharded call, [B, 2k+3] (see below)
    // soft_full statistics (max, sum exp) of s/T into sf_stats[b * sf_stride + {0, 1}]
    // when sf_stats is non-null: from the full pass's per-CTA pairs
    // sf_partial [B, sf_nblk, 2], or (-inf, 0) when sf_partial is null
    const float* sf_partial;
    int sf_nblk;
    float* sf_stats;
    int sf_stride;
};

__device__ __forceinline__ float gate_raw(float s, float lam, float tau, float T) {
    const float g = 1.f / (1.f + expf(-(lam * (s - tau))));
    return g * expf(s / T);
}

// alphas and indices of one query from its got <= k winners (scores s_sv, global
// rows rows_sv, best first), run by one warp (retrieval.py:143-158): warmup
// softmax(top / T); gate raw / (Z + 1e-8), then / (sum top + 1e-8).  Shared by
// the single-call selection and the merge of a sharded call.
__device__ void write_alphas(int got, int k, bool gate, float lam, float tau, float T, float Z,
                             float* s_sv, const int64_t* rows_sv, float* al, int32_t* ix) {
    const int l = threadIdx.x & 31;
    if (!gate) {
        // softmax(top / T) (retrieval.py:146); s_sv[0] is the maximum
        const float mx = got > 0 ? s_sv[0] / T : 0.f;
        float den = 0.f;
        for (int i = l; i < got; i += 32) den += expf(s_sv[i] / T - mx);
        den = warp_sum(den);
        for (int i = l; i < got; i += 32) al[i] = expf(s_sv[i] / T - mx) / den;
    } else {
        // raw / (sum raw + 1e-8), then / (sum top + 1e-8) (retrieval.py:150-155)
        float tot = 0.f;
        for (int i = l; i < got; i += 32) {
            const float v = gate_raw(s_sv[i], lam, tau, T) / (Z + 1e-8f);
            s_sv[i] = v;
            tot += v;
        }
        tot = warp_sum(tot);
        for (int i = l; i < got; i += 32) al[i] = s_sv[i] / (tot + 1e-8f);
    }
    for (int i = l; i < got; i += 32) ix[i] = static_cast<int32_t>(rows_sv[i]);
    __syncwarp();
    for (int i = got + l; i < k; i += 32) { al[i] = 0.f; ix[i] = got > 0 ? static_cast<int32_t>(rows_sv[0]) : 0; }
}

// soft_full statistics of query b (see SelectArgs), by the whole block.
__device__ void write_softmax_stats(const SelectArgs& a, int b, float* red) {
    float mx = -INFINITY, zs = 0.f;
    if (a.sf_partial) {
        const float* p = a.sf_partial + static_cast<int64_t>(b) * a.sf_nblk * 2;
        for (int i = threadIdx.x; i < a.sf_nblk; i += blockDim.x) mx = fmaxf(mx, p[2 * i]);
        mx = block_reduce(mx, true, red);
        for (int i = threadIdx.x; i < a.sf_nblk; i += blockDim.x) zs += p[2 * i + 1] * expf(p[2 * i] - mx);
        zs = block_reduce(zs, false, red);
    }
    if (threadIdx.x == 0) {
        a.sf_stats[static_cast<int64_t>(b) * a.sf_stride] = mx;
        a.sf_stats[static_cast<int64_t>(b) * a.sf_stride + 1] = zs;
    }
}

// The result of query b's selection from its got <= k winners (scores s_sv,
// global rows rows_sv, best first) and the gate sum Z: the rank's summary in a
// sharded call, else alphas and indices.
__device__ void emit_selection(const SelectArgs& a, int b, int got, bool gate, float lam, float tau, float Z,
                               float* s_sv, int64_t* rows_sv) {
    if (a.summary) {
        float* sm = a.summary + static_cast<int64_t>(b) * summary_width(a.k);
        for (int i = threadIdx.x; i < a.k; i += blockDim.x) {
            sm[i] = i < got ? s_sv[i] : -INFINITY;
            sm[a.k + i] = __int_as_float(i < got ? static_cast<int32_t>(rows_sv[i]) : -1);
        }
        if (threadIdx.x == 0) sm[2 * a.k] = gate ? Z : 0.f;
        return;
    }
    if (threadIdx.x < 32) {
        if (threadIdx.x == 0 && got < a.k) raise_status(a.status, DWA_STATUS_FEW_CANDIDATES);
        write_alphas(got, a.k, gate, lam, tau, a.T, Z, s_sv, rows_sv, a.alphas + static_cast<int64_t>(b) * a.k,
                     a.indices + static_cast<int64_t>(b) * a.k);
    }
}

// Selection of one query by a cluster of CL CTAs (grid (CL, B), clusters
// (CL, 1, 1), kSelThreads threads).  CTA r takes the candidate positions
// [n*r/CL, n*(r+1)/CL): score, gate term and key staged in shared memory (in
// passes of up to local_cap when there are more), adds its share of the gate
// sum Z, selects its local top k and stores it, with its Z share, into cluster
// rank 0's shared memory.  After one cluster barrier rank 0 adds the Z shares
// in rank order and selects the top k of the CL*k pushed slots; the keys order
// (score or gate term, then pool row) is the single-block selection's, so the
// winners are the same.  The last rank also writes the soft_full statistics.
constexpr int kSelThreads = 512;
constexpr int kSelCluster = 8;
constexpr int kSelLocalKeys = 14336;   // candidates a CTA stages (168 KB of keys and scores)

// Dynamic shared memory: keys [cap], pushed keys [CL*k], scores [cap], pushed
// scores [CL*k], cap = max(local_cap, CL*k).
__host__ __device__ inline size_t select_cluster_smem(int64_t local_cap, int CL, int k) {
    const int64_t ck = static_cast<int64_t>(CL) * k;
    const int64_t cap = local_cap > ck ? local_cap : ck;
    return static_cast<size_t>(cap + ck) * (sizeof(uint64_t) + sizeof(float));
}

__global__ void __launch_bounds__(kSelThreads) select_cluster_kernel(SelectArgs a, int local_cap) {
    pdl_enter();
    __shared__ uint64_t sel_key[kMaxK];
    __shared__ int64_t sel_pos[kMaxK];
    __shared__ int64_t s_lo[kMaxK + 1], s_base[kMaxK + 1];
    __shared__ float red[33];
    __shared__ int m_got[kSelCluster];     // rank 0: each rank's number of winners
    __shared__ float m_z[kSelCluster];     // rank 0: each rank's share of Z
    __shared__ float s_sv[kMaxK];
    extern __shared__ __align__(16) unsigned char sel_sm[];
    cooperative_groups::cluster_group cl = cooperative_groups::this_cluster();
    cluster_arrive_relaxed();
    const int CL = static_cast<int>(cl.num_blocks()), r = static_cast<int>(cl.block_rank());
    const int b = blockIdx.y, tid = threadIdx.x, k = a.k;
    const int ck = CL * k, cap = local_cap > ck ? local_cap : ck;
    uint64_t* skeys = reinterpret_cast<uint64_t*>(sel_sm);
    uint64_t* mkeys = skeys + cap;
    float* sscore = reinterpret_cast<float*>(mkeys + ck);
    float* mscore = sscore + cap;
    for (int j = tid; j <= a.m; j += blockDim.x) {
        s_lo[j] = a.probe_lo[static_cast<int64_t>(b) * (a.m + 1) + j];
        s_base[j] = a.cand_base[static_cast<int64_t>(b) * (a.m + 1) + j];
    }
    if (a.sf_stats && r == CL - 1) write_softmax_stats(a, b, red);
    __syncthreads();
    const int64_t n = s_base[a.m];
    const int64_t p_lo = n * r / CL, p_hi = n * (r + 1) / CL;
    const float lam = __ldg(a.lambda_val), tau = __ldg(a.tau), T = a.T;
    const bool gate = !a.is_warmup;
    const bool rank_raw = gate && lam < 0.f;
    float zacc = 0.f;
    // Candidates beyond the staging capacity are taken in passes: the running
    // winners stay at the front of the staging arrays and each pass stages up
    // to local_cap - carried new candidates behind them.  Keys are unique
    // (score or gate term, then pool row), so the winners do not depend on
    // the passes.
    auto key_at = [&](int64_t i) { return skeys[i]; };
    int carried = 0, got = 0;
    constexpr int U = 4;
    for (int64_t q0 = p_lo;;) {
        const int64_t room = cap - carried;     // cap >= k >= carried
        if (room <= 0) {
            raise_status(a.status, DWA_STATUS_LIST_OVERFLOW);
            break;
        }
        const int64_t q1 = p_hi - q0 > room ? q0 + room : p_hi;
        for (int64_t p0 = q0; p0 < q1; p0 += kSelThreads * U) {
            float sv[U];
            int64_t rowv[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int64_t p = p0 + u * kSelThreads + tid;
                sv[u] = 0.f;
                rowv[u] = 0;
                if (p < q1) {
                    int lo = 0, hi = a.m - 1;
                    while (lo < hi) {
                        const int mid = (lo + hi + 1) >> 1;
                        if (s_base[mid] <= p) lo = mid; else hi = mid - 1;
                    }
                    rowv[u] = s_lo[lo] + (p - s_base[lo]);
                    sv[u] = a.sfull ? a.sfull[static_cast<int64_t>(b) * a.N + rowv[u]]
                                    : a.scores[static_cast<int64_t>(b) * a.K_cap + p];
                }
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int64_t p = p0 + u * kSelThreads + tid;
                if (p < q1) {
                    const float raw = gate ? gate_raw(sv[u], lam, tau, T) : 0.f;
                    zacc += raw;
                    skeys[carried + (p - q0)] = make_key(rank_raw ? raw : sv[u], static_cast<uint32_t>(rowv[u] + a.row_lo));
                    sscore[carried + (p - q0)] = sv[u];
                }
            }
        }
        __syncthreads();
        got = block_topk(carried + (q1 - q0), k, key_at, sel_key, sel_pos);
        q0 = q1;
        if (q0 >= p_hi) break;
        // carry this pass's winners to the front (k <= kMaxK <= kSelThreads)
        uint64_t kw = 0;
        float sw = 0.f;
        if (tid < got) {
            kw = sel_key[tid];
            sw = sscore[sel_pos[tid]];
        }
        __syncthreads();
        if (tid < got) {
            skeys[tid] = kw;
            sscore[tid] = sw;
        }
        carried = got;
        __syncthreads();
    }
    const float zshare = gate ? block_reduce(zacc, false, red) : 0.f;
    __syncthreads();
    // push the local winners (slots past got: key 0, below every real key)
    // and the Z share into rank 0
    cluster_wait();
    {
        uint64_t* mk = cl.map_shared_rank(mkeys, 0);
        float* ms = cl.map_shared_rank(mscore, 0);
        for (int i = tid; i < k; i += blockDim.x) {
            mk[r * k + i] = i < got ? sel_key[i] : 0ull;
            ms[r * k + i] = i < got ? sscore[sel_pos[i]] : 0.f;
        }
        if (tid == 0) {
            cl.map_shared_rank(m_got, 0)[r] = got;
            cl.map_shared_rank(m_z, 0)[r] = zshare;
        }
    }
    cl.sync();
    if (r != 0) return;
    // rank 0: the top k of the CL*k slots (Z shares added in rank order)
    int total = 0;
    float Z = 0.f;
    for (int src = 0; src < CL; ++src) {
        total += m_got[src];
        Z += m_z[src];
    }
    auto mkey_at = [&](int64_t i) { return mkeys[i]; };
    const int fin = block_topk(ck, total < k ? total : k, mkey_at, sel_key, sel_pos);
    for (int i = tid; i < fin; i += blockDim.x) {
        s_sv[i] = mscore[sel_pos[i]];
        sel_pos[i] = static_cast<int64_t>(0xFFFFFFFFu - static_cast<uint32_t>(sel_key[i] & 0xFFFFFFFFu));
    }
    __syncthreads();
    emit_selection(a, b, fin, gate, lam, tau, Z, s_sv, sel_pos);
}

// Merge of a sharded call: per query, the global top-k of the world ranks'
// summaries (ties to the lower global row), Z = sum of the ranks' partial
// sums in rank order, alphas as in the single call; and the soft_full
// statistics (max, sum exp) of s/T combined over the ranks into stats[b].
struct MergeArgs {
    const float* summaries;   // [world, B, 2k+3]
    int world, B, k;
    float T;
    int is_warmup;
    const float* lambda_val;
    const float* tau;
    float* alphas;
    int32_t* indices;
    float* stats;             // [B, 2] or null
    uint32_t* status;
};

__global__ void __launch_bounds__(1024) merge_kernel(MergeArgs a) {
    pdl_enter();
    __shared__ uint64_t sel_key[kMaxK];
    __shared__ int64_t sel_pos[kMaxK];
    __shared__ float s_sv[kMaxK];
    __shared__ int s_valid;
    extern __shared__ uint64_t mkeys[];
    const int b = blockIdx.x, W = summary_width(a.k);
    const float lam = __ldg(a.lambda_val), tau = __ldg(a.tau), T = a.T;
    const bool gate = !a.is_warmup;
    const bool rank_raw = gate && lam < 0.f;
    const int n = a.world * a.k;
    if (threadIdx.x == 0) s_valid = 0;
    __syncthreads();
    int valid = 0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float* sm = a.summaries + (static_cast<int64_t>(i / a.k) * a.B + b) * W;
        const int j = i % a.k;
        const int32_t row = __float_as_int(sm[a.k + j]);
        const float sv = sm[j];
        // a missing candidate gets its position as key: distinct, and below
        // every real key (whose top 32 bits are an ordered float >= 2^23)
        mkeys[i] = row >= 0 ? make_key(rank_raw ? gate_raw(sv, lam, tau, T) : sv, static_cast<uint32_t>(row))
                            : static_cast<uint64_t>(i);
        valid += row >= 0;
    }
    atomicAdd(&s_valid, valid);
    __syncthreads();
    auto key_at = [&](int64_t i) { return mkeys[i]; };
    int got = block_topk(n, a.k, key_at, sel_key, sel_pos);
    got = got < s_valid ? got : s_valid;
    for (int i = threadIdx.x; i < got; i += blockDim.x) {
        const int64_t pos = sel_pos[i];
        const float* sm = a.summaries + ((pos / a.k) * a.B + b) * W;
        s_sv[i] = sm[pos % a.k];
        sel_pos[i] = __float_as_int(sm[a.k + pos % a.k]);
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        float Z = 0.f, M = -INFINITY;
        if (threadIdx.x == 0) {
            if (got < a.k) raise_status(a.status, DWA_STATUS_FEW_CANDIDATES);
            for (int p = 0; p < a.world; ++p) {
                const float* sm = a.summaries + (static_cast<int64_t>(p) * a.B + b) * W;
                Z += sm[2 * a.k];
                M = fmaxf(M, sm[2 * a.k + 1]);
            }
            if (a.stats) {
                float zs = 0.f;
                for (int p = 0; p < a.world; ++p) {
                    const float* sm = a.summaries + (static_cast<int64_t>(p) * a.B + b) * W;
                    if (sm[2 * a.k + 1] != -INFINITY) zs += sm[2 * a.k + 2] * expf(sm[2 * a.k + 1] - M);
                }
                a.stats[2 * b] = M;
                a.stats[2 * b + 1] = zs;
            }
        }
        Z = __shfl_sync(0xffffffffu, Z, 0);
        write_alphas(got, a.k, gate, lam, tau, T, Z, s_sv, sel_pos, a.alphas + static_cast<int64_t>(b) * a.k,
                     a.indices + static_cast<int64_t>(b) * a.k);
    }
}

__global__ void full_probe_kernel(int B, int64_t N, int64_t* probe_lo, int64_t* cand_base) {
    pdl_enter();
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    probe_lo[2 * b] = 0; probe_lo[2 * b + 1] = 0;
    cand_base[2 * b] = 0; cand_base[2 * b + 1] = N;
}

// ------------------------------------------------------------------ host ---
struct RetWorkspace {
    uint32_t* status;
    float* q;
    float* qw;
    float* c_score;
    int32_t* topc;
    int64_t* probe_lo;
    int64_t* cand_base;
    float* scores;
    float* sfull;
    float* partial;
    float* stats;
    int32_t* list_start;   // [C+1] probe CSR of the list-inverted fine pass
    int32_t* list_ent;     // [B*m_eff]
    int m_eff;
    int64_t K_cap;
    int nblk;
    size_t bytes;
};

constexpr int kFullRows = 256;
constexpr int kMaxScanGrid = 1024;            // CTAs of a key scan

// The list-inverted fine pass: batches above the key scans' 32 queries.
static bool fine_by_lists(const DwaRetrieveDims& d, bool ivf, bool want_sf) {
    return ivf && !want_sf && d.d_k == 64 && d.S <= 4 && d.B > 32;
}

static RetWorkspace carve_ret(void* base, const DwaRetrieveDims& d, bool ivf, bool want_sf) {
    Carver c(base);
    RetWorkspace w{};
    w.status = static_cast<uint32_t*>(base);
    w.m_eff = ivf ? (d.m < d.C ? d.m : d.C) : 1;
    w.K_cap = ivf ? static_cast<int64_t>(w.m_eff) * d.max_list : d.N;
    w.nblk = static_cast<int>((d.N + kFullRows - 1) / kFullRows);
    w.q = c.take<float>(static_cast<size_t>(d.B) * d.S * d.d_k);
    w.qw = c.take<float>(static_cast<size_t>(d.B) * d.S * d.d_k);
    w.probe_lo = c.take<int64_t>(static_cast<size_t>(d.B) * (w.m_eff + 1));
    w.cand_base = c.take<int64_t>(static_cast<size_t>(d.B) * (w.m_eff + 1));
    if (ivf) {
        w.c_score = c.take<float>(static_cast<size_t>(d.B) * d.C);
        w.topc = c.take<int32_t>(static_cast<size_t>(d.B) * w.m_eff);
        if (!want_sf) w.scores = c.take<float>(static_cast<size_t>(d.B) * w.K_cap);
        if (fine_by_lists(d, ivf, want_sf) && d.C <= kFlMaxLists) {
            w.list_start = c.take<int32_t>(static_cast<size_t>(d.C) + 1);
            w.list_ent = c.take<int32_t>(static_cast<size_t>(d.B) * w.m_eff);
        }
    }
    const bool full_pass = !ivf || want_sf;
    if (!ivf && !want_sf) w.sfull = c.take<float>(static_cast<size_t>(d.B) * d.N);
    if (full_pass) {
        // the key scans launch at most min(ceil(N/32), kMaxScanGrid) CTAs (32- or
        // 64-row blocks), the generic pass ceil(N/256)
        const size_t part_blocks = std::max<size_t>(
            static_cast<size_t>(w.nblk),
            std::min<size_t>(static_cast<size_t>((d.N + 31) / 32), kMaxScanGrid));
        w.partial = c.take<float>(static_cast<size_t>(d.B) * part_blocks * 2);
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
    if (qbytes * 8 > 48 * 1024 || static_cast<size_t>(d->d_A) * sizeof(float) > 48 * 1024)
        return fail(DWA_ERR_UNSUPPORTED, "S*d_k or d_A too large for shared memory staging");
    if (d->S > 16) return fail(DWA_ERR_UNSUPPORTED, "S > 16");
    return DWA_OK;
}

}  // namespace dwa

using namespace dwa;

extern "C" size_t dwa_retrieve_workspace_bytes(const DwaRetrieveDims* dims, int use_ivf,
                                               int want_soft_full) {
    if (check_ret(dims, use_ivf)) return 0;
    return carve_ret(nullptr, *dims, use_ivf != 0, want_soft_full != 0).bytes;
}

// Steps 1-2 of a retrieval call, shared by the forward and the VJP: raw
// queries q = W_Q z into w.q; normalised queries into w.qw; with IVF the top-m
// lists of every query and their candidate ranges (probe_lo, cand_base) clipped
// to the key rows [row_lo, row_lo + N); without IVF one range of all N rows.
// lanes != nullptr (soft_full on, so the full key scan needs only qw): the
// normalised queries come from query_norm_kernel on `st`, and the coarse
// scores + top-m run on lanes->aux[0], concurrently with the scan the caller
// launches next on `st`; the caller joins the lanes before the selection.
static int launch_queries_and_probes(cudaStream_t st, const DwaRetrieveDims& d, bool ivf, bool dk64,
                                     const void* z, const float* W_Q, const float* aspect_weights,
                                     const float* centroids, const int64_t* list_offsets, int64_t row_lo,
                                     int64_t n_global, const RetWorkspace& w, Lanes* lanes = nullptr) {
    const size_t qsh = static_cast<size_t>(d.S) * d.d_k * sizeof(float);
    // 1. raw aspect queries q = W_Q z
    const int rows = d.S * d.d_k;
    const dim3 gq((rows + kProjRows - 1) / kProjRows, (d.B + kProjQ - 1) / kProjQ);
    const dim3 gq_big((rows + 7) / 8, (d.B + 15) / 16);
    if (d.B > 16 && d.z_dtype == DWA_BF16)
        DWA_TIMED("query", st, launch_pdl(query_proj_kernel<__nv_bfloat16, 8, 16, 2>, gq_big, kProjThreads, 0, st,
                                          static_cast<const __nv_bfloat16*>(z), W_Q, d.B, rows, d.d_A, w.q));
    else if (d.B > 16)
        DWA_TIMED("query", st, launch_pdl(query_proj_kernel<float, 8, 16, 2>, gq_big, kProjThreads, 0, st,
                                          static_cast<const float*>(z), W_Q, d.B, rows, d.d_A, w.q));
    else if (d.z_dtype == DWA_BF16)
        DWA_TIMED("query", st, launch_pdl(query_proj_kernel<__nv_bfloat16>, gq, kProjThreads, 0, st,
                                          static_cast<const __nv_bfloat16*>(z), W_Q, d.B, rows, d.d_A, w.q));
    else
        DWA_TIMED("query", st, launch_pdl(query_proj_kernel<float>, gq, kProjThreads, 0, st,
                                          static_cast<const float*>(z), W_Q, d.B, rows, d.d_A, w.q));
    DWA_LAUNCH_CHECK("query_proj_kernel");
    ++g_launches_total;

    // 2. normalised queries qw; with IVF also the coarse scores, the top-m lists
    //    and their candidate ranges: one cluster per query when the C list keys
    //    fit in shared memory, else three kernels
    const int CL = ivf ? std::min(kCoarseCluster, (d.C + 63) / 64) : 1;
    const int cpp = coarse_topm_cpp(d.C, CL, d.S);
    const size_t ct_smem = coarse_topm_smem(d.C, d.S, d.d_k, cpp);
    const bool fused_coarse = ivf && d.C <= kStageKeys && ct_smem <= 200 * 1024;
    const bool overlap = fused_coarse && lanes != nullptr;
    if (!fused_coarse || overlap) {
        DWA_TIMED("query_norm", st, launch_pdl(query_norm_kernel, d.B, 32 * d.S, 0, st, w.q, aspect_weights,
                                               d.S, d.d_k, w.qw));
        DWA_LAUNCH_CHECK("query_norm_kernel");
        ++g_launches_total;
    }
    cudaStream_t cst = st;
    if (overlap) {
        int rc = lanes->depend(lanes->aux[0], st, 1);   // the coarse lane starts after the raw queries
        if (rc) return rc;
        cst = lanes->aux[0];
    }
    if (fused_coarse) {
        const size_t sm = ct_smem;
        CoarseTopmArgs ca;
        ca.q = w.q; ca.aspect_w = aspect_weights; ca.centroids = centroids;
        ca.S = d.S; ca.d_k = d.d_k; ca.C = d.C; ca.m = w.m_eff;
        ca.list_off = list_offsets; ca.n_global = n_global; ca.row_lo = row_lo; ca.row_hi = row_lo + d.N;
        ca.max_list = d.max_list; ca.qw = overlap ? nullptr : w.qw; ca.top_clusters = w.topc;
        ca.probe_lo = w.probe_lo; ca.cand_base = w.cand_base; ca.status = w.status;
        auto fn = dk64 ? coarse_topm_kernel<64> : coarse_topm_kernel<0>;
        {   // static + dynamic shared memory may pass 48 KB at any size
            int dv = 0;
            DWA_CUDA_TRY(cudaGetDevice(&dv));
            static bool ct_attr[2][64] = {};
            if (dv < 0 || dv >= 64 || !ct_attr[dk64][dv]) {
                DWA_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
                if (dv >= 0 && dv < 64) ct_attr[dk64][dv] = true;
            }
        }
        DWA_TIMED("coarse", cst, launch_pdl_cluster(fn, dim3(CL, d.B), dim3(cpp * d.S), sm, cst, dim3(CL, 1, 1), ca));
        DWA_LAUNCH_CHECK("coarse_topm_kernel");
        ++g_launches_total;
    } else if (ivf) {
        dim3 gc((d.C + 63) / 64, d.B);
        const int cth = 64 * d.S;                       // S <= 16 (checked on entry)
        const size_t csh = qsh + static_cast<size_t>(d.S) * 64 * sizeof(float);
        if (dk64)
            DWA_TIMED("coarse", st, launch_pdl(coarse_kernel<64>, gc, cth, csh, st, 
                                        w.qw, centroids, d.S, d.d_k, d.C, w.c_score));
        else
            DWA_TIMED("coarse", st, launch_pdl(coarse_kernel<0>, gc, cth, csh, st, 
                                        w.qw, centroids, d.S, d.d_k, d.C, w.c_score));
        DWA_LAUNCH_CHECK("coarse_kernel");
        const size_t tsh = d.C <= kStageKeys ? static_cast<size_t>(d.C) * 8 : 0;
        {
            int dv = 0;
            DWA_CUDA_TRY(cudaGetDevice(&dv));
            static bool tm_attr[64] = {};
            if (dv < 0 || dv >= 64 || !tm_attr[dv]) {
                DWA_CUDA_TRY(cudaFuncSetAttribute(topm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  static_cast<int>(kStageKeys * 8)));
                if (dv >= 0 && dv < 64) tm_attr[dv] = true;
            }
        }
        DWA_TIMED("topm", st, launch_pdl(topm_kernel, d.B, 512, tsh, st, w.c_score, d.C, w.m_eff, list_offsets,
                                                                 n_global, row_lo, row_lo + d.N,
                                                                 d.max_list, w.topc, w.probe_lo,
                                                                 w.cand_base, w.status));
        DWA_LAUNCH_CHECK("topm_kernel");
        g_launches_total += 2;
    } else {
        launch_pdl(full_probe_kernel, (d.B + 127) / 128, 128, 0, st, d.B, d.N, w.probe_lo, w.cand_base);
        DWA_LAUNCH_CHECK("full_probe_kernel");
        ++g_launches_total;
    }
    return DWA_OK;
}

// One retrieval call.  shard == nullptr: the whole pool (dwa_retrieve).
// Otherwise pool_keys holds the rows [row_lo, row_lo + N) of an n_global-row
// pool and, instead of alphas / indices, the call writes this rank's summary
// [B, 2k+3] (see summary_width) and leaves soft_full as raw scores.
static int retrieve_impl(void* stream, const DwaRetrieveDims* dims, const DwaShard* shard, int use_ivf,
                         int is_warmup, const float* lambda_val, const void* z, const float* W_Q,
                         const float* aspect_weights, const float* tau, const float* centroids,
                         const int64_t* list_offsets, const float* pool_keys, float* alphas,
                         int32_t* indices, float* soft_full, float* summary, void* workspace,
                         size_t workspace_bytes) {
    int rc = check_ret(dims, use_ivf);
    if (rc) return rc;
    const DwaRetrieveDims& d = *dims;
    const bool ivf = use_ivf != 0, want_sf = soft_full != nullptr;
    if (!lambda_val || !z || !W_Q || !aspect_weights || !tau || !pool_keys ||
        (shard ? !summary : (!alphas || !indices)))
        return fail(DWA_ERR_INVALID_ARG, "a required pointer is NULL");
    const int64_t row_lo = shard ? shard->row_lo : 0, n_global = shard ? shard->n_global : d.N;
    if (ivf && (!centroids || !list_offsets))
        return fail(DWA_ERR_INVALID_ARG, "IVF needs centroids and list_offsets");
    const RetWorkspace w = carve_ret(workspace, d, ivf, want_sf);
    if (!workspace || reinterpret_cast<uintptr_t>(workspace) % 256 != 0)
        return fail(DWA_ERR_WORKSPACE, "workspace must be non-NULL and 256-byte aligned");
    if (workspace_bytes < w.bytes)
        return fail(DWA_ERR_WORKSPACE, "workspace too small: need " + std::to_string(w.bytes));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const size_t qsh = static_cast<size_t>(d.S) * d.d_k * sizeof(float);
    // d_k = 64 with 16-byte aligned keys takes the unrolled scoring; the fine
    // and the full pass always take the same variant (bit-identical scores).
    const bool dk64 = d.d_k == 64 && reinterpret_cast<uintptr_t>(pool_keys) % 16 == 0 &&
                      (!ivf || reinterpret_cast<uintptr_t>(centroids) % 16 == 0);

    // with soft_full the full scan needs only the normalised queries: the coarse
    // top-m runs beside it on a lane that the selection waits for
    std::unique_ptr<Lanes> lanes;
    if (ivf && want_sf) {
        lanes.reset(new Lanes(st));
        if ((rc = lanes->rc)) return rc;
    }
    if ((rc = launch_queries_and_probes(st, d, ivf, dk64, z, W_Q, aspect_weights, centroids, list_offsets,
                                        row_lo, n_global, w, lanes.get())))
        return rc;
    float* sfull = want_sf ? soft_full : w.sfull;
    // Scoring variant, the same for the full and the fine pass so both give
    // bit-identical scores (d_k = 64): the CUDA-core key scan for B <= 16, the
    // tensor-core key scan for 16 < B <= 32 with S <= 4, else the generic
    // kernels.  DWA_SCORES=tc (tensor-core scan wherever B <= 32) or
    // DWA_SCORES=generic select another variant, for comparisons.
    int dev = 0, dev_sms = 148;
    DWA_CUDA_TRY(cudaGetDevice(&dev));
    DWA_CUDA_TRY(cudaDeviceGetAttribute(&dev_sms, cudaDevAttrMultiProcessorCount, dev));
    dev_sms = std::min(dev_sms, kMaxScanGrid);
    const char* variant = std::getenv("DWA_SCORES");
    const bool ask_tc = variant && std::strcmp(variant, "tc") == 0;
    const bool ask_generic = variant && std::strcmp(variant, "generic") == 0;
    const bool scan_shape = dk64 && !ask_generic && static_cast<int64_t>(d.S) * d.N < (int64_t(1) << 31);
    // tensor-core scan
    const int nq = d.B <= 16 ? 16 : 32;
    const int tc_stages = sc::ring_stages(nq, d.S);
    const size_t tc_smem = sc::smem_bytes(tc_stages, nq, d.S);
    bool use_tc = scan_shape && d.B <= 32 && (ask_tc || d.B > 16) && d.S <= sc::MAXS &&
                  d.S * nq <= 128 && tc_smem <= sc::kSmemLimit;
    // CUDA-core scan: full pass with QB query chains, fine pass <8, true>
    const int qb = d.B <= 4 ? 4 : d.B <= 8 ? 8 : 16;
    auto scan_full_smem = [&](int st) {
        return qb == 16 ? ks::smem_bytes<16>(st, 16, d.S) : ks::smem_bytes<8>(st, qb, d.S);
    };
    int scan_stages = 0, fine_stages = 0;
    for (int st = 3; st >= 2 && !scan_stages; --st)
        if (scan_full_smem(st) <= ks::kSmemLimit) scan_stages = st;
    for (int st = 3; st >= 2 && !fine_stages; --st)
        if (ks::smem_bytes<8>(st, d.B, d.S) <= ks::kSmemLimit) fine_stages = st;
    bool use_scan = scan_shape && !use_tc && d.B <= ks::MAX_QB && scan_stages && fine_stages;
    CUtensorMap tm_scores;
    if (use_tc || use_scan) {
        auto enc = tc::tensor_map_encoder();
        cuuint64_t dims2[2] = {64, static_cast<cuuint64_t>(d.S) * static_cast<cuuint64_t>(d.N)};
        cuuint64_t strides2[1] = {64 * sizeof(float)};
        cuuint32_t box2[2] = {use_tc ? 32u : static_cast<cuuint32_t>(ks::KQ),
                              static_cast<cuuint32_t>(use_tc ? sc::BOX : ks::BOX)};
        cuuint32_t es2[2] = {1, 1};
        const bool ok = enc && enc(&tm_scores, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(pool_keys),
                                   dims2, strides2, box2, es2, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                   use_tc ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
        if (!ok) use_tc = use_scan = false;
    }
    static bool tc_attr[2][64] = {}, scan_attr[4][64] = {};
    const int ti = nq == 16 ? 0 : 1;
    if (use_tc && (dev < 0 || dev >= 64 || !tc_attr[ti][dev])) {
        const void* fn = nq == 16 ? reinterpret_cast<const void*>(sc::key_scan_tc_kernel<16>)
                                  : reinterpret_cast<const void*>(sc::key_scan_tc_kernel<32>);
        DWA_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(sc::kSmemLimit)));
        if (dev >= 0 && dev < 64) tc_attr[ti][dev] = true;
    }
    const int qi = qb == 4 ? 0 : qb == 8 ? 1 : 2;
    if (use_scan && (dev < 0 || dev >= 64 || !scan_attr[qi][dev] || !scan_attr[3][dev])) {
        const void* fns[2] = {
            qb == 4   ? reinterpret_cast<const void*>(ks::key_scan_kernel<4, false>)
            : qb == 8 ? reinterpret_cast<const void*>(ks::key_scan_kernel<8, false>)
                      : reinterpret_cast<const void*>(ks::key_scan_kernel<16, false>),
            reinterpret_cast<const void*>(ks::key_scan_kernel<8, true>)};
        for (const void* fn : fns)
            DWA_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              static_cast<int>(ks::kSmemLimit)));
        if (dev >= 0 && dev < 64) scan_attr[qi][dev] = scan_attr[3][dev] = true;
    }
    // mode 0: full pass into `out` = s_full [B, N]; mode 1: fine pass into scores [B, K_cap]
    auto launch_scores = [&](int mode, float* out, int* blocks_out) -> int {
        kt::Args ka{};
        ka.N = d.N; ka.S = d.S; ka.B = d.B; ka.invT = 1.f / d.T; ka.mode = mode;
        ka.qw = w.qw; ka.out = out; ka.partial = w.partial; ka.status = w.status;
        int rows, box;
        if (use_tc) {
            rows = sc::ROWS; box = sc::BOX; ka.stages = tc_stages;
        } else {
            rows = mode == 1 ? ks::tile_rows<8>() : qb == 16 ? ks::tile_rows<16>() : ks::tile_rows<8>();
            box = ks::BOX;
            ka.stages = mode == 1 ? fine_stages : scan_stages;
        }
        int64_t work;
        if (mode == 0) {
            ka.nblk = (d.N + box - 1) / box;
            work = ka.nblk;
        } else {
            ka.tiles_per_list = (d.max_list + rows - 1) / rows;
            ka.m = w.m_eff;
            ka.ntiles = d.B * w.m_eff * ka.tiles_per_list;
            ka.probe_lo = w.probe_lo; ka.cand_base = w.cand_base; ka.K_cap = w.K_cap;
            work = ka.ntiles;
        }
        const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(work, dev_sms)));
        const char* name = mode == 0 ? "full_scores" : "fine";
        if (use_tc) {
            if (nq == 16)
                DWA_TIMED(name, st, launch_pdl(sc::key_scan_tc_kernel<16>, blocks, sc::THREADS, tc_smem, st, tm_scores, ka));
            else
                DWA_TIMED(name, st, launch_pdl(sc::key_scan_tc_kernel<32>, blocks, sc::THREADS, tc_smem, st, tm_scores, ka));
            DWA_LAUNCH_CHECK("key_scan_tc_kernel");
        } else {
            const size_t smem = mode == 1 ? ks::smem_bytes<8>(fine_stages, d.B, d.S) : scan_full_smem(scan_stages);
            if (mode == 1)
                DWA_TIMED(name, st, (launch_pdl(ks::key_scan_kernel<8, true>, blocks, ks::THREADS, smem, st, tm_scores, ka)));
            else if (qb == 4)
                DWA_TIMED(name, st, (launch_pdl(ks::key_scan_kernel<4, false>, blocks, ks::THREADS, smem, st, tm_scores, ka)));
            else if (qb == 8)
                DWA_TIMED(name, st, (launch_pdl(ks::key_scan_kernel<8, false>, blocks, ks::THREADS, smem, st, tm_scores, ka)));
            else
                DWA_TIMED(name, st, (launch_pdl(ks::key_scan_kernel<16, false>, blocks, ks::THREADS, smem, st, tm_scores, ka)));
            DWA_LAUNCH_CHECK("key_scan_kernel");
        }
        ++g_launches_total;
        if (blocks_out) *blocks_out = blocks;
        return DWA_OK;
    };

    // 3. full-pool raw scores (soft_full or full search)
    int sf_blocks = w.nblk;
    if ((!ivf || want_sf) && (use_tc || use_scan)) {
        if ((rc = launch_scores(0, sfull, &sf_blocks))) return rc;
    } else if (!ivf || want_sf) {
        constexpr int NB = 8;
        if (dk64)
            DWA_TIMED("full_scores", st,
                      launch_pdl(full_scores_kernel<NB, 64>, w.nblk, kFullRows, NB * qsh, st, 
                          w.qw, pool_keys, d.N, d.S, d.d_k, d.B, 1.f / d.T, sfull, w.partial));
        else
            DWA_TIMED("full_scores", st,
                      launch_pdl(full_scores_kernel<NB, 0>, w.nblk, kFullRows, NB * qsh, st, 
                          w.qw, pool_keys, d.N, d.S, d.d_k, d.B, 1.f / d.T, sfull, w.partial));
        DWA_LAUNCH_CHECK("full_scores_kernel");
        ++g_launches_total;
    }
    if (lanes && (rc = lanes->join())) return rc;   // the probed lists are known from here on
    // 4. fine scores of the probed lists (read from the full pass when it ran)
    if (ivf && !want_sf && (use_tc || use_scan)) {
        if ((rc = launch_scores(1, w.scores, nullptr))) return rc;
    } else if (fine_by_lists(d, ivf, want_sf) && dk64) {
        if (w.list_start) {
            const size_t lsm = 2 * static_cast<size_t>(d.C) * sizeof(int);
            if (lsm > 48 * 1024)
                DWA_CUDA_TRY(cudaFuncSetAttribute(probe_lists_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  static_cast<int>(lsm)));
            DWA_TIMED("probe_lists", st, launch_pdl(probe_lists_kernel, 1, 1024, lsm, st, w.topc, w.cand_base, d.B,
                                                    w.m_eff, d.C, w.list_start, w.list_ent));
            DWA_LAUNCH_CHECK("probe_lists_kernel");
            ++g_launches_total;
        }
        dim3 gl(static_cast<unsigned>((d.max_list + kFlRows * kFlChunks - 1) / (kFlRows * kFlChunks)), d.C);
        DWA_TIMED("fine", st, launch_pdl(fine_lists_kernel, gl, 256, 0, st, w.qw, pool_keys, d.N, d.S, d.B,
                                         w.m_eff, w.topc, w.probe_lo, w.cand_base, w.K_cap, w.list_start,
                                         w.list_ent, w.scores));
        DWA_LAUNCH_CHECK("fine_lists_kernel");
        ++g_launches_total;
    } else if (ivf && !want_sf) {
        dim3 gf(static_cast<unsigned>((d.max_list + 255) / 256), w.m_eff, d.B);
        if (dk64)
            DWA_TIMED("fine", st, launch_pdl(fine_kernel<64>, gf, 256, qsh, st, 
                                      w.qw, pool_keys, d.N, d.S, d.d_k, w.m_eff, w.probe_lo,
                                      w.cand_base, w.K_cap, w.scores));
        else
            DWA_TIMED("fine", st, launch_pdl(fine_kernel<0>, gf, 256, qsh, st, 
                                      w.qw, pool_keys, d.N, d.S, d.d_k, w.m_eff, w.probe_lo,
                                      w.cand_base, w.K_cap, w.scores));
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
    sa.row_lo = row_lo;
    sa.summary = shard ? summary : nullptr;
    sa.sf_partial = want_sf ? w.partial : nullptr;
    sa.sf_nblk = sf_blocks;
    sa.sf_stats = shard ? summary + 2 * d.k + 1 : want_sf ? w.stats : nullptr;
    sa.sf_stride = shard ? summary_width(d.k) : 2;
    // one cluster of CL CTAs per query stages the candidates (about 512 per
    // CTA) when they fit, else one block per query re-reads them every pass
    // (candidate sets beyond the cluster's staging capacity are taken in passes)
    int sel_cl = static_cast<int>(std::min<int64_t>(kSelCluster, std::max<int64_t>(1, (w.K_cap + 511) / 512)));
    int64_t local_cap = std::min<int64_t>((w.K_cap + sel_cl - 1) / sel_cl, kSelLocalKeys);
    {
        const size_t ssh = select_cluster_smem(local_cap, sel_cl, d.k);
        {
            // static + dynamic shared memory may pass 48 KB at any size
            int dv = 0;
            DWA_CUDA_TRY(cudaGetDevice(&dv));
            static bool attr_set[64] = {};
            if (dv < 0 || dv >= 64 || !attr_set[dv]) {
                DWA_CUDA_TRY(cudaFuncSetAttribute(select_cluster_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  static_cast<int>(select_cluster_smem(kSelLocalKeys, kSelCluster, kMaxK))));
                if (dv >= 0 && dv < 64) attr_set[dv] = true;
            }
        }
        DWA_TIMED("select", st, launch_pdl_cluster(select_cluster_kernel, dim3(sel_cl, d.B), dim3(kSelThreads), ssh, st,
                                                   dim3(sel_cl, 1, 1), sa, static_cast<int>(local_cap)));
    }
    DWA_LAUNCH_CHECK("select_cluster_kernel");
    ++g_launches_total;
    // 6. normalise soft_full in place with the statistics the selection wrote
    //    (a rank of a sharded call only writes them into its summary; the merge
    //    normalises)
    if (want_sf && !shard) {
        dim3 ga(static_cast<unsigned>((d.N + 2047) / 2048), d.B);
        DWA_TIMED("softmax_apply", st,
                  launch_pdl(softmax_apply_kernel, ga, 256, 0, st, soft_full, d.N, 1.f / d.T, w.stats));
        DWA_LAUNCH_CHECK("softmax_apply_kernel");
        ++g_launches_total;
    }
    return DWA_OK;
}

extern "C" int dwa_retrieve(void* stream, const DwaRetrieveDims* dims, int use_ivf, int is_warmup,
                            const float* lambda_val, const void* z, const float* W_Q,
                            const float* aspect_weights, const float* tau, const float* centroids,
                            const int64_t* list_offsets, const float* pool_keys, float* alphas,
                            int32_t* indices, float* soft_full, void* workspace,
                            size_t workspace_bytes) {
    return retrieve_impl(stream, dims, nullptr, use_ivf, is_warmup, lambda_val, z, W_Q, aspect_weights,
                         tau, centroids, list_offsets, pool_keys, alphas, indices, soft_full, nullptr,
                         workspace, workspace_bytes);
}

extern "C" int dwa_retrieve_local(void* stream, const DwaRetrieveDims* dims, const DwaShard* shard,
                                  int use_ivf, int is_warmup, const float* lambda_val, const void* z,
                                  const float* W_Q, const float* aspect_weights, const float* tau,
                                  const float* centroids, const int64_t* list_offsets,
                                  const float* pool_keys, float* summary, float* soft_full,
                                  void* workspace, size_t workspace_bytes) {
    if (!shard || !dims) return fail(DWA_ERR_INVALID_ARG, "dims and shard are required");
    if (dims->N == 0) {
        // a rank that holds no rows contributes an empty summary
        if (!summary || dims->B <= 0 || dims->k <= 0 || dims->k > kMaxK)
            return fail(DWA_ERR_INVALID_ARG, "summary, B and k (<= 256) are required");
        launch_pdl(empty_summary_kernel, dims->B, 128, 0, static_cast<cudaStream_t>(stream), summary, dims->k);
        DWA_LAUNCH_CHECK("empty_summary_kernel");
        ++g_launches_total;
        return DWA_OK;
    }
    if (shard->row_lo < 0 || shard->n_global <= 0 || shard->row_lo + dims->N > shard->n_global ||
        shard->n_global >= (int64_t(1) << 31))
        return fail(DWA_ERR_INVALID_ARG, "shard rows [row_lo, row_lo + N) must lie in [0, n_global < 2^31)");
    return retrieve_impl(stream, dims, shard, use_ivf, is_warmup, lambda_val, z, W_Q, aspect_weights, tau,
                         centroids, list_offsets, pool_keys, nullptr, nullptr, soft_full, summary, workspace,
                         workspace_bytes);
}

extern "C" size_t dwa_retrieve_merge_workspace_bytes(const DwaRetrieveDims* dims) {
    if (!dims || dims->B <= 0) return 0;
    return 256 + ((static_cast<size_t>(dims->B) * 2 * sizeof(float) + 255) / 256) * 256;
}

extern "C" int dwa_retrieve_merge(void* stream, const DwaRetrieveDims* dims, int world,
                                  const float* summaries, int is_warmup, const float* lambda_val,
                                  const float* tau, float* alphas, int32_t* indices, float* soft_full,
                                  void* workspace, size_t workspace_bytes) {
    if (!dims) return fail(DWA_ERR_INVALID_ARG, "dims is NULL");
    const DwaRetrieveDims& d = *dims;
    if (world < 1 || d.B <= 0 || d.k <= 0 || d.N < 0) return fail(DWA_ERR_INVALID_ARG, "bad world / B / k / N");
    if (d.k > kMaxK) return fail(DWA_ERR_UNSUPPORTED, "k > 256");
    if (static_cast<int64_t>(world) * d.k > 4096) return fail(DWA_ERR_UNSUPPORTED, "world * k > 4096");
    if (!(d.T > 0.f)) return fail(DWA_ERR_INVALID_ARG, "T must be > 0");
    if (!summaries || !lambda_val || !tau || !alphas || !indices)
        return fail(DWA_ERR_INVALID_ARG, "a required pointer is NULL");
    if (!workspace || reinterpret_cast<uintptr_t>(workspace) % 256 != 0)
        return fail(DWA_ERR_WORKSPACE, "workspace must be non-NULL and 256-byte aligned");
    if (workspace_bytes < dwa_retrieve_merge_workspace_bytes(dims))
        return fail(DWA_ERR_WORKSPACE, "workspace too small");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    MergeArgs ma;
    ma.summaries = summaries; ma.world = world; ma.B = d.B; ma.k = d.k; ma.T = d.T;
    ma.is_warmup = is_warmup; ma.lambda_val = lambda_val; ma.tau = tau;
    ma.alphas = alphas; ma.indices = indices;
    ma.status = static_cast<uint32_t*>(workspace);
    float* stats = reinterpret_cast<float*>(static_cast<char*>(workspace) + 256);
    ma.stats = soft_full ? stats : nullptr;
    const size_t msh = static_cast<size_t>(world) * d.k * sizeof(uint64_t);
    DWA_TIMED("merge", st, launch_pdl(merge_kernel, d.B, 1024, msh, st, ma));
    DWA_LAUNCH_CHECK("merge_kernel");
    ++g_launches_total;
    if (soft_full && d.N > 0) {
        dim3 ga(static_cast<unsigned>((d.N + 2047) / 2048), d.B);
        DWA_TIMED("softmax_apply", st, launch_pdl(softmax_apply_kernel, ga, 256, 0, st, soft_full, d.N, 1.f / d.T, stats));
        DWA_LAUNCH_CHECK("softmax_apply_kernel");
        ++g_launches_total;
    }
    return DWA_OK;
}

extern "C" int dwa_sequence_mean(void* stream, int B, int T, int d, int dtype, const void* h_A,
                                 float* z) {
    if (B <= 0 || T <= 0 || d <= 0 || !h_A || !z)
        return fail(DWA_ERR_INVALID_ARG, "dwa_sequence_mean: bad sizes or NULL pointer");
    if (dtype != DWA_F32 && dtype != DWA_BF16) return fail(DWA_ERR_INVALID_ARG, "bad dtype");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int es = dtype == DWA_BF16 ? 2 : 4;
    if (d % 8 == 0 && reinterpret_cast<uintptr_t>(h_A) % 16 == 0) {
        if (dtype == DWA_BF16)
            DWA_TIMED("seq_mean", st, launch_column_sum8(st, static_cast<const __nv_bfloat16*>(h_A), B, T, d, 1, z));
        else
            DWA_TIMED("seq_mean", st, launch_column_sum8(st, static_cast<const float*>(h_A), B, T, d, 1, z));
    } else {
        dim3 g((d + 63) / 64, B);
        if (dtype == DWA_BF16)
            DWA_TIMED("seq_mean", st, launch_pdl(column_sum_kernel<__nv_bfloat16>, g, 1024, 0, st, 
                                          static_cast<const __nv_bfloat16*>(h_A), T, d, 1, z));
        else
            DWA_TIMED("seq_mean", st, launch_pdl(column_sum_kernel<float>, g, 1024, 0, st, 
                                          static_cast<const float*>(h_A), T, d, 1, z));
    }
    (void)es;
    DWA_LAUNCH_CHECK("column_sum_kernel");
    ++g_launches_total;
    return DWA_OK;
}

// ---------------------------------------------------- allocation-free ---
// dwa_retrieve_noalloc runs the retrieval above with its scratch taken from
// this file-scope device array instead of a caller workspace.  Every GPU that
// loads libdwa keeps these 8 MiB until the process exits.  In host code the
// name g_retrieve_scratch is only a stand-in for the symbol, not a device
// address: the address a kernel may use comes from cudaGetSymbolAddress, with
// the device current.  The looked-up address is cached per CUDA context (the
// module, and so the array, is loaded once per context), so a driver-API
// context other than the primary one, or a primary context re-created after
// cudaDeviceReset, gets its own lookup instead of a stale address.
namespace dwa {
constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;
static __device__ __align__(256) unsigned char g_retrieve_scratch[kNoAllocScratchBytes];

using PFN_ctx_current = CUresult (*)(CUcontext*);

static PFN_ctx_current ctx_current_fn() {
    static PFN_ctx_current fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_ctx_current>(p);
    });
    return fn;
}

struct ScratchSlot {
    CUcontext ctx;
    void* addr;
};
constexpr int kScratchSlots = 64;
static std::mutex g_scratch_mu;
static ScratchSlot g_scratch_slots[kScratchSlots];
static int g_scratch_next = 0;

static int scratch_address(void** out) {
    PFN_ctx_current cur = ctx_current_fn();
    if (!cur) return fail(DWA_ERR_CUDA, "cuCtxGetCurrent unavailable");
    CUcontext ctx = nullptr;
    if (cur(&ctx) != CUDA_SUCCESS) return fail(DWA_ERR_CUDA, "cuCtxGetCurrent failed");
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (ctx)
        for (int i = 0; i < kScratchSlots; ++i)
            if (g_scratch_slots[i].ctx == ctx && g_scratch_slots[i].addr) {
                *out = g_scratch_slots[i].addr;
                return DWA_OK;
            }
    // no context yet (this look-up makes the device's primary context current)
    // or a context that has not used the array: look its address up
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_retrieve_scratch);
    if (e != cudaSuccess || p == nullptr)
        return fail(DWA_ERR_CUDA, std::string("cudaGetSymbolAddress(g_retrieve_scratch): ") +
                                      cudaGetErrorString(e));
    if (cur(&ctx) != CUDA_SUCCESS || ctx == nullptr)
        return fail(DWA_ERR_CUDA, "no current CUDA context after the symbol look-up");
    // a context handle can be reused after its context is destroyed: the
    // newest lookup for a handle wins, older slots are recycled round-robin
    g_scratch_slots[g_scratch_next] = ScratchSlot{ctx, p};
    g_scratch_next = (g_scratch_next + 1) % kScratchSlots;
    *out = p;
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

extern "C" int dwa_retrieve_noalloc_status(void* stream, uint32_t* status, int clear) {
    void* scratch = nullptr;
    if (int rc = scratch_address(&scratch)) return rc;
    return dwa_workspace_status(stream, scratch, status, clear);
}
#include "retrieval_bwd.cuh"
