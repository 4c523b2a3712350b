// Key-cache scan on the CUDA cores: scores of key rows against the queries.
//
//   score(row, b) = sum_s  (q[b,s] . k[s,row]) * inv(row, s),
//   inv(row, s)   = 1 / (sqrt(|k[s,row]|^2) + 1e-8)
//
// (src/dwa/retrieval.py:100-118, aspect weights folded into q).  With B <= 16
// queries there are at most 17 FMAs per key float, so the scan can be bound by
// HBM; what limits a CUDA-core version is shared memory: every query value a
// thread multiplies is a broadcast load that costs one wavefront per float per
// warp.  A thread therefore scores R rows at once (R = 4 for B <= 8), so each
// query load feeds R rows: per 56 KB of keys about 1.3K wavefront-cycles of
// shared memory and 1K cycles of FMA issue per SM against 2.5K cycles of HBM.
//
// Persistent CTAs of 256 threads (one per SM, ~180 KB shared memory):
//   warp 0      TMA producer: per item one quarter-aspect (16 floats) of a
//               tile of ROWS = 224*R rows, as 64-row boxes with 64-byte
//               swizzle, into a ring of `stages` 56 KB slots; partial tiles
//               load only the boxes they need
//   warps 1-7   consumers: thread t of consumer warp w scores rows
//               w*32R + 32i + lane (i < R).  Per item, 4R conflict-free
//               16-byte loads take its rows' 16 floats into registers and the
//               slot is released at once; per 4 floats one broadcast load per
//               query feeds 4R FMAs, with the |k|^2 chains alongside.  After the last
//               quarter of an aspect: one IEEE reciprocal per row and
//               score += dot * inv per (row, query).
// Full pass: rows split over the CTAs as in key_tiles.cuh; writes s_full
// [B, N] (coalesced per query) and the online softmax statistics of s/T per
// query (per warp and tile: max and sum of exp over its rows, merged into lane
// j's running pair for query j) -> partial [B, grid, 2].  Fine pass: tiles of
// the probed lists of each query (query b only), written to scores [B, K_cap].
// A (row, query) score is the same FMA chain in the same order in both passes,
// so the two passes give bit-identical scores.  Every wait is bounded
// (DWA_STATUS_WAIT_TIMEOUT).
#pragma once

#include "key_tiles.cuh"

namespace dwa {
namespace ks {

// 8 warps: every SM sub-partition holds 2, so a thread may use 255 registers
// (R*16 key floats and 2*R*QB accumulators live at once).
constexpr int CONSUMER_WARPS = 7;
constexpr int THREADS = 32 + 32 * CONSUMER_WARPS;   // 256
constexpr int BOX = 64;                  // rows per TMA box (4 KB)
constexpr int KQ = 16;                   // floats per row per item (a quarter of d_k = 64)
constexpr int MAX_QB = 16;
constexpr size_t kSmemLimit = 227 * 1024 - 4096;   // leaves room for static shared memory

// Rows per thread for a query block of QB queries (registers: R*16 key floats,
// R*QB dot and score accumulators).
template <int QB> constexpr int rows_per_thread() { return 4; }
template <int QB> constexpr int tile_rows() { return 32 * rows_per_thread<QB>() * CONSUMER_WARPS; }
template <int QB> constexpr uint32_t slot_bytes() { return tile_rows<QB>() * KQ * 4; }

// With 16 query chains the dot products run as packed pairs of queries
// (fma.rn.f32x2: lane h of a pair is exactly fmaf(k, q_{2p+h}, dot), so the
// scores are bit-identical to scalar FMAs in the same order), which halves the
// FMA instructions of the loop.
template <int QB> constexpr bool paired() { return QB > 8; }

// Dynamic shared memory for `stages` slots and nq x S query vectors (and,
// for paired queries, the same vectors interleaved by query pair).
template <int QB>
inline size_t smem_bytes(int stages, int nq, int S) {
    return 1024 + static_cast<size_t>(stages) * slot_bytes<QB>() +
           static_cast<size_t>(nq) * S * 64 * sizeof(float) * (paired<QB>() ? 2 : 1) +
           2 * static_cast<size_t>(stages) * 8;
}

__device__ __forceinline__ unsigned long long pack2(float lo, float hi) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void unpack2(unsigned long long v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
// d.lo = fma(a.lo, b.lo, d.lo), d.hi = fma(a.hi, b.hi, d.hi), round to nearest
__device__ __forceinline__ void ffma2(unsigned long long& d, unsigned long long a, unsigned long long b) {
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(d) : "l"(a), "l"(b));
}

// QB: queries scored per row (full pass, B <= QB, padded with zero queries);
// FINE: the fine pass (one query per tile, chains of query t.b only).
template <int QB, bool FINE>
__global__ void __launch_bounds__(THREADS, 1) key_scan_kernel(const __grid_constant__ CUtensorMap tm,
                                                              kt::Args a) {
    constexpr int CW = CONSUMER_WARPS;
    constexpr int R = rows_per_thread<QB>();
    constexpr int ROWS = tile_rows<QB>();
    constexpr uint32_t SLOT = slot_bytes<QB>();
    constexpr int J = FINE ? 1 : QB;   // query chains per row
    constexpr bool PAIRED = !FINE && paired<QB>();
    extern __shared__ uint8_t dyn[];
    const int stages = a.stages, S = a.S;
    uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dyn) + 1023) & ~uintptr_t(1023));
    const int nq = FINE ? a.B : QB;    // query vectors staged
    float* qs = reinterpret_cast<float*>(ring + static_cast<size_t>(stages) * SLOT);   // [nq][S][64]
    // paired queries: [S][32 element pairs][QB/2 query pairs][2 elements][2 queries]
    float* qp = qs + nq * S * 64;
    uint64_t* full = reinterpret_cast<uint64_t*>(qp + (PAIRED ? nq * S * 64 : 0));
    uint64_t* empty = full + stages;
    __shared__ float red_m[CW][32], red_z[CW][32];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        tc::prefetch_tmap(&tm);
        for (int i = 0; i < stages; ++i) {
            tc::mbar_init(&full[i], 1);
            tc::mbar_init(&empty[i], CW);
        }
        tc::fence_barrier_init();
    }
    __syncthreads();
    pdl_enter();   // the queries come from the previous kernel

    int64_t row_lo, row_hi;
    const int ntile = kt::tile_count<ROWS, BOX>(a, blockIdx.x, gridDim.x, row_lo, row_hi);

    if (warp == 0) {
        // ------------------------------------------------------- producer
        if (lane == 0) {
            int it = 0;
            bool ok = true;
            for (int i = 0; i < ntile && ok; ++i) {
                const kt::Tile t = kt::tile_at<ROWS>(a, i, blockIdx.x, gridDim.x, row_lo, row_hi);
                if (!t.valid) continue;
                const int nbox = (t.rows + BOX - 1) / BOX;
                for (int s = 0; s < S && ok; ++s) {
                    for (int kq = 0; kq < 4; ++kq, ++it) {
                        const int slot = it % stages;
                        if (it >= stages && !tc::mbar_wait_bounded(&empty[slot], ((it / stages) - 1) & 1)) {
                            raise_status(a.status, DWA_STATUS_WAIT_TIMEOUT);
                            ok = false;
                            break;
                        }
                        const int y = static_cast<int>(static_cast<int64_t>(s) * a.N + t.row0);
                        uint8_t* dst = ring + static_cast<size_t>(slot) * SLOT;
                        tc::mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(nbox) * BOX * KQ * 4);
                        for (int bx = 0; bx < nbox; ++bx)
                            kt::tma_load_2d(dst + bx * BOX * KQ * 4, &tm, &full[slot], kq * KQ, y + bx * BOX);
                    }
                }
            }
            // drain: the last issued loads must have landed before exit
            for (int i = (it > stages ? it - stages : 0); i < it; ++i)
                if (!tc::mbar_wait_bounded(&full[i % stages], (i / stages) & 1)) {
                    raise_status(a.status, DWA_STATUS_WAIT_TIMEOUT);
                    break;
                }
        }
        __syncwarp();
        return;
    }

    // ----------------------------------------------------------- consumers
    // the queries are staged while the producer's first loads are in flight
    for (int i = threadIdx.x - 32; i < nq * S * 16; i += 32 * CW) {
        const int qb = i / (S * 16);
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (qb < a.B) v = reinterpret_cast<const float4*>(a.qw)[i];
        reinterpret_cast<float4*>(qs)[i] = v;
        if constexpr (PAIRED) {
            const int rem = i - qb * S * 16, s4 = rem >> 4, e0 = (rem & 15) * 4;   // aspect, first element
            const float x[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int e = e0 + u;
                qp[((s4 * 32 + (e >> 1)) * (QB / 2) + (qb >> 1)) * 4 + (e & 1) * 2 + (qb & 1)] = x[u];
            }
        }
    }
    asm volatile("bar.sync 2, %0;" ::"r"(CW * 32) : "memory");
    const int cw = warp - 1;
    const int rbase = cw * 32 * R + lane;   // tile row of chain i: rbase + 32*i
    const float invT = a.invT;
    float m_run = -INFINITY, z_run = 0.f;   // lane j: statistics of query j over this warp's rows
    int it = 0;
    bool ok = true;
    for (int ti = 0; ti < ntile && ok; ++ti) {
        const kt::Tile t = kt::tile_at<ROWS>(a, ti, blockIdx.x, gridDim.x, row_lo, row_hi);
        if (!t.valid) continue;
        const bool warp_active = cw * 32 * R < t.rows;
        const float* qt = FINE ? qs + t.b * S * 64 : qs;
        constexpr int JD = PAIRED ? 1 : J;     // scalar dot chains (the paired ones live in dot2)
        constexpr int JP = PAIRED ? J / 2 : 1;
        float sc[R][J], dot[R][JD], nrm[R];
        unsigned long long dot2[R][JP];
#pragma unroll
        for (int i = 0; i < R; ++i) {
            nrm[i] = 0.f;
#pragma unroll
            for (int j = 0; j < J; ++j) sc[i][j] = 0.f;
#pragma unroll
            for (int j = 0; j < JD; ++j) dot[i][j] = 0.f;
#pragma unroll
            for (int p = 0; p < JP; ++p) dot2[i][p] = 0ull;
        }
        for (int s = 0; s < S && ok; ++s) {
            for (int kq = 0; kq < 4; ++kq, ++it) {
                const int slot = it % stages;
                if (!tc::mbar_wait_bounded(&full[slot], (it / stages) & 1)) {
                    if (lane == 0) raise_status(a.status, DWA_STATUS_WAIT_TIMEOUT);
                    ok = false;
                    break;
                }
                if (!warp_active) {
                    __syncwarp();
                    if (lane == 0) kt::mbar_arrive(&empty[slot]);
                    continue;
                }
                const uint8_t* sp = ring + static_cast<size_t>(slot) * SLOT;
                const float* qa = qt + s * 64 + kq * KQ;   // query j of this quarter: qa + j*S*64
                if constexpr (PAIRED) {
                    // query pair p of element pair ep: qp + ((s*32 + ep)*(J/2) + p)*4
                    const float* qpa = qp + (s * 32 + kq * (KQ / 2)) * (J / 2) * 4;
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        float4 kc[R];
#pragma unroll
                        for (int i = 0; i < R; ++i) {
                            const int rr = rbase + 32 * i;
                            kc[i] = *reinterpret_cast<const float4*>(sp + rr * (KQ * 4) + ((c ^ ((rr >> 1) & 3)) << 4));
                        }
#pragma unroll
                        for (int i = 0; i < R; ++i) {
                            nrm[i] = fmaf(kc[i].x, kc[i].x, nrm[i]);
                            nrm[i] = fmaf(kc[i].y, kc[i].y, nrm[i]);
                            nrm[i] = fmaf(kc[i].z, kc[i].z, nrm[i]);
                            nrm[i] = fmaf(kc[i].w, kc[i].w, nrm[i]);
                        }
                        unsigned long long kx[R], ky[R], kz[R], kw[R];
#pragma unroll
                        for (int i = 0; i < R; ++i) {
                            kx[i] = pack2(kc[i].x, kc[i].x);
                            ky[i] = pack2(kc[i].y, kc[i].y);
                            kz[i] = pack2(kc[i].z, kc[i].z);
                            kw[i] = pack2(kc[i].w, kc[i].w);
                        }
#pragma unroll
                        for (int p = 0; p < J / 2; ++p) {
                            // (q_2p, q_2p+1) of elements 4c, 4c+1 and of 4c+2, 4c+3
                            const ulonglong2 b01 = *reinterpret_cast<const ulonglong2*>(qpa + ((2 * c) * (J / 2) + p) * 4);
                            const ulonglong2 b23 = *reinterpret_cast<const ulonglong2*>(qpa + ((2 * c + 1) * (J / 2) + p) * 4);
                            // component-major: the R rows' chains are independent, so a
                            // chain's next FMA is R instructions after its last
#pragma unroll
                            for (int i = 0; i < R; ++i) ffma2(dot2[i][p], kx[i], b01.x);
#pragma unroll
                            for (int i = 0; i < R; ++i) ffma2(dot2[i][p], ky[i], b01.y);
#pragma unroll
                            for (int i = 0; i < R; ++i) ffma2(dot2[i][p], kz[i], b23.x);
#pragma unroll
                            for (int i = 0; i < R; ++i) ffma2(dot2[i][p], kw[i], b23.y);
                        }
                    }
                    __syncwarp();
                    if (lane == 0) kt::mbar_arrive(&empty[slot]);
                } else if constexpr (J > 8) {
                    // 16 query chains: the key registers hold one float4 chunk of
                    // the R rows at a time (the accumulators take the rest), and
                    // the slot is released after the last chunk
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        float4 kc[R];
#pragma unroll
                        for (int i = 0; i < R; ++i) {
                            const int rr = rbase + 32 * i;
                            kc[i] = *reinterpret_cast<const float4*>(sp + rr * (KQ * 4) + ((c ^ ((rr >> 1) & 3)) << 4));
                        }
#pragma unroll
                        for (int i = 0; i < R; ++i) {
                            nrm[i] = fmaf(kc[i].x, kc[i].x, nrm[i]);
                            nrm[i] = fmaf(kc[i].y, kc[i].y, nrm[i]);
                            nrm[i] = fmaf(kc[i].z, kc[i].z, nrm[i]);
                            nrm[i] = fmaf(kc[i].w, kc[i].w, nrm[i]);
                        }
#pragma unroll
                        for (int j = 0; j < J; ++j) {
                            const float4 qv = *reinterpret_cast<const float4*>(qa + j * S * 64 + c * 4);
#pragma unroll
                            for (int i = 0; i < R; ++i) {
                                dot[i][j] = fmaf(kc[i].x, qv.x, dot[i][j]);
                                dot[i][j] = fmaf(kc[i].y, qv.y, dot[i][j]);
                                dot[i][j] = fmaf(kc[i].z, qv.z, dot[i][j]);
                                dot[i][j] = fmaf(kc[i].w, qv.w, dot[i][j]);
                            }
                        }
                    }
                    __syncwarp();
                    if (lane == 0) kt::mbar_arrive(&empty[slot]);
                } else {
                float4 kv[R][4];
#pragma unroll
                for (int i = 0; i < R; ++i) {
                    const int rr = rbase + 32 * i;
#pragma unroll
                    for (int c = 0; c < 4; ++c)
                        kv[i][c] = *reinterpret_cast<const float4*>(sp + rr * (KQ * 4) + ((c ^ ((rr >> 1) & 3)) << 4));
                }
                __syncwarp();
                if (lane == 0) kt::mbar_arrive(&empty[slot]);
#pragma unroll
                for (int c = 0; c < 4; ++c) {
#pragma unroll
                    for (int i = 0; i < R; ++i) {
                        nrm[i] = fmaf(kv[i][c].x, kv[i][c].x, nrm[i]);
                        nrm[i] = fmaf(kv[i][c].y, kv[i][c].y, nrm[i]);
                        nrm[i] = fmaf(kv[i][c].z, kv[i][c].z, nrm[i]);
                        nrm[i] = fmaf(kv[i][c].w, kv[i][c].w, nrm[i]);
                    }
#pragma unroll
                    for (int j = 0; j < J; ++j) {
                        const float4 qv = *reinterpret_cast<const float4*>(qa + j * S * 64 + c * 4);
#pragma unroll
                        for (int i = 0; i < R; ++i) {
                            dot[i][j] = fmaf(kv[i][c].x, qv.x, dot[i][j]);
                            dot[i][j] = fmaf(kv[i][c].y, qv.y, dot[i][j]);
                            dot[i][j] = fmaf(kv[i][c].z, qv.z, dot[i][j]);
                            dot[i][j] = fmaf(kv[i][c].w, qv.w, dot[i][j]);
                        }
                    }
                }
                }
                if (kq == 3) {
#pragma unroll
                    for (int i = 0; i < R; ++i) {
                        const float inv = 1.f / (sqrtf(nrm[i]) + 1e-8f);
                        if constexpr (PAIRED) {
#pragma unroll
                            for (int p = 0; p < JP; ++p) {
                                float lo, hi;
                                unpack2(dot2[i][p], lo, hi);
                                sc[i][2 * p] = fmaf(lo, inv, sc[i][2 * p]);
                                sc[i][2 * p + 1] = fmaf(hi, inv, sc[i][2 * p + 1]);
                                dot2[i][p] = 0ull;
                            }
                        } else {
#pragma unroll
                            for (int j = 0; j < J; ++j) { sc[i][j] = fmaf(dot[i][j], inv, sc[i][j]); dot[i][j] = 0.f; }
                        }
                        nrm[i] = 0.f;
                    }
                }
            }
        }
        if (!ok || !warp_active) continue;
        if (!FINE) {
#pragma unroll
            for (int j = 0; j < QB; ++j) {
                if (j < a.B) {
                    float x[R], mt = -INFINITY;
#pragma unroll
                    for (int i = 0; i < R; ++i) {
                        const int rr = rbase + 32 * i;
                        const bool valid = rr < t.rows;
                        if (valid) a.out[static_cast<int64_t>(j) * a.N + t.row0 + rr] = sc[i][j];
                        x[i] = valid ? sc[i][j] * invT : -INFINITY;
                        mt = fmaxf(mt, x[i]);
                    }
                    mt = warp_max(mt);
                    if (mt != -INFINITY) {
                        float e = 0.f;
#pragma unroll
                        for (int i = 0; i < R; ++i) e += __expf(x[i] - mt);
                        const float zt = warp_sum(e);
                        if (lane == j) {
                            const float mn = fmaxf(m_run, mt);
                            z_run = z_run * __expf(m_run - mn) + zt * __expf(mt - mn);
                            m_run = mn;
                        }
                    }
                }
            }
        } else {
#pragma unroll
            for (int i = 0; i < R; ++i) {
                const int rr = rbase + 32 * i;
                if (rr < t.rows) a.out[static_cast<int64_t>(t.b) * a.K_cap + t.obase + rr] = sc[i][0];
            }
        }
    }
    if (!FINE) {
        // CTA reduction of the online statistics (consumer warps only)
        red_m[cw][lane] = m_run;
        red_z[cw][lane] = z_run;
        asm volatile("bar.sync 1, %0;" ::"r"(CW * 32) : "memory");
        if (cw == 0 && lane < a.B && lane < QB) {
            const int j = lane;
            float M = -INFINITY;
            for (int w = 0; w < CW; ++w) M = fmaxf(M, red_m[w][j]);
            float Z = 0.f;
            for (int w = 0; w < CW; ++w)
                if (red_m[w][j] != -INFINITY) Z += red_z[w][j] * expf(red_m[w][j] - M);
            a.partial[(static_cast<int64_t>(j) * gridDim.x + blockIdx.x) * 2] = M;
            a.partial[(static_cast<int64_t>(j) * gridDim.x + blockIdx.x) * 2 + 1] = Z;
        }
    }
}

}  // namespace ks
}  // namespace dwa
