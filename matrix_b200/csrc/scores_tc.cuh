// Tensor-core scan of the key cache (tcgen05 kind::tf32, A operand in TMEM).
//
//   score(row, b) = sum_s  (q[b,s] . k[s,row]) * inv(row, s),
//   inv(row, s)   = 1 / (sqrt(|k[s,row]|^2) + 1e-8)
//
// (src/dwa/retrieval.py:100-118, aspect weights folded into q).  Per aspect the
// dot products of a 128-row tile with all queries are one M=128, N=NQ, K=64
// MMA chain.  fp32 keys and queries are split into tf32 parts, x = hi + lo
// (both exact in tf32), and hi.qhi + hi.qlo + lo.qhi is accumulated in fp32,
// which carries ~22 bits of each operand (the dropped lo.qlo is ~2^-22
// relative).
//
// The keys reach the tensor core from TMEM, not shared memory: with N <= 32 an
// A operand read from shared memory would cost more shared-memory bandwidth
// than the HBM stream delivers.  Shared memory carries the TMA ring, one
// converter read per key and the small query operands.
//
// Persistent CTAs, 384 threads, one per SM, holding two independent pipelines
// (groups g = 0, 1); group g takes the CTA's tiles i with i % 2 == g:
//   warp g        TMA producer: one 128-row x 64-float aspect of a tile per
//                 item (32-row boxes, 128-byte swizzle) into the group's ring
//                 of `stages` slots
//   warp 2 + g    single-thread MMA issuer (warp 2 also allocates 512 TMEM
//                 columns); tcgen05 commits track the issuing thread, so the
//                 two issuers do not wait on each other
//   warps 4+4g..  4 worker warps; thread = tile row = TMEM lane.  Per aspect:
//                 read the row from the ring (conflict-free through the
//                 swizzle), |k|^2 in four partial chains, reciprocal; then,
//                 once the group's previous MMAs have read the A buffer, the
//                 hi/lo split written into it with tcgen05.st.  Per tile:
//                 accumulators -> registers, score per query in aspect order,
//                 output, and (full pass) per-warp online softmax statistics
//                 of s/T.
// TMEM columns: A buffers [0,128) and [128,256) (hi 64 + lo 64 each),
// accumulators [256,384) and [384,512) (S * NQ <= 128 each).
// The same kernel serves the full pass (every pool row) and the fine pass (the
// rows of each query's probed lists), so both give bit-identical scores.
// Every wait is bounded (DWA_STATUS_WAIT_TIMEOUT); at exit each MMA issuer
// waits for its last MMAs before TMEM is released.
#pragma once

#include "key_tiles.cuh"

namespace dwa {
namespace sc {

constexpr int ROWS = 128;                // rows per tile = TMEM lanes = MMA M
constexpr int BOX = 32;                  // rows per TMA box
constexpr uint32_t HALF = ROWS * 128;    // 16 KB: 32 floats x 128 rows
constexpr uint32_t SLOT = 2 * HALF;      // 32 KB: one aspect of one tile
constexpr int MAXS = 8;                  // aspects; S * NQ <= 128 accumulator columns
constexpr int MAX_STAGES = 3;             // ring slots per group
constexpr int THREADS = 384;             // 2 producers, 2 MMA issuers, 8 workers
constexpr int WORKER_WARPS = 8;
constexpr uint32_t TMEM_COLS = 512;
constexpr size_t kSmemLimit = 227 * 1024 - 2048;   // leaves room for static shared memory

// Dynamic shared memory: two rings of `stages` slots, query operands (hi, lo
// per aspect), reciprocal norms [2 groups][MAXS][ROWS], barriers.
inline size_t smem_bytes(int stages, int nq, int S) {
    return 1024 + static_cast<size_t>(2 * stages) * SLOT + static_cast<size_t>(S) * 2 * nq * 256 +
           2 * MAXS * ROWS * sizeof(float) + 256;
}

inline int ring_stages(int nq, int S) {
    int st = MAX_STAGES;
    while (st > 2 && smem_bytes(st, nq, S) > kSmemLimit) --st;
    return st;
}

__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                       uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d),
        "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}

// 32 consecutive 32-bit columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
        "%29, %30, %31, %32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
        "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]),
        "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]),
        "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t tf32_hi(float x) { return __float_as_uint(x) & 0xFFFFE000u; }

// Byte offset of element k (0..63) of row r in a 128-byte-swizzled K-major
// operand made of two 32-float halves of `half_bytes` each.
__device__ __forceinline__ uint32_t sw_off(int r, int k, uint32_t half_bytes) {
    return (k >> 5) * half_bytes + r * 128 + ((((k & 31) >> 2) ^ (r & 7)) << 4) + ((k & 3) << 2);
}

template <int NQ>
__global__ void __launch_bounds__(THREADS, 1) key_scan_tc_kernel(const __grid_constant__ CUtensorMap tm,
                                                                 kt::Args a) {
    static_assert(NQ == 16 || NQ == 32, "N of the MMA: 16 or 32 queries");
    constexpr uint32_t QHALF = NQ * 128;   // one 32-float half of a query operand
    constexpr uint32_t QOP = 2 * QHALF;    // one (aspect, term) query operand
    constexpr int SPL = 32 / NQ;           // aspects per 32-column accumulator load
    constexpr int SMAX = 128 / NQ;         // aspects that fit the accumulator buffer
    // D f32, A/B tf32, both K-major, N = NQ, M = 128
    constexpr uint32_t IDESC = (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(NQ >> 3) << 17) |
                               (static_cast<uint32_t>(ROWS >> 4) << 24);
    extern __shared__ uint8_t dyn[];
    const int stages = a.stages, S = a.S;   // stages: ring slots per group
    uint8_t* rings = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dyn) + 1023) & ~uintptr_t(1023));
    uint8_t* qop = rings + static_cast<size_t>(2 * stages) * SLOT;            // [S][2][QOP]
    float* inv_tab = reinterpret_cast<float*>(qop + static_cast<size_t>(S) * 2 * QOP);  // [2][MAXS][ROWS]
    uint64_t* bars = reinterpret_cast<uint64_t*>(inv_tab + 2 * MAXS * ROWS);
    // per group g: raw_full[stages], raw_free[stages], a_full, a_free, d_full, drain
    const int nbar = 2 * stages + 4;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * nbar);
    __shared__ float red_m[WORKER_WARPS][32], red_z[WORKER_WARPS][32];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_enter();   // the queries come from the previous kernel
    // role: warps 0-1 producers, 2-3 MMA issuers, 4-7 / 8-11 workers of group 0 / 1
    const int g = warp < 4 ? (warp & 1) : ((warp - 4) >> 2);
    uint8_t* ring = rings + static_cast<size_t>(g * stages) * SLOT;
    uint64_t* raw_full = bars + g * nbar;
    uint64_t* raw_free = raw_full + stages;
    uint64_t* a_full = raw_free + stages;   // 4 worker warps: A buffer written
    uint64_t* a_free = a_full + 1;          // MMA commit: A buffer read
    uint64_t* d_full = a_free + 1;          // MMA commit: tile accumulated
    uint64_t* drain = d_full + 1;           // MMA commit at exit

    // query operands: hi / lo tf32 parts in the swizzled K-major layout
    for (int i = threadIdx.x; i < S * NQ * 64; i += blockDim.x) {
        const int k = i & 63, b = (i >> 6) % NQ, s = i / (64 * NQ);
        const float v = b < a.B ? a.qw[(static_cast<int64_t>(b) * S + s) * 64 + k] : 0.f;
        const float hi = __uint_as_float(tf32_hi(v)), lo = __uint_as_float(tf32_hi(v - hi));
        const uint32_t o = sw_off(b, k, QHALF);
        *reinterpret_cast<float*>(qop + (s * 2 + 0) * QOP + o) = hi;
        *reinterpret_cast<float*>(qop + (s * 2 + 1) * QOP + o) = lo;
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    if (threadIdx.x == 0) {
        tc::prefetch_tmap(&tm);
        for (int gg = 0; gg < 2; ++gg) {
            uint64_t* b = bars + gg * nbar;
            for (int i = 0; i < stages; ++i) {
                tc::mbar_init(&b[i], 1);
                tc::mbar_init(&b[stages + i], 4);
            }
            tc::mbar_init(&b[2 * stages + 0], 4);
            tc::mbar_init(&b[2 * stages + 1], 1);
            tc::mbar_init(&b[2 * stages + 2], 1);
            tc::mbar_init(&b[2 * stages + 3], 1);
        }
        tc::fence_barrier_init();
    }
    if (warp == 2) {
        tc::tmem_alloc(tmem_slot, TMEM_COLS);
        tc::tmem_relinquish();
        tc::tc_fence_before();
    }
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    int64_t row_lo, row_hi;
    const int ntile = kt::tile_count<ROWS, BOX>(a, blockIdx.x, gridDim.x, row_lo, row_hi);
    auto tile = [&](int i) { return kt::tile_at<ROWS>(a, i, blockIdx.x, gridDim.x, row_lo, row_hi); };

    if (warp < 2) {
        // ------------------------------------------------------- producer of group g
        if (lane == 0) {
            int it = 0;
            bool ok = true;
            for (int i = g; i < ntile && ok; i += 2) {
                const kt::Tile t = tile(i);
                if (!t.valid) continue;
                const int nbox = (t.rows + BOX - 1) / BOX;
                for (int s = 0; s < S; ++s, ++it) {
                    const int slot = it % stages;
                    if (it >= stages && !tc::mbar_wait_bounded(&raw_free[slot], ((it / stages) - 1) & 1)) {
                        raise_status(a.status, DWA_STATUS_WAIT_TIMEOUT);
                        ok = false;
                        break;
                    }
                    const int y = static_cast<int>(static_cast<int64_t>(s) * a.N + t.row0);
                    uint8_t* dst = ring + static_cast<size_t>(slot) * SLOT;
                    tc::mbar_arrive_expect_tx(&raw_full[slot], static_cast<uint32_t>(nbox) * BOX * 256);
                    for (int bx = 0; bx < nbox; ++bx) {
                        kt::tma_load_2d(dst + bx * BOX * 128, &tm, &raw_full[slot], 0, y + bx * BOX);
                        kt::tma_load_2d(dst + HALF + bx * BOX * 128, &tm, &raw_full[slot], 32, y + bx * BOX);
                    }
                }
            }
            // drain: the last issued loads must have landed before exit
            for (int i = (it > stages ? it - stages : 0); i < it; ++i)
                if (!tc::mbar_wait_bounded(&raw_full[i % stages], (i / stages) & 1)) {
                    raise_status(a.status, DWA_STATUS_WAIT_TIMEOUT);
                    break;
                }
        }
        __syncwarp();
    } else if (warp < 4) {
        // ------------------------------------------------------- MMA issuer of group g
        if (lane == 0) {
            int cnt = 0;
            bool ok = true;
            const uint32_t ahi = tmem + g * 128, alo = ahi + 64;
            for (int i = g; i < ntile && ok; i += 2) {
                if (!tile(i).valid) continue;
                for (int s = 0; s < S; ++s, ++cnt) {
                    if (!tc::mbar_wait_bounded(a_full, cnt & 1)) {
                        raise_status(a.status, DWA_STATUS_WAIT_TIMEOUT);
                        ok = false;
                        break;
                    }
                    tc::tc_fence_after();
                    const uint32_t d = tmem + 256 + g * 128 + s * NQ;
                    const uint32_t bhi = tc::smem_u32(qop + (s * 2 + 0) * QOP);
                    const uint32_t blo = tc::smem_u32(qop + (s * 2 + 1) * QOP);
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                        const uint32_t ob = (kk >> 2) * QHALF + (kk & 3) * 32;
                        const uint64_t dbh = tc::sw128_desc(bhi + ob, 16, 1024);
                        const uint64_t dbl = tc::sw128_desc(blo + ob, 16, 1024);
                        mma_ts(d, ahi + kk * 8, dbh, IDESC, kk > 0 ? 1u : 0u);
                        mma_ts(d, ahi + kk * 8, dbl, IDESC, 1u);
                        mma_ts(d, alo + kk * 8, dbh, IDESC, 1u);
                    }
                    tc::mma_commit(a_free);
                    if (s == S - 1) tc::mma_commit(d_full);
                }
            }
            // every issued MMA has completed before TMEM is released
            tc::mma_commit(drain);
            if (!tc::mbar_wait_bounded(drain, 0)) raise_status(a.status, DWA_STATUS_WAIT_TIMEOUT);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------- workers of group g
        const int q = warp & 3, r = q * 32 + lane;
        const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
        const uint32_t A = tmem + lane_addr + g * 128, D = tmem + lane_addr + 256 + g * 128;
        float* inv_g = inv_tab + g * MAXS * ROWS;
        const float invT = a.invT;
        float m_run = -INFINITY, z_run = 0.f;   // lane j: statistics of query j over this warp's rows
        int it = 0, n_tiles = 0;
        bool ok = true;
        for (int i = g; i < ntile && ok; i += 2) {
            const kt::Tile t = tile(i);
            if (!t.valid) continue;
            for (int s = 0; s < S; ++s, ++it) {
                const int slot = it % stages;
                if (!tc::mbar_wait_bounded(&raw_full[slot], (it / stages) & 1)) {
                    if (lane == 0) raise_status(a.status, DWA_STATUS_WAIT_TIMEOUT);
                    ok = false;
                    break;
                }
                float4 v[16];
                const uint8_t* rp = ring + static_cast<size_t>(slot) * SLOT + r * 128;
#pragma unroll
                for (int c = 0; c < 16; ++c)
                    v[c] = *reinterpret_cast<const float4*>(rp + (c >> 3) * HALF + (((c & 7) ^ (r & 7)) << 4));
                __syncwarp();
                if (lane == 0) kt::mbar_arrive(&raw_free[slot]);
                // |k|^2 as four interleaved partial chains
                float n4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int c = 0; c < 16; ++c) {
                    float& n = n4[c & 3];
                    n = fmaf(v[c].x, v[c].x, n);
                    n = fmaf(v[c].y, v[c].y, n);
                    n = fmaf(v[c].z, v[c].z, n);
                    n = fmaf(v[c].w, v[c].w, n);
                }
                inv_g[s * ROWS + r] = 1.f / (sqrtf((n4[0] + n4[1]) + (n4[2] + n4[3])) + 1e-8f);
                // the A buffer is free once the MMAs of this group's previous aspect completed
                if (it >= 1 && !tc::mbar_wait_bounded(a_free, (it - 1) & 1)) {
                    if (lane == 0) raise_status(a.status, DWA_STATUS_WAIT_TIMEOUT);
                    ok = false;
                    break;
                }
                tc::tc_fence_after();
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    uint32_t hi[32], lo[32];
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        const float4 x = v[h * 8 + c];
                        hi[c * 4 + 0] = tf32_hi(x.x);
                        hi[c * 4 + 1] = tf32_hi(x.y);
                        hi[c * 4 + 2] = tf32_hi(x.z);
                        hi[c * 4 + 3] = tf32_hi(x.w);
                        lo[c * 4 + 0] = tf32_hi(x.x - __uint_as_float(hi[c * 4 + 0]));
                        lo[c * 4 + 1] = tf32_hi(x.y - __uint_as_float(hi[c * 4 + 1]));
                        lo[c * 4 + 2] = tf32_hi(x.z - __uint_as_float(hi[c * 4 + 2]));
                        lo[c * 4 + 3] = tf32_hi(x.w - __uint_as_float(hi[c * 4 + 3]));
                    }
                    tmem_st32(A + h * 32, hi);
                    tmem_st32(A + 64 + h * 32, lo);
                }
                tmem_wait_st();
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) kt::mbar_arrive(a_full);
            }
            if (!ok) break;
            // ---- epilogue of this group's tile
            if (!tc::mbar_wait_bounded(d_full, n_tiles & 1)) {
                if (lane == 0) raise_status(a.status, DWA_STATUS_WAIT_TIMEOUT);
                ok = false;
                break;
            }
            tc::tc_fence_after();
            ++n_tiles;
            float sc[NQ];
#pragma unroll
            for (int j = 0; j < NQ; ++j) sc[j] = 0.f;
#pragma unroll
            for (int s2 = 0; s2 < SMAX; s2 += SPL) {
                if (s2 < S) {
                    float dv[32];
                    tc::tmem_ld32(D + s2 * NQ, dv);
#pragma unroll
                    for (int u = 0; u < SPL; ++u) {
                        if (s2 + u < S) {
                            const float inv = inv_g[(s2 + u) * ROWS + r];
#pragma unroll
                            for (int j = 0; j < NQ; ++j) sc[j] = fmaf(dv[u * NQ + j], inv, sc[j]);
                        }
                    }
                }
            }
            tc::tc_fence_before();
            const bool valid = r < t.rows;
            if (a.mode == 0) {
                const int64_t n = t.row0 + r;
#pragma unroll
                for (int j = 0; j < NQ; ++j) {
                    if (j < a.B) {
                        if (valid) a.out[static_cast<int64_t>(j) * a.N + n] = sc[j];
                        const float x = valid ? sc[j] * invT : -INFINITY;
                        const float mt = warp_max(x);
                        if (mt != -INFINITY) {
                            const float zt = warp_sum(__expf(x - mt));
                            if (lane == j) {
                                const float mn = fmaxf(m_run, mt);
                                z_run = z_run * __expf(m_run - mn) + zt * __expf(mt - mn);
                                m_run = mn;
                            }
                        }
                    }
                }
            } else if (valid) {
                float v = 0.f;
#pragma unroll
                for (int j = 0; j < NQ; ++j) v = (j == t.b) ? sc[j] : v;
                a.out[static_cast<int64_t>(t.b) * a.K_cap + t.obase + r] = v;
            }
        }
        if (a.mode == 0) {
            // CTA reduction of the online statistics (worker warps only)
            const int w = warp - 4;
            red_m[w][lane] = m_run;
            red_z[w][lane] = z_run;
            asm volatile("bar.sync 1, %0;" ::"r"(WORKER_WARPS * 32) : "memory");
            if (w == 0 && lane < a.B && lane < NQ) {
                const int j = lane;
                float M = -INFINITY;
                for (int u = 0; u < WORKER_WARPS; ++u) M = fmaxf(M, red_m[u][j]);
                float Z = 0.f;
                for (int u = 0; u < WORKER_WARPS; ++u)
                    if (red_m[u][j] != -INFINITY) Z += red_z[u][j] * expf(red_m[u][j] - M);
                a.partial[(static_cast<int64_t>(j) * gridDim.x + blockIdx.x) * 2] = M;
                a.partial[(static_cast<int64_t>(j) * gridDim.x + blockIdx.x) * 2 + 1] = Z;
            }
        }
    }
    __syncthreads();
    if (warp == 2) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, TMEM_COLS);
    }
}

}  // namespace sc
}  // namespace dwa
