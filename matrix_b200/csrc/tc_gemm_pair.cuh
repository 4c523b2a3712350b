// Persistent bf16 GEMM on CTA pairs (tcgen05 cta_group::2).
//
// A cluster of two CTAs on neighbouring SMs computes 256 x BN output tiles with
// M = 256 MMAs issued by the even CTA (the leader): each CTA stages its own 128
// rows of A and its own BN/2 columns of B per k-block, and the pair's MMA reads
// both halves, so a CTA moves (128 + BN/2) x 64 operand elements per k-block
// for a 128 x BN share of the tile where a single-CTA 128 x BN tile moves
// (128 + BN) x 64: a third less operand traffic through L2 at BN = 256.  The
// accumulator rows 0-127 live in the leader's TMEM, rows 128-255 in the
// peer's; each CTA drains its own with the per-warp epilogue of the persistent
// kernel.
//   full[s]       leader only: its producer's arrive + expect_tx of both CTAs'
//                 bytes; both CTAs' TMA loads complete_tx on it
//   empty[s]      each CTA: the leader's MMA commit, signalled to the pair
//   acc_full[b]   each CTA: the leader's commit of a finished tile, signalled to the pair
//   acc_empty[b]  leader only: one arrive per epilogue warp of both CTAs
// Every mbarrier wait is bounded; both CTAs reach the two cluster barriers
// (after set-up, before teardown) on every path.  No TMA load here uses
// cluster multicast: each CTA loads only into its own shared memory.
#pragma once

#include "tc_gemm.cuh"

namespace dwa {
namespace tc {

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// shared::cluster address of the variable at `addr` in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// mbar_wait_bounded with cluster-scope acquire (arrivals from the peer CTA)
static __device__ __noinline__ bool mbar_wait_bounded_cluster(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
        if (mbar_try_wait_cluster(bar, parity)) return true;
        if (global_timer_ns() - t0 > kWaitLimitNs) return false;
    }
}
// TMA load into this CTA's shared memory whose completion is counted on the
// leader's barrier (a shared::cluster address)
__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* tm, uint32_t bar_cluster, int c0,
                                                 int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(bar_cluster), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}
__device__ __forceinline__ void mma_bf16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// arrive on the barrier at this offset in both CTAs of the pair once the
// issuing thread's MMAs complete
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
    asm volatile(
        "{\n\t.reg .b16 m;\n\t"
        "mov.b16 m, 3;\n\t"
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}\n" ::"r"(
            smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

template <int BN, int STAGES, int EW = kPersEpiWarps>
struct PairSmem {
    static constexpr uint32_t A_STAGE = BM * BK * 2;          // this CTA's 128 rows of A
    static constexpr uint32_t B_STAGE = (BN / 2) * BK * 2;    // this CTA's BN/2 columns of B
    static constexpr uint32_t RING = STAGES * (A_STAGE + B_STAGE);
    static constexpr uint32_t STAGE_LD = 33;
    static constexpr uint32_t WARP_STAGE = 32 * STAGE_LD * 4;
    static constexpr uint32_t EPI_OFF = RING;
    static constexpr uint32_t BAR_OFF = EPI_OFF + EW * WARP_STAGE;
    static constexpr uint32_t NBAR = 2 * STAGES + 5;        // full, empty, acc_full[2], acc_empty[2], drain
    static constexpr uint32_t BYTES = 1024 + BAR_OFF + NBAR * 8 + 16;
    static_assert(BYTES <= 227 * 1024, "pair GEMM shared memory above the per-CTA limit");
};

// Instruction descriptor of a cta_group::2 kind::f16 MMA: D fp32, A/B bf16, M = 256.
template <int BN, bool A_MN, bool B_MN>
__host__ __device__ constexpr uint32_t instr_desc_bf16_pair() {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((A_MN ? 1u : 0u) << 15) | ((B_MN ? 1u : 0u) << 16) |
           (static_cast<uint32_t>(BN >> 3) << 17) | (static_cast<uint32_t>((2 * BM) >> 4) << 24);
}

template <int BN, int STAGES, bool A_MN, bool B_MN, class Epi, int EW = kPersEpiWarps>
__global__ void __launch_bounds__(gemm_threads<EW>(), 1)
    gemm_bf16_pair(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M, int N,
                   int K, int batch, int a_batched, int b_batched, Epi epi, uint32_t* status) {
    static_assert(BN == 256, "pair GEMM: BN 256 (N = 256 MMAs, 128 B columns per CTA)");
    using L = PairSmem<BN, STAGES, EW>;
    constexpr int PM = 2 * BM;                  // rows of a pair tile
    constexpr int HBN = BN / 2;                 // B columns staged per CTA
    constexpr uint32_t TMEM_COLS = 2 * BN;
    extern __shared__ uint8_t dyn_smem[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(dyn_smem) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * L::A_STAGE;
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
    uint64_t* empty_bar = full_bar + STAGES;
    uint64_t* acc_full = empty_bar + STAGES;
    uint64_t* acc_empty = acc_full + 2;
    uint64_t* drain_bar = acc_empty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
    __shared__ float s_red[EW];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
    const int tiles_n = (N + BN - 1) / BN, tiles_m = (M + PM - 1) / PM;
    const int tiles = tiles_n * tiles_m * batch;
    const int nkb = (K + BK - 1) / BK;

    if (threadIdx.x == 0) {
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 2 * EW);
        }
        mbar_init(drain_bar, 1);
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, TMEM_COLS);
        tmem_relinquish_pair();
        tc_fence_before();
    }
    __syncthreads();
    cluster_sync_all();       // both CTAs' barriers initialised before any cross-CTA signal
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_enter();   // operands and epilogue inputs come from earlier kernels

    if (warp == 0) {
        if (lane == 0) {
            // both CTAs load their halves; the leader expects the pair's bytes
            int it = 0;
            bool ok = true;
            for (int t = pair; t < tiles && ok; t += npairs) {
                const int n0 = (t % tiles_n) * BN, m0 = ((t / tiles_n) % tiles_m) * PM + static_cast<int>(rank) * BM;
                const int bz = t / (tiles_n * tiles_m);
                const int za = a_batched ? bz : 0, zb = b_batched ? bz : 0;
                const int nb0 = n0 + static_cast<int>(rank) * HBN;
                for (int kb = 0; kb < nkb; ++kb, ++it) {
                    const int s = it % STAGES;
                    if (it >= STAGES && !mbar_wait_bounded(&empty_bar[s], ((it / STAGES) - 1) & 1)) {
                        raise_status(status, DWA_STATUS_WAIT_TIMEOUT);
                        ok = false;
                        break;
                    }
                    const uint32_t fb = mapa_shared(smem_u32(&full_bar[s]), 0);
                    if (leader) mbar_arrive_expect_tx(&full_bar[s], 2 * (L::A_STAGE + L::B_STAGE));
                    const int k0 = kb * BK;
                    uint8_t* a = sA + s * L::A_STAGE;
                    uint8_t* b = sB + s * L::B_STAGE;
                    if (A_MN) {
#pragma unroll
                        for (int h = 0; h < BM / 64; ++h) tma_load_3d_pair(a + h * 8192, &tmA, fb, m0 + 64 * h, k0, za);
                    } else {
                        tma_load_3d_pair(a, &tmA, fb, k0, m0, za);
                    }
                    if (B_MN) {
#pragma unroll
                        for (int h = 0; h < HBN / 64; ++h) tma_load_3d_pair(b + h * 8192, &tmB, fb, nb0 + 64 * h, k0, zb);
                    } else {
                        tma_load_3d_pair(b, &tmB, fb, k0, nb0, zb);
                    }
                }
            }
            // the leader's full barriers count both CTAs' bytes: every issued
            // copy of the pair has landed once its last phases complete
            if (leader)
                for (int i = (it > STAGES ? it - STAGES : 0); i < it; ++i)
                    if (!mbar_wait_bounded(&full_bar[i % STAGES], (i / STAGES) & 1)) {
                        raise_status(status, DWA_STATUS_WAIT_TIMEOUT);
                        break;
                    }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            constexpr uint32_t idesc = instr_desc_bf16_pair<BN, A_MN, B_MN>();
            int it = 0, li = 0;
            bool ok = true;
            for (int t = pair; t < tiles && ok; t += npairs, ++li) {
                const int buf = li & 1;
                if (li >= 2 && !mbar_wait_bounded_cluster(&acc_empty[buf], ((li >> 1) - 1) & 1)) {
                    raise_status(status, DWA_STATUS_WAIT_TIMEOUT);
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem + static_cast<uint32_t>(buf * BN);
                for (int kb = 0; kb < nkb; ++kb, ++it) {
                    const int s = it % STAGES;
                    if (!mbar_wait_bounded(&full_bar[s], (it / STAGES) & 1)) {
                        raise_status(status, DWA_STATUS_WAIT_TIMEOUT);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_base = smem_u32(sA + s * L::A_STAGE);
                    const uint32_t b_base = smem_u32(sB + s * L::B_STAGE);
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk)
                        mma_bf16_pair(d_tmem, operand_desc<A_MN>(a_base, kk), operand_desc<B_MN>(b_base, kk), idesc,
                                      (kb | kk) != 0 ? 1u : 0u);
                    mma_commit_pair(&empty_bar[s]);
                }
                if (ok) mma_commit_pair(&acc_full[buf]);
            }
            // every MMA this thread issued has completed before TMEM is released
            mma_commit_pair(drain_bar);
            if (!mbar_wait_bounded(drain_bar, 0)) raise_status(status, DWA_STATUS_WAIT_TIMEOUT);
        }
        __syncwarp();
    } else {
        const int q = warp & 3;        // TMEM lane quarter this warp may read
        const int e = warp - 2;        // epilogue warp 0..EW-1
        const int grp = e >> 2;        // column group 0..EW/4-1
        constexpr int LD = L::STAGE_LD;
        constexpr int CPW = BN / 32 / (EW / 4);     // chunks per warp and tile
        static_assert(CPW >= 1 && (BN / 32) % (EW / 4) == 0, "column chunks split evenly over the groups");
        constexpr bool PRE = sizeof(typename Epi::Frag) <= 40;   // registers for two chunks' operands
        float* stg = reinterpret_cast<float*>(smem + L::EPI_OFF + e * L::WARP_STAGE);
        const int fr_row = lane >> 2, fr_col = (lane & 3) * 8;   // fragment: row within 8, first column
        typename Epi::Frag nxt[4];
        auto load_chunk = [&](int t, int ci, typename Epi::Frag* f) {
            if (t >= tiles) return;
            const int n0 = (t % tiles_n) * BN, m0 = ((t / tiles_n) % tiles_m) * PM + static_cast<int>(rank) * BM;
            const int bz = t / (tiles_n * tiles_m);
            const int col0 = n0 + (grp + ci * (EW / 4)) * 32 + fr_col, cnt = min(8, N - col0);
#pragma unroll
            for (int it = 0; it < 4; ++it) {
                const int row = m0 + q * 32 + it * 8 + fr_row;
                if (row < M && cnt > 0) epi.load(bz, row, col0, cnt, f[it]);
            }
        };
        if (PRE) load_chunk(pair, 0, nxt);
        int li = 0;
        for (int t = pair; t < tiles; t += npairs, ++li) {
            const int n0 = (t % tiles_n) * BN, m0 = ((t / tiles_n) % tiles_m) * PM + static_cast<int>(rank) * BM;
            const int bz = t / (tiles_n * tiles_m);
            const int buf = li & 1;
            const bool ok = mbar_wait_bounded(&acc_full[buf], (li >> 1) & 1);
            if (!epi_all<EW>(ok)) {
                if (lane == 0) raise_status(status, DWA_STATUS_WAIT_TIMEOUT);
                break;
            }
            tc_fence_after();
            float cta_acc = 0.f;
#pragma unroll 1
            for (int ci = 0; ci < CPW; ++ci) {
                const int c = grp + ci * (EW / 4);
                const int col0 = n0 + c * 32 + fr_col, cnt = min(8, N - col0);
                typename Epi::Frag frag[4];
                if constexpr (PRE) {
#pragma unroll
                    for (int it = 0; it < 4; ++it) frag[it] = nxt[it];
                    if (ci + 1 < CPW) load_chunk(t, ci + 1, nxt);
                    else load_chunk(t + npairs, 0, nxt);
                } else {
                    load_chunk(t, ci, frag);
                }
                float v[32];
                tmem_ld32(tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(buf * BN + c * 32), v);
                if (ci == CPW - 1) {           // this warp's part of the accumulator read out
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_remote(mapa_shared(smem_u32(&acc_empty[buf]), 0));
                }
                __syncwarp();                  // the previous chunk's staging reads are done
#pragma unroll
                for (int i = 0; i < 32; ++i) stg[lane * LD + i] = v[i];
                __syncwarp();
#pragma unroll
                for (int it = 0; it < 4; ++it) {
                    const int rr = it * 8 + fr_row, row = m0 + q * 32 + rr;
                    float part = 0.f;
                    if (row < M && cnt > 0) {
                        float w8[8];
#pragma unroll
                        for (int i = 0; i < 8; ++i) w8[i] = stg[rr * LD + fr_col + i];
                        part = epi.finish(bz, row, col0, w8, cnt, frag[it]);
                    }
                    if (Epi::kReduce == 1) {
                        part += __shfl_xor_sync(0xffffffffu, part, 1);
                        part += __shfl_xor_sync(0xffffffffu, part, 2);
                        if ((lane & 3) == 0 && row < M && cnt > 0) epi.row_done(bz, row, part);
                    } else if (Epi::kReduce == 2) {
                        cta_acc += part;
                    }
                }
            }
            if (Epi::kReduce == 2) {
                cta_acc = warp_sum(cta_acc);
                if (lane == 0) s_red[e] = cta_acc;
                asm volatile("bar.sync 1, %0;" ::"n"(32 * EW) : "memory");
                if (e == 0 && lane == 0) {
                    float tsum = 0.f;
                    for (int i = 0; i < EW; ++i) tsum += s_red[i];
                    epi.cta_done(bz, tsum);
                }
            }
        }
    }
    __syncthreads();
    cluster_sync_all();       // the pair's MMAs and copies are done with both CTAs' memory
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, TMEM_COLS);
    }
}

template <int BN, int STAGES, bool A_MN, bool B_MN, class Epi, int EW = kPersEpiWarps>
int launch_gemm_bf16_pair(const Operand& A, const Operand& B, int M, int N, int K, int batch, const Epi& epi,
                          uint32_t* status, cudaStream_t stream) {
    CUtensorMap ta, tb;
    std::string why;
    if (!make_operand_map(&ta, A, M, K, batch, BM, &why) || !make_operand_map(&tb, B, N, K, batch, BN / 2, &why))
        return fail(DWA_ERR_INVALID_ARG, "tensor map: " + why);
    using L = PairSmem<BN, STAGES, EW>;
    auto kern = gemm_bf16_pair<BN, STAGES, A_MN, B_MN, Epi, EW>;
    static bool attr_set[64] = {};  // per instantiation and device
    int dev = 0;
    DWA_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        DWA_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(L::BYTES)));
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    const int64_t tiles = static_cast<int64_t>((N + BN - 1) / BN) * ((M + 2 * BM - 1) / (2 * BM)) * batch;
    const int pairs = static_cast<int>(std::min<int64_t>(tiles, sm_count() / 2));
    DWA_CUDA_TRY(launch_pdl_cluster(kern, dim3(2 * pairs), dim3(gemm_threads<EW>()), L::BYTES, stream, dim3(2, 1, 1),
                                    ta, tb, M, N, K, batch, static_cast<int>(A.bstride != 0),
                                    static_cast<int>(B.bstride != 0), epi, status));
    DWA_LAUNCH_CHECK("gemm_bf16_pair");
    return DWA_OK;
}

}  // namespace tc
}  // namespace dwa
