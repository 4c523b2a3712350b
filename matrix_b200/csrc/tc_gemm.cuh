// Batched bf16 GEMM on the sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
//   C[b](m, n) = sum_k A[b](m, k) * B[b](n, k)      fp32 accumulation in TMEM
//
// followed by a caller-supplied epilogue functor that receives each output row
// segment in registers.  Either operand may be K-major (k contiguous) or
// MN-major (m / n contiguous); both are staged by TMA with the 128-byte
// swizzle and consumed directly by tcgen05.mma through shared-memory matrix
// descriptors, so no transposes are materialised in HBM.
//
// CTA tile 128 x BN x 64, STAGES-deep TMA ring, one CTA per output tile:
//   warp 0      TMA producer (one elected lane)
//   warp 1      TMEM allocator + MMA issuer (one elected lane)
//   warps 2..17 epilogue: tcgen05.ld into a shared fp32 tile, then a coalesced
//               pass (8 columns per lane) through the epilogue functor
// Every mbarrier wait is bounded (kWaitLimitNs); a wait that runs out sets
// DWA_STATUS_WAIT_TIMEOUT in the status word and the CTA winds down, freeing
// its TMEM.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include "dwa_common.cuh"

namespace dwa {
namespace tc {

constexpr int BM = 128;
constexpr int BK = 64;  // bf16 elements per k-block = 128 bytes = one swizzle row

// Host description of one operand.  Element (mn, k) of batch item b lives at
//   K-major : ptr + b*bstride + mn*ld + k
//   MN-major: ptr + b*bstride + k*ld + mn
// (element units).  bstride == 0 means the operand is shared by all items.
struct Operand {
    const void* ptr;
    bool mn_major;
    int64_t ld;
    int64_t bstride;
};

// ------------------------------------------------------------------ PTX ----
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for the phase with the given parity to complete; gives up after
// kWaitLimitNs and returns false.
static __device__ __noinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (global_timer_ns() - t0 > kWaitLimitNs) return false;
    }
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* tm) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tm)) : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* tm, uint64_t* bar, int c0,
                                            int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(slot)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void mma_bf16_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane; the wait is part of
// the same statement, so no use of the registers can be scheduled before it.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor, 128-byte swizzle, sm_100 format:
// start>>4 [0,14), LBO>>4 [16,30), SBO>>4 [32,46), version=1 [46,48),
// base offset 0 [49,52), layout SWIZZLE_128B = 2 [61,64).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1) << 46;
    d |= static_cast<uint64_t>(2) << 61;
    return d;
}

// Instruction descriptor of tcgen05.mma kind::f16: D fp32, A/B bf16, M=128.
template <int BN, bool A_MN, bool B_MN>
__host__ __device__ constexpr uint32_t instr_desc_bf16() {
    return (1u << 4)                       // D format: f32
           | (1u << 7)                     // A format: bf16
           | (1u << 10)                    // B format: bf16
           | ((A_MN ? 1u : 0u) << 15)      // A major: 0 = K, 1 = MN
           | ((B_MN ? 1u : 0u) << 16)      // B major
           | (static_cast<uint32_t>(BN >> 3) << 17)
           | (static_cast<uint32_t>(BM >> 4) << 24);
}

// Descriptor of k-step kk (16 elements) inside one staged k-block.
// K-major: rows of 128 B, 8-row atoms 1024 B apart; advance 32 B per k-step.
// MN-major: 64-element MN chunks (8 KB each, one TMA box of 64 k-rows) LBO
// apart; 8 k-rows per 1024 B atom; advance 16 k-rows = 2048 B per k-step.
template <bool MN>
__device__ __forceinline__ uint64_t operand_desc(uint32_t base, int kk) {
    if (MN) return sw128_desc(base + kk * 2048, 8192, 1024);
    return sw128_desc(base + kk * 32, 16, 1024);
}

template <int BN, int STAGES>
struct SmemLayout {
    static constexpr uint32_t A_STAGE = BM * BK * 2;
    static constexpr uint32_t B_STAGE = BN * BK * 2;
    static constexpr uint32_t BAR_OFF = STAGES * (A_STAGE + B_STAGE);
    // the epilogue reuses the stage buffers for the fp32 accumulator tile
    static_assert(BM * (BN + 4) * 4 <= BAR_OFF, "epilogue tile must fit in the stage buffers");
    static constexpr uint32_t BYTES = 1024 /*align slack*/ + BAR_OFF + (2 * STAGES + 1) * 8 + 16;
};

// Epilogue protocol.  Epi provides
//   struct Frag;  void load(int b, int row, int col0, int cnt, Frag&) const
//   float finish(int b, int row, int col0, const float* v, int cnt, const Frag&) const
//     v[0..cnt) = C[b](row, col0 + i), cnt <= 8 (col0 a multiple of 8 when
//     cnt == 8); returns a partial for the reductions;
//   static constexpr int kReduce;   0 none, 1 per row, 2 per CTA
//   void row_done(int b, int row, float acc) const   (kReduce == 1)
//   void cta_done(int b, float acc) const            (kReduce == 2)
// EW epilogue warps (16: one CTA per SM; 8: with BN = 128 and 3 stages two CTAs
// fit on an SM, so one CTA's epilogue overlaps the other's mainloop).
constexpr int kEpiWarps = 16;
template <int EW> constexpr int gemm_threads() { return 64 + 32 * EW; }   // + TMA warp + MMA warp
constexpr int kGemmThreads = gemm_threads<kEpiWarps>();

template <int BN, int STAGES, bool A_MN, bool B_MN, class Epi, int EW = kEpiWarps>
__global__ void __launch_bounds__(gemm_threads<EW>(), EW == 8 ? 2 : 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     int M, int N, int K, int a_batched, int b_batched, Epi epi, uint32_t* status) {
    using L = SmemLayout<BN, STAGES>;
    constexpr uint32_t TMEM_COLS = BN;
    extern __shared__ uint8_t dyn_smem[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(dyn_smem) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * L::A_STAGE;
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
    uint64_t* empty_bar = full_bar + STAGES;
    uint64_t* done_bar = empty_bar + STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
    __shared__ float s_red[EW];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM, bz = blockIdx.z;
    const int nkb = (K + BK - 1) / BK;

    if (threadIdx.x == 0) {
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        mbar_init(done_bar, 1);
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, TMEM_COLS);
        tmem_relinquish();
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_enter();   // operands and epilogue inputs come from earlier kernels

    if (warp == 0) {
        if (lane == 0) {
            const int za = a_batched ? bz : 0, zb = b_batched ? bz : 0;
            int issued = 0;
            for (int kb = 0; kb < nkb; ++kb) {
                const int s = kb % STAGES;
                if (kb >= STAGES && !mbar_wait_bounded(&empty_bar[s], ((kb / STAGES) - 1) & 1)) {
                    raise_status(status, DWA_STATUS_WAIT_TIMEOUT);
                    break;
                }
                mbar_arrive_expect_tx(&full_bar[s], L::A_STAGE + L::B_STAGE);
                const int k0 = kb * BK;
                uint8_t* a = sA + s * L::A_STAGE;
                uint8_t* b = sB + s * L::B_STAGE;
                if (A_MN) {
#pragma unroll
                    for (int h = 0; h < BM / 64; ++h)
                        tma_load_3d(a + h * 8192, &tmA, &full_bar[s], m0 + 64 * h, k0, za);
                } else {
                    tma_load_3d(a, &tmA, &full_bar[s], k0, m0, za);
                }
                if (B_MN) {
#pragma unroll
                    for (int h = 0; h < BN / 64; ++h)
                        tma_load_3d(b + h * 8192, &tmB, &full_bar[s], n0 + 64 * h, k0, zb);
                } else {
                    tma_load_3d(b, &tmB, &full_bar[s], k0, n0, zb);
                }
                issued = kb + 1;
            }
            // Drain: wait until every issued copy has landed before the CTA may exit.
            for (int kb = (issued > STAGES ? issued - STAGES : 0); kb < issued; ++kb)
                if (!mbar_wait_bounded(&full_bar[kb % STAGES], (kb / STAGES) & 1)) {
                    raise_status(status, DWA_STATUS_WAIT_TIMEOUT);
                    break;
                }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = instr_desc_bf16<BN, A_MN, B_MN>();
            for (int kb = 0; kb < nkb; ++kb) {
                const int s = kb % STAGES;
                if (!mbar_wait_bounded(&full_bar[s], (kb / STAGES) & 1)) {
                    raise_status(status, DWA_STATUS_WAIT_TIMEOUT);
                    break;
                }
                tc_fence_after();
                const uint32_t a_base = smem_u32(sA + s * L::A_STAGE);
                const uint32_t b_base = smem_u32(sB + s * L::B_STAGE);
#pragma unroll
                for (int kk = 0; kk < BK / 16; ++kk)
                    mma_bf16_ss(tmem, operand_desc<A_MN>(a_base, kk), operand_desc<B_MN>(b_base, kk),
                                idesc, (kb | kk) != 0 ? 1u : 0u);
                mma_commit(&empty_bar[s]);
            }
            mma_commit(done_bar);
        }
        __syncwarp();
    } else {
        // Epilogue.  Phase 1: TMEM -> shared tile (fp32, row stride BN+4 floats),
        // thread = row; warp w may only read TMEM lanes 32*(w%4).., so the EW
        // warps form EW/4 column groups of one warp per lane quarter.  The stage
        // buffers are free: every TMA load was consumed by an MMA and done_bar
        // fires after the last MMA completes.
        const int q = warp & 3;
        const int e = warp - 2;        // epilogue warp 0..EW-1
        const int grp = e >> 2;        // column group 0..EW/4-1
        const bool ok = mbar_wait_bounded(done_bar, 0);
        if (!ok && lane == 0) raise_status(status, DWA_STATUS_WAIT_TIMEOUT);
        tc_fence_after();
        constexpr int LD = BN + 4;
        float* tile = reinterpret_cast<float*>(smem);
        if (ok) {
            const int r_local = q * 32 + lane;
            for (int c = grp; c < BN / 32; c += EW / 4) {
                if (n0 + c * 32 >= N) break;
                float v[32];
                tmem_ld32(tmem + (static_cast<uint32_t>(q * 32) << 16) + c * 32, v);
                float4* dst = reinterpret_cast<float4*>(tile + r_local * LD + c * 32);
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
            }
        }
        tc_fence_before();
        asm volatile("bar.sync 1, %0;" ::"n"(32 * EW) : "memory");
        // Phase 2: coalesced.  LPR lanes cover one row (8 columns each); each
        // warp first loads the epilogue operands of PF rows, then finishes them.
        constexpr int LPR = BN / 8, RPW = 32 / LPR, PF = 4;
        constexpr int STEP = EW * RPW;
        const int sub = lane / LPR, li = lane % LPR;
        const int col0 = n0 + li * 8;
        const int cnt = min(8, N - col0);
        float cta_acc = 0.f;
        if (ok) {
            for (int base = e * RPW + sub; base < BM; base += STEP * PF) {
                typename Epi::Frag frag[PF];
#pragma unroll
                for (int u = 0; u < PF; ++u) {
                    const int rr = base + u * STEP, row = m0 + rr;
                    if (rr < BM && row < M && cnt > 0) epi.load(bz, row, col0, cnt, frag[u]);
                }
#pragma unroll
                for (int u = 0; u < PF; ++u) {
                    const int rr = base + u * STEP, row = m0 + rr;
                    float part = 0.f;
                    if (rr < BM && row < M && cnt > 0) {
                        const float4* src = reinterpret_cast<const float4*>(tile + rr * LD + li * 8);
                        const float4 a = src[0], b = src[1];
                        const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
                        part = epi.finish(bz, row, col0, v, cnt, frag[u]);
                    }
                    if (Epi::kReduce == 1) {
#pragma unroll
                        for (int o = LPR / 2; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
                        if (li == 0 && rr < BM && row < M) epi.row_done(bz, row, part);
                    } else if (Epi::kReduce == 2) {
                        cta_acc += part;
                    }
                }
            }
        }
        if (Epi::kReduce == 2) {
            cta_acc = warp_sum(cta_acc);
            if (lane == 0) s_red[e] = cta_acc;
        }
    }
    __syncthreads();
    if (Epi::kReduce == 2 && threadIdx.x == 0) {
        float t = 0.f;
        for (int i = 0; i < EW; ++i) t += s_red[i];
        epi.cta_done(bz, t);
    }
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

// --------------------------------------------------- persistent variant ---
// One CTA per SM loops over the output tiles (tile t = blockIdx.x + i *
// gridDim.x, column block fastest, then row block, then batch item, so the
// CTAs running at once share their operands in L2).  Two TMEM accumulators
// (2 x BN columns): while the epilogue warps drain tile i from one, the MMA
// warp accumulates tile i+1 into the other, and the producer keeps the TMA
// ring full across tile boundaries.  Eight epilogue warps (320 threads, so a
// thread may hold 168 registers) each drain 32 x 32 chunks through their own
// 4 KB staging area beside the ring, with no block-wide barrier inside a tile.
//   acc_full[buf]   MMA commit: tile accumulated in buffer buf
//   acc_empty[buf]  one arrive per epilogue warp: buffer buf read out
constexpr int kPersEpiWarps = 8;
template <int BN, int STAGES, int EW = kPersEpiWarps>
struct PSmem {
    static constexpr uint32_t A_STAGE = BM * BK * 2;
    static constexpr uint32_t B_STAGE = BN * BK * 2;
    static constexpr uint32_t RING = STAGES * (A_STAGE + B_STAGE);
    static constexpr uint32_t STAGE_LD = 33;                 // floats per staged row: conflict-free scalar access
    static constexpr uint32_t WARP_STAGE = 32 * STAGE_LD * 4;  // one warp's 32 x 32 chunk
    static constexpr uint32_t EPI_OFF = RING;
    static constexpr uint32_t BAR_OFF = EPI_OFF + EW * WARP_STAGE;
    static constexpr uint32_t NBAR = 2 * STAGES + 5;        // full, empty, acc_full[2], acc_empty[2], drain
    static constexpr uint32_t BYTES = 1024 + BAR_OFF + NBAR * 8 + 16;
    static_assert(BYTES <= 227 * 1024, "persistent GEMM shared memory above the per-CTA limit");
};

// True on every epilogue thread when `ok` holds on all of them (named barrier 1).
template <int EW>
__device__ __forceinline__ bool epi_all(bool ok) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 q, %1, 0;\n\t"
        "bar.red.and.pred p, 1, %2, q;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(r)
        : "r"(static_cast<uint32_t>(ok)), "n"(32 * EW)
        : "memory");
    return r != 0;
}

template <int BN, int STAGES, bool A_MN, bool B_MN, class Epi, int EW = kPersEpiWarps>
__global__ void __launch_bounds__(gemm_threads<EW>(), 1)
    gemm_bf16_persistent(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                         int M, int N, int K, int batch, int a_batched, int b_batched, Epi epi,
                         uint32_t* status) {
    using L = PSmem<BN, STAGES, EW>;
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
    const int tiles_n = (N + BN - 1) / BN, tiles_m = (M + BM - 1) / BM;
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
            mbar_init(&acc_empty[b], EW);
        }
        mbar_init(drain_bar, 1);
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, TMEM_COLS);
        tmem_relinquish();
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_enter();   // operands and epilogue inputs come from earlier kernels

    if (warp == 0) {
        if (lane == 0) {
            int it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
                const int n0 = (t % tiles_n) * BN, m0 = ((t / tiles_n) % tiles_m) * BM;
                const int bz = t / (tiles_n * tiles_m);
                const int za = a_batched ? bz : 0, zb = b_batched ? bz : 0;
                for (int kb = 0; kb < nkb; ++kb, ++it) {
                    const int s = it % STAGES;
                    if (it >= STAGES && !mbar_wait_bounded(&empty_bar[s], ((it / STAGES) - 1) & 1)) {
                        raise_status(status, DWA_STATUS_WAIT_TIMEOUT);
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full_bar[s], L::A_STAGE + L::B_STAGE);
                    const int k0 = kb * BK;
                    uint8_t* a = sA + s * L::A_STAGE;
                    uint8_t* b = sB + s * L::B_STAGE;
                    if (A_MN) {
#pragma unroll
                        for (int h = 0; h < BM / 64; ++h)
                            tma_load_3d(a + h * 8192, &tmA, &full_bar[s], m0 + 64 * h, k0, za);
                    } else {
                        tma_load_3d(a, &tmA, &full_bar[s], k0, m0, za);
                    }
                    if (B_MN) {
#pragma unroll
                        for (int h = 0; h < BN / 64; ++h)
                            tma_load_3d(b + h * 8192, &tmB, &full_bar[s], n0 + 64 * h, k0, zb);
                    } else {
                        tma_load_3d(b, &tmB, &full_bar[s], k0, n0, zb);
                    }
                }
            }
            // every issued copy must have landed before the CTA may exit
            for (int i = (it > STAGES ? it - STAGES : 0); i < it; ++i)
                if (!mbar_wait_bounded(&full_bar[i % STAGES], (i / STAGES) & 1)) {
                    raise_status(status, DWA_STATUS_WAIT_TIMEOUT);
                    break;
                }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = instr_desc_bf16<BN, A_MN, B_MN>();
            int it = 0, li = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++li) {
                const int buf = li & 1;
                if (li >= 2 && !mbar_wait_bounded(&acc_empty[buf], ((li >> 1) - 1) & 1)) {
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
                        mma_bf16_ss(d_tmem, operand_desc<A_MN>(a_base, kk), operand_desc<B_MN>(b_base, kk),
                                    idesc, (kb | kk) != 0 ? 1u : 0u);
                    mma_commit(&empty_bar[s]);
                }
                if (ok) mma_commit(&acc_full[buf]);
            }
            // every MMA this thread issued has completed before TMEM is released
            mma_commit(drain_bar);
            if (!mbar_wait_bounded(drain_bar, 0)) raise_status(status, DWA_STATUS_WAIT_TIMEOUT);
        }
        __syncwarp();
    } else {
        // Each epilogue warp drains its own 32 x 32 chunks: TMEM lane quarter
        // q = warp % 4 (the lanes it may read), chunks grp, grp + EW/4, ... of
        // the tile's BN/32 column chunks.  A chunk goes TMEM -> registers (row
        // per lane) -> the warp's own staging area -> registers again with
        // four lanes per row and eight columns each, so the epilogue's global
        // loads and stores are coalesced; only __syncwarp orders the staging,
        // and the warps proceed independently within a tile.  The epilogue
        // operands of the warp's next chunk (this tile's, or its next tile's
        // first) are loaded before the current chunk is drained.
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
            const int n0 = (t % tiles_n) * BN, m0 = ((t / tiles_n) % tiles_m) * BM;
            const int bz = t / (tiles_n * tiles_m);
            const int col0 = n0 + (grp + ci * (EW / 4)) * 32 + fr_col, cnt = min(8, N - col0);
#pragma unroll
            for (int it = 0; it < 4; ++it) {
                const int row = m0 + q * 32 + it * 8 + fr_row;
                if (row < M && cnt > 0) epi.load(bz, row, col0, cnt, f[it]);
            }
        };
        if (PRE) load_chunk(blockIdx.x, 0, nxt);
        int li = 0;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++li) {
            const int n0 = (t % tiles_n) * BN, m0 = ((t / tiles_n) % tiles_m) * BM;
            const int bz = t / (tiles_n * tiles_m);
            const int buf = li & 1;
            const bool ok = mbar_wait_bounded(&acc_full[buf], (li >> 1) & 1);
            // every epilogue thread leaves together, or none does (the named
            // barrier of the per-CTA reduction must be reached by all of them)
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
                    else load_chunk(t + gridDim.x, 0, nxt);
                } else {
                    load_chunk(t, ci, frag);
                }
                float v[32];
                tmem_ld32(tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(buf * BN + c * 32), v);
                if (ci == CPW - 1) {           // this warp's part of the accumulator read out
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&acc_empty[buf]);
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
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

// ------------------------------------------------------------------ host ---
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

// Builds the 3-D tensor map {inner, outer, batch} of an operand for the box
// the kernel loads.  Returns false (with a message) when TMA cannot address it.
bool make_operand_map(CUtensorMap* tm, const Operand& op, int64_t mn_extent, int64_t k_extent,
                      int batch, int box_mn, std::string* why);

// True when the operand satisfies the TMA rules (16-byte aligned base and
// strides) and covers at least one full box in each dimension.
bool tc_operand_ok(const Operand& op, int64_t mn_extent, int64_t k_extent, int box_mn);

template <int BN, int STAGES, bool A_MN, bool B_MN, class Epi, int EW = kEpiWarps>
int launch_gemm_bf16(const Operand& A, const Operand& B, int M, int N, int K, int batch,
                     const Epi& epi, uint32_t* status, cudaStream_t stream) {
    static_assert(BN % 64 == 0 && BN >= 64 && BN <= 256, "BN must be 64, 128, 192 or 256");
    static_assert(BN == 64 || BN == 128 || BN == 256, "TMEM allocation needs a power of two");
    CUtensorMap ta, tb;
    std::string why;
    if (!make_operand_map(&ta, A, M, K, batch, BM, &why) ||
        !make_operand_map(&tb, B, N, K, batch, BN, &why))
        return fail(DWA_ERR_INVALID_ARG, "tensor map: " + why);
    using L = SmemLayout<BN, STAGES>;
    auto kern = gemm_bf16_kernel<BN, STAGES, A_MN, B_MN, Epi, EW>;
    static bool attr_set[64] = {};  // per instantiation and device
    int dev = 0;
    DWA_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        DWA_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(L::BYTES)));
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM, batch);
    launch_pdl(kern, grid, gemm_threads<EW>(), L::BYTES, stream, ta, tb, M, N, K, A.bstride != 0, B.bstride != 0,
                                                   epi, status);
    DWA_LAUNCH_CHECK("gemm_bf16_kernel");
    return DWA_OK;
}


int sm_count();
bool pair_gemm();   // CTA-pair kernel allowed (DWA_GEMM not classic / single)
bool persistent_gemm();

template <int BN, int STAGES, bool A_MN, bool B_MN, class Epi, int EW = kPersEpiWarps>
int launch_gemm_bf16_persistent(const Operand& A, const Operand& B, int M, int N, int K, int batch,
                                const Epi& epi, uint32_t* status, cudaStream_t stream) {
    static_assert(BN == 128 || BN == 256, "persistent GEMM: BN 128 or 256");
    CUtensorMap ta, tb;
    std::string why;
    if (!make_operand_map(&ta, A, M, K, batch, BM, &why) ||
        !make_operand_map(&tb, B, N, K, batch, BN, &why))
        return fail(DWA_ERR_INVALID_ARG, "tensor map: " + why);
    using L = PSmem<BN, STAGES, EW>;
    auto kern = gemm_bf16_persistent<BN, STAGES, A_MN, B_MN, Epi, EW>;
    static bool attr_set[64] = {};  // per instantiation and device
    int dev = 0;
    DWA_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        DWA_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(L::BYTES)));
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    const int64_t tiles = static_cast<int64_t>((N + BN - 1) / BN) * ((M + BM - 1) / BM) * batch;
    const int grid = static_cast<int>(std::min<int64_t>(tiles, sm_count()));
    launch_pdl(kern, dim3(grid), gemm_threads<EW>(), L::BYTES, stream, ta, tb, M, N, K, batch,
               A.bstride != 0, B.bstride != 0, epi, status);
    DWA_LAUNCH_CHECK("gemm_bf16_persistent");
    return DWA_OK;
}

}  // namespace tc
}  // namespace dwa
