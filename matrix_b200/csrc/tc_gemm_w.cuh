// The assembled weight W[b] = W_base + acc[b] (acc = the factor product) as a
// persistent tcgen05 GEMM whose epilogue moves W_base in and W (fp32) and
// W_act (bf16) out with TMA instead of per-thread loads and stores.
//
// Mainloop, producer and MMA warps as in gemm_bf16_persistent (two TMEM
// accumulators, one CTA per SM looping over 128 x 256 tiles); BN = 256 and
// three ring stages, which leave room for the epilogue's staging.  Each of
// the 8 epilogue warps drains 32 x 32 chunks of its TMEM lane quarter:
//   - lane 0 loads the chunk's W_base box (32 x 32 fp32, 128-byte swizzle)
//     into one of the warp's two fp32 slots, one chunk ahead (per-slot
//     mbarrier, bounded wait);
//   - lane r (row r of the chunk) reads its accumulator row from TMEM, adds
//     its W_base row from the slot (16-byte chunk c of row r sits at c ^ (r%8),
//     so the 32 lanes' accesses spread over the banks), writes the fp32 sum
//     back in place and its bf16 copy into the warp's bf16 slot (64-byte
//     swizzle: chunk c of row r at c ^ ((r/2)%4));
//   - lane 0 stores both boxes with cp.async.bulk.tensor (one bulk group per
//     chunk) and, before a slot is written again, waits until the bulk group
//     that read it is done reading.
// No load here uses cluster multicast.
#pragma once

#include "tc_gemm.cuh"

namespace dwa {
namespace tc {

__device__ __forceinline__ void tma_load_2d_cta(void* dst, const CUtensorMap* tm, uint64_t* bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* tm, const void* src, int c0, int c1, int c2) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(tm)),
                 "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

constexpr int kWStages = 3;
struct WSmem {
    static constexpr int EW = kPersEpiWarps;
    static constexpr uint32_t A_STAGE = BM * BK * 2;
    static constexpr uint32_t B_STAGE = 256 * BK * 2;
    static constexpr uint32_t RING = kWStages * (A_STAGE + B_STAGE);
    static constexpr uint32_t F32_SLOT = 32 * 32 * 4;                 // 4 KB, 1024-byte aligned
    static constexpr uint32_t BF16_SLOT = 32 * 32 * 2;                // 2 KB
    static constexpr uint32_t WARP_BYTES = 2 * F32_SLOT + BF16_SLOT;  // 10 KB
    static constexpr uint32_t EPI_OFF = RING;
    static constexpr uint32_t BAR_OFF = EPI_OFF + EW * WARP_BYTES;
    static constexpr uint32_t NBAR = 2 * kWStages + 5 + 2 * EW;      // ring, acc_full/empty, drain, W_base slots
    static constexpr uint32_t BYTES = 1024 + BAR_OFF + NBAR * 8 + 16;
    static_assert(BYTES <= 227 * 1024, "W GEMM shared memory above the per-CTA limit");
    static_assert(RING % 1024 == 0 && WARP_BYTES % 1024 == 0, "swizzled slots need 1024-byte alignment");
};

// A = Ug [batch][M = d_B][K] (K-major), B = Vs [batch][K][N = d_A] (MN-major).
__global__ void __launch_bounds__(gemm_threads<kPersEpiWarps>(), 1)
    gemm_w_tma(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmWb, const __grid_constant__ CUtensorMap tmWo,
               const __grid_constant__ CUtensorMap tmWa, int M, int N, int K, int batch, uint32_t* status) {
    constexpr int BN = 256, STAGES = kWStages, EW = kPersEpiWarps;
    using L = WSmem;
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
    uint64_t* wb_bar = drain_bar + 1;                // [EW][2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(wb_bar + 2 * EW);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles_n = (N + BN - 1) / BN, tiles_m = (M + BM - 1) / BM;
    const int tiles = tiles_n * tiles_m * batch;
    const int nkb = (K + BK - 1) / BK;

    if (threadIdx.x == 0) {
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
        prefetch_tmap(&tmWb);
        prefetch_tmap(&tmWo);
        prefetch_tmap(&tmWa);
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], EW);
        }
        mbar_init(drain_bar, 1);
        for (int i = 0; i < 2 * EW; ++i) mbar_init(&wb_bar[i], 1);
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
    pdl_enter();   // operands and W_base come from earlier kernels

    if (warp == 0) {
        if (lane == 0) {
            int it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
                const int n0 = (t % tiles_n) * BN, m0 = ((t / tiles_n) % tiles_m) * BM;
                const int bz = t / (tiles_n * tiles_m);
                for (int kb = 0; kb < nkb; ++kb, ++it) {
                    const int s = it % STAGES;
                    if (it >= STAGES && !mbar_wait_bounded(&empty_bar[s], ((it / STAGES) - 1) & 1)) {
                        raise_status(status, DWA_STATUS_WAIT_TIMEOUT);
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full_bar[s], L::A_STAGE + L::B_STAGE);
                    const int k0 = kb * BK;
                    tma_load_3d(sA + s * L::A_STAGE, &tmA, &full_bar[s], k0, m0, bz);
                    uint8_t* b = sB + s * L::B_STAGE;
#pragma unroll
                    for (int h = 0; h < BN / 64; ++h) tma_load_3d(b + h * 8192, &tmB, &full_bar[s], n0 + 64 * h, k0, bz);
                }
            }
            for (int i = (it > STAGES ? it - STAGES : 0); i < it; ++i)
                if (!mbar_wait_bounded(&full_bar[i % STAGES], (i / STAGES) & 1)) {
                    raise_status(status, DWA_STATUS_WAIT_TIMEOUT);
                    break;
                }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = instr_desc_bf16<BN, false, true>();
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
                        mma_bf16_ss(d_tmem, operand_desc<false>(a_base, kk), operand_desc<true>(b_base, kk), idesc,
                                    (kb | kk) != 0 ? 1u : 0u);
                    mma_commit(&empty_bar[s]);
                }
                if (ok) mma_commit(&acc_full[buf]);
            }
            mma_commit(drain_bar);
            if (!mbar_wait_bounded(drain_bar, 0)) raise_status(status, DWA_STATUS_WAIT_TIMEOUT);
        }
        __syncwarp();
    } else {
        const int q = warp & 3;        // TMEM lane quarter this warp may read
        const int e = warp - 2;        // epilogue warp 0..EW-1
        const int grp = e >> 2;        // column group 0..EW/4-1
        constexpr int CPW = BN / 32 / (EW / 4);     // chunks per warp and tile
        uint8_t* wbase = smem + L::EPI_OFF + e * L::WARP_BYTES;
        auto f32s = [&](int slot) { return wbase + slot * L::F32_SLOT; };
        uint8_t* b16s = wbase + 2 * L::F32_SLOT;
        uint64_t* bars = wb_bar + 2 * e;
        // chunk g of this warp: tile blockIdx.x + (g / CPW) * gridDim.x, column chunk g % CPW
        int issued = 0;                // chunks whose W_base load lane 0 has issued
        auto issue_wbase = [&](int g) {
            const int t = blockIdx.x + (g / CPW) * gridDim.x;
            if (t >= tiles) return;
            const int n0 = (t % tiles_n) * BN, m0 = ((t / tiles_n) % tiles_m) * BM;
            const int c = grp + (g % CPW) * (EW / 4);
            mbar_arrive_expect_tx(&bars[g & 1], L::F32_SLOT);
            tma_load_2d_cta(f32s(g & 1), &tmWb, &bars[g & 1], n0 + c * 32, m0 + q * 32);
            issued = g + 1;
        };
        if (lane == 0) issue_wbase(0);
        __syncwarp();
        int li = 0, g = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++li) {
            const int n0 = (t % tiles_n) * BN, m0 = ((t / tiles_n) % tiles_m) * BM;
            const int bz = t / (tiles_n * tiles_m);
            const int buf = li & 1;
            if (!__all_sync(0xffffffffu, mbar_wait_bounded(&acc_full[buf], (li >> 1) & 1))) {
                if (lane == 0) raise_status(status, DWA_STATUS_WAIT_TIMEOUT);
                ok = false;
                break;
            }
            tc_fence_after();
#pragma unroll 1
            for (int ci = 0; ci < CPW; ++ci, ++g) {
                const int c = grp + ci * (EW / 4);
                // both slots and the bf16 slot are free once the earlier chunks'
                // stores have read them; then the next chunk's W_base goes out
                if (lane == 0) {
                    bulk_wait_read_all();
                    issue_wbase(g + 1);
                }
                __syncwarp();
                float v[32];
                tmem_ld32(tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(buf * BN + c * 32), v);
                if (ci == CPW - 1) {           // this warp's part of the accumulator read out
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&acc_empty[buf]);
                }
                if (!mbar_wait_bounded(&bars[g & 1], (g >> 1) & 1)) {
                    if (lane == 0) raise_status(status, DWA_STATUS_WAIT_TIMEOUT);
                    ok = false;
                }
                if (!__all_sync(0xffffffffu, ok)) break;
                uint8_t* fr = f32s(g & 1) + lane * 128;
                uint8_t* br = b16s + lane * 64;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float4* pa = reinterpret_cast<float4*>(fr + (((2 * j) ^ (lane & 7)) << 4));
                    float4* pb = reinterpret_cast<float4*>(fr + (((2 * j + 1) ^ (lane & 7)) << 4));
                    float4 a = *pa, b = *pb;
                    a.x += v[8 * j + 0]; a.y += v[8 * j + 1]; a.z += v[8 * j + 2]; a.w += v[8 * j + 3];
                    b.x += v[8 * j + 4]; b.y += v[8 * j + 5]; b.z += v[8 * j + 6]; b.w += v[8 * j + 7];
                    *pa = a;
                    *pb = b;
                    uint4 h;
                    __nv_bfloat162 t0 = __floats2bfloat162_rn(a.x, a.y), t1 = __floats2bfloat162_rn(a.z, a.w);
                    __nv_bfloat162 t2 = __floats2bfloat162_rn(b.x, b.y), t3 = __floats2bfloat162_rn(b.z, b.w);
                    h.x = *reinterpret_cast<uint32_t*>(&t0);
                    h.y = *reinterpret_cast<uint32_t*>(&t1);
                    h.z = *reinterpret_cast<uint32_t*>(&t2);
                    h.w = *reinterpret_cast<uint32_t*>(&t3);
                    *reinterpret_cast<uint4*>(br + ((j ^ ((lane >> 1) & 3)) << 4)) = h;
                }
                fence_proxy_async_smem();      // this lane's writes, visible to the bulk copies
                __syncwarp();
                if (lane == 0) {
                    tma_store_3d(&tmWo, f32s(g & 1), n0 + c * 32, m0 + q * 32, bz);
                    tma_store_3d(&tmWa, b16s, n0 + c * 32, m0 + q * 32, bz);
                    bulk_commit();
                }
                __syncwarp();
            }
        }
        if (lane == 0) {
            bulk_wait_all();
            // W_base loads issued but not consumed (only on an error path) land
            // before the CTA exits
            for (int h = g; h < issued; ++h)
                if (!mbar_wait_bounded(&bars[h & 1], (h >> 1) & 1)) {
                    raise_status(status, DWA_STATUS_WAIT_TIMEOUT);
                    break;
                }
        }
        __syncwarp();
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

// Tensor maps of the epilogue: W_base [d_B, d_A] fp32, W [B, d_B, d_A] fp32,
// W_act [B, d_B, d_A] bf16, all with 32 x 32 boxes.
bool make_w_epilogue_maps(CUtensorMap* wb, CUtensorMap* wo, CUtensorMap* wa, const float* W_base, float* W_out,
                          void* W_act, int d_B, int d_A, int batch, std::string* why);

inline int launch_gemm_w_tma(const Operand& A, const Operand& B, int M, int N, int K, int batch, const float* W_base,
                             float* W_out, void* W_act, uint32_t* status, cudaStream_t stream) {
    CUtensorMap ta, tb, twb, two, twa;
    std::string why;
    if (!make_operand_map(&ta, A, M, K, batch, BM, &why) || !make_operand_map(&tb, B, N, K, batch, 256, &why) ||
        !make_w_epilogue_maps(&twb, &two, &twa, W_base, W_out, W_act, M, N, batch, &why))
        return fail(DWA_ERR_INVALID_ARG, "tensor map: " + why);
    static bool attr_set[64] = {};
    int dev = 0;
    DWA_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        DWA_CUDA_TRY(cudaFuncSetAttribute(gemm_w_tma, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(WSmem::BYTES)));
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    const int64_t tiles = static_cast<int64_t>((N + 255) / 256) * ((M + BM - 1) / BM) * batch;
    const int grid = static_cast<int>(std::min<int64_t>(tiles, sm_count()));
    launch_pdl(gemm_w_tma, dim3(grid), gemm_threads<kPersEpiWarps>(), WSmem::BYTES, stream, ta, tb, twb, two, twa,
               M, N, K, batch, status);
    DWA_LAUNCH_CHECK("gemm_w_tma");
    return DWA_OK;
}

}  // namespace tc
}  // namespace dwa
