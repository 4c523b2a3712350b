// Work split shared by the key-cache scoring kernels (CUDA-core and tensor-core
// scans): which key rows a persistent CTA scores, in which order.
//
// Full pass: the pool's rows are cut into BOX-row blocks and CTA c takes the
// contiguous blocks [nblk*c/grid, nblk*(c+1)/grid), walked as ROWS-row tiles
// (the last one partial), so every CTA streams the same number of bytes.
// Fine pass: tile g covers rows [tt*ROWS, (tt+1)*ROWS) of probed list j of
// query b (g = (b*m + j)*tiles_per_list + tt); CTA c takes g = c, c+grid, ...
// Tiles past the end of a list are invalid and skipped by every role alike.
#pragma once

#include "tc_gemm.cuh"

namespace dwa {
namespace kt {

struct Args {
    int64_t N;
    int S, B;
    float invT;              // 1 / T
    int mode;                // 0: full pass over [0, N); 1: fine pass over the probed lists
    int stages;              // TMA ring slots
    int64_t nblk;            // full: ceil(N / BOX)
    int ntiles;              // fine: B * m * tiles_per_list
    int tiles_per_list;      // fine
    int m;                   // fine: lists per query
    const int64_t* probe_lo;   // fine [B, m+1]: first key row of each probed list
    const int64_t* cand_base;  // fine [B, m+1]: output offset of each probed list
    int64_t K_cap;             // fine: row stride of out
    const float* qw;           // [B, S, 64]
    float* out;                // full: s_full [B, N]; fine: scores [B, K_cap]
    float* partial;            // full: [B, gridDim, 2] (max, sum exp) of s/T
    uint32_t* status;
};

struct Tile {
    bool valid;
    int b;          // fine: the query
    int64_t row0;   // first key row
    int rows;       // rows of the tile that belong to it (<= ROWS)
    int64_t obase;  // fine: output offset of the tile's first row
};

// Number of tile slots CTA `blk` walks (valid or not) and, for the full pass,
// its row range.
template <int ROWS, int BOX>
__device__ __forceinline__ int tile_count(const Args& a, int blk, int grid, int64_t& row_lo,
                                          int64_t& row_hi) {
    if (a.mode == 0) {
        row_lo = (a.nblk * blk / grid) * BOX;
        row_hi = (a.nblk * (blk + 1) / grid) * BOX;
        if (row_hi > a.N) row_hi = a.N;
        return row_hi > row_lo ? static_cast<int>((row_hi - row_lo + ROWS - 1) / ROWS) : 0;
    }
    row_lo = row_hi = 0;
    return blk < a.ntiles ? (a.ntiles - 1 - blk) / grid + 1 : 0;
}

template <int ROWS>
__device__ __forceinline__ Tile tile_at(const Args& a, int i, int blk, int grid, int64_t row_lo,
                                        int64_t row_hi) {
    Tile t{};
    if (a.mode == 0) {
        t.valid = true;
        t.b = 0;
        t.row0 = row_lo + static_cast<int64_t>(i) * ROWS;
        t.rows = static_cast<int>(row_hi - t.row0 < ROWS ? row_hi - t.row0 : ROWS);
        t.obase = 0;
    } else {
        const int g = blk + i * grid;
        const int per_b = a.m * a.tiles_per_list;
        t.b = g / per_b;
        const int j = (g / a.tiles_per_list) % a.m, tt = g % a.tiles_per_list;
        const int64_t* cb = a.cand_base + static_cast<int64_t>(t.b) * (a.m + 1);
        const int64_t size = cb[j + 1] - cb[j];
        const int64_t off = static_cast<int64_t>(tt) * ROWS;
        t.valid = off < size;
        t.row0 = a.probe_lo[static_cast<int64_t>(t.b) * (a.m + 1) + j] + off;
        t.rows = static_cast<int>(size - off < ROWS ? size - off : ROWS);
        t.obase = cb[j] + off;
    }
    return t;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* tm, uint64_t* bar, int c0,
                                            int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(tc::smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(tc::smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc::smem_u32(bar)) : "memory");
}

}  // namespace kt
}  // namespace dwa
