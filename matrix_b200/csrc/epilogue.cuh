// Helpers shared by the GEMM epilogue functors (assembly and key cache):
// 8-wide vector loads / stores of f32 and bf16 rows, a vector float reduction,
// the no-reduction base and the operator() the CUDA-core GEMM calls.
#pragma once

#include "dwa_common.cuh"

namespace dwa {

// 8 consecutive elements through 16-byte accesses (the pointer must be 16-byte
// aligned for bf16, 16-byte aligned for fp32 pairs of float4).
__device__ __forceinline__ void load8(const float* p, float* v) {
    const float4 a = reinterpret_cast<const float4*>(p)[0];
    const float4 b = reinterpret_cast<const float4*>(p)[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void load8(const __nv_bfloat16* p, float* v) {
    const uint4 t = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&t);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(h[j]);
        v[2 * j] = f.x;
        v[2 * j + 1] = f.y;
    }
}
__device__ __forceinline__ void store8(float* p, const float* v) {
    reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}
// Streaming store (st.global.cs): for outputs no kernel of the same call reads
// again, so they do not evict operands that are still being re-read from L2.
__device__ __forceinline__ void store8_stream(float* p, const float* v) {
    __stcs(reinterpret_cast<float4*>(p), make_float4(v[0], v[1], v[2], v[3]));
    __stcs(reinterpret_cast<float4*>(p) + 1, make_float4(v[4], v[5], v[6], v[7]));
}
__device__ __forceinline__ void store8(__nv_bfloat16* p, const float* v) {
    uint4 t;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&t);
#pragma unroll
    for (int j = 0; j < 4; ++j) h[j] = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
    *reinterpret_cast<uint4*>(p) = t;
}
__device__ __forceinline__ void red_add4(float* p, float a, float b, float c, float d) {
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c),
                 "f"(d)
                 : "memory");
}

// ------------------------------------------------------------ epilogues ----
// Epilogue functors.  The tensor-core GEMM calls load() for several rows first
// (global operands into a register fragment) and finish() afterwards, so the
// loads of those rows are in flight together; the CUDA-core GEMM calls
// operator(), i.e. both back to back.  The vector path covers 8 columns
// starting at a multiple of 8; other segments take the scalar path in finish().
struct NoReduce {
    static constexpr int kReduce = 0;
    __device__ void row_done(int, int, float) const {}
    __device__ void cta_done(int, float) const {}
};

#define DWA_EPI_CALL                                                                    \
    __device__ float operator()(int b, int row, int col0, const float* v, int cnt) const { \
        Frag f;                                                                           \
        load(b, row, col0, cnt, f);                                                       \
        return finish(b, row, col0, v, cnt, f);                                           \
    }

}  // namespace dwa
