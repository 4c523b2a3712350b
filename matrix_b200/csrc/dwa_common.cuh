// Shared device/host helpers for libdwa: element access, status word, bounded
// waits, last-error plumbing.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <string>

#include "../../include/dwa.h"

namespace dwa {

// ---------------------------------------------------------------------------
// host-side error reporting
// ---------------------------------------------------------------------------
void set_last_error(const std::string& msg);
int fail(int code, const std::string& msg);

#define DWA_CUDA_TRY(expr)                                                        \
    do {                                                                          \
        cudaError_t _e = (expr);                                                  \
        if (_e != cudaSuccess)                                                    \
            return ::dwa::fail(DWA_ERR_CUDA, std::string(#expr " failed: ") +     \
                                                 cudaGetErrorString(_e));         \
    } while (0)

#define DWA_LAUNCH_CHECK(what)                                                    \
    do {                                                                          \
        cudaError_t _e = cudaGetLastError();                                      \
        if (_e != cudaSuccess)                                                    \
            return ::dwa::fail(DWA_ERR_CUDA, std::string("launch of " what        \
                                                 " failed: ") + cudaGetErrorString(_e)); \
    } while (0)

// Kernel timing hook (dwa_profile_kernel): event pair recorded around the
// launches of one named kernel.
void prof_begin(const char* name, cudaStream_t st);
void prof_end(const char* name, cudaStream_t st);
#define DWA_TIMED(name, st, ...)      \
    do {                              \
        ::dwa::prof_begin(name, st);  \
        __VA_ARGS__;                  \
        ::dwa::prof_end(name, st);    \
    } while (0)

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }
inline size_t dtype_bytes(int dt) { return dt == DWA_BF16 ? 2 : 4; }

// Carves aligned sub-buffers out of a caller workspace.  The first 256 bytes
// hold the device status word.
struct Carver {
    char* base;
    size_t off = 256;
    explicit Carver(void* p) : base(static_cast<char*>(p)) {}
    template <class T>
    T* take(size_t count) {
        off = align_up(off, 256);
        T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
        off += count * sizeof(T);
        return p;
    }
    size_t bytes() const { return align_up(off, 256); }
};

// ---------------------------------------------------------------------------
// device helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float load_elem(const void* p, int64_t i, int dt) {
    return dt == DWA_BF16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i])
                          : static_cast<const float*>(p)[i];
}

__device__ __forceinline__ void store_elem(void* p, int64_t i, int dt, float v) {
    if (dt == DWA_BF16)
        static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
    else
        static_cast<float*>(p)[i] = v;
}

template <class T> struct Elem;
template <> struct Elem<float> {
    static __device__ __forceinline__ float to_f(float v) { return v; }
    static __device__ __forceinline__ float from_f(float v) { return v; }
    static constexpr int dtype = DWA_F32;
};
template <> struct Elem<__nv_bfloat16> {
    static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
    static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
    static constexpr int dtype = DWA_BF16;
};

__device__ __forceinline__ void raise_status(uint32_t* status, uint32_t bits) {
    if (status) atomicOr(status, bits);
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Upper bound of any device-side wait.  A healthy wait ends in microseconds.
constexpr uint64_t kWaitLimitNs = 1000ull * 1000ull * 1000ull;  // 1 s

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

}  // namespace dwa
