// Shared device/host helpers for libdwa: element access, status word, bounded
// waits, last-error plumbing.
#pragma once

#include <cooperative_groups.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <string>
#include <utility>

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

// Programmatic dependent launch.  Every kernel of the library is launched with
// launch_pdl, which lets the next kernel of the same stream (or CUDA graph) be
// scheduled while this one drains, and every kernel calls pdl_enter() before it
// touches global memory that an earlier kernel wrote: griddepcontrol.wait returns
// once the preceding kernel has completed and its writes are visible; then
// launch_dependents allows the following kernel to start its prologue.  Both are
// no-ops for a kernel launched without the attribute.  DWA_PDL=0 disables it.
__device__ __forceinline__ void pdl_enter() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

bool pdl_enabled();
bool serialized();   // dwa_profile_serialize is on

// Split cluster barrier: arrive early, wait just before the first access to
// another CTA's shared memory (every CTA of the cluster has then started).
__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }

template <class... KArgs, class... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// launch_pdl for a kernel run as thread-block clusters of `cluster` CTAs
// (each grid dimension a multiple of the cluster's).
template <class... KArgs, class... Args>
inline cudaError_t launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                      cudaStream_t st, dim3 cluster, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = cluster.x;
    attr[1].val.clusterDim.y = cluster.y;
    attr[1].val.clusterDim.z = cluster.z;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

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

// Intra-call concurrency: per-device auxiliary streams and events, created on
// first use.  A Lanes object holds the device's lock from construction to
// destruction, so the record/wait pairs of one call are not interleaved with
// another host thread's.  Everything is stream-ordered (capturable in a graph).
struct Lanes {
    cudaStream_t main = nullptr;
    cudaStream_t aux[2] = {nullptr, nullptr};
    cudaEvent_t ev[8] = {};
    int dev = -1;
    int rc = 0;
    explicit Lanes(cudaStream_t st);   // forks aux[0], aux[1] off `main`
    ~Lanes();
    // `to` waits for everything enqueued so far on `from` (event slot `slot`)
    int depend(cudaStream_t to, cudaStream_t from, int slot);
    int join();                         // main waits for both aux streams
};

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

// out[b][j] = sum_t x[b][t][j]   (divided by T when `mean`), x [B, T, d].
// Grid (ceil(d/64), B), 1024 threads: lane l of warp w sums columns c0+2l,
// c0+2l+1 over rows t = w, w+32, ... (16 loads in flight per thread); the 32
// warp partials are then added in a fixed order, so the result is
// deterministic.
template <class T>
__global__ void __launch_bounds__(1024) column_sum_kernel(const T* __restrict__ x, int T_, int d,
                                                          int mean, float* __restrict__ out) {
    pdl_enter();
    __shared__ float part[32][65];
    const int b = blockIdx.y, lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int c = blockIdx.x * 64 + 2 * lane;
    const T* p = x + static_cast<int64_t>(b) * T_ * d;
    float a0 = 0.f, a1 = 0.f;
    for (int t0 = w; t0 < T_; t0 += 32 * 16) {
        float v0[16], v1[16];
#pragma unroll
        for (int u = 0; u < 16; ++u) {
            const int t = t0 + 32 * u;
            const T* q = p + static_cast<int64_t>(t) * d;
            v0[u] = (t < T_ && c < d) ? Elem<T>::to_f(q[c]) : 0.f;
            v1[u] = (t < T_ && c + 1 < d) ? Elem<T>::to_f(q[c + 1]) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < 16; ++u) { a0 += v0[u]; a1 += v1[u]; }
    }
    part[w][2 * lane] = a0;
    part[w][2 * lane + 1] = a1;
    __syncthreads();
    if (threadIdx.x < 64) {
        const int j = blockIdx.x * 64 + threadIdx.x;
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i) s += part[i][threadIdx.x];
        if (j < d) out[static_cast<int64_t>(b) * d + j] = mean ? s / static_cast<float>(T_) : s;
    }
}

// Same sums with 8 consecutive columns per lane (16-byte loads for bf16, two
// for fp32): grid (ceil(d/256), B, split) launched as clusters of (1, 1, split)
// CTAs, 512 threads.  CTA z of a cluster sums the rows
// [T*z/split, T*(z+1)/split) (warp w takes rows w, w+16, ...; U = 8 rows in
// flight per lane for bf16, held as raw 16-byte words until they land, 4 for
// fp32), adds its 16 warp partials in warp order, and cluster rank 0 adds
// the split CTAs' sums in rank order out of their shared memory: deterministic
// for a given split.  d % 8 == 0 and a 16-byte aligned x required.
namespace tc {
int sm_count();   // streaming multiprocessors of the current device (abi.cu)
}

template <class T> constexpr int column_sum8_rows() { return sizeof(T) == 2 ? 8 : 4; }

template <class T>
__global__ void __launch_bounds__(512, 2) column_sum8_kernel(const T* __restrict__ x, int T_, int d,
                                                          int mean, float* __restrict__ out) {
    pdl_enter();
    constexpr int U = column_sum8_rows<T>();
    __shared__ float part[16][257];
    __shared__ float tot[256];
    const int b = blockIdx.y, lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int split = gridDim.z, z = blockIdx.z;
    const int t_lo = static_cast<int>(static_cast<int64_t>(T_) * z / split);
    const int t_hi = static_cast<int>(static_cast<int64_t>(T_) * (z + 1) / split);
    const int c = blockIdx.x * 256 + 8 * lane;
    const T* p = x + static_cast<int64_t>(b) * T_ * d;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (c < d) {
        for (int t0 = t_lo + w; t0 < t_hi; t0 += 16 * U) {
            uint4 r[U], r2[sizeof(T) == 2 ? 1 : U];
            const T* q0 = p + static_cast<int64_t>(t0) * d + c;
            const int64_t step = 16 * static_cast<int64_t>(d);
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const uint4* q = reinterpret_cast<const uint4*>(q0 + u * step);
                const bool in = t0 + 16 * u < t_hi;
                r[u] = in ? q[0] : make_uint4(0u, 0u, 0u, 0u);
                if constexpr (sizeof(T) == 4) r2[u] = in ? q[1] : make_uint4(0u, 0u, 0u, 0u);
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                if constexpr (sizeof(T) == 2) {
                    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&r[u]);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float2 f = __bfloat1622float2(h[j]);
                        acc[2 * j] += f.x;
                        acc[2 * j + 1] += f.y;
                    }
                } else {
                    acc[0] += __uint_as_float(r[u].x); acc[1] += __uint_as_float(r[u].y);
                    acc[2] += __uint_as_float(r[u].z); acc[3] += __uint_as_float(r[u].w);
                    acc[4] += __uint_as_float(r2[u].x); acc[5] += __uint_as_float(r2[u].y);
                    acc[6] += __uint_as_float(r2[u].z); acc[7] += __uint_as_float(r2[u].w);
                }
            }
        }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) part[w][8 * lane + j] = acc[j];
    __syncthreads();
    if (threadIdx.x < 256) {
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) s += part[i][threadIdx.x];
        tot[threadIdx.x] = s;
    }
    if (split > 1) {
        cooperative_groups::cluster_group cl = cooperative_groups::this_cluster();
        cl.sync();
        if (cl.block_rank() == 0 && threadIdx.x < 256) {
            float s = 0.f;
            for (int r = 0; r < split; ++r) s += cl.map_shared_rank(tot, r)[threadIdx.x];
            const int col = blockIdx.x * 256 + threadIdx.x;
            if (col < d) out[static_cast<int64_t>(b) * d + col] = mean ? s / static_cast<float>(T_) : s;
        }
        cl.sync();   // every CTA's sums stay in place until rank 0 has read them
    } else if (threadIdx.x < 256) {
        const int col = blockIdx.x * 256 + threadIdx.x;
        if (col < d) out[static_cast<int64_t>(b) * d + col] = mean ? tot[threadIdx.x] / static_cast<float>(T_) : tot[threadIdx.x];
    }
}

// Launch of column_sum8_kernel over x [B, T, d]: at most 8 CTAs (one cluster)
// per (column block, b), at least one round of loads (16 warps x U rows) each,
// and no more CTAs than one wave at two per SM (measured on B 16 x T 1024 x
// d 2048 bf16: 22 us with two CTAs per column block, 31 us with eight).  At
// two 512-thread CTAs per SM a thread has 64 registers: eight raw bf16 rows
// (32 registers) fit, eight fp32 rows would spill.
template <class T>
inline cudaError_t launch_column_sum8(cudaStream_t st, const T* x, int B, int T_, int d, int mean, float* out) {
    const int rows = 16 * column_sum8_rows<T>();
    int split = (T_ + rows - 1) / rows;
    const int units = B * ((d + 255) / 256);
    const int wave = 2 * tc::sm_count() / (units > 0 ? units : 1);
    if (split > wave) split = wave;
    split = split < 1 ? 1 : split > 8 ? 8 : split;
    return launch_pdl_cluster(column_sum8_kernel<T>, dim3((d + 255) / 256, B, split), dim3(512), 0, st,
                              dim3(1, 1, split), x, T_, d, mean, out);
}

}  // namespace dwa
