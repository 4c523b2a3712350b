// libdwa host plumbing: version, status strings, per-thread last error,
// device status readback, launch counters and TMA tensor-map encoding.
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "dwa_common.cuh"
#include "tc_gemm.cuh"

namespace dwa {

std::atomic<uint64_t> g_launches_total{0}, g_launches_tc{0}, g_launches_simt{0};

// Serialised launches (dwa_profile_serialize): no programmatic dependent
// launch and no concurrent lanes, so that an event pair around one kernel
// measures that kernel alone and per-kernel times add up to the step.
static std::atomic<int> g_serialize{0};

bool serialized() { return g_serialize.load(std::memory_order_relaxed) != 0; }

bool pdl_enabled() {
    static const bool on = [] {
        const char* v = std::getenv("DWA_PDL");
        return !(v && std::strcmp(v, "0") == 0);
    }();
    return on && !serialized();
}

static thread_local std::string t_last_error;

void set_last_error(const std::string& msg) { t_last_error = msg; }

int fail(int code, const std::string& msg) {
    set_last_error(msg);
    return code;
}

struct ProfEntry {
    char name[32];
    cudaEvent_t start, stop;
};
static std::mutex g_prof_mu;
static ProfEntry g_prof[64];
static int g_prof_n = 0;
static std::atomic<int> g_prof_active{0};

static ProfEntry* prof_find(const char* name) {
    for (int i = 0; i < g_prof_n; ++i)
        if (std::strncmp(g_prof[i].name, name, sizeof(g_prof[i].name)) == 0) return &g_prof[i];
    return nullptr;
}

// Inside a stream capture the record becomes an external event node of the
// graph, so every replay records the event again.
static void prof_record(cudaEvent_t ev, cudaStream_t st) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(st, &cs) == cudaSuccess && cs == cudaStreamCaptureStatusActive)
        cudaEventRecordWithFlags(ev, st, cudaEventRecordExternal);
    else
        cudaEventRecord(ev, st);
}

void prof_begin(const char* name, cudaStream_t st) {
    if (!g_prof_active.load(std::memory_order_relaxed)) return;
    std::lock_guard<std::mutex> lk(g_prof_mu);
    if (ProfEntry* e = prof_find(name)) prof_record(e->start, st);
}

void prof_end(const char* name, cudaStream_t st) {
    if (!g_prof_active.load(std::memory_order_relaxed)) return;
    std::lock_guard<std::mutex> lk(g_prof_mu);
    if (ProfEntry* e = prof_find(name)) prof_record(e->stop, st);
}

struct LaneState {
    std::mutex mu;
    bool ready = false;
    cudaStream_t aux[2];
    cudaEvent_t ev[8];
};
static LaneState g_lanes[64];

Lanes::Lanes(cudaStream_t st) : main(st) {
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        rc = fail(DWA_ERR_CUDA, "Lanes: no current device");
        dev = -1;
        return;
    }
    LaneState& L = g_lanes[dev];
    L.mu.lock();
    if (!L.ready) {
        bool ok = true;
        for (auto& a : L.aux) ok = ok && cudaStreamCreateWithFlags(&a, cudaStreamNonBlocking) == cudaSuccess;
        for (auto& e : L.ev) ok = ok && cudaEventCreateWithFlags(&e, cudaEventDisableTiming) == cudaSuccess;
        if (!ok) {
            rc = fail(DWA_ERR_CUDA, "Lanes: stream/event creation failed");
            return;
        }
        L.ready = true;
    }
    for (int i = 0; i < 8; ++i) ev[i] = L.ev[i];
    if (serialized()) {   // every lane is the main stream: kernels run one after another
        aux[0] = aux[1] = main;
        return;
    }
    aux[0] = L.aux[0];
    aux[1] = L.aux[1];
    if ((rc = depend(aux[0], main, 0))) return;
    rc = depend(aux[1], main, 0);
}

Lanes::~Lanes() {
    if (dev >= 0) g_lanes[dev].mu.unlock();
}

int Lanes::depend(cudaStream_t to, cudaStream_t from, int slot) {
    if (to == from) return DWA_OK;
    if (cudaEventRecord(ev[slot], from) != cudaSuccess || cudaStreamWaitEvent(to, ev[slot], 0) != cudaSuccess)
        return fail(DWA_ERR_CUDA, "Lanes: event record/wait failed");
    return DWA_OK;
}

int Lanes::join() {
    int r = depend(main, aux[0], 6);
    return r ? r : depend(main, aux[1], 7);
}

namespace tc {

// Streaming multiprocessors of the current device (cached per device).
int sm_count() {
    static int cache[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (!cache[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

// DWA_GEMM=classic or DWA_GEMM=single keeps GEMMs off the CTA-pair kernel.
bool pair_gemm() {
    static const bool on = [] {
        const char* v = std::getenv("DWA_GEMM");
        return !(v && (std::strcmp(v, "classic") == 0 || std::strcmp(v, "single") == 0));
    }();
    return on;
}

// DWA_GEMM=classic selects the one-tile-per-CTA GEMM instead of the persistent one.
bool persistent_gemm() {
    static const bool on = [] {
        const char* v = std::getenv("DWA_GEMM");
        return !(v && std::strcmp(v, "classic") == 0);
    }();
    return on;
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// W_base [d_B, d_A] fp32, W [batch, d_B, d_A] fp32 (128-byte swizzle) and
// W_act [batch, d_B, d_A] bf16 (64-byte swizzle), 32 x 32 boxes: the TMA maps
// of the W GEMM's epilogue.
bool make_w_epilogue_maps(CUtensorMap* wb, CUtensorMap* wo, CUtensorMap* wa, const float* W_base, float* W_out,
                          void* W_act, int d_B, int d_A, int batch, std::string* why) {
    auto enc = tensor_map_encoder();
    if (!enc) {
        *why = "cuTensorMapEncodeTiled unavailable";
        return false;
    }
    const cuuint64_t A = static_cast<cuuint64_t>(d_A), Bd = static_cast<cuuint64_t>(d_B);
    const cuuint32_t box[3] = {32, 32, 1}, es[3] = {1, 1, 1};
    const cuuint64_t dims2[2] = {A, Bd}, str2[1] = {A * 4};
    const cuuint64_t dims3[3] = {A, Bd, static_cast<cuuint64_t>(batch)};
    const cuuint64_t strf[2] = {A * 4, A * Bd * 4}, strh[2] = {A * 2, A * Bd * 2};
    CUresult r = enc(wb, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(W_base), dims2, str2, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r == CUDA_SUCCESS)
        r = enc(wo, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, W_out, dims3, strf, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r == CUDA_SUCCESS)
        r = enc(wa, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, W_act, dims3, strh, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        *why = "cuTensorMapEncodeTiled error " + std::to_string(static_cast<int>(r)) + " (W epilogue maps)";
        return false;
    }
    return true;
}

bool tc_operand_ok(const Operand& op, int64_t mn_extent, int64_t k_extent, int box_mn) {
    const int64_t es = 2;
    if (reinterpret_cast<uintptr_t>(op.ptr) % 16 != 0) return false;
    if ((op.ld * es) % 16 != 0 || (op.bstride * es) % 16 != 0) return false;
    if (k_extent < BK) return false;
    if (op.mn_major) {
        if (mn_extent < 64 || op.ld < mn_extent) return false;
    } else {
        if (mn_extent < box_mn || op.ld < k_extent) return false;
    }
    return mn_extent < (int64_t(1) << 31) && k_extent < (int64_t(1) << 31);
}

bool make_operand_map(CUtensorMap* tm, const Operand& op, int64_t mn_extent, int64_t k_extent,
                      int batch, int box_mn, std::string* why) {
    auto enc = tensor_map_encoder();
    if (!enc) {
        *why = "cuTensorMapEncodeTiled unavailable";
        return false;
    }
    const int64_t inner = op.mn_major ? mn_extent : k_extent;
    const int64_t outer = op.mn_major ? k_extent : mn_extent;
    const bool batched = op.bstride != 0;
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer),
                          static_cast<cuuint64_t>(batched ? batch : 1)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(op.ld * 2),
                             static_cast<cuuint64_t>(batched ? op.bstride * 2 : op.ld * 2 * outer)};
    cuuint32_t box[3] = {64, static_cast<cuuint32_t>(op.mn_major ? 64 : box_mn), 1};
    cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(op.ptr), dims,
                           strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        char buf[160];
        std::snprintf(buf, sizeof(buf), "cuTensorMapEncodeTiled error %d (inner %lld outer %lld ld %lld)",
                      static_cast<int>(r), static_cast<long long>(inner),
                      static_cast<long long>(outer), static_cast<long long>(op.ld));
        *why = buf;
        return false;
    }
    return true;
}

}  // namespace tc
}  // namespace dwa

extern "C" const char* dwa_version(void) { return "dwa-b200 0.1 (sm_100a)"; }

extern "C" int dwa_abi_version(void) { return DWA_ABI_VERSION; }

extern "C" const char* dwa_status_string(int status) {
    switch (status) {
        case DWA_OK: return "ok";
        case DWA_ERR_INVALID_ARG: return "invalid argument";
        case DWA_ERR_UNSUPPORTED: return "unsupported";
        case DWA_ERR_CUDA: return "CUDA error";
        case DWA_ERR_WORKSPACE: return "workspace error";
        case DWA_ERR_DEVICE: return "device status error";
        default: return "unknown status";
    }
}

extern "C" int dwa_last_error(char* buf, size_t buf_bytes) {
    const std::string& e = dwa::t_last_error;
    if (buf && buf_bytes) {
        const size_t n = e.size() < buf_bytes - 1 ? e.size() : buf_bytes - 1;
        std::memcpy(buf, e.data(), n);
        buf[n] = '\0';
    }
    return static_cast<int>(e.size());
}

extern "C" int dwa_workspace_status(void* stream, void* workspace, uint32_t* status, int clear) {
    if (!workspace || !status) return dwa::fail(DWA_ERR_INVALID_ARG, "NULL workspace or status");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    DWA_CUDA_TRY(cudaMemcpyAsync(status, workspace, sizeof(uint32_t), cudaMemcpyDeviceToHost, st));
    DWA_CUDA_TRY(cudaStreamSynchronize(st));
    if (clear) {
        DWA_CUDA_TRY(cudaMemsetAsync(workspace, 0, sizeof(uint32_t), st));
        DWA_CUDA_TRY(cudaStreamSynchronize(st));
    }
    return *status ? DWA_ERR_DEVICE : DWA_OK;
}

extern "C" void dwa_launch_counters(uint64_t* total, uint64_t* tensor_core_gemms,
                                    uint64_t* simt_gemms) {
    if (total) *total = dwa::g_launches_total.load();
    if (tensor_core_gemms) *tensor_core_gemms = dwa::g_launches_tc.load();
    if (simt_gemms) *simt_gemms = dwa::g_launches_simt.load();
}

extern "C" void dwa_profile_serialize(int on) { dwa::g_serialize.store(on ? 1 : 0); }

extern "C" int dwa_profile_kernel(const char* kernel, void* start_event, void* stop_event) {
    if (!kernel || std::strlen(kernel) >= sizeof(dwa::ProfEntry::name))
        return dwa::fail(DWA_ERR_INVALID_ARG, "kernel name missing or too long");
    std::lock_guard<std::mutex> lk(dwa::g_prof_mu);
    dwa::ProfEntry* e = dwa::prof_find(kernel);
    if (!start_event || !stop_event) {
        if (e) {
            *e = dwa::g_prof[dwa::g_prof_n - 1];
            --dwa::g_prof_n;
        }
    } else {
        if (!e) {
            if (dwa::g_prof_n >= 64) return dwa::fail(DWA_ERR_UNSUPPORTED, "too many timed kernels");
            e = &dwa::g_prof[dwa::g_prof_n++];
            std::snprintf(e->name, sizeof(e->name), "%s", kernel);
        }
        e->start = static_cast<cudaEvent_t>(start_event);
        e->stop = static_cast<cudaEvent_t>(stop_event);
    }
    dwa::g_prof_active.store(dwa::g_prof_n > 0);
    return DWA_OK;
}

extern "C" void dwa_profile_clear(void) {
    std::lock_guard<std::mutex> lk(dwa::g_prof_mu);
    dwa::g_prof_n = 0;
    dwa::g_prof_active.store(0);
}
