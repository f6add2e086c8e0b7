// Library-wide state of libpolykern: thread-local last error, the device status
// word, the cached SM count and the runtime-resolved TMA descriptor encoder.
#include <cudaTypedefs.h>

#include <atomic>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "pk_common.cuh"

__device__ int pk_device_status_word = 0;

namespace pk {

// Device address of the status word on the current device, looked up once per device.
// The lookup is serialised: two host threads making their first call on one device would
// otherwise both write the cache slot.  (A cudaDeviceReset invalidates the address; the
// library is not meant to outlive a reset of its context.)
static std::mutex g_status_mutex;

int* device_status_ptr() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    static int* cache[64] = {nullptr};
    std::lock_guard<std::mutex> lock(g_status_mutex);
    if (!cache[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, pk_device_status_word) == cudaSuccess) cache[dev] = static_cast<int*>(p);
    }
    return cache[dev];
}

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}

int cuda_fail(cudaError_t err, const char* what) {
    g_last_error = std::string(what) + ": " + cudaGetErrorName(err) + " (" + cudaGetErrorString(err) + ")";
    return PK_ERR_CUDA;
}

int num_sms() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    // Racing first calls store the same value; atomics keep that well defined.
    static std::atomic<int> cache[64];
    if (dev < 0 || dev >= 64) return 148;
    int n = cache[dev].load(std::memory_order_relaxed);
    if (n == 0) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cache[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::once_flag g_encode_once;

CUresult encode_tiled(CUtensorMap* map, CUtensorMapDataType dt, cuuint32_t rank, void* base,
                      const cuuint64_t* dims, const cuuint64_t* strides_bytes, const cuuint32_t* box,
                      CUtensorMapSwizzle swizzle) {
    std::call_once(g_encode_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    if (!g_encode) return CUDA_ERROR_NOT_FOUND;
    cuuint32_t elem_strides[5] = {1, 1, 1, 1, 1};
    return g_encode(map, dt, rank, base, dims, strides_bytes, box, elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

// ---------------------------------------------------------------------------------
// Optional launch timing: when enabled, launchers bracket their main kernel with CUDA
// events recorded on the launch stream; pk_profile_query() resolves them.

struct ProfRecord {
    std::vector<std::pair<cudaEvent_t, cudaEvent_t>> pending;
    std::vector<cudaEvent_t> free_events;
};
static std::mutex g_prof_mutex;
static bool g_prof_on = false;
static std::map<std::string, ProfRecord> g_prof;

static cudaEvent_t take_event(ProfRecord& r) {
    if (!r.free_events.empty()) {
        cudaEvent_t e = r.free_events.back();
        r.free_events.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}

bool profiling() { return g_prof_on; }

static std::atomic<int64_t> g_launches{0};

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

void prof_begin(const char* name, cudaStream_t stream, void** token) {
    *token = nullptr;
    if (!g_prof_on) return;
    std::lock_guard<std::mutex> lock(g_prof_mutex);
    ProfRecord& r = g_prof[name];
    cudaEvent_t e = take_event(r);
    cudaEventRecord(e, stream);
    *token = e;
}

void prof_end(const char* name, cudaStream_t stream, void* token) {
    if (!token) return;
    std::lock_guard<std::mutex> lock(g_prof_mutex);
    ProfRecord& r = g_prof[name];
    cudaEvent_t e = take_event(r);
    cudaEventRecord(e, stream);
    r.pending.emplace_back(static_cast<cudaEvent_t>(token), e);
}

}  // namespace pk

extern "C" {

int pk_profile_enable(int on) {
    std::lock_guard<std::mutex> lock(pk::g_prof_mutex);
    pk::g_prof_on = on != 0;
    return 0;
}

int pk_profile_query(const char* name, double* total_ms, int64_t* launches) {
    if (!name || !total_ms || !launches) return pk::fail(PK_ERR_ARG, "pk_profile_query: null argument");
    std::lock_guard<std::mutex> lock(pk::g_prof_mutex);
    *total_ms = 0.0;
    *launches = 0;
    auto it = pk::g_prof.find(name);
    if (it == pk::g_prof.end()) return 0;
    pk::ProfRecord& r = it->second;
    for (auto& pr : r.pending) {
        cudaError_t e = cudaEventSynchronize(pr.second);
        if (e != cudaSuccess) return pk::cuda_fail(e, "pk_profile_query: cudaEventSynchronize");
        float ms = 0.f;
        e = cudaEventElapsedTime(&ms, pr.first, pr.second);
        if (e != cudaSuccess) return pk::cuda_fail(e, "pk_profile_query: cudaEventElapsedTime");
        *total_ms += ms;
        *launches += 1;
        r.free_events.push_back(pr.first);
        r.free_events.push_back(pr.second);
    }
    r.pending.clear();
    return 0;
}

int64_t pk_launch_count(int reset) {
    return reset ? pk::g_launches.exchange(0) : pk::g_launches.load();
}

const char* pk_version(void) { return "polykern 0.1 (sm_100a)"; }

const char* pk_last_error(void) { return pk::g_last_error.c_str(); }

int pk_device_status(int reset) {
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return pk::cuda_fail(e, "pk_device_status: cudaDeviceSynchronize");
    int value = 0;
    e = cudaMemcpyFromSymbol(&value, pk_device_status_word, sizeof(int));
    if (e != cudaSuccess) return pk::cuda_fail(e, "pk_device_status: read status word");
    if (reset) {
        int zero = 0;
        e = cudaMemcpyToSymbol(pk_device_status_word, &zero, sizeof(int));
        if (e != cudaSuccess) return pk::cuda_fail(e, "pk_device_status: clear status word");
    }
    return value;
}

}  // extern "C"
