// pk_poly_gemm_noalloc: the polynomial matrix product for callers that cannot
// allocate device memory.
//
// pk_poly_gemm needs a scratch workspace (the operands are re-staged into K-major
// bf16 hi/lo or float64 sub-planes before the tensor-core product).  Some callers
// cannot provide one: code running where cudaMalloc is unavailable or forbidden, such
// as a plugin host that owns every device allocation itself, a process that must not
// grow its memory footprint after start-up, or code that cannot link an allocator.
// This entry point takes the scratch from a fixed array in the library's own device
// memory instead, so the caller passes only inputs and outputs.
//
// Limits and behaviour
//   - The array holds PK_NOALLOC_SCRATCH_BYTES (64 MiB).  Every GPU that loads the
//     library keeps it reserved until the process exits.  A product whose workspace
//     (pk_poly_gemm_workspace_query) is larger is rejected with PK_ERR_UNSUPPORTED;
//     bf16 operands read in place need none.
//   - The first call on a device looks up the array's device address for that device
//     (cudaGetSymbolAddress with the device current).  Make that first call before any
//     stream capture begins.
//   - All calls share the one array and it keeps the contents of the last call.  The
//     product overwrites every scratch byte it reads, so nothing needs clearing between
//     calls.  Calls whose work overlaps on the GPU (different streams, or host threads
//     without ordering) race on the array: order them on one stream.
//   - Nothing here calls cudaMalloc, cudaFree or any allocating library routine.
#include <mutex>

#include "pk_common.cuh"

static __device__ __align__(256) unsigned char pk_noalloc_scratch[PK_NOALLOC_SCRATCH_BYTES];

namespace {

std::mutex g_scratch_mutex;
void* g_scratch_ptr[64] = {nullptr};

// Device address of pk_noalloc_scratch on the current device (looked up once per device).
int scratch_for_current_device(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return pk::cuda_fail(e, "pk_poly_gemm_noalloc: cudaGetDevice");
    if (dev < 0 || dev >= 64) return pk::fail(PK_ERR_UNSUPPORTED, "pk_poly_gemm_noalloc: device index above 63");
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, pk_noalloc_scratch);
        if (e != cudaSuccess) return pk::cuda_fail(e, "pk_poly_gemm_noalloc: cudaGetSymbolAddress(scratch)");
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return PK_OK;
}

}  // namespace

extern "C" int pk_poly_gemm_noalloc(int dtype, int degree, int64_t batch, int64_t M, int64_t N, int64_t K,
                                    const void* const* a_planes, int64_t a_bs, int64_t a_rs, int64_t a_cs,
                                    const void* const* b_planes, int64_t b_bs, int64_t b_rs, int64_t b_cs,
                                    void* const* c_planes, int64_t c_bs, int64_t c_rs, int a_complex_from,
                                    int b_complex_from, void* stream) {
    size_t need = 0;
    const int qrc = pk_poly_gemm_workspace_query(dtype, degree, batch, M, N, K, a_planes, a_bs, a_rs, a_cs, b_planes,
                                                 b_bs, b_rs, b_cs, a_complex_from, b_complex_from, &need);
    if (qrc != PK_OK) return qrc;
    if (need > PK_NOALLOC_SCRATCH_BYTES)
        return pk::fail(PK_ERR_UNSUPPORTED,
                        "pk_poly_gemm_noalloc: this product needs " + std::to_string(need) +
                            " bytes of scratch but the built-in scratch array holds " +
                            std::to_string(static_cast<unsigned long long>(PK_NOALLOC_SCRATCH_BYTES)) +
                            " bytes; use pk_poly_gemm with a caller-provided workspace");
    void* scratch = nullptr;
    const int rc = scratch_for_current_device(&scratch);
    if (rc != PK_OK) return rc;
    return pk_poly_gemm(dtype, degree, batch, M, N, K, a_planes, a_bs, a_rs, a_cs, b_planes, b_bs, b_rs, b_cs,
                        c_planes, c_bs, c_rs, a_complex_from, b_complex_from, scratch, PK_NOALLOC_SCRATCH_BYTES,
                        stream);
}
