/*
 * polykern.h - C ABI of libpolykern.so, the sm_100a kernels behind the PolyTensor
 * truncated Taylor-series hot path.
 *
 * A "series" of degree n is a tuple of n+1 coefficient tensors ("planes") c_0..c_n
 * representing p(t) = sum_k c_k t^k truncated after t^n.  Every entry point takes
 * one device pointer per plane (a host array of n+1 pointers), the shared shape and
 * element strides of those planes, and a cudaStream_t (passed as void*).  Work is
 * enqueued asynchronously on that stream.
 *
 * Conventions
 *   - Return value: 0 on success, negative on failure.  pk_last_error() returns a
 *     thread-local description of the last failure on the calling thread.
 *   - Ownership: the caller allocates every input, output and workspace buffer.
 *     The library never allocates or frees device memory and keeps no pointer
 *     after a call returns.
 *   - Strides are in elements of the plane's storage type (a complex128 element
 *     counts as one element).
 *   - No entry point has a CPU fallback: a missing GPU or an unsupported
 *     configuration is an error.
 *
 * Each declaration cites the reference function it replaces (paths inside the
 * samuel-gunn/poly-tensors project).
 */
#ifndef POLYKERN_H
#define POLYKERN_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define PK_API __attribute__((visibility("default")))
#else
#define PK_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Storage / arithmetic types of a plane. */
enum pk_dtype {
    PK_F32 = 0,   /* float32 planes; products use a 3-term bf16 split on tcgen05 (fp32 accumulate) */
    PK_F64 = 1,   /* float64 planes; DMMA (mma.sync f64) */
    PK_BF16 = 2,  /* bfloat16 planes; tcgen05 kind::f16, fp32 accumulate */
    PK_F16 = 3,   /* float16 planes; tcgen05 kind::f16, fp32 accumulate */
    PK_C128 = 4   /* complex128 planes (interleaved re/im); DMMA on planar parts */
};

/* Status codes. */
enum pk_status {
    PK_OK = 0,
    PK_ERR_ARG = -1,          /* invalid argument (null pointer, negative size, bad stride) */
    PK_ERR_UNSUPPORTED = -2,  /* configuration outside what the kernels implement */
    PK_ERR_CUDA = -3,         /* a CUDA runtime/driver call failed */
    PK_ERR_WORKSPACE = -4,    /* workspace missing or too small */
    PK_ERR_TIMEOUT = -5       /* a device-side wait gave up (see pk_device_status) */
};

#define PK_MAX_PLANES 16   /* degree <= 15 */

/* Library identification and diagnostics. */
PK_API const char* pk_version(void);
PK_API const char* pk_last_error(void);

/*
 * Device-side status word: kernels whose internal waits time out write a nonzero
 * code here instead of hanging.  pk_device_status() synchronises the current
 * device and returns (and with reset != 0, clears) that word.
 */
PK_API int pk_device_status(int reset);

/*
 * Launch timing for benchmarks: after pk_profile_enable(1), each entry point records
 * CUDA events on its stream around its main kernel (named "poly_gemm", ...).
 * pk_profile_query() waits for the recorded events of `kernel`, returns their summed
 * duration and count, and forgets them.  No counterpart in the reference.
 */
PK_API int pk_profile_enable(int on);
PK_API int pk_profile_query(const char* kernel, double* total_ms, int64_t* launches);

/*
 * Polynomial (block-Toeplitz) matrix product, C_k = sum_{i=0..k} A_i @ B_{k-i},
 * k = 0..degree, for a batch of matrices.
 * Replaces plain_polynomial_product(matrix=True)   (src/polytensors/_plain.py:118-128)
 * as reached from mm/bmm/matmul/mv/dot/addmm/linear (src/polytensors/_range_ops.py:160-176),
 * including real-base / complex-direction promotion     (src/polytensors/_plain.py:77-80).
 *
 *   a_planes[p]: batch x M x K, element (b,m,k) at b*a_bs + m*a_rs + k*a_cs
 *   b_planes[p]: batch x K x N, element (b,k,n) at b*b_bs + k*b_rs + n*b_cs
 *   c_planes[p]: batch x M x N, element (b,m,n) at b*c_bs + m*c_rs + n   (written, not accumulated)
 *   dtype:       PK_F32 / PK_BF16 / PK_F16 / PK_F64 for real planes.  With PK_C128,
 *                planes with index >= a_complex_from (resp. b_complex_from) are
 *                complex128 and lower planes are float64 (a real base with complex
 *                directions); pass degree+1 for "no complex plane".  Output plane k
 *                is complex128 iff some term A_i B_{k-i} has a complex factor.
 *   workspace:   device buffer of at least pk_poly_gemm_workspace_size(...) bytes,
 *                16-byte aligned.
 */
PK_API size_t pk_poly_gemm_workspace_size(int dtype, int degree, int64_t batch,
                                   int64_t M, int64_t N, int64_t K,
                                   int a_complex_from, int b_complex_from);
PK_API int pk_poly_gemm(int dtype, int degree, int64_t batch, int64_t M, int64_t N, int64_t K,
                 const void* const* a_planes, int64_t a_bs, int64_t a_rs, int64_t a_cs,
                 const void* const* b_planes, int64_t b_bs, int64_t b_rs, int64_t b_cs,
                 void* const* c_planes, int64_t c_bs, int64_t c_rs,
                 int a_complex_from, int b_complex_from,
                 void* workspace, size_t workspace_bytes, void* stream);

/*
 * pk_poly_gemm without a workspace argument, for callers that cannot allocate device
 * memory (a plugin host that owns every allocation, a process that must not grow its
 * device footprint after start-up, code with no allocator to link).  The scratch comes
 * from a fixed PK_NOALLOC_SCRATCH_BYTES array in the library's device memory, held on
 * every GPU that loads the library until the process exits.  Products needing more
 * scratch than that (pk_poly_gemm_workspace_size) fail with PK_ERR_UNSUPPORTED.  The
 * first call on a device looks up the array's address; make it before any stream
 * capture.  All calls share the array: calls that overlap on the GPU race, so order
 * them on one stream.  Allocates nothing.
 * No counterpart in the reference (an addition of this library).
 */
#define PK_NOALLOC_SCRATCH_BYTES (64ull << 20)
PK_API int pk_poly_gemm_noalloc(int dtype, int degree, int64_t batch, int64_t M, int64_t N, int64_t K,
                                const void* const* a_planes, int64_t a_bs, int64_t a_rs, int64_t a_cs,
                                const void* const* b_planes, int64_t b_bs, int64_t b_rs, int64_t b_cs,
                                void* const* c_planes, int64_t c_bs, int64_t c_rs,
                                int a_complex_from, int b_complex_from, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* POLYKERN_H */
