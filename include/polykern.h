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

/* Library identification and diagnostics (no counterpart in the reference: its rules are Python
 * that raises on failure, where these entry points return status codes). */
PK_API const char* pk_version(void);
PK_API const char* pk_last_error(void);

/*
 * Device-side status word: kernels whose internal waits time out write a nonzero
 * code here instead of hanging.  pk_device_status() synchronises the current
 * device and returns (and with reset != 0, clears) that word.  No counterpart in the reference.
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
 * Number of kernels the library has launched in this process (all entry points, all
 * devices and streams), for counting launches inside a timed region; reset != 0 returns
 * the count and sets it to zero.  No counterpart in the reference.
 */
PK_API int64_t pk_launch_count(int reset);

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
 *   workspace:   device buffer of at least pk_poly_gemm_workspace_query(...) bytes for
 *                this call (pk_poly_gemm_workspace_size(...) bounds every call of the
 *                shape); may be null when the query returns 0.  bf16 operands whose
 *                planes are 16-byte aligned with k or rows contiguous (other strides
 *                multiples of 8 elements, rows not overlapping) are read in place and
 *                need no workspace; every other operand is staged through it.
 */
PK_API size_t pk_poly_gemm_workspace_size(int dtype, int degree, int64_t batch,
                                   int64_t M, int64_t N, int64_t K,
                                   int a_complex_from, int b_complex_from);
/* Workspace bytes the pk_poly_gemm call with these operands needs (*bytes; 0 = none).
 * The reference has no workspace (its products are separate PyTorch GEMMs); this pairs
 * with pk_poly_gemm, which replaces src/polytensors/_plain.py:118-128. */
PK_API int pk_poly_gemm_workspace_query(int dtype, int degree, int64_t batch,
                                        int64_t M, int64_t N, int64_t K,
                                        const void* const* a_planes, int64_t a_bs, int64_t a_rs, int64_t a_cs,
                                        const void* const* b_planes, int64_t b_bs, int64_t b_rs, int64_t b_cs,
                                        int a_complex_from, int b_complex_from, size_t* bytes);
PK_API int pk_poly_gemm(int dtype, int degree, int64_t batch, int64_t M, int64_t N, int64_t K,
                 const void* const* a_planes, int64_t a_bs, int64_t a_rs, int64_t a_cs,
                 const void* const* b_planes, int64_t b_bs, int64_t b_rs, int64_t b_cs,
                 void* const* c_planes, int64_t c_bs, int64_t c_rs,
                 int a_complex_from, int b_complex_from,
                 void* workspace, size_t workspace_bytes, void* stream);
/* pk_poly_gemm (accumulate = 0) or pk_poly_gemm_accumulate (accumulate != 0) for operands
 * whose A planes are zero outside a band, as the causal attention products are:
 *   band 1: A[b][m][k] may be nonzero only for k >= m + band_offset,
 *   band 2: A[b][m][k] may be nonzero only for k <= m + band_offset,
 *   band 3: only the outputs C[b][m][n] with n <= m + band_offset are wanted (causal scores);
 *           the others are unspecified (zero where a whole output tile lies beyond the band),
 *   band 0: no band (plain product).
 * For bands 1 and 2, k blocks outside the band of a whole row tile are skipped (the caller
 * guarantees the skipped entries are zero; the product may still read some of them).  Replaces the same products as
 * pk_poly_gemm; the reference evaluates them over the full (masked) score matrices
 * (src/polytensors/_decompositions.py:28-43). */
PK_API int pk_poly_gemm_banded(int dtype, int degree, int64_t batch, int64_t M, int64_t N, int64_t K,
                 const void* const* a_planes, int64_t a_bs, int64_t a_rs, int64_t a_cs,
                 const void* const* b_planes, int64_t b_bs, int64_t b_rs, int64_t b_cs,
                 void* const* c_planes, int64_t c_bs, int64_t c_rs,
                 int a_complex_from, int b_complex_from, int accumulate, int band, int64_t band_offset,
                 void* workspace, size_t workspace_bytes, void* stream);
/* C_k += sum_{i+j=k} A_i B_j: pk_poly_gemm accumulating into the existing output planes
 * (the beta = alpha = 1 case of addmm, src/polytensors/_range_ops.py:160-176).  Same
 * arguments and workspace. */
PK_API int pk_poly_gemm_accumulate(int dtype, int degree, int64_t batch, int64_t M, int64_t N, int64_t K,
                 const void* const* a_planes, int64_t a_bs, int64_t a_rs, int64_t a_cs,
                 const void* const* b_planes, int64_t b_bs, int64_t b_rs, int64_t b_cs,
                 void* const* c_planes, int64_t c_bs, int64_t c_rs,
                 int a_complex_from, int b_complex_from,
                 void* workspace, size_t workspace_bytes, void* stream);

/*
 * float32 polynomial product whose operands may arrive already split for the bf16 tensor
 * cores: with a_hilo != 0, a_planes holds 2(n+1) bfloat16 planes hi_0, lo_0, hi_1, lo_1, ...
 * (x_k ~= hi_k + lo_k, strides in bf16 elements) that are read in place — no staging pass —
 * either k-contiguous or rows-contiguous, 16-byte aligned, other strides multiples of 8
 * elements; with a_hilo == 0, n+1 float32 planes as in pk_poly_gemm (staged into the
 * workspace).  Likewise for B.  Output: n+1 float32 planes, written or (accumulate != 0)
 * added to; band / band_offset as in pk_poly_gemm_banded.  degree <= 7 when an operand is
 * pre-split.  Used by the float32 attention (probability and score-gradient planes come out of
 * the score kernels already split).  Replaces the same rule as pk_poly_gemm
 * (src/polytensors/_plain.py:118-128) for that case.
 */
PK_API int pk_poly_gemm_hilo_workspace_query(int degree, int64_t batch, int64_t M, int64_t N, int64_t K,
                                             const void* const* a_planes, int64_t a_bs, int64_t a_rs, int64_t a_cs,
                                             int a_hilo, const void* const* b_planes, int64_t b_bs, int64_t b_rs,
                                             int64_t b_cs, int b_hilo, size_t* bytes);
PK_API int pk_poly_gemm_hilo(int degree, int64_t batch, int64_t M, int64_t N, int64_t K, const void* const* a_planes,
                             int64_t a_bs, int64_t a_rs, int64_t a_cs, int a_hilo, const void* const* b_planes,
                             int64_t b_bs, int64_t b_rs, int64_t b_cs, int b_hilo, void* const* c_planes,
                             int64_t c_bs, int64_t c_rs, int accumulate, int band, int64_t band_offset,
                             void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------------
 * Elementwise series operations.  out = f(a) or f(a, b) for every element, all planes
 * at once.  Shapes broadcast through strides (0 for a broadcast dimension, at most 6
 * dimensions); out, a and b share `shape` and the storage dtype (PK_F32, PK_F64,
 * PK_BF16, PK_F16; bf16/f16 compute in float).  a_planes / b_planes is degree+1 for a
 * series operand or 1 for a constant operand (its higher coefficients are zero).  out
 * may alias a (in-place update, e.g. an SGD step) when their strides are equal.
 */
enum pk_series_op {
    PK_OP_COPY = 0,        /* out = a */
    PK_OP_AFFINE = 1,      /* out = p0*a + p1 (p1 on the constant term): neg, scale, add/rsub scalar */
    PK_OP_EXP = 2,         /* src/polytensors/_plain.py:153-159 */
    PK_OP_LOG = 3,         /* src/polytensors/_plain.py:162-171 */
    PK_OP_SQRT = 4,        /* src/polytensors/_series.py:72-81, _plain.py:294-298 */
    PK_OP_RSQRT = 5,       /* src/polytensors/_series.py:83-96 */
    PK_OP_RECIPROCAL = 6,  /* src/polytensors/_range_ops.py:157-158 */
    PK_OP_TANH = 7,        /* src/polytensors/_plain.py:303-304 */
    PK_OP_SIGMOID = 8,     /* src/polytensors/_plain.py:303-304 */
    PK_OP_GELU = 9,        /* exact GELU, src/polytensors/_plain.py:305-309 */
    PK_OP_POWI = 10,       /* a^p0, p0 a nonnegative integer, src/polytensors/_dispatch.py:419-429 */
    PK_OP_ADD = 32,        /* out = a + p0*b, src/polytensors/_range_ops.py:137-142 */
    PK_OP_MUL = 33,        /* Cauchy product, src/polytensors/_range_ops.py:143-144 */
    PK_OP_DIV = 34,        /* series quotient, src/polytensors/_range_ops.py:86-93 */
    PK_OP_GELU_BWD = 35,   /* a = gradient, b = input: a * gelu'(b), src/polytensors/_plain.py:310-315 */
    PK_OP_TANH_BWD = 36,   /* a = gradient, b = output: a * (1 - b^2), src/polytensors/_plain.py:316-320 */
    PK_OP_SIGMOID_BWD = 37 /* a = gradient, b = output: a * b * (1 - b), src/polytensors/_plain.py:321-325 */
};
/*
 * Extended-range series (the reference's default mode, src/polytensors/_scaled.py,
 * src/polytensors/_range_ops.py): each coefficient element is a mantissa m (float32 for
 * float32 / bfloat16 / float16 series, float64 for float64; |m| in [1, 2), 0 or non-finite) and an
 * int32 binary exponent e, value m * 2^e.  Planes are contiguous (numel elements).
 * pk_scaled_from:  values (dtype) -> (m, e + base_exponent), normalised.
 * pk_scaled_to:    (m, e - exponent_offset) -> values of dtype (only this step can overflow or
 *                  underflow, as the reference's to_tensor).
 * pk_scaled_series_map: PK_OP_COPY / AFFINE (p0 a + p1) / ADD (a + p0 b) / MUL (truncated Cauchy
 *                  product, terms added in order) / DIV (quotient recurrence) / EXP (exp of the base
 *                  from its logarithm, then the exponential recurrence) over (m, e) planes,
 *                  strides and broadcasting as pk_series_map.
 * pk_scaled_reduce: out[o][i] = sum_r x[o][r][i], aligned to the largest exponent of the nonzero
 *                  terms of each sum.
 */
PK_API int pk_scaled_from(int dtype, int degree, int64_t numel, const void* const* x, void* const* m,
                          int32_t* const* e, int32_t base_exponent, void* stream);
PK_API int pk_scaled_to(int dtype, int mantissa_dtype, int degree, int64_t numel, const void* const* m,
                        const int32_t* const* e, int32_t exponent_offset, void* const* out, void* stream);
PK_API int pk_scaled_series_map(int op, int mantissa_dtype, int degree, int ndim, const int64_t* shape,
                                void* const* out_m, int32_t* const* out_e, const int64_t* out_strides,
                                const void* const* a_m, const int32_t* const* a_e, int a_planes,
                                const int64_t* a_strides, const void* const* b_m, const int32_t* const* b_e,
                                int b_planes, const int64_t* b_strides, double p0, double p1, void* stream);
PK_API int pk_scaled_reduce(int mantissa_dtype, int degree, int64_t outer, int64_t red, int64_t inner,
                            const void* const* m, const int32_t* const* e, void* const* out_m,
                            int32_t* const* out_e, void* stream);

/* float32 planes (numel contiguous elements each, degree + 1 of them) -> bf16 hi/lo pairs
 * out = [hi_0, lo_0, hi_1, ...] with hi = bf16(x) and lo = bf16(x - hi) (round to nearest): the
 * operand form read in place by pk_poly_gemm_hilo and the float32 attention kernels.  No
 * counterpart in the reference (its float32 products are single PyTorch matmuls). */
PK_API int pk_split_hilo(int degree, int64_t numel, const void* const* x, void* const* out, void* stream);

PK_API int pk_series_map(int op, int dtype, int degree, int ndim, const int64_t* shape,
                         void* const* out, const int64_t* out_strides,
                         const void* const* a, int a_planes, const int64_t* a_strides,
                         const void* const* b, int b_planes, const int64_t* b_strides,
                         double p0, double p1, void* stream);
/* pk_series_map on series with complex planes: plane k of out / a / b holds interleaved
 * (re, im) pairs of real_dtype (PK_F32 -> complex64, PK_F64 -> complex128) when bit k of
 * out_complex / a_complex / b_complex is set, else real values of real_dtype; strides count
 * elements.  Every operation of pk_series_map; PK_OP_TANH, PK_OP_GELU and PK_OP_GELU_BWD need a
 * real base (plane 0 of their series argument), which the caller checks.  Replaces the
 * reference's plain-range rules on complex coefficients (src/polytensors/_plain.py, with the
 * real-base / complex-direction promotion of :77-80). */
PK_API int pk_series_map_complex(int op, int real_dtype, int degree, int ndim, const int64_t* shape,
                                 void* const* out, const int64_t* out_strides, uint32_t out_complex,
                                 const void* const* a, int a_planes, const int64_t* a_strides, uint32_t a_complex,
                                 const void* const* b, int b_planes, const int64_t* b_strides, uint32_t b_complex,
                                 double p0, double p1, void* stream);

/*
 * out[o, i] = scale * sum_r x[o, r, i] for every plane; x is contiguous [outer][red][inner],
 * out contiguous [outer][inner].  Replaces the per-plane sum/mean of
 * src/polytensors/_range_ops.py:178-193 (mean: scale = 1/count).  float32 / float64.
 */
PK_API int pk_series_reduce(int dtype, int degree, int64_t outer, int64_t red, int64_t inner,
                            const void* const* x, void* const* out, double scale, void* stream);

/*
 * Embedding rows: out[i, :] = src[idx[i], :] (gather, src/polytensors/_dispatch.py:530-532) and
 * its backward out[idx[i], :] += src[i, :] over a zeroed (n_rows, dim) output, skipping
 * idx == padding_idx (src/polytensors/_dispatch.py:683-685).  idx is a device int64 array;
 * out-of-range indices are skipped and reported through pk_device_status.  float32 / float64.
 */
PK_API int pk_series_gather_rows(int dtype, int degree, int64_t n_idx, int64_t dim, const int64_t* idx,
                                 const void* const* src, int64_t src_rs, int64_t n_rows,
                                 void* const* out, void* stream);
PK_API int pk_series_scatter_add_rows(int dtype, int degree, int64_t n_idx, int64_t dim, const int64_t* idx,
                                      int64_t padding_idx, const void* const* src, int64_t src_rs,
                                      int64_t n_rows, void* const* out, void* stream);

/* ---------------------------------------------------------------------------------
 * Row-wise series kernels over a (rows, cols) view: plane k of row r starts at
 * planes[k] + r * row_stride and its cols elements are contiguous.
 */

/*
 * RMSNorm: y = x (*) rsqrt(mean_row(x (*) x) + eps) (*) w, (*) the truncated Cauchy product.
 * Replaces the decomposition of src/polytensors/_decompositions.py:14-22 and generalises the
 * degree-1 kernels of src/polytensors/_norm_kernels.py:6-38 (gate src/polytensors/_fused_norm.py:11-21).
 * w: NULL (no weight), or w_planes = 1 (constant weight) / degree+1 planes of cols elements.
 * rstd (optional): receives the per-row rsqrt series, [rows][degree+1] in float (float64 for PK_F64),
 * which pk_rmsnorm_bwd needs.
 */
PK_API int pk_rmsnorm_fwd(int dtype, int degree, int64_t rows, int64_t cols,
                          const void* const* x, int64_t x_rs, const void* const* w, int w_planes,
                          double eps, void* const* y, int64_t y_rs, void* rstd, void* stream);
/*
 * Gradient series of pk_rmsnorm_fwd for the output-gradient series g: dx, and (if dw is not NULL)
 * dw (degree+1 planes of cols elements; needs a workspace of pk_rmsnorm_bwd_workspace_size bytes).
 */
PK_API size_t pk_rmsnorm_bwd_workspace_size(int dtype, int degree, int64_t rows, int64_t cols);
PK_API int pk_rmsnorm_bwd(int dtype, int degree, int64_t rows, int64_t cols,
                          const void* const* x, int64_t x_rs, const void* const* w, int w_planes,
                          const void* const* g, int64_t g_rs, const void* rstd,
                          void* const* dx, int64_t dx_rs, void* const* dw,
                          void* workspace, size_t workspace_bytes, void* stream);

/*
 * Softmax / log-softmax along rows (log = 1 for log_softmax), and their backward rules:
 * src/polytensors/_plain.py:262-273 (forward), :342-347 (softmax backward), :348-354
 * (log-softmax backward; y is the forward output).
 */
PK_API int pk_softmax_fwd(int dtype, int degree, int64_t rows, int64_t cols,
                          const void* const* x, int64_t x_rs, int log, void* const* y, int64_t y_rs,
                          void* stream);
PK_API int pk_softmax_bwd(int dtype, int degree, int64_t rows, int64_t cols,
                          const void* const* g, int64_t g_rs, const void* const* y, int64_t y_rs, int log,
                          void* const* dx, int64_t dx_rs, void* stream);

/*
 * Cross entropy of (rows, cols) logits series with int64 class targets (device array):
 * loss[k][r] = -log_softmax_k(z[r])[target[r]], 0 where target == ignore_index; softcap > 0
 * first maps z -> softcap * tanh(z / softcap) as a series.  Loss planes and the per-row
 * statistics (stats: [rows][degree+1]) are float for PK_F32/PK_BF16/PK_F16 and double for PK_F64.
 * pk_cross_entropy_bwd: dz = d/dz of sum_r <g[.][r], loss[.][r]> as a series, for the per-row
 * gradient series g (same precision as the loss); rows with target == ignore_index get 0.
 * Replaces F.cross_entropy = log_softmax + nll_loss in plain range (src/polytensors/_plain.py:326-332,
 * src/polytensors/_dispatch.py:537-562) and generalises the degree-1 fused kernels
 * (src/polytensors/_cross_entropy_kernels.py:19-85, src/polytensors/_fused_cross_entropy.py:54-76).
 */
PK_API int pk_cross_entropy_fwd(int dtype, int degree, int64_t rows, int64_t cols,
                                const void* const* z, int64_t z_rs, const int64_t* target,
                                int64_t ignore_index, double softcap, void* const* loss, void* stats,
                                void* stream);
PK_API int pk_cross_entropy_bwd(int dtype, int degree, int64_t rows, int64_t cols,
                                const void* const* z, int64_t z_rs, const int64_t* target,
                                int64_t ignore_index, double softcap, const void* stats,
                                const void* const* g, void* const* dz, int64_t dz_rs, void* stream);

/*
 * Attention score kernels for series attention built from pk_poly_gemm contractions
 * (the reference's decomposition, src/polytensors/_decompositions.py:28-43, evaluated a
 * block of heads at a time).  Rows are score rows of (rows / q_len) matrices; row r is query
 * r % q_len; with causal != 0, keys beyond query + causal_shift are masked out.
 * pk_attn_probs: P = softmax(scale * scores) as series (src/polytensors/_plain.py:262-273),
 *   stats [rows][degree+1] = (lse_0, logz_1..n), float (double for PK_F64).
 * pk_attn_dscores: d scores = scale * P (*) (dP - dsum) from the probabilities P of pk_attn_probs,
 *   dsum [rows][degree+1] = sum_d dO (*) O (src/polytensors/_plain.py:342-347); masked entries
 *   (P = 0) get zero.  dscores may alias dprobs.
 */
PK_API int pk_attn_probs(int dtype, int degree, int64_t rows, int64_t cols, int64_t q_len,
                         const void* const* scores, int64_t s_rs, double scale, int causal,
                         int64_t causal_shift, void* const* probs, int64_t p_rs, void* stats, void* stream);
PK_API int pk_attn_dscores(int dtype, int degree, int64_t rows, int64_t cols,
                           const void* const* probs, int64_t p_rs, const void* const* dprobs, int64_t dp_rs,
                           const void* dsum, double scale, void* const* dscores, int64_t ds_rs, void* stream);
/* dsum[row][k] = (sum_d dO (*) O)_k over the rows of the attention output and its gradient
 * (rows x cols planes, row strides do_rs / o_rs elements): the row term of the score gradient,
 * sum_d dO (*) O (src/polytensors/_plain.py:342-347 applied to the attention's P V product).
 * dsum is float32 ([rows][degree+1]; float64 for PK_F64). */
PK_API int pk_attn_dsum(int dtype, int degree, int64_t rows, int64_t cols, const void* const* dO, int64_t do_rs,
                        const void* const* O, int64_t o_rs, void* dsum, void* stream);
/* float32 forms whose probabilities and score gradients are bf16 hi/lo pairs (2(n+1) planes
 * hi_0, lo_0, hi_1, ...; x ~= hi + lo), the operand form pk_poly_gemm_hilo reads without staging.
 * Scores and dprobs stay float32 (n+1 planes).  degree <= 7; outputs must not alias inputs.
 * They replace the same reference rules as pk_attn_probs / pk_attn_dscores
 * (src/polytensors/_plain.py:262-273, :342-347). */
PK_API int pk_attn_probs_hilo(int degree, int64_t rows, int64_t cols, int64_t q_len,
                              const void* const* scores, int64_t s_rs, double scale, int causal,
                              int64_t causal_shift, void* const* probs, int64_t p_rs, void* stats, void* stream);
PK_API int pk_attn_dscores_hilo(int degree, int64_t rows, int64_t cols,
                                const void* const* probs, int64_t p_rs, const void* const* dprobs, int64_t dp_rs,
                                const void* dsum, double scale, void* const* dscores, int64_t ds_rs, void* stream);

/*
 * Series flash attention forward in one kernel: O = softmax(scale * Q K^T, causal) V with
 * truncated Cauchy products, bfloat16 planes, fp32 accumulation, degree <= 3, head dim 64 or
 * 128.  q/o: [bh][L][D], k/v: [bh][S][D], contiguous, 16-byte aligned.  Key index j is
 * admissible for query i when j <= i (causal != 0).  Generalises the degree-1 Triton forward
 * (src/polytensors/_attention_kernels.py:27-82) and replaces the decomposition of
 * src/polytensors/_decompositions.py:28-43 (whose (L, S) score series it never forms).
 * dtype PK_F32 (float32 attention, head dim 64): q, k, v each hold 2(n+1) bf16 planes
 * hi_0, lo_0, hi_1, ... with x ~= hi + lo, every product evaluated as hi*hi + hi*lo + lo*hi
 * with fp32 accumulation; o holds n+1 float32 planes.
 */
PK_API int pk_flash_attn_fwd(int dtype, int degree, int64_t bh, int64_t L, int64_t S, int64_t D,
                             const void* const* q, const void* const* k, const void* const* v,
                             void* const* o, int causal, double scale, void* stats, void* stream);
/*   stats (optional, may be null): float32 [bh][L][degree+1], the softmax normaliser series of
 *   every query row as pk_attn_probs writes it (lse_0, logz_1..n), for the backward. */

/*
 * Attention score products with the softmax in the epilogue, for the series attention
 * backward (bfloat16 planes, degree <= 3).  Operands as in pk_poly_gemm (batch x M x K and
 * batch x K x N, element strides), read in place: every plane 16-byte aligned with k or
 * rows contiguous and the other strides multiples of 8 elements (PK_ERR_UNSUPPORTED
 * otherwise).  Row values (stats, dsum): float32 [batch][M][degree+1], batch entries
 * stats_bs / dsum_bs floats apart.  Query index of row r is r + causal_shift; with causal
 * != 0, key j is admissible for it when j <= r + causal_shift.  causal == 1 writes the zeros
 * of every inadmissible entry; causal == 2 writes them only within 192 keys of the admissible
 * region (the most that band-limited consumers such as pk_poly_gemm_banded read there) and
 * leaves 64-key tiles lying wholly further out unwritten.
 *
 * pk_attn_probs_gemm:   probs = exp-series(scale * Q K^T - stats) on admissible keys, 0 elsewhere
 *                       (pk_poly_gemm followed by pk_attn_probs with the forward's stats).
 * pk_attn_dscores_gemm: dscores = scale * probs (*) (dO V^T - dsum)
 *                       (pk_poly_gemm followed by pk_attn_dscores).
 * Together they replace the score and softmax-backward steps of the reference's attention
 * backward (src/polytensors/_decompositions.py:28-43 through src/polytensors/_plain.py:342-347;
 * degree-1 Triton form src/polytensors/_attention_kernels.py:84-201).
 * dtype PK_F32 (float32 attention, reduction <= 64): every plane array — operands, probs and
 * the output — holds 2(n+1) bf16 planes hi_0, lo_0, hi_1, ... (x ~= hi + lo); products are
 * hi*hi + hi*lo + lo*hi in fp32 and the outputs are written split the same way, ready for
 * pk_poly_gemm_hilo.
 *
 * In this form pk_attn_dscores_gemm writes its output key-major, dscores[b][key][query] at
 * b * ds_bs + key * ds_rs + query (the transpose of the bf16 layout), so that its stores are
 * coalesced; both gradient products read that layout in place.
 */
PK_API int pk_attn_probs_gemm(int dtype, int degree, int64_t batch, int64_t M, int64_t N, int64_t K,
                              const void* const* q, int64_t q_bs, int64_t q_rs, int64_t q_cs,
                              const void* const* kt, int64_t kt_bs, int64_t kt_rs, int64_t kt_cs,
                              void* const* probs, int64_t p_bs, int64_t p_rs,
                              const void* stats, int64_t stats_bs, double scale, int causal,
                              int64_t causal_shift, void* stream);
PK_API int pk_attn_dscores_gemm(int dtype, int degree, int64_t batch, int64_t M, int64_t N, int64_t K,
                                const void* const* dout, int64_t do_bs, int64_t do_rs, int64_t do_cs,
                                const void* const* vt, int64_t vt_bs, int64_t vt_rs, int64_t vt_cs,
                                const void* const* probs, int64_t p_bs, int64_t p_rs,
                                const void* dsum, int64_t dsum_bs, double scale, int causal,
                                int64_t causal_shift, void* const* dscores, int64_t ds_bs, int64_t ds_rs,
                                void* stream);

/*
 * pk_poly_gemm without a workspace argument, for callers that cannot allocate device
 * memory (a plugin host that owns every allocation, a process that must not grow its
 * device footprint after start-up, code with no allocator to link).  The scratch comes
 * from a fixed PK_NOALLOC_SCRATCH_BYTES array in the library's device memory, held on
 * every GPU that loads the library until the process exits.  Products needing more
 * scratch than that (pk_poly_gemm_workspace_query) fail with PK_ERR_UNSUPPORTED.  The
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
