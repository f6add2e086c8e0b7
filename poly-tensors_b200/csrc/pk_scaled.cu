// Extended-range series arithmetic: every coefficient element is a mantissa m (|m| in [1, 2), or 0,
// or a non-finite value) and a binary exponent e (int32), value = m * 2^e, so products and sums
// whose values leave the range of the storage dtype stay finite until a result is converted back.
// This is the reference's default (non-plain-range) representation (src/polytensors/_scaled.py:
// normalisation :82-103, add :260-271, mul :279-288, div :290-298, sum :303-324, to_tensor
// :334-342) and its series rules over it (src/polytensors/_range_ops.py:26-120 with the
// coefficient convolution of src/polytensors/_scaled_matmul.py:38-40).  Planes are contiguous;
// mantissas are float (for float32 / bfloat16 / float16 series) or double (float64).
#include <algorithm>
#include <climits>

#include "pk_common.cuh"
#include "pk_series.cuh"

namespace pk {

template <typename C>
struct SV {
    C m;
    int e;
};

__device__ __forceinline__ float sc_frexp(float v, int* ex) { return frexpf(v, ex); }
__device__ __forceinline__ double sc_frexp(double v, int* ex) { return frexp(v, ex); }
__device__ __forceinline__ float sc_ldexp(float v, int ex) { return ldexpf(v, ex); }
__device__ __forceinline__ double sc_ldexp(double v, int ex) { return ldexp(v, ex); }

// v * 2^e normalised: |m| in [1, 2) for finite nonzero v (the reference keeps [1, 2) so that a
// finite maximum converts without a nonrepresentable power of two); zero and non-finite values
// keep their value and the exponent (exponents are clamped to +-1e9).
template <typename C>
__device__ __forceinline__ SV<C> sc_norm(C v, long long e) {
    SV<C> r;
    if (v == C(0) || !isfinite(v)) {
        r.m = v;
        r.e = static_cast<int>(max(min(e, 1000000000LL), -1000000000LL));
        return r;
    }
    int ex = 0;
    const C f = sc_frexp(v, &ex);  // v = f 2^ex, |f| in [1/2, 1)
    r.m = f * C(2);
    const long long t = e + ex - 1;
    r.e = static_cast<int>(max(min(t, 1000000000LL), -1000000000LL));
    return r;
}

template <typename C>
__device__ __forceinline__ SV<C> sc_mul(SV<C> a, SV<C> b) {
    return sc_norm<C>(a.m * b.m, static_cast<long long>(a.e) + b.e);
}

template <typename C>
__device__ __forceinline__ SV<C> sc_div(SV<C> a, SV<C> b) {
    return sc_norm<C>(a.m / b.m, static_cast<long long>(a.e) - b.e);
}

// aligned to the larger exponent of the nonzero operands (the reference takes the other operand's
// exponent where one mantissa is zero)
template <typename C>
__device__ __forceinline__ SV<C> sc_add(SV<C> a, SV<C> b) {
    int E = max(a.e, b.e);
    if (a.m == C(0)) E = b.e;
    if (b.m == C(0)) E = a.e;
    const C x = sc_ldexp(a.m, max(a.e - E, -100000));
    const C y = sc_ldexp(b.m, max(b.e - E, -100000));
    return sc_norm<C>(x + y, E);
}

template <typename C>
__device__ __forceinline__ SV<C> sc_neg(SV<C> a) {
    a.m = -a.m;
    return a;
}

// value of m 2^e, exact until the final overflow or underflow
template <typename C>
__device__ __forceinline__ C sc_value(C m, long long e) {
    return sc_ldexp(m, static_cast<int>(max(min(e, 100000LL), -100000LL)));
}

struct ScaledMapParams {
    int op, np, ndim, contig, a_np, b_np;
    int64_t numel;
    int64_t shape[6], so[6], sa[6], sb[6];
    double p0, p1;
    void* om[PK_MAX_PLANES];
    int* oe[PK_MAX_PLANES];
    const void* am[PK_MAX_PLANES];
    const int* ae[PK_MAX_PLANES];
    const void* bm[PK_MAX_PLANES];
    const int* be[PK_MAX_PLANES];
};

template <typename C, int NP>
__global__ void __launch_bounds__(256) scaled_map_kernel(const ScaledMapParams p) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < p.numel; idx += stride) {
        int64_t oo = idx, oa = idx, ob = idx;
        if (!p.contig) {
            oo = oa = ob = 0;
            int64_t rem = idx;
            for (int d = p.ndim - 1; d >= 0; --d) {
                const int64_t c = rem % p.shape[d];
                rem /= p.shape[d];
                oo += c * p.so[d];
                oa += c * p.sa[d];
                ob += c * p.sb[d];
            }
        }
        SV<C> a[NP], b[NP], y[NP];
#pragma unroll
        for (int k = 0; k < NP; ++k) {
            a[k] = (k < p.a_np && k < p.np) ? SV<C>{static_cast<const C*>(p.am[k])[oa], p.ae[k][oa]} : SV<C>{C(0), 0};
            b[k] = (p.bm[0] != nullptr && k < p.b_np && k < p.np) ? SV<C>{static_cast<const C*>(p.bm[k])[ob], p.be[k][ob]}
                                                                 : SV<C>{C(0), 0};
        }
        switch (p.op) {
            case PK_OP_ADD: {  // a + p0 * b
                const SV<C> s = sc_norm<C>(C(p.p0), 0);
#pragma unroll
                for (int k = 0; k < NP; ++k) y[k] = sc_add<C>(a[k], sc_mul<C>(b[k], s));
                break;
            }
            case PK_OP_AFFINE: {  // p0 * a + p1
                const SV<C> s = sc_norm<C>(C(p.p0), 0);
#pragma unroll
                for (int k = 0; k < NP; ++k) y[k] = sc_mul<C>(a[k], s);
                y[0] = sc_add<C>(y[0], sc_norm<C>(C(p.p1), 0));
                break;
            }
            case PK_OP_MUL:  // C_k = ((0 + a_0 b_k) + a_1 b_{k-1}) + ...
#pragma unroll
                for (int k = 0; k < NP; ++k) {
                    SV<C> acc{C(0), 0};
#pragma unroll
                    for (int i = 0; i <= k; ++i) acc = sc_add<C>(acc, sc_mul<C>(a[i], b[k - i]));
                    y[k] = acc;
                }
                break;
            case PK_OP_DIV:  // q_k = (a_k - sum_{i=1..k} b_i q_{k-i}) / b_0
#pragma unroll
                for (int k = 0; k < NP; ++k) {
                    SV<C> r = a[k];
#pragma unroll
                    for (int i = 1; i <= k; ++i) r = sc_add<C>(r, sc_neg<C>(sc_mul<C>(b[i], y[k - i])));
                    y[k] = sc_div<C>(r, b[0]);
                }
                break;
            case PK_OP_EXP: {
                // y_0 = exp(x_0) from its logarithm: 2^floor(x_0 / ln 2) times exp of the remainder,
                // in double, so exp(x_0) beyond the dtype's range stays finite (the reference's
                // ScaledTensor.from_log, src/polytensors/_scaled.py:226-250); then
                // y_k = (x_1 / k) y_{k-1} + sum_{i=2..k} (x_i (i/k)) y_{k-i} in scaled arithmetic
                // (src/polytensors/_series.py:31-42)
                const double v = static_cast<double>(sc_value<C>(a[0].m, a[0].e));
                if (isfinite(v)) {
                    const double ln2 = 0.69314718055994530942;
                    const double E = floor(v / ln2);
                    const double E_c = fmax(fmin(E, 1.0e9), -1.0e9);
                    const double r = v - E_c * ln2;
                    y[0] = sc_norm<C>(static_cast<C>(exp(r)), static_cast<long long>(E_c));
                } else {
                    y[0] = sc_norm<C>(static_cast<C>(exp(v)), 0);
                }
#pragma unroll
                for (int k = 1; k < NP; ++k) {
                    SV<C> acc = sc_mul<C>(sc_div<C>(a[1], sc_norm<C>(C(k), 0)), y[k - 1]);
#pragma unroll
                    for (int i = 2; i <= k; ++i)
                        acc = sc_add<C>(acc, sc_mul<C>(sc_mul<C>(a[i], sc_norm<C>(C(i) / C(k), 0)), y[k - i]));
                    y[k] = acc;
                }
                break;
            }
            default:  // copy
#pragma unroll
                for (int k = 0; k < NP; ++k) y[k] = a[k];
        }
#pragma unroll
        for (int k = 0; k < NP; ++k) {
            if (k >= p.np) continue;
            static_cast<C*>(p.om[k])[oo] = y[k].m;
            p.oe[k][oo] = y[k].e;
        }
    }
}

template <typename C>
static void launch_scaled_map(const ScaledMapParams& p, int grid, cudaStream_t s) {
    switch (p.np) {
        case 1: PK_LAUNCHED(scaled_map_kernel<C, 1><<<grid, 256, 0, s>>>(p)); break;
        case 2: PK_LAUNCHED(scaled_map_kernel<C, 2><<<grid, 256, 0, s>>>(p)); break;
        case 3: PK_LAUNCHED(scaled_map_kernel<C, 3><<<grid, 256, 0, s>>>(p)); break;
        case 4: PK_LAUNCHED(scaled_map_kernel<C, 4><<<grid, 256, 0, s>>>(p)); break;
        case 5: case 6: PK_LAUNCHED(scaled_map_kernel<C, 6><<<grid, 256, 0, s>>>(p)); break;
        case 7: case 8: case 9: PK_LAUNCHED(scaled_map_kernel<C, 9><<<grid, 256, 0, s>>>(p)); break;
        default: PK_LAUNCHED(scaled_map_kernel<C, 16><<<grid, 256, 0, s>>>(p)); break;
    }
}

// Conversions over contiguous planes: from values (T) to (m, e + base), and from (m, e - base) to T;
// blockIdx.y selects the plane.
struct ScaledPlanesParams {
    int np;
    int64_t numel;
    int base;
    const void* x[PK_MAX_PLANES];  // values (from) or mantissas (to)
    const int* xe[PK_MAX_PLANES];  // exponents (to)
    void* y[PK_MAX_PLANES];        // mantissas (from) or values (to)
    int* ye[PK_MAX_PLANES];        // exponents (from)
};

template <typename T, typename C>
__global__ void __launch_bounds__(256) scaled_from_kernel(const ScaledPlanesParams p) {
    const int k = blockIdx.y;
    if (k >= p.np) return;
    const T* x = static_cast<const T*>(p.x[k]);
    C* m = static_cast<C*>(p.y[k]);
    int* e = p.ye[k];
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < p.numel; i += stride) {
        const SV<C> v = sc_norm<C>(to_c<C>(x[i]), p.base);
        m[i] = v.m;
        e[i] = v.e;
    }
}

template <typename T, typename C>
__global__ void __launch_bounds__(256) scaled_to_kernel(const ScaledPlanesParams p) {
    const int k = blockIdx.y;
    if (k >= p.np) return;
    const C* m = static_cast<const C*>(p.x[k]);
    const int* e = p.xe[k];
    T* out = static_cast<T*>(p.y[k]);
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < p.numel; i += stride)
        out[i] = from_c<T>(sc_value<C>(m[i], static_cast<long long>(e[i]) - p.base));
}

// out[o, i] = sum_r x[o, r, i]: aligned to the largest exponent of the nonzero terms of each sum
struct ScaledReduceParams {
    int np;
    int64_t outer, red, inner;
    const void* m[PK_MAX_PLANES];
    const int* e[PK_MAX_PLANES];
    void* om[PK_MAX_PLANES];
    int* oe[PK_MAX_PLANES];
};

template <typename C>
__global__ void __launch_bounds__(256) scaled_reduce_kernel(const ScaledReduceParams p) {
    const int k = blockIdx.y;
    if (k >= p.np) return;
    const int64_t total = p.outer * p.inner;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total; t += stride) {
        const int64_t o = t / p.inner, i = t % p.inner;
        const C* mp = static_cast<const C*>(p.m[k]) + o * p.red * p.inner + i;
        const int* ep = p.e[k] + o * p.red * p.inner + i;
        int E = INT_MIN;
        for (int64_t r = 0; r < p.red; ++r)
            if (mp[r * p.inner] != C(0)) E = max(E, ep[r * p.inner]);
        if (E == INT_MIN) E = 0;
        C s = C(0);
        for (int64_t r = 0; r < p.red; ++r) s += sc_ldexp(mp[r * p.inner], max(ep[r * p.inner] - E, -100000));
        const SV<C> v = sc_norm<C>(s, E);
        static_cast<C*>(p.om[k])[t] = v.m;
        p.oe[k][t] = v.e;
    }
}

static int scaled_grid(int64_t work) {
    return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(ceil_div(work, 256), 65535)));
}

static int scaled_planes(ScaledPlanesParams& p, const char* what, int degree, int64_t numel, const void* const* x,
                         const int32_t* const* xe, void* const* y, int32_t* const* ye, int base) {
    if (degree < 0 || degree >= PK_MAX_PLANES || numel < 0 || !x || !y)
        return fail(PK_ERR_ARG, std::string(what) + ": bad arguments");
    p.np = degree + 1;
    p.numel = numel;
    p.base = base;
    for (int k = 0; k < p.np; ++k) {
        if (!x[k] || !y[k] || (xe && !xe[k]) || (ye && !ye[k])) return fail(PK_ERR_ARG, std::string(what) + ": null plane");
        p.x[k] = x[k];
        p.y[k] = y[k];
        p.xe[k] = xe ? xe[k] : nullptr;
        p.ye[k] = ye ? ye[k] : nullptr;
    }
    return PK_OK;
}

}  // namespace pk

using namespace pk;

extern "C" {

int pk_scaled_from(int dtype, int degree, int64_t numel, const void* const* x, void* const* m, int32_t* const* e,
                   int32_t base_exponent, void* stream) {
    if (!e) return fail(PK_ERR_ARG, "pk_scaled_from: null exponent planes");
    ScaledPlanesParams p{};
    if (int rc = scaled_planes(p, "pk_scaled_from", degree, numel, x, nullptr, m, e, base_exponent)) return rc;
    if (numel == 0) return PK_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const dim3 grid(scaled_grid(numel), p.np);
    switch (dtype) {
        case PK_F32: PK_LAUNCHED(scaled_from_kernel<float, float><<<grid, 256, 0, s>>>(p)); break;
        case PK_F64: PK_LAUNCHED(scaled_from_kernel<double, double><<<grid, 256, 0, s>>>(p)); break;
        case PK_BF16: PK_LAUNCHED(scaled_from_kernel<__nv_bfloat16, float><<<grid, 256, 0, s>>>(p)); break;
        case PK_F16: PK_LAUNCHED(scaled_from_kernel<__half, float><<<grid, 256, 0, s>>>(p)); break;
        default: return fail(PK_ERR_UNSUPPORTED, "pk_scaled_from: unsupported dtype");
    }
    PK_CHECK_LAUNCH("pk_scaled_from");
    return PK_OK;
}

int pk_scaled_to(int dtype, int mantissa_dtype, int degree, int64_t numel, const void* const* m,
                 const int32_t* const* e, int32_t exponent_offset, void* const* out, void* stream) {
    if (!e) return fail(PK_ERR_ARG, "pk_scaled_to: null exponent planes");
    ScaledPlanesParams p{};
    if (int rc = scaled_planes(p, "pk_scaled_to", degree, numel, m, e, out, nullptr, exponent_offset)) return rc;
    if (numel == 0) return PK_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const dim3 grid(scaled_grid(numel), p.np);
    if (mantissa_dtype == PK_F64) {
        if (dtype != PK_F64) return fail(PK_ERR_UNSUPPORTED, "pk_scaled_to: float64 mantissas convert to float64");
        PK_LAUNCHED(scaled_to_kernel<double, double><<<grid, 256, 0, s>>>(p));
    } else if (mantissa_dtype == PK_F32) {
        switch (dtype) {
            case PK_F32: PK_LAUNCHED(scaled_to_kernel<float, float><<<grid, 256, 0, s>>>(p)); break;
            case PK_BF16: PK_LAUNCHED(scaled_to_kernel<__nv_bfloat16, float><<<grid, 256, 0, s>>>(p)); break;
            case PK_F16: PK_LAUNCHED(scaled_to_kernel<__half, float><<<grid, 256, 0, s>>>(p)); break;
            default: return fail(PK_ERR_UNSUPPORTED, "pk_scaled_to: unsupported dtype");
        }
    } else {
        return fail(PK_ERR_UNSUPPORTED, "pk_scaled_to: mantissas are float32 or float64");
    }
    PK_CHECK_LAUNCH("pk_scaled_to");
    return PK_OK;
}

int pk_scaled_series_map(int op, int mantissa_dtype, int degree, int ndim, const int64_t* shape,
                         void* const* out_m, int32_t* const* out_e, const int64_t* out_strides,
                         const void* const* a_m, const int32_t* const* a_e, int a_planes, const int64_t* a_strides,
                         const void* const* b_m, const int32_t* const* b_e, int b_planes, const int64_t* b_strides,
                         double p0, double p1, void* stream) {
    if (degree < 0 || degree >= PK_MAX_PLANES) return fail(PK_ERR_UNSUPPORTED, "pk_scaled_series_map: degree out of range");
    if (ndim < 0 || ndim > 6) return fail(PK_ERR_UNSUPPORTED, "pk_scaled_series_map: more than 6 dimensions");
    if (op != PK_OP_COPY && op != PK_OP_AFFINE && op != PK_OP_ADD && op != PK_OP_MUL && op != PK_OP_DIV &&
        op != PK_OP_EXP)
        return fail(PK_ERR_UNSUPPORTED, "pk_scaled_series_map: copy, affine, add, mul, div and exp only");
    const bool binary = op == PK_OP_ADD || op == PK_OP_MUL || op == PK_OP_DIV;
    const int np = degree + 1;
    if (!out_m || !out_e || !a_m || !a_e || (binary && (!b_m || !b_e)))
        return fail(PK_ERR_ARG, "pk_scaled_series_map: null plane array");
    if (a_planes != 1 && a_planes != np) return fail(PK_ERR_ARG, "pk_scaled_series_map: a_planes must be 1 or degree+1");
    if (binary && b_planes != 1 && b_planes != np)
        return fail(PK_ERR_ARG, "pk_scaled_series_map: b_planes must be 1 or degree+1");
    ScaledMapParams p{};
    p.op = op;
    p.np = np;
    p.ndim = ndim;
    p.a_np = a_planes;
    p.b_np = binary ? b_planes : 0;
    p.p0 = p0;
    p.p1 = p1;
    p.numel = 1;
    bool dense = true;
    int64_t expect = 1;
    for (int d = ndim - 1; d >= 0; --d) {
        if (shape[d] < 0) return fail(PK_ERR_ARG, "pk_scaled_series_map: negative extent");
        p.numel *= shape[d];
        p.shape[d] = shape[d];
        p.so[d] = out_strides[d];
        p.sa[d] = a_strides[d];
        p.sb[d] = binary ? b_strides[d] : 0;
        if (shape[d] != 1) {
            dense = dense && p.so[d] == expect && p.sa[d] == expect && (!binary || p.sb[d] == expect);
            expect *= shape[d];
        }
    }
    p.contig = dense ? 1 : 0;
    if (p.numel == 0) return PK_OK;
    for (int k = 0; k < np; ++k) {
        if (!out_m[k] || !out_e[k]) return fail(PK_ERR_ARG, "pk_scaled_series_map: null output plane");
        p.om[k] = out_m[k];
        p.oe[k] = out_e[k];
    }
    for (int k = 0; k < a_planes; ++k) {
        if (!a_m[k] || !a_e[k]) return fail(PK_ERR_ARG, "pk_scaled_series_map: null input plane");
        p.am[k] = a_m[k];
        p.ae[k] = a_e[k];
    }
    if (binary)
        for (int k = 0; k < b_planes; ++k) {
            if (!b_m[k] || !b_e[k]) return fail(PK_ERR_ARG, "pk_scaled_series_map: null input plane");
            p.bm[k] = b_m[k];
            p.be[k] = b_e[k];
        }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int grid = scaled_grid(p.numel);
    void* tok;
    prof_begin("scaled_map", s, &tok);
    if (mantissa_dtype == PK_F64) launch_scaled_map<double>(p, grid, s);
    else if (mantissa_dtype == PK_F32) launch_scaled_map<float>(p, grid, s);
    else return fail(PK_ERR_UNSUPPORTED, "pk_scaled_series_map: mantissas are float32 or float64");
    prof_end("scaled_map", s, tok);
    PK_CHECK_LAUNCH("pk_scaled_series_map");
    return PK_OK;
}

int pk_scaled_reduce(int mantissa_dtype, int degree, int64_t outer, int64_t red, int64_t inner, const void* const* m,
                     const int32_t* const* e, void* const* out_m, int32_t* const* out_e, void* stream) {
    if (degree < 0 || degree >= PK_MAX_PLANES || outer < 0 || red < 0 || inner < 0 || !m || !e || !out_m || !out_e)
        return fail(PK_ERR_ARG, "pk_scaled_reduce: bad arguments");
    ScaledReduceParams p{};
    p.np = degree + 1;
    p.outer = outer;
    p.red = red;
    p.inner = inner;
    for (int k = 0; k < p.np; ++k) {
        if (!m[k] || !e[k] || !out_m[k] || !out_e[k]) return fail(PK_ERR_ARG, "pk_scaled_reduce: null plane");
        p.m[k] = m[k];
        p.e[k] = e[k];
        p.om[k] = out_m[k];
        p.oe[k] = out_e[k];
    }
    if (outer * inner == 0) return PK_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const dim3 grid(scaled_grid(outer * inner), p.np);
    if (mantissa_dtype == PK_F64) PK_LAUNCHED(scaled_reduce_kernel<double><<<grid, 256, 0, s>>>(p));
    else if (mantissa_dtype == PK_F32) PK_LAUNCHED(scaled_reduce_kernel<float><<<grid, 256, 0, s>>>(p));
    else return fail(PK_ERR_UNSUPPORTED, "pk_scaled_reduce: mantissas are float32 or float64");
    PK_CHECK_LAUNCH("pk_scaled_reduce");
    return PK_OK;
}

}  // extern "C"
