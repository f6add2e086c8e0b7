// Complex compute type for series whose directions (or base) are complex.
//
// The reference lets a PolyTensor carry complex coefficient planes — typically a real base with
// complex directions (src/polytensors/_tensor.py:37-126, _plain.py:77-80) — and its plain-range
// rules are ordinary PyTorch arithmetic, so every series rule works on complex planes.  The
// series helpers of pk_series.cuh are templates over the compute type; instantiating them with
// cplx<R> gives the same recurrences in complex arithmetic.  Functions of the base: exp, log,
// sqrt and rsqrt are the principal complex functions; tanh and erf take the real part only (their
// callers, tanh and GELU, accept a real base only, which the host checks).
#pragma once

#include <type_traits>

#include "pk_series.cuh"

namespace pk {

template <typename R>
struct cplx {
    R re, im;
    __host__ __device__ constexpr cplx() : re(R(0)), im(R(0)) {}
    __host__ __device__ constexpr cplx(R r, R i) : re(r), im(i) {}
    // a real number of any arithmetic type (series code writes C(1), C(k), C(0.5), C(p0))
    template <typename S, typename = typename std::enable_if<std::is_arithmetic<S>::value>::type>
    __host__ __device__ constexpr cplx(S r) : re(static_cast<R>(r)), im(R(0)) {}
    __device__ __forceinline__ cplx& operator+=(const cplx& o) {
        re += o.re;
        im += o.im;
        return *this;
    }
    __device__ __forceinline__ cplx& operator-=(const cplx& o) {
        re -= o.re;
        im -= o.im;
        return *this;
    }
    __device__ __forceinline__ cplx& operator*=(const cplx& o) {
        const R r = re * o.re - im * o.im;
        im = re * o.im + im * o.re;
        re = r;
        return *this;
    }
};

template <typename R>
__device__ __forceinline__ cplx<R> operator+(cplx<R> a, const cplx<R>& b) { return a += b; }
template <typename R>
__device__ __forceinline__ cplx<R> operator-(cplx<R> a, const cplx<R>& b) { return a -= b; }
template <typename R>
__device__ __forceinline__ cplx<R> operator*(cplx<R> a, const cplx<R>& b) { return a *= b; }
template <typename R>
__device__ __forceinline__ cplx<R> operator-(const cplx<R>& a) { return cplx<R>(-a.re, -a.im); }
// a / b by scaling with the larger component of b (Smith's method), so |b|^2 never overflows
template <typename R>
__device__ __forceinline__ cplx<R> operator/(const cplx<R>& a, const cplx<R>& b) {
    if (b.im == R(0)) return cplx<R>(a.re / b.re, a.im / b.re);
    if (fabs(b.re) >= fabs(b.im)) {
        const R r = b.im / b.re, d = b.re + b.im * r;
        return cplx<R>((a.re + a.im * r) / d, (a.im - a.re * r) / d);
    }
    const R r = b.re / b.im, d = b.re * r + b.im;
    return cplx<R>((a.re * r + a.im) / d, (a.im * r - a.re) / d);
}

template <typename R>
__device__ __forceinline__ cplx<R> c_exp(const cplx<R>& z) {
    const R m = c_exp(z.re);
    if (z.im == R(0)) return cplx<R>(m, R(0));
    return cplx<R>(m * cos(z.im), m * sin(z.im));
}
template <typename R>
__device__ __forceinline__ cplx<R> c_log(const cplx<R>& z) {
    if (z.im == R(0) && z.re >= R(0)) return cplx<R>(c_log(z.re), R(0));
    return cplx<R>(c_log(hypot(z.re, z.im)), atan2(z.im, z.re));
}
// principal square root: (sqrt((|z| + a) / 2), sign(b) sqrt((|z| - a) / 2)) for z = a + ib
template <typename R>
__device__ __forceinline__ cplx<R> c_sqrt(const cplx<R>& z) {
    if (z.im == R(0) && z.re >= R(0)) return cplx<R>(c_sqrt(z.re), R(0));
    const R m = hypot(z.re, z.im);
    const R u = c_sqrt((m + fabs(z.re)) * R(0.5));
    if (z.re >= R(0)) return cplx<R>(u, z.im / (R(2) * u));
    return cplx<R>(fabs(z.im) / (R(2) * u), z.im >= R(0) ? u : -u);
}
template <typename R>
__device__ __forceinline__ cplx<R> c_rsqrt(const cplx<R>& z) {
    if (z.im == R(0) && z.re > R(0)) return cplx<R>(c_rsqrt(z.re), R(0));
    return cplx<R>(R(1)) / c_sqrt(z);
}
template <typename R>
__device__ __forceinline__ cplx<R> c_tanh(const cplx<R>& z) { return cplx<R>(c_tanh(z.re), R(0)); }
template <typename R>
__device__ __forceinline__ cplx<R> c_erf(const cplx<R>& z) { return cplx<R>(c_erf(z.re), R(0)); }

}  // namespace pk
