// Truncated power-series arithmetic on register arrays.
//
// A series of NP coefficients s[0..NP-1] stands for sum_k s[k] t^k, truncated after
// t^(NP-1).  All loops have compile-time bounds so the arrays stay in registers.
// Recurrences follow the power-series ODEs of each function (y' = f'(x) x'), which give
// the same coefficients as the reference's rules (src/polytensors/_plain.py,
// src/polytensors/_series.py) up to rounding.
#pragma once

#include "pk_common.cuh"

namespace pk {

// 1/k for the series recurrences (k is a compile-time constant after unrolling).
template <typename C>
__device__ __forceinline__ constexpr C inv_int(int k) {
    return C(1.0 / static_cast<double>(k));
}

// Storage <-> compute conversions.  bf16 / f16 planes are computed in float.
template <typename T> struct Compute { using type = T; };
template <> struct Compute<__nv_bfloat16> { using type = float; };
template <> struct Compute<__half> { using type = float; };

template <typename C, typename T> __device__ __forceinline__ C to_c(T v) { return static_cast<C>(v); }
template <> __device__ __forceinline__ float to_c<float, __nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> __device__ __forceinline__ float to_c<float, __half>(__half v) { return __half2float(v); }
template <typename T, typename C> __device__ __forceinline__ T from_c(C v) { return static_cast<T>(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_c<__nv_bfloat16, float>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ __half from_c<__half, float>(float v) { return __float2half_rn(v); }

// exp/log/erf/... in the compute precision
__device__ __forceinline__ float c_exp(float x) { return expf(x); }
__device__ __forceinline__ double c_exp(double x) { return exp(x); }
__device__ __forceinline__ float c_log(float x) { return logf(x); }
__device__ __forceinline__ double c_log(double x) { return log(x); }
__device__ __forceinline__ float c_sqrt(float x) { return sqrtf(x); }
__device__ __forceinline__ double c_sqrt(double x) { return sqrt(x); }
__device__ __forceinline__ float c_rsqrt(float x) { return rsqrtf(x); }
__device__ __forceinline__ double c_rsqrt(double x) { return rsqrt(x); }
__device__ __forceinline__ float c_tanh(float x) { return tanhf(x); }
__device__ __forceinline__ double c_tanh(double x) { return tanh(x); }
__device__ __forceinline__ float c_erf(float x) { return erff(x); }
__device__ __forceinline__ double c_erf(double x) { return erf(x); }

// out = a (*) b, truncated
template <int NP, typename C>
__device__ __forceinline__ void s_mul(const C (&a)[NP], const C (&b)[NP], C (&out)[NP]) {
    C r[NP];
#pragma unroll
    for (int k = 0; k < NP; ++k) {
        C acc = a[0] * b[k];
#pragma unroll
        for (int i = 1; i <= k; ++i) acc += a[i] * b[k - i];
        r[k] = acc;
    }
#pragma unroll
    for (int k = 0; k < NP; ++k) out[k] = r[k];
}

// acc += a (*) b (one multiply-add per term; acc must not alias a or b)
template <int NP, typename C>
__device__ __forceinline__ void s_mul_acc(const C (&a)[NP], const C (&b)[NP], C (&acc)[NP]) {
#pragma unroll
    for (int k = 0; k < NP; ++k) {
#pragma unroll
        for (int i = 0; i <= k; ++i) acc[k] += a[i] * b[k - i];
    }
}

// out = base - a (*) b
template <int NP, typename C>
__device__ __forceinline__ void s_sub_mul(const C (&base)[NP], const C (&a)[NP], const C (&b)[NP], C (&out)[NP]) {
    C r[NP];
#pragma unroll
    for (int k = 0; k < NP; ++k) {
        C acc = base[k];
#pragma unroll
        for (int i = 0; i <= k; ++i) acc -= a[i] * b[k - i];
        r[k] = acc;
    }
#pragma unroll
    for (int k = 0; k < NP; ++k) out[k] = r[k];
}

// Sum of squares accumulated in two halves: cross += sum over i < k - i of x_i x_{k-i}, diag +=
// x_{k/2}^2 for even k, so that x (*) x = 2 cross + diag takes about half the multiply-adds of a
// general product (the factor 2 is applied once, after the accumulation).
template <int NP, typename C>
__device__ __forceinline__ void s_square_acc(const C (&x)[NP], C (&cross)[NP], C (&diag)[NP]) {
#pragma unroll
    for (int k = 0; k < NP; ++k) {
#pragma unroll
        for (int i = 0; 2 * i < k; ++i) cross[k] += x[i] * x[k - i];
        if (k % 2 == 0) diag[k] += x[k / 2] * x[k / 2];
    }
}

// out = a / b (quotient recurrence, src/polytensors/_range_ops.py:86-93)
template <int NP, typename C>
__device__ __forceinline__ void s_div(const C (&a)[NP], const C (&b)[NP], C (&out)[NP]) {
    C q[NP];
    const C inv = C(1) / b[0];
#pragma unroll
    for (int k = 0; k < NP; ++k) {
        C r = a[k];
#pragma unroll
        for (int i = 1; i <= k; ++i) r -= b[i] * q[k - i];
        q[k] = r * inv;
    }
#pragma unroll
    for (int k = 0; k < NP; ++k) out[k] = q[k];
}

// y = exp(x): y_0 = exp(x_0), k y_k = sum_{i=1..k} i x_i y_{k-i}
template <int NP, typename C>
__device__ __forceinline__ void s_exp(const C (&x)[NP], C (&y)[NP]) {
    C r[NP];
    r[0] = c_exp(x[0]);
#pragma unroll
    for (int k = 1; k < NP; ++k) {
        C acc = C(0);
#pragma unroll
        for (int i = 1; i <= k; ++i) acc += C(i) * x[i] * r[k - i];
        r[k] = acc * inv_int<C>(k);
    }
#pragma unroll
    for (int k = 0; k < NP; ++k) y[k] = r[k];
}

// exp of the directions only: e = exp(x - x_0) (e_0 = 1)
template <int NP, typename C>
__device__ __forceinline__ void s_exp_dir(const C (&x)[NP], C (&e)[NP]) {
    e[0] = C(1);
#pragma unroll
    for (int k = 1; k < NP; ++k) {
        C acc = C(0);
#pragma unroll
        for (int i = 1; i <= k; ++i) acc += C(i) * x[i] * e[k - i];
        e[k] = acc * inv_int<C>(k);
    }
}

// log of a series whose constant term is 1 (directions normalised), y_0 = 0:
// y_k = u_k - sum_{i=1..k-1} (i/k) y_i u_{k-i}   (src/polytensors/_plain.py:162-171)
template <int NP, typename C>
__device__ __forceinline__ void s_log1(const C (&u)[NP], C (&y)[NP]) {
    y[0] = C(0);
#pragma unroll
    for (int k = 1; k < NP; ++k) {
        C acc = u[k] * C(k);
#pragma unroll
        for (int i = 1; i < k; ++i) acc -= C(i) * y[i] * u[k - i];
        y[k] = acc * inv_int<C>(k);
    }
}

template <int NP, typename C>
__device__ __forceinline__ void s_log(const C (&x)[NP], C (&y)[NP]) {
    C u[NP];
    const C inv = C(1) / x[0];
    u[0] = C(1);
#pragma unroll
    for (int k = 1; k < NP; ++k) u[k] = x[k] * inv;
    C r[NP];
    s_log1<NP, C>(u, r);
    r[0] = c_log(x[0]);
#pragma unroll
    for (int k = 0; k < NP; ++k) y[k] = r[k];
}

// y = x^(-1/2) from 2 x y' + x' y = 0 with normalised directions
// (src/polytensors/_series.py:83-96):  y_k = -sum_{i=1..k} ((2k-i)/(2k)) u_i y_{k-i}
template <int NP, typename C>
__device__ __forceinline__ void s_rsqrt(const C (&x)[NP], C (&y)[NP]) {
    C u[NP], r[NP];
    const C inv = C(1) / x[0];
#pragma unroll
    for (int k = 1; k < NP; ++k) u[k] = x[k] * inv;
    r[0] = c_rsqrt(x[0]);
#pragma unroll
    for (int k = 1; k < NP; ++k) {
        C acc = C(0);
#pragma unroll
        for (int i = 1; i <= k; ++i) acc += C(2 * k - i) * u[i] * r[k - i];
        r[k] = -acc * inv_int<C>(2 * k);
    }
#pragma unroll
    for (int k = 0; k < NP; ++k) y[k] = r[k];
}

// y = sqrt(x): y_k = (x_k - sum_{i=1..k-1} y_i y_{k-i}) / (2 y_0)   (src/polytensors/_series.py:72-81)
template <int NP, typename C>
__device__ __forceinline__ void s_sqrt(const C (&x)[NP], C (&y)[NP]) {
    C r[NP];
    r[0] = c_sqrt(x[0]);
    const C inv2 = C(1) / (C(2) * r[0]);
#pragma unroll
    for (int k = 1; k < NP; ++k) {
        C acc = x[k];
#pragma unroll
        for (int i = 1; i < k; ++i) acc -= r[i] * r[k - i];
        r[k] = acc * inv2;
    }
#pragma unroll
    for (int k = 0; k < NP; ++k) y[k] = r[k];
}

// Series of a function y = f(x) with y' = g x' where g = G(y) is computed alongside:
// k y_k = sum_{i=1..k} i x_i g_{k-i}.
// tanh: g = 1 - y^2; sigmoid: g = y (1 - y).  dydx (optional) receives the g series.
template <int NP, typename C>
__device__ __forceinline__ void s_tanh(const C (&x)[NP], C (&y)[NP], C (&g)[NP]) {
    C r[NP], gg[NP];
    r[0] = c_tanh(x[0]);
    gg[0] = C(1) - r[0] * r[0];
#pragma unroll
    for (int k = 1; k < NP; ++k) {
        C acc = C(0);
#pragma unroll
        for (int i = 1; i <= k; ++i) acc += C(i) * x[i] * gg[k - i];
        r[k] = acc * inv_int<C>(k);
        C sq = C(0);
#pragma unroll
        for (int i = 0; i <= k; ++i) sq += r[i] * r[k - i];
        gg[k] = -sq;
    }
#pragma unroll
    for (int k = 0; k < NP; ++k) {
        y[k] = r[k];
        g[k] = gg[k];
    }
}

template <int NP, typename C>
__device__ __forceinline__ void s_sigmoid(const C (&x)[NP], C (&y)[NP], C (&g)[NP]) {
    C r[NP], gg[NP];
    r[0] = C(1) / (C(1) + c_exp(-x[0]));
    gg[0] = r[0] * (C(1) - r[0]);
#pragma unroll
    for (int k = 1; k < NP; ++k) {
        C acc = C(0);
#pragma unroll
        for (int i = 1; i <= k; ++i) acc += C(i) * x[i] * gg[k - i];
        r[k] = acc * inv_int<C>(k);
        C p = r[k] * (C(1) - r[0]);
#pragma unroll
        for (int i = 0; i < k; ++i) p -= r[i] * r[k - i];
        gg[k] = p;
    }
#pragma unroll
    for (int k = 0; k < NP; ++k) {
        y[k] = r[k];
        g[k] = gg[k];
    }
}

// Exact GELU, f(x) = x Phi(x), from the coupled series of Phi(x) and phi(x):
// Phi' = phi x',  phi' = -x phi x'.  Returns y = f(x) and d = f'(x) = Phi(x) + x phi(x).
template <int NP, typename C>
__device__ __forceinline__ void s_gelu(const C (&x)[NP], C (&y)[NP], C (&d)[NP]) {
    C Phi[NP], phi[NP], w[NP];  // w = x * phi (series)
    const C inv_sqrt2 = C(0.70710678118654752440);
    const C inv_sqrt2pi = C(0.39894228040143267794);
    Phi[0] = C(0.5) * (C(1) + c_erf(x[0] * inv_sqrt2));
    phi[0] = c_exp(C(-0.5) * x[0] * x[0]) * inv_sqrt2pi;
    w[0] = x[0] * phi[0];
#pragma unroll
    for (int k = 1; k < NP; ++k) {
        C a = C(0), b = C(0);
#pragma unroll
        for (int i = 1; i <= k; ++i) {
            a += C(i) * x[i] * phi[k - i];
            b += C(i) * x[i] * w[k - i];
        }
        Phi[k] = a * inv_int<C>(k);
        phi[k] = -b * inv_int<C>(k);
        C ww = C(0);
#pragma unroll
        for (int i = 0; i <= k; ++i) ww += x[i] * phi[k - i];
        w[k] = ww;
    }
    C r[NP];
    s_mul<NP, C>(x, Phi, r);
#pragma unroll
    for (int k = 0; k < NP; ++k) {
        y[k] = r[k];
        d[k] = Phi[k] + w[k];
    }
}

}  // namespace pk
