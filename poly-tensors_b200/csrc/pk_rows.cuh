// Block-level helpers for row-wise series kernels (one CTA per row).
#pragma once

#include "pk_series.cuh"

namespace pk {

// Sum NP values across the block; every thread receives the totals.
// `scratch` must hold (blockDim.x / 32) * NP values of A.
template <int NP, typename A>
__device__ __forceinline__ void block_sum(A (&v)[NP], A* scratch) {
#pragma unroll
    for (int k = 0; k < NP; ++k) {
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v[k] += __shfl_xor_sync(0xffffffffu, v[k], off);
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) {
#pragma unroll
        for (int k = 0; k < NP; ++k) scratch[warp * NP + k] = v[k];
    }
    __syncthreads();
    // every warp reduces the per-warp partials itself: with P = nw rounded up to a power of two,
    // lane j holds warp (j mod P)'s partial (zero past nw) and a butterfly over offsets < P gives
    // every lane the total; all warps run the same butterfly, so all threads agree bit for bit
    int pw = 1;
    while (pw < nw) pw <<= 1;
    const int src = lane & (pw - 1);
#pragma unroll
    for (int k = 0; k < NP; ++k) v[k] = src < nw ? scratch[src * NP + k] : A(0);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        if (off < pw) {
#pragma unroll
            for (int k = 0; k < NP; ++k) v[k] += __shfl_xor_sync(0xffffffffu, v[k], off);
        }
    }
}

// Combine (m, S[]) pairs where S is scaled by exp(-m): the online log-sum-exp state of a
// softmax series.  Every thread receives the combined state.
template <int NP, typename A>
__device__ __forceinline__ void block_lse_combine(A& m, A (&S)[NP], A* scratch) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const A mo = __shfl_xor_sync(0xffffffffu, m, off);
        A So[NP];
#pragma unroll
        for (int k = 0; k < NP; ++k) So[k] = __shfl_xor_sync(0xffffffffu, S[k], off);
        const A mn = fmax(m, mo);
        const A fa = (m == -INFINITY) ? A(0) : c_exp(m - mn);
        const A fb = (mo == -INFINITY) ? A(0) : c_exp(mo - mn);
#pragma unroll
        for (int k = 0; k < NP; ++k) S[k] = S[k] * fa + So[k] * fb;
        m = mn;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) {
        scratch[warp * (NP + 1)] = m;
#pragma unroll
        for (int k = 0; k < NP; ++k) scratch[warp * (NP + 1) + 1 + k] = S[k];
    }
    __syncthreads();
    A mm = -INFINITY;
    for (int w = 0; w < nw; ++w) mm = fmax(mm, scratch[w * (NP + 1)]);
    A tot[NP];
#pragma unroll
    for (int k = 0; k < NP; ++k) tot[k] = A(0);
    for (int w = 0; w < nw; ++w) {
        const A mw = scratch[w * (NP + 1)];
        const A f = (mw == -INFINITY) ? A(0) : c_exp(mw - mm);
#pragma unroll
        for (int k = 0; k < NP; ++k) tot[k] += scratch[w * (NP + 1) + 1 + k] * f;
    }
    m = mm;
#pragma unroll
    for (int k = 0; k < NP; ++k) S[k] = tot[k];
}

// Fold one element's series x (compute precision) into a thread's online state:
// S_k += exp(x_0 - m) e_k(x), e = exp of the directions.
template <int NP, typename A>
__device__ __forceinline__ void lse_accumulate(A& m, A (&S)[NP], const A (&x)[NP]) {
    if (x[0] == -INFINITY) return;  // masked entries contribute nothing
    if (x[0] > m) {
        const A f = (m == -INFINITY) ? A(0) : c_exp(m - x[0]);
#pragma unroll
        for (int k = 0; k < NP; ++k) S[k] *= f;
        m = x[0];
    }
    A e[NP];
    s_exp_dir<NP, A>(x, e);
    const A w = c_exp(x[0] - m);
#pragma unroll
    for (int k = 0; k < NP; ++k) S[k] += w * e[k];
}

// From the combined state: lse_0 = m + log S_0 and the log-normaliser directions
// logz_k = [log(S / S_0)]_k, k >= 1 (logz_0 slot receives lse_0).
template <int NP, typename A>
__device__ __forceinline__ void lse_finish(A m, const A (&S)[NP], A (&lse)[NP]) {
    A u[NP];
    const A inv = A(1) / S[0];
    u[0] = A(1);
#pragma unroll
    for (int k = 1; k < NP; ++k) u[k] = S[k] * inv;
    s_log1<NP, A>(u, lse);
    lse[0] = m + c_log(S[0]);
}

}  // namespace pk

namespace pk {

// ---------------------------------------------------------------------------------
// Vectorised row access: each thread handles ROW_VEC consecutive elements of a row per
// step, loaded with one 8-32 byte access per plane when the launch marked all planes
// (and row strides) as ROW_VEC-aligned, element by element otherwise (row tails too).

constexpr int ROW_VEC = 4;

// Elements of the step starting at c0 that lie before `end` (at most ROW_VEC).
__device__ __forceinline__ int vec_count(int64_t end, int64_t c0) {
    const int64_t r = end - c0;
    return r >= ROW_VEC ? ROW_VEC : static_cast<int>(r);
}

template <typename T>
__device__ __forceinline__ void load_vec4(const T* p, float (&v)[4]);
// (generic loads: the row kernels also read their shared-memory stages through this helper)
template <>
__device__ __forceinline__ void load_vec4<float>(const float* p, float (&v)[4]) {
    const float4 t = *reinterpret_cast<const float4*>(p);
    v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
}
template <>
__device__ __forceinline__ void load_vec4<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[4]) {
    const uint2 t = *reinterpret_cast<const uint2*>(p);
    const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&t.x);
    const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&t.y);
    v[0] = __low2float(a); v[1] = __high2float(a); v[2] = __low2float(b); v[3] = __high2float(b);
}
template <>
__device__ __forceinline__ void load_vec4<__half>(const __half* p, float (&v)[4]) {
    const uint2 t = *reinterpret_cast<const uint2*>(p);
    const __half2 a = *reinterpret_cast<const __half2*>(&t.x);
    const __half2 b = *reinterpret_cast<const __half2*>(&t.y);
    v[0] = __low2float(a); v[1] = __high2float(a); v[2] = __low2float(b); v[3] = __high2float(b);
}
__device__ __forceinline__ void load_vec4d(const double* p, double (&v)[4]) {
    const double2 a = reinterpret_cast<const double2*>(p)[0];
    const double2 b = reinterpret_cast<const double2*>(p)[1];
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}

template <typename T>
__device__ __forceinline__ void store_vec4(T* p, const float (&v)[4]);
template <>
__device__ __forceinline__ void store_vec4<float>(float* p, const float (&v)[4]) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
}
template <>
__device__ __forceinline__ void store_vec4<__nv_bfloat16>(__nv_bfloat16* p, const float (&v)[4]) {
    __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]), b = __floats2bfloat162_rn(v[2], v[3]);
    uint2 t;
    t.x = *reinterpret_cast<uint32_t*>(&a);
    t.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(p) = t;
}
template <>
__device__ __forceinline__ void store_vec4<__half>(__half* p, const float (&v)[4]) {
    __half2 a = __floats2half2_rn(v[0], v[1]), b = __floats2half2_rn(v[2], v[3]);
    uint2 t;
    t.x = *reinterpret_cast<uint32_t*>(&a);
    t.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(p) = t;
}
__device__ __forceinline__ void store_vec4d(double* p, const double (&v)[4]) {
    reinterpret_cast<double2*>(p)[0] = make_double2(v[0], v[1]);
    reinterpret_cast<double2*>(p)[1] = make_double2(v[2], v[3]);
}

// x[u][k] = plane k, element off + u (u < valid; zero beyond)
template <int NP, typename T, typename C>
__device__ __forceinline__ void load_planes4(const void* const* planes, int np, int64_t off, int valid, bool vec,
                                             C (&x)[ROW_VEC][NP]) {
#pragma unroll
    for (int k = 0; k < NP; ++k) {
        const T* src = static_cast<const T*>(planes[k]) + off;
        C v[4] = {C(0), C(0), C(0), C(0)};
        if (k < np) {
            if (vec && valid == ROW_VEC) {
                if constexpr (sizeof(C) == 8) load_vec4d(reinterpret_cast<const double*>(src), v);
                else load_vec4<T>(src, v);
            } else {
#pragma unroll
                for (int u = 0; u < ROW_VEC; ++u)
                    if (u < valid) v[u] = to_c<C>(src[u]);
            }
        }
#pragma unroll
        for (int u = 0; u < ROW_VEC; ++u) x[u][k] = v[u];
    }
}

template <int NP, typename T, typename C>
__device__ __forceinline__ void store_planes4(void* const* planes, int np, int64_t off, int valid, bool vec,
                                              const C (&y)[ROW_VEC][NP]) {
#pragma unroll
    for (int k = 0; k < NP; ++k) {
        if (k >= np) continue;
        T* dst = static_cast<T*>(planes[k]) + off;
        C v[4];
#pragma unroll
        for (int u = 0; u < ROW_VEC; ++u) v[u] = y[u][k];
        if (vec && valid == ROW_VEC) {
            if constexpr (sizeof(C) == 8) store_vec4d(reinterpret_cast<double*>(dst), v);
            else store_vec4<T>(dst, v);
        } else {
#pragma unroll
            for (int u = 0; u < ROW_VEC; ++u)
                if (u < valid) dst[u] = from_c<T>(v[u]);
        }
    }
}

// float32 values written as bf16 hi/lo pairs: planes[2k] = hi_k = bf16(y_k), planes[2k + 1] =
// lo_k = bf16(y_k - hi_k), so that y_k ~= hi_k + lo_k to about 2^-16 relative (the split the
// float32 tensor-core products read; the same rounding as the operand staging).
template <int NP>
__device__ __forceinline__ void store_planes4_hilo(void* const* planes, int np, int64_t off, int valid, bool vec,
                                                   const float (&y)[ROW_VEC][NP]) {
#pragma unroll
    for (int k = 0; k < NP; ++k) {
        if (k >= np) continue;
        __nv_bfloat16* hi = static_cast<__nv_bfloat16*>(planes[2 * k]) + off;
        __nv_bfloat16* lo = static_cast<__nv_bfloat16*>(planes[2 * k + 1]) + off;
        float h[4], l[4];
#pragma unroll
        for (int u = 0; u < ROW_VEC; ++u) {
            h[u] = __bfloat162float(__float2bfloat16_rn(y[u][k]));
            l[u] = y[u][k] - h[u];
        }
        if (vec && valid == ROW_VEC) {
            store_vec4<__nv_bfloat16>(hi, h);
            store_vec4<__nv_bfloat16>(lo, l);
        } else {
#pragma unroll
            for (int u = 0; u < ROW_VEC; ++u)
                if (u < valid) {
                    hi[u] = __float2bfloat16_rn(h[u]);
                    lo[u] = __float2bfloat16_rn(l[u]);
                }
        }
    }
}

// bf16 hi/lo pairs (planes[2k], planes[2k + 1]) read back as float32 hi + lo.
template <int NP>
__device__ __forceinline__ void load_planes4_hilo(const void* const* planes, int np, int64_t off, int valid, bool vec,
                                                  float (&x)[ROW_VEC][NP]) {
#pragma unroll
    for (int k = 0; k < NP; ++k) {
        float h[4] = {0.f, 0.f, 0.f, 0.f}, l[4] = {0.f, 0.f, 0.f, 0.f};
        if (k < np) {
            const __nv_bfloat16* hi = static_cast<const __nv_bfloat16*>(planes[2 * k]) + off;
            const __nv_bfloat16* lo = static_cast<const __nv_bfloat16*>(planes[2 * k + 1]) + off;
            if (vec && valid == ROW_VEC) {
                load_vec4<__nv_bfloat16>(hi, h);
                load_vec4<__nv_bfloat16>(lo, l);
            } else {
#pragma unroll
                for (int u = 0; u < ROW_VEC; ++u)
                    if (u < valid) {
                        h[u] = __bfloat162float(hi[u]);
                        l[u] = __bfloat162float(lo[u]);
                    }
            }
        }
#pragma unroll
        for (int u = 0; u < ROW_VEC; ++u) x[u][k] = h[u] + l[u];
    }
}

// Whether planes (base pointers) and a row stride allow ROW_VEC-element vector access.
inline bool row_vec_ok(const void* const* planes, int np, int64_t row_stride, int elem_bytes) {
    const uintptr_t align = static_cast<uintptr_t>(ROW_VEC) * elem_bytes;
    if (row_stride % ROW_VEC) return false;
    for (int k = 0; k < np; ++k)
        if (reinterpret_cast<uintptr_t>(planes[k]) % (align > 16 ? 16 : align)) return false;
    return true;
}

// Online log-sum-exp state update for up to four elements at once (one rescale per group).
template <int NP, typename A>
__device__ __forceinline__ void lse_accumulate4(A& m, A (&S)[NP], const A (&x)[ROW_VEC][NP], int valid) {
    A gmax = -INFINITY;
#pragma unroll
    for (int u = 0; u < ROW_VEC; ++u)
        if (u < valid) gmax = fmax(gmax, x[u][0]);
    if (gmax == -INFINITY) return;
    if (gmax > m) {
        const A f = (m == -INFINITY) ? A(0) : c_exp(m - gmax);
#pragma unroll
        for (int k = 0; k < NP; ++k) S[k] *= f;
        m = gmax;
    }
#pragma unroll
    for (int u = 0; u < ROW_VEC; ++u) {
        if (u >= valid || x[u][0] == -INFINITY) continue;
        A e[NP];
        s_exp_dir<NP, A>(x[u], e);
        const A w = c_exp(x[u][0] - m);
#pragma unroll
        for (int k = 0; k < NP; ++k) S[k] += w * e[k];
    }
}

}  // namespace pk
