// RMSNorm of a series along the last dimension, with an optional weight series:
//   y = x (*) rsqrt(mean(x (*) x) + eps) (*) w        ((*) = truncated Cauchy product)
// Replaces the reference's decomposition (src/polytensors/_decompositions.py:14-22),
// which issues ~10 full-size launches per plane pair, and generalises its degree-1 fused
// Triton kernels (src/polytensors/_norm_kernels.py:6-38) to any degree.  One CTA owns a
// row: a first pass reduces the n+1 coefficients of mean(x (*) x), the CTA evaluates the
// rsqrt series of the row, and a second pass (an L2 hit) writes y.
//
// Backward, as series arithmetic (the reference's wrapper autograd through the same
// decomposition):  with gy = G (*) w,  d = sum_row gy (*) x,
//   dx = r (*) gy - (r (*) r (*) r (*) d / cols) (*) x,   dw = sum_rows G (*) (x (*) r).
#include <algorithm>

#include <cooperative_groups.h>

#include "pk_rows.cuh"

namespace pk {

struct NormParams {
    int np;
    int64_t rows, cols;
    int64_t x_rs, y_rs, g_rs;
    int w_np;  // 0 = no weight, 1 = constant weight, np = weight series
    double eps;
    const void* x[PK_MAX_PLANES];
    const void* w[PK_MAX_PLANES];
    const void* g[PK_MAX_PLANES];
    void* y[PK_MAX_PLANES];   // forward output / backward dx
    void* dw_part;            // backward: [gridDim.x][np][cols] partial weight gradients (compute type)
    void* rstd;               // [rows][np] rsqrt series per row (compute type)
    int vec;                  // planes and row strides allow ROW_VEC-element vector access
    int* status;              // device status word for waits that time out
};

template <int NP, typename T, typename C>
__device__ __forceinline__ void load_elem(const void* const* planes, int np, int64_t off, C (&v)[NP]) {
#pragma unroll
    for (int k = 0; k < NP; ++k) v[k] = k < np ? to_c<C>(static_cast<const T*>(planes[k])[off]) : C(0);
}

template <int NP, typename T, typename C>
__device__ __forceinline__ void load_weight(const NormParams& p, int64_t c, C (&w)[NP]) {
#pragma unroll
    for (int k = 0; k < NP; ++k) w[k] = (k < p.w_np) ? to_c<C>(static_cast<const T*>(p.w[k])[c]) : C(0);
    if (p.w_np == 0) w[0] = C(1);
}

template <int NP, typename T, typename C>
__device__ __forceinline__ void load_weight4(const NormParams& p, int64_t c0, int valid, C (&w)[ROW_VEC][NP]) {
    if (p.w_np == 0) {
#pragma unroll
        for (int u = 0; u < ROW_VEC; ++u) {
#pragma unroll
            for (int k = 0; k < NP; ++k) w[u][k] = C(k == 0 ? 1 : 0);
        }
        return;
    }
    load_planes4<NP, T, C>(p.w, p.w_np, c0, valid, p.vec != 0, w);
}

template <typename T, int NP>
__global__ void __launch_bounds__(512) rmsnorm_fwd_kernel(const NormParams p) {
    using C = typename Compute<T>::type;
    __shared__ C scratch[16 * NP];
    for (int64_t row = blockIdx.x; row < p.rows; row += gridDim.x) {
        const int64_t xb = row * p.x_rs;
        C acc[NP];
#pragma unroll
        for (int k = 0; k < NP; ++k) acc[k] = C(0);
        for (int64_t c0 = static_cast<int64_t>(threadIdx.x) * ROW_VEC; c0 < p.cols;
             c0 += static_cast<int64_t>(blockDim.x) * ROW_VEC) {
            const int valid = vec_count(p.cols, c0);
            C x[ROW_VEC][NP];
            load_planes4<NP, T, C>(p.x, p.np, xb + c0, valid, p.vec != 0, x);
#pragma unroll
            for (int u = 0; u < ROW_VEC; ++u) {
                C sq[NP];
                s_mul<NP, C>(x[u], x[u], sq);
#pragma unroll
                for (int k = 0; k < NP; ++k) acc[k] += sq[k];
            }
        }
        block_sum<NP, C>(acc, scratch);
        C m[NP], r[NP];
        const C inv_cols = C(1) / C(p.cols);
#pragma unroll
        for (int k = 0; k < NP; ++k) m[k] = acc[k] * inv_cols;
        m[0] += C(p.eps);
        s_rsqrt<NP, C>(m, r);
        if (p.rstd && threadIdx.x < p.np) {
#pragma unroll
            for (int k = 0; k < NP; ++k)
                if (k == static_cast<int>(threadIdx.x)) static_cast<C*>(p.rstd)[row * p.np + k] = r[k];
        }
        const int64_t yb = row * p.y_rs;
        for (int64_t c0 = static_cast<int64_t>(threadIdx.x) * ROW_VEC; c0 < p.cols;
             c0 += static_cast<int64_t>(blockDim.x) * ROW_VEC) {
            const int valid = vec_count(p.cols, c0);
            C x[ROW_VEC][NP], w[ROW_VEC][NP], t[ROW_VEC][NP];
            load_planes4<NP, T, C>(p.x, p.np, xb + c0, valid, p.vec != 0, x);
            if (p.w_np) load_weight4<NP, T, C>(p, c0, valid, w);
#pragma unroll
            for (int u = 0; u < ROW_VEC; ++u) {
                s_mul<NP, C>(x[u], r, t[u]);
                if (p.w_np) s_mul<NP, C>(t[u], w[u], t[u]);
            }
            store_planes4<NP, T, C>(p.y, p.np, yb + c0, valid, p.vec != 0, t);
        }
    }
}

// The same forward with the row held in registers: thread t owns columns (s * blockDim + t) * 4
// .. +3 for s < STEPS, issues every load of its share of the row at once, and writes y from the
// registers after the row's reduction, so x is read from HBM exactly once and never re-read.
template <typename T, int NP, int STEPS>
__global__ void __launch_bounds__(512, 1) rmsnorm_fwd_reg_kernel(const NormParams p) {
    using C = typename Compute<T>::type;
    __shared__ C scratch[16 * NP];
    const int64_t span = static_cast<int64_t>(blockDim.x) * ROW_VEC;
    for (int64_t row = blockIdx.x; row < p.rows; row += gridDim.x) {
        const int64_t xb = row * p.x_rs;
        C x[STEPS][ROW_VEC][NP];
#pragma unroll
        for (int s = 0; s < STEPS; ++s) {
            const int64_t c0 = s * span + static_cast<int64_t>(threadIdx.x) * ROW_VEC;
            load_planes4<NP, T, C>(p.x, p.np, xb + c0, max(0, vec_count(p.cols, c0)), p.vec != 0, x[s]);
        }
        C acc[NP];
#pragma unroll
        for (int k = 0; k < NP; ++k) acc[k] = C(0);
#pragma unroll
        for (int s = 0; s < STEPS; ++s) {
#pragma unroll
            for (int u = 0; u < ROW_VEC; ++u) {
                C sq[NP];
                s_mul<NP, C>(x[s][u], x[s][u], sq);
#pragma unroll
                for (int k = 0; k < NP; ++k) acc[k] += sq[k];
            }
        }
        block_sum<NP, C>(acc, scratch);
        C m[NP], r[NP];
        const C inv_cols = C(1) / C(p.cols);
#pragma unroll
        for (int k = 0; k < NP; ++k) m[k] = acc[k] * inv_cols;
        m[0] += C(p.eps);
        s_rsqrt<NP, C>(m, r);
        if (p.rstd && threadIdx.x < p.np) {
#pragma unroll
            for (int k = 0; k < NP; ++k)
                if (k == static_cast<int>(threadIdx.x)) static_cast<C*>(p.rstd)[row * p.np + k] = r[k];
        }
        const int64_t yb = row * p.y_rs;
#pragma unroll
        for (int s = 0; s < STEPS; ++s) {
            const int64_t c0 = s * span + static_cast<int64_t>(threadIdx.x) * ROW_VEC;
            const int valid = max(0, vec_count(p.cols, c0));
            C w[ROW_VEC][NP], t[ROW_VEC][NP];
            if (p.w_np) load_weight4<NP, T, C>(p, c0, valid, w);
#pragma unroll
            for (int u = 0; u < ROW_VEC; ++u) {
                s_mul<NP, C>(x[s][u], r, t[u]);
                if (p.w_np) s_mul<NP, C>(t[u], w[u], t[u]);
            }
            store_planes4<NP, T, C>(p.y, p.np, yb + c0, valid, p.vec != 0, t);
        }
    }
}

// Rows bulk-prefetched into L2 beyond the one streaming into shared memory.  Measured at 16384 x
// 4096 float32 rows (degree 4 / degree 1): forward 0.56 / 0.20 ms with 2 rows, 0.40 / 0.18 with 1,
// 0.45 / 0.18 with none; backward 0.78 / 0.31 ms with 1 or 2 rows, 0.72 / 0.29 with none (deeper
// prefetch competes with the rows being read for HBM and L2 capacity).
#ifndef PK_NORM_FWD_L2_AHEAD
#define PK_NORM_FWD_L2_AHEAD 1
#endif
#ifndef PK_NORM_BWD_L2_AHEAD
#define PK_NORM_BWD_L2_AHEAD 0
#endif
constexpr int NORM_FWD_L2_AHEAD = PK_NORM_FWD_L2_AHEAD;
constexpr int NORM_BWD_L2_AHEAD = PK_NORM_BWD_L2_AHEAD;

// The forward with the next row streaming in while this one is computed: thread t owns the column
// quads q = s * blockDim + t (s < STEPS) and copies its quads of the NEXT row's x planes into the
// second of two shared-memory stages with cp.async before it works on the current row, so HBM
// reads continue through the row reduction and the stores.  A thread reads back only what it
// copied, so the stages need no block barrier; the weight series of its columns stays in registers.
template <typename T, int NP, int STEPS>
__global__ void __launch_bounds__(512, 1) rmsnorm_fwd_stream_kernel(const NormParams p) {
    using C = float;
    __shared__ C scratch[16 * NP];
    extern __shared__ __align__(16) unsigned char dyn[];
    T* const stages = reinterpret_cast<T*>(dyn);  // [2][NP][cols]
    constexpr int VB = ROW_VEC * static_cast<int>(sizeof(T));
    const int64_t quads = p.cols / ROW_VEC, stage_elems = NP * p.cols;
    const C inv_cols = C(1) / C(p.cols);
    C w[STEPS][ROW_VEC][NP];
#pragma unroll
    for (int s = 0; s < STEPS; ++s) {
        const int64_t q = static_cast<int64_t>(s) * blockDim.x + threadIdx.x;
        load_weight4<NP, T, C>(p, q * ROW_VEC, q < quads ? ROW_VEC : 0, w[s]);
    }
    auto issue = [&](int64_t row, int stage) {
        T* st = stages + stage * stage_elems;
#pragma unroll
        for (int s = 0; s < STEPS; ++s) {
            const int64_t q = static_cast<int64_t>(s) * blockDim.x + threadIdx.x;
            if (q < quads) {
#pragma unroll
                for (int k = 0; k < NP; ++k)
                    cp_async_vec<VB>(st + k * p.cols + q * ROW_VEC,
                                     static_cast<const T*>(p.x[k]) + row * p.x_rs + q * ROW_VEC);
            }
        }
        cp_async_commit();
    };
    // rows further ahead go to L2 only (one bulk prefetch per plane), so more of HBM's latency is
    // covered than two shared-memory stages allow
    auto prefetch = [&](int64_t row) {
        if (row < p.rows && threadIdx.x < NP)
            prefetch_l2(static_cast<const T*>(p.x[threadIdx.x]) + row * p.x_rs, static_cast<size_t>(p.cols) * sizeof(T));
    };
    int64_t row = blockIdx.x;
    if (row < p.rows) issue(row, 0);
#pragma unroll
    for (int a = 1; a <= NORM_FWD_L2_AHEAD; ++a) prefetch(row + static_cast<int64_t>(a) * gridDim.x);
    for (int64_t i = 0; row < p.rows; ++i, row += gridDim.x) {
        const int stage = static_cast<int>(i & 1);
        const int64_t nrow = row + gridDim.x;
        if (NORM_FWD_L2_AHEAD > 0) prefetch(row + static_cast<int64_t>(NORM_FWD_L2_AHEAD + 1) * gridDim.x);
        if (nrow < p.rows) issue(nrow, stage ^ 1);
        else cp_async_commit();  // an empty group keeps the wait count below uniform
        cp_async_wait<1>();      // this thread's copies of `row` have landed
        const T* const xs = stages + stage * stage_elems;
        C acc[NP], diag[NP];
#pragma unroll
        for (int k = 0; k < NP; ++k) acc[k] = diag[k] = C(0);
#pragma unroll
        for (int s = 0; s < STEPS; ++s) {
            const int64_t q = static_cast<int64_t>(s) * blockDim.x + threadIdx.x;
            if (q >= quads) continue;
            C xv[NP][ROW_VEC];
#pragma unroll
            for (int k = 0; k < NP; ++k) load_vec4<T>(xs + k * p.cols + q * ROW_VEC, xv[k]);
#pragma unroll
            for (int u = 0; u < ROW_VEC; ++u) {
                C x[NP];
#pragma unroll
                for (int k = 0; k < NP; ++k) x[k] = xv[k][u];
                s_square_acc<NP, C>(x, acc, diag);
            }
        }
#pragma unroll
        for (int k = 0; k < NP; ++k) acc[k] = C(2) * acc[k] + diag[k];
        block_sum<NP, C>(acc, scratch);
        C m[NP], r[NP];
#pragma unroll
        for (int k = 0; k < NP; ++k) m[k] = acc[k] * inv_cols;
        m[0] += C(p.eps);
        s_rsqrt<NP, C>(m, r);
        if (p.rstd && threadIdx.x < NP) {
#pragma unroll
            for (int k = 0; k < NP; ++k)
                if (k == static_cast<int>(threadIdx.x)) static_cast<C*>(p.rstd)[row * NP + k] = r[k];
        }
        const int64_t yb = row * p.y_rs;
#pragma unroll
        for (int s = 0; s < STEPS; ++s) {
            const int64_t q = static_cast<int64_t>(s) * blockDim.x + threadIdx.x;
            if (q >= quads) continue;
            C xv[NP][ROW_VEC], out[ROW_VEC][NP];
#pragma unroll
            for (int k = 0; k < NP; ++k) load_vec4<T>(xs + k * p.cols + q * ROW_VEC, xv[k]);
#pragma unroll
            for (int u = 0; u < ROW_VEC; ++u) {
                C x[NP];
#pragma unroll
                for (int k = 0; k < NP; ++k) x[k] = xv[k][u];
                s_mul<NP, C>(x, r, out[u]);
                if (p.w_np) s_mul<NP, C>(out[u], w[s][u], out[u]);
            }
            store_planes4<NP, T, C>(p.y, NP, yb + q * ROW_VEC, ROW_VEC, true, out);
        }
    }
    cp_async_wait<0>();
}

// Each CTA walks rows blockIdx.x, blockIdx.x + gridDim.x, ... and keeps its weight-gradient
// partial sums for the columns it owns in shared memory (np x cols values).
template <typename T, int NP>
__global__ void __launch_bounds__(512) rmsnorm_bwd_kernel(const NormParams p) {
    using C = typename Compute<T>::type;
    __shared__ C scratch[16 * NP];
    extern __shared__ __align__(16) unsigned char dyn[];
    C* dwp = reinterpret_cast<C*>(dyn);  // [NP][cols] when p.dw_part != nullptr
    const bool want_dw = p.dw_part != nullptr;
    if (want_dw)
        for (int64_t i = threadIdx.x; i < static_cast<int64_t>(NP) * p.cols; i += blockDim.x) dwp[i] = C(0);
    const C inv_cols = C(1) / C(p.cols);
    for (int64_t row = blockIdx.x; row < p.rows; row += gridDim.x) {
        const int64_t xb = row * p.x_rs, gb = row * p.g_rs;
        C r[NP];
#pragma unroll
        for (int k = 0; k < NP; ++k) r[k] = k < p.np ? static_cast<const C*>(p.rstd)[row * p.np + k] : C(0);
        C d[NP];
#pragma unroll
        for (int k = 0; k < NP; ++k) d[k] = C(0);
        for (int64_t c0 = static_cast<int64_t>(threadIdx.x) * ROW_VEC; c0 < p.cols;
             c0 += static_cast<int64_t>(blockDim.x) * ROW_VEC) {
            const int valid = vec_count(p.cols, c0);
            C x[ROW_VEC][NP], g[ROW_VEC][NP], w[ROW_VEC][NP];
            load_planes4<NP, T, C>(p.x, p.np, xb + c0, valid, p.vec != 0, x);
            load_planes4<NP, T, C>(p.g, p.np, gb + c0, valid, p.vec != 0, g);
            if (p.w_np) load_weight4<NP, T, C>(p, c0, valid, w);
#pragma unroll
            for (int u = 0; u < ROW_VEC; ++u) {
                C gy[NP], t[NP];
                if (p.w_np) s_mul<NP, C>(g[u], w[u], gy);
                else {
#pragma unroll
                    for (int k = 0; k < NP; ++k) gy[k] = g[u][k];
                }
                s_mul<NP, C>(gy, x[u], t);
#pragma unroll
                for (int k = 0; k < NP; ++k) d[k] += t[k];
            }
        }
        block_sum<NP, C>(d, scratch);
        C r2[NP], r3[NP], coef[NP];
        s_mul<NP, C>(r, r, r2);
        s_mul<NP, C>(r2, r, r3);
        s_mul<NP, C>(r3, d, coef);
#pragma unroll
        for (int k = 0; k < NP; ++k) coef[k] *= inv_cols;
        const int64_t yb = row * p.y_rs;
        for (int64_t c0 = static_cast<int64_t>(threadIdx.x) * ROW_VEC; c0 < p.cols;
             c0 += static_cast<int64_t>(blockDim.x) * ROW_VEC) {
            const int valid = vec_count(p.cols, c0);
            C x[ROW_VEC][NP], g[ROW_VEC][NP], w[ROW_VEC][NP], out[ROW_VEC][NP];
            load_planes4<NP, T, C>(p.x, p.np, xb + c0, valid, p.vec != 0, x);
            load_planes4<NP, T, C>(p.g, p.np, gb + c0, valid, p.vec != 0, g);
            if (p.w_np) load_weight4<NP, T, C>(p, c0, valid, w);
#pragma unroll
            for (int u = 0; u < ROW_VEC; ++u) {
                C gy[NP], a[NP], b[NP];
                if (p.w_np) s_mul<NP, C>(g[u], w[u], gy);
                else {
#pragma unroll
                    for (int k = 0; k < NP; ++k) gy[k] = g[u][k];
                }
                s_mul<NP, C>(r, gy, a);
                s_mul<NP, C>(coef, x[u], b);
#pragma unroll
                for (int k = 0; k < NP; ++k) out[u][k] = a[k] - b[k];
                if (want_dw && u < valid) {
                    C xr[NP], gx[NP];
                    s_mul<NP, C>(x[u], r, xr);
                    s_mul<NP, C>(g[u], xr, gx);
                    // vector layout: [k][u][cols/4], consecutive threads on consecutive words
                    const int64_t slot = p.vec ? u * (p.cols / ROW_VEC) + c0 / ROW_VEC : c0 + u;
#pragma unroll
                    for (int k = 0; k < NP; ++k) dwp[k * p.cols + slot] += gx[k];
                }
            }
            store_planes4<NP, T, C>(p.y, p.np, yb + c0, valid, p.vec != 0, out);
        }
    }
    if (want_dw) {
        __syncthreads();
        C* out = static_cast<C*>(p.dw_part) + static_cast<int64_t>(blockIdx.x) * p.np * p.cols;
        const int64_t q = p.cols / ROW_VEC;
        for (int64_t i = threadIdx.x; i < static_cast<int64_t>(p.np) * p.cols; i += blockDim.x) {
            const int64_t k = i / p.cols, c = i % p.cols;
            out[i] = dwp[k * p.cols + (p.vec ? (c % ROW_VEC) * q + c / ROW_VEC : c)];
        }
    }
}

// The backward with whole rows in registers and one CTA per row (persistent over rows): for short
// series a row's x and g fit the registers of one CTA, so no cluster exchange is needed and
// several CTAs per SM keep rows in flight while others reduce.  Thread t owns the column quads
// s * blockDim + t (s < STEPS) of every row; with W the weight series and the weight-gradient
// partials of those columns stay in registers, written per CTA to dw_part[blockIdx.x] at the end.
// Per element: rg = r (*) g, dw += rg (*) x, a = rg (*) w, row sum += a (*) x (= r (*) gy (*) x),
// then dx = a - (r (*) r (*) sum / cols) (*) x.
template <typename T, int NP, int STEPS, bool W>
__global__ void __launch_bounds__(256) rmsnorm_bwd_reg_kernel(const NormParams p) {
    using C = typename Compute<T>::type;
    __shared__ C scratch[8 * NP];
    const int64_t span = static_cast<int64_t>(blockDim.x) * ROW_VEC;
    const C inv_cols = C(1) / C(p.cols);
    C w[STEPS][ROW_VEC][NP], dwa[STEPS][ROW_VEC][NP];
#pragma unroll
    for (int s = 0; s < STEPS; ++s) {
        const int64_t c0 = s * span + static_cast<int64_t>(threadIdx.x) * ROW_VEC;
        if constexpr (W) load_weight4<NP, T, C>(p, c0, max(0, vec_count(p.cols, c0)), w[s]);
#pragma unroll
        for (int u = 0; u < ROW_VEC; ++u) {
#pragma unroll
            for (int k = 0; k < NP; ++k) {
                dwa[s][u][k] = C(0);
                if constexpr (!W) w[s][u][k] = C(k == 0 ? 1 : 0);
            }
        }
    }
    for (int64_t row = blockIdx.x; row < p.rows; row += gridDim.x) {
        C x[STEPS][ROW_VEC][NP], g[STEPS][ROW_VEC][NP];
#pragma unroll
        for (int s = 0; s < STEPS; ++s) {
            const int64_t c0 = s * span + static_cast<int64_t>(threadIdx.x) * ROW_VEC;
            const int valid = max(0, vec_count(p.cols, c0));
            load_planes4<NP, T, C>(p.x, p.np, row * p.x_rs + c0, valid, p.vec != 0, x[s]);
            load_planes4<NP, T, C>(p.g, p.np, row * p.g_rs + c0, valid, p.vec != 0, g[s]);
        }
        C r[NP], d[NP];
#pragma unroll
        for (int k = 0; k < NP; ++k) {
            r[k] = k < p.np ? static_cast<const C*>(p.rstd)[row * p.np + k] : C(0);
            d[k] = C(0);
        }
#pragma unroll
        for (int s = 0; s < STEPS; ++s) {
#pragma unroll
            for (int u = 0; u < ROW_VEC; ++u) {
                C rg[NP], a[NP];
                s_mul<NP, C>(r, g[s][u], rg);
                if constexpr (W) s_mul_acc<NP, C>(rg, x[s][u], dwa[s][u]);
                s_mul<NP, C>(rg, w[s][u], a);
                s_mul_acc<NP, C>(a, x[s][u], d);
#pragma unroll
                for (int k = 0; k < NP; ++k) g[s][u][k] = a[k];
            }
        }
        block_sum<NP, C>(d, scratch);
        C coef[NP];
        s_mul<NP, C>(r, r, coef);
        s_mul<NP, C>(coef, d, coef);
#pragma unroll
        for (int k = 0; k < NP; ++k) coef[k] *= inv_cols;
#pragma unroll
        for (int s = 0; s < STEPS; ++s) {
            const int64_t c0 = s * span + static_cast<int64_t>(threadIdx.x) * ROW_VEC;
            C out[ROW_VEC][NP];
#pragma unroll
            for (int u = 0; u < ROW_VEC; ++u) s_sub_mul<NP, C>(g[s][u], coef, x[s][u], out[u]);
            store_planes4<NP, T, C>(p.y, p.np, row * p.y_rs + c0, max(0, vec_count(p.cols, c0)), p.vec != 0, out);
        }
    }
    if constexpr (W) {
        if (p.dw_part != nullptr) {
            C* part = static_cast<C*>(p.dw_part) + static_cast<int64_t>(blockIdx.x) * p.np * p.cols;
#pragma unroll
            for (int s = 0; s < STEPS; ++s) {
                const int64_t c0 = s * span + static_cast<int64_t>(threadIdx.x) * ROW_VEC;
#pragma unroll
                for (int u = 0; u < ROW_VEC; ++u) {
                    if (c0 + u >= p.cols) continue;
#pragma unroll
                    for (int k = 0; k < NP; ++k)
                        if (k < p.np) part[k * p.cols + c0 + u] = dwa[s][u][k];
                }
            }
        }
    }
}

// The backward with each row split over a cluster of CL CTAs: CTA rank h owns columns
// [h * cols/CL, (h+1) * cols/CL), holds its x and g in registers (thread t: columns
// h * cols/CL + (s * blockDim + t) * 4 .. +3, s < STEPS), so both passes read registers and x, g
// come from HBM once.  The row sum d = sum gy (*) x is combined through distributed shared memory
// (every CTA adds the CL partials in rank order, so they agree bit for bit); the per-row slots are
// double-buffered so one cluster barrier per row suffices.  Several CTAs fit per SM, so one row's
// loads overlap another row's arithmetic.  Weight-gradient partials accumulate in shared memory
// per cluster ([k][u][part/4] layout), written to dw_part[cluster][k][cols].
template <typename T, int NP, int STEPS, int CL>
__global__ void __launch_bounds__(256, 2) rmsnorm_bwd_cluster_kernel(const NormParams p) {
    using C = typename Compute<T>::type;
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    __shared__ C scratch[16 * NP];
    __shared__ C dslot[2][NP];
    extern __shared__ __align__(16) unsigned char dyn[];
    C* dwp = reinterpret_cast<C*>(dyn);
    const int h = static_cast<int>(cluster.block_rank());
    const int64_t half = p.cols / CL, q = half / ROW_VEC;  // "half": this CTA's share of the row
    const int64_t cbase = h * half;
    const int64_t n_clusters = gridDim.x / CL, cid = blockIdx.x / CL;
    const bool want_dw = p.dw_part != nullptr;
    if (want_dw)
        for (int64_t i = threadIdx.x; i < static_cast<int64_t>(NP) * half; i += blockDim.x) dwp[i] = C(0);
    const C* slots[CL];
#pragma unroll
    for (int j = 0; j < CL; ++j) slots[j] = cluster.map_shared_rank(&dslot[0][0], j);
    const C inv_cols = C(1) / C(p.cols);
    const int64_t span = static_cast<int64_t>(blockDim.x) * ROW_VEC;
    int par = 0;
    for (int64_t row = cid; row < p.rows; row += n_clusters, par ^= 1) {
        const int64_t xb = row * p.x_rs + cbase, gb = row * p.g_rs + cbase;
        C x[STEPS][ROW_VEC][NP], g[STEPS][ROW_VEC][NP];
#pragma unroll
        for (int s = 0; s < STEPS; ++s) {
            const int64_t c0 = s * span + static_cast<int64_t>(threadIdx.x) * ROW_VEC;
            const int valid = max(0, vec_count(half, c0));
            load_planes4<NP, T, C>(p.x, p.np, xb + c0, valid, true, x[s]);
            load_planes4<NP, T, C>(p.g, p.np, gb + c0, valid, true, g[s]);
        }
        C r[NP];
#pragma unroll
        for (int k = 0; k < NP; ++k) r[k] = k < p.np ? static_cast<const C*>(p.rstd)[row * p.np + k] : C(0);
        C d[NP];
#pragma unroll
        for (int k = 0; k < NP; ++k) d[k] = C(0);
#pragma unroll
        for (int s = 0; s < STEPS; ++s) {
            const int64_t c0 = s * span + static_cast<int64_t>(threadIdx.x) * ROW_VEC;
            const int valid = max(0, vec_count(half, c0));
            C w[ROW_VEC][NP];
            if (p.w_np) load_weight4<NP, T, C>(p, cbase + c0, valid, w);
#pragma unroll
            for (int u = 0; u < ROW_VEC; ++u) {
                // gx = g (*) x serves both the weight gradient (gx (*) r) and the row sum
                // (gy (*) x = w (*) gx); g then becomes gy = g (*) w for the second pass
                C gx[NP];
                s_mul<NP, C>(g[s][u], x[s][u], gx);
                if (want_dw && u < valid) {
                    C gxr[NP];
                    s_mul<NP, C>(gx, r, gxr);
                    const int64_t slot = u * q + c0 / ROW_VEC;
#pragma unroll
                    for (int k = 0; k < NP; ++k) dwp[k * half + slot] += gxr[k];
                }
                if (p.w_np) {
                    C t[NP];
                    s_mul<NP, C>(w[u], gx, t);
                    s_mul<NP, C>(g[s][u], w[u], g[s][u]);
#pragma unroll
                    for (int k = 0; k < NP; ++k) d[k] += t[k];
                } else {
#pragma unroll
                    for (int k = 0; k < NP; ++k) d[k] += gx[k];
                }
            }
        }
        block_sum<NP, C>(d, scratch);
        if (threadIdx.x == 0) {
#pragma unroll
            for (int k = 0; k < NP; ++k) dslot[par][k] = d[k];
        }
        cluster.sync();
#pragma unroll
        for (int k = 0; k < NP; ++k) {
            C t = slots[0][par * NP + k];
#pragma unroll
            for (int j = 1; j < CL; ++j) t += slots[j][par * NP + k];
            d[k] = t;
        }
        C r2[NP], r3[NP], coef[NP];
        s_mul<NP, C>(r, r, r2);
        s_mul<NP, C>(r2, r, r3);
        s_mul<NP, C>(r3, d, coef);
#pragma unroll
        for (int k = 0; k < NP; ++k) coef[k] *= inv_cols;
        const int64_t yb = row * p.y_rs + cbase;
#pragma unroll
        for (int s = 0; s < STEPS; ++s) {
            const int64_t c0 = s * span + static_cast<int64_t>(threadIdx.x) * ROW_VEC;
            C out[ROW_VEC][NP];
#pragma unroll
            for (int u = 0; u < ROW_VEC; ++u) {
                C a[NP], b[NP];
                s_mul<NP, C>(r, g[s][u], a);
                s_mul<NP, C>(coef, x[s][u], b);
#pragma unroll
                for (int k = 0; k < NP; ++k) out[u][k] = a[k] - b[k];
            }
            store_planes4<NP, T, C>(p.y, p.np, yb + c0, max(0, vec_count(half, c0)), true, out);
        }
    }
    if (want_dw) {
        __syncthreads();
        C* out = static_cast<C*>(p.dw_part) + cid * p.np * p.cols + cbase;
        for (int64_t i = threadIdx.x; i < static_cast<int64_t>(p.np) * half; i += blockDim.x) {
            const int64_t k = i / half, c = i % half;
            out[k * p.cols + c] = dwp[k * half + (c % ROW_VEC) * q + c / ROW_VEC];
        }
    }
    cluster.sync();  // the peer may still read this CTA's row slots
}

// The cluster backward with the next row streaming in while this one is computed.  CTA rank h
// of a CL-CTA cluster owns columns [h * cols/CL, (h+1) * cols/CL); thread t owns the column
// quads q = s * blockDim + t (s < STEPS) of every row.  Each thread copies its own quads of the
// NEXT row's x and g planes into a second shared-memory stage with cp.async while it computes
// the current row from the first (rows further ahead are bulk-prefetched into L2), so HBM reads
// never wait for the arithmetic, the row exchange or the stores; since a thread reads back only
// what it copied, the stages need no block barrier.  The weight series and the weight-gradient
// partial sums of the thread's columns stay in registers for the whole launch.  For float planes
// the first pass leaves a = r (*) g (*) w in the g stage, so the second pass is dx = a - coef (*) x.
// The CTAs of a cluster exchange their row partials of d by pushing them into each other's shared
// memory (st.async completing bytes on the receiver's mbarrier, one barrier and slot set per row
// parity), so no cluster-wide barrier (and no release of the previous row's stores) sits in the
// row loop.
template <typename T, int NP, int STEPS, int CL>
__global__ void __launch_bounds__(STEPS == 1 ? 512 : 256, 1) rmsnorm_bwd_stream_kernel(const NormParams p) {
    using C = float;
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    __shared__ C scratch[16 * NP];
    __shared__ C xslot[2][CL][NP];  // [row parity][sender rank][k]
    __shared__ __align__(8) uint64_t xbar[2];
    extern __shared__ __align__(16) unsigned char dyn[];
    T* const stages = reinterpret_cast<T*>(dyn);  // [2][x planes, g planes][NP][half]
    constexpr int VB = ROW_VEC * static_cast<int>(sizeof(T));
    const int h = static_cast<int>(cluster.block_rank());
    const int64_t half = p.cols / CL, quads = half / ROW_VEC, cbase = h * half;
    const int64_t stage_elems = 2 * NP * half;
    const int64_t n_clusters = gridDim.x / CL, cid = blockIdx.x / CL;
    const bool want_dw = p.dw_part != nullptr;
    if (threadIdx.x == 0) {
        mbar_init(&xbar[0], 1);
        mbar_init(&xbar[1], 1);
        fence_mbar_init();
    }
    cluster.sync();  // every CTA's barriers are initialised before any peer signals them
    const C inv_cols = C(1) / C(p.cols);

    C w[STEPS][ROW_VEC][NP], dwa[STEPS][ROW_VEC][NP];
#pragma unroll
    for (int s = 0; s < STEPS; ++s) {
        const int64_t q = static_cast<int64_t>(s) * blockDim.x + threadIdx.x;
        load_weight4<NP, T, C>(p, cbase + q * ROW_VEC, q < quads ? ROW_VEC : 0, w[s]);
#pragma unroll
        for (int u = 0; u < ROW_VEC; ++u) {
#pragma unroll
            for (int k = 0; k < NP; ++k) dwa[s][u][k] = C(0);
        }
    }
    auto issue = [&](int64_t row, int stage) {
        T* st = stages + stage * stage_elems;
#pragma unroll
        for (int s = 0; s < STEPS; ++s) {
            const int64_t q = static_cast<int64_t>(s) * blockDim.x + threadIdx.x;
            if (q < quads) {
                const int64_t off = cbase + q * ROW_VEC;
#pragma unroll
                for (int k = 0; k < NP; ++k) {
                    cp_async_vec<VB>(st + k * half + q * ROW_VEC, static_cast<const T*>(p.x[k]) + row * p.x_rs + off);
                    cp_async_vec<VB>(st + (NP + k) * half + q * ROW_VEC,
                                     static_cast<const T*>(p.g[k]) + row * p.g_rs + off);
                }
            }
        }
        cp_async_commit();
    };
    // rows further ahead go to L2 only (one bulk prefetch per plane segment), so more of HBM's
    // latency is covered than two shared-memory stages allow
    auto prefetch = [&](int64_t row) {
        if (row < p.rows && threadIdx.x < 2 * NP) {
            const int k = threadIdx.x % NP;
            const T* base = threadIdx.x < NP ? static_cast<const T*>(p.x[k]) + row * p.x_rs
                                             : static_cast<const T*>(p.g[k]) + row * p.g_rs;
            prefetch_l2(base + cbase, static_cast<size_t>(half) * sizeof(T));
        }
    };
    auto load_r = [&](int64_t row, C (&r)[NP]) {
#pragma unroll
        for (int k = 0; k < NP; ++k) r[k] = static_cast<const C*>(p.rstd)[row * NP + k];
    };

    int64_t row = cid;
    C rn[NP];
    if (row < p.rows) {
        issue(row, 0);
        load_r(row, rn);
    }
#pragma unroll
    for (int a = 1; a <= NORM_BWD_L2_AHEAD; ++a) prefetch(row + a * n_clusters);
    int par = 0;
    for (int64_t i = 0; row < p.rows; ++i, row += n_clusters, par ^= 1) {
        const int stage = static_cast<int>(i & 1);
        const int64_t nrow = row + n_clusters;
        if (NORM_BWD_L2_AHEAD > 0) prefetch(row + (NORM_BWD_L2_AHEAD + 1) * n_clusters);
        if (nrow < p.rows) issue(nrow, stage ^ 1);
        else cp_async_commit();  // an empty group keeps the wait count below uniform
        C r[NP];
#pragma unroll
        for (int k = 0; k < NP; ++k) r[k] = rn[k];
        if (nrow < p.rows) load_r(nrow, rn);
        cp_async_wait<1>();  // this thread's copies of `row` have landed
        T* const xs = stages + stage * stage_elems;
        T* const gs = xs + NP * half;

        C d[NP];
#pragma unroll
        for (int k = 0; k < NP; ++k) d[k] = C(0);
#pragma unroll
        for (int s = 0; s < STEPS; ++s) {
            const int64_t q = static_cast<int64_t>(s) * blockDim.x + threadIdx.x;
            if (q >= quads) continue;
            C xv[NP][ROW_VEC], gv[NP][ROW_VEC];
#pragma unroll
            for (int k = 0; k < NP; ++k) {
                load_vec4<T>(xs + k * half + q * ROW_VEC, xv[k]);
                load_vec4<T>(gs + k * half + q * ROW_VEC, gv[k]);
            }
#pragma unroll
            for (int u = 0; u < ROW_VEC; ++u) {
                C x[NP], g[NP], rg[NP], a[NP];
#pragma unroll
                for (int k = 0; k < NP; ++k) {
                    x[k] = xv[k][u];
                    g[k] = gv[k][u];
                }
                // rg = r (*) g feeds the weight gradient (rg (*) x) and a = rg (*) w, the first
                // term of dx; the row sum is accumulated as a (*) x = r (*) (gy (*) x), gy = g (*) w
                // (r is constant along the row, so the row total is r (*) d and the coefficient
                // below takes r (*) r instead of r^3)
                s_mul<NP, C>(r, g, rg);
                if (want_dw) s_mul_acc<NP, C>(rg, x, dwa[s][u]);
                s_mul<NP, C>(rg, w[s][u], a);
                s_mul_acc<NP, C>(a, x, d);
                if constexpr (sizeof(T) == 4) {
#pragma unroll
                    for (int k = 0; k < NP; ++k) gv[k][u] = a[k];  // g of element u is no longer needed
                }
            }
            if constexpr (sizeof(T) == 4) {
#pragma unroll
                for (int k = 0; k < NP; ++k) store_vec4<T>(gs + k * half + q * ROW_VEC, gv[k]);
            }
        }
        block_sum<NP, C>(d, scratch);
        if (threadIdx.x == 0) {
            mbar_arrive_expect_tx(&xbar[par], (CL - 1) * NP * static_cast<uint32_t>(sizeof(C)));
#pragma unroll
            for (int j = 0; j < CL; ++j) {
                if (j == h) continue;
                const uint32_t slot = cluster_map_u32(&xslot[par][h][0], j), bar = cluster_map_u32(&xbar[par], j);
#pragma unroll
                for (int k = 0; k < NP; ++k) st_async_f32(slot + 4 * k, d[k], bar);
            }
        }
        // barrier xbar[par] serves every second row: its (i / 2)-th phase is this row's
        const bool ok = mbar_wait_bounded(&xbar[par], static_cast<uint32_t>(i >> 1) & 1u, p.status, 501);
        if (__syncthreads_or(!ok)) break;  // the whole CTA leaves together (the peer's wait ends too)
        // the partials in rank order, so every CTA of the cluster forms the same sum
#pragma unroll
        for (int k = 0; k < NP; ++k) {
            C t = h == 0 ? d[k] : xslot[par][0][k];
#pragma unroll
            for (int j = 1; j < CL; ++j) t += j == h ? d[k] : xslot[par][j][k];
            d[k] = t;
        }
        // d holds r (*) sum gy (*) x here, so coef = r^3 (*) sum gy (*) x / cols = r (*) r (*) d / cols
        C coef[NP];
        s_mul<NP, C>(r, r, coef);
        s_mul<NP, C>(coef, d, coef);
#pragma unroll
        for (int k = 0; k < NP; ++k) coef[k] *= inv_cols;
        const int64_t yb = row * p.y_rs + cbase;
#pragma unroll
        for (int s = 0; s < STEPS; ++s) {
            const int64_t q = static_cast<int64_t>(s) * blockDim.x + threadIdx.x;
            if (q >= quads) continue;
            C xv[NP][ROW_VEC], av[NP][ROW_VEC];
#pragma unroll
            for (int k = 0; k < NP; ++k) {
                load_vec4<T>(xs + k * half + q * ROW_VEC, xv[k]);
                load_vec4<T>(gs + k * half + q * ROW_VEC, av[k]);
            }
            C out[ROW_VEC][NP];
#pragma unroll
            for (int u = 0; u < ROW_VEC; ++u) {
                C x[NP], a[NP];
#pragma unroll
                for (int k = 0; k < NP; ++k) {
                    x[k] = xv[k][u];
                    a[k] = av[k][u];
                }
                if constexpr (sizeof(T) != 4) {
                    C rg[NP];
                    s_mul<NP, C>(r, a, rg);  // the stage holds g: a = r (*) g (*) w
                    s_mul<NP, C>(rg, w[s][u], a);
                }
                s_sub_mul<NP, C>(a, coef, x, out[u]);
            }
            store_planes4<NP, T, C>(p.y, NP, yb + q * ROW_VEC, ROW_VEC, true, out);
        }
    }
    cp_async_wait<0>();
    if (want_dw) {
        C* out = static_cast<C*>(p.dw_part) + cid * NP * p.cols + cbase;
#pragma unroll
        for (int s = 0; s < STEPS; ++s) {
            const int64_t q = static_cast<int64_t>(s) * blockDim.x + threadIdx.x;
            if (q >= quads) continue;
#pragma unroll
            for (int k = 0; k < NP; ++k) {
                C v[ROW_VEC];
#pragma unroll
                for (int u = 0; u < ROW_VEC; ++u) v[u] = dwa[s][u][k];
                store_vec4<C>(out + k * p.cols + q * ROW_VEC, v);
            }
        }
    }
    cluster.sync();  // no CTA leaves while a peer may still write into its shared memory
}

// dw[k][c] = sum_b part[b][k][c].  A CTA covers 32 consecutive values with 8 lanes of partials
// each (warp j sums partials j, j+8, ...; coalesced 128-byte rows), then combines the 8 lanes.
template <typename T, int NP>
__global__ void __launch_bounds__(256) rmsnorm_dw_reduce_kernel(const NormParams p, int parts) {
    using C = typename Compute<T>::type;
    __shared__ C lanes[8][33];
    const int64_t total = static_cast<int64_t>(p.np) * p.cols;
    const int col = threadIdx.x & 31, lane = threadIdx.x >> 5;
    const int64_t i = static_cast<int64_t>(blockIdx.x) * 32 + col;
    C s = C(0);
    if (i < total) {
        const C* src = static_cast<const C*>(p.dw_part) + i;
#pragma unroll 4
        for (int b = lane; b < parts; b += 8) s += src[static_cast<int64_t>(b) * total];
    }
    lanes[lane][col] = s;
    __syncthreads();
    if (lane == 0 && i < total) {
        C t = C(0);
#pragma unroll
        for (int l = 0; l < 8; ++l) t += lanes[l][col];
        const int k = static_cast<int>(i / p.cols);
        static_cast<T*>(const_cast<void*>(p.g[k]))[i % p.cols] = from_c<T>(t);
    }
}

static int norm_threads(int64_t cols) { return cols >= 2048 ? 512 : (cols >= 512 ? 256 : 128); }

// Launch the register-resident forward when a row fits: STEPS vectors of 4 columns per thread,
// at most 512 threads, float compute, degree <= 5.  Returns false when it does not apply.
// Weight-gradient partials [parts][np][cols] -> dw planes.
template <typename T, int NP>
static int reduce_dw(const NormParams& p, void* const* dw, int parts, cudaStream_t s) {
    NormParams q = p;
    for (int k = 0; k < p.np; ++k) q.g[k] = dw[k];
    const int64_t total = static_cast<int64_t>(p.np) * p.cols;
    PK_LAUNCHED(rmsnorm_dw_reduce_kernel<T, NP><<<static_cast<int>(ceil_div(total, 32)), 256, 0, s>>>(q, parts));
    PK_CHECK_LAUNCH("pk_rmsnorm_bwd: weight reduction");
    return PK_OK;
}

// Series lengths below these use the register kernels instead of the streaming ones.  At degree 1
// (16384 x 4096 float32) the register forward takes 0.175 ms against 0.185 streaming, while the
// streaming backward takes 0.286 ms against 0.366 with registers.
#ifndef PK_NORM_FWD_STREAM_MIN_NP
#define PK_NORM_FWD_STREAM_MIN_NP 3
#endif
#ifndef PK_NORM_BWD_STREAM_MIN_NP
#define PK_NORM_BWD_STREAM_MIN_NP 1
#endif

// Tuning of the streaming backward: the cluster size tried first, and the half-row width (in
// column quads) from which a thread takes two quads per row.
#ifndef PK_NORM_BWD_CL
#define PK_NORM_BWD_CL 2
#endif
#ifndef PK_NORM_BWD_STEP2_QUADS
#define PK_NORM_BWD_STEP2_QUADS 256
#endif

// The streaming backward (rmsnorm_bwd_stream_kernel) for rows that split into CL-CTA clusters of
// at most 512 threads x 4 columns with two stages of x and g in shared memory.  Returns 1 when the
// shape does not suit it (the caller uses another kernel), else a status.
template <typename T, int NP, int CL>
static int bwd_stream(NormParams& p, void* const* dw, void* ws, size_t ws_bytes, cudaStream_t s) {
    if (p.np != NP || !p.vec || p.cols % (CL * ROW_VEC)) return 1;
    const int64_t half = p.cols / CL, quads = half / ROW_VEC;
    const size_t smem = 2 * 2 * static_cast<size_t>(NP) * half * sizeof(T);
    if (quads < 64 || quads > 512 || smem > 200 * 1024) return 1;
    // two column quads per thread once a half row has 256 of them: the per-row work (block
    // reduction, exchange, rsqrt-series coefficients) is shared by twice the elements
    const int steps = quads >= PK_NORM_BWD_STEP2_QUADS ? 2 : 1;
    const int threads = static_cast<int>(round_up(ceil_div(quads, steps), 32));
    auto kern = steps == 2 ? rmsnorm_bwd_stream_kernel<T, NP, 2, CL> : rmsnorm_bwd_stream_kernel<T, NP, 1, CL>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return cuda_fail(e, "pk_rmsnorm_bwd: cudaFuncSetAttribute");
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(CL);
    cfg.blockDim = dim3(static_cast<unsigned>(threads));
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = CL;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    // only as many clusters as can be resident at once: rows are dealt out statically, so a
    // cluster that waited for a free slot would finish its rows after all the others
    int resident = 0;
    e = cudaOccupancyMaxActiveClusters(&resident, kern, &cfg);
    if (e != cudaSuccess) return cuda_fail(e, "pk_rmsnorm_bwd: cluster occupancy query");
    if (resident < 1) return 1;
    const int64_t clusters =
        std::min<int64_t>({p.rows, static_cast<int64_t>(resident), static_cast<int64_t>(num_sms()) * 4 / CL});
    if (dw) {
        const size_t need = static_cast<size_t>(clusters) * p.np * p.cols * sizeof(float);
        if (!ws || ws_bytes < need) return fail(PK_ERR_WORKSPACE, "pk_rmsnorm_bwd: workspace too small");
        p.dw_part = ws;
    }
    cfg.gridDim = dim3(static_cast<unsigned>(CL * clusters));
    void* tok;
    prof_begin("rmsnorm_bwd", s, &tok);
    e = cudaLaunchKernelEx(&cfg, kern, p);
    if (e == cudaSuccess) ::pk::note_launch();
    if (e != cudaSuccess) return cuda_fail(e, "pk_rmsnorm_bwd: cluster launch");
    PK_CHECK_LAUNCH("pk_rmsnorm_bwd");
    if (dw) {
        const int st = reduce_dw<T, NP>(p, dw, static_cast<int>(clusters), s);
        if (st != PK_OK) return st;
    }
    prof_end("rmsnorm_bwd", s, tok);
    return PK_OK;
}

// The register backward (rmsnorm_bwd_reg_kernel) for rows of at most 256 threads x 4 quads with
// vector-aligned planes.  Returns 1 when the shape does not suit it, else a status.  Used up to
// degree 1: at 16384 x 4096 float32 it takes 0.267 ms against 0.300 streaming at degree 1, but
// 1.49 against 0.72 ms at degree 4 with a weight series (the registers then hold one row per SM).
#ifndef PK_NORM_BWD_REG_MAX_NP
#define PK_NORM_BWD_REG_MAX_NP 2
#endif
template <typename T, int NP>
static int bwd_reg(NormParams& p, void* const* dw, void* ws, size_t ws_bytes, cudaStream_t s) {
    if (p.np != NP || !p.vec || p.cols % ROW_VEC) return 1;
    const int64_t quads = p.cols / ROW_VEC;
    const int steps = quads <= 256 ? 1 : (quads <= 512 ? 2 : (quads <= 1024 ? 4 : 0));
    if (!steps || quads < 32) return 1;
    const int threads = static_cast<int>(round_up(ceil_div(quads, steps), 32));
    const bool weighted = p.w_np != 0 || dw != nullptr;
    const void* fn = nullptr;
    if (weighted)
        fn = steps == 1 ? reinterpret_cast<const void*>(rmsnorm_bwd_reg_kernel<T, NP, 1, true>)
             : steps == 2 ? reinterpret_cast<const void*>(rmsnorm_bwd_reg_kernel<T, NP, 2, true>)
                          : reinterpret_cast<const void*>(rmsnorm_bwd_reg_kernel<T, NP, 4, true>);
    else
        fn = steps == 1 ? reinterpret_cast<const void*>(rmsnorm_bwd_reg_kernel<T, NP, 1, false>)
             : steps == 2 ? reinterpret_cast<const void*>(rmsnorm_bwd_reg_kernel<T, NP, 2, false>)
                          : reinterpret_cast<const void*>(rmsnorm_bwd_reg_kernel<T, NP, 4, false>);
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, threads, 0) != cudaSuccess || per_sm < 1) return 1;
    // the weight-gradient partials take one [np][cols] slice per CTA of the workspace, which is
    // sized for at most 4 CTAs per SM
    const int64_t grid = std::min<int64_t>(p.rows, static_cast<int64_t>(num_sms()) * std::min(per_sm, 4));
    if (dw) {
        const size_t need = static_cast<size_t>(grid) * p.np * p.cols * sizeof(float);
        if (!ws || ws_bytes < need) return fail(PK_ERR_WORKSPACE, "pk_rmsnorm_bwd: workspace too small");
        p.dw_part = ws;
    }
    void* tok;
    prof_begin("rmsnorm_bwd", s, &tok);
    const int g = static_cast<int>(grid);
    if (weighted) {
        if (steps == 1) PK_LAUNCHED(rmsnorm_bwd_reg_kernel<T, NP, 1, true><<<g, threads, 0, s>>>(p));
        else if (steps == 2) PK_LAUNCHED(rmsnorm_bwd_reg_kernel<T, NP, 2, true><<<g, threads, 0, s>>>(p));
        else PK_LAUNCHED(rmsnorm_bwd_reg_kernel<T, NP, 4, true><<<g, threads, 0, s>>>(p));
    } else {
        if (steps == 1) PK_LAUNCHED(rmsnorm_bwd_reg_kernel<T, NP, 1, false><<<g, threads, 0, s>>>(p));
        else if (steps == 2) PK_LAUNCHED(rmsnorm_bwd_reg_kernel<T, NP, 2, false><<<g, threads, 0, s>>>(p));
        else PK_LAUNCHED(rmsnorm_bwd_reg_kernel<T, NP, 4, false><<<g, threads, 0, s>>>(p));
    }
    PK_CHECK_LAUNCH("pk_rmsnorm_bwd");
    if (dw) {
        const int st = reduce_dw<T, NP>(p, dw, g, s);
        if (st != PK_OK) return st;
    }
    prof_end("rmsnorm_bwd", s, tok);
    return PK_OK;
}

// Launch the streaming forward when two stages of a row fit in shared memory and the row fits
// 512 threads x STEPS x 4 columns (vector-aligned planes, float compute, degree <= 5).  Returns
// false when it does not apply.
template <typename T, int NP>
static bool stream_row_forward(const NormParams& p, cudaStream_t s) {
    using C = typename Compute<T>::type;
    if constexpr (sizeof(C) != 4 || NP > 6) {
        return false;
    } else {
        if (p.np != NP || !p.vec || p.cols % ROW_VEC) return false;
        const int64_t quads = p.cols / ROW_VEC;
        const int steps = quads <= 512 ? 1 : (quads <= 1024 ? 2 : 0);
        const size_t smem = 2 * static_cast<size_t>(NP) * p.cols * sizeof(T);
        if (!steps || quads < 64 || smem > 200 * 1024) return false;
        const int threads = static_cast<int>(round_up(ceil_div(quads, steps), 32));
        auto kern = steps == 1 ? rmsnorm_fwd_stream_kernel<T, NP, 1> : rmsnorm_fwd_stream_kernel<T, NP, 2>;
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
            cudaSuccess)
            return false;
        int per_sm = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem) != cudaSuccess || per_sm < 1)
            return false;
        const int grid = static_cast<int>(std::min<int64_t>(p.rows, static_cast<int64_t>(num_sms()) * per_sm));
        PK_LAUNCHED(kern<<<grid, threads, smem, s>>>(p));
        return true;
    }
}

template <typename T, int NP>
static bool reg_row_forward(const NormParams& p, cudaStream_t s) {
    using C = typename Compute<T>::type;
    if constexpr (sizeof(C) != 4 || NP > 6) {
        return false;
    } else {
        const int64_t quads = ceil_div(p.cols, ROW_VEC);
        int steps = 0;
        int64_t threads = 0;
        for (int st : {1, 2, 4}) {
            threads = round_up(ceil_div(quads, st), 32);
            if (threads <= 256 || (st == 4 && threads <= 512)) {
                steps = st;
                break;
            }
        }
        if (steps == 0) return false;
        int per_sm = 0;
        const void* fn = steps == 1 ? reinterpret_cast<const void*>(rmsnorm_fwd_reg_kernel<T, NP, 1>)
                         : steps == 2 ? reinterpret_cast<const void*>(rmsnorm_fwd_reg_kernel<T, NP, 2>)
                                      : reinterpret_cast<const void*>(rmsnorm_fwd_reg_kernel<T, NP, 4>);
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, static_cast<int>(threads), 0) != cudaSuccess ||
            per_sm < 1)
            return false;
        const int grid = static_cast<int>(std::min<int64_t>(p.rows, static_cast<int64_t>(num_sms()) * per_sm));
        const int th = static_cast<int>(threads);
        if (steps == 1) PK_LAUNCHED(rmsnorm_fwd_reg_kernel<T, NP, 1><<<grid, th, 0, s>>>(p));
        else if (steps == 2) PK_LAUNCHED(rmsnorm_fwd_reg_kernel<T, NP, 2><<<grid, th, 0, s>>>(p));
        else PK_LAUNCHED(rmsnorm_fwd_reg_kernel<T, NP, 4><<<grid, th, 0, s>>>(p));
        return true;
    }
}

template <typename T, int NP>
static int run_norm(bool backward, NormParams& p, void* const* dw, void* ws, size_t ws_bytes, cudaStream_t s) {
    using C = typename Compute<T>::type;
    {
        const int eb = static_cast<int>(sizeof(T));
        bool ok = p.cols % ROW_VEC == 0 && row_vec_ok(p.x, p.np, p.x_rs, eb) &&
                  row_vec_ok(reinterpret_cast<const void* const*>(p.y), p.np, p.y_rs, eb);
        if (backward) ok = ok && row_vec_ok(p.g, p.np, p.g_rs, eb);
        if (p.w_np) ok = ok && row_vec_ok(p.w, p.w_np, 0, eb);
        p.vec = ok ? 1 : 0;
    }
    const int threads = norm_threads(p.cols);
    if (!backward) {
        void* tok;
        prof_begin("rmsnorm_fwd", s, &tok);
        if (!(NP >= PK_NORM_FWD_STREAM_MIN_NP && stream_row_forward<T, NP>(p, s)) && !reg_row_forward<T, NP>(p, s)) {
            const int grid = static_cast<int>(std::min<int64_t>(p.rows, static_cast<int64_t>(num_sms()) * 8));
            PK_LAUNCHED(rmsnorm_fwd_kernel<T, NP><<<grid, threads, 0, s>>>(p));
        }
        prof_end("rmsnorm_fwd", s, tok);
        PK_CHECK_LAUNCH("pk_rmsnorm_fwd");
        return PK_OK;
    }
    if constexpr (sizeof(C) == 4 && NP <= PK_NORM_BWD_REG_MAX_NP) {
        const int st = bwd_reg<T, NP>(p, dw, ws, ws_bytes, s);
        if (st != 1) return st;
    }
    if constexpr (sizeof(C) == 4 && NP <= 6 && NP >= PK_NORM_BWD_STREAM_MIN_NP) {
        // next rows streamed into shared memory: half rows over 2-CTA clusters, quarter rows
        // over 4-CTA clusters for rows too long for a pair (a 4-CTA split of 4096-column rows
        // measured slower: 3.4 against 4.0 TB/s)
        int st = bwd_stream<T, NP, PK_NORM_BWD_CL>(p, dw, ws, ws_bytes, s);
        if (st == 1) st = bwd_stream<T, NP, 2>(p, dw, ws, ws_bytes, s);
        if (st == 1) st = bwd_stream<T, NP, 4>(p, dw, ws, ws_bytes, s);
        if (st != 1) return st;
    }
    const size_t smem = dw ? static_cast<size_t>(NP) * p.cols * sizeof(C) : 0;
    if (smem > 200 * 1024) return fail(PK_ERR_UNSUPPORTED, "pk_rmsnorm_bwd: row too long for the weight-gradient buffer");
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(rmsnorm_bwd_kernel<T, NP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        if (e != cudaSuccess) return cuda_fail(e, "pk_rmsnorm_bwd: cudaFuncSetAttribute");
    }
    // rows split over 2-CTA clusters with x and g in registers (vector-aligned planes, float compute)
    if constexpr (sizeof(C) == 4 && NP <= 5) {
        // pairs of CTAs (a 4-CTA split measured slower: its per-row cluster barrier costs more
        // than the extra occupancy gains); each CTA's half row fits 256 threads x STEPS x 4 columns
        constexpr int cl = 2;
        int steps = 0;
        int64_t cthreads = 0;
        if (p.vec && p.cols >= 512 && p.cols % (cl * ROW_VEC) == 0) {
            const int64_t quads = p.cols / cl / ROW_VEC;
            for (int st : {1, 2}) {
                cthreads = round_up(ceil_div(quads, st), 32);
                if (cthreads <= 256) {
                    steps = st;
                    break;
                }
            }
        }
        if (steps) {
            const size_t csmem = dw ? static_cast<size_t>(NP) * (p.cols / cl) * sizeof(C) : 0;
            auto kern = steps == 1 ? rmsnorm_bwd_cluster_kernel<T, NP, 1, cl> : rmsnorm_bwd_cluster_kernel<T, NP, 2, cl>;
            if (csmem > 48 * 1024) {
                cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                     static_cast<int>(csmem));
                if (e != cudaSuccess) return cuda_fail(e, "pk_rmsnorm_bwd: cudaFuncSetAttribute");
            }
            int per_sm = 0;
            cudaError_t e =
                cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, static_cast<int>(cthreads), csmem);
            if (e != cudaSuccess) return cuda_fail(e, "pk_rmsnorm_bwd: occupancy query");
            per_sm = std::max(1, std::min(per_sm, 4));
            const int64_t clusters = std::min<int64_t>(p.rows, static_cast<int64_t>(num_sms()) * per_sm / cl);
            if (dw) {
                const size_t need = static_cast<size_t>(clusters) * p.np * p.cols * sizeof(C);
                if (!ws || ws_bytes < need) return fail(PK_ERR_WORKSPACE, "pk_rmsnorm_bwd: workspace too small");
                p.dw_part = ws;
            }
            cudaLaunchConfig_t cfg{};
            cfg.gridDim = dim3(static_cast<unsigned>(cl * clusters));
            cfg.blockDim = dim3(static_cast<unsigned>(cthreads));
            cfg.dynamicSmemBytes = csmem;
            cfg.stream = s;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = static_cast<unsigned>(cl);
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            void* tok;
            prof_begin("rmsnorm_bwd", s, &tok);
            e = cudaLaunchKernelEx(&cfg, kern, p);
            if (e == cudaSuccess) ::pk::note_launch();
            if (e != cudaSuccess) return cuda_fail(e, "pk_rmsnorm_bwd: cluster launch");
            PK_CHECK_LAUNCH("pk_rmsnorm_bwd");
            if (dw) {
                NormParams q = p;
                for (int k = 0; k < p.np; ++k) q.g[k] = dw[k];
                const int64_t total = static_cast<int64_t>(p.np) * p.cols;
                PK_LAUNCHED(rmsnorm_dw_reduce_kernel<T, NP><<<static_cast<int>(ceil_div(total, 32)), 256, 0, s>>>(
                    q, static_cast<int>(clusters)));
                PK_CHECK_LAUNCH("pk_rmsnorm_bwd: weight reduction");
            }
            prof_end("rmsnorm_bwd", s, tok);
            return PK_OK;
        }
    }
    // as many CTAs as fit on the SMs at once (registers and the weight-gradient buffer decide)
    const int bthreads = std::min(threads, 256);
    int per_sm = 0;
    {
        cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, rmsnorm_bwd_kernel<T, NP>, bthreads, smem);
        if (e != cudaSuccess) return cuda_fail(e, "pk_rmsnorm_bwd: occupancy query");
        per_sm = std::max(1, std::min(per_sm, 4));
    }
    int grid = static_cast<int>(std::min<int64_t>(p.rows, static_cast<int64_t>(num_sms()) * per_sm));
    if (dw) {
        const size_t need = static_cast<size_t>(grid) * p.np * p.cols * sizeof(C);
        if (!ws || ws_bytes < need) return fail(PK_ERR_WORKSPACE, "pk_rmsnorm_bwd: workspace too small");
        p.dw_part = ws;
    }
    void* tok;
    prof_begin("rmsnorm_bwd", s, &tok);
    PK_LAUNCHED(rmsnorm_bwd_kernel<T, NP><<<grid, bthreads, smem, s>>>(p));
    PK_CHECK_LAUNCH("pk_rmsnorm_bwd");
    if (dw) {
        NormParams q = p;
        for (int k = 0; k < p.np; ++k) q.g[k] = dw[k];
        const int64_t total = static_cast<int64_t>(p.np) * p.cols;
        PK_LAUNCHED(rmsnorm_dw_reduce_kernel<T, NP><<<static_cast<int>(ceil_div(total, 32)), 256, 0, s>>>(q, grid));
        PK_CHECK_LAUNCH("pk_rmsnorm_bwd: weight reduction");
    }
    prof_end("rmsnorm_bwd", s, tok);
    return PK_OK;
}

template <typename T>
static int run_norm_np(bool bwd, NormParams& p, void* const* dw, void* ws, size_t wsb, cudaStream_t s) {
    switch (p.np) {
        case 1: return run_norm<T, 1>(bwd, p, dw, ws, wsb, s);
        case 2: return run_norm<T, 2>(bwd, p, dw, ws, wsb, s);
        case 3: return run_norm<T, 3>(bwd, p, dw, ws, wsb, s);
        case 4: return run_norm<T, 4>(bwd, p, dw, ws, wsb, s);
        case 5: return run_norm<T, 5>(bwd, p, dw, ws, wsb, s);
        case 6: return run_norm<T, 6>(bwd, p, dw, ws, wsb, s);
        case 7: case 8: case 9: return run_norm<T, 9>(bwd, p, dw, ws, wsb, s);
        default: return run_norm<T, 16>(bwd, p, dw, ws, wsb, s);
    }
}

static int compute_size(int dtype) { return dtype == PK_F64 ? 8 : 4; }

}  // namespace pk

using namespace pk;

extern "C" {

size_t pk_rmsnorm_bwd_workspace_size(int dtype, int degree, int64_t rows, int64_t cols) {
    if (degree < 0 || degree >= PK_MAX_PLANES || rows < 0 || cols < 0) return 0;
    const int64_t grid = std::min<int64_t>(rows, static_cast<int64_t>(num_sms()) * 4);
    return static_cast<size_t>(std::max<int64_t>(grid, 1) * (degree + 1) * cols * compute_size(dtype)) + 256;
}

int pk_rmsnorm_fwd(int dtype, int degree, int64_t rows, int64_t cols, const void* const* x, int64_t x_rs,
                   const void* const* w, int w_planes, double eps, void* const* y, int64_t y_rs, void* rstd,
                   void* stream) {
    if (degree < 0 || degree >= PK_MAX_PLANES) return fail(PK_ERR_UNSUPPORTED, "pk_rmsnorm_fwd: degree out of range");
    if (rows < 0 || cols <= 0) return fail(PK_ERR_ARG, "pk_rmsnorm_fwd: bad shape");
    NormParams p{};
    p.np = degree + 1;
    p.rows = rows;
    p.cols = cols;
    p.x_rs = x_rs;
    p.y_rs = y_rs;
    p.eps = eps;
    p.w_np = w ? w_planes : 0;
    if (w && w_planes != 1 && w_planes != p.np) return fail(PK_ERR_ARG, "pk_rmsnorm_fwd: w_planes must be 1 or degree+1");
    p.rstd = rstd;
    for (int k = 0; k < p.np; ++k) {
        p.x[k] = x[k];
        p.y[k] = y[k];
    }
    for (int k = 0; k < p.w_np; ++k) p.w[k] = w[k];
    if (rows == 0) return PK_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    switch (dtype) {
        case PK_F32: return run_norm_np<float>(false, p, nullptr, nullptr, 0, s);
        case PK_F64: return run_norm_np<double>(false, p, nullptr, nullptr, 0, s);
        case PK_BF16: return run_norm_np<__nv_bfloat16>(false, p, nullptr, nullptr, 0, s);
        case PK_F16: return run_norm_np<__half>(false, p, nullptr, nullptr, 0, s);
    }
    return fail(PK_ERR_UNSUPPORTED, "pk_rmsnorm_fwd: unsupported dtype");
}

int pk_rmsnorm_bwd(int dtype, int degree, int64_t rows, int64_t cols, const void* const* x, int64_t x_rs,
                   const void* const* w, int w_planes, const void* const* g, int64_t g_rs, const void* rstd,
                   void* const* dx, int64_t dx_rs, void* const* dw, void* workspace, size_t workspace_bytes,
                   void* stream) {
    if (degree < 0 || degree >= PK_MAX_PLANES) return fail(PK_ERR_UNSUPPORTED, "pk_rmsnorm_bwd: degree out of range");
    if (rows < 0 || cols <= 0 || !rstd) return fail(PK_ERR_ARG, "pk_rmsnorm_bwd: bad arguments");
    NormParams p{};
    p.np = degree + 1;
    p.rows = rows;
    p.cols = cols;
    p.x_rs = x_rs;
    p.g_rs = g_rs;
    p.y_rs = dx_rs;
    p.w_np = w ? w_planes : 0;
    if (w && w_planes != 1 && w_planes != p.np) return fail(PK_ERR_ARG, "pk_rmsnorm_bwd: w_planes must be 1 or degree+1");
    p.rstd = const_cast<void*>(rstd);
    p.status = device_status_ptr();
    for (int k = 0; k < p.np; ++k) {
        p.x[k] = x[k];
        p.g[k] = g[k];
        p.y[k] = dx[k];
    }
    for (int k = 0; k < p.w_np; ++k) p.w[k] = w[k];
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (rows == 0) {
        if (dw) {
            const size_t esz = dtype == PK_F64 ? 8 : (dtype == PK_F32 ? 4 : 2);
            for (int k = 0; k < p.np; ++k) {
                cudaError_t e = cudaMemsetAsync(dw[k], 0, cols * esz, s);
                if (e != cudaSuccess) return cuda_fail(e, "pk_rmsnorm_bwd: memset");
            }
        }
        return PK_OK;
    }
    void* ws = workspace ? reinterpret_cast<void*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255))
                         : nullptr;
    const size_t wsb = workspace ? workspace_bytes - (static_cast<char*>(ws) - static_cast<char*>(workspace)) : 0;
    switch (dtype) {
        case PK_F32: return run_norm_np<float>(true, p, dw, ws, wsb, s);
        case PK_F64: return run_norm_np<double>(true, p, dw, ws, wsb, s);
        case PK_BF16: return run_norm_np<__nv_bfloat16>(true, p, dw, ws, wsb, s);
        case PK_F16: return run_norm_np<__half>(true, p, dw, ws, wsb, s);
    }
    return fail(PK_ERR_UNSUPPORTED, "pk_rmsnorm_bwd: unsupported dtype");
}

}  // extern "C"
