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
#pragma unroll
                    for (int k = 0; k < NP; ++k) dwp[k * p.cols + c0 + u] += gx[k];
                }
            }
            store_planes4<NP, T, C>(p.y, p.np, yb + c0, valid, p.vec != 0, out);
        }
    }
    if (want_dw) {
        __syncthreads();
        C* out = static_cast<C*>(p.dw_part) + static_cast<int64_t>(blockIdx.x) * p.np * p.cols;
        for (int64_t i = threadIdx.x; i < static_cast<int64_t>(p.np) * p.cols; i += blockDim.x) out[i] = dwp[i];
    }
}

// dw[k][c] = sum_b part[b][k][c]
template <typename T, int NP>
__global__ void rmsnorm_dw_reduce_kernel(const NormParams p, int parts, void* const* dw_planes_unused) {
    using C = typename Compute<T>::type;
    const int64_t total = static_cast<int64_t>(p.np) * p.cols;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        C s = C(0);
        for (int b = 0; b < parts; ++b) s += static_cast<const C*>(p.dw_part)[static_cast<int64_t>(b) * total + i];
        const int k = static_cast<int>(i / p.cols);
        static_cast<T*>(const_cast<void*>(p.g[k]))[i % p.cols] = from_c<T>(s);
    }
}

static int norm_threads(int64_t cols) { return cols >= 2048 ? 512 : (cols >= 512 ? 256 : 128); }

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
        const int grid = static_cast<int>(std::min<int64_t>(p.rows, static_cast<int64_t>(num_sms()) * 8));
        void* tok;
        prof_begin("rmsnorm_fwd", s, &tok);
        rmsnorm_fwd_kernel<T, NP><<<grid, threads, 0, s>>>(p);
        prof_end("rmsnorm_fwd", s, tok);
        PK_CHECK_LAUNCH("pk_rmsnorm_fwd");
        return PK_OK;
    }
    const size_t smem = dw ? static_cast<size_t>(NP) * p.cols * sizeof(C) : 0;
    if (smem > 200 * 1024) return fail(PK_ERR_UNSUPPORTED, "pk_rmsnorm_bwd: row too long for the weight-gradient buffer");
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(rmsnorm_bwd_kernel<T, NP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        if (e != cudaSuccess) return cuda_fail(e, "pk_rmsnorm_bwd: cudaFuncSetAttribute");
    }
    int per_sm = 4;
    if (smem > 0) per_sm = static_cast<int>(std::max<size_t>(1, std::min<size_t>(4, (220 * 1024) / (smem + 4096))));
    int grid = static_cast<int>(std::min<int64_t>(p.rows, static_cast<int64_t>(num_sms()) * per_sm));
    if (dw) {
        const size_t need = static_cast<size_t>(grid) * p.np * p.cols * sizeof(C);
        if (!ws || ws_bytes < need) return fail(PK_ERR_WORKSPACE, "pk_rmsnorm_bwd: workspace too small");
        p.dw_part = ws;
    }
    void* tok;
    prof_begin("rmsnorm_bwd", s, &tok);
    rmsnorm_bwd_kernel<T, NP><<<grid, threads, smem, s>>>(p);
    prof_end("rmsnorm_bwd", s, tok);
    PK_CHECK_LAUNCH("pk_rmsnorm_bwd");
    if (dw) {
        NormParams q = p;
        for (int k = 0; k < p.np; ++k) q.g[k] = dw[k];
        const int64_t total = static_cast<int64_t>(p.np) * p.cols;
        const int g2 = static_cast<int>(std::min<int64_t>(ceil_div(total, 256), 4096));
        rmsnorm_dw_reduce_kernel<T, NP><<<g2, 256, 0, s>>>(q, grid, nullptr);
        PK_CHECK_LAUNCH("pk_rmsnorm_bwd: weight reduction");
    }
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
