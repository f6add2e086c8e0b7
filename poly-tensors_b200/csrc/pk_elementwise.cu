// Elementwise series operations, reductions and row gathers over coefficient planes.
//
// One launch evaluates an operation for every coefficient plane at once (each thread
// holds the n+1 coefficients of its element in registers), instead of the reference's
// O(n^2) Python loop of full-size ATen launches per operation:
//   Cauchy product / quotient   src/polytensors/_range_ops.py:133-149, :86-93, _plain.py:118-128
//   constant fast path          src/polytensors/_range_ops.py:109-132
//   exp / log / sqrt / rsqrt    src/polytensors/_plain.py:153-171, _series.py:72-96
//   tanh / sigmoid / GELU       src/polytensors/_plain.py:256-259, :283-325
//   sum / mean                  src/polytensors/_range_ops.py:178-193
//   embedding (+ backward)      src/polytensors/_dispatch.py:530-532, :683-685
//   SGD add_(alpha)             src/polytensors/_range_ops.py:95-103, :133-149
#include <algorithm>

#include "pk_common.cuh"
#include "pk_rows.cuh"
#include "pk_series.cuh"
#include "pk_complex.cuh"

namespace pk {

constexpr int MAP_MAX_DIMS = 6;

struct MapParams {
    int op, np;
    int ndim;
    int contig;
    int a_np, b_np;
    int64_t numel;
    int64_t shape[MAP_MAX_DIMS];
    int64_t so[MAP_MAX_DIMS], sa[MAP_MAX_DIMS], sb[MAP_MAX_DIMS];
    double p0, p1;
    void* out[PK_MAX_PLANES];
    const void* a[PK_MAX_PLANES];
    const void* b[PK_MAX_PLANES];
};

// y = op(a, b) for one element's series (the operation table of pk_series_map).
template <int NP, typename C>
__device__ __forceinline__ void apply_op(const MapParams& p, const C (&a)[NP], const C (&b)[NP], C (&y)[NP]) {
    switch (p.op) {
        case PK_OP_COPY:
#pragma unroll
            for (int k = 0; k < NP; ++k) y[k] = a[k];
            break;
        case PK_OP_AFFINE:
#pragma unroll
            for (int k = 0; k < NP; ++k) y[k] = C(p.p0) * a[k];
            y[0] += C(p.p1);
            break;
        case PK_OP_EXP: s_exp<NP, C>(a, y); break;
        case PK_OP_LOG: s_log<NP, C>(a, y); break;
        case PK_OP_SQRT: s_sqrt<NP, C>(a, y); break;
        case PK_OP_RSQRT: s_rsqrt<NP, C>(a, y); break;
        case PK_OP_RECIPROCAL: {
            C one[NP];
#pragma unroll
            for (int k = 0; k < NP; ++k) one[k] = C(k == 0 ? 1 : 0);
            s_div<NP, C>(one, a, y);
            break;
        }
        case PK_OP_TANH: { C g[NP]; s_tanh<NP, C>(a, y, g); break; }
        case PK_OP_SIGMOID: { C g[NP]; s_sigmoid<NP, C>(a, y, g); break; }
        case PK_OP_GELU: { C d[NP]; s_gelu<NP, C>(a, y, d); break; }
        case PK_OP_POWI: {
            // repeated multiplication, as the reference's integer-power rule
            // (src/polytensors/_dispatch.py:419-429); x^2 is one Cauchy product (_plain.py:291-293)
            const int n = static_cast<int>(p.p0);
#pragma unroll
            for (int k = 0; k < NP; ++k) y[k] = C(k == 0 ? 1 : 0);
            for (int r = 0; r < n; ++r) s_mul<NP, C>(y, a, y);
            break;
        }
        case PK_OP_ADD:
#pragma unroll
            for (int k = 0; k < NP; ++k) y[k] = a[k] + C(p.p0) * b[k];
            break;
        case PK_OP_MUL: s_mul<NP, C>(a, b, y); break;
        case PK_OP_DIV: s_div<NP, C>(a, b, y); break;
        case PK_OP_GELU_BWD: {  // a = incoming gradient series, b = GELU input
            C v[NP], d[NP];
            s_gelu<NP, C>(b, v, d);
            s_mul<NP, C>(a, d, y);
            break;
        }
        case PK_OP_TANH_BWD: {  // a = gradient, b = tanh output: G (1 - Y^2)
            C sq[NP];
            s_mul<NP, C>(b, b, sq);
#pragma unroll
            for (int k = 0; k < NP; ++k) sq[k] = (k == 0 ? C(1) : C(0)) - sq[k];
            s_mul<NP, C>(a, sq, y);
            break;
        }
        case PK_OP_SIGMOID_BWD: {  // a = gradient, b = sigmoid output: G Y (1 - Y)
            C om[NP], t[NP];
#pragma unroll
            for (int k = 0; k < NP; ++k) om[k] = (k == 0 ? C(1) : C(0)) - b[k];
            s_mul<NP, C>(b, om, t);
            s_mul<NP, C>(a, t, y);
            break;
        }
        default:
#pragma unroll
            for (int k = 0; k < NP; ++k) y[k] = C(0);
    }
}

template <typename T, int NP>
__global__ void __launch_bounds__(256) series_map_kernel(const MapParams p) {
    using C = typename Compute<T>::type;
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
        C a[NP], b[NP], y[NP];
#pragma unroll
        for (int k = 0; k < NP; ++k) {
            a[k] = (k < p.a_np && k < p.np) ? to_c<C>(static_cast<const T*>(p.a[k])[oa]) : C(0);
            b[k] = (p.b[0] != nullptr && k < p.b_np && k < p.np) ? to_c<C>(static_cast<const T*>(p.b[k])[ob]) : C(0);
        }
        apply_op<NP, C>(p, a, b, y);
#pragma unroll
        for (int k = 0; k < NP; ++k)
            if (k < p.np) static_cast<T*>(p.out[k])[oo] = from_c<T>(y[k]);
    }
}

// Dense operands with vector-aligned planes: Q groups of four consecutive elements per thread and
// step (the groups of a warp lie 512 elements apart, so each load instruction of a warp covers
// whole lines), every group's loads issued before any arithmetic, one 8-32 byte access per plane
// (partial groups element by element).  Measured at 16384 x 4096 float32 (GELU forward and
// backward plus a series product, through the API): one group per thread and one block per 1024
// elements (no grid-stride loop) ran at 6.47 / 6.57 TB/s at degree 1 / 4, against 5.8 / 6.2 with
// the grid capped at 16 blocks per SM, and two groups per thread did not help.
#ifndef PK_MAP_QUADS
#define PK_MAP_QUADS 1
#endif
#ifndef PK_MAP_BLOCKS_PER_SM
#define PK_MAP_BLOCKS_PER_SM 0
#endif
template <typename T, int NP, int Q>
__global__ void __launch_bounds__(256) series_map_vec_kernel(const MapParams p) {
    using C = typename Compute<T>::type;
    const int64_t chunk = static_cast<int64_t>(blockDim.x) * ROW_VEC;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * chunk * Q;
    const int a_np = min(p.a_np, p.np);
    const int b_np = p.b[0] != nullptr ? min(p.b_np, p.np) : 0;
    for (int64_t base = static_cast<int64_t>(blockIdx.x) * chunk * Q + static_cast<int64_t>(threadIdx.x) * ROW_VEC;
         base < p.numel; base += stride) {
        C a[Q][ROW_VEC][NP], b[Q][ROW_VEC][NP];
        int valid[Q];
#pragma unroll
        for (int q = 0; q < Q; ++q) {
            const int64_t off = base + q * chunk;
            valid[q] = off < p.numel ? vec_count(p.numel, off) : 0;
            load_planes4<NP, T, C>(p.a, a_np, off, valid[q], true, a[q]);
            load_planes4<NP, T, C>(p.b, b_np, off, valid[q], true, b[q]);
        }
#pragma unroll
        for (int q = 0; q < Q; ++q) {
            if (valid[q] <= 0) continue;
            C y[ROW_VEC][NP];
#pragma unroll
            for (int u = 0; u < ROW_VEC; ++u) apply_op<NP, C>(p, a[q][u], b[q][u], y[u]);
            store_planes4<NP, T, C>(p.out, p.np, base + q * chunk, valid[q], true, y);
        }
    }
}

template <typename T, int NP>
static void launch_map_np(const MapParams& p, int grid, bool vec, cudaStream_t s) {
    if (vec) {
        // two groups per thread for short series (more bytes in flight per thread at little
        // register cost), one for longer ones
        constexpr int Q = NP <= 3 ? PK_MAP_QUADS : 1;
        const int64_t blocks = ceil_div(p.numel, 256 * ROW_VEC * Q);
        const int64_t cap = PK_MAP_BLOCKS_PER_SM > 0 ? static_cast<int64_t>(num_sms()) * PK_MAP_BLOCKS_PER_SM : blocks;
        const int g = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(blocks, cap)));
        PK_LAUNCHED(series_map_vec_kernel<T, NP, Q><<<g, 256, 0, s>>>(p));
    } else {
        PK_LAUNCHED(series_map_kernel<T, NP><<<grid, 256, 0, s>>>(p));
    }
}

// Series with complex planes (a real base with complex directions, or complex throughout):
// planes flagged in a mask hold interleaved (re, im) pairs of R, the others plain R values; the
// arithmetic runs in cplx<R> through the same operation table.  Strides count elements (a
// complex element is one element).  Element by element with strided indexing: the complex forms
// serve API completeness, not the configs' hot loops.
template <typename R>
__device__ __forceinline__ cplx<R> load_cplx(const void* plane, int64_t off, bool is_complex) {
    if (is_complex) {
        const R* q = static_cast<const R*>(plane) + 2 * off;
        return cplx<R>(q[0], q[1]);
    }
    return cplx<R>(static_cast<const R*>(plane)[off], R(0));
}

template <typename R, int NP>
__global__ void __launch_bounds__(256) series_map_cplx_kernel(const MapParams p, uint32_t a_cm, uint32_t b_cm,
                                                                uint32_t o_cm) {
    using C = cplx<R>;
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
        C a[NP], b[NP], y[NP];
#pragma unroll
        for (int k = 0; k < NP; ++k) {
            a[k] = (k < p.a_np && k < p.np) ? load_cplx<R>(p.a[k], oa, (a_cm >> k) & 1u) : C(0);
            b[k] = (p.b[0] != nullptr && k < p.b_np && k < p.np) ? load_cplx<R>(p.b[k], ob, (b_cm >> k) & 1u) : C(0);
        }
        apply_op<NP, C>(p, a, b, y);
#pragma unroll
        for (int k = 0; k < NP; ++k) {
            if (k >= p.np) continue;
            if ((o_cm >> k) & 1u) {
                R* q = static_cast<R*>(p.out[k]) + 2 * oo;
                q[0] = y[k].re;
                q[1] = y[k].im;
            } else {
                static_cast<R*>(p.out[k])[oo] = y[k].re;
            }
        }
    }
}

template <typename R>
static void launch_map_cplx(const MapParams& p, int grid, uint32_t a_cm, uint32_t b_cm, uint32_t o_cm,
                            cudaStream_t s) {
    switch (p.np) {
        case 1: PK_LAUNCHED(series_map_cplx_kernel<R, 1><<<grid, 256, 0, s>>>(p, a_cm, b_cm, o_cm)); break;
        case 2: PK_LAUNCHED(series_map_cplx_kernel<R, 2><<<grid, 256, 0, s>>>(p, a_cm, b_cm, o_cm)); break;
        case 3: PK_LAUNCHED(series_map_cplx_kernel<R, 3><<<grid, 256, 0, s>>>(p, a_cm, b_cm, o_cm)); break;
        case 4: PK_LAUNCHED(series_map_cplx_kernel<R, 4><<<grid, 256, 0, s>>>(p, a_cm, b_cm, o_cm)); break;
        case 5: case 6: PK_LAUNCHED(series_map_cplx_kernel<R, 6><<<grid, 256, 0, s>>>(p, a_cm, b_cm, o_cm)); break;
        case 7: case 8: case 9: PK_LAUNCHED(series_map_cplx_kernel<R, 9><<<grid, 256, 0, s>>>(p, a_cm, b_cm, o_cm)); break;
        default: PK_LAUNCHED(series_map_cplx_kernel<R, 16><<<grid, 256, 0, s>>>(p, a_cm, b_cm, o_cm)); break;
    }
}

template <typename T>
static void launch_map_t(const MapParams& p, int grid, bool vec, cudaStream_t s) {
    switch (p.np) {
        case 1: launch_map_np<T, 1>(p, grid, vec, s); break;
        case 2: launch_map_np<T, 2>(p, grid, vec, s); break;
        case 3: launch_map_np<T, 3>(p, grid, vec, s); break;
        case 4: launch_map_np<T, 4>(p, grid, vec, s); break;
        case 5: launch_map_np<T, 5>(p, grid, vec, s); break;
        case 6: launch_map_np<T, 6>(p, grid, vec, s); break;
        case 7: case 8: case 9: launch_map_np<T, 9>(p, grid, vec, s); break;
        default: launch_map_np<T, 16>(p, grid, vec, s); break;
    }
}

static bool is_binary(int op) { return op >= PK_OP_ADD; }

static bool dense(int ndim, const int64_t* shape, const int64_t* st) {
    int64_t expect = 1;
    for (int d = ndim - 1; d >= 0; --d) {
        if (shape[d] != 1 && st[d] != expect) return false;
        expect *= shape[d];
    }
    return true;
}

// ---------------------------------------------------------------------------------
// Reductions: out[o, i] = scale * sum_r x[o, r, i]  (x, out contiguous)

struct ReduceParams {
    int np;
    int64_t outer, red, inner;
    int64_t red_chunk;
    double scale;
    const void* x[PK_MAX_PLANES];
    void* out[PK_MAX_PLANES];
};

template <typename T, int NP>
__global__ void __launch_bounds__(256) reduce_rows_kernel(const ReduceParams p) {
    using C = typename Compute<T>::type;
    using A = typename std::conditional<sizeof(C) == 8, double, float>::type;
    __shared__ A partial[8][NP];
    for (int64_t o = blockIdx.x; o < p.outer; o += gridDim.x) {
        A acc[NP];
#pragma unroll
        for (int k = 0; k < NP; ++k) acc[k] = A(0);
        const int64_t base = o * p.red;
        for (int64_t r = threadIdx.x; r < p.red; r += blockDim.x) {
#pragma unroll
            for (int k = 0; k < NP; ++k)
                if (k < p.np) acc[k] += to_c<C>(static_cast<const T*>(p.x[k])[base + r]);
        }
#pragma unroll
        for (int k = 0; k < NP; ++k) {
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) acc[k] += __shfl_xor_sync(0xffffffffu, acc[k], off);
        }
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
        if (lane == 0) {
#pragma unroll
            for (int k = 0; k < NP; ++k) partial[warp][k] = acc[k];
        }
        __syncthreads();
        if (threadIdx.x < NP && threadIdx.x < p.np) {
            A s = A(0);
            for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) s += partial[w][threadIdx.x];
            static_cast<T*>(p.out[threadIdx.x])[o] = from_c<T>(static_cast<C>(s * A(p.scale)));
        }
        __syncthreads();
    }
}

// Column reduction; blockIdx.y splits the reduced axis into chunks combined with atomics
// (the output is zeroed first) when there are too few columns to fill the GPU.
template <typename T, int NP>
__global__ void __launch_bounds__(256) reduce_cols_kernel(const ReduceParams p, int atomic) {
    using C = typename Compute<T>::type;
    const int64_t cols = p.outer * p.inner;
    const int64_t r0 = static_cast<int64_t>(blockIdx.y) * p.red_chunk;
    const int64_t r1 = min(p.red, r0 + p.red_chunk);
    for (int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; c < cols;
         c += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t o = c / p.inner, i = c % p.inner;
        C acc[NP];
#pragma unroll
        for (int k = 0; k < NP; ++k) acc[k] = C(0);
        for (int64_t r = r0; r < r1; ++r) {
            const int64_t off = (o * p.red + r) * p.inner + i;
#pragma unroll
            for (int k = 0; k < NP; ++k)
                if (k < p.np) acc[k] += to_c<C>(static_cast<const T*>(p.x[k])[off]);
        }
#pragma unroll
        for (int k = 0; k < NP; ++k) {
            if (k >= p.np) continue;
            const C v = acc[k] * C(p.scale);
            if (atomic) atomicAdd(static_cast<C*>(p.out[k]) + c, v);
            else static_cast<T*>(p.out[k])[c] = from_c<T>(v);
        }
    }
}

// ---------------------------------------------------------------------------------
// Row gather / scatter-add (embedding forward / backward)

struct RowParams {
    int np;
    int64_t n_idx, dim, n_rows;
    int64_t src_rs;  // row stride of the source planes
    int64_t padding_idx;
    const int64_t* idx;
    const void* src[PK_MAX_PLANES];
    void* dst[PK_MAX_PLANES];
    int* status;
};

template <typename T>
__global__ void gather_rows_kernel(const RowParams p) {
    const int64_t total = p.n_idx * p.dim;
    for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
         e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t i = e / p.dim, c = e % p.dim;
        const int64_t row = p.idx[i];
        const bool ok = row >= 0 && row < p.n_rows;
        if (!ok) pk_record_status(p.status, 201);
        for (int k = 0; k < p.np; ++k)
            static_cast<T*>(p.dst[k])[e] = ok ? static_cast<const T*>(p.src[k])[row * p.src_rs + c] : T(0);
    }
}

template <typename T>
__global__ void scatter_add_rows_kernel(const RowParams p) {
    const int64_t total = p.n_idx * p.dim;
    for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
         e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t i = e / p.dim, c = e % p.dim;
        const int64_t row = p.idx[i];
        if (row == p.padding_idx) continue;
        if (row < 0 || row >= p.n_rows) {
            pk_record_status(p.status, 202);
            continue;
        }
        for (int k = 0; k < p.np; ++k)
            atomicAdd(static_cast<T*>(p.dst[k]) + row * p.dim + c, static_cast<const T*>(p.src[k])[i * p.src_rs + c]);
    }
}

template <typename T, int NP>
static void launch_reduce(const ReduceParams& p, bool rows, int atomic, dim3 grid, cudaStream_t s) {
    if (rows) PK_LAUNCHED(reduce_rows_kernel<T, NP><<<grid, 256, 0, s>>>(p));
    else PK_LAUNCHED(reduce_cols_kernel<T, NP><<<grid, 256, 0, s>>>(p, atomic));
}

template <typename T>
static void launch_reduce_np(const ReduceParams& p, bool rows, int atomic, dim3 grid, cudaStream_t s) {
    switch (p.np) {
        case 1: launch_reduce<T, 1>(p, rows, atomic, grid, s); break;
        case 2: launch_reduce<T, 2>(p, rows, atomic, grid, s); break;
        case 3: launch_reduce<T, 3>(p, rows, atomic, grid, s); break;
        case 4: launch_reduce<T, 4>(p, rows, atomic, grid, s); break;
        case 5: launch_reduce<T, 5>(p, rows, atomic, grid, s); break;
        case 6: launch_reduce<T, 6>(p, rows, atomic, grid, s); break;
        case 7: case 8: case 9: launch_reduce<T, 9>(p, rows, atomic, grid, s); break;
        default: launch_reduce<T, 16>(p, rows, atomic, grid, s); break;
    }
}

static int grid_for(int64_t work, int per_block = 256) {
    const int64_t blocks = ceil_div(std::max<int64_t>(work, 1), per_block);
    return static_cast<int>(std::min<int64_t>(blocks, static_cast<int64_t>(num_sms()) * 16));
}

// float32 planes -> bf16 hi/lo pairs (hi = bf16(x), lo = bf16(x - hi)), the operand form of the
// float32 tensor-core products: one read of x and one write of each pair, four elements per
// thread and step; blockIdx.y selects the plane.
struct SplitParams {
    int64_t numel;
    const float* x[PK_MAX_PLANES];
    __nv_bfloat16* out[2 * PK_MAX_PLANES];
    int vec;
};

__global__ void __launch_bounds__(256) split_hilo_kernel(const SplitParams p) {
    const int k = blockIdx.y;
    const float* x = p.x[k];
    __nv_bfloat16* hi = p.out[2 * k];
    __nv_bfloat16* lo = p.out[2 * k + 1];
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x * ROW_VEC;
    for (int64_t off = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * ROW_VEC; off < p.numel;
         off += stride) {
        const int valid = vec_count(p.numel, off);
        float v[4] = {0.f, 0.f, 0.f, 0.f}, h[4], l[4];
        if (p.vec && valid == ROW_VEC) load_vec4<float>(x + off, v);
        else
            for (int u = 0; u < valid; ++u) v[u] = x[off + u];
#pragma unroll
        for (int u = 0; u < ROW_VEC; ++u) {
            h[u] = __bfloat162float(__float2bfloat16_rn(v[u]));
            l[u] = v[u] - h[u];
        }
        if (p.vec && valid == ROW_VEC) {
            store_vec4<__nv_bfloat16>(hi + off, h);
            store_vec4<__nv_bfloat16>(lo + off, l);
        } else {
            for (int u = 0; u < valid; ++u) {
                hi[off + u] = __float2bfloat16_rn(h[u]);
                lo[off + u] = __float2bfloat16_rn(l[u]);
            }
        }
    }
}

// Validated parameters of one pk_series_map / pk_series_map_complex call (p.numel == 0: nothing to do).
static int fill_map_params(MapParams& p, const char* what, int op, int degree, int ndim, const int64_t* shape,
                           void* const* out, const int64_t* out_strides, const void* const* a, int a_planes,
                           const int64_t* a_strides, const void* const* b, int b_planes, const int64_t* b_strides,
                           double p0, double p1) {
    const std::string w(what);
    if (degree < 0 || degree >= PK_MAX_PLANES) return fail(PK_ERR_UNSUPPORTED, w + ": degree out of range");
    if (ndim < 0 || ndim > MAP_MAX_DIMS) return fail(PK_ERR_UNSUPPORTED, w + ": more than 6 dimensions");
    const int np = degree + 1;
    const bool binary = is_binary(op);
    if (op < 0 || op > PK_OP_SIGMOID_BWD || (op > PK_OP_POWI && op < PK_OP_ADD))
        return fail(PK_ERR_ARG, w + ": unknown op " + std::to_string(op));
    if (!out || !a || (binary && !b)) return fail(PK_ERR_ARG, w + ": null plane array");
    if (a_planes != 1 && a_planes != np) return fail(PK_ERR_ARG, w + ": a_planes must be 1 or degree+1");
    if (binary && b_planes != 1 && b_planes != np) return fail(PK_ERR_ARG, w + ": b_planes must be 1 or degree+1");
    p.op = op;
    p.np = np;
    p.ndim = ndim;
    p.a_np = a_planes;
    p.b_np = binary ? b_planes : 0;
    p.p0 = p0;
    p.p1 = p1;
    p.numel = 1;
    for (int d = 0; d < ndim; ++d) {
        if (shape[d] < 0) return fail(PK_ERR_ARG, w + ": negative extent");
        p.numel *= shape[d];
        p.shape[d] = shape[d];
        p.so[d] = out_strides[d];
        p.sa[d] = a_strides[d];
        p.sb[d] = binary ? b_strides[d] : 0;
    }
    if (p.numel == 0) return PK_OK;
    for (int k = 0; k < np; ++k) {
        if (!out[k]) return fail(PK_ERR_ARG, w + ": null output plane");
        p.out[k] = out[k];
    }
    for (int k = 0; k < a_planes; ++k) {
        if (!a[k]) return fail(PK_ERR_ARG, w + ": null input plane");
        p.a[k] = a[k];
    }
    if (binary) {
        for (int k = 0; k < b_planes; ++k) {
            if (!b[k]) return fail(PK_ERR_ARG, w + ": null input plane");
            p.b[k] = b[k];
        }
    }
    p.contig = dense(ndim, shape, out_strides) && dense(ndim, shape, a_strides) &&
               (!binary || dense(ndim, shape, b_strides));
    return PK_OK;
}

}  // namespace pk

using namespace pk;

extern "C" {

int pk_split_hilo(int degree, int64_t numel, const void* const* x, void* const* out, void* stream) {
    if (degree < 0 || degree >= PK_MAX_PLANES) return fail(PK_ERR_UNSUPPORTED, "pk_split_hilo: degree out of range");
    if (numel < 0 || !x || !out) return fail(PK_ERR_ARG, "pk_split_hilo: bad arguments");
    if (numel == 0) return PK_OK;
    SplitParams p{};
    p.numel = numel;
    bool vec = true;
    for (int k = 0; k <= degree; ++k) {
        p.x[k] = static_cast<const float*>(x[k]);
        p.out[2 * k] = static_cast<__nv_bfloat16*>(out[2 * k]);
        p.out[2 * k + 1] = static_cast<__nv_bfloat16*>(out[2 * k + 1]);
        if (!p.x[k] || !p.out[2 * k] || !p.out[2 * k + 1]) return fail(PK_ERR_ARG, "pk_split_hilo: null plane");
        vec = vec && reinterpret_cast<uintptr_t>(p.x[k]) % 16 == 0 && reinterpret_cast<uintptr_t>(p.out[2 * k]) % 8 == 0 &&
              reinterpret_cast<uintptr_t>(p.out[2 * k + 1]) % 8 == 0;
    }
    p.vec = vec ? 1 : 0;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int64_t blocks = ceil_div(numel, 256 * ROW_VEC);
    const int gx = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(blocks, 0x7fffffff)));
    void* tok;
    prof_begin("split_hilo", s, &tok);
    PK_LAUNCHED(split_hilo_kernel<<<dim3(gx, degree + 1), 256, 0, s>>>(p));
    prof_end("split_hilo", s, tok);
    PK_CHECK_LAUNCH("pk_split_hilo");
    return PK_OK;
}

int pk_series_map(int op, int dtype, int degree, int ndim, const int64_t* shape, void* const* out,
                  const int64_t* out_strides, const void* const* a, int a_planes, const int64_t* a_strides,
                  const void* const* b, int b_planes, const int64_t* b_strides, double p0, double p1,
                  void* stream) {
    MapParams p{};
    if (int rc = fill_map_params(p, "pk_series_map", op, degree, ndim, shape, out, out_strides, a, a_planes,
                                 a_strides, b, b_planes, b_strides, p0, p1))
        return rc;
    if (p.numel == 0) return PK_OK;
    const int np = p.np;
    const bool binary = is_binary(op);
    const int grid = grid_for(p.numel);
    bool vec = p.contig != 0;
    if (vec) {
        const int esz = dtype == PK_F64 ? 8 : (dtype == PK_F32 ? 4 : 2);
        vec = row_vec_ok(p.out, np, 0, esz) && row_vec_ok(p.a, std::min(a_planes, np), 0, esz) &&
              (!binary || row_vec_ok(p.b, std::min(b_planes, np), 0, esz));
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    void* tok;
    prof_begin("series_map", s, &tok);
    switch (dtype) {
        case PK_F32: launch_map_t<float>(p, grid, vec, s); break;
        case PK_F64: launch_map_t<double>(p, grid, vec, s); break;
        case PK_BF16: launch_map_t<__nv_bfloat16>(p, grid, vec, s); break;
        case PK_F16: launch_map_t<__half>(p, grid, vec, s); break;
        default: return fail(PK_ERR_UNSUPPORTED, "pk_series_map: unsupported dtype");
    }
    prof_end("series_map", s, tok);
    PK_CHECK_LAUNCH("pk_series_map");
    return PK_OK;
}

int pk_series_map_complex(int op, int real_dtype, int degree, int ndim, const int64_t* shape, void* const* out,
                          const int64_t* out_strides, uint32_t out_complex, const void* const* a, int a_planes,
                          const int64_t* a_strides, uint32_t a_complex, const void* const* b, int b_planes,
                          const int64_t* b_strides, uint32_t b_complex, double p0, double p1, void* stream) {
    MapParams p{};
    if (int rc = fill_map_params(p, "pk_series_map_complex", op, degree, ndim, shape, out, out_strides, a,
                                 a_planes, a_strides, b, b_planes, b_strides, p0, p1))
        return rc;
    if (p.numel == 0) return PK_OK;
    const int grid = grid_for(p.numel);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    void* tok;
    prof_begin("series_map", s, &tok);
    switch (real_dtype) {
        case PK_F32: launch_map_cplx<float>(p, grid, a_complex, b_complex, out_complex, s); break;
        case PK_F64: launch_map_cplx<double>(p, grid, a_complex, b_complex, out_complex, s); break;
        default: return fail(PK_ERR_UNSUPPORTED, "pk_series_map_complex: real_dtype must be PK_F32 or PK_F64");
    }
    prof_end("series_map", s, tok);
    PK_CHECK_LAUNCH("pk_series_map_complex");
    return PK_OK;
}

int pk_series_reduce(int dtype, int degree, int64_t outer, int64_t red, int64_t inner, const void* const* x,
                     void* const* out, double scale, void* stream) {
    if (degree < 0 || degree >= PK_MAX_PLANES) return fail(PK_ERR_UNSUPPORTED, "pk_series_reduce: degree out of range");
    if (outer < 0 || red < 0 || inner < 0) return fail(PK_ERR_ARG, "pk_series_reduce: negative extent");
    ReduceParams p{};
    p.np = degree + 1;
    p.outer = outer;
    p.red = red;
    p.inner = inner;
    p.scale = scale;
    for (int k = 0; k < p.np; ++k) {
        p.x[k] = x[k];
        p.out[k] = out[k];
    }
    if (outer * inner == 0) return PK_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t esz = dtype == PK_F64 ? 8 : (dtype == PK_F32 ? 4 : 2);
    if (red == 0) {
        for (int k = 0; k < p.np; ++k) {
            cudaError_t e = cudaMemsetAsync(out[k], 0, outer * inner * esz, s);
            if (e != cudaSuccess) return cuda_fail(e, "pk_series_reduce: memset");
        }
        return PK_OK;
    }
    if (inner == 1) {
        const dim3 grid(static_cast<unsigned>(std::min<int64_t>(outer, 65535LL * 16)));
        if (dtype == PK_F32) launch_reduce_np<float>(p, true, 0, grid, s);
        else if (dtype == PK_F64) launch_reduce_np<double>(p, true, 0, grid, s);
        else return fail(PK_ERR_UNSUPPORTED, "pk_series_reduce: row reduction supports float32/float64");
    } else {
        const int64_t cols = outer * inner;
        int64_t splits = 1;
        const int64_t want = static_cast<int64_t>(num_sms()) * 8 * 256;
        if (cols < want && red > 64) splits = std::min<int64_t>(ceil_div(want, cols), ceil_div(red, 64));
        splits = std::min<int64_t>(splits, 65535);
        p.red_chunk = ceil_div(red, splits);
        splits = ceil_div(red, p.red_chunk);
        const int atomic = splits > 1 ? 1 : 0;
        if (dtype != PK_F32 && dtype != PK_F64)
            return fail(PK_ERR_UNSUPPORTED, "pk_series_reduce: column reduction supports float32/float64");
        if (atomic) {
            for (int k = 0; k < p.np; ++k) {
                cudaError_t e = cudaMemsetAsync(out[k], 0, cols * esz, s);
                if (e != cudaSuccess) return cuda_fail(e, "pk_series_reduce: memset");
            }
        }
        const dim3 grid(static_cast<unsigned>(std::min<int64_t>(ceil_div(cols, 256), 65535)),
                        static_cast<unsigned>(splits));
        if (dtype == PK_F32) launch_reduce_np<float>(p, false, atomic, grid, s);
        else launch_reduce_np<double>(p, false, atomic, grid, s);
    }
    PK_CHECK_LAUNCH("pk_series_reduce");
    return PK_OK;
}

int pk_series_gather_rows(int dtype, int degree, int64_t n_idx, int64_t dim, const int64_t* idx,
                          const void* const* src, int64_t src_rs, int64_t n_rows, void* const* out, void* stream) {
    if (degree < 0 || degree >= PK_MAX_PLANES) return fail(PK_ERR_UNSUPPORTED, "pk_series_gather_rows: degree");
    RowParams p{};
    p.np = degree + 1;
    p.n_idx = n_idx;
    p.dim = dim;
    p.n_rows = n_rows;
    p.src_rs = src_rs;
    p.idx = idx;
    p.status = device_status_ptr();
    for (int k = 0; k < p.np; ++k) {
        p.src[k] = src[k];
        p.dst[k] = out[k];
    }
    if (n_idx * dim == 0) return PK_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int grid = grid_for(n_idx * dim);
    if (dtype == PK_F32) PK_LAUNCHED(gather_rows_kernel<float><<<grid, 256, 0, s>>>(p));
    else if (dtype == PK_F64) PK_LAUNCHED(gather_rows_kernel<double><<<grid, 256, 0, s>>>(p));
    else return fail(PK_ERR_UNSUPPORTED, "pk_series_gather_rows: float32/float64 only");
    PK_CHECK_LAUNCH("pk_series_gather_rows");
    return PK_OK;
}

int pk_series_scatter_add_rows(int dtype, int degree, int64_t n_idx, int64_t dim, const int64_t* idx,
                               int64_t padding_idx, const void* const* src, int64_t src_rs, int64_t n_rows,
                               void* const* out, void* stream) {
    if (degree < 0 || degree >= PK_MAX_PLANES) return fail(PK_ERR_UNSUPPORTED, "pk_series_scatter_add_rows: degree");
    RowParams p{};
    p.np = degree + 1;
    p.n_idx = n_idx;
    p.dim = dim;
    p.n_rows = n_rows;
    p.src_rs = src_rs;
    p.idx = idx;
    p.padding_idx = padding_idx;
    p.status = device_status_ptr();
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t esz = dtype == PK_F64 ? 8 : 4;
    if (dtype != PK_F32 && dtype != PK_F64) return fail(PK_ERR_UNSUPPORTED, "pk_series_scatter_add_rows: dtype");
    for (int k = 0; k < p.np; ++k) {
        p.src[k] = src[k];
        p.dst[k] = out[k];
        cudaError_t e = cudaMemsetAsync(out[k], 0, n_rows * dim * esz, s);
        if (e != cudaSuccess) return cuda_fail(e, "pk_series_scatter_add_rows: memset");
    }
    if (n_idx * dim == 0) return PK_OK;
    const int grid = grid_for(n_idx * dim);
    if (dtype == PK_F32) PK_LAUNCHED(scatter_add_rows_kernel<float><<<grid, 256, 0, s>>>(p));
    else PK_LAUNCHED(scatter_add_rows_kernel<double><<<grid, 256, 0, s>>>(p));
    PK_CHECK_LAUNCH("pk_series_scatter_add_rows");
    return PK_OK;
}

}  // extern "C"
