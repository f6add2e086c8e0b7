// Softmax family and cross entropy of series along the last dimension.
//
// For a row of logits series x(c) (c = class) with base log-sum-exp lse_0, the reference
// (src/polytensors/_plain.py:262-273) forms E = exp(x - lse_0) as series, Z = sum_c E,
// log Z, and log_softmax = x - log Z.  Because exp(x(c)) = exp(x_0(c)) e(c) with e the
// exponential of the directions only, Z_k = sum_c exp(x_0(c) - m) e_k(c) / S_0 for any
// shift m: one streaming pass with an online maximum (the flash-softmax rescaling applied
// to all n+1 sums at once) yields lse_0 and the log-normaliser series logz_1..n.  A second
// pass writes log_softmax_k = x_k - logz_k (k >= 1), x_0 - lse_0 (k = 0), or its exponential.
//
// Cross entropy never writes log_softmax: loss_k = logz_k - x_k[y] (loss_0 = lse_0 - x_0[y]),
// and its backward is dx = g (*) P - g e_y with P the softmax series recomputed per
// element (src/polytensors/_plain.py:348-354 after the NLL scatter of
// src/polytensors/_dispatch.py:556-562), optionally through a softcap z -> c tanh(z/c)
// (src/polytensors/_cross_entropy_kernels.py:7-17, generalised to any degree).
#include <type_traits>
#include <algorithm>

#include "pk_rows.cuh"

namespace pk {

struct SoftmaxParams {
    int np;
    int64_t rows, cols;
    int64_t x_rs, y_rs, g_rs;
    int log;              // softmax: write log_softmax (1) or softmax (0)
    double softcap;       // cross entropy: 0 = none
    int64_t ignore_index;
    const int64_t* target;
    const void* x[PK_MAX_PLANES];
    const void* y[PK_MAX_PLANES];   // backward: forward output
    const void* g[PK_MAX_PLANES];   // backward: incoming gradient (per element, or per row for CE)
    void* out[PK_MAX_PLANES];
    void* stats;                    // CE / attention: [rows][np] (lse_0, logz_1..n), compute type
    // attention score rows: row r is query (r % q_len) of its matrix; entries scale * x,
    // masked (causal: key > query + causal_shift) entries excluded
    double scale;
    int causal;
    int64_t q_len, causal_shift;
    const void* dsum;               // attention backward: [rows][np] sum_d dO (*) O, compute type
    int vec;                        // every plane and row stride allows ROW_VEC-element vector access
};

template <int NP, typename T, typename C>
__device__ __forceinline__ void load_row_elem(const void* const* planes, int np, int64_t off, C (&v)[NP]) {
#pragma unroll
    for (int k = 0; k < NP; ++k) v[k] = k < np ? to_c<C>(static_cast<const T*>(planes[k])[off]) : C(0);
}

// z -> c tanh(z / c) as a series; d receives the derivative series 1 - tanh^2(z / c).
template <int NP, typename C>
__device__ __forceinline__ void softcap_series(C (&z)[NP], C cap, C (&d)[NP]) {
    C u[NP], t[NP];
    const C inv = C(1) / cap;
#pragma unroll
    for (int k = 0; k < NP; ++k) u[k] = z[k] * inv;
    s_tanh<NP, C>(u, t, d);
#pragma unroll
    for (int k = 0; k < NP; ++k) z[k] = cap * t[k];
}

// Pass 1 of every kernel here: the online log-sum-exp state of a row (keys <= limit when limit >= 0).
template <typename T, int NP, typename C>
__device__ __forceinline__ void row_lse(const SoftmaxParams& p, int64_t xb, C* scratch, C (&lse)[NP],
                                        C scale = C(1), int64_t limit = -1) {
    C m = -INFINITY, S[NP];
#pragma unroll
    for (int k = 0; k < NP; ++k) S[k] = C(0);
    const int64_t end = (limit < 0 || limit >= p.cols) ? p.cols : limit + 1;  // limit < 0: every key
    for (int64_t c0 = static_cast<int64_t>(threadIdx.x) * ROW_VEC; c0 < end; c0 += static_cast<int64_t>(blockDim.x) * ROW_VEC) {
        const int valid = vec_count(end, c0);
        C x[ROW_VEC][NP];
        load_planes4<NP, T, C>(p.x, p.np, xb + c0, valid, p.vec != 0, x);
#pragma unroll
        for (int u = 0; u < ROW_VEC; ++u) {
#pragma unroll
            for (int k = 0; k < NP; ++k) x[u][k] *= scale;
            if (p.softcap != 0.0) {
                C d[NP];
                softcap_series<NP, C>(x[u], C(p.softcap), d);
            }
        }
        lse_accumulate4<NP, C>(m, S, x, valid);
    }
    block_lse_combine<NP, C>(m, S, scratch);
    lse_finish<NP, C>(m, S, lse);
}

template <typename T, int NP>
__global__ void __launch_bounds__(512) softmax_fwd_kernel(const SoftmaxParams p) {
    using C = typename Compute<T>::type;
    __shared__ C scratch[16 * (NP + 1)];
    for (int64_t row = blockIdx.x; row < p.rows; row += gridDim.x) {
        const int64_t xb = row * p.x_rs, yb = row * p.y_rs;
        C lse[NP];
        row_lse<T, NP, C>(p, xb, scratch, lse);
        for (int64_t c0 = static_cast<int64_t>(threadIdx.x) * ROW_VEC; c0 < p.cols;
             c0 += static_cast<int64_t>(blockDim.x) * ROW_VEC) {
            const int valid = vec_count(p.cols, c0);
            C x[ROW_VEC][NP];
            load_planes4<NP, T, C>(p.x, p.np, xb + c0, valid, p.vec != 0, x);
#pragma unroll
            for (int u = 0; u < ROW_VEC; ++u) {
                x[u][0] -= lse[0];
#pragma unroll
                for (int k = 1; k < NP; ++k) x[u][k] -= lse[k];
                if (!p.log) s_exp<NP, C>(x[u], x[u]);
            }
            store_planes4<NP, T, C>(p.out, p.np, yb + c0, valid, p.vec != 0, x);
        }
    }
}

// log: dx = G - exp(Y) (*) sum_row G        (src/polytensors/_plain.py:348-354)
// not log: dx = Y (*) (G - sum_row G (*) Y)   (src/polytensors/_plain.py:342-347)
template <typename T, int NP>
__global__ void __launch_bounds__(512) softmax_bwd_kernel(const SoftmaxParams p) {
    using C = typename Compute<T>::type;
    __shared__ C scratch[16 * NP];
    for (int64_t row = blockIdx.x; row < p.rows; row += gridDim.x) {
        const int64_t gb = row * p.g_rs, yb = row * p.y_rs, ob = row * p.x_rs;
        C s[NP];
#pragma unroll
        for (int k = 0; k < NP; ++k) s[k] = C(0);
        for (int64_t c0 = static_cast<int64_t>(threadIdx.x) * ROW_VEC; c0 < p.cols;
             c0 += static_cast<int64_t>(blockDim.x) * ROW_VEC) {
            const int valid = vec_count(p.cols, c0);
            C g[ROW_VEC][NP], y[ROW_VEC][NP];
            load_planes4<NP, T, C>(p.g, p.np, gb + c0, valid, p.vec != 0, g);
            if (!p.log) load_planes4<NP, T, C>(p.y, p.np, yb + c0, valid, p.vec != 0, y);
#pragma unroll
            for (int u = 0; u < ROW_VEC; ++u) {
                if (p.log) {
#pragma unroll
                    for (int k = 0; k < NP; ++k) s[k] += g[u][k];
                } else {
                    C t[NP];
                    s_mul<NP, C>(g[u], y[u], t);
#pragma unroll
                    for (int k = 0; k < NP; ++k) s[k] += t[k];
                }
            }
        }
        block_sum<NP, C>(s, scratch);
        for (int64_t c0 = static_cast<int64_t>(threadIdx.x) * ROW_VEC; c0 < p.cols;
             c0 += static_cast<int64_t>(blockDim.x) * ROW_VEC) {
            const int valid = vec_count(p.cols, c0);
            C g[ROW_VEC][NP], y[ROW_VEC][NP], r[ROW_VEC][NP];
            load_planes4<NP, T, C>(p.g, p.np, gb + c0, valid, p.vec != 0, g);
            load_planes4<NP, T, C>(p.y, p.np, yb + c0, valid, p.vec != 0, y);
#pragma unroll
            for (int u = 0; u < ROW_VEC; ++u) {
                if (p.log) {
                    C e[NP], t[NP];
                    s_exp<NP, C>(y[u], e);
                    s_mul<NP, C>(e, s, t);
#pragma unroll
                    for (int k = 0; k < NP; ++k) r[u][k] = g[u][k] - t[k];
                } else {
                    C d[NP];
#pragma unroll
                    for (int k = 0; k < NP; ++k) d[k] = g[u][k] - s[k];
                    s_mul<NP, C>(y[u], d, r[u]);
                }
            }
            store_planes4<NP, T, C>(p.out, p.np, ob + c0, valid, p.vec != 0, r);
        }
    }
}

// Cross entropy forward: per-row loss series and the row statistics for backward.
template <typename T, int NP>
__global__ void __launch_bounds__(512) ce_fwd_kernel(const SoftmaxParams p) {
    using C = typename Compute<T>::type;
    __shared__ C scratch[16 * (NP + 1)];
    for (int64_t row = blockIdx.x; row < p.rows; row += gridDim.x) {
        const int64_t xb = row * p.x_rs;
        C lse[NP];
        row_lse<T, NP, C>(p, xb, scratch, lse);
        if (threadIdx.x == 0) {
            const int64_t y = p.target[row];
            const bool valid = y != p.ignore_index && y >= 0 && y < p.cols;
            C zy[NP];
#pragma unroll
            for (int k = 0; k < NP; ++k) zy[k] = C(0);
            if (valid) {
                load_row_elem<NP, T, C>(p.x, p.np, xb + y, zy);
                if (p.softcap != 0.0) {
                    C d[NP];
                    softcap_series<NP, C>(zy, C(p.softcap), d);
                }
            }
#pragma unroll
            for (int k = 0; k < NP; ++k) {
                if (k >= p.np) continue;
                static_cast<C*>(p.out[k])[row] = valid ? lse[k] - zy[k] : C(0);
                static_cast<C*>(p.stats)[row * p.np + k] = lse[k];
            }
        }
        __syncthreads();
    }
}

// Cross entropy backward: dz = d (*) [g (*) P - g e_y], d = softcap derivative series (or 1).
template <typename T, int NP>
__global__ void __launch_bounds__(512) ce_bwd_kernel(const SoftmaxParams p) {
    using C = typename Compute<T>::type;
    for (int64_t row = blockIdx.x; row < p.rows; row += gridDim.x) {
        const int64_t y = p.target[row];
        const bool valid = y != p.ignore_index && y >= 0 && y < p.cols;
        C g[NP], lse[NP];
#pragma unroll
        for (int k = 0; k < NP; ++k) {
            g[k] = (valid && k < p.np) ? static_cast<const C*>(p.g[k])[row] : C(0);
            lse[k] = k < p.np ? static_cast<const C*>(p.stats)[row * p.np + k] : C(0);
        }
        const int64_t xb = row * p.x_rs, ob = row * p.y_rs;
        for (int64_t c0 = static_cast<int64_t>(threadIdx.x) * ROW_VEC; c0 < p.cols;
             c0 += static_cast<int64_t>(blockDim.x) * ROW_VEC) {
            const int valid = vec_count(p.cols, c0);
            C z[ROW_VEC][NP], r[ROW_VEC][NP];
            load_planes4<NP, T, C>(p.x, p.np, xb + c0, valid, p.vec != 0, z);
#pragma unroll
            for (int u = 0; u < ROW_VEC; ++u) {
                C d[NP], ls[NP], P[NP];
                if (p.softcap != 0.0) softcap_series<NP, C>(z[u], C(p.softcap), d);
                ls[0] = z[u][0] - lse[0];
#pragma unroll
                for (int k = 1; k < NP; ++k) ls[k] = z[u][k] - lse[k];
                s_exp<NP, C>(ls, P);
                s_mul<NP, C>(g, P, r[u]);
                if (c0 + u == y) {
#pragma unroll
                    for (int k = 0; k < NP; ++k) r[u][k] -= g[k];
                }
                if (p.softcap != 0.0) s_mul<NP, C>(r[u], d, r[u]);
            }
            store_planes4<NP, T, C>(p.out, p.np, ob + c0, valid, p.vec != 0, r);
        }
    }
}

// Attention probabilities from raw score series x = Q K^T (all planes):  P = softmax(scale * x)
// along keys with causal masking, written as series; stats receive (lse_0, logz_1..n) per row.
// HILO (float32 scores only): P is written as bf16 hi/lo pairs (2 np output planes), the operand
// form of the float32 tensor-core products that consume it.
template <typename T, int NP, bool HILO = false>
__global__ void __launch_bounds__(512) attn_probs_kernel(const SoftmaxParams p) {
    using C = typename Compute<T>::type;
    __shared__ C scratch[16 * (NP + 1)];
    const C sc = C(p.scale);
    for (int64_t row = blockIdx.x; row < p.rows; row += gridDim.x) {
        const int64_t xb = row * p.x_rs, yb = row * p.y_rs;
        const int64_t limit = p.causal ? (row % p.q_len) + p.causal_shift : p.cols - 1;  // last admissible key
        C lse[NP];
        row_lse<T, NP, C>(p, xb, scratch, lse, sc, limit);
        const bool empty = !(lse[0] > -INFINITY) || lse[0] != lse[0];
        if (empty) {
#pragma unroll
            for (int k = 0; k < NP; ++k) lse[k] = C(0);
            lse[0] = INFINITY;  // a row without admissible keys: P = 0 (and 0 output)
        }
        if (threadIdx.x == 0) {
#pragma unroll
            for (int k = 0; k < NP; ++k)
                if (k < p.np) static_cast<C*>(p.stats)[row * p.np + k] = lse[k];
        }
        for (int64_t c0 = static_cast<int64_t>(threadIdx.x) * ROW_VEC; c0 < p.cols;
             c0 += static_cast<int64_t>(blockDim.x) * ROW_VEC) {
            const int valid = vec_count(p.cols, c0);
            C x[ROW_VEC][NP];
            load_planes4<NP, T, C>(p.x, p.np, xb + c0, valid, p.vec != 0, x);
#pragma unroll
            for (int u = 0; u < ROW_VEC; ++u) {
                if (c0 + u <= limit && !empty) {
                    x[u][0] = x[u][0] * sc - lse[0];
#pragma unroll
                    for (int k = 1; k < NP; ++k) x[u][k] = x[u][k] * sc - lse[k];
                    s_exp<NP, C>(x[u], x[u]);
                } else {
#pragma unroll
                    for (int k = 0; k < NP; ++k) x[u][k] = C(0);
                }
            }
            if constexpr (HILO) store_planes4_hilo<NP>(p.out, p.np, yb + c0, valid, p.vec != 0, x);
            else store_planes4<NP, T, C>(p.out, p.np, yb + c0, valid, p.vec != 0, x);
        }
    }
}

// Score gradient of attention, the series form of the softmax backward
// (src/polytensors/_plain.py:342-347) through the score scaling:
//   d scores = scale * P (*) (dP - dsum_row),   dsum_row = sum_d dO (*) O.
// P arrives in p.y, dP in p.g, the output goes to p.out (may alias p.g); masked entries
// have P = 0 and so get a zero gradient.  HILO (float32 only): P arrives and the output leaves as
// bf16 hi/lo pairs (2 np planes each); dP stays float32.
template <typename T, int NP, bool HILO = false>
__global__ void __launch_bounds__(256) attn_dscores_kernel(const SoftmaxParams p) {
    using C = typename Compute<T>::type;
    const C sc = C(p.scale);
    for (int64_t row = blockIdx.x; row < p.rows; row += gridDim.x) {
        const int64_t yb = row * p.y_rs, gb = row * p.g_rs, ob = row * p.x_rs;
        C ds[NP];
#pragma unroll
        for (int k = 0; k < NP; ++k) ds[k] = k < p.np ? static_cast<const C*>(p.dsum)[row * p.np + k] : C(0);
        for (int64_t c0 = static_cast<int64_t>(threadIdx.x) * ROW_VEC; c0 < p.cols;
             c0 += static_cast<int64_t>(blockDim.x) * ROW_VEC) {
            const int valid = vec_count(p.cols, c0);
            C P[ROW_VEC][NP], g[ROW_VEC][NP], r[ROW_VEC][NP];
            if constexpr (HILO) load_planes4_hilo<NP>(p.y, p.np, yb + c0, valid, p.vec != 0, P);
            else load_planes4<NP, T, C>(p.y, p.np, yb + c0, valid, p.vec != 0, P);
            load_planes4<NP, T, C>(p.g, p.np, gb + c0, valid, p.vec != 0, g);
#pragma unroll
            for (int u = 0; u < ROW_VEC; ++u) {
#pragma unroll
                for (int k = 0; k < NP; ++k) g[u][k] -= ds[k];
                s_mul<NP, C>(P[u], g[u], r[u]);
#pragma unroll
                for (int k = 0; k < NP; ++k) r[u][k] *= sc;
            }
            if constexpr (HILO) store_planes4_hilo<NP>(p.out, p.np, ob + c0, valid, p.vec != 0, r);
            else store_planes4<NP, T, C>(p.out, p.np, ob + c0, valid, p.vec != 0, r);
        }
    }
}

// dsum[row][k] = (sum_d dO (*) O)_k, the row term of the attention score gradient: one warp per
// row, four elements per lane and step, the n+1 sums reduced across the warp.  Rows of dO and O
// are contiguous (row strides do_rs / o_rs elements).
struct DsumParams {
    int np;
    int64_t rows, cols, do_rs, o_rs;
    const void* dO[PK_MAX_PLANES];
    const void* O[PK_MAX_PLANES];
    void* dsum;  // [rows][np], compute type
    int vec;
};

template <typename T, int NP>
__global__ void __launch_bounds__(256) attn_dsum_kernel(const DsumParams p) {
    using C = typename Compute<T>::type;
    const int lane = threadIdx.x & 31;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); row < p.rows;
         row += warps) {
        C acc[NP];
#pragma unroll
        for (int k = 0; k < NP; ++k) acc[k] = C(0);
        for (int64_t c0 = static_cast<int64_t>(lane) * ROW_VEC; c0 < p.cols; c0 += 32 * ROW_VEC) {
            const int valid = vec_count(p.cols, c0);
            C g[ROW_VEC][NP], o[ROW_VEC][NP];
            load_planes4<NP, T, C>(p.dO, p.np, row * p.do_rs + c0, valid, p.vec != 0, g);
            load_planes4<NP, T, C>(p.O, p.np, row * p.o_rs + c0, valid, p.vec != 0, o);
#pragma unroll
            for (int u = 0; u < ROW_VEC; ++u) s_mul_acc<NP, C>(g[u], o[u], acc);
        }
#pragma unroll
        for (int k = 0; k < NP; ++k) {
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) acc[k] += __shfl_xor_sync(0xffffffffu, acc[k], off);
        }
        if (lane < p.np) {
#pragma unroll
            for (int k = 0; k < NP; ++k)
                if (k == lane) static_cast<C*>(p.dsum)[row * p.np + k] = acc[k];
        }
    }
}

template <typename T>
static void launch_dsum(const DsumParams& p, cudaStream_t s) {
    // one warp per row (no row loop): the rows are short, so parallelism, not reuse, hides latency
    const int grid = static_cast<int>(std::min<int64_t>(ceil_div(p.rows, 8), 0x7fffffff));
    switch (p.np) {
        case 1: PK_LAUNCHED(attn_dsum_kernel<T, 1><<<grid, 256, 0, s>>>(p)); break;
        case 2: PK_LAUNCHED(attn_dsum_kernel<T, 2><<<grid, 256, 0, s>>>(p)); break;
        case 3: PK_LAUNCHED(attn_dsum_kernel<T, 3><<<grid, 256, 0, s>>>(p)); break;
        case 4: PK_LAUNCHED(attn_dsum_kernel<T, 4><<<grid, 256, 0, s>>>(p)); break;
        case 5: case 6: PK_LAUNCHED(attn_dsum_kernel<T, 6><<<grid, 256, 0, s>>>(p)); break;
        case 7: case 8: case 9: PK_LAUNCHED(attn_dsum_kernel<T, 9><<<grid, 256, 0, s>>>(p)); break;
        default: PK_LAUNCHED(attn_dsum_kernel<T, 16><<<grid, 256, 0, s>>>(p)); break;
    }
}

enum { SM_FWD = 0, SM_BWD = 1, CE_FWD = 2, CE_BWD = 3, ATTN_P = 4, ATTN_DS = 5, ATTN_P_HILO = 6, ATTN_DS_HILO = 7 };

static int row_threads(int64_t cols) { return cols >= 4096 ? 512 : (cols >= 1024 ? 256 : 128); }

template <typename T, int NP>
static void launch_rows(int which, const SoftmaxParams& p, cudaStream_t s) {
    const int threads = row_threads(p.cols);
    const int grid = static_cast<int>(std::min<int64_t>(p.rows, static_cast<int64_t>(num_sms()) * 8));
    switch (which) {
        case SM_FWD: PK_LAUNCHED(softmax_fwd_kernel<T, NP><<<grid, threads, 0, s>>>(p)); break;
        case SM_BWD: PK_LAUNCHED(softmax_bwd_kernel<T, NP><<<grid, threads, 0, s>>>(p)); break;
        case CE_FWD: PK_LAUNCHED(ce_fwd_kernel<T, NP><<<grid, threads, 0, s>>>(p)); break;
        case ATTN_P: PK_LAUNCHED(attn_probs_kernel<T, NP><<<grid, threads, 0, s>>>(p)); break;
        case ATTN_DS: PK_LAUNCHED(attn_dscores_kernel<T, NP><<<grid, std::min(threads, 256), 0, s>>>(p)); break;
        case ATTN_P_HILO:
            if constexpr (std::is_same<T, float>::value)
                PK_LAUNCHED(attn_probs_kernel<T, NP, true><<<grid, threads, 0, s>>>(p));
            break;
        case ATTN_DS_HILO:
            if constexpr (std::is_same<T, float>::value)
                PK_LAUNCHED(attn_dscores_kernel<T, NP, true><<<grid, std::min(threads, 256), 0, s>>>(p));
            break;
        default: PK_LAUNCHED(ce_bwd_kernel<T, NP><<<grid, threads, 0, s>>>(p)); break;
    }
}

template <typename T>
static void launch_rows_np(int which, const SoftmaxParams& p, cudaStream_t s) {
    switch (p.np) {
        case 1: launch_rows<T, 1>(which, p, s); break;
        case 2: launch_rows<T, 2>(which, p, s); break;
        case 3: launch_rows<T, 3>(which, p, s); break;
        case 4: launch_rows<T, 4>(which, p, s); break;
        case 5: launch_rows<T, 5>(which, p, s); break;
        case 6: launch_rows<T, 6>(which, p, s); break;
        case 7: case 8: case 9: launch_rows<T, 9>(which, p, s); break;
        default: launch_rows<T, 16>(which, p, s); break;
    }
}

static int elem_bytes(int dtype) { return dtype == PK_F64 ? 8 : (dtype == PK_F32 ? 4 : 2); }

static int dispatch_rows(int which, int dtype, SoftmaxParams& p, void* stream, const char* what) {
    if (p.rows == 0 || p.cols == 0) return PK_OK;
    {
        const int eb = elem_bytes(dtype);
        bool ok = p.cols % ROW_VEC == 0;
        const void* const* sets[4] = {p.x, p.y, p.g, reinterpret_cast<const void* const*>(p.out)};
        const int64_t strides[4] = {p.x_rs, p.y_rs, p.g_rs, 0};
        // hi/lo kinds: the probabilities (y, for the score gradient) and the output are 2 np bf16 planes
        const bool hilo = which == ATTN_P_HILO || which == ATTN_DS_HILO;
        const bool split_set[4] = {false, hilo, false, hilo};
        for (int i = 0; i < 4 && ok; ++i) {
            if (!sets[i][0]) continue;
            ok = split_set[i] ? row_vec_ok(sets[i], 2 * p.np, strides[i], 2) : row_vec_ok(sets[i], p.np, strides[i], eb);
        }
        // output planes share the row stride of their input role (x_rs or y_rs)
        ok = ok && p.x_rs % ROW_VEC == 0 && p.y_rs % ROW_VEC == 0 && p.g_rs % ROW_VEC == 0;
        p.vec = ok ? 1 : 0;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    void* tok;
    prof_begin(what, s, &tok);
    switch (dtype) {
        case PK_F32: launch_rows_np<float>(which, p, s); break;
        case PK_F64: launch_rows_np<double>(which, p, s); break;
        case PK_BF16: launch_rows_np<__nv_bfloat16>(which, p, s); break;
        case PK_F16: launch_rows_np<__half>(which, p, s); break;
        default: return fail(PK_ERR_UNSUPPORTED, std::string(what) + ": unsupported dtype");
    }
    prof_end(what, s, tok);
    PK_CHECK_LAUNCH(what);
    return PK_OK;
}

static int check_common(int degree, int64_t rows, int64_t cols, const char* what) {
    if (degree < 0 || degree >= PK_MAX_PLANES) return fail(PK_ERR_UNSUPPORTED, std::string(what) + ": degree out of range");
    if (rows < 0 || cols < 0) return fail(PK_ERR_ARG, std::string(what) + ": negative extent");
    return PK_OK;
}

}  // namespace pk

using namespace pk;

extern "C" {

int pk_softmax_fwd(int dtype, int degree, int64_t rows, int64_t cols, const void* const* x, int64_t x_rs, int log,
                   void* const* y, int64_t y_rs, void* stream) {
    if (int rc = check_common(degree, rows, cols, "pk_softmax_fwd")) return rc;
    SoftmaxParams p{};
    p.np = degree + 1;
    p.rows = rows;
    p.cols = cols;
    p.x_rs = x_rs;
    p.y_rs = y_rs;
    p.log = log;
    for (int k = 0; k < p.np; ++k) {
        p.x[k] = x[k];
        p.out[k] = y[k];
    }
    return dispatch_rows(SM_FWD, dtype, p, stream, "softmax_fwd");
}

int pk_softmax_bwd(int dtype, int degree, int64_t rows, int64_t cols, const void* const* g, int64_t g_rs,
                   const void* const* y, int64_t y_rs, int log, void* const* dx, int64_t dx_rs, void* stream) {
    if (int rc = check_common(degree, rows, cols, "pk_softmax_bwd")) return rc;
    SoftmaxParams p{};
    p.np = degree + 1;
    p.rows = rows;
    p.cols = cols;
    p.g_rs = g_rs;
    p.y_rs = y_rs;
    p.x_rs = dx_rs;
    p.log = log;
    for (int k = 0; k < p.np; ++k) {
        p.g[k] = g[k];
        p.y[k] = y[k];
        p.out[k] = dx[k];
    }
    return dispatch_rows(SM_BWD, dtype, p, stream, "softmax_bwd");
}

int pk_cross_entropy_fwd(int dtype, int degree, int64_t rows, int64_t cols, const void* const* z, int64_t z_rs,
                         const int64_t* target, int64_t ignore_index, double softcap, void* const* loss, void* stats,
                         void* stream) {
    if (int rc = check_common(degree, rows, cols, "pk_cross_entropy_fwd")) return rc;
    if (!target || !stats) return fail(PK_ERR_ARG, "pk_cross_entropy_fwd: null target or stats");
    if (cols == 0) return fail(PK_ERR_ARG, "pk_cross_entropy_fwd: no classes");
    SoftmaxParams p{};
    p.np = degree + 1;
    p.rows = rows;
    p.cols = cols;
    p.x_rs = z_rs;
    p.target = target;
    p.ignore_index = ignore_index;
    p.softcap = softcap;
    p.stats = stats;
    for (int k = 0; k < p.np; ++k) {
        p.x[k] = z[k];
        p.out[k] = loss[k];
    }
    return dispatch_rows(CE_FWD, dtype, p, stream, "cross_entropy_fwd");
}

int pk_cross_entropy_bwd(int dtype, int degree, int64_t rows, int64_t cols, const void* const* z, int64_t z_rs,
                         const int64_t* target, int64_t ignore_index, double softcap, const void* stats,
                         const void* const* g, void* const* dz, int64_t dz_rs, void* stream) {
    if (int rc = check_common(degree, rows, cols, "pk_cross_entropy_bwd")) return rc;
    if (!target || !stats) return fail(PK_ERR_ARG, "pk_cross_entropy_bwd: null target or stats");
    SoftmaxParams p{};
    p.np = degree + 1;
    p.rows = rows;
    p.cols = cols;
    p.x_rs = z_rs;
    p.y_rs = dz_rs;
    p.target = target;
    p.ignore_index = ignore_index;
    p.softcap = softcap;
    p.stats = const_cast<void*>(stats);
    for (int k = 0; k < p.np; ++k) {
        p.x[k] = z[k];
        p.g[k] = g[k];
        p.out[k] = dz[k];
    }
    return dispatch_rows(CE_BWD, dtype, p, stream, "cross_entropy_bwd");
}

int pk_attn_probs(int dtype, int degree, int64_t rows, int64_t cols, int64_t q_len, const void* const* scores,
                  int64_t s_rs, double scale, int causal, int64_t causal_shift, void* const* probs, int64_t p_rs,
                  void* stats, void* stream) {
    if (int rc = check_common(degree, rows, cols, "pk_attn_probs")) return rc;
    if (!stats || q_len <= 0) return fail(PK_ERR_ARG, "pk_attn_probs: null stats or bad q_len");
    SoftmaxParams p{};
    p.np = degree + 1;
    p.rows = rows;
    p.cols = cols;
    p.x_rs = s_rs;
    p.y_rs = p_rs;
    p.scale = scale;
    p.causal = causal;
    p.q_len = q_len;
    p.causal_shift = causal_shift;
    p.stats = stats;
    for (int k = 0; k < p.np; ++k) {
        p.x[k] = scores[k];
        p.out[k] = probs[k];
    }
    return dispatch_rows(ATTN_P, dtype, p, stream, "attn_probs");
}

int pk_attn_dscores(int dtype, int degree, int64_t rows, int64_t cols, const void* const* probs, int64_t p_rs,
                    const void* const* dprobs, int64_t dp_rs, const void* dsum, double scale, void* const* dscores,
                    int64_t ds_rs, void* stream) {
    if (int rc = check_common(degree, rows, cols, "pk_attn_dscores")) return rc;
    if (!dsum) return fail(PK_ERR_ARG, "pk_attn_dscores: null dsum");
    SoftmaxParams p{};
    p.np = degree + 1;
    p.rows = rows;
    p.cols = cols;
    p.y_rs = p_rs;
    p.g_rs = dp_rs;
    p.x_rs = ds_rs;
    p.scale = scale;
    p.dsum = dsum;
    for (int k = 0; k < p.np; ++k) {
        p.y[k] = probs[k];
        p.g[k] = dprobs[k];
        p.out[k] = dscores[k];
    }
    return dispatch_rows(ATTN_DS, dtype, p, stream, "attn_dscores");
}

int pk_attn_dsum(int dtype, int degree, int64_t rows, int64_t cols, const void* const* dO, int64_t do_rs,
                 const void* const* O, int64_t o_rs, void* dsum, void* stream) {
    if (int rc = check_common(degree, rows, cols, "pk_attn_dsum")) return rc;
    if (!dsum || !dO || !O) return fail(PK_ERR_ARG, "pk_attn_dsum: null pointer");
    if (rows == 0) return PK_OK;
    DsumParams p{};
    p.np = degree + 1;
    p.rows = rows;
    p.cols = cols;
    p.do_rs = do_rs;
    p.o_rs = o_rs;
    p.dsum = dsum;
    for (int k = 0; k < p.np; ++k) {
        if (!dO[k] || !O[k]) return fail(PK_ERR_ARG, "pk_attn_dsum: null plane");
        p.dO[k] = dO[k];
        p.O[k] = O[k];
    }
    const int eb = elem_bytes(dtype);
    p.vec = (cols % ROW_VEC == 0 && row_vec_ok(p.dO, p.np, do_rs, eb) && row_vec_ok(p.O, p.np, o_rs, eb)) ? 1 : 0;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    void* tok;
    prof_begin("attn_dsum", s, &tok);
    switch (dtype) {
        case PK_F32: launch_dsum<float>(p, s); break;
        case PK_F64: launch_dsum<double>(p, s); break;
        case PK_BF16: launch_dsum<__nv_bfloat16>(p, s); break;
        case PK_F16: launch_dsum<__half>(p, s); break;
        default: return fail(PK_ERR_UNSUPPORTED, "pk_attn_dsum: unsupported dtype");
    }
    prof_end("attn_dsum", s, tok);
    PK_CHECK_LAUNCH("pk_attn_dsum");
    return PK_OK;
}

int pk_attn_probs_hilo(int degree, int64_t rows, int64_t cols, int64_t q_len, const void* const* scores, int64_t s_rs,
                       double scale, int causal, int64_t causal_shift, void* const* probs, int64_t p_rs, void* stats,
                       void* stream) {
    if (int rc = check_common(degree, rows, cols, "pk_attn_probs_hilo")) return rc;
    if (2 * (degree + 1) > PK_MAX_PLANES) return fail(PK_ERR_UNSUPPORTED, "pk_attn_probs_hilo: degree > 7");
    if (!stats || q_len <= 0) return fail(PK_ERR_ARG, "pk_attn_probs_hilo: null stats or bad q_len");
    SoftmaxParams p{};
    p.np = degree + 1;
    p.rows = rows;
    p.cols = cols;
    p.x_rs = s_rs;
    p.y_rs = p_rs;
    p.scale = scale;
    p.causal = causal;
    p.q_len = q_len;
    p.causal_shift = causal_shift;
    p.stats = stats;
    for (int k = 0; k < p.np; ++k) p.x[k] = scores[k];
    for (int k = 0; k < 2 * p.np; ++k) p.out[k] = probs[k];
    return dispatch_rows(ATTN_P_HILO, PK_F32, p, stream, "attn_probs");
}

int pk_attn_dscores_hilo(int degree, int64_t rows, int64_t cols, const void* const* probs, int64_t p_rs,
                         const void* const* dprobs, int64_t dp_rs, const void* dsum, double scale,
                         void* const* dscores, int64_t ds_rs, void* stream) {
    if (int rc = check_common(degree, rows, cols, "pk_attn_dscores_hilo")) return rc;
    if (2 * (degree + 1) > PK_MAX_PLANES) return fail(PK_ERR_UNSUPPORTED, "pk_attn_dscores_hilo: degree > 7");
    if (!dsum) return fail(PK_ERR_ARG, "pk_attn_dscores_hilo: null dsum");
    SoftmaxParams p{};
    p.np = degree + 1;
    p.rows = rows;
    p.cols = cols;
    p.y_rs = p_rs;
    p.g_rs = dp_rs;
    p.x_rs = ds_rs;
    p.scale = scale;
    p.dsum = dsum;
    for (int k = 0; k < p.np; ++k) p.g[k] = dprobs[k];
    for (int k = 0; k < 2 * p.np; ++k) {
        p.y[k] = probs[k];
        p.out[k] = dscores[k];
    }
    return dispatch_rows(ATTN_DS_HILO, PK_F32, p, stream, "attn_dscores");
}

}  // extern "C"
