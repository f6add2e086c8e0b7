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
#pragma unroll
    for (int k = 0; k < NP; ++k) {
        A s = A(0);
        for (int w = 0; w < nw; ++w) s += scratch[w * NP + k];
        v[k] = s;
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
