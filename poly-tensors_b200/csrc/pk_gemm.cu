// Polynomial (block-Toeplitz) matrix product  C_k = sum_{i+j=k} A_i B_j,  k = 0..n.
//
// Replaces plain_polynomial_product(matrix=True) (src/polytensors/_plain.py:118-128),
// which issues (n+1)(n+2)/2 separate GEMMs plus n(n+1)/2 full-size additions.  Here
// output plane k is one GEMM over a concatenated reduction axis: the k+1 products
// A_i B_{k-i} are accumulated in the same tensor-memory accumulator, so every output
// plane is written once and no partial sums ever reach HBM.
//
// Paths
//   float32 / bf16 / f16 : tcgen05.mma kind::f16 (TMEM accumulators, TMA-fed, persistent,
//                          warp-specialised).  float32 operands are split into bf16
//                          hi + lo; each product is a_hi b_hi + a_hi b_lo + a_lo b_hi.
//   float64 / complex128 : mma.sync m16n8k4 f64 (DMMA); a complex product is a sum of
//                          real products over planar re / im / -im sub-planes.
#include <algorithm>
#include <cstring>
#include <vector>

#include "pk_common.cuh"
#include "pk_gemm_prep.cuh"

namespace pk {

// =====================================================================================
// Operand staging (see pk_gemm_prep.cuh)

template <int KIND>
struct StageTraits;
template <>
struct StageTraits<STAGE_SPLIT_BF16> {
    using T = float;
    static constexpr int NOUT = 2;
};
template <>
struct StageTraits<STAGE_COPY_16> {
    using T = uint16_t;
    static constexpr int NOUT = 1;
};
template <>
struct StageTraits<STAGE_F64> {
    using T = double;
    static constexpr int NOUT = 1;
};
template <>
struct StageTraits<STAGE_C128_A> {
    using T = double2;
    static constexpr int NOUT = 3;
};
template <>
struct StageTraits<STAGE_C128_B> {
    using T = double2;
    static constexpr int NOUT = 2;
};

template <typename T>
__device__ __forceinline__ T zero_of() {
    return T{};
}

// Grid: x = ceil(Kp/64) k-tiles, y = ceil(rows/32) row tiles, z = batch * planes.
// Only planes whose kind equals KIND are processed by this instantiation.
template <int KIND>
__global__ void __launch_bounds__(256) stage_kernel(const StageParams p) {
    using T = typename StageTraits<KIND>::T;
    __shared__ T tile[32][65];
    const int z = blockIdx.z;
    const int pi = z % p.planes;
    const int64_t b = z / p.planes;
    const StagePlane pl = p.plane[pi];
    if (pl.kind != KIND) return;
    const T* src = static_cast<const T*>(pl.src) + b * p.s_b;
    const int64_t r0 = static_cast<int64_t>(blockIdx.y) * 32;
    const int64_t k0 = static_cast<int64_t>(blockIdx.x) * 64;
    const int t = threadIdx.x;

    if (p.s_k == 1 || p.s_r != 1) {
        // k is the fast index of the source (or neither is): threads sweep k.
        const int tx = t & 63, ty = t >> 6;
        for (int rr = ty; rr < 32; rr += 4) {
            const int64_t r = r0 + rr, k = k0 + tx;
            tile[rr][tx] = (r < p.rows && k < p.K) ? src[r * p.s_r + k * p.s_k] : zero_of<T>();
        }
    } else {
        // rows are the fast index of the source: threads sweep rows, then transpose.
        const int tx = t & 31, ty = t >> 5;
        for (int kk = ty; kk < 64; kk += 8) {
            const int64_t r = r0 + tx, k = k0 + kk;
            tile[tx][kk] = (r < p.rows && k < p.K) ? src[r * p.s_r + k * p.s_k] : zero_of<T>();
        }
    }
    __syncthreads();

    const int lane = t & 31, warp = t >> 5;
    const int64_t sub0 = b * p.subs_per_batch + pl.dst_sub;
    for (int rr = warp; rr < 32; rr += 8) {
        const int64_t r = r0 + rr;
        const int64_t k = k0 + 2 * lane;
        if (r >= p.rows || k >= p.Kp) continue;  // Kp is even, so k+1 < Kp as well
        const T v0 = tile[rr][2 * lane], v1 = tile[rr][2 * lane + 1];
        if constexpr (KIND == STAGE_SPLIT_BF16) {
            __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(p.dst);
            const __nv_bfloat16 h0 = __float2bfloat16_rn(v0), h1 = __float2bfloat16_rn(v1);
            const __nv_bfloat16 l0 = __float2bfloat16_rn(v0 - __bfloat162float(h0));
            const __nv_bfloat16 l1 = __float2bfloat16_rn(v1 - __bfloat162float(h1));
            const int64_t base_hi = ((sub0 + 0) * p.rows + r) * p.Kp + k;
            const int64_t base_lo = ((sub0 + 1) * p.rows + r) * p.Kp + k;
            *reinterpret_cast<__nv_bfloat162*>(dst + base_hi) = __halves2bfloat162(h0, h1);
            *reinterpret_cast<__nv_bfloat162*>(dst + base_lo) = __halves2bfloat162(l0, l1);
        } else if constexpr (KIND == STAGE_COPY_16) {
            uint16_t* dst = static_cast<uint16_t*>(p.dst);
            const int64_t base = (sub0 * p.rows + r) * p.Kp + k;
            *reinterpret_cast<uint32_t*>(dst + base) = static_cast<uint32_t>(v0) | (static_cast<uint32_t>(v1) << 16);
        } else if constexpr (KIND == STAGE_F64) {
            double* dst = static_cast<double*>(p.dst);
            const int64_t base = (sub0 * p.rows + r) * p.Kp + k;
            *reinterpret_cast<double2*>(dst + base) = make_double2(v0, v1);
        } else {
            double* dst = static_cast<double*>(p.dst);
            const int64_t base_re = ((sub0 + 0) * p.rows + r) * p.Kp + k;
            const int64_t base_im = ((sub0 + 1) * p.rows + r) * p.Kp + k;
            *reinterpret_cast<double2*>(dst + base_re) = make_double2(v0.x, v1.x);
            *reinterpret_cast<double2*>(dst + base_im) = make_double2(v0.y, v1.y);
            if constexpr (KIND == STAGE_C128_A) {
                const int64_t base_ni = ((sub0 + 2) * p.rows + r) * p.Kp + k;
                *reinterpret_cast<double2*>(dst + base_ni) = make_double2(-v0.y, -v1.y);
            }
        }
    }
}

// float32 -> bf16 hi/lo staging, fast paths.  split4 writes the hi/lo pairs of four
// consecutive k of one row (two 8-byte stores).
__device__ __forceinline__ void split4_store(__nv_bfloat16* hi, __nv_bfloat16* lo, const float (&v)[4]) {
    uint32_t h[2], l[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const __nv_bfloat16 h0 = __float2bfloat16_rn(v[2 * i]), h1 = __float2bfloat16_rn(v[2 * i + 1]);
        const __nv_bfloat16 l0 = __float2bfloat16_rn(v[2 * i] - __bfloat162float(h0));
        const __nv_bfloat16 l1 = __float2bfloat16_rn(v[2 * i + 1] - __bfloat162float(h1));
        h[i] = static_cast<uint32_t>(__bfloat16_as_ushort(h0)) | (static_cast<uint32_t>(__bfloat16_as_ushort(h1)) << 16);
        l[i] = static_cast<uint32_t>(__bfloat16_as_ushort(l0)) | (static_cast<uint32_t>(__bfloat16_as_ushort(l1)) << 16);
    }
    *reinterpret_cast<uint2*>(hi) = make_uint2(h[0], h[1]);
    *reinterpret_cast<uint2*>(lo) = make_uint2(l[0], l[1]);
}

// k contiguous in the source (s_k == 1): each source row (batch entry, plane, row) is a "line"
// of K floats.  A line gets `lpl` lanes (the power of two >= its 4-float groups, at most 32; a
// warp takes 32 / lpl lines at once), its indices are decoded once, and the lanes stride over its
// groups of four k: 16-byte loads when rows are 16-byte aligned, 8-byte hi and lo stores.
__global__ void __launch_bounds__(256) split_direct_kernel(const __grid_constant__ StageParams p, int64_t batch,
                                                           int vec, int lpl) {
    const int64_t kv = p.Kp / 4;
    const int64_t lines = batch * p.planes * p.rows;
    const int lane = threadIdx.x & 31;
    const int per_warp = 32 / lpl, sub = lane / lpl, j0 = lane % lpl;
    const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(p.dst);
    for (int64_t y = warp * per_warp + sub; y < lines; y += nwarps * per_warp) {
        const int64_t r = y % p.rows;
        const int64_t bp = y / p.rows;
        const int pi = static_cast<int>(bp % p.planes);
        const int64_t b = bp / p.planes;
        const StagePlane& pl = p.plane[pi];
        const float* src = static_cast<const float*>(pl.src) + b * p.s_b + r * p.s_r;
        const int64_t sub0 = b * p.subs_per_batch + pl.dst_sub;
        __nv_bfloat16* hi = dst + (sub0 * p.rows + r) * p.Kp;
        __nv_bfloat16* lo = dst + ((sub0 + 1) * p.rows + r) * p.Kp;
#pragma unroll 4
        for (int64_t jj = j0; jj < kv; jj += lpl) {
            const int64_t k = jj * 4;
            float v[4] = {0.f, 0.f, 0.f, 0.f};
            if (vec && k + 4 <= p.K) {
                const float4 t = *reinterpret_cast<const float4*>(src + k);
                v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
            } else {
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    if (k + i < p.K) v[i] = src[k + i];
            }
            split4_store(hi + k, lo + k, v);
        }
    }
}

// rows contiguous in the source (s_r == 1): a 64 x 64 tile is read along rows and written
// along k through shared memory.  grid: x = k tiles, y = row tiles, z = batch * planes.  With
// `vec` (16-byte aligned planes, s_k and s_b multiples of 4) a thread reads four rows of one k
// with one 16-byte load.
__global__ void __launch_bounds__(256) split_transpose_kernel(const __grid_constant__ StageParams p, int vec) {
    __shared__ float tile[64][65];
    const int z = blockIdx.z;
    const int pi = z % p.planes;
    const int64_t b = z / p.planes;
    const StagePlane& pl = p.plane[pi];
    const float* src = static_cast<const float*>(pl.src) + b * p.s_b;
    const int64_t r0 = static_cast<int64_t>(blockIdx.y) * 64, k0 = static_cast<int64_t>(blockIdx.x) * 64;
    const int t = threadIdx.x;
    if (vec && r0 + 64 <= p.rows) {
        const int tr = (t & 15) * 4, tk = t >> 4;  // 16 groups of four rows x 16 k per pass
#pragma unroll
        for (int kk = tk; kk < 64; kk += 16) {
            const int64_t k = k0 + kk;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (k < p.K) v = *reinterpret_cast<const float4*>(src + r0 + tr + k * p.s_k);
            tile[kk][tr] = v.x;
            tile[kk][tr + 1] = v.y;
            tile[kk][tr + 2] = v.z;
            tile[kk][tr + 3] = v.w;
        }
    } else {
        const int tr = t & 63, tk = t >> 6;  // 64 rows x 4 k per pass, rows fastest (coalesced)
        for (int kk = tk; kk < 64; kk += 4) {
            const int64_t r = r0 + tr, k = k0 + kk;
            tile[kk][tr] = (r < p.rows && k < p.K) ? src[r + k * p.s_k] : 0.f;
        }
    }
    __syncthreads();
    const int tk4 = (t & 15) * 4, tr = t >> 4;  // 16 rows x 16 four-k groups per pass
    __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(p.dst);
    const int64_t sub0 = b * p.subs_per_batch + pl.dst_sub;
    for (int rr = tr; rr < 64; rr += 16) {
        const int64_t r = r0 + rr, k = k0 + tk4;
        if (r >= p.rows || k >= p.Kp) continue;
        float v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = tile[tk4 + i][rr];
        split4_store(dst + (sub0 * p.rows + r) * p.Kp + k, dst + ((sub0 + 1) * p.rows + r) * p.Kp + k, v);
    }
}

// 16-bit copy staging (bf16 / f16 planes), fast paths: k contiguous -> 8-byte copies of four
// elements; rows contiguous -> 64 x 64 transpose through shared memory.
__global__ void __launch_bounds__(256) copy16_direct_kernel(const StageParams p, int64_t batch, int vec) {
    const int64_t kv = p.Kp / 4;
    const int64_t total = batch * p.planes * p.rows * kv;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t k = (i % kv) * 4;
        const int64_t y = i / kv;
        const int64_t r = y % p.rows;
        const int pi = static_cast<int>((y / p.rows) % p.planes);
        const int64_t b = y / (p.rows * p.planes);
        const StagePlane pl = p.plane[pi];
        const uint16_t* src = static_cast<const uint16_t*>(pl.src) + b * p.s_b + r * p.s_r;
        uint16_t v[4] = {0, 0, 0, 0};
        if (vec && k + 4 <= p.K) {
            const uint2 t = *reinterpret_cast<const uint2*>(src + k);
            v[0] = t.x & 0xFFFFu; v[1] = t.x >> 16; v[2] = t.y & 0xFFFFu; v[3] = t.y >> 16;
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (k + j < p.K) v[j] = src[k + j];
        }
        const int64_t sub0 = b * p.subs_per_batch + pl.dst_sub;
        uint16_t* dst = static_cast<uint16_t*>(p.dst) + (sub0 * p.rows + r) * p.Kp + k;
        *reinterpret_cast<uint2*>(dst) = make_uint2(static_cast<uint32_t>(v[0]) | (static_cast<uint32_t>(v[1]) << 16),
                                                    static_cast<uint32_t>(v[2]) | (static_cast<uint32_t>(v[3]) << 16));
    }
}

__global__ void __launch_bounds__(256) copy16_transpose_kernel(const StageParams p) {
    __shared__ uint16_t tile[64][66];
    const int z = blockIdx.z;
    const int pi = z % p.planes;
    const int64_t b = z / p.planes;
    const StagePlane pl = p.plane[pi];
    const uint16_t* src = static_cast<const uint16_t*>(pl.src) + b * p.s_b;
    const int64_t r0 = static_cast<int64_t>(blockIdx.y) * 64, k0 = static_cast<int64_t>(blockIdx.x) * 64;
    const int t = threadIdx.x;
    {
        const int tr = t & 63, tk = t >> 6;
        for (int kk = tk; kk < 64; kk += 4) {
            const int64_t r = r0 + tr, k = k0 + kk;
            tile[kk][tr] = (r < p.rows && k < p.K) ? src[r + k * p.s_k] : uint16_t(0);
        }
    }
    __syncthreads();
    const int tk4 = (t & 15) * 4, tr = t >> 4;
    uint16_t* dst = static_cast<uint16_t*>(p.dst);
    const int64_t sub0 = b * p.subs_per_batch + pl.dst_sub;
    for (int rr = tr; rr < 64; rr += 16) {
        const int64_t r = r0 + rr, k = k0 + tk4;
        if (r >= p.rows || k >= p.Kp) continue;
        *reinterpret_cast<uint2*>(dst + (sub0 * p.rows + r) * p.Kp + k) =
            make_uint2(static_cast<uint32_t>(tile[tk4][rr]) | (static_cast<uint32_t>(tile[tk4 + 1][rr]) << 16),
                       static_cast<uint32_t>(tile[tk4 + 2][rr]) | (static_cast<uint32_t>(tile[tk4 + 3][rr]) << 16));
    }
}

static int launch_stage(const StageParams& p, int64_t batch, bool has_kind[5], cudaStream_t stream) {
    if (has_kind[STAGE_COPY_16] && !has_kind[STAGE_SPLIT_BF16] && !has_kind[STAGE_F64] &&
        !has_kind[STAGE_C128_A] && !has_kind[STAGE_C128_B] && p.rows > 0 && p.Kp > 0 && batch > 0) {
        if (p.s_k == 1) {
            bool vec = p.s_r % 4 == 0 && p.s_b % 4 == 0;
            for (int k = 0; k < p.planes; ++k)
                if (reinterpret_cast<uintptr_t>(p.plane[k].src) % 8) vec = false;
            const int64_t total = batch * p.planes * p.rows * (p.Kp / 4);
            const int grid = static_cast<int>(std::min<int64_t>(ceil_div(total, 256), static_cast<int64_t>(num_sms()) * 32));
            PK_LAUNCHED(copy16_direct_kernel<<<grid, 256, 0, stream>>>(p, batch, vec ? 1 : 0));
            PK_CHECK_LAUNCH("pk_poly_gemm: copy kernel launch");
            return PK_OK;
        }
        if (p.s_r == 1 && ceil_div(p.rows, 64) <= 65535 && batch * p.planes <= 65535) {
            dim3 grid(static_cast<unsigned>(ceil_div(p.Kp, 64)), static_cast<unsigned>(ceil_div(p.rows, 64)),
                      static_cast<unsigned>(batch * p.planes));
            PK_LAUNCHED(copy16_transpose_kernel<<<grid, 256, 0, stream>>>(p));
            PK_CHECK_LAUNCH("pk_poly_gemm: copy transpose kernel launch");
            return PK_OK;
        }
    }
    if (has_kind[STAGE_SPLIT_BF16] && !has_kind[STAGE_COPY_16] && !has_kind[STAGE_F64] &&
        !has_kind[STAGE_C128_A] && !has_kind[STAGE_C128_B] && p.rows > 0 && p.Kp > 0 && batch > 0) {
        if (p.s_k == 1) {
            bool vec = p.s_r % 4 == 0 && p.s_b % 4 == 0;
            for (int k = 0; k < p.planes; ++k)
                if (reinterpret_cast<uintptr_t>(p.plane[k].src) % 16) vec = false;
            const int64_t kv = p.Kp / 4;
            int lpl = 1;
            while (lpl < 32 && lpl < kv) lpl <<= 1;
            const int64_t lines = batch * p.planes * p.rows;
            const int64_t warps = ceil_div(lines, 32 / lpl);
            const int grid = static_cast<int>(std::min<int64_t>(ceil_div(warps, 8), static_cast<int64_t>(num_sms()) * 16));
            PK_LAUNCHED(split_direct_kernel<<<grid, 256, 0, stream>>>(p, batch, vec ? 1 : 0, lpl));
            PK_CHECK_LAUNCH("pk_poly_gemm: split kernel launch");
            return PK_OK;
        }
        if (p.s_r == 1 && ceil_div(p.rows, 64) <= 65535 && batch * p.planes <= 65535) {
            dim3 grid(static_cast<unsigned>(ceil_div(p.Kp, 64)), static_cast<unsigned>(ceil_div(p.rows, 64)),
                      static_cast<unsigned>(batch * p.planes));
            bool vec = p.s_k % 4 == 0 && p.s_b % 4 == 0;
            for (int k = 0; k < p.planes; ++k)
                if (reinterpret_cast<uintptr_t>(p.plane[k].src) % 16) vec = false;
            PK_LAUNCHED(split_transpose_kernel<<<grid, 256, 0, stream>>>(p, vec ? 1 : 0));
            PK_CHECK_LAUNCH("pk_poly_gemm: split transpose kernel launch");
            return PK_OK;
        }
    }
    if (p.rows == 0 || p.Kp == 0 || batch == 0) return PK_OK;
    const int64_t gx = ceil_div(p.Kp, 64), gy = ceil_div(p.rows, 32), gz = batch * p.planes;
    if (gy > 65535 || gz > 65535) return fail(PK_ERR_UNSUPPORTED, "pk_poly_gemm: operand too large to stage");
    dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(gy), static_cast<unsigned>(gz));
    if (has_kind[STAGE_SPLIT_BF16]) PK_LAUNCHED(stage_kernel<STAGE_SPLIT_BF16><<<grid, 256, 0, stream>>>(p));
    if (has_kind[STAGE_COPY_16]) PK_LAUNCHED(stage_kernel<STAGE_COPY_16><<<grid, 256, 0, stream>>>(p));
    if (has_kind[STAGE_F64]) PK_LAUNCHED(stage_kernel<STAGE_F64><<<grid, 256, 0, stream>>>(p));
    if (has_kind[STAGE_C128_A]) PK_LAUNCHED(stage_kernel<STAGE_C128_A><<<grid, 256, 0, stream>>>(p));
    if (has_kind[STAGE_C128_B]) PK_LAUNCHED(stage_kernel<STAGE_C128_B><<<grid, 256, 0, stream>>>(p));
    PK_CHECK_LAUNCH("pk_poly_gemm: stage kernel launch");
    return PK_OK;
}

// =====================================================================================
// tcgen05 path

constexpr int TC_BM = 128;
// k blocks (of 64) accumulated in tensor memory before a float32 product adds the segment into
// its fp32 register sum (see the seg_iters comment in pk_poly_gemm)
#ifndef PK_F32_SEGMENT
#define PK_F32_SEGMENT 16
#endif
constexpr int PK_F32_SEGMENT_KBLOCKS = PK_F32_SEGMENT;
constexpr int TC_EPI_WARPS = 8;  // two per TMEM lane quadrant, each draining half of the columns
constexpr int TC_THREADS = 64 + 32 * TC_EPI_WARPS;  // warp 0: TMA, warp 1: MMA + TMEM owner, rest: epilogue
// The float32 (split) product keeps a tile's running fp32 sum in the epilogue's registers, so it
// has four epilogue warps per lane quadrant (a quarter of the columns each): at 256-column tiles
// that is 64 sums per thread, which fit beside the loads without spilling.
template <bool SPLIT>
struct TcWarps {
    static constexpr int EPI = SPLIT ? 16 : TC_EPI_WARPS;
    static constexpr int GROUPS = EPI / 4;  // column groups per lane quadrant
    static constexpr int THREADS = 64 + 32 * EPI;
};

// One tensor map per operand plane (3-D: k or rows innermost, then the other, then batch).
// float32 products use a[0] / b[0] only, over the whole staged workspace.
struct TcMaps {
    CUtensorMap a[PK_MAX_PLANES];
    CUtensorMap b[PK_MAX_PLANES];
};

struct TcParams {
    int planes, batch;
    int a_mn, b_mn;  // operand read MN-major (direct bf16 / f16 planes with rows contiguous)
    int in_fmt;      // MMA input format: 1 = bf16 (also the float32 hi/lo split), 0 = f16
    int M, N;
    int kblocks;
    int tiles_m, tiles_n, group_m;
    int total_tiles;
    int out_kind;  // 0 = f32, 1 = bf16, 2 = f16
    int vec_ok;    // output rows 16-byte aligned: vectorised stores allowed
    int accumulate;  // C += product (read-modify-write) instead of C = product
    int band;        // 0: every k; 1: only k >= m + band_off contributes; 2: only k <= m + band_off;
                     // 3: only outputs n <= m + band_off are needed (causal scores)
    int64_t band_off;
    int K;           // reduction length (banded k ranges)
    int seg_iters;   // float32 split: k-block iterations per accumulation segment (0 = one segment per tile)
    int a_pre, b_pre;  // float32 split: operand given as bf16 hi/lo planes read in place (maps 2i, 2i+1)
    int64_t c_bs, c_rs;
    void* c[PK_MAX_PLANES];
    int* status;
};

struct TileCoord {
    int plane, b, tm, tn;
};

// The k-th tile of this CTA.  Tiles come heaviest first (below), so a plain round robin gives the
// low-numbered CTAs the most work in every round; the boustrophedon order (snake_rank) alternates
// the direction each round, which evens out the per-CTA totals.
#ifndef PK_TC_SNAKE
#define PK_TC_SNAKE 1
#endif
__device__ __forceinline__ int tc_tile_rank(int k) {
    if constexpr (PK_TC_SNAKE != 0) return snake_rank(k);
    return k * static_cast<int>(gridDim.x) + static_cast<int>(blockIdx.x);
}

// Tiles are ordered heaviest first (output plane n has n+1 products), then by batch,
// then in groups of `group_m` row tiles so that CTAs running concurrently share
// operand tiles in L2.
__device__ __forceinline__ TileCoord decode_tile(const TcParams& p, int t) {
    TileCoord c;
    const int per_b = p.tiles_m * p.tiles_n;
    const int per_plane = p.batch * per_b;
    c.plane = p.planes - 1 - t / per_plane;
    int r = t % per_plane;
    c.b = r / per_b;
    r %= per_b;
    const int span = p.group_m * p.tiles_n;
    const int first_m = (r / span) * p.group_m;
    const int gsize = min(p.tiles_m - first_m, p.group_m);
    c.tm = first_m + (r % span) % gsize;
    c.tn = (r % span) / gsize;
    return c;
}

// The k blocks an output tile needs.  A banded product (a causal attention product) only has
// nonzeros for k >= m + off (band 1) or k <= m + off (band 2) in row m; k blocks entirely
// outside the band of every row of the tile are neither loaded nor multiplied.  Band 3 asks only
// for the outputs n <= m + off: tiles whose columns all lie beyond that get an empty range (their
// outputs are written as zeros, or left as they are when accumulating).
__device__ __forceinline__ void tile_kblocks(const TcParams& p, int tm, int tn, int bn, int& kb0, int& kb1) {
    kb0 = 0;
    kb1 = p.kblocks;
    if (p.band == 0) return;
    const int64_t m0 = static_cast<int64_t>(tm) * TC_BM;
    const int64_t m1 = (m0 + TC_BM - 1 < p.M - 1) ? m0 + TC_BM - 1 : static_cast<int64_t>(p.M) - 1;
    if (p.band == 3) {
        if (static_cast<int64_t>(tn) * bn > m1 + p.band_off) kb1 = 0;
        return;
    }
    if (p.band == 1) {
        const int64_t lo = m0 + p.band_off;
        const int64_t b = lo <= 0 ? 0 : lo / TC_BK;
        kb0 = static_cast<int>(b < p.kblocks ? b : p.kblocks);
    } else {
        int64_t hi = m1 + p.band_off;
        if (hi > static_cast<int64_t>(p.K) - 1) hi = static_cast<int64_t>(p.K) - 1;
        const int64_t b = hi < 0 ? 0 : hi / TC_BK + 1;
        kb1 = static_cast<int>(b < p.kblocks ? b : p.kblocks);
    }
}

template <int BN, bool SPLIT>
struct TcConfig {
    static constexpr int NSUB = SPLIT ? 2 : 1;
    static constexpr int A_BYTES = TC_BM * TC_BK * 2;
    static constexpr int B_BYTES = BN * TC_BK * 2;
    static constexpr int STAGE_BYTES = NSUB * (A_BYTES + B_BYTES);
    static constexpr int STAGES = (196 * 1024) / STAGE_BYTES;
    static constexpr int TMEM_COLS = 2 * BN;  // double-buffered accumulator
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
    static_assert(STAGES >= 2, "need at least two pipeline stages");
    static_assert(TMEM_COLS == 128 || TMEM_COLS == 256 || TMEM_COLS == 512, "TMEM allocation must be a power of two");
};

__device__ __forceinline__ void store_row_chunk(const TcParams& p, int plane, int b, int row, int col0,
                                                const uint32_t (&r)[32]) {
    if (row >= p.M) return;
    const int64_t off = static_cast<int64_t>(b) * p.c_bs + static_cast<int64_t>(row) * p.c_rs + col0;
    const bool full = (col0 + 32 <= p.N) && p.vec_ok;
    if (p.out_kind == 0) {
        float* dst = static_cast<float*>(p.c[plane]) + off;
        if (full) {
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
                float4 v = make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]), __uint_as_float(r[j + 2]),
                                       __uint_as_float(r[j + 3]));
                if (p.accumulate) {
                    const float4 o = *reinterpret_cast<const float4*>(dst + j);
                    v.x += o.x; v.y += o.y; v.z += o.z; v.w += o.w;
                }
                *reinterpret_cast<float4*>(dst + j) = v;
            }
        } else {
            for (int j = 0; j < 32 && col0 + j < p.N; ++j)
                dst[j] = __uint_as_float(r[j]) + (p.accumulate ? dst[j] : 0.f);
        }
    } else {
        uint16_t* dst = static_cast<uint16_t*>(p.c[plane]) + off;
        float prev[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) prev[j] = 0.f;
        if (p.accumulate) {
            if (full) {
#pragma unroll
                for (int j = 0; j < 32; j += 8) {
                    const uint4 o = *reinterpret_cast<const uint4*>(dst + j);
                    const uint32_t w[4] = {o.x, o.y, o.z, o.w};
#pragma unroll
                    for (int t = 0; t < 4; ++t) {
                        const uint16_t lo = static_cast<uint16_t>(w[t] & 0xFFFFu), hi = static_cast<uint16_t>(w[t] >> 16);
                        prev[j + 2 * t] = p.out_kind == 1 ? __bfloat162float(__ushort_as_bfloat16(lo))
                                                          : __half2float(__ushort_as_half(lo));
                        prev[j + 2 * t + 1] = p.out_kind == 1 ? __bfloat162float(__ushort_as_bfloat16(hi))
                                                              : __half2float(__ushort_as_half(hi));
                    }
                }
            } else {
                for (int j = 0; j < 32 && col0 + j < p.N; ++j)
                    prev[j] = p.out_kind == 1 ? __bfloat162float(__ushort_as_bfloat16(dst[j]))
                                              : __half2float(__ushort_as_half(dst[j]));
            }
        }
        uint32_t packed[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const float x0 = __uint_as_float(r[2 * j]) + prev[2 * j], x1 = __uint_as_float(r[2 * j + 1]) + prev[2 * j + 1];
            uint16_t h0, h1;
            if (p.out_kind == 1) {
                h0 = __bfloat16_as_ushort(__float2bfloat16_rn(x0));
                h1 = __bfloat16_as_ushort(__float2bfloat16_rn(x1));
            } else {
                h0 = __half_as_ushort(__float2half_rn(x0));
                h1 = __half_as_ushort(__float2half_rn(x1));
            }
            packed[j] = static_cast<uint32_t>(h0) | (static_cast<uint32_t>(h1) << 16);
        }
        if (full) {
#pragma unroll
            for (int j = 0; j < 16; j += 4)
                *reinterpret_cast<uint4*>(dst + 2 * j) = make_uint4(packed[j], packed[j + 1], packed[j + 2], packed[j + 3]);
        } else {
            for (int j = 0; j < 32 && col0 + j < p.N; ++j)
                dst[j] = static_cast<uint16_t>((packed[j / 2] >> (16 * (j & 1))) & 0xFFFFu);
        }
    }
}

// W = 32: store_row_chunk.  W = 16 (a quarter of a 64-column float32 tile): the first 16 values of
// r, float32 output (the only output kind of the split product).
__device__ __forceinline__ void store_row_chunk_n(const TcParams& p, int plane, int b, int row, int col0,
                                                  const uint32_t (&r)[32], int W) {
    if (W == 32) {
        store_row_chunk(p, plane, b, row, col0, r);
        return;
    }
    if (row >= p.M) return;
    const int64_t off = static_cast<int64_t>(b) * p.c_bs + static_cast<int64_t>(row) * p.c_rs + col0;
    float* dst = static_cast<float*>(p.c[plane]) + off;
    if ((col0 + 16 <= p.N) && p.vec_ok) {
#pragma unroll
        for (int j = 0; j < 16; j += 4) {
            float4 v = make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]), __uint_as_float(r[j + 2]),
                                   __uint_as_float(r[j + 3]));
            if (p.accumulate) {
                const float4 o = *reinterpret_cast<const float4*>(dst + j);
                v.x += o.x; v.y += o.y; v.z += o.z; v.w += o.w;
            }
            *reinterpret_cast<float4*>(dst + j) = v;
        }
    } else {
        for (int j = 0; j < 16 && col0 + j < p.N; ++j)
            dst[j] = __uint_as_float(r[j]) + (p.accumulate ? dst[j] : 0.f);
    }
}

template <int BN, bool SPLIT>
__global__ void __launch_bounds__(TcWarps<SPLIT>::THREADS, 1)
    tc_poly_gemm_kernel(const __grid_constant__ TcMaps maps, const TcParams p) {
    using Cfg = TcConfig<BN, SPLIT>;
    constexpr int STAGES = Cfg::STAGES;
    constexpr int NSUB = Cfg::NSUB;

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES);
    uint64_t* empty_bar = full_bar + STAGES;
    uint64_t* acc_full = empty_bar + STAGES;
    uint64_t* acc_empty = acc_full + 2;
    uint64_t* drain_bar = acc_empty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(&acc_full[s], 1);
            mbar_init(&acc_empty[s], 32 * TcWarps<SPLIT>::EPI);
        }
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        fence_mbar_init();
        const int nmaps = SPLIT ? 1 : p.planes;
        for (int i = 0; i < nmaps; ++i) {
            tma_prefetch_desc(&maps.a[i]);
            tma_prefetch_desc(&maps.b[i]);
        }
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            uint32_t stage = 0, phase = 0;
            int issued_parity[STAGES];
#pragma unroll
            for (int s = 0; s < STAGES; ++s) issued_parity[s] = -1;
            bool ok = true;
            for (int rk = 0, t = tc_tile_rank(0); t < p.total_tiles && ok; t = tc_tile_rank(++rk)) {
                const TileCoord tc = decode_tile(p, t);
                int kb0, kb1;
                tile_kblocks(p, tc.tm, tc.tn, BN, kb0, kb1);
                for (int i = 0; i <= tc.plane && ok; ++i) {
                    const int j = tc.plane - i;
                    for (int kb = kb0; kb < kb1; ++kb) {
                        if (!mbar_wait_or_abort(&empty_bar[stage], phase ^ 1, abort_flag, p.status, 101)) {
                            ok = false;
                            break;
                        }
                        uint8_t* st = smem + stage * Cfg::STAGE_BYTES;
                        mbar_arrive_expect_tx(&full_bar[stage], Cfg::STAGE_BYTES);
                        if constexpr (SPLIT) {
                            // staged workspace: z walks (batch, plane, hi/lo) sub-planes; a pre-split
                            // operand has one map per hi / lo plane, K-major or MN-major (64-row atoms)
                            const int za = (tc.b * p.planes + i) * NSUB;
                            const int zb = (tc.b * p.planes + j) * NSUB;
#pragma unroll
                            for (int h = 0; h < NSUB; ++h) {
                                uint8_t* dst = st + h * Cfg::A_BYTES;
                                if (!p.a_pre) {
                                    tma_load_3d(dst, &maps.a[0], &full_bar[stage], kb * TC_BK, tc.tm * TC_BM, za + h);
                                } else if (p.a_mn) {
#pragma unroll
                                    for (int hh = 0; hh < TC_BM / 64; ++hh)
                                        tma_load_3d(dst + hh * 8192, &maps.a[2 * i + h], &full_bar[stage],
                                                    tc.tm * TC_BM + hh * 64, kb * TC_BK, tc.b);
                                } else {
                                    tma_load_3d(dst, &maps.a[2 * i + h], &full_bar[stage], kb * TC_BK, tc.tm * TC_BM,
                                                tc.b);
                                }
                            }
#pragma unroll
                            for (int h = 0; h < NSUB; ++h) {
                                uint8_t* dst = st + NSUB * Cfg::A_BYTES + h * Cfg::B_BYTES;
                                if (!p.b_pre) {
                                    tma_load_3d(dst, &maps.b[0], &full_bar[stage], kb * TC_BK, tc.tn * BN, zb + h);
                                } else if (p.b_mn) {
#pragma unroll
                                    for (int hh = 0; hh < BN / 64; ++hh)
                                        tma_load_3d(dst + hh * 8192, &maps.b[2 * j + h], &full_bar[stage],
                                                    tc.tn * BN + hh * 64, kb * TC_BK, tc.b);
                                } else {
                                    tma_load_3d(dst, &maps.b[2 * j + h], &full_bar[stage], kb * TC_BK, tc.tn * BN, tc.b);
                                }
                            }
                        } else {
                            // one map per plane, z = batch; MN-major tiles arrive as 64-row atoms
                            if (p.a_mn) {
#pragma unroll
                                for (int h = 0; h < TC_BM / 64; ++h)
                                    tma_load_3d(st + h * 8192, &maps.a[i], &full_bar[stage], tc.tm * TC_BM + h * 64,
                                                kb * TC_BK, tc.b);
                            } else {
                                tma_load_3d(st, &maps.a[i], &full_bar[stage], kb * TC_BK, tc.tm * TC_BM, tc.b);
                            }
                            uint8_t* sb = st + Cfg::A_BYTES;
                            if (p.b_mn) {
#pragma unroll
                                for (int h = 0; h < BN / 64; ++h)
                                    tma_load_3d(sb + h * 8192, &maps.b[j], &full_bar[stage], tc.tn * BN + h * 64,
                                                kb * TC_BK, tc.b);
                            } else {
                                tma_load_3d(sb, &maps.b[j], &full_bar[stage], kb * TC_BK, tc.tn * BN, tc.b);
                            }
                        }
                        issued_parity[stage] = static_cast<int>(phase);
                        if (++stage == STAGES) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                }
            }
            if (!ok) {
                // Let copies already in flight land before the CTA (and its shared memory) exits:
                // the last load issued into stage s completes phase issued_parity[s] of full_bar[s].
                for (int s = 0; s < STAGES; ++s) {
                    if (issued_parity[s] < 0) continue;
                    const uint64_t t0 = pk_globaltimer();
                    while (!mbar_try_wait(&full_bar[s], static_cast<uint32_t>(issued_parity[s])) &&
                           pk_globaltimer() - t0 < 1000000000ull) {
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            // MN-major operands: transpose bits 15 (A) / 16 (B) of the instruction descriptor
            const uint32_t idesc = f16_idesc(static_cast<uint32_t>(p.in_fmt), TC_BM, BN) |
                                   (static_cast<uint32_t>(p.a_mn) << 15) | (static_cast<uint32_t>(p.b_mn) << 16);
            uint32_t stage = 0, phase = 0;
            uint32_t abuf = 0, aphase = 0;
            bool ok = true;
            bool issued = false;
            for (int rk = 0, t = tc_tile_rank(0); t < p.total_tiles && ok; t = tc_tile_rank(++rk)) {
                const TileCoord tc = decode_tile(p, t);
                int kb0, kb1;
                tile_kblocks(p, tc.tm, tc.tn, BN, kb0, kb1);
                if (kb1 <= kb0) continue;  // no k block in the band: the epilogue writes the zeros
                const int iters = (tc.plane + 1) * (kb1 - kb0);
                // float32: the reduction runs in segments of seg_iters k blocks, each into a fresh
                // accumulator (the two buffers alternate), summed by the epilogue in fp32 registers
                const int seg = (SPLIT && p.seg_iters > 0) ? p.seg_iters : iters;
                for (int s0 = 0; s0 < iters && ok; s0 += seg) {
                const int s1 = min(iters, s0 + seg);
                if (!mbar_wait_or_abort(&acc_empty[abuf], aphase ^ 1, abort_flag, p.status, 102)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + abuf * BN;
                for (int it = s0; it < s1; ++it) {
                    if (!mbar_wait_or_abort(&full_bar[stage], phase, abort_flag, p.status, 103)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t st = smem_u32(smem + stage * Cfg::STAGE_BYTES);
                    const uint32_t a_hi = st, a_lo = st + Cfg::A_BYTES;
                    const uint32_t b_hi = st + NSUB * Cfg::A_BYTES, b_lo = b_hi + Cfg::B_BYTES;
                    // descriptors built once per stage; a 16-wide k step advances the start address
                    // field: 32 bytes along a K-major swizzled row, 16 rows (2048 bytes) MN-major
                    const uint64_t ahd = p.a_mn ? sw128_mnmajor_desc_lbo(a_hi, 8192) : sw128_kmajor_desc(a_hi);
                    const uint64_t bhd = p.b_mn ? sw128_mnmajor_desc_lbo(b_hi, 8192) : sw128_kmajor_desc(b_hi);
                    const uint64_t a_step = p.a_mn ? (2048 >> 4) : (32 >> 4);
                    const uint64_t b_step = p.b_mn ? (2048 >> 4) : (32 >> 4);
#pragma unroll
                    for (int kk = 0; kk < TC_BK / 16; ++kk) {
                        tc_mma_f16(d_tmem, ahd + kk * a_step, bhd + kk * b_step, idesc, (it > s0 || kk > 0) ? 1u : 0u);
                        if constexpr (SPLIT) {
                            const uint64_t ald = p.a_mn ? sw128_mnmajor_desc_lbo(a_lo, 8192) : sw128_kmajor_desc(a_lo);
                            const uint64_t bld = p.b_mn ? sw128_mnmajor_desc_lbo(b_lo, 8192) : sw128_kmajor_desc(b_lo);
                            tc_mma_f16(d_tmem, ahd + kk * a_step, bld + kk * b_step, idesc, 1u);
                            tc_mma_f16(d_tmem, ald + kk * a_step, bhd + kk * b_step, idesc, 1u);
                        }
                    }
                    issued = true;
                    tc_commit(&empty_bar[stage]);  // frees this smem stage once the MMAs above retire
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (!ok) break;
                tc_commit(&acc_full[abuf]);  // accumulator (segment) ready for the epilogue
                if (++abuf == 2) {
                    abuf = 0;
                    aphase ^= 1;
                }
                }
            }
            if (!ok && issued) {
                // Drain: wait (bounded) until every MMA issued so far has retired, so that none
                // still writes TMEM or reads shared memory when the CTA releases them.
                tc_commit(drain_bar);
                const uint64_t t0 = pk_globaltimer();
                while (!mbar_try_wait(drain_bar, 0) && pk_globaltimer() - t0 < 1000000000ull) {
                }
            }
        }
    } else {
        // ---------------- epilogue: TMEM -> registers -> global ----------------
        // warp w drains lanes 32*(w%4).. (its TMEM lane quadrant) and column group (w-2)/4 (of two,
        // or four for the float32 product)
        const uint32_t lane_base = 32u * (warp & 3);
        const int half = (warp - 2) >> 2;
        uint32_t abuf = 0, aphase = 0;
        for (int rk = 0, t = tc_tile_rank(0); t < p.total_tiles; t = tc_tile_rank(++rk)) {
            const TileCoord tc = decode_tile(p, t);
            const int row = tc.tm * TC_BM + lane_base + lane;
            int kb0, kb1;
            tile_kblocks(p, tc.tm, tc.tn, BN, kb0, kb1);
            if (kb1 <= kb0) {
                // empty band: the product is zero (nothing to add when accumulating)
                if (!p.accumulate) {
                    uint32_t z[32];
#pragma unroll
                    for (int j = 0; j < 32; ++j) z[j] = 0u;
                    constexpr int GC = BN / TcWarps<SPLIT>::GROUPS;  // columns of this warp's group
                    for (int c = 0; c < GC; c += 32)
                        store_row_chunk_n(p, tc.plane, tc.b, row, tc.tn * BN + half * GC + c, z, GC < 32 ? GC : 32);
                }
                continue;
            }
            if constexpr (SPLIT) {
                // the tile's segments: each accumulator is read into registers and released at once,
                // the partial sums added with round-to-nearest fp32 adds; stores after the last one
                const int iters = (tc.plane + 1) * (kb1 - kb0);
                const int seg = p.seg_iters > 0 ? p.seg_iters : iters;
                const int nseg = (iters + seg - 1) / seg;
                constexpr int GC = BN / TcWarps<SPLIT>::GROUPS;  // this thread's columns: 64, 32 or 16
                constexpr int W = 16;                              // columns per TMEM load (registers)
                constexpr int CH = GC / W;
                float sum[CH][W];
#pragma unroll
                for (int c = 0; c < CH; ++c)
#pragma unroll
                    for (int j = 0; j < W; ++j) sum[c][j] = 0.f;
                bool ok = true;
                for (int sg = 0; sg < nseg; ++sg) {
                    if (!mbar_wait_or_abort(&acc_full[abuf], aphase, abort_flag, p.status, 104)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll
                    for (int c = 0; c < CH; ++c) {
                        uint32_t r[W];
                        const uint32_t taddr = tmem_base + (lane_base << 16) + abuf * BN + half * GC + c * W;
                        tmem_ld_32x32b_x16(taddr, r);
                        tmem_ld_wait();
#pragma unroll
                        for (int j = 0; j < W; ++j) sum[c][j] = __fadd_rn(sum[c][j], __uint_as_float(r[j]));
                    }
                    tc_fence_before();
                    mbar_arrive(&acc_empty[abuf]);
                    if (++abuf == 2) {
                        abuf = 0;
                        aphase ^= 1;
                    }
                }
                if (!ok) break;
#pragma unroll
                for (int c = 0; c < CH; ++c) {
                    uint32_t r[32];
#pragma unroll
                    for (int j = 0; j < W; ++j) r[j] = __float_as_uint(sum[c][j]);
                    store_row_chunk_n(p, tc.plane, tc.b, row, tc.tn * BN + half * GC + c * W, r, W);
                }
            } else {
            if (!mbar_wait_or_abort(&acc_full[abuf], aphase, abort_flag, p.status, 104)) break;
            tc_fence_after();
#pragma unroll 1
            for (int c = half * (BN / 64); c < (half + 1) * (BN / 64); ++c) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(tmem_base + (lane_base << 16) + abuf * BN + c * 32, r);
                tmem_ld_wait();
                store_row_chunk(p, tc.plane, tc.b, row, tc.tn * BN + c * 32, r);
            }
            tc_fence_before();
            mbar_arrive(&acc_empty[abuf]);
            if (++abuf == 2) {
                abuf = 0;
                aphase ^= 1;
            }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
    }
}

template <int BN, bool SPLIT>
static int launch_tc(TcParams& p, const TcOperand& a, const TcOperand& b, cudaStream_t stream) {
    using Cfg = TcConfig<BN, SPLIT>;
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(tc_poly_gemm_kernel<BN, SPLIT>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES);
        if (e != cudaSuccess) return cuda_fail(e, "pk_poly_gemm: cudaFuncSetAttribute");
        attr_set[dev] = true;
    }
    TcMaps maps;
    std::memset(&maps, 0, sizeof(maps));
    // float32 operands are staged (one map over the workspace) or pre-split hi/lo planes read in
    // place (one map per hi and lo plane)
    p.a_pre = (SPLIT && a.mode != OPM_STAGED) ? 1 : 0;
    p.b_pre = (SPLIT && b.mode != OPM_STAGED) ? 1 : 0;
    int rc = encode_operand(maps.a, a, p.a_pre ? 2 * p.planes : p.planes, SPLIT && !p.a_pre, TC_BM);
    if (rc) return rc;
    rc = encode_operand(maps.b, b, p.b_pre ? 2 * p.planes : p.planes, SPLIT && !p.b_pre, BN);
    if (rc) return rc;
    p.a_mn = a.mode == OPM_MNMAJOR ? 1 : 0;
    p.b_mn = b.mode == OPM_MNMAJOR ? 1 : 0;
    p.tiles_m = static_cast<int>(ceil_div(p.M, TC_BM));
    p.tiles_n = static_cast<int>(ceil_div(p.N, BN));
    // row-tile groups of 16: a wave of ~148 tiles spans 16 row tiles x ~9 column tiles, so each
    // operand panel is re-read by fewer waves than with a flat 8-row group (L2 reuse)
    p.group_m = 16;
    const int64_t total = static_cast<int64_t>(p.tiles_m) * p.tiles_n * p.batch * p.planes;
    if (total > 0x7fffffff) return fail(PK_ERR_UNSUPPORTED, "pk_poly_gemm: too many tiles");
    p.total_tiles = static_cast<int>(total);
    const int grid = static_cast<int>(std::min<int64_t>(total, num_sms()));
    void* tok;
    prof_begin("poly_gemm", stream, &tok);
    PK_LAUNCHED(tc_poly_gemm_kernel<BN, SPLIT><<<grid, TcWarps<SPLIT>::THREADS, Cfg::SMEM_BYTES, stream>>>(maps, p));
    prof_end("poly_gemm", stream, tok);
    PK_CHECK_LAUNCH("pk_poly_gemm: tcgen05 kernel launch");
    return PK_OK;
}

// =====================================================================================
// All-planes tcgen05 product (bf16 / f16 planes, degree <= 3)
//
// For output tile (b, tm, tn) the accumulators of EVERY output plane live in tensor memory
// (plane k at column k * AP_BN).  Per 64-wide k block the TMA warp loads each plane's A and B
// k-block once (n+1 ring stages) and the MMA warp issues all (n+1)(n+2)/2 products A_i B_j from
// them; the per-plane kernel above instead loads the operands of each product separately
// (sum_k (k+1) operand pairs per k block against n+1 here: 10 against 4 at degree 3), which makes
// narrow products (N = 128, e.g. attention head dimensions) L2-bandwidth bound.  The accumulator
// set (NP x 128 <= 512 columns) is single-buffered: the epilogue drains it and releases it before
// the next tile's products start, a small share of a tile when the reduction is long.

constexpr int AP_BN = 128;
constexpr int AP_A_BYTES = TC_BM * TC_BK * 2;
constexpr int AP_STAGE_BYTES = AP_A_BYTES + AP_BN * TC_BK * 2;  // one plane's A and B k-block
constexpr int AP_STAGES = 6;
constexpr int AP_SMEM_BYTES = AP_STAGES * AP_STAGE_BYTES + 1024 + 256;

__device__ __forceinline__ TileCoord ap_decode(const TcParams& p, int t) {
    TileCoord c;
    c.plane = 0;
    if (p.band == 1 || p.band == 2) {
        // banded product: a row tile's k-block count falls (band 1) or rises (band 2) with its
        // index, so row tiles in decreasing cost order, then batch entries, then column tiles
        // (dealt out with snake_rank, the CTAs' loads stay balanced)
        const int per_m = p.batch * p.tiles_n;
        const int i = t / per_m, rem = t % per_m;
        c.tm = p.band == 1 ? i : p.tiles_m - 1 - i;
        c.b = rem / p.tiles_n;
        c.tn = rem % p.tiles_n;
        return c;
    }
    // batch entry, then groups of group_m row tiles (CTAs running together share B tiles in L2)
    const int per_b = p.tiles_m * p.tiles_n;
    c.b = t / per_b;
    const int r = t % per_b;
    const int span = p.group_m * p.tiles_n;
    const int first_m = (r / span) * p.group_m;
    const int gsize = min(p.tiles_m - first_m, p.group_m);
    c.tm = first_m + (r % span) % gsize;
    c.tn = (r % span) / gsize;
    return c;
}

template <int NP>
__global__ void __launch_bounds__(TC_THREADS, 1)
    tc_allplanes_kernel(const __grid_constant__ TcMaps maps, const TcParams p) {
    constexpr int TMEM_COLS = NP * AP_BN <= 128 ? 128 : (NP * AP_BN <= 256 ? 256 : 512);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + AP_STAGES * AP_STAGE_BYTES);
    uint64_t* empty_bar = full_bar + AP_STAGES;
    uint64_t* acc_full = empty_bar + AP_STAGES;
    uint64_t* acc_empty = acc_full + 1;
    uint64_t* drain_bar = acc_empty + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < AP_STAGES; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        mbar_init(acc_full, 1);
        mbar_init(acc_empty, 32 * TC_EPI_WARPS);
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        fence_mbar_init();
        for (int i = 0; i < NP; ++i) {
            tma_prefetch_desc(&maps.a[i]);
            tma_prefetch_desc(&maps.b[i]);
        }
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer: plane i's A and B k-block into one ring stage ----------------
        if (lane == 0) {
            uint32_t stage = 0, phase = 0;
            int issued_parity[AP_STAGES];
#pragma unroll
            for (int s = 0; s < AP_STAGES; ++s) issued_parity[s] = -1;
            bool ok = true;
            for (int rk = 0, t = snake_rank(0); t < p.total_tiles && ok; t = snake_rank(++rk)) {
                const TileCoord tc = ap_decode(p, t);
                int kb0, kb1;
                tile_kblocks(p, tc.tm, tc.tn, AP_BN, kb0, kb1);
                for (int kb = kb0; kb < kb1 && ok; ++kb) {
                    for (int i = 0; i < NP; ++i) {
                        if (!mbar_wait_or_abort(&empty_bar[stage], phase ^ 1, abort_flag, p.status, 111)) {
                            ok = false;
                            break;
                        }
                        uint8_t* st = smem + stage * AP_STAGE_BYTES;
                        mbar_arrive_expect_tx(&full_bar[stage], AP_STAGE_BYTES);
                        if (p.a_mn) {
#pragma unroll
                            for (int h = 0; h < TC_BM / 64; ++h)
                                tma_load_3d(st + h * 8192, &maps.a[i], &full_bar[stage], tc.tm * TC_BM + h * 64,
                                            kb * TC_BK, tc.b);
                        } else {
                            tma_load_3d(st, &maps.a[i], &full_bar[stage], kb * TC_BK, tc.tm * TC_BM, tc.b);
                        }
                        uint8_t* sb = st + AP_A_BYTES;
                        if (p.b_mn) {
#pragma unroll
                            for (int h = 0; h < AP_BN / 64; ++h)
                                tma_load_3d(sb + h * 8192, &maps.b[i], &full_bar[stage], tc.tn * AP_BN + h * 64,
                                            kb * TC_BK, tc.b);
                        } else {
                            tma_load_3d(sb, &maps.b[i], &full_bar[stage], kb * TC_BK, tc.tn * AP_BN, tc.b);
                        }
                        issued_parity[stage] = static_cast<int>(phase);
                        if (++stage == AP_STAGES) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                }
            }
            if (!ok) {
                for (int s = 0; s < AP_STAGES; ++s) {
                    if (issued_parity[s] < 0) continue;
                    const uint64_t t0 = pk_globaltimer();
                    while (!mbar_try_wait(&full_bar[s], static_cast<uint32_t>(issued_parity[s])) &&
                           pk_globaltimer() - t0 < 1000000000ull) {
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer: all products of a k block from its NP resident stages ----------------
        if (lane == 0) {
            const uint32_t idesc = f16_idesc(static_cast<uint32_t>(p.in_fmt), TC_BM, AP_BN) |
                                   (static_cast<uint32_t>(p.a_mn) << 15) | (static_cast<uint32_t>(p.b_mn) << 16);
            const uint64_t a_step = p.a_mn ? (2048 >> 4) : (32 >> 4);
            const uint64_t b_step = p.b_mn ? (2048 >> 4) : (32 >> 4);
            uint32_t stage = 0, phase = 0, aphase = 0;
            bool ok = true, issued = false;
            for (int rk = 0, t = snake_rank(0); t < p.total_tiles && ok; t = snake_rank(++rk)) {
                const TileCoord tc = ap_decode(p, t);
                int kb0, kb1;
                tile_kblocks(p, tc.tm, tc.tn, AP_BN, kb0, kb1);
                if (kb1 <= kb0) continue;  // empty band: the epilogue writes the zeros
                if (!mbar_wait_or_abort(acc_empty, aphase ^ 1, abort_flag, p.status, 112)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                for (int kb = kb0; kb < kb1 && ok; ++kb) {
                    uint32_t st[NP];
#pragma unroll
                    for (int i = 0; i < NP; ++i) {
                        if (!mbar_wait_or_abort(&full_bar[stage], phase, abort_flag, p.status, 113)) {
                            ok = false;
                            break;
                        }
                        st[i] = stage;
                        if (++stage == AP_STAGES) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                    if (!ok) break;
                    tc_fence_after();
                    uint64_t ad[NP], bd[NP];
#pragma unroll
                    for (int i = 0; i < NP; ++i) {
                        const uint32_t a_s = smem_u32(smem + st[i] * AP_STAGE_BYTES);
                        const uint32_t b_s = a_s + AP_A_BYTES;
                        ad[i] = p.a_mn ? sw128_mnmajor_desc_lbo(a_s, 8192) : sw128_kmajor_desc(a_s);
                        bd[i] = p.b_mn ? sw128_mnmajor_desc_lbo(b_s, 8192) : sw128_kmajor_desc(b_s);
                    }
#pragma unroll
                    for (int k = 0; k < NP; ++k) {
#pragma unroll
                        for (int i = 0; i <= k; ++i) {
#pragma unroll
                            for (int kk = 0; kk < TC_BK / 16; ++kk)
                                tc_mma_f16(tmem_base + k * AP_BN, ad[i] + kk * a_step, bd[k - i] + kk * b_step, idesc,
                                           (kb > kb0 || i > 0 || kk > 0) ? 1u : 0u);
                        }
                    }
                    issued = true;
#pragma unroll
                    for (int i = 0; i < NP; ++i) tc_commit(&empty_bar[st[i]]);
                }
                if (!ok) break;
                tc_commit(acc_full);
                aphase ^= 1;
            }
            if (!ok && issued) {
                tc_commit(drain_bar);
                const uint64_t t0 = pk_globaltimer();
                while (!mbar_try_wait(drain_bar, 0) && pk_globaltimer() - t0 < 1000000000ull) {
                }
            }
        }
    } else {
        // ---------------- epilogue: every plane of the tile, TMEM -> registers -> global ----------------
        // warp w drains lanes 32*(w%4).. (its TMEM lane quadrant) and column half (w-2)/4 of each plane
        const uint32_t lane_base = 32u * (warp & 3);
        const int half = (warp - 2) >> 2;
        uint32_t aphase = 0;
        for (int rk = 0, t = snake_rank(0); t < p.total_tiles; t = snake_rank(++rk)) {
            const TileCoord tc = ap_decode(p, t);
            const int row = tc.tm * TC_BM + lane_base + lane;
            int kb0, kb1;
            tile_kblocks(p, tc.tm, tc.tn, AP_BN, kb0, kb1);
            if (kb1 <= kb0) {
                if (!p.accumulate) {
                    uint32_t z[32];
#pragma unroll
                    for (int j = 0; j < 32; ++j) z[j] = 0u;
                    for (int k = 0; k < NP; ++k)
                        for (int c = half * (AP_BN / 64); c < (half + 1) * (AP_BN / 64); ++c)
                            store_row_chunk(p, k, tc.b, row, tc.tn * AP_BN + c * 32, z);
                }
                continue;
            }
            if (!mbar_wait_or_abort(acc_full, aphase, abort_flag, p.status, 114)) break;
            tc_fence_after();
#pragma unroll 1
            for (int k = 0; k < NP; ++k) {
#pragma unroll 1
                for (int c = half * (AP_BN / 64); c < (half + 1) * (AP_BN / 64); ++c) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(tmem_base + (lane_base << 16) + k * AP_BN + c * 32, r);
                    tmem_ld_wait();
                    store_row_chunk(p, k, tc.b, row, tc.tn * AP_BN + c * 32, r);
                }
            }
            tc_fence_before();
            mbar_arrive(acc_empty);
            aphase ^= 1;
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

template <int NP>
static int launch_allplanes(TcParams& p, const TcOperand& a, const TcOperand& b, cudaStream_t stream) {
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(tc_allplanes_kernel<NP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             AP_SMEM_BYTES);
        if (e != cudaSuccess) return cuda_fail(e, "pk_poly_gemm: cudaFuncSetAttribute");
        attr_set[dev] = true;
    }
    TcMaps maps;
    std::memset(&maps, 0, sizeof(maps));
    int rc = encode_operand(maps.a, a, p.planes, false, TC_BM);
    if (rc) return rc;
    rc = encode_operand(maps.b, b, p.planes, false, AP_BN);
    if (rc) return rc;
    p.a_mn = a.mode == OPM_MNMAJOR ? 1 : 0;
    p.b_mn = b.mode == OPM_MNMAJOR ? 1 : 0;
    p.tiles_m = static_cast<int>(ceil_div(p.M, TC_BM));
    p.tiles_n = static_cast<int>(ceil_div(p.N, AP_BN));
    p.group_m = 8;
    const int64_t total = static_cast<int64_t>(p.tiles_m) * p.tiles_n * p.batch;
    if (total > 0x7fffffff) return fail(PK_ERR_UNSUPPORTED, "pk_poly_gemm: too many tiles");
    p.total_tiles = static_cast<int>(total);
    const int grid = static_cast<int>(std::min<int64_t>(total, num_sms()));
    void* tok;
    prof_begin("poly_gemm", stream, &tok);
    PK_LAUNCHED(tc_allplanes_kernel<NP><<<grid, TC_THREADS, AP_SMEM_BYTES, stream>>>(maps, p));
    prof_end("poly_gemm", stream, tok);
    PK_CHECK_LAUNCH("pk_poly_gemm: tcgen05 all-planes kernel launch");
    return PK_OK;
}

// =====================================================================================
// DMMA path (float64, complex128)

constexpr int DM_BM = 128, DM_BN = 128, DM_BK = 16, DM_LD = 20, DM_STAGES = 3;
constexpr int DM_THREADS = 256;
constexpr int DM_MAX_OUT = 2 * PK_MAX_PLANES;
constexpr int DM_MAX_SEG = 2 * PK_MAX_PLANES * (PK_MAX_PLANES + 1);

struct DmOut {
    double* ptr;   // plane base (as doubles)
    int mult;      // 1 for a float64 plane, 2 for an interleaved complex128 plane
    int part;      // 0 = real part / real plane, 1 = imaginary part
    int seg_begin, seg_end;
};

struct DmParams {
    int M, N;
    int batch;
    int64_t Kp;
    int kblocks;
    int n_out;
    int64_t a_subs, b_subs;  // sub-planes per batch entry
    const double* ws_a;
    const double* ws_b;
    int64_t c_bs, c_rs;
    DmOut out[DM_MAX_OUT];
    uint8_t seg_a[DM_MAX_SEG];
    uint8_t seg_b[DM_MAX_SEG];
    int order[DM_MAX_OUT];  // output sub-planes, heaviest first
    int accumulate;         // C += product
};

__device__ __forceinline__ void cp_async_16(void* smem, const void* gmem, bool valid) {
    const int n = valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem), "r"(n) : "memory");
}

__device__ __forceinline__ void dmma_16x8x4(double (&d)[4], double a0, double a1, double b0) {
    asm volatile(
        "mma.sync.aligned.m16n8k4.row.col.f64.f64.f64.f64 {%0, %1, %2, %3}, {%4, %5}, {%6}, {%0, %1, %2, %3};"
        : "+d"(d[0]), "+d"(d[1]), "+d"(d[2]), "+d"(d[3])
        : "d"(a0), "d"(a1), "d"(b0));
}

// Grid: x = N tiles, y = M tiles, z = batch * n_out (heaviest output sub-planes first).
__global__ void __launch_bounds__(DM_THREADS, 1) dmma_poly_gemm_kernel(const DmParams p) {
    extern __shared__ __align__(16) double dsm[];
    double* sA = dsm;                                 // [STAGES][BM][LD]
    double* sB = dsm + DM_STAGES * DM_BM * DM_LD;     // [STAGES][BN][LD]

    const int zo = blockIdx.z / p.batch;  // z = (output rank) * batch + b: heaviest outputs launch first
    const int64_t b = blockIdx.z % p.batch;
    const DmOut out = p.out[p.order[zo]];
    const int m0 = blockIdx.y * DM_BM, n0 = blockIdx.x * DM_BN;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int wm = warp >> 2, wn = warp & 3;  // 2 x 4 warps, 64 x 32 each
    const int g = lane >> 2, tg = lane & 3;

    double acc[4][4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[i][j][e] = 0.0;

    const int nseg = out.seg_end - out.seg_begin;
    const int total = nseg * p.kblocks;

    auto load_stage = [&](int it, int st) {
        const int s = out.seg_begin + it / p.kblocks;
        const int kb = it % p.kblocks;
        const double* ga = p.ws_a + ((b * p.a_subs + p.seg_a[s]) * p.M) * p.Kp + static_cast<int64_t>(kb) * DM_BK;
        const double* gb = p.ws_b + ((b * p.b_subs + p.seg_b[s]) * p.N) * p.Kp + static_cast<int64_t>(kb) * DM_BK;
        double* da = sA + st * DM_BM * DM_LD;
        double* db = sB + st * DM_BN * DM_LD;
#pragma unroll
        for (int c = tid; c < DM_BM * DM_BK / 2; c += DM_THREADS) {
            const int r = c >> 3, kc = (c & 7) * 2;
            const bool va = (m0 + r) < p.M;
            cp_async_16(da + r * DM_LD + kc, va ? ga + static_cast<int64_t>(m0 + r) * p.Kp + kc : p.ws_a, va);
            const bool vb = (n0 + r) < p.N;
            cp_async_16(db + r * DM_LD + kc, vb ? gb + static_cast<int64_t>(n0 + r) * p.Kp + kc : p.ws_b, vb);
        }
    };

#pragma unroll
    for (int s = 0; s < DM_STAGES - 1; ++s) {
        if (s < total) load_stage(s, s);
        cp_async_commit();
    }
    for (int it = 0; it < total; ++it) {
        cp_async_wait<DM_STAGES - 2>();
        __syncthreads();
        const int nxt = it + DM_STAGES - 1;
        if (nxt < total) load_stage(nxt, nxt % DM_STAGES);
        cp_async_commit();
        const double* a = sA + (it % DM_STAGES) * DM_BM * DM_LD + (wm * 64) * DM_LD;
        const double* bb = sB + (it % DM_STAGES) * DM_BN * DM_LD + (wn * 32) * DM_LD;
#pragma unroll
        for (int kk = 0; kk < DM_BK; kk += 4) {
            double af[4][2], bf[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                af[i][0] = a[(i * 16 + g) * DM_LD + kk + tg];
                af[i][1] = a[(i * 16 + g + 8) * DM_LD + kk + tg];
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) bf[j] = bb[(j * 8 + g) * DM_LD + kk + tg];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) dmma_16x8x4(acc[i][j], af[i][0], af[i][1], bf[j]);
        }
    }
    cp_async_wait<0>();

    // Epilogue: rows g / g+8, columns 2*tg, 2*tg+1 of each 16 x 8 fragment.
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int row = m0 + wm * 64 + i * 16 + g + ((e >> 1) ? 8 : 0);
                const int col = n0 + wn * 32 + j * 8 + tg * 2 + (e & 1);
                if (row < p.M && col < p.N) {
                    const int64_t idx = b * p.c_bs + static_cast<int64_t>(row) * p.c_rs + col;
                    double* dst = out.ptr + idx * out.mult + out.part;
                    *dst = acc[i][j][e] + (p.accumulate ? *dst : 0.0);
                }
            }
        }
    }
}

// Zero-fill output planes for K == 0 (an empty sum).
__global__ void zero_planes_kernel(void* const* planes_dev_unused, char* base, int64_t rows, int64_t cols,
                                   int64_t rs, int64_t bs, int64_t batch, int elem_bytes) {
    const int64_t total = batch * rows * cols;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t b = i / (rows * cols), r = (i / cols) % rows, c = i % cols;
        char* dst = base + (b * bs + r * rs + c) * elem_bytes;
        for (int e = 0; e < elem_bytes; ++e) dst[e] = 0;
    }
}

static int elem_size(int dtype) {
    switch (dtype) {
        case PK_F32: return 4;
        case PK_F64: return 8;
        case PK_BF16:
        case PK_F16: return 2;
        case PK_C128: return 16;
    }
    return 0;
}

struct GemmPlan {
    int a_mode = OPM_STAGED, b_mode = OPM_STAGED;
    bool unaddressable = false;  // a pre-split (hi/lo) operand the tensor maps cannot read in place
    int64_t Kp = 0;
    int64_t a_subs = 0, b_subs = 0;  // per batch entry
    size_t a_bytes = 0, b_bytes = 0, total = 0;
    std::vector<int> a_first, b_first;  // first sub-plane of each plane
};

static GemmPlan plan_gemm(int dtype, int degree, int64_t batch, int64_t M, int64_t N, int64_t K, int acf, int bcf) {
    GemmPlan g;
    const int P = degree + 1;
    g.a_first.resize(P);
    g.b_first.resize(P);
    int64_t esz;
    if (dtype == PK_F32 || dtype == PK_BF16 || dtype == PK_F16) {
        g.Kp = round_up(std::max<int64_t>(K, 1), 8);
        const int ns = dtype == PK_F32 ? 2 : 1;
        for (int p = 0; p < P; ++p) {
            g.a_first[p] = p * ns;
            g.b_first[p] = p * ns;
        }
        g.a_subs = g.b_subs = static_cast<int64_t>(P) * ns;
        esz = 2;
    } else {
        g.Kp = round_up(std::max<int64_t>(K, 1), 16);
        for (int p = 0; p < P; ++p) {
            const bool ca = dtype == PK_C128 && p >= acf, cb = dtype == PK_C128 && p >= bcf;
            g.a_first[p] = static_cast<int>(g.a_subs);
            g.a_subs += ca ? 3 : 1;
            g.b_first[p] = static_cast<int>(g.b_subs);
            g.b_subs += cb ? 2 : 1;
        }
        esz = 8;
    }
    g.a_bytes = static_cast<size_t>(round_up(batch * g.a_subs * M * g.Kp * esz, 1024));
    g.b_bytes = static_cast<size_t>(round_up(batch * g.b_subs * N * g.Kp * esz, 1024));
    g.total = g.a_bytes + g.b_bytes + 1024;  // +1024: alignment slack for the caller's pointer
    return g;
}

// The plan for one call: operands read in place need no workspace.
// float32 operands may come pre-split (a_hilo / b_hilo): 2(n+1) bf16 planes hi_0, lo_0, hi_1, ...
// read in place, so they are never staged.
static GemmPlan plan_call(int dtype, int degree, int64_t batch, int64_t M, int64_t N, int64_t K, int acf, int bcf,
                          const void* const* a_planes, int64_t a_bs, int64_t a_rs, int64_t a_cs,
                          const void* const* b_planes, int64_t b_bs, int64_t b_rs, int64_t b_cs, int a_hilo = 0,
                          int b_hilo = 0) {
    GemmPlan g = plan_gemm(dtype, degree, batch, M, N, K, acf, bcf);
    const int P = degree + 1;
    g.a_mode = a_hilo ? operand_mode(PK_BF16, a_planes, 2 * P, batch, M, K, a_bs, a_rs, a_cs)
                      : operand_mode(dtype, a_planes, P, batch, M, K, a_bs, a_rs, a_cs);
    g.b_mode = b_hilo ? operand_mode(PK_BF16, b_planes, 2 * P, batch, N, K, b_bs, b_cs, b_rs)
                      : operand_mode(dtype, b_planes, P, batch, N, K, b_bs, b_cs, b_rs);
    g.unaddressable = (a_hilo && g.a_mode == OPM_STAGED) || (b_hilo && g.b_mode == OPM_STAGED);
    if (g.a_mode != OPM_STAGED) g.a_bytes = 0;
    if (g.b_mode != OPM_STAGED) g.b_bytes = 0;
    g.total = (g.a_bytes + g.b_bytes) ? g.a_bytes + g.b_bytes + 1024 : 0;
    return g;
}

}  // namespace pk

using namespace pk;

extern "C" {

int pk_poly_gemm_workspace_query(int dtype, int degree, int64_t batch, int64_t M, int64_t N, int64_t K,
                                 const void* const* a_planes, int64_t a_bs, int64_t a_rs, int64_t a_cs,
                                 const void* const* b_planes, int64_t b_bs, int64_t b_rs, int64_t b_cs,
                                 int a_complex_from, int b_complex_from, size_t* bytes) {
    if (!bytes) return fail(PK_ERR_ARG, "pk_poly_gemm_workspace_query: null result pointer");
    *bytes = 0;
    if (degree < 0 || degree >= PK_MAX_PLANES || batch < 0 || M < 0 || N < 0 || K < 0 || elem_size(dtype) == 0)
        return fail(PK_ERR_ARG, "pk_poly_gemm_workspace_query: invalid dtype, degree or size");
    if (batch == 0 || M == 0 || N == 0 || K == 0) return PK_OK;  // nothing is staged
    if (!a_planes || !b_planes) return fail(PK_ERR_ARG, "pk_poly_gemm_workspace_query: null operand plane array");
    for (int p = 0; p <= degree; ++p)
        if (!a_planes[p] || !b_planes[p])
            return fail(PK_ERR_ARG, "pk_poly_gemm_workspace_query: null operand plane pointer");
    *bytes = plan_call(dtype, degree, batch, M, N, K, a_complex_from, b_complex_from, a_planes, a_bs, a_rs, a_cs,
                       b_planes, b_bs, b_rs, b_cs)
                 .total;
    return PK_OK;
}

size_t pk_poly_gemm_workspace_size(int dtype, int degree, int64_t batch, int64_t M, int64_t N, int64_t K,
                                   int a_complex_from, int b_complex_from) {
    if (degree < 0 || degree >= PK_MAX_PLANES || batch < 0 || M < 0 || N < 0 || K < 0) return 0;
    if (elem_size(dtype) == 0) return 0;
    return plan_gemm(dtype, degree, batch, M, N, K, a_complex_from, b_complex_from).total;
}

}  // extern "C"

namespace pk {

static int poly_gemm(int dtype, int degree, int64_t batch, int64_t M, int64_t N, int64_t K, const void* const* a_planes,
                     int64_t a_bs, int64_t a_rs, int64_t a_cs, const void* const* b_planes, int64_t b_bs, int64_t b_rs,
                     int64_t b_cs, void* const* c_planes, int64_t c_bs, int64_t c_rs, int a_complex_from,
                     int b_complex_from, void* workspace, size_t workspace_bytes, void* stream_ptr, int accumulate,
                     int band = 0, int64_t band_off = 0, int a_hilo = 0, int b_hilo = 0) {
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    if (degree < 0 || degree >= PK_MAX_PLANES)
        return fail(PK_ERR_UNSUPPORTED, "pk_poly_gemm: degree must be in [0, " + std::to_string(PK_MAX_PLANES - 1) + "]");
    if (batch < 0 || M < 0 || N < 0 || K < 0) return fail(PK_ERR_ARG, "pk_poly_gemm: negative size");
    const int esz = elem_size(dtype);
    if (esz == 0) return fail(PK_ERR_UNSUPPORTED, "pk_poly_gemm: unknown dtype " + std::to_string(dtype));
    if (M > 0x7fffffff || N > 0x7fffffff || K > 0x7fffffff)
        return fail(PK_ERR_UNSUPPORTED, "pk_poly_gemm: dimension exceeds 2^31-1");
    const int P = degree + 1;
    if (dtype != PK_C128) {
        a_complex_from = P;
        b_complex_from = P;
    } else {
        a_complex_from = std::max(0, std::min(a_complex_from, P));
        b_complex_from = std::max(0, std::min(b_complex_from, P));
    }
    if (batch == 0 || M == 0 || N == 0) return PK_OK;  // empty output: nothing to read or write
    if (!c_planes) return fail(PK_ERR_ARG, "pk_poly_gemm: null output plane array");
    for (int p = 0; p < P; ++p)
        if (!c_planes[p]) return fail(PK_ERR_ARG, "pk_poly_gemm: null output plane pointer");

    if (K == 0) {  // empty reduction: the operands may have no storage at all
        if (accumulate) return PK_OK;
        for (int p = 0; p < P; ++p) {
            const bool cplx = dtype == PK_C128 && (p >= a_complex_from || p >= b_complex_from);
            const int e = dtype == PK_C128 ? (cplx ? 16 : 8) : esz;
            PK_LAUNCHED(zero_planes_kernel<<<592, 256, 0, stream>>>(nullptr, static_cast<char*>(c_planes[p]), M, N, c_rs, c_bs,
                                                        batch, e));
        }
        PK_CHECK_LAUNCH("pk_poly_gemm: zero fill");
        return PK_OK;
    }

    if (!a_planes || !b_planes) return fail(PK_ERR_ARG, "pk_poly_gemm: null operand plane array");
    if ((a_hilo || b_hilo) && (dtype != PK_F32 || 2 * P > PK_MAX_PLANES))
        return fail(PK_ERR_UNSUPPORTED, "pk_poly_gemm_hilo: pre-split operands are float32 products of degree <= 7");
    for (int p = 0; p < (a_hilo ? 2 * P : P); ++p)
        if (!a_planes[p]) return fail(PK_ERR_ARG, "pk_poly_gemm: null operand plane pointer");
    for (int p = 0; p < (b_hilo ? 2 * P : P); ++p)
        if (!b_planes[p]) return fail(PK_ERR_ARG, "pk_poly_gemm: null operand plane pointer");
    const GemmPlan g = plan_call(dtype, degree, batch, M, N, K, a_complex_from, b_complex_from, a_planes, a_bs, a_rs,
                                 a_cs, b_planes, b_bs, b_rs, b_cs, a_hilo, b_hilo);
    if (g.unaddressable)
        return fail(PK_ERR_UNSUPPORTED,
                    "pk_poly_gemm_hilo: pre-split planes need 16-byte aligned bases, k or rows contiguous and the "
                    "other strides multiples of 8 elements");
    if (g.total > 0 && (!workspace || workspace_bytes < g.total))
        return fail(PK_ERR_WORKSPACE, "pk_poly_gemm: workspace of " + std::to_string(g.total) + " bytes required");
    char* ws = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(workspace) + 1023) & ~uintptr_t(1023));
    void* ws_a = ws;
    void* ws_b = ws + g.a_bytes;

    // ---- stage operands into K-major sub-planes
    StageParams sa{}, sb{};
    bool kinds_a[5] = {false, false, false, false, false}, kinds_b[5] = {false, false, false, false, false};
    for (int p = 0; p < P; ++p) {
        int ka, kb;
        if (dtype == PK_F32) ka = kb = STAGE_SPLIT_BF16;
        else if (dtype == PK_BF16 || dtype == PK_F16) ka = kb = STAGE_COPY_16;
        else {
            ka = (dtype == PK_C128 && p >= a_complex_from) ? STAGE_C128_A : STAGE_F64;
            kb = (dtype == PK_C128 && p >= b_complex_from) ? STAGE_C128_B : STAGE_F64;
        }
        sa.plane[p] = {a_planes[p], g.a_first[p], ka};
        sb.plane[p] = {b_planes[p], g.b_first[p], kb};
        kinds_a[ka] = true;
        kinds_b[kb] = true;
    }
    sa.planes = sb.planes = P;
    sa.rows = M; sa.K = K; sa.Kp = g.Kp; sa.s_b = a_bs; sa.s_r = a_rs; sa.s_k = a_cs;
    sa.subs_per_batch = g.a_subs; sa.dst = ws_a;
    sb.rows = N; sb.K = K; sb.Kp = g.Kp; sb.s_b = b_bs; sb.s_r = b_cs; sb.s_k = b_rs;
    sb.subs_per_batch = g.b_subs; sb.dst = ws_b;
    sa.elem_bytes = sb.elem_bytes = (dtype == PK_F64 || dtype == PK_C128) ? 8 : 2;
    int rc = g.a_mode == OPM_STAGED ? launch_stage(sa, batch, kinds_a, stream) : PK_OK;
    if (rc) return rc;
    rc = g.b_mode == OPM_STAGED ? launch_stage(sb, batch, kinds_b, stream) : PK_OK;
    if (rc) return rc;

    if (dtype == PK_F32 || dtype == PK_BF16 || dtype == PK_F16) {
        if (batch * P * 2 > 0x7fffffff) return fail(PK_ERR_UNSUPPORTED, "pk_poly_gemm: batch too large");
        TcParams tp{};
        tp.planes = P;
        tp.batch = static_cast<int>(batch);
        tp.M = static_cast<int>(M);
        tp.N = static_cast<int>(N);
        tp.kblocks = static_cast<int>(ceil_div(g.Kp, TC_BK));
        tp.out_kind = dtype == PK_F32 ? 0 : (dtype == PK_BF16 ? 1 : 2);
        tp.c_bs = c_bs;
        tp.c_rs = c_rs;
        const int align_elems = 16 / esz;
        bool vec = (c_rs % align_elems == 0) && (c_bs % align_elems == 0);
        for (int p = 0; p < P; ++p) {
            tp.c[p] = c_planes[p];
            if (reinterpret_cast<uintptr_t>(c_planes[p]) % 16 != 0) vec = false;
        }
        tp.vec_ok = vec ? 1 : 0;
        tp.accumulate = accumulate;
        tp.band = band;
        tp.band_off = band_off;
        tp.K = static_cast<int>(K);
        // float32: the tensor core's fp32 accumulation loses precision in proportion to the number
        // of k steps summed into one accumulator (measured: plane error ~3.7e-9 per k element at
        // 8192^3, i.e. 1.4e-4 at degree 4), so the reduction of an output tile runs in segments of
        // PK_F32_SEGMENT_KBLOCKS 64-wide k blocks whose results are added in fp32 registers
        tp.seg_iters = dtype == PK_F32 ? PK_F32_SEGMENT_KBLOCKS : 0;
        tp.status = device_status_ptr();
        const int64_t tiles256 = ceil_div(M, TC_BM) * ceil_div(N, 256) * batch * P;
        // 256-column tiles when N fills them (a 128-wide N would leave half of every MMA on the
        // zero fill past N) and there are at least two such tiles per SM
        const bool wide = tiles256 >= 2 * num_sms() && N > 192;
        const bool f16 = dtype == PK_F16;
        const TcOperand oa{g.a_mode, M, K, g.Kp, batch, a_planes, a_bs, a_rs, a_cs,
                           static_cast<const char*>(ws_a), g.a_first.data(), g.a_subs, f16};
        const TcOperand ob{g.b_mode, N, K, g.Kp, batch, b_planes, b_bs, b_cs, b_rs,
                           static_cast<const char*>(ws_b), g.b_first.data(), g.b_subs, f16};
        tp.in_fmt = f16 ? 0 : 1;
        // N <= 64 (e.g. attention head dimensions): 64-column tiles; a 128-column tile would spend
        // half of every MMA on the zero fill beyond N
        const bool narrow = N <= 64;
        if (dtype == PK_F32) {
            if (narrow) return launch_tc<64, true>(tp, oa, ob, stream);
            return wide ? launch_tc<256, true>(tp, oa, ob, stream) : launch_tc<128, true>(tp, oa, ob, stream);
        }
        // degree <= 3 with enough output tiles: every plane of a tile at once (operands loaded once
        // per k block for all products)
        const int64_t ap_tiles = ceil_div(M, TC_BM) * ceil_div(N, AP_BN) * batch;
        if (P >= 2 && P <= 4 && ap_tiles >= num_sms()) {
            switch (P) {
                case 2: return launch_allplanes<2>(tp, oa, ob, stream);
                case 3: return launch_allplanes<3>(tp, oa, ob, stream);
                default: return launch_allplanes<4>(tp, oa, ob, stream);
            }
        }
        if (narrow) return launch_tc<64, false>(tp, oa, ob, stream);
        return wide ? launch_tc<256, false>(tp, oa, ob, stream) : launch_tc<128, false>(tp, oa, ob, stream);
    }

    // ---- DMMA path: build the per-output segment lists
    DmParams dp{};
    dp.M = static_cast<int>(M);
    dp.N = static_cast<int>(N);
    dp.batch = static_cast<int>(batch);
    dp.Kp = g.Kp;
    dp.kblocks = static_cast<int>(g.Kp / DM_BK);
    dp.a_subs = g.a_subs;
    dp.b_subs = g.b_subs;
    dp.ws_a = static_cast<const double*>(ws_a);
    dp.ws_b = static_cast<const double*>(ws_b);
    dp.c_bs = c_bs;
    dp.c_rs = c_rs;
    dp.accumulate = accumulate;
    int nseg = 0, nout = 0;
    for (int k = 0; k < P; ++k) {
        const bool out_complex = dtype == PK_C128 && (k >= a_complex_from || k >= b_complex_from);
        for (int part = 0; part < (out_complex ? 2 : 1); ++part) {
            DmOut& o = dp.out[nout];
            o.ptr = static_cast<double*>(c_planes[k]);
            o.mult = out_complex ? 2 : 1;
            o.part = part;
            o.seg_begin = nseg;
            for (int i = 0; i <= k; ++i) {
                const int j = k - i;
                const bool ca = dtype == PK_C128 && i >= a_complex_from;
                const bool cb = dtype == PK_C128 && j >= b_complex_from;
                const int ar = g.a_first[i], ai = ar + 1, ani = ar + 2;
                const int br = g.b_first[j], bi = br + 1;
                auto add = [&](int sa_, int sb_) {
                    dp.seg_a[nseg] = static_cast<uint8_t>(sa_);
                    dp.seg_b[nseg] = static_cast<uint8_t>(sb_);
                    ++nseg;
                };
                if (part == 0) {  // real part: re*re - im*im
                    add(ar, br);
                    if (ca && cb) add(ani, bi);
                } else {  // imaginary part: re*im + im*re
                    if (cb) add(ar, bi);
                    if (ca) add(ai, br);
                }
            }
            o.seg_end = nseg;
            ++nout;
        }
    }
    dp.n_out = nout;
    std::vector<int> order(nout);
    for (int i = 0; i < nout; ++i) order[i] = i;
    std::stable_sort(order.begin(), order.end(), [&](int x, int y) {
        return (dp.out[x].seg_end - dp.out[x].seg_begin) > (dp.out[y].seg_end - dp.out[y].seg_begin);
    });
    for (int i = 0; i < nout; ++i) dp.order[i] = order[i];
    const int smem = DM_STAGES * (DM_BM + DM_BN) * DM_LD * static_cast<int>(sizeof(double));
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(dmma_poly_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return cuda_fail(e, "pk_poly_gemm: cudaFuncSetAttribute (dmma)");
        attr_set[dev] = true;
    }
    const int64_t gz = batch * nout;
    if (gz > 65535 || ceil_div(M, DM_BM) > 65535) return fail(PK_ERR_UNSUPPORTED, "pk_poly_gemm: grid too large");
    dim3 grid(static_cast<unsigned>(ceil_div(N, DM_BN)), static_cast<unsigned>(ceil_div(M, DM_BM)),
              static_cast<unsigned>(gz));
    void* tok;
    prof_begin("poly_gemm", stream, &tok);
    PK_LAUNCHED(dmma_poly_gemm_kernel<<<grid, DM_THREADS, smem, stream>>>(dp));
    prof_end("poly_gemm", stream, tok);
    PK_CHECK_LAUNCH("pk_poly_gemm: dmma kernel launch");
    return PK_OK;
}

}  // namespace pk

extern "C" {

int pk_poly_gemm(int dtype, int degree, int64_t batch, int64_t M, int64_t N, int64_t K, const void* const* a_planes,
                 int64_t a_bs, int64_t a_rs, int64_t a_cs, const void* const* b_planes, int64_t b_bs, int64_t b_rs,
                 int64_t b_cs, void* const* c_planes, int64_t c_bs, int64_t c_rs, int a_complex_from,
                 int b_complex_from, void* workspace, size_t workspace_bytes, void* stream) {
    return poly_gemm(dtype, degree, batch, M, N, K, a_planes, a_bs, a_rs, a_cs, b_planes, b_bs, b_rs, b_cs, c_planes,
                     c_bs, c_rs, a_complex_from, b_complex_from, workspace, workspace_bytes, stream, 0);
}

int pk_poly_gemm_banded(int dtype, int degree, int64_t batch, int64_t M, int64_t N, int64_t K,
                        const void* const* a_planes, int64_t a_bs, int64_t a_rs, int64_t a_cs,
                        const void* const* b_planes, int64_t b_bs, int64_t b_rs, int64_t b_cs,
                        void* const* c_planes, int64_t c_bs, int64_t c_rs, int a_complex_from, int b_complex_from,
                        int accumulate, int band, int64_t band_offset, void* workspace, size_t workspace_bytes,
                        void* stream) {
    if (band < 0 || band > 3) return fail(PK_ERR_ARG, "pk_poly_gemm_banded: band must be 0, 1, 2 or 3");
    return poly_gemm(dtype, degree, batch, M, N, K, a_planes, a_bs, a_rs, a_cs, b_planes, b_bs, b_rs, b_cs, c_planes,
                     c_bs, c_rs, a_complex_from, b_complex_from, workspace, workspace_bytes, stream, accumulate ? 1 : 0,
                     band, band_offset);
}

int pk_poly_gemm_accumulate(int dtype, int degree, int64_t batch, int64_t M, int64_t N, int64_t K,
                            const void* const* a_planes, int64_t a_bs, int64_t a_rs, int64_t a_cs,
                            const void* const* b_planes, int64_t b_bs, int64_t b_rs, int64_t b_cs,
                            void* const* c_planes, int64_t c_bs, int64_t c_rs, int a_complex_from, int b_complex_from,
                            void* workspace, size_t workspace_bytes, void* stream) {
    return poly_gemm(dtype, degree, batch, M, N, K, a_planes, a_bs, a_rs, a_cs, b_planes, b_bs, b_rs, b_cs, c_planes,
                     c_bs, c_rs, a_complex_from, b_complex_from, workspace, workspace_bytes, stream, 1);
}

int pk_poly_gemm_hilo_workspace_query(int degree, int64_t batch, int64_t M, int64_t N, int64_t K,
                                      const void* const* a_planes, int64_t a_bs, int64_t a_rs, int64_t a_cs, int a_hilo,
                                      const void* const* b_planes, int64_t b_bs, int64_t b_rs, int64_t b_cs, int b_hilo,
                                      size_t* bytes) {
    if (!bytes) return fail(PK_ERR_ARG, "pk_poly_gemm_hilo_workspace_query: null result pointer");
    *bytes = 0;
    if (degree < 0 || 2 * (degree + 1) > PK_MAX_PLANES || batch < 0 || M < 0 || N < 0 || K < 0)
        return fail(PK_ERR_ARG, "pk_poly_gemm_hilo_workspace_query: invalid degree or size");
    if (batch == 0 || M == 0 || N == 0 || K == 0) return PK_OK;
    if (!a_planes || !b_planes) return fail(PK_ERR_ARG, "pk_poly_gemm_hilo_workspace_query: null operand plane array");
    const GemmPlan g = plan_call(PK_F32, degree, batch, M, N, K, degree + 1, degree + 1, a_planes, a_bs, a_rs, a_cs,
                                 b_planes, b_bs, b_rs, b_cs, a_hilo ? 1 : 0, b_hilo ? 1 : 0);
    if (g.unaddressable)
        return fail(PK_ERR_UNSUPPORTED, "pk_poly_gemm_hilo_workspace_query: pre-split planes not addressable in place");
    *bytes = g.total;
    return PK_OK;
}

int pk_poly_gemm_hilo(int degree, int64_t batch, int64_t M, int64_t N, int64_t K, const void* const* a_planes,
                      int64_t a_bs, int64_t a_rs, int64_t a_cs, int a_hilo, const void* const* b_planes, int64_t b_bs,
                      int64_t b_rs, int64_t b_cs, int b_hilo, void* const* c_planes, int64_t c_bs, int64_t c_rs,
                      int accumulate, int band, int64_t band_offset, void* workspace, size_t workspace_bytes,
                      void* stream) {
    if (band < 0 || band > 3) return fail(PK_ERR_ARG, "pk_poly_gemm_hilo: band must be 0, 1, 2 or 3");
    return poly_gemm(PK_F32, degree, batch, M, N, K, a_planes, a_bs, a_rs, a_cs, b_planes, b_bs, b_rs, b_cs, c_planes,
                     c_bs, c_rs, degree + 1, degree + 1, workspace, workspace_bytes, stream, accumulate ? 1 : 0, band,
                     band_offset, a_hilo ? 1 : 0, b_hilo ? 1 : 0);
}

}  // extern "C"

