// Attention score products with the softmax work in the epilogue (bfloat16 planes, degree <= 3).
//
// The series attention backward (the reference's SDPA decomposition, src/polytensors/
// _decompositions.py:28-43, differentiated through its bmm and softmax-backward rules,
// src/polytensors/_plain.py:342-347) needs, per block of queries and keys,
//
//   P  = exp(scale * Q K^T - lse)          the probabilities, from the forward's row statistics
//   dS = scale * P (*) (dO V^T - dsum)     the score gradient
//
// with every product a truncated Cauchy product over the n+1 coefficient planes.  Both are a
// polynomial matrix product followed by an elementwise series function of ALL its output
// planes, so one CTA tile here holds every plane of a 128 x 64 block of the product in tensor
// memory (n+1 accumulators, double-buffered: 2 (n+1) 64 <= 512 columns) and the epilogue warps
// apply the series function on the way out.  The score planes are written once, as P or dS,
// and never re-read for the softmax.
//
// Per 64-wide k block the TMA warp loads A_i and B_i (i = 0..n) once into n+1 ring stages and the
// MMA warp issues all (n+1)(n+2)/2 products A_i B_j (i + j <= n) from them, so each operand tile is
// read once per k block instead of once per product.  With a causal mask, tiles whose keys all
// lie after their last query are neither loaded nor multiplied: the epilogue writes their zeros.
#include <algorithm>
#include <cstring>

#include "pk_common.cuh"
#include "pk_gemm_prep.cuh"
#include "pk_series.cuh"

namespace pk {

constexpr int AG_BM = 128;
constexpr int AG_BN = 64;
constexpr int AG_EPI_WARPS = 8;                    // two per TMEM lane quadrant, 32 columns each
constexpr int AG_THREADS = 64 + 32 * AG_EPI_WARPS;  // warp 0: TMA, warp 1: MMA + TMEM owner
constexpr int AG_A_BYTES = AG_BM * TC_BK * 2;
constexpr int AG_B_BYTES = AG_BN * TC_BK * 2;
constexpr int AG_STAGE_BYTES = AG_A_BYTES + AG_B_BYTES;  // one plane's A and B k-block
constexpr int AG_STAGES = 8;
constexpr int AG_SMEM_BYTES = AG_STAGES * AG_STAGE_BYTES + 1024 + 256;
constexpr int AG_MAX_NP = 4;

enum { AG_PROBS = 0, AG_DSCORES = 1 };

struct AgMaps {
    CUtensorMap a[AG_MAX_NP];
    CUtensorMap b[AG_MAX_NP];
};

struct AgParams {
    int batch, M, N;
    int kblocks, tiles_m, tiles_n, group_m, total_tiles;
    int a_mn, b_mn;
    int causal;
    int64_t shift;     // query index of row r is r + shift
    float scale;
    int vec_ok;        // 16-byte vector access to the output (and probability) planes
    int64_t c_bs, c_rs;
    void* c[AG_MAX_NP];
    int64_t p_bs, p_rs;              // AG_DSCORES: probability planes
    const void* pr[AG_MAX_NP];
    const float* rowv;               // AG_PROBS: (lse_0, logz_1..n); AG_DSCORES: dsum; per row
    int64_t rowv_bs;                 // floats between batch entries (rows are NP floats apart)
    int* status;
};

struct AgTile {
    int b, tm, tn;
};

__device__ __forceinline__ AgTile ag_decode(const AgParams& p, int t) {
    AgTile c;
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

// Every key of the tile lies after the last query of its rows: all probabilities are zero.
__device__ __forceinline__ bool ag_masked(const AgParams& p, const AgTile& c) {
    if (!p.causal) return false;
    const int64_t last_row = min(c.tm * AG_BM + AG_BM - 1, p.M - 1);
    return static_cast<int64_t>(c.tn) * AG_BN > last_row + p.shift;
}

__device__ __forceinline__ void ag_load16(const __nv_bfloat16* src, bool vec, int valid, float (&v)[16]) {
    if (vec && valid == 16) {
        const uint4 a = reinterpret_cast<const uint4*>(src)[0];
        const uint4 b = reinterpret_cast<const uint4*>(src)[1];
        const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int t = 0; t < 8; ++t) {
            v[2 * t] = __uint_as_float(w[t] << 16);
            v[2 * t + 1] = __uint_as_float(w[t] & 0xFFFF0000u);
        }
    } else {
#pragma unroll
        for (int t = 0; t < 16; ++t) v[t] = t < valid ? __bfloat162float(src[t]) : 0.f;
    }
}

__device__ __forceinline__ void ag_store16(__nv_bfloat16* dst, bool vec, int valid, const float (&v)[16]) {
    if (vec && valid == 16) {
        uint32_t w[8];
#pragma unroll
        for (int t = 0; t < 8; ++t)
            w[t] = static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(v[2 * t]))) |
                   (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(v[2 * t + 1]))) << 16);
        reinterpret_cast<uint4*>(dst)[0] = make_uint4(w[0], w[1], w[2], w[3]);
        reinterpret_cast<uint4*>(dst)[1] = make_uint4(w[4], w[5], w[6], w[7]);
    } else {
        for (int t = 0; t < valid; ++t) dst[t] = __float2bfloat16_rn(v[t]);
    }
}

template <int NP, int MODE>
__global__ void __launch_bounds__(AG_THREADS, 1)
    attn_score_gemm_kernel(const __grid_constant__ AgMaps maps, const AgParams p) {
    constexpr int TMEM_COLS = 2 * NP * AG_BN <= 128 ? 128 : (2 * NP * AG_BN <= 256 ? 256 : 512);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + AG_STAGES * AG_STAGE_BYTES);
    uint64_t* empty_bar = full_bar + AG_STAGES;
    uint64_t* acc_full = empty_bar + AG_STAGES;
    uint64_t* acc_empty = acc_full + 2;
    uint64_t* drain_bar = acc_empty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < AG_STAGES; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(&acc_full[s], 1);
            mbar_init(&acc_empty[s], 32 * AG_EPI_WARPS);
        }
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
        // ---------------- TMA producer: plane i of k block kb into one ring stage ----------------
        if (lane == 0) {
            uint32_t stage = 0, phase = 0;
            int issued_parity[AG_STAGES];
#pragma unroll
            for (int s = 0; s < AG_STAGES; ++s) issued_parity[s] = -1;
            bool ok = true;
            for (int t = blockIdx.x; t < p.total_tiles && ok; t += gridDim.x) {
                const AgTile tc = ag_decode(p, t);
                if (ag_masked(p, tc)) continue;
                for (int kb = 0; kb < p.kblocks && ok; ++kb) {
                    for (int i = 0; i < NP; ++i) {
                        if (!mbar_wait_or_abort(&empty_bar[stage], phase ^ 1, abort_flag, p.status, 121)) {
                            ok = false;
                            break;
                        }
                        uint8_t* st = smem + stage * AG_STAGE_BYTES;
                        mbar_arrive_expect_tx(&full_bar[stage], AG_STAGE_BYTES);
                        if (p.a_mn) {
#pragma unroll
                            for (int h = 0; h < AG_BM / 64; ++h)
                                tma_load_3d(st + h * 8192, &maps.a[i], &full_bar[stage], tc.tm * AG_BM + h * 64,
                                            kb * TC_BK, tc.b);
                        } else {
                            tma_load_3d(st, &maps.a[i], &full_bar[stage], kb * TC_BK, tc.tm * AG_BM, tc.b);
                        }
                        if (p.b_mn)
                            tma_load_3d(st + AG_A_BYTES, &maps.b[i], &full_bar[stage], tc.tn * AG_BN, kb * TC_BK, tc.b);
                        else
                            tma_load_3d(st + AG_A_BYTES, &maps.b[i], &full_bar[stage], kb * TC_BK, tc.tn * AG_BN, tc.b);
                        issued_parity[stage] = static_cast<int>(phase);
                        if (++stage == AG_STAGES) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                }
            }
            if (!ok) {
                for (int s = 0; s < AG_STAGES; ++s) {
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
            const uint32_t idesc = f16_idesc(1u, AG_BM, AG_BN) | (static_cast<uint32_t>(p.a_mn) << 15) |
                                   (static_cast<uint32_t>(p.b_mn) << 16);
            uint32_t stage = 0, phase = 0;
            uint32_t abuf = 0, aphase = 0;
            bool ok = true, issued = false;
            for (int t = blockIdx.x; t < p.total_tiles && ok; t += gridDim.x) {
                const AgTile tc = ag_decode(p, t);
                if (ag_masked(p, tc)) continue;
                if (!mbar_wait_or_abort(&acc_empty[abuf], aphase ^ 1, abort_flag, p.status, 122)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + abuf * (NP * AG_BN);
                for (int kb = 0; kb < p.kblocks && ok; ++kb) {
                    uint32_t st[NP];
#pragma unroll
                    for (int i = 0; i < NP; ++i) {
                        if (!mbar_wait_or_abort(&full_bar[stage], phase, abort_flag, p.status, 123)) {
                            ok = false;
                            break;
                        }
                        st[i] = stage;
                        if (++stage == AG_STAGES) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                    if (!ok) break;
                    tc_fence_after();
#pragma unroll
                    for (int k = 0; k < NP; ++k) {
#pragma unroll
                        for (int i = 0; i <= k; ++i) {
                            const uint32_t a_s = smem_u32(smem + st[i] * AG_STAGE_BYTES);
                            const uint32_t b_s = smem_u32(smem + st[k - i] * AG_STAGE_BYTES) + AG_A_BYTES;
#pragma unroll
                            for (int kk = 0; kk < TC_BK / 16; ++kk) {
                                const uint64_t ad = p.a_mn ? sw128_mnmajor_desc_lbo(a_s + kk * 2048, 8192)
                                                           : sw128_kmajor_desc(a_s + kk * 32);
                                const uint64_t bd = p.b_mn ? sw128_mnmajor_desc_lbo(b_s + kk * 2048, 8192)
                                                           : sw128_kmajor_desc(b_s + kk * 32);
                                tc_mma_f16(d_tmem + k * AG_BN, ad, bd, idesc, (kb > 0 || i > 0 || kk > 0) ? 1u : 0u);
                            }
                        }
                    }
                    issued = true;
#pragma unroll
                    for (int i = 0; i < NP; ++i) tc_commit(&empty_bar[st[i]]);
                }
                if (!ok) break;
                tc_commit(&acc_full[abuf]);
                if (++abuf == 2) {
                    abuf = 0;
                    aphase ^= 1;
                }
            }
            if (!ok && issued) {
                tc_commit(drain_bar);
                const uint64_t t0 = pk_globaltimer();
                while (!mbar_try_wait(drain_bar, 0) && pk_globaltimer() - t0 < 1000000000ull) {
                }
            }
        }
    } else {
        // ---------------- epilogue: series softmax / score gradient, TMEM -> global ----------------
        // warp w drains TMEM lanes 32*(w%4).. (its lane quadrant) and columns 32*((w-2)/4)..+31
        const uint32_t lane_base = 32u * (warp & 3);
        const int half = (warp - 2) >> 2;
        const bool vec = p.vec_ok != 0;
        const float sc = p.scale;
        uint32_t abuf = 0, aphase = 0;
        for (int t = blockIdx.x; t < p.total_tiles; t += gridDim.x) {
            const AgTile tc = ag_decode(p, t);
            const int r = tc.tm * AG_BM + static_cast<int>(lane_base) + lane;
            const int col0 = tc.tn * AG_BN + half * 32;
            const bool masked_tile = ag_masked(p, tc);
            if (!masked_tile) {
                if (!mbar_wait_or_abort(&acc_full[abuf], aphase, abort_flag, p.status, 124)) break;
                tc_fence_after();
            }
            const bool row_ok = r < p.M;
            float rv[NP];
#pragma unroll
            for (int k = 0; k < NP; ++k) rv[k] = row_ok ? p.rowv[tc.b * p.rowv_bs + static_cast<int64_t>(r) * NP + k] : 0.f;
            const int64_t last_key = p.causal ? static_cast<int64_t>(r) + p.shift : static_cast<int64_t>(p.N) - 1;
#pragma unroll 1
            for (int c = 0; c < 2; ++c) {
                const int cb = col0 + c * 16;
                float y[NP][16];
                if (!masked_tile) {
                    uint32_t x[NP][16];
#pragma unroll
                    for (int k = 0; k < NP; ++k)
                        tmem_ld_32x32b_x16(tmem_base + (lane_base << 16) + abuf * (NP * AG_BN) + k * AG_BN + half * 32 +
                                               c * 16,
                                           x[k]);
                    tmem_ld_wait();
                    if constexpr (MODE == AG_PROBS) {
                        const bool live = rv[0] < INFINITY;
#pragma unroll
                        for (int u = 0; u < 16; ++u) {
                            float s[NP];
#pragma unroll
                            for (int k = 0; k < NP; ++k) s[k] = sc * __uint_as_float(x[k][u]) - rv[k];
                            if (live && cb + u <= last_key) {
                                s_exp<NP, float>(s, s);
                            } else {
#pragma unroll
                                for (int k = 0; k < NP; ++k) s[k] = 0.f;
                            }
#pragma unroll
                            for (int k = 0; k < NP; ++k) y[k][u] = s[k];
                        }
                    } else {
                        const int valid = row_ok ? max(0, min(16, p.N - cb)) : 0;
                        float P[NP][16];
#pragma unroll
                        for (int k = 0; k < NP; ++k) {
                            if (valid > 0) {
                                ag_load16(static_cast<const __nv_bfloat16*>(p.pr[k]) + tc.b * p.p_bs +
                                              static_cast<int64_t>(r) * p.p_rs + cb,
                                          vec, valid, P[k]);
                            } else {
#pragma unroll
                                for (int u = 0; u < 16; ++u) P[k][u] = 0.f;
                            }
                        }
#pragma unroll
                        for (int u = 0; u < 16; ++u) {
                            float g[NP], pu[NP], d[NP];
#pragma unroll
                            for (int k = 0; k < NP; ++k) {
                                g[k] = __uint_as_float(x[k][u]) - rv[k];
                                pu[k] = P[k][u];
                            }
                            s_mul<NP, float>(pu, g, d);
#pragma unroll
                            for (int k = 0; k < NP; ++k) y[k][u] = sc * d[k];
                        }
                    }
                } else {
#pragma unroll
                    for (int k = 0; k < NP; ++k)
#pragma unroll
                        for (int u = 0; u < 16; ++u) y[k][u] = 0.f;
                }
                if (row_ok && cb < p.N) {
                    const int valid = min(16, p.N - cb);
#pragma unroll
                    for (int k = 0; k < NP; ++k)
                        ag_store16(static_cast<__nv_bfloat16*>(p.c[k]) + tc.b * p.c_bs + static_cast<int64_t>(r) * p.c_rs +
                                       cb,
                                   vec, valid, y[k]);
                }
            }
            if (!masked_tile) {
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
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

template <int NP, int MODE>
static int launch_ag(const AgMaps& maps, AgParams& p, cudaStream_t stream) {
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(attn_score_gemm_kernel<NP, MODE>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, AG_SMEM_BYTES);
        if (e != cudaSuccess) return cuda_fail(e, "pk_attn_score_gemm: cudaFuncSetAttribute");
        attr_set[dev] = true;
    }
    const int grid = static_cast<int>(std::min<int64_t>(p.total_tiles, num_sms()));
    void* tok;
    prof_begin(MODE == AG_PROBS ? "attn_probs_gemm" : "attn_dscores_gemm", stream, &tok);
    attn_score_gemm_kernel<NP, MODE><<<grid, AG_THREADS, AG_SMEM_BYTES, stream>>>(maps, p);
    prof_end(MODE == AG_PROBS ? "attn_probs_gemm" : "attn_dscores_gemm", stream, tok);
    PK_CHECK_LAUNCH("pk_attn_score_gemm: kernel launch");
    return PK_OK;
}

static int attn_score_gemm(int mode, const char* what, int dtype, int degree, int64_t batch, int64_t M, int64_t N,
                           int64_t K, const void* const* a_planes, int64_t a_bs, int64_t a_rs, int64_t a_cs,
                           const void* const* b_planes, int64_t b_bs, int64_t b_rs, int64_t b_cs,
                           void* const* c_planes, int64_t c_bs, int64_t c_rs, const void* const* probs, int64_t p_bs,
                           int64_t p_rs, const void* rowv, int64_t rowv_bs, double scale, int causal,
                           int64_t causal_shift, void* stream_ptr) {
    const std::string w(what);
    if (dtype != PK_BF16) return fail(PK_ERR_UNSUPPORTED, w + ": bfloat16 planes only");
    if (degree < 0 || degree >= AG_MAX_NP) return fail(PK_ERR_UNSUPPORTED, w + ": degree must be in [0, 3]");
    if (batch < 0 || M < 0 || N < 0 || K < 0) return fail(PK_ERR_ARG, w + ": negative size");
    if (M > 0x7fffffff || N > 0x7fffffff || K > 0x7fffffff || batch > 0x7fffffff)
        return fail(PK_ERR_UNSUPPORTED, w + ": dimension exceeds 2^31-1");
    if (batch == 0 || M == 0 || N == 0) return PK_OK;
    if (K == 0) return fail(PK_ERR_UNSUPPORTED, w + ": empty reduction");
    const int P = degree + 1;
    if (!a_planes || !b_planes || !c_planes || !rowv) return fail(PK_ERR_ARG, w + ": null plane array or row values");
    for (int k = 0; k < P; ++k)
        if (!a_planes[k] || !b_planes[k] || !c_planes[k]) return fail(PK_ERR_ARG, w + ": null plane pointer");
    if (mode == AG_DSCORES) {
        if (!probs) return fail(PK_ERR_ARG, w + ": null probability planes");
        for (int k = 0; k < P; ++k)
            if (!probs[k]) return fail(PK_ERR_ARG, w + ": null probability plane pointer");
    }
    const int am = operand_mode(dtype, a_planes, P, batch, M, K, a_bs, a_rs, a_cs);
    const int bm = operand_mode(dtype, b_planes, P, batch, N, K, b_bs, b_cs, b_rs);
    if (am == OPM_STAGED || bm == OPM_STAGED)
        return fail(PK_ERR_UNSUPPORTED, w + ": operand planes must be 16-byte aligned with k or rows contiguous "
                                            "and the other strides multiples of 8 elements");

    AgMaps maps;
    std::memset(&maps, 0, sizeof(maps));
    const TcOperand oa{am, M, K, K, batch, a_planes, a_bs, a_rs, a_cs, nullptr, nullptr, 0};
    const TcOperand ob{bm, N, K, K, batch, b_planes, b_bs, b_cs, b_rs, nullptr, nullptr, 0};
    int rc = encode_operand(maps.a, oa, P, false, AG_BM);
    if (rc) return rc;
    rc = encode_operand(maps.b, ob, P, false, AG_BN);
    if (rc) return rc;

    AgParams p{};
    p.batch = static_cast<int>(batch);
    p.M = static_cast<int>(M);
    p.N = static_cast<int>(N);
    p.kblocks = static_cast<int>(ceil_div(K, TC_BK));
    p.tiles_m = static_cast<int>(ceil_div(M, AG_BM));
    p.tiles_n = static_cast<int>(ceil_div(N, AG_BN));
    p.group_m = 8;
    const int64_t total = static_cast<int64_t>(p.tiles_m) * p.tiles_n * batch;
    if (total > 0x7fffffff) return fail(PK_ERR_UNSUPPORTED, w + ": too many tiles");
    p.total_tiles = static_cast<int>(total);
    p.a_mn = am == OPM_MNMAJOR;
    p.b_mn = bm == OPM_MNMAJOR;
    p.causal = causal ? 1 : 0;
    p.shift = causal_shift;
    p.scale = static_cast<float>(scale);
    p.c_bs = c_bs;
    p.c_rs = c_rs;
    p.p_bs = p_bs;
    p.p_rs = p_rs;
    bool vec = c_rs % 8 == 0 && (batch == 1 || c_bs % 8 == 0);
    for (int k = 0; k < P; ++k) {
        p.c[k] = c_planes[k];
        if (reinterpret_cast<uintptr_t>(c_planes[k]) % 16) vec = false;
        if (mode == AG_DSCORES) {
            p.pr[k] = probs[k];
            if (reinterpret_cast<uintptr_t>(probs[k]) % 16) vec = false;
        }
    }
    if (mode == AG_DSCORES && (p_rs % 8 != 0 || (batch > 1 && p_bs % 8 != 0))) vec = false;
    p.vec_ok = vec ? 1 : 0;
    p.rowv = static_cast<const float*>(rowv);
    p.rowv_bs = rowv_bs;
    p.status = device_status_ptr();
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    switch (P * 2 + mode) {
        case 2: return launch_ag<1, AG_PROBS>(maps, p, stream);
        case 3: return launch_ag<1, AG_DSCORES>(maps, p, stream);
        case 4: return launch_ag<2, AG_PROBS>(maps, p, stream);
        case 5: return launch_ag<2, AG_DSCORES>(maps, p, stream);
        case 6: return launch_ag<3, AG_PROBS>(maps, p, stream);
        case 7: return launch_ag<3, AG_DSCORES>(maps, p, stream);
        case 8: return launch_ag<4, AG_PROBS>(maps, p, stream);
        default: return launch_ag<4, AG_DSCORES>(maps, p, stream);
    }
}

}  // namespace pk

using namespace pk;

extern "C" {

int pk_attn_probs_gemm(int dtype, int degree, int64_t batch, int64_t M, int64_t N, int64_t K,
                       const void* const* q, int64_t q_bs, int64_t q_rs, int64_t q_cs, const void* const* kt,
                       int64_t kt_bs, int64_t kt_rs, int64_t kt_cs, void* const* probs, int64_t p_bs, int64_t p_rs,
                       const void* stats, int64_t stats_bs, double scale, int causal, int64_t causal_shift,
                       void* stream) {
    return attn_score_gemm(AG_PROBS, "pk_attn_probs_gemm", dtype, degree, batch, M, N, K, q, q_bs, q_rs, q_cs, kt,
                           kt_bs, kt_rs, kt_cs, probs, p_bs, p_rs, nullptr, 0, 0, stats, stats_bs, scale, causal,
                           causal_shift, stream);
}

int pk_attn_dscores_gemm(int dtype, int degree, int64_t batch, int64_t M, int64_t N, int64_t K,
                         const void* const* dout, int64_t do_bs, int64_t do_rs, int64_t do_cs, const void* const* vt,
                         int64_t vt_bs, int64_t vt_rs, int64_t vt_cs, const void* const* probs, int64_t p_bs,
                         int64_t p_rs, const void* dsum, int64_t dsum_bs, double scale, int causal,
                         int64_t causal_shift, void* const* dscores, int64_t ds_bs, int64_t ds_rs, void* stream) {
    return attn_score_gemm(AG_DSCORES, "pk_attn_dscores_gemm", dtype, degree, batch, M, N, K, dout, do_bs, do_rs,
                           do_cs, vt, vt_bs, vt_rs, vt_cs, dscores, ds_bs, ds_rs, probs, p_bs, p_rs, dsum, dsum_bs,
                           scale, causal, causal_shift, stream);
}

}  // extern "C"
