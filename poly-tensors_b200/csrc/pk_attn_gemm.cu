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
// A work unit is 128 rows of A (queries) against a run of up to AG_CHUNK 64-column tiles of B
// (keys): the unit's A planes (all n+1 planes, the whole reduction, k <= 128) are loaded once into
// shared memory and stay resident while B streams through a ring of per-plane 64 x 64 k-blocks,
// so A crosses L2 once per unit instead of once per tile.  Per k block the MMA warp issues all
// (n+1)(n+2)/2 products A_i B_j (i + j <= n) from the resident A and n+1 ring stages.  Units are
// ordered so CTAs running together share a B chunk in L2.  With a causal mask, tiles whose keys
// all lie after their last query are neither loaded nor multiplied: the epilogue writes zeros.
#include <algorithm>
#include <cstring>
#include <vector>

#include "pk_common.cuh"
#include "pk_gemm_prep.cuh"
#include "pk_series.cuh"

namespace pk {

constexpr int AG_BM = 128;
constexpr int AG_BN = 64;
constexpr int AG_EPI_WARPS = 16;                   // four per TMEM lane quadrant, 16 columns each
constexpr int AG_THREADS = 64 + 32 * AG_EPI_WARPS;  // warp 0: TMA, warp 1: MMA + TMEM owner
constexpr int AG_A_BYTES = AG_BM * TC_BK * 2;     // one plane's 128 x 64 A k-block
constexpr int AG_B_BYTES = AG_BN * TC_BK * 2;     // one plane's 64 x 64 B k-block (a ring stage)
constexpr int AG_MAX_K = 128;                     // reduction held resident (head dimension)
constexpr int AG_MAX_STAGES = 24;
constexpr int AG_WARP_OUT = 32 * 16 * 2;          // one epilogue warp's 32 rows x 16 columns of one plane, bf16
constexpr int AG_OUT_BYTES = AG_EPI_WARPS * 2 * AG_WARP_OUT;  // 2 buffers per epilogue warp (TMA-store staging)
constexpr int AG_SMEM_BUDGET = 224 * 1024;        // resident A + B ring + output staging
constexpr int AG_SMEM_BYTES = AG_SMEM_BUDGET + 1024 + 512;
constexpr int AG_CHUNK = 8;                       // B tiles per work unit
constexpr int AG_MAX_NP = 4;
constexpr int AG_MAX_SHAPES = 4096;               // unit shapes (chunk, row tile) the cost order holds
constexpr int64_t AG_FAR_KEYS = 192;              // causal == 2: zero tiles written up to this far out

enum { AG_PROBS = 0, AG_DSCORES = 1 };

// Plane i (sub-plane h of NS: bf16 planes NS = 1; float32 attention NS = 2, x ~= hi + lo) at index
// i * NS + h of each array.
struct AgMaps {
    CUtensorMap a[2 * AG_MAX_NP];
    CUtensorMap b[2 * AG_MAX_NP];
    CUtensorMap c[2 * AG_MAX_NP];  // output planes, boxes of 16 columns x 32 rows (per-warp TMA stores)
};

struct AgParams {
    int batch, M, N;
    int kblocks, tiles_m, tiles_n, n_chunks, total_units;
    int nstages;       // B ring stages
    int a_bytes;       // resident A bytes (NP * kblocks * AG_A_BYTES)
    int a_mn, b_mn;
    int causal;
    int skip_far;      // masked tiles starting more than AG_FAR_KEYS keys past their rows are not written
    int64_t shift;     // query index of row r is r + shift
    float scale;
    int vec_ok;        // 16-byte vector access to the output (and probability) planes
    int tma_store;     // output planes written by TMA stores from shared-memory staging
    int64_t c_bs, c_rs;
    void* c[2 * AG_MAX_NP];
    int64_t p_bs, p_rs;              // AG_DSCORES: probability planes
    const void* pr[2 * AG_MAX_NP];
    const float* rowv;               // AG_PROBS: (lse_0, logz_1..n); AG_DSCORES: dsum; per row
    int64_t rowv_bs;                 // floats between batch entries (rows are NP floats apart)
    int* status;
    // Unit schedule.  n_groups == 0: natural order (batch entry, B chunk, row tile).  Otherwise the
    // unit shapes (B chunk, row tile) in classes of equal live-tile count, heaviest class first:
    // class g holds shapes order[grp_first[g] .. grp_first[g+1]) for every batch entry, ranks
    // grp_cum[g] .. grp_cum[g+1] (batch entry outer, row tile fastest within a chunk).
    int n_groups;
    int grp_first[AG_CHUNK + 2];
    int grp_cum[AG_CHUNK + 2];
    uint16_t order[AG_MAX_SHAPES];   // chunk * tiles_m + row tile
};

struct AgTile {
    int b, tm, tn;
};

// Unit of schedule rank u -> (batch entry, B chunk, row tile), the row tile fastest within a
// class so that CTAs running together work on the same B chunk.  Tiles of the unit: tn in
// [tn0, tn1).
struct AgUnit {
    int b, tm, tn0, tn1;
};

__device__ __forceinline__ AgUnit ag_unit(const AgParams& p, int u) {
    AgUnit c;
    int chunk;
    if (p.n_groups == 0) {
        const int per_b = p.n_chunks * p.tiles_m;
        c.b = u / per_b;
        const int r = u % per_b;
        chunk = r / p.tiles_m;
        c.tm = r % p.tiles_m;
    } else {
        int g = 0;
        while (g + 1 < p.n_groups && u >= p.grp_cum[g + 1]) ++g;
        const int local = u - p.grp_cum[g];
        const int gsize = p.grp_first[g + 1] - p.grp_first[g];
        c.b = local / gsize;
        const int code = p.order[p.grp_first[g] + local % gsize];
        chunk = code / p.tiles_m;
        c.tm = code % p.tiles_m;
    }
    c.tn0 = chunk * AG_CHUNK;
    c.tn1 = min(p.tiles_n, c.tn0 + AG_CHUNK);
    return c;
}


// Every key of the tile lies after the last query of its rows: all probabilities are zero.
__device__ __forceinline__ bool ag_masked(const AgParams& p, const AgTile& c) {
    if (!p.causal) return false;
    const int64_t last_row = min(c.tm * AG_BM + AG_BM - 1, p.M - 1);
    return static_cast<int64_t>(c.tn) * AG_BN > last_row + p.shift;
}

// exp of a series with the constant term through the fast exponential intrinsic (the
// probabilities are stored as bfloat16, far coarser than its error); directions by the ODE
// recurrence k y_k = sum_{i=1..k} i x_i y_{k-i}.
template <int NP>
__device__ __forceinline__ void s_exp_fast(float (&x)[NP]) {
    float r[NP];
    r[0] = __expf(x[0]);
#pragma unroll
    for (int k = 1; k < NP; ++k) {
        float acc = 0.f;
#pragma unroll
        for (int i = 1; i <= k; ++i) acc += float(i) * x[i] * r[k - i];
        r[k] = acc * inv_int<float>(k);
    }
#pragma unroll
    for (int k = 0; k < NP; ++k) x[k] = r[k];
}

// NS = 1: bfloat16 planes.  NS = 2 (float32 attention): every operand, probability and output plane
// is a pair of bf16 planes (hi, lo) with x ~= hi + lo; each product is evaluated as
// a_hi b_hi + a_hi b_lo + a_lo b_hi (fp32 accumulation) and outputs are split the same way.
template <int NP, int MODE, int NS>
__global__ void __launch_bounds__(AG_THREADS, 1)
    attn_score_gemm_kernel(const __grid_constant__ AgMaps maps, const __grid_constant__ AgParams p) {
    constexpr int TMEM_COLS = 2 * NP * AG_BN <= 128 ? 128 : (2 * NP * AG_BN <= 256 ? 256 : 512);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* a_res = smem;                // [plane][kblock] 16 KB boxes
    uint8_t* ring = smem + p.a_bytes;     // B stages, 8 KB each
    uint8_t* out_stage = smem + AG_SMEM_BUDGET - AG_OUT_BYTES;  // [epilogue warp][buffer] 1 KB blocks
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + AG_SMEM_BUDGET);
    uint64_t* empty_bar = full_bar + AG_MAX_STAGES;
    uint64_t* acc_full = empty_bar + AG_MAX_STAGES;
    uint64_t* acc_empty = acc_full + 2;
    uint64_t* a_full = acc_empty + 2;
    uint64_t* a_empty = a_full + 1;
    uint64_t* drain_bar = a_empty + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int nst = p.nstages;

    if (threadIdx.x == 0) {
        for (int s = 0; s < nst; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(&acc_full[s], 1);
            mbar_init(&acc_empty[s], 32 * AG_EPI_WARPS);
        }
        mbar_init(a_full, 1);
        mbar_init(a_empty, 1);
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        fence_mbar_init();
        for (int i = 0; i < NP * NS; ++i) {
            tma_prefetch_desc(&maps.a[i]);
            tma_prefetch_desc(&maps.b[i]);
            if (p.tma_store) tma_prefetch_desc(&maps.c[i]);
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
        // ---------------- TMA producer: a unit's A planes once, then its B k-blocks ----------------
        if (lane == 0) {
            uint32_t stage = 0, phase = 0, a_phase = 0;
            int issued_parity[AG_MAX_STAGES];
            for (int s = 0; s < nst; ++s) issued_parity[s] = -1;
            int a_issued = -1;
            bool ok = true;
            for (int rk = 0, u = snake_rank(0); u < p.total_units && ok; u = snake_rank(++rk)) {
                const AgUnit un = ag_unit(p, u);
                if (ag_masked(p, AgTile{un.b, un.tm, un.tn0})) continue;  // every tile of the unit masked
                if (!mbar_wait_or_abort(a_empty, a_phase ^ 1, abort_flag, p.status, 125)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(a_full, static_cast<uint32_t>(p.a_bytes));
                for (int i = 0; i < NP * NS; ++i) {
                    for (int kb = 0; kb < p.kblocks; ++kb) {
                        uint8_t* dst = a_res + (i * p.kblocks + kb) * AG_A_BYTES;
                        if (p.a_mn) {
#pragma unroll
                            for (int h = 0; h < AG_BM / 64; ++h)
                                tma_load_3d(dst + h * 8192, &maps.a[i], a_full, un.tm * AG_BM + h * 64, kb * TC_BK, un.b);
                        } else {
                            tma_load_3d(dst, &maps.a[i], a_full, kb * TC_BK, un.tm * AG_BM, un.b);
                        }
                    }
                }
                a_issued = static_cast<int>(a_phase);
                a_phase ^= 1;
                for (int tn = un.tn0; tn < un.tn1 && ok; ++tn) {
                    if (ag_masked(p, AgTile{un.b, un.tm, tn})) break;  // later tiles are masked too
                    for (int kb = 0; kb < p.kblocks && ok; ++kb) {
                        // stage order within a k block: sub-plane major (all hi planes, then all lo)
                        for (int t = 0; t < NP * NS; ++t) {
                            const int i = (t % NP) * NS + t / NP;  // map index of plane t % NP, sub t / NP
                            if (!mbar_wait_or_abort(&empty_bar[stage], phase ^ 1, abort_flag, p.status, 121)) {
                                ok = false;
                                break;
                            }
                            uint8_t* st = ring + stage * AG_B_BYTES;
                            mbar_arrive_expect_tx(&full_bar[stage], AG_B_BYTES);
                            if (p.b_mn)
                                tma_load_3d(st, &maps.b[i], &full_bar[stage], tn * AG_BN, kb * TC_BK, un.b);
                            else
                                tma_load_3d(st, &maps.b[i], &full_bar[stage], kb * TC_BK, tn * AG_BN, un.b);
                            issued_parity[stage] = static_cast<int>(phase);
                            if (++stage == static_cast<uint32_t>(nst)) {
                                stage = 0;
                                phase ^= 1;
                            }
                        }
                    }
                }
            }
            if (!ok) {
                // let copies in flight land before the CTA (and its shared memory) exits (bounded)
                for (int s = 0; s < nst; ++s) {
                    if (issued_parity[s] < 0) continue;
                    const uint64_t t0 = pk_globaltimer();
                    while (!mbar_try_wait(&full_bar[s], static_cast<uint32_t>(issued_parity[s])) &&
                           pk_globaltimer() - t0 < 1000000000ull) {
                    }
                }
                if (a_issued >= 0) {
                    const uint64_t t0 = pk_globaltimer();
                    while (!mbar_try_wait(a_full, static_cast<uint32_t>(a_issued)) &&
                           pk_globaltimer() - t0 < 1000000000ull) {
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t idesc = f16_idesc(1u, AG_BM, AG_BN) | (static_cast<uint32_t>(p.a_mn) << 15) |
                                   (static_cast<uint32_t>(p.b_mn) << 16);
            uint32_t stage = 0, phase = 0, a_par = 0;
            uint32_t abuf = 0, aphase = 0;
            bool ok = true, issued = false;
            for (int rk = 0, u = snake_rank(0); u < p.total_units && ok; u = snake_rank(++rk)) {
                const AgUnit un = ag_unit(p, u);
                if (ag_masked(p, AgTile{un.b, un.tm, un.tn0})) continue;
                if (!mbar_wait_or_abort(a_full, a_par, abort_flag, p.status, 126)) {
                    ok = false;
                    break;
                }
                a_par ^= 1;
                tc_fence_after();
                for (int tn = un.tn0; tn < un.tn1 && ok; ++tn) {
                    if (ag_masked(p, AgTile{un.b, un.tm, tn})) break;
                    if (!mbar_wait_or_abort(&acc_empty[abuf], aphase ^ 1, abort_flag, p.status, 122)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + abuf * (NP * AG_BN);
                    for (int kb = 0; kb < p.kblocks && ok; ++kb) {
                        uint32_t st[NP * NS];
#pragma unroll
                        for (int i = 0; i < NP * NS; ++i) {
                            if (!mbar_wait_or_abort(&full_bar[stage], phase, abort_flag, p.status, 123)) {
                                ok = false;
                                break;
                            }
                            st[i] = stage;
                            if (++stage == static_cast<uint32_t>(nst)) {
                                stage = 0;
                                phase ^= 1;
                            }
                        }
                        if (!ok) break;
                        tc_fence_after();
                        // descriptors built once per k block; each 16-wide k step advances the
                        // start address field by a constant (32 B K-major, 2048 B MN-major)
                        uint64_t ad[NP][NS], bd[NP][NS];
#pragma unroll
                        for (int i = 0; i < NP; ++i) {
#pragma unroll
                            for (int h = 0; h < NS; ++h) {
                                const uint32_t a_s = smem_u32(a_res + ((i * NS + h) * p.kblocks + kb) * AG_A_BYTES);
                                const uint32_t b_s = smem_u32(ring + st[h * NP + i] * AG_B_BYTES);
                                ad[i][h] = p.a_mn ? sw128_mnmajor_desc_lbo(a_s, 8192) : sw128_kmajor_desc(a_s);
                                bd[i][h] = p.b_mn ? sw128_mnmajor_desc_lbo(b_s, 8192) : sw128_kmajor_desc(b_s);
                            }
                        }
                        const uint64_t a_step = p.a_mn ? 2048 >> 4 : 32 >> 4;
                        const uint64_t b_step = p.b_mn ? 2048 >> 4 : 32 >> 4;
                        // consecutive MMAs go to different accumulators (k varies fastest), so no
                        // MMA waits on the previous one's accumulation
#pragma unroll
                        for (int kk = 0; kk < TC_BK / 16; ++kk) {
#pragma unroll
                            for (int i = 0; i < NP; ++i) {
#pragma unroll
                                for (int k = i; k < NP; ++k) {
                                    tc_mma_f16(d_tmem + k * AG_BN, ad[i][0] + kk * a_step, bd[k - i][0] + kk * b_step,
                                               idesc, (kb > 0 || i > 0 || kk > 0) ? 1u : 0u);
                                    if constexpr (NS == 2) {
                                        tc_mma_f16(d_tmem + k * AG_BN, ad[i][0] + kk * a_step,
                                                   bd[k - i][1] + kk * b_step, idesc, 1u);
                                        tc_mma_f16(d_tmem + k * AG_BN, ad[i][1] + kk * a_step,
                                                   bd[k - i][0] + kk * b_step, idesc, 1u);
                                    }
                                }
                            }
                        }
                        issued = true;
#pragma unroll
                        for (int i = 0; i < NP * NS; ++i) tc_commit(&empty_bar[st[i]]);
                    }
                    if (!ok) break;
                    tc_commit(&acc_full[abuf]);
                    if (++abuf == 2) {
                        abuf = 0;
                        aphase ^= 1;
                    }
                }
                if (!ok) break;
                tc_commit(a_empty);  // the unit's A may be overwritten once its products retire
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
        // warp w drains TMEM lanes 32*(w%4).. (its lane quadrant) and columns 16*((w-2)/4)..+15,
        // eight columns at a time, each element's n+1 coefficients transformed in place
        const uint32_t lane_base = 32u * (warp & 3);
        const int grp = (warp - 2) >> 2;
        const bool vec = p.vec_ok != 0;
        const float sc = p.scale;
        uint32_t abuf = 0, aphase = 0;
        // A wait that fails (timeout or abort) turns its tile into zeros; every warp still runs the
        // same tile sequence, so the quadrants' named barriers always match.
        for (int rk = 0, u = snake_rank(0); u < p.total_units; u = snake_rank(++rk)) {
          const AgUnit un = ag_unit(p, u);
          // the unit's rows are this thread's rows in every tile: their statistics are read once
          const int r = un.tm * AG_BM + static_cast<int>(lane_base) + lane;
          const bool row_ok = r < p.M;
          float rv[NP];
#pragma unroll
          for (int k = 0; k < NP; ++k) rv[k] = row_ok ? p.rowv[un.b * p.rowv_bs + static_cast<int64_t>(r) * NP + k] : 0.f;
          for (int tn = un.tn0; tn < un.tn1; ++tn) {
            const AgTile tc{un.b, un.tm, tn};
            bool masked_tile = ag_masked(p, tc);
            if (masked_tile && p.skip_far) {
                // far above the diagonal: no consumer reads these zeros (the decision depends on
                // the tile only, so every warp of the CTA skips the same tiles)
                const int64_t last_row = min(tc.tm * AG_BM + AG_BM - 1, p.M - 1);
                if (static_cast<int64_t>(tc.tn) * AG_BN > last_row + p.shift + AG_FAR_KEYS) continue;
            }
            const int64_t last_key = p.causal ? static_cast<int64_t>(r) + p.shift : static_cast<int64_t>(p.N) - 1;
            const bool live = MODE == AG_PROBS ? rv[0] < INFINITY : true;
            // tile entirely inside the matrix and below the causal diagonal: no per-element tests
            const bool interior = (tc.tn + 1) * AG_BN <= p.N &&
                                  (!p.causal || static_cast<int64_t>(tc.tn + 1) * AG_BN - 1 <=
                                                    static_cast<int64_t>(tc.tm) * AG_BM + p.shift);
            const int cbase = tc.tn * AG_BN + grp * 16;
            // score gradient: this thread's 16 probabilities of every plane, requested before the
            // accumulator wait so that their latency overlaps it (bf16 pairs, zero outside the matrix)
            // bf16: all 16 columns of every plane loaded before the accumulator wait; float32 (hi/lo
            // pairs): each 8-column half loaded just before its use (registers), pw[k * NS + h][0..3]
            uint32_t pw[NP * NS][NS == 1 ? 8 : 4];
            if constexpr (MODE == AG_DSCORES) {
                // the unit's next tile: its probability rows (64 columns = one 128-byte line per
                // row and plane) go to L2 now, a whole tile ahead of their loads
                const int ncol = (tn + 1) * AG_BN;
                if (grp == 0 && row_ok && tn + 1 < un.tn1 && ncol < p.N && !ag_masked(p, AgTile{un.b, un.tm, tn + 1})) {
#pragma unroll
                    for (int k = 0; k < NP * NS; ++k)
                        prefetch_l2_line(static_cast<const __nv_bfloat16*>(p.pr[k]) + tc.b * p.p_bs +
                                         static_cast<int64_t>(r) * p.p_rs + ncol);
                }
                const int valid16 = row_ok ? max(0, min(16, p.N - cbase)) : 0;
#pragma unroll
                for (int k = 0; k < (NS == 1 ? NP : 0); ++k) {
                    const __nv_bfloat16* src = static_cast<const __nv_bfloat16*>(p.pr[k]) + tc.b * p.p_bs +
                                               static_cast<int64_t>(r) * p.p_rs + cbase;
                    if (masked_tile) {
#pragma unroll
                        for (int t = 0; t < 8; ++t) pw[k][t] = 0u;
                    } else if (vec && valid16 == 16) {
                        const uint4 w0 = reinterpret_cast<const uint4*>(src)[0];
                        const uint4 w1 = reinterpret_cast<const uint4*>(src)[1];
                        pw[k][0] = w0.x; pw[k][1] = w0.y; pw[k][2] = w0.z; pw[k][3] = w0.w;
                        pw[k][4] = w1.x; pw[k][5] = w1.y; pw[k][6] = w1.z; pw[k][7] = w1.w;
                    } else {
#pragma unroll
                        for (int t = 0; t < 8; ++t) {
                            const uint32_t lo = 2 * t < valid16 ? __bfloat16_as_ushort(src[2 * t]) : 0u;
                            const uint32_t hi = 2 * t + 1 < valid16 ? __bfloat16_as_ushort(src[2 * t + 1]) : 0u;
                            pw[k][t] = lo | (hi << 16);
                        }
                    }
                }
            }
            if (!masked_tile) {
                if (mbar_wait_or_abort(&acc_full[abuf], aphase, abort_flag, p.status, 124)) tc_fence_after();
                else masked_tile = true;  // no accumulator to read: write zeros
            }
            // this thread's 16 columns of every plane as bf16 pairs, ypk[k][0..7], stored after both
            // halves; float32 (hi/lo pairs): one 8-column half at a time, ypk[k * NS + h][0..3],
            // stored as soon as it is formed (registers)
            // the split probabilities keep all 16 columns too, so that each row's 32-byte sector of a
            // plane leaves in one go
            constexpr bool FULL = NS == 1 || MODE == AG_PROBS;
            constexpr int YW = FULL ? 8 : 4;
            uint32_t ypk[NP * NS][YW];
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                const int cb = cbase + c * 8;
                if constexpr (MODE == AG_DSCORES && NS == 2) {
                    const int valid8 = row_ok ? max(0, min(8, p.N - cb)) : 0;
#pragma unroll
                    for (int k = 0; k < NP * NS; ++k) {
                        const __nv_bfloat16* src = static_cast<const __nv_bfloat16*>(p.pr[k]) + tc.b * p.p_bs +
                                                   static_cast<int64_t>(r) * p.p_rs + cb;
                        if (masked_tile) {
#pragma unroll
                            for (int t = 0; t < 4; ++t) pw[k][t] = 0u;
                        } else if (vec && valid8 == 8) {
                            const uint4 w0 = *reinterpret_cast<const uint4*>(src);
                            pw[k][0] = w0.x; pw[k][1] = w0.y; pw[k][2] = w0.z; pw[k][3] = w0.w;
                        } else {
#pragma unroll
                            for (int t = 0; t < 4; ++t) {
                                const uint32_t lo = 2 * t < valid8 ? __bfloat16_as_ushort(src[2 * t]) : 0u;
                                const uint32_t hi = 2 * t + 1 < valid8 ? __bfloat16_as_ushort(src[2 * t + 1]) : 0u;
                                pw[k][t] = lo | (hi << 16);
                            }
                        }
                    }
                }
                if (!masked_tile) {
                    uint32_t x[NP][8];
#pragma unroll
                    for (int k = 0; k < NP; ++k)
                        tmem_ld_32x32b_x8(tmem_base + (lane_base << 16) + abuf * (NP * AG_BN) + k * AG_BN + grp * 16 +
                                              c * 8,
                                          x[k]);
                    tmem_ld_wait();
                    if (c == 1) {
                        // the accumulator is in registers: release it to the next tile's products
                        tc_fence_before();
                        mbar_arrive(&acc_empty[abuf]);
                        if (++abuf == 2) {
                            abuf = 0;
                            aphase ^= 1;
                        }
                    }
#pragma unroll
                    for (int e = 0; e < 8; e += 2) {
                        float v2[2][NP];
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            float* v = v2[h];
                            const int ee = e + h;
                            if constexpr (MODE == AG_PROBS) {
#pragma unroll
                                for (int k = 0; k < NP; ++k) v[k] = sc * __uint_as_float(x[k][ee]) - rv[k];
                                if (interior ? live : (live && cb + ee <= last_key)) {
                                    s_exp_fast<NP>(v2[h]);
                                } else {
#pragma unroll
                                    for (int k = 0; k < NP; ++k) v[k] = 0.f;
                                }
                            } else {
                                float g[NP], pe[NP], d[NP];
#pragma unroll
                                for (int k = 0; k < NP; ++k) {
                                    g[k] = __uint_as_float(x[k][ee]) - rv[k];
                                    const int wi = NS == 1 ? c * 4 + ee / 2 : ee / 2;
                                    const uint32_t wbits = pw[k * NS][wi];
                                    pe[k] = __uint_as_float((ee & 1) ? (wbits & 0xFFFF0000u) : (wbits << 16));
                                    if constexpr (NS == 2) {
                                        const uint32_t lbits = pw[k * NS + 1][wi];
                                        pe[k] += __uint_as_float((ee & 1) ? (lbits & 0xFFFF0000u) : (lbits << 16));
                                    }
                                }
                                s_mul<NP, float>(pe, g, d);
#pragma unroll
                                for (int k = 0; k < NP; ++k) v[k] = sc * d[k];
                            }
                        }
#pragma unroll
                        for (int k = 0; k < NP; ++k) {
                            const uint32_t hb = bf16x2_bits(v2[0][k], v2[1][k]);
                            const int yi = FULL ? c * 4 + e / 2 : e / 2;
                            ypk[k * NS][yi] = hb;
                            if constexpr (NS == 2) {
                                // lo = bf16(x - hi): the part of x the rounded hi misses
                                ypk[k * NS + 1][yi] = bf16x2_bits(v2[0][k] - __uint_as_float(hb << 16),
                                                                  v2[1][k] - __uint_as_float(hb & 0xFFFF0000u));
                            }
                        }
                    }
                } else {
#pragma unroll
                    for (int k = 0; k < NP * NS; ++k)
#pragma unroll
                        for (int t = 0; t < 4; ++t) ypk[k][FULL ? c * 4 + t : t] = 0u;
                }
                if constexpr (NS == 2 && !FULL) {
                    // split score gradient, stored key-major (plane [key][query], c_rs apart per key):
                    // for each of the half's 8 keys the warp's 32 lanes write 32 consecutive queries
                    const int valid = row_ok ? max(0, min(8, p.N - cb)) : 0;
#pragma unroll
                    for (int k = 0; k < NP * NS; ++k) {
                        unsigned short* dst = static_cast<unsigned short*>(p.c[k]) + tc.b * p.c_bs +
                                              static_cast<int64_t>(cb) * p.c_rs + r;
#pragma unroll
                        for (int t = 0; t < 8; ++t)
                            if (t < valid)
                                dst[static_cast<int64_t>(t) * p.c_rs] =
                                    static_cast<unsigned short>((ypk[k][t / 2] >> (16 * (t & 1))) & 0xFFFFu);
                    }
                }
            }
            if constexpr (NS == 2 && FULL) {
                // split probabilities: each row's 16 columns of every hi / lo plane as one 32-byte store pair
                const int valid = row_ok ? max(0, min(16, p.N - cbase)) : 0;
#pragma unroll
                for (int k = 0; k < NP * NS; ++k) {
                    if (valid <= 0) break;
                    __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(p.c[k]) + tc.b * p.c_bs +
                                         static_cast<int64_t>(r) * p.c_rs + cbase;
                    if (vec && valid == 16) {
                        uint4* d4 = reinterpret_cast<uint4*>(dst);
                        d4[0] = make_uint4(ypk[k][0], ypk[k][1], ypk[k][2], ypk[k][3]);
                        d4[1] = make_uint4(ypk[k][4], ypk[k][5], ypk[k][6], ypk[k][7]);
                    } else {
                        for (int t = 0; t < valid; ++t)
                            dst[t] = __ushort_as_bfloat16(
                                static_cast<unsigned short>((ypk[k][t / 2] >> (16 * (t & 1))) & 0xFFFFu));
                    }
                }
            } else if constexpr (NS == 2) {
                // stored half by half above
            } else if (p.tma_store) {
                // Per plane: the warp writes its 32 rows x 16 columns into its own staging block
                // (row t at 32 t bytes) and its lane 0 stores the block with TMA, so no other warp
                // takes part and the only synchronisation is within the warp.  Two blocks per warp
                // alternate; a block is rewritten only after its previous store has read it.
                const int q = warp & 3, ew = warp - 2;
#pragma unroll
                for (int k = 0; k < NP * NS; ++k) {
                    uint8_t* blk = out_stage + (ew * 2 + (k & 1)) * AG_WARP_OUT;
                    if (lane == 0) {
                        if (k == 0) bulk_wait_group_read<0>();
                        else bulk_wait_group_read<1>();
                    }
                    __syncwarp();
                    uint8_t* row = blk + lane * 32;
                    *reinterpret_cast<uint4*>(row) = make_uint4(ypk[k][0], ypk[k][1], ypk[k][2], ypk[k][3]);
                    *reinterpret_cast<uint4*>(row + 16) = make_uint4(ypk[k][4], ypk[k][5], ypk[k][6], ypk[k][7]);
                    fence_proxy_async();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_3d(&maps.c[k], blk, tc.tn * AG_BN + grp * 16, tc.tm * AG_BM + q * 32, tc.b);
                        bulk_commit_group();
                    }
                }
            } else if (row_ok) {
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    const int cb = cbase + c * 8;
                    const int valid = max(0, min(8, p.N - cb));
                    if (valid <= 0) continue;
#pragma unroll
                    for (int k = 0; k < NP * NS; ++k) {
                        __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(p.c[k]) + tc.b * p.c_bs +
                                             static_cast<int64_t>(r) * p.c_rs + cb;
                        if (vec && valid == 8) {
                            *reinterpret_cast<uint4*>(dst) =
                                make_uint4(ypk[k][c * 4], ypk[k][c * 4 + 1], ypk[k][c * 4 + 2], ypk[k][c * 4 + 3]);
                        } else {
                            for (int t = 0; t < valid; ++t)
                                dst[t] = __ushort_as_bfloat16(
                                    static_cast<unsigned short>((ypk[k][c * 4 + t / 2] >> (16 * (t & 1))) & 0xFFFFu));
                        }
                    }
                }
            }
          }
        }
        if (p.tma_store && lane == 0)
            bulk_wait_group_all();  // this warp's stores have completed before the CTA exits
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

template <int NP, int MODE, int NS>
static int launch_ag(const AgMaps& maps, AgParams& p, cudaStream_t stream) {
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(attn_score_gemm_kernel<NP, MODE, NS>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, AG_SMEM_BYTES);
        if (e != cudaSuccess) return cuda_fail(e, "pk_attn_score_gemm: cudaFuncSetAttribute");
        attr_set[dev] = true;
    }
    const int grid = static_cast<int>(std::min<int64_t>(p.total_units, num_sms()));
    void* tok;
    prof_begin(MODE == AG_PROBS ? "attn_probs_gemm" : "attn_dscores_gemm", stream, &tok);
    PK_LAUNCHED(attn_score_gemm_kernel<NP, MODE, NS><<<grid, AG_THREADS, AG_SMEM_BYTES, stream>>>(maps, p));
    prof_end(MODE == AG_PROBS ? "attn_probs_gemm" : "attn_dscores_gemm", stream, tok);
    PK_CHECK_LAUNCH("pk_attn_score_gemm: kernel launch");
    return PK_OK;
}

// Output plane map for the epilogue's TMA stores: boxes of 16 columns (32 bytes) x 32 rows, no
// swizzle (one epilogue warp's block of one plane).
static int encode_out_map(CUtensorMap* map, const void* base, int64_t cols, int64_t rows, int64_t batch,
                          int64_t row_bytes, int64_t batch_bytes) {
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows),
                                static_cast<cuuint64_t>(batch)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(row_bytes), static_cast<cuuint64_t>(batch_bytes)};
    const cuuint32_t box[3] = {16u, 32u, 1u};
    CUresult r = encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
                              CU_TENSOR_MAP_SWIZZLE_NONE);
    return r == CUDA_SUCCESS ? PK_OK : fail(PK_ERR_CUDA, "pk_attn_score_gemm: cuTensorMapEncodeTiled failed");
}

static int attn_score_gemm(int mode, const char* what, int dtype, int degree, int64_t batch, int64_t M, int64_t N,
                           int64_t K, const void* const* a_planes, int64_t a_bs, int64_t a_rs, int64_t a_cs,
                           const void* const* b_planes, int64_t b_bs, int64_t b_rs, int64_t b_cs,
                           void* const* c_planes, int64_t c_bs, int64_t c_rs, const void* const* probs, int64_t p_bs,
                           int64_t p_rs, const void* rowv, int64_t rowv_bs, double scale, int causal,
                           int64_t causal_shift, void* stream_ptr) {
    const std::string w(what);
    // bfloat16 planes, or float32 attention given as bf16 (hi, lo) plane pairs: every plane array
    // then holds 2(n+1) pointers hi_0, lo_0, hi_1, ... (operands, probabilities and outputs alike)
    if (dtype != PK_BF16 && dtype != PK_F32)
        return fail(PK_ERR_UNSUPPORTED, w + ": bfloat16 planes or float32 as bf16 hi/lo pairs only");
    const int NS = dtype == PK_F32 ? 2 : 1;
    if (degree < 0 || degree >= AG_MAX_NP) return fail(PK_ERR_UNSUPPORTED, w + ": degree must be in [0, 3]");
    if (batch < 0 || M < 0 || N < 0 || K < 0) return fail(PK_ERR_ARG, w + ": negative size");
    if (M > 0x7fffffff || N > 0x7fffffff || K > 0x7fffffff || batch > 0x7fffffff)
        return fail(PK_ERR_UNSUPPORTED, w + ": dimension exceeds 2^31-1");
    if (batch == 0 || M == 0 || N == 0) return PK_OK;
    if (K == 0) return fail(PK_ERR_UNSUPPORTED, w + ": empty reduction");
    if (K > AG_MAX_K / NS)
        return fail(PK_ERR_UNSUPPORTED, w + (NS == 2 ? ": float32 reduction (head dimension) above 64"
                                                     : ": reduction (head dimension) above 128"));
    const int P = degree + 1;
    const int NPL = P * NS;  // plane pointers per array
    if (!a_planes || !b_planes || !c_planes || !rowv) return fail(PK_ERR_ARG, w + ": null plane array or row values");
    for (int k = 0; k < NPL; ++k)
        if (!a_planes[k] || !b_planes[k] || !c_planes[k]) return fail(PK_ERR_ARG, w + ": null plane pointer");
    if (mode == AG_DSCORES) {
        if (!probs) return fail(PK_ERR_ARG, w + ": null probability planes");
        for (int k = 0; k < NPL; ++k)
            if (!probs[k]) return fail(PK_ERR_ARG, w + ": null probability plane pointer");
    }
    const int am = operand_mode(PK_BF16, a_planes, NPL, batch, M, K, a_bs, a_rs, a_cs);
    const int bm = operand_mode(PK_BF16, b_planes, NPL, batch, N, K, b_bs, b_cs, b_rs);
    if (am == OPM_STAGED || bm == OPM_STAGED)
        return fail(PK_ERR_UNSUPPORTED, w + ": operand planes must be 16-byte aligned with k or rows contiguous "
                                            "and the other strides multiples of 8 elements");

    AgMaps maps;
    std::memset(&maps, 0, sizeof(maps));
    const TcOperand oa{am, M, K, K, batch, a_planes, a_bs, a_rs, a_cs, nullptr, nullptr, 0, false};
    const TcOperand ob{bm, N, K, K, batch, b_planes, b_bs, b_cs, b_rs, nullptr, nullptr, 0, false};
    int rc = encode_operand(maps.a, oa, NPL, false, AG_BM);
    if (rc) return rc;
    rc = encode_operand(maps.b, ob, NPL, false, AG_BN);
    if (rc) return rc;

    AgParams p{};
    p.batch = static_cast<int>(batch);
    p.M = static_cast<int>(M);
    p.N = static_cast<int>(N);
    p.kblocks = static_cast<int>(ceil_div(K, TC_BK));
    p.tiles_m = static_cast<int>(ceil_div(M, AG_BM));
    p.tiles_n = static_cast<int>(ceil_div(N, AG_BN));
    p.n_chunks = static_cast<int>(ceil_div(p.tiles_n, AG_CHUNK));
    const int64_t total = static_cast<int64_t>(p.tiles_m) * p.n_chunks * batch;
    if (total > 0x7fffffff) return fail(PK_ERR_UNSUPPORTED, w + ": too many tiles");
    p.total_units = static_cast<int>(total);
    p.a_bytes = NPL * p.kblocks * AG_A_BYTES;
    // the split form stores its outputs directly (no TMA-store staging), so the staging area's
    // shared memory goes to the B ring: 12 stages at degree 3, so that the next tile's stages
    // load while a tile's products run
    const int out_bytes = NS == 1 ? AG_OUT_BYTES : 0;
    p.nstages = std::min(AG_MAX_STAGES, (AG_SMEM_BUDGET - out_bytes - p.a_bytes) / AG_B_BYTES);
    // a k block's NPL B stages must be resident together; bf16 keeps two more for prefetch
    if (p.a_bytes + out_bytes > AG_SMEM_BUDGET || p.nstages < NPL + (NS == 1 ? 2 : 0))
        return fail(PK_ERR_UNSUPPORTED, w + ": reduction too long for the resident operand");
    p.a_mn = am == OPM_MNMAJOR;
    p.b_mn = bm == OPM_MNMAJOR;
    p.causal = causal ? 1 : 0;
    p.skip_far = causal == 2 ? 1 : 0;
    p.shift = causal_shift;
    p.scale = static_cast<float>(scale);
    p.c_bs = c_bs;
    p.c_rs = c_rs;
    p.p_bs = p_bs;
    p.p_rs = p_rs;
    bool vec = c_rs % 8 == 0 && (batch == 1 || c_bs % 8 == 0);
    // TMA stores of the output planes: 16-byte aligned bases and row / batch strides, rows and
    // batch entries not overlapping
    bool tstore = vec && c_rs >= N && (batch == 1 || c_bs >= M * c_rs);
    for (int k = 0; k < NPL; ++k) {
        p.c[k] = c_planes[k];
        if (reinterpret_cast<uintptr_t>(c_planes[k]) % 16) vec = tstore = false;
        if (mode == AG_DSCORES) {
            p.pr[k] = probs[k];
            if (reinterpret_cast<uintptr_t>(probs[k]) % 16) vec = false;
        }
    }
    if (mode == AG_DSCORES && (p_rs % 8 != 0 || (batch > 1 && p_bs % 8 != 0))) vec = false;
    p.vec_ok = vec ? 1 : 0;
    if (tstore) {
        const int64_t sb = batch > 1 ? c_bs * 2 : M * c_rs * 2;
        for (int k = 0; k < NPL && tstore; ++k)
            if (encode_out_map(&maps.c[k], c_planes[k], N, M, batch, c_rs * 2, sb) != PK_OK) tstore = false;
    }
    p.tma_store = (tstore && NS == 1) ? 1 : 0;
    p.rowv = static_cast<const float*>(rowv);
    p.rowv_bs = rowv_bs;
    p.status = device_status_ptr();
    // Schedule: unit shapes by live (unmasked) tile count, heaviest first, so that the rounds of
    // the snake deal comparable units together (causal masking makes a static round-robin over
    // the natural order leave some SMs with far more tiles than others).  Fully masked units stay
    // in the schedule as the last class: their epilogue writes the zero tiles.
    p.n_groups = 0;
    if (static_cast<int64_t>(p.tiles_m) * p.n_chunks <= AG_MAX_SHAPES) {
        std::vector<int> by_cost[AG_CHUNK + 1];
        for (int ch = 0; ch < p.n_chunks; ++ch) {
            for (int tm = 0; tm < p.tiles_m; ++tm) {
                const int tn0 = ch * AG_CHUNK, tn1 = std::min(p.tiles_n, tn0 + AG_CHUNK);
                const int64_t last_row = std::min<int64_t>(static_cast<int64_t>(tm) * AG_BM + AG_BM - 1, M - 1);
                int cost = 0;
                for (int tn = tn0; tn < tn1; ++tn)
                    if (!p.causal || static_cast<int64_t>(tn) * AG_BN <= last_row + p.shift) ++cost;
                by_cost[cost].push_back(ch * p.tiles_m + tm);
            }
        }
        int s = 0, g = 0;
        int64_t rank = 0;
        for (int cost = AG_CHUNK; cost >= 0; --cost) {
            if (by_cost[cost].empty()) continue;
            p.grp_first[g] = s;
            p.grp_cum[g] = static_cast<int>(rank);
            for (int code : by_cost[cost]) p.order[s++] = static_cast<uint16_t>(code);
            rank += static_cast<int64_t>(by_cost[cost].size()) * batch;
            ++g;
        }
        p.grp_first[g] = s;
        p.grp_cum[g] = static_cast<int>(rank);
        p.n_groups = g;
    }
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    switch ((P * 2 + mode) * 2 + (NS - 1)) {
        case 4: return launch_ag<1, AG_PROBS, 1>(maps, p, stream);
        case 5: return launch_ag<1, AG_PROBS, 2>(maps, p, stream);
        case 6: return launch_ag<1, AG_DSCORES, 1>(maps, p, stream);
        case 7: return launch_ag<1, AG_DSCORES, 2>(maps, p, stream);
        case 8: return launch_ag<2, AG_PROBS, 1>(maps, p, stream);
        case 9: return launch_ag<2, AG_PROBS, 2>(maps, p, stream);
        case 10: return launch_ag<2, AG_DSCORES, 1>(maps, p, stream);
        case 11: return launch_ag<2, AG_DSCORES, 2>(maps, p, stream);
        case 12: return launch_ag<3, AG_PROBS, 1>(maps, p, stream);
        case 13: return launch_ag<3, AG_PROBS, 2>(maps, p, stream);
        case 14: return launch_ag<3, AG_DSCORES, 1>(maps, p, stream);
        case 15: return launch_ag<3, AG_DSCORES, 2>(maps, p, stream);
        case 16: return launch_ag<4, AG_PROBS, 1>(maps, p, stream);
        case 17: return launch_ag<4, AG_PROBS, 2>(maps, p, stream);
        case 18: return launch_ag<4, AG_DSCORES, 1>(maps, p, stream);
        default: return launch_ag<4, AG_DSCORES, 2>(maps, p, stream);
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
