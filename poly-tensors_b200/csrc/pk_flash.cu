// Series flash attention, forward: O = softmax(scale * Q K^T, causal) V with every product
// a truncated Cauchy product, in one kernel (bfloat16 storage, fp32 accumulation).
//
// The reference evaluates this as its SDPA decomposition (src/polytensors/_decompositions.py:28-43)
// with the full (L, S) score series materialised per coefficient plane; its degree-1 Triton
// kernel (src/polytensors/_attention_kernels.py:27-82) is the single-kernel form for degree 1.
// Here, for degree n <= 3, one CTA owns 128 query rows and a 64-wide slice of the output
// columns and streams 64-key blocks:
//
//   S_k   = sum_{a+b=k} Q_a K_b^T                 tcgen05 (A = Q, B = K from shared memory),
//                                                  all n+1 planes accumulated in TMEM
//   E     = exp(scale*S - m) as a series           16 softmax warps: 4 per TMEM lane quadrant
//                                                  (32 query rows), each owning 16 of the 64
//                                                  keys; row maxima and normaliser partials
//                                                  combine through shared memory.
//                                                  E_0 = exp(scale*S_0 - m), e = exp of the
//                                                  directions; l_k += sum_keys E_k
//   O~_k += sum_{a+b=k} E_a V_b                   tcgen05 with A = E (bf16) written back into
//                                                  TMEM over the spent score columns, B = V read
//                                                  MN-major straight from the caller's planes
//   O     = O~ (/) l                               series division in the epilogue
//
// Both contractions issue one MMA per left plane: Q_a (or E_a) meets K_0 .. K_{n-a} (V_0 ..
// V_{n-a}), whose products land in the adjacent TMEM planes a .. n, and those right planes sit in
// consecutive ring stages, so the n+1-a products are one MMA of N = 64 (n+1-a) columns (n+1 MMAs
// per 16-wide k step instead of (n+1)(n+2)/2, each Q plane read from shared memory once).
//
// The running maximum m is only raised (and O~, l rescaled) when a block's maximum exceeds it
// by more than FA_TAU, so most blocks skip the TMEM read-modify-write of O~; a stale m only
// scales E by at most e^FA_TAU, which fp32 accumulation absorbs.
#include <algorithm>
#include <cstring>

#include "pk_common.cuh"
#include "pk_series.cuh"

namespace pk {

constexpr int FA_BM = 128;           // query rows per CTA
constexpr int FA_BN = 64;            // keys per block
constexpr int FA_DS = 64;            // output columns per CTA
constexpr int FA_STAGES = 10;
constexpr int FA_TILE = 64 * 64 * 2;        // K chunk [64 keys][64 d] or V slice [64 keys][64 d], bf16
constexpr int FA_QTILE = FA_BM * 64 * 2;    // Q chunk [128][64], bf16
constexpr float FA_TAU = 8.0f;
constexpr int FA_SOFTMAX_WARPS = 16;         // 4 per TMEM lane quadrant, each owning 16 keys of a block
constexpr int FA_THREADS = 64 + 32 * FA_SOFTMAX_WARPS;
constexpr int FA_MAX_NP = 4;

// Plane a, sub-plane h (NS = 2: float32 planes as bf16 hi / lo pairs) at index a * NS + h.
struct FlashMaps {
    CUtensorMap q[2 * FA_MAX_NP];
    CUtensorMap k[2 * FA_MAX_NP];
    CUtensorMap v[2 * FA_MAX_NP];
};

struct FlashParams {
    int bh, L, S, D;
    int n_slices, q_tiles, causal;
    float scale;
    void* o[FA_MAX_NP];
    float* stats;  // optional: per query row (lse_0, logz_1..n) of the softmax series
    int* status;
};

template <int NP>
struct FlashCfg {
    static constexpr int S_COLS = NP * FA_BN;     // score / probability planes
    static constexpr int O_BASE = S_COLS;
    static constexpr int USED = 2 * NP * 64;
    static constexpr int TMEM_COLS = USED <= 128 ? 128 : (USED <= 256 ? 256 : 512);
};

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    return static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(lo))) |
           (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(hi))) << 16);
}

// NS = 1: bfloat16 planes, bf16 output.  NS = 2 (float32 attention): Q, K, V arrive as bf16
// (hi, lo) plane pairs; every product is a_hi b_hi + a_hi b_lo + a_lo b_hi, the probabilities are
// written into TMEM as hi pairs (columns 16g .. 16g+7 of a key group) and lo pairs (16g+8 ..
// 16g+15, the columns whose fp32 scores the same warp has already read), and O is float32.
template <int NP, int DCH, int NS>
__global__ void __launch_bounds__(FA_THREADS, 1)
    flash_fwd_kernel(const __grid_constant__ FlashMaps maps, const FlashParams p) {
    using Cfg = FlashCfg<NP>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sq = smem;
    uint8_t* ring = sq + NP * NS * DCH * FA_QTILE;
    uint64_t* full = reinterpret_cast<uint64_t*>(ring + FA_STAGES * FA_TILE);
    uint64_t* empty = full + FA_STAGES;
    uint64_t* q_full = empty + FA_STAGES;
    uint64_t* s_full = q_full + 1;
    uint64_t* p_ready = s_full + 1;
    uint64_t* pv_done = p_ready + 1;
    uint64_t* drain = pv_done + 1;
    uint64_t* s0_full = drain + 1;   // score plane 0 final (its only product Q_0 K_0 is done)
    uint64_t* p0_ready = s0_full + 1;  // probability plane 0 written (and O rescaled)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(p0_ready + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    float* red = reinterpret_cast<float*>(tmem_slot + 4);  // [4 key groups][128 rows][NP + 1]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int slice = blockIdx.x % p.n_slices;
    const int qt = p.q_tiles - 1 - static_cast<int>(blockIdx.x) / p.n_slices;  // heaviest (latest) tiles first
    const int bh = blockIdx.y;
    const int q0 = qt * FA_BM;
    int nblocks = (p.S + FA_BN - 1) / FA_BN;
    if (p.causal) nblocks = min(nblocks, (min(q0 + FA_BM, p.L) - 1) / FA_BN + 1);

    if (threadIdx.x == 0) {
        for (int s = 0; s < FA_STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(q_full, 1);
        mbar_init(s_full, 1);
        mbar_init(p_ready, 32 * FA_SOFTMAX_WARPS);
        mbar_init(pv_done, 1);
        mbar_init(drain, 1);
        mbar_init(s0_full, 1);
        mbar_init(p0_ready, 32 * FA_SOFTMAX_WARPS);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            mbar_arrive_expect_tx(q_full, NP * NS * DCH * FA_QTILE);
            for (int a = 0; a < NP * NS; ++a)
                for (int c = 0; c < DCH; ++c)
                    tma_load_3d(sq + (a * DCH + c) * FA_QTILE, &maps.q[a], q_full, c * 64, q0, bh);
            uint32_t stage = 0, phase = 0;
            int issued_parity[FA_STAGES];
#pragma unroll
            for (int s = 0; s < FA_STAGES; ++s) issued_parity[s] = -1;
            bool ok = true;
            for (int j = 0; j < nblocks && ok; ++j) {
                for (int t = 0; t < NS * NP * (DCH + 1) && ok; ++t) {
                    if (!mbar_wait_or_abort(&empty[stage], phase ^ 1, abort_flag, p.status, 401)) {
                        ok = false;
                        break;
                    }
                    uint8_t* dst = ring + stage * FA_TILE;
                    mbar_arrive_expect_tx(&full[stage], FA_TILE);
                    if (t < NS * NP * DCH) {
                        // head-dimension chunk major, then sub-plane, plane minor: a chunk's K planes
                        // of one sub-plane fill consecutive stages (one wide MMA reads them together)
                        const int c = t / (NS * NP), h = (t / NP) % NS, b = t % NP;
                        tma_load_3d(dst, &maps.k[b * NS + h], &full[stage], c * 64, j * FA_BN, bh);
                    } else {
                        const int u = t - NS * NP * DCH, h = u / NP, b = u % NP;
                        tma_load_3d(dst, &maps.v[b * NS + h], &full[stage], slice * FA_DS, j * FA_BN, bh);
                    }
                    issued_parity[stage] = static_cast<int>(phase);
                    if (++stage == FA_STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            {
                // Let every copy issued (Q included) land before the CTA can exit.
                const uint64_t t0 = pk_globaltimer();
                while (!mbar_try_wait(q_full, 0) && pk_globaltimer() - t0 < 1000000000ull) {
                }
            }
            if (!ok) {
                for (int s = 0; s < FA_STAGES; ++s) {
                    if (issued_parity[s] < 0) continue;
                    const uint64_t t0 = pk_globaltimer();
                    while (!mbar_try_wait(&full[s], static_cast<uint32_t>(issued_parity[s])) &&
                           pk_globaltimer() - t0 < 1000000000ull) {
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            // instruction descriptors without the N field; N = 64 m sets (8 m) << 17
            constexpr uint32_t idesc_qk0 = f16_idesc(1u, FA_BM, 0);
            constexpr uint32_t idesc_pv0 = f16_idesc(1u, FA_BM, 0) | (1u << 16);  // B (V) MN-major
            auto n_field = [](int m) { return static_cast<uint32_t>(FA_BN / 8 * m) << 17; };
            uint32_t stage = 0, phase = 0;
            bool ok = mbar_wait_or_abort(q_full, 0, abort_flag, p.status, 402);
            bool issued = false;
            // Shared-memory descriptors are built once; a tile or 16-wide k step further on only
            // advances the start-address field (bytes >> 4), so the single issuing thread spends
            // a couple of integer adds per MMA instead of rebuilding two descriptors.
            const uint64_t q_desc = sw128_kmajor_desc(smem_u32(sq));
            const uint64_t ring_kdesc = sw128_kmajor_desc(smem_u32(ring));
            const uint64_t ring_vdesc = sw128_mnmajor_desc_lbo(smem_u32(ring), FA_TILE);
            // The products of one left plane with the right planes b0 .. b1-1 go to the adjacent
            // accumulator planes a+b0 .. a+b1-1 and read consecutive ring stages, so they are ONE
            // MMA of N = 64 (b1 - b0) columns (K-major: 8-row groups 1024 B apart run on into the
            // next stage; MN-major V: 64-column atoms FA_TILE apart), split in two where the
            // stages wrap around the ring's end (`wrap` = planes before it).
            auto segments = [](int b0, int b1, int wrap, auto&& issue) {
                if (b0 < wrap) issue(b0, min(b1, wrap));
                if (b1 > wrap) issue(max(b0, wrap), b1);
            };
            for (int j = 0; j < nblocks && ok; ++j) {
                if (j > 0 && !mbar_wait_or_abort(pv_done, (j - 1) & 1, abort_flag, p.status, 403)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                // S_k = sum_{a+b=k} Q_a K_b^T over the head dimension (DCH chunks of 64)
                for (int c = 0; c < DCH && ok; ++c) {
                    uint32_t kst[NS][NP];
                    for (int h = 0; h < NS && ok; ++h) {
                        for (int b = 0; b < NP; ++b) {
                            if (!mbar_wait_or_abort(&full[stage], phase, abort_flag, p.status, 404)) {
                                ok = false;
                                break;
                            }
                            kst[h][b] = stage;
                            if (++stage == FA_STAGES) {
                                stage = 0;
                                phase ^= 1;
                            }
                        }
                    }
                    if (!ok) break;
                    tc_fence_after();
                    // products of sub-planes (hq of Q, hk of K): (hi, hi), then for float32 (hi, lo), (lo, hi)
                    auto qk = [&](int a, int b0, int b1) {
#pragma unroll
                        for (int cb = 0; cb < (NS == 2 ? 3 : 1); ++cb) {
                            const int hq = cb == 2 ? 1 : 0, hk = cb == 1 ? 1 : 0;
                            const int wrap = min(NP, FA_STAGES - static_cast<int>(kst[hk][0]));
                            const uint64_t qd = q_desc + (((a * NS + hq) * DCH + c) * FA_QTILE >> 4);
                            segments(b0, b1, wrap, [&](int s0, int s1) {
                                const uint64_t kd = ring_kdesc + (kst[hk][s0] * FA_TILE >> 4);
#pragma unroll
                                for (int kk = 0; kk < 4; ++kk)
                                    tc_mma_f16(tmem + (a + s0) * FA_BN, qd + kk * 2, kd + kk * 2,
                                               idesc_qk0 | n_field(s1 - s0),
                                               (c == 0 && a == 0 && kk == 0 && cb == 0) ? 0u : 1u);
                            });
                        }
                    };
                    if (c + 1 < DCH) {
                        qk(0, 0, NP);
                    } else {
                        // S_0 = Q_0 K_0^T is complete once the last chunk's Q_0 K_0 product is
                        // issued: the softmax warps start on plane 0 while the other products run
                        qk(0, 0, 1);
                        tc_commit(s0_full);
                        qk(0, 1, NP);
                    }
#pragma unroll
                    for (int a = 1; a < NP; ++a) qk(a, 0, NP - a);
                    issued = true;
#pragma unroll
                    for (int h = 0; h < NS; ++h)
#pragma unroll
                        for (int b = 0; b < NP; ++b) tc_commit(&empty[kst[h][b]]);
                }
                if (!ok) break;
                tc_commit(s_full);
                // O~_k += sum_{a+b=k} E_a V_b, E_a in TMEM: the bf16 pairs of keys 16kk..16kk+15 sit in
                // columns 16kk..16kk+7 of S_a (written by the warp that owned those scores).  The E_0
                // products run first (as soon as plane 0 is written), the V_b stages are kept until
                // the higher planes' products have been issued too.
                if (!mbar_wait_or_abort(p0_ready, j & 1, abort_flag, p.status, 409)) {
                    ok = false;
                    break;
                }
                uint32_t vst[NS][NP];
                for (int h = 0; h < NS && ok; ++h) {
                    for (int b = 0; b < NP; ++b) {
                        if (!mbar_wait_or_abort(&full[stage], phase, abort_flag, p.status, 406)) {
                            ok = false;
                            break;
                        }
                        vst[h][b] = stage;
                        if (++stage == FA_STAGES) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                }
                if (!ok) break;
                tc_fence_after();
                // products (he of E, hv of V): (hi, hi), then for float32 (hi, lo), (lo, hi); E's lo
                // pairs of keys 16kk.. sit 8 columns after its hi pairs
                auto pv = [&](int a) {
#pragma unroll
                    for (int cb = 0; cb < (NS == 2 ? 3 : 1); ++cb) {
                        const int he = cb == 2 ? 1 : 0, hv = cb == 1 ? 1 : 0;
                        const int vwrap = min(NP, FA_STAGES - static_cast<int>(vst[hv][0]));
                        segments(0, NP - a, vwrap, [&](int s0, int s1) {
                            const uint64_t vd = ring_vdesc + (vst[hv][s0] * FA_TILE >> 4);
#pragma unroll
                            for (int kk = 0; kk < 4; ++kk)
                                tc_mma_f16_ts(tmem + Cfg::O_BASE + (a + s0) * FA_DS, tmem + a * FA_BN + kk * 16 + he * 8,
                                              vd + kk * (2048 >> 4), idesc_pv0 | n_field(s1 - s0),
                                              (j == 0 && a == 0 && kk == 0 && cb == 0) ? 0u : 1u);
                        });
                    }
                };
                pv(0);
                if (!mbar_wait_or_abort(p_ready, j & 1, abort_flag, p.status, 405)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int a = 1; a < NP; ++a) pv(a);
#pragma unroll
                for (int h = 0; h < NS; ++h)
#pragma unroll
                    for (int b = 0; b < NP; ++b) tc_commit(&empty[vst[h][b]]);
                tc_commit(pv_done);
            }
            if (!ok && issued) {
                tc_commit(drain);
                const uint64_t t0 = pk_globaltimer();
                while (!mbar_try_wait(drain, 0) && pk_globaltimer() - t0 < 1000000000ull) {
                }
            }
        }
    } else {
        // ---------------- softmax + epilogue ----------------
        // warp w (2..17) accesses TMEM lanes 32*(w%4)..+31 (query rows); key group g = (w-2)/4
        // owns keys 16g..16g+15 of every block and output columns 16g..16g+15 of the slice.
        const int quad = warp & 3;
        const int g = (warp - 2) >> 2;
        const uint32_t lane_base = 32u * quad;
        const int row = static_cast<int>(lane_base) + lane;
        const uint32_t trow = tmem + (lane_base << 16);
        const int q = q0 + row;
        const float sc = p.scale;
        float m_used = -INFINITY;
        float l[NP];
#pragma unroll
        for (int k = 0; k < NP; ++k) l[k] = 0.f;
        auto quad_sync = [&]() { asm volatile("bar.sync %0, %1;" ::"r"(1 + quad), "r"(128) : "memory"); };
        bool ok = true;
        for (int j = 0; j < nblocks; ++j) {
            // ---- phase 1: plane 0 (final once Q_0 K_0 is multiplied): row maxima, the rescale of
            // O~ when the maximum moved, E_0 = exp(scale * S_0 - m) and its bf16 pairs over S_0
            if (!mbar_wait_or_abort(s0_full, j & 1, abort_flag, p.status, 407)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const int key0 = j * FA_BN + g * 16;
            const int last_key = p.causal ? min(q, p.S - 1) : p.S - 1;
            uint32_t r0[16];
            tmem_ld_32x32b_x16(trow + g * 16, r0);
            tmem_ld_wait();
            float pmax = -INFINITY;
#pragma unroll
            for (int t = 0; t < 16; ++t)
                if (key0 + t <= last_key) pmax = fmaxf(pmax, sc * __uint_as_float(r0[t]));
            red[(g * 128 + row) * (NP + 1)] = pmax;
            quad_sync();
            float bmax = -INFINITY;
#pragma unroll
            for (int gg = 0; gg < 4; ++gg) bmax = fmaxf(bmax, red[(gg * 128 + row) * (NP + 1)]);
            quad_sync();  // the partial maxima are read before the next block overwrites them
            float f = 1.f;
            bool rescale = false;
            if (bmax > -INFINITY && (m_used == -INFINITY || bmax > m_used + FA_TAU)) {
                if (m_used != -INFINITY) {
                    f = __expf(m_used - bmax);
                    rescale = true;
#pragma unroll
                    for (int k = 0; k < NP; ++k) l[k] *= f;
                }
                m_used = bmax;
            }
            float w[16];  // E_0 of this warp's 16 keys
            {
                uint32_t packed0[8];
#pragma unroll
                for (int t = 0; t < 16; ++t) {
                    const bool live = key0 + t <= last_key && m_used > -INFINITY;
                    w[t] = live ? __expf(sc * __uint_as_float(r0[t]) - m_used) : 0.f;
                    l[0] += w[t];
                }
#pragma unroll
                for (int t = 0; t < 8; ++t) packed0[t] = pack_bf16x2(w[2 * t], w[2 * t + 1]);
                tmem_st_32x32b_x8(trow + g * 16, packed0);
                if constexpr (NS == 2) {
                    // lo = bf16(E - hi), the part of E the rounded hi misses
                    uint32_t lo0[8];
#pragma unroll
                    for (int t = 0; t < 8; ++t)
                        lo0[t] = pack_bf16x2(w[2 * t] - __uint_as_float(packed0[t] << 16),
                                             w[2 * t + 1] - __uint_as_float(packed0[t] & 0xFFFF0000u));
                    tmem_st_32x32b_x8(trow + g * 16 + 8, lo0);
                }
            }
            // rescale this warp's 16 columns of every O~ plane where the row maximum moved
            if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
                for (int k = 0; k < NP; ++k) {
                    uint32_t o[16];
                    const uint32_t addr = trow + Cfg::O_BASE + k * FA_DS + g * 16;
                    tmem_ld_32x32b_x16(addr, o);
                    tmem_ld_wait();
#pragma unroll
                    for (int t = 0; t < 16; ++t) o[t] = __float_as_uint(__uint_as_float(o[t]) * f);
                    tmem_st_32x32b_x16(addr, o);
                }
            }
            tmem_st_wait();
            tc_fence_before();
            mbar_arrive(p0_ready);
            // ---- phase 2: planes 1..n once all products are in: E_k = E_0 e_k with e the
            // exponential series of the directions (k e_k = sum_i i x_i e_{k-i}), bf16 over S_k
            if constexpr (NP > 1) {
                if (!mbar_wait_or_abort(s_full, j & 1, abort_flag, p.status, 410)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                uint32_t r[NP][16];
#pragma unroll
                for (int k = 1; k < NP; ++k) tmem_ld_32x32b_x16(trow + k * FA_BN + g * 16, r[k]);
                tmem_ld_wait();
                uint32_t packed[NP][8];
                uint32_t packed_lo[NS == 2 ? NP : 1][8];
#pragma unroll
                for (int t = 0; t < 16; t += 2) {
                    float e2[2][NP];
#pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        float x[NP], e[NP];
                        x[0] = 0.f;
#pragma unroll
                        for (int k = 1; k < NP; ++k) x[k] = sc * __uint_as_float(r[k][t + u]);
                        s_exp_dir<NP, float>(x, e);
#pragma unroll
                        for (int k = 1; k < NP; ++k) {
                            e2[u][k] = w[t + u] * e[k];
                            l[k] += e2[u][k];
                        }
                    }
#pragma unroll
                    for (int k = 1; k < NP; ++k) {
                        packed[k][t / 2] = pack_bf16x2(e2[0][k], e2[1][k]);
                        if constexpr (NS == 2)
                            packed_lo[k][t / 2] = pack_bf16x2(e2[0][k] - __uint_as_float(packed[k][t / 2] << 16),
                                                              e2[1][k] - __uint_as_float(packed[k][t / 2] & 0xFFFF0000u));
                    }
                }
#pragma unroll
                for (int k = 1; k < NP; ++k) {
                    tmem_st_32x32b_x8(trow + k * FA_BN + g * 16, packed[k]);
                    if constexpr (NS == 2) tmem_st_32x32b_x8(trow + k * FA_BN + g * 16 + 8, packed_lo[k]);
                }
                tmem_st_wait();
                tc_fence_before();
            }
            mbar_arrive(p_ready);
        }
        // epilogue: combine the four normaliser partials of each row, O = O~ (/) l for this
        // warp's 16 output columns, written as bf16
        if (ok) {
#pragma unroll
            for (int k = 0; k < NP; ++k) red[(g * 128 + row) * (NP + 1) + 1 + k] = l[k];
            quad_sync();
            float lt[NP];
#pragma unroll
            for (int k = 0; k < NP; ++k) {
                lt[k] = 0.f;
#pragma unroll
                for (int gg = 0; gg < 4; ++gg) lt[k] += red[(gg * 128 + row) * (NP + 1) + 1 + k];
            }
            if (p.stats && slice == 0 && g == 0 && q < p.L) {
                // the row's softmax normaliser as a series: lse_0 = m + log l_0 and the
                // directions of log(l / l_0); a row without admissible keys gets lse_0 = +inf
                float st[NP];
                if (lt[0] > 0.f) {
                    float u[NP];
                    const float inv0 = 1.f / lt[0];
                    u[0] = 1.f;
#pragma unroll
                    for (int k = 1; k < NP; ++k) u[k] = lt[k] * inv0;
                    s_log1<NP, float>(u, st);
                    st[0] = m_used + logf(lt[0]);
                } else {
#pragma unroll
                    for (int k = 0; k < NP; ++k) st[k] = 0.f;
                    st[0] = INFINITY;
                }
                float* dst = p.stats + (static_cast<int64_t>(bh) * p.L + q) * NP;
#pragma unroll
                for (int k = 0; k < NP; ++k) dst[k] = st[k];
            }
            if (mbar_wait_or_abort(pv_done, (nblocks - 1) & 1, abort_flag, p.status, 408)) {
                tc_fence_after();
                const float inv = lt[0] > 0.f ? 1.f / lt[0] : 0.f;
                uint32_t r[NP][16];
#pragma unroll
                for (int k = 0; k < NP; ++k) tmem_ld_32x32b_x16(trow + Cfg::O_BASE + k * FA_DS + g * 16, r[k]);
                tmem_ld_wait();
                float o[NP][16];
#pragma unroll
                for (int t = 0; t < 16; ++t) {
#pragma unroll
                    for (int k = 0; k < NP; ++k) {
                        float acc = __uint_as_float(r[k][t]);
#pragma unroll
                        for (int c2 = 1; c2 <= k; ++c2) acc -= lt[c2] * o[k - c2][t];
                        o[k][t] = acc * inv;
                    }
                }
                if (q < p.L && NS == 2) {
#pragma unroll
                    for (int k = 0; k < NP; ++k) {
                        float* dst = static_cast<float*>(p.o[k]) + (static_cast<int64_t>(bh) * p.L + q) * p.D +
                                     slice * FA_DS + g * 16;
                        float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
                        for (int t = 0; t < 4; ++t)
                            d4[t] = make_float4(o[k][4 * t], o[k][4 * t + 1], o[k][4 * t + 2], o[k][4 * t + 3]);
                    }
                } else if (q < p.L) {
#pragma unroll
                    for (int k = 0; k < NP; ++k) {
                        uint32_t w[8];
#pragma unroll
                        for (int t = 0; t < 8; ++t) w[t] = pack_bf16x2(o[k][2 * t], o[k][2 * t + 1]);
                        __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(p.o[k]) +
                                             (static_cast<int64_t>(bh) * p.L + q) * p.D + slice * FA_DS + g * 16;
                        uint4* d4 = reinterpret_cast<uint4*>(dst);
                        d4[0] = make_uint4(w[0], w[1], w[2], w[3]);
                        d4[1] = make_uint4(w[4], w[5], w[6], w[7]);
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, Cfg::TMEM_COLS);
    }
}

static int encode_plane_map(CUtensorMap* map, const void* base, int64_t rows, int64_t D, int64_t bh, int box_rows) {
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(rows),
                                static_cast<cuuint64_t>(bh)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(D * 2), static_cast<cuuint64_t>(rows * D * 2)};
    const cuuint32_t box[3] = {64u, static_cast<cuuint32_t>(box_rows), 1u};
    CUresult r = encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
                              CU_TENSOR_MAP_SWIZZLE_128B);
    if (r != CUDA_SUCCESS)
        return fail(PK_ERR_CUDA, "pk_flash_attn_fwd: cuTensorMapEncodeTiled failed (" + std::to_string(r) + ")");
    return PK_OK;
}

template <int NP, int DCH, int NS>
static int launch_flash(const FlashMaps& maps, const FlashParams& p, cudaStream_t s) {
    const int smem = NP * NS * DCH * FA_QTILE + FA_STAGES * FA_TILE + 1024 + 512 + 4 * 128 * (NP + 1) * 4;
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(flash_fwd_kernel<NP, DCH, NS>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return cuda_fail(e, "pk_flash_attn_fwd: cudaFuncSetAttribute");
        attr_set[dev] = true;
    }
    dim3 grid(static_cast<unsigned>(p.q_tiles * p.n_slices), static_cast<unsigned>(p.bh));
    void* tok;
    prof_begin("flash_attn_fwd", s, &tok);
    PK_LAUNCHED(flash_fwd_kernel<NP, DCH, NS><<<grid, FA_THREADS, smem, s>>>(maps, p));
    prof_end("flash_attn_fwd", s, tok);
    PK_CHECK_LAUNCH("pk_flash_attn_fwd");
    return PK_OK;
}

}  // namespace pk

using namespace pk;

extern "C" int pk_flash_attn_fwd(int dtype, int degree, int64_t bh, int64_t L, int64_t S, int64_t D,
                                 const void* const* q, const void* const* k, const void* const* v, void* const* o,
                                 int causal, double scale, void* stats, void* stream) {
    // bfloat16 planes; or float32 attention with q / k / v given as bf16 (hi, lo) plane pairs
    // (2(n+1) pointers each: hi_0, lo_0, hi_1, ...) and float32 output planes
    if (dtype != PK_BF16 && dtype != PK_F32)
        return fail(PK_ERR_UNSUPPORTED, "pk_flash_attn_fwd: bfloat16 planes, or float32 as bf16 hi/lo pairs");
    const int NS = dtype == PK_F32 ? 2 : 1;
    if (degree < 0 || degree >= FA_MAX_NP) return fail(PK_ERR_UNSUPPORTED, "pk_flash_attn_fwd: degree must be <= 3");
    if (NS == 1 && D != 64 && D != 128)
        return fail(PK_ERR_UNSUPPORTED, "pk_flash_attn_fwd: head dimension must be 64 or 128");
    if (NS == 2 && D != 64) return fail(PK_ERR_UNSUPPORTED, "pk_flash_attn_fwd: float32 head dimension must be 64");
    if (bh <= 0 || L <= 0 || S <= 0) return bh == 0 || L == 0 ? PK_OK : fail(PK_ERR_ARG, "pk_flash_attn_fwd: empty keys");
    if (bh > 65535 || L > (1LL << 30) || S > (1LL << 30)) return fail(PK_ERR_UNSUPPORTED, "pk_flash_attn_fwd: too large");
    const int NP = degree + 1;
    FlashMaps maps;
    memset(&maps, 0, sizeof(maps));
    for (int a = 0; a < NP * NS; ++a) {
        if (!q[a] || !k[a] || !v[a]) return fail(PK_ERR_ARG, "pk_flash_attn_fwd: null plane");
        if ((reinterpret_cast<uintptr_t>(q[a]) | reinterpret_cast<uintptr_t>(k[a]) | reinterpret_cast<uintptr_t>(v[a])) %
            16)
            return fail(PK_ERR_ARG, "pk_flash_attn_fwd: planes must be 16-byte aligned");
        int rc = encode_plane_map(&maps.q[a], q[a], L, D, bh, FA_BM);
        if (!rc) rc = encode_plane_map(&maps.k[a], k[a], S, D, bh, FA_BN);
        if (!rc) rc = encode_plane_map(&maps.v[a], v[a], S, D, bh, FA_BN);
        if (rc) return rc;
    }
    for (int a = 0; a < NP; ++a) {
        if (!o[a]) return fail(PK_ERR_ARG, "pk_flash_attn_fwd: null output plane");
        if (reinterpret_cast<uintptr_t>(o[a]) % 16) return fail(PK_ERR_ARG, "pk_flash_attn_fwd: planes must be 16-byte aligned");
    }
    FlashParams p{};
    p.bh = static_cast<int>(bh);
    p.L = static_cast<int>(L);
    p.S = static_cast<int>(S);
    p.D = static_cast<int>(D);
    p.n_slices = static_cast<int>(D / FA_DS);
    p.q_tiles = static_cast<int>(ceil_div(L, FA_BM));
    p.causal = causal ? 1 : 0;
    p.scale = static_cast<float>(scale);
    for (int a = 0; a < NP; ++a) p.o[a] = o[a];
    p.stats = static_cast<float*>(stats);
    p.status = device_status_ptr();
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int dch = static_cast<int>(D / 64);
    if (NS == 2) {
        switch (NP) {
            case 1: return launch_flash<1, 1, 2>(maps, p, s);
            case 2: return launch_flash<2, 1, 2>(maps, p, s);
            case 3: return launch_flash<3, 1, 2>(maps, p, s);
            default: return launch_flash<4, 1, 2>(maps, p, s);
        }
    }
#define PK_FLASH(NPV)                                                              \
    case NPV: return dch == 1 ? launch_flash<NPV, 1, 1>(maps, p, s) : launch_flash<NPV, 2, 1>(maps, p, s);
    switch (NP) {
        PK_FLASH(1)
        PK_FLASH(2)
        PK_FLASH(3)
        PK_FLASH(4)
    }
#undef PK_FLASH
    return fail(PK_ERR_UNSUPPORTED, "pk_flash_attn_fwd: degree");
}
