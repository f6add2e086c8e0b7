// Operand staging for the polynomial matrix product.
//
// Every operand plane (A_p: M x K, B_p: K x N, any element strides) is rewritten
// once into a K-major workspace "sub-plane" [rows][Kp] so that the product kernels
// read tiles with TMA (tcgen05 path) or 16-byte cp.async (DMMA path) no matter how
// the caller's planes were laid out (transposed weights, batch views, ...).
//
//   float32  -> two bfloat16 sub-planes (hi, lo) with x ~= hi + lo: the product
//               kernel evaluates a*b ~= a_hi b_hi + a_hi b_lo + a_lo b_hi on the
//               bf16 tensor cores, accumulating in fp32.
//   bf16/f16 -> one sub-plane of the same type.
//   float64  -> one float64 sub-plane.
//   complex128 (interleaved) -> float64 sub-planes (re, im) and, for A, -im, so that
//               the complex product is a plain sum of real products.
#pragma once

#include "pk_common.cuh"

namespace pk {

// Which sub-planes one staged source plane produces.
enum StageKind {
    STAGE_SPLIT_BF16 = 0,  // f32 -> (hi, lo) bf16
    STAGE_COPY_16 = 1,     // bf16 -> bf16 or f16 -> f16
    STAGE_F64 = 2,         // f64 -> f64
    STAGE_C128_A = 3,      // c128 -> (re, im, -im) f64
    STAGE_C128_B = 4       // c128 -> (re, im) f64
};

struct StagePlane {
    const void* src;   // plane base pointer
    int64_t dst_sub;   // index of the first destination sub-plane (within this batch entry)
    int kind;          // StageKind
};

struct StageParams {
    StagePlane plane[PK_MAX_PLANES];
    int planes;
    int64_t rows, K, Kp;          // operand viewed as rows x K
    int64_t s_b, s_r, s_k;        // source element strides (batch, row, k)
    int64_t subs_per_batch;       // destination sub-planes per batch entry
    void* dst;                    // workspace base
    int elem_bytes;               // destination element size (2 or 8)
};

// =====================================================================================
// tcgen05 operand access (shared by the polynomial product and the attention score kernels)

constexpr int TC_BK = 64;  // k extent of one operand tile: 64 bf16 = one 128-byte swizzle row

// How the kernel reads an operand's planes (bf16 / f16 products; float32 products always
// read the staged hi/lo workspace through one map).
enum OperandMode {
    OPM_STAGED = 0,   // K-major workspace sub-planes written by the staging kernels
    OPM_KMAJOR = 1,   // the caller's planes, k contiguous: 64 x rows boxes
    OPM_MNMAJOR = 2   // the caller's planes, rows contiguous: 64 (rows) x 64 (k) boxes
};

// Whether a bf16 operand's planes can be read in place by the tensor maps: 16-byte aligned
// bases, one contiguous axis (k or rows) and the other strides multiples of 16 bytes that do
// not make rows (or batch entries) overlap.  s_rows / s_k: element strides along the rows
// (M or N) and along k.
inline int operand_mode(int dtype, const void* const* planes, int P, int64_t batch, int64_t rows, int64_t K,
                        int64_t s_b, int64_t s_rows, int64_t s_k) {
    if (dtype != PK_BF16 && dtype != PK_F16) return OPM_STAGED;
    for (int p = 0; p < P; ++p)
        if (reinterpret_cast<uintptr_t>(planes[p]) % 16) return OPM_STAGED;
    if (s_k == 1 && s_rows % 8 == 0 && s_rows >= K && (batch == 1 || (s_b % 8 == 0 && s_b >= rows * s_rows)))
        return OPM_KMAJOR;
    if (s_rows == 1 && s_k % 8 == 0 && s_k >= rows && (batch == 1 || (s_b % 8 == 0 && s_b >= K * s_k)))
        return OPM_MNMAJOR;
    return OPM_STAGED;
}

// 3-D 16-bit (bf16, or f16 with f16 = true) tensor map with the 128-byte swizzle: dims
// {d0 (innermost), d1, d2}, byte strides {s1, s2} of dims 1 and 2, box {64, box1, 1}.
inline int encode_map3(CUtensorMap* map, const void* base, int64_t d0, int64_t d1, int64_t d2, int64_t s1,
                       int64_t s2, int box1, bool f16 = false) {
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(d0), static_cast<cuuint64_t>(d1), static_cast<cuuint64_t>(d2)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(s1), static_cast<cuuint64_t>(s2)};
    const cuuint32_t box[3] = {static_cast<cuuint32_t>(TC_BK), static_cast<cuuint32_t>(box1), 1u};
    CUresult r = encode_tiled(map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                              const_cast<void*>(base), dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (r != CUDA_SUCCESS) return fail(PK_ERR_CUDA, "pk_poly_gemm: cuTensorMapEncodeTiled failed (" + std::to_string(r) + ")");
    return PK_OK;
}

// One operand of a tcgen05 product as the kernel reads it.
struct TcOperand {
    int mode;                      // OperandMode
    int64_t rows;                  // M for A, N for B
    int64_t K, Kp;
    int64_t batch;
    const void* const* planes;     // caller planes (direct modes)
    int64_t s_b, s_rows, s_k;      // caller element strides (direct modes)
    const char* ws;                // staged workspace base
    const int* first;              // first staged sub-plane of each plane
    int64_t subs;                  // staged sub-planes per batch entry
    bool f16;                      // float16 planes (bfloat16 otherwise)
};

// Per-plane maps (bf16 / f16 products), or one map over the whole staged workspace (float32).
inline int encode_operand(CUtensorMap* maps, const TcOperand& o, int planes, bool split, int box_rows) {
    if (split)
        return encode_map3(&maps[0], o.ws, o.Kp, o.rows, o.batch * o.subs, o.Kp * 2, o.rows * o.Kp * 2, box_rows);
    for (int p = 0; p < planes; ++p) {
        int rc;
        if (o.mode == OPM_KMAJOR) {
            const int64_t sb = o.batch > 1 ? o.s_b * 2 : o.rows * o.s_rows * 2;
            rc = encode_map3(&maps[p], o.planes[p], o.K, o.rows, o.batch, o.s_rows * 2, sb, box_rows, o.f16);
        } else if (o.mode == OPM_MNMAJOR) {
            const int64_t sb = o.batch > 1 ? o.s_b * 2 : o.K * o.s_k * 2;
            rc = encode_map3(&maps[p], o.planes[p], o.rows, o.K, o.batch, o.s_k * 2, sb, 64, o.f16);
        } else {
            const char* base = o.ws + static_cast<int64_t>(o.first[p]) * o.rows * o.Kp * 2;
            rc = encode_map3(&maps[p], base, o.Kp, o.rows, o.batch, o.Kp * 2, o.subs * o.rows * o.Kp * 2, box_rows,
                             o.f16);
        }
        if (rc) return rc;
    }
    return PK_OK;
}

}  // namespace pk
