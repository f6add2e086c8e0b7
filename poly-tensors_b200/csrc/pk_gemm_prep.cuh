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

}  // namespace pk
