// lalb_tc_gemm.cuh -- the tcgen05 tf32-split GEMM (lalb_tc_gemm.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

#include "lalb_internal.cuh"

// Y[m][n] = rowscale[m] * colscale[n] * sum_k A[m][k] B[n][k] + bias[n];
// A = a_hi (+ a_lo), B = b_hi (+ b_lo), every part exactly representable in
// tf32, or A raw fp32 with split_a set.  Row-major, K a multiple of 32, 16-byte aligned.
struct TcGemmParts {
    int M, N, K;
    const float *a_hi, *a_lo;   // [M][K]; a_lo nullable
    const float *b_hi, *b_lo;   // [N][K]; b_lo nullable
    float *Y;                   // [M][N]
    const float *rowscale;      // [M], nullable
    const float *colscale;      // [N], nullable
    const float *bias;          // [N], nullable
    int split_a;                // a_lo null: a_hi is raw fp32 and the kernel forms
                                // hi (its tf32 truncation) and lo = A - hi itself
};

int lalb_tc_gemm_tf32(lalb_ctx *ctx, const TcGemmParts &p, cudaStream_t s);
