// lalb_logic_gemm.cuh -- the seed STE model's logic layers from their int8
// codes on the tcgen05 tensor cores (lalb_logic_gemm.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "lalb_internal.cuh"

// Workspace bytes of calls with up to max_M rows of X.
size_t lalb_logic_gemm_ws_bytes(int rows, int K, int max_M);
// Y [M][rows] = srow[n] * (codes [rows][K] int8 . X [M][K] fp32) + bias[n]
// (bias may be null); codes and X 16-byte aligned, K % 32 == 0, ws 256-byte
// aligned with ws_bytes >= lalb_logic_gemm_ws_bytes(rows, K, M).
int lalb_logic_gemm(lalb_ctx *ctx, const int8_t *codes, const float *srow, const float *bias, int rows, int K,
                    const float *X, int M, void *ws, size_t ws_bytes, float *Y, cudaStream_t s);
