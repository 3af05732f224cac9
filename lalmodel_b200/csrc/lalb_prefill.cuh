// lalb_prefill.cuh -- the batched (prefill) Q4_K x Q8 matmul (lalb_prefill.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

#include "lalb_internal.cuh"

size_t lalb_prefill_ws_bytes(int rows, int K, int T);
int lalb_prefill_matmul(lalb_ctx *ctx, const void *W, int rows, int K, const float *X, int T, void *ws,
                        float *Y, cudaStream_t s);
