// lalb_kernels.cuh -- argument blocks and launchers shared between the
// kernel files and the decoder.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "lalb.h"

// activation input of a matvec
enum : int {
    kInF32 = 0,     // fp32 vector, quantized in the prologue
    kInF32Rms = 1,  // fp32 vector, RMS-normalised (unit or gamma weights) then quantized
    kInQ8 = 2,      // already quantized (xq, sx, sumq)
};

// epilogue of a Q4_K matvec
enum : int {
    kEpiStore = 0,   // y[r] = acc
    kEpiResid = 1,   // y[r] = resid[r] + acc (resid may alias y)
    kEpiSwiglu = 2,  // 64-row tiles: 32 gate + 32 up rows -> silu(g)*u -> Q8
};

struct Q4kGemvArgs {
    const uint8_t *W;
    int rows, K;
    const float *x;        // kInF32 / kInF32Rms
    const float *gamma;    // kInF32Rms, nullable (unit weights)
    const int8_t *xq;      // kInQ8
    const float *sx;
    const int32_t *sumq;
    float *y;              // kEpiStore / kEpiResid
    const float *resid;    // kEpiResid
    int32_t *isum;         // nullable: exact int32 sub-block dots [rows][K/32]
    int8_t *aq;            // kEpiSwiglu: quantized product [rows/2]
    float *asx;            //   its per-32 scales [rows/64]
    int32_t *asumq;        //   its per-32 sums [rows/64]
    float *act_out;        //   nullable: the fp32 product [rows/2]
    int unit;              // CTA row split granularity (64 for kEpiSwiglu)
    int act_bulk;          // set by the launcher: activations arrive by bulk copy
    int wr, teams;         // set by the launcher: warps per row, teams per CTA
    int nstages;           // set by the launcher
    unsigned int *status;  // set by the launcher
};

struct Q8HeadArgs {
    const int8_t *W;       // [rows][K], the full matrix (row_begin is absolute)
    const float *sw;       // [rows]
    int K, row_begin, row_end;
    const float *x;        // kInF32 / kInF32Rms
    const float *gamma;
    const int8_t *xq;      // kInQ8
    const float *sx;
    float *logits;         // [row_end-row_begin], nullable
    int32_t *isum;         // nullable [row_end-row_begin][K/32]
    int32_t *argmax;       // nullable
    unsigned long long *best;  // argmax reduction scratch (8 bytes)
    unsigned int *ticket;      // CTA ticket counter (4 bytes)
    int nstages;
    unsigned int *status;
};

int lalb_launch_q4k_gemv(lalb_ctx *ctx, const Q4kGemvArgs &a, int in, int epi,
                         cudaStream_t stream, bool pdl, int ctas_per_sm);
int lalb_launch_q8_head(lalb_ctx *ctx, const Q8HeadArgs &a, int in, cudaStream_t stream,
                        bool pdl, int ctas_per_sm);
