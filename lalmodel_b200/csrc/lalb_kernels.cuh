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

// One decode token in a single persistent, cooperative kernel.
struct PersistArgs {
    int n_layer, hidden, q_rows, kv_rows, ffn, vocab;
    const lalb_layer_weights *layers;  // device array [n_layer]
    const int8_t *lm_w;
    const float *lm_s;
    const float *h_in;                  // [hidden]
    float *h;                           // [hidden] residual stream
    float *qkv;                         // [q_rows + 2*kv_rows]
    int8_t *aq;                         // [ffn] quantized SwiGLU product
    float *asx;                         // [ffn/32]
    int32_t *asumq;                     // [ffn/32]
    float *logits;                      // [vocab], nullable
    int32_t *argmax;                    // nullable
    unsigned int *gbar;                 // [4*n_layer] grid-barrier arrival counters (zero)
    unsigned long long *best;           // argmax key (zero)
    unsigned int *ticket;               // CTAs done with the LM head (zero)
    unsigned int *status;
    // nullable: per CTA and phase, the global timer (ns) when the CTA's
    // consumers finished the phase's work and when they left its grid
    // barrier: [gridDim.x][n_phase][2]
    unsigned long long *trace;
};

// Limits of the persistent kernel (checked by the decoder).
constexpr int kPersistMaxHidden = 4096;   // K of qkv, gate/up, head; q_rows
constexpr int kPersistMaxFfn = 20480;     // K of down
int lalb_persist_smem_bytes();
int lalb_persist_max_tiles();
int lalb_launch_persist(lalb_ctx *ctx, const PersistArgs &a, cudaStream_t stream);
