// lalb_kernels.cuh -- argument blocks and launchers shared between the
// kernel files and the decoder.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "lalb.h"
#include "lalb_attention.cuh"

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
    float eps;             // kInF32Rms: RMSNorm epsilon
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
    int w_l2_first;        // the weights may come from the preceding kernel: before the
                           //   dependency wait they are only prefetched into L2
    int wr, teams;         // set by the launcher: warps per row, teams per CTA
    int nstages;           // set by the launcher
    unsigned int *status;  // set by the launcher
};

struct Q8HeadArgs {
    const int8_t *W;       // [rows][K], the full matrix (row_begin is absolute)
    const float *sw;       // [rows]
    int K, row_begin, row_end;
    const float *x;        // kInF32 / kInF32Rms
    const float *gamma;    // kInF32Rms, nullable (unit weights)
    float eps;             // kInF32Rms: RMSNorm epsilon
    const int8_t *xq;      // kInQ8
    const float *sx;
    float *logits;         // [row_end-row_begin], nullable
    int32_t *isum;         // nullable [row_end-row_begin][K/32]
    int32_t *argmax;       // nullable
    unsigned long long *best;  // argmax reduction scratch (8 bytes)
    unsigned int *ticket;      // CTA ticket counter (4 bytes)
    int nstages;
    unsigned int *status;
    int fail_argmax;           // nonzero: publish argmax = -1 when the status word is raised
};

int lalb_launch_q4k_gemv(lalb_ctx *ctx, const Q4kGemvArgs &a, int in, int epi,
                         cudaStream_t stream, bool pdl, int ctas_per_sm);
int lalb_launch_q8_head(lalb_ctx *ctx, const Q8HeadArgs &a, int in, cudaStream_t stream,
                        bool pdl, int ctas_per_sm);

// Decode attention (lalb_attention.cu): shape check, the standalone kernel
// (ctas CTAs; the position from *pos_ptr when given) and the kernel that
// advances a decoder's position word after a token.
int lalb_attention_check(int n_head, int n_kv, int hd);
int lalb_launch_attention(lalb_ctx *ctx, const lalb::AttnStep &a, const int *pos_ptr, int max_ctx,
                          int ctas, cudaStream_t s);
int lalb_launch_advance_position(lalb_ctx *ctx, int *pos, cudaStream_t s);
int lalb_launch_set_position(lalb_ctx *ctx, int *pos, int value, cudaStream_t s);

// One decode token in a single persistent, cooperative kernel, optionally
// tensor-parallel over n_rank GPUs.  Every rank holds a contiguous shard of
// the rows of gate/up, down and the LM head, all rows of qkv and o
// (lalb_tp_range), and an exchange buffer with the full activations.  A CTA
// stores its gate/up and down output rows into every rank's buffer (peer
// memory over NVLink); qkv and o outputs stay in the rank's own buffer, and
// the barriers after them are the rank's own.
constexpr int kPersistMaxRanks = 8;

struct PersistRank {                    // one rank's weight shards (device)
    const lalb_layer_weights *layers;   // [n_layer] row shards of the 4 matrices
    const int8_t *lm_w;                 // LM-head row shard [rows][hidden]
    const float *lm_s;
};

struct PersistArgs {
    int n_layer, hidden, q_rows, kv_rows, ffn, vocab;
    int ppl;                            // phases per layer: 4, or 5 with attention
    int norm;                           // nonzero: some RMSNorm weight vector is set
    int head_dim, max_ctx;              // attention (ppl == 5)
    double rope_theta;
    float *const *kv_cache;             // attention: [n_layer][2] (k, v) cache pointers
    int n_rank;                         // ranks in total (1: one GPU holds every row)
    int rank0, ranks_here;              // the ranks this launch computes, one CTA group each
    int cta_per_rank;                   // CTAs per rank (equal on every rank)
    int remote;                         // nonzero: some ranks are other GPUs (system scope)
    PersistRank rk[kPersistMaxRanks];   // [rank - rank0]
    unsigned char *xb[kPersistMaxRanks];   // every rank's exchange buffer (peer pointers)
    const float *h_in;                  // [hidden] token input, same on every rank
    float rms_eps;                      // RMSNorm epsilon
    const float *out_norm;              // nullable: RMSNorm weights before the LM head
    float *logits;                      // nullable: [vocab] (each rank writes its rows)
    int32_t *argmax;                    // nullable
    unsigned int *status;
    unsigned long long wait_ns;         // bound on a grid or cross-GPU wait (global timer)
    // nullable: per CTA and phase, timeline and counters (lalb_decoder_trace_step)
    unsigned long long *trace;
};

// Layout of one rank's exchange buffer (byte offsets; identical on every rank).
struct PersistXLayout {
    size_t gbar;      // u32 [ppl*n_layer]: this rank's CTAs done with each phase (monotonic
                      //   across tokens), then u32 [ppl*n_layer]: other ranks done (one
                      //   arrival per rank per phase), then u32: ranks' LM-head keys in
    size_t seq;       // u32: tokens completed by this rank
    size_t ticket;    // u32: this rank's CTAs done with the LM head (reset per token)
    size_t pos;       // i32: decode position (attention), advanced after every token
    size_t best;      // u64: this rank's argmax key (reset per token)
    size_t keys;      // u64 [kPersistMaxRanks]: every rank's argmax key for the token
    size_t h;         // f32 [hidden]: residual stream
    size_t q;         // f32 [q_rows + 2*kv_rows]: the qkv projection
    size_t att;       // f32 [q_rows]: attention output
    size_t att_cnt;   // u32 [n_head]: attention chunk arrivals (0 between phases)
    size_t att_part;  // f64 [n_head][8][head_dim + 2]: attention chunk partials
    size_t aq;        // i8  [ffn]: quantized SwiGLU product
    size_t asx;       // f32 [ffn/32]
    size_t asumq;     // i32 [ffn/32]
    size_t total;
};
__host__ __device__ inline PersistXLayout lalb_persist_xlayout(int n_layer, int hidden, int q_rows,
                                                               int kv_rows, int ffn, int head_dim) {
    auto up = [](size_t v) { return (v + 127) / 128 * 128; };
    const int ppl = head_dim > 0 ? 5 : 4;
    const int n_head = head_dim > 0 ? q_rows / head_dim : 0;
    PersistXLayout L;
    L.gbar = 0;
    L.seq = up((size_t)(2 * ppl * n_layer + 1) * 4);
    L.ticket = L.seq + 4;
    L.pos = L.seq + 8;
    L.best = L.seq + 16;
    L.keys = L.seq + 128;
    L.h = L.keys + 128;
    L.q = L.h + up((size_t)hidden * 4);
    L.att = L.q + up((size_t)(q_rows + 2 * kv_rows) * 4);
    L.att_cnt = L.att + up((size_t)(head_dim > 0 ? q_rows : 0) * 4);
    L.att_part = L.att_cnt + up((size_t)n_head * 4);
    L.aq = L.att_part + up((size_t)n_head * 8 * (head_dim + 2) * 8);
    L.asx = L.aq + up((size_t)ffn);
    L.asumq = L.asx + up((size_t)(ffn / 32) * 4);
    L.total = L.asumq + up((size_t)(ffn / 32) * 4);
    return L;
}

// Rows [row0, row1) of matrix `which` that rank r of n holds: 0 qkv, 1 o,
// 2 gate/up (whole 64-row gate/up tiles), 3 down, 4 LM head.
__host__ __device__ inline void lalb_tp_range(const lalb_decoder_cfg &c, int which, int n, int r,
                                              int *row0, int *row1) {
    int units, unit = 1;
    switch (which) {
        // qkv and o are small (16 MB per layer at the 7B shape): every rank
        // holds all their rows and computes q and the residual update
        // itself, so only gate/up, down and the head exchange across GPUs
        case 0: *row0 = 0; *row1 = c.q_rows + 2 * c.kv_rows; return;
        case 1: *row0 = 0; *row1 = c.hidden; return;
        case 3: units = c.hidden; break;
        case 2: units = 2 * c.ffn / 64; unit = 64; break;
        default: units = c.vocab; break;
    }
    // 32-bit: units < 2^24 and r <= 8 (the decoder checks the shapes)
    *row0 = (int)((unsigned)r * (unsigned)units / (unsigned)n) * unit;
    *row1 = (int)((unsigned)(r + 1) * (unsigned)units / (unsigned)n) * unit;
}

// Limits of the persistent kernel (checked by the decoder).
constexpr int kPersistMaxHidden = 4096;   // K of qkv, gate/up, head; q_rows
constexpr int kPersistMaxFfn = 20480;     // K of down
int lalb_persist_smem_bytes();
int lalb_persist_max_tiles();
int lalb_launch_persist(lalb_ctx *ctx, const PersistArgs &a, cudaStream_t stream);
