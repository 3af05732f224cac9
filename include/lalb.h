/*
 * lalb.h -- C ABI of the B200 (sm_100a) quantized-matmul hot path of LAL.
 *
 * Plain C99, includable from the reference engine's C sources.  Every entry
 * point returns an int status (0 = LALB_OK, negative = lalb_status); none
 * exits, prints or falls back to the CPU.  All tensor arguments are DEVICE
 * pointers owned by the caller unless a name ends in _host; the library owns
 * only the context (a status word, a small scratch area and, for decoders,
 * activation buffers).  Work is enqueued on the caller's stream
 * (lalb_stream = cudaStream_t; NULL = the legacy default stream).
 *
 * Formats
 *   Q4_K  144-byte super-block per 256 weights, llama.cpp layout:
 *         fp16 d | fp16 dmin | 12 bytes packed 6-bit scales/mins | 128 bytes
 *         of 4-bit quants (32-byte group g holds sub-block 2g in the low
 *         nibbles and 2g+1 in the high nibbles); w = d*sc_j*q - dmin*m_j.
 *         A matrix is row-major: row r is K/256 consecutive blocks.
 *   Q8 activations  per 32-block: int8 q = clamp(roundf(x/s), +-127) with
 *         fp32 s = amax/127, plus sumq = sum of the 32 q (int32).
 *   Q8 LM head  int8 [rows][K] with one fp32 scale per row.
 *
 * Reference interfaces replaced (paths inside the reference project):
 *   lal_matmul_q4_k         runtime/lal_q4k_kernel.h (README.md:130,210)
 *   lal_lm_head_int8_range  runtime/lal_q8_kernel.h  (README.md:131,211)
 *   unpack_scales_6bit      (README.md:212)
 *   the lal_cuda.h pattern  runtime/lal_cuda.h:12-97 (extern "C", resident
 *                           device weights, runtime/lal_cuda.h:56-68)
 * The reference's kernel headers are absent from its snapshot; the
 * signatures below keep their names and argument meaning (weights, row
 * range, activation, output) with explicit sizes, a context and a stream.
 */
#ifndef LALB_H
#define LALB_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define LALB_API __attribute__((visibility("default")))
#else
#define LALB_API
#endif

#define LALB_ABI_VERSION 3
#define LALB_QK_K 256
#define LALB_QB 32
#define LALB_Q4K_BLOCK_BYTES 144

typedef enum {
    LALB_OK = 0,
    LALB_ERR_INVALID = -1,     /* bad pointer, size, alignment or state */
    LALB_ERR_CUDA = -2,        /* a CUDA runtime call failed */
    LALB_ERR_NOMEM = -3,       /* device or host allocation failed */
    LALB_ERR_UNSUPPORTED = -4, /* shape outside what the kernels handle */
    LALB_ERR_TIMEOUT = -5,     /* a bounded device wait gave up */
    LALB_ERR_COMM = -6,        /* multi-GPU communicator failure */
    LALB_ERR_DEVICE = -7       /* not an sm_100 device */
} lalb_status;

typedef struct lalb_ctx lalb_ctx;
typedef void *lalb_stream;

/* ---- context --------------------------------------------------------- */
LALB_API int         lalb_abi_version(void);
LALB_API const char *lalb_status_string(int status);
/* Binds the calling thread to `device` and allocates the context's status
 * word and scratch (a few hundred bytes).  Fails with LALB_ERR_DEVICE on a
 * device other than compute capability 10.0. */
LALB_API int         lalb_init(int device, lalb_ctx **out);
LALB_API int         lalb_destroy(lalb_ctx *ctx);
/* Text of the last error recorded on this context ("" if none). */
LALB_API const char *lalb_last_error(const lalb_ctx *ctx);
/* Synchronises the device and returns the device-side status word, a set
 * of bits: 1 = a bounded wait expired, 2 = a decode position outside the KV
 * cache was refused (0 = neither); reset != 0 clears it. */
LALB_API int         lalb_device_status(lalb_ctx *ctx, int reset);

/* ---- formats ---------------------------------------------------------- */
/* Host helper (no GPU): 12 packed bytes -> out16[0..7] scales,
 * out16[8..15] mins.  Replaces unpack_scales_6bit (README.md:212). */
LALB_API int lalb_unpack_scales_6bit(const uint8_t *scales12, uint8_t *out16);

/* Seeded N(0, sigma) fill of n floats (element i of stream `seed` is a
 * function of seed and offset+i only). */
LALB_API int lalb_fill_normal(lalb_ctx *ctx, float *out, size_t n, uint64_t seed,
                              uint64_t offset, float sigma, lalb_stream stream);

/* Min-max Q4_K quantization of w [rows][K] (K % 256 == 0) into
 * blocks [rows][K/256][144] (the converter's quantizer; README.md:48,154). */
LALB_API int lalb_q4k_quantize(lalb_ctx *ctx, const float *w, int rows, int K,
                               void *blocks, lalb_stream stream);

/* Per-row int8 quantization of an LM head w [rows][K]: s = amax/127,
 * q = clamp(roundf(w/s), +-127). */
LALB_API int lalb_q8_quantize_rows(lalb_ctx *ctx, const float *w, int rows, int K,
                                   int8_t *q, float *s, lalb_stream stream);

/* Per-32-block int8 activation quantizer for M vectors of K (K % 32 == 0):
 * xq [M][K], sx [M][K/32], sumq [M][K/32] (sumq may be NULL). */
LALB_API int lalb_quantize_act(lalb_ctx *ctx, const float *x, int M, int K,
                               int8_t *xq, float *sx, int32_t *sumq,
                               lalb_stream stream);

/* ---- Q4_K x Q8 matvec (decode, batch 1) --------------------------------
 * y[r] = sum_j sx_j * (d*sc_j*isum_j - dmin*m_j*sumq_j) over the 32-wide
 * sub-blocks j of row r, isum_j = the exact int32 dot of the 32 4-bit quants
 * with the 32 int8 activations.  The activation quantizer is fused: x is
 * fp32 [K].  W must be 16-byte aligned; K % 256 == 0, K <= 32768.
 * Replaces lal_matmul_q4_k (runtime/lal_q4k_kernel.h, README.md:130,210). */
LALB_API int lalb_matmul_q4_k(lalb_ctx *ctx, const void *W, int rows, int K,
                              const float *x, float *y, lalb_stream stream);

/* Same product on an activation already quantized by lalb_quantize_act.
 * isum (nullable) receives the int32 sub-block dots [rows][K/32]. */
LALB_API int lalb_matmul_q4_k_q8(lalb_ctx *ctx, const void *W, int rows, int K,
                                 const int8_t *xq, const float *sx,
                                 const int32_t *sumq, float *y, int32_t *isum,
                                 lalb_stream stream);

/* ---- Q8 LM head --------------------------------------------------------
 * For r in [row_begin, row_end): logits[r - row_begin] =
 *   sw[r] * sum_b sx_b * isum_b(r)   (isum_b = int32 dot of 32-block b)
 * with x (fp32 [K], K % 32 == 0, K <= 4096) quantized in the prologue.
 * argmax (nullable, device int32) receives the absolute row index of the
 * first maximum logit in the range.  W rows are K bytes; W + r*K must be
 * 16-byte aligned.  Calls on one context must not overlap on the GPU (the
 * argmax reduction uses the context's scratch).
 * Replaces lal_lm_head_int8_range (runtime/lal_q8_kernel.h,
 * README.md:131,211). */
LALB_API int lalb_lm_head_int8_range(lalb_ctx *ctx, const int8_t *W, const float *sw,
                                     int K, int row_begin, int row_end,
                                     const float *x, float *logits, int32_t *argmax,
                                     lalb_stream stream);

/* Same on a pre-quantized activation; isum (nullable) gets
 * [row_end-row_begin][K/32] int32 block dots. */
LALB_API int lalb_lm_head_int8_q8(lalb_ctx *ctx, const int8_t *W, const float *sw,
                                  int K, int row_begin, int row_end,
                                  const int8_t *xq, const float *sx, float *logits,
                                  int32_t *isum, int32_t *argmax, lalb_stream stream);

/* ---- decode attention (one layer, one token) ----------------------------
 * attention_forward after apply_rope (runtime/lal_runtime.c:833-882 and
 * :137-153, called as the layer forward calls them, :310-327), generalised
 * to grouped KV heads.  qkv = q [n_head*head_dim] | k [n_kv_head*head_dim]
 * | v [n_kv_head*head_dim] fp32.  RoPE at position pos on every q and k
 * head (pairs d, d + head_dim/2; angle pos * rope_theta^(-2d/head_dim));
 * the rotated k and the v go to row pos of k_cache / v_cache
 * ([max_ctx][n_kv_head*head_dim] fp32, 16-byte aligned); head h attends KV
 * head h / (n_head / n_kv_head) over positions 0..pos with scores scaled by
 * 1/sqrt(head_dim): out [n_head*head_dim] = sum_j softmax_j v_j (the
 * softmax's sum + 1e-12 in the denominator, as in the reference).  RoPE,
 * scores, softmax and the weighted sum are computed in double and rounded
 * to float once per value.  head_dim 32, 64, 128 or 256; n_kv_head divides
 * n_head; 0 <= pos < max_ctx; rope_theta > 1 (the reference uses 10000). */
LALB_API int lalb_attention_decode(lalb_ctx *ctx, const float *qkv, int n_head, int n_kv_head,
                                   int head_dim, int pos, int max_ctx, float rope_theta,
                                   float *k_cache, float *v_cache, float *out,
                                   lalb_stream stream);

/* ---- next-token sampling after the LM head --------------------------------
 * generate_text's sampling (models/ste_train.c:2229-2318) on device logits:
 *   adjusted = logits; ids < n_masked_low_ids -> -1e30 (the reference masks
 *   its 3 special ids); every distinct token of history[0..n_history) once:
 *   adjusted /= rep_penalty if > 0, else *= rep_penalty (the reference:
 *   1.5); no_repeat_ngram = n >= 2 bans (-1e30) every token that would
 *   complete an n-gram already in the history (the reference: 3);
 *   temperature <= 0.01: the first maximum (sample_argmax, :1503-1509);
 *   else the top_k largest (value descending, ties to the lower id),
 *   p_j = exp((a_j - a_0) / temperature) (float subtraction and division,
 *   the exponential in double rounded to float once), running float sums;
 *   the nucleus ends at the first j whose running sum exceeds top_p * sum
 *   (the reference: 0.9); r = u * (that running sum); the token is the
 *   first j of the nucleus with r < running sum.
 * u: device float in [0, 1) (nullable when greedy), so that a captured
 * graph can be fed a new draw per token.  ws: device workspace of
 * lalb_sample_ws_bytes(vocab, top_k) bytes (8-byte aligned; no contents
 * carried between calls).  token (device int32) gets the id; topk_id /
 * topk_prob (nullable, top_k entries) the ranked ids and their p_j.
 * Limits: 1 <= top_k <= 256, vocab up to 8192 * (16384 / top_k) ids. */
typedef struct {
    float temperature;
    int top_k;
    float top_p;
    float rep_penalty;     /* 1: off */
    int no_repeat_ngram;   /* 0: off */
    int n_masked_low_ids;  /* 0: none */
} lalb_sampling;
LALB_API int lalb_sample_ws_bytes(int vocab, int top_k, size_t *bytes);
LALB_API int lalb_sample(lalb_ctx *ctx, const float *logits, int vocab, const int32_t *history,
                         int n_history, const lalb_sampling *params, const float *u, void *ws,
                         int32_t *token, int32_t *topk_id, float *topk_prob, lalb_stream stream);

/* Allocation-free LM head.  This entry point has no counterpart in the
 * reference.  It is for callers that cannot call cudaMalloc: an engine whose
 * own memory pool owns the device and forbids libraries from allocating (a
 * cudaMalloc would also stall every stream on the device), or code that
 * cannot create a lalb_ctx because creating one allocates.  It computes
 * exactly what lalb_lm_head_int8_range computes, on the current device, with
 * no context and no allocation: its argmax reduction state (16 bytes) lives
 * in a 256-byte static device array that every GPU loading the library holds
 * until the process exits.  That need does not grow with the row count or K,
 * so the sizes it rejects are the kernel's own: K > 4096 returns
 * LALB_ERR_UNSUPPORTED; K not a multiple of 32, an inverted range, a null or
 * misaligned pointer return LALB_ERR_INVALID.  Errors are reported only
 * through the returned status (there is no context to hold a message),
 * except one that happens on the GPU after the call has returned: if a
 * bounded wait inside the kernel expires, the logits of the range are
 * incomplete and *argmax is set to -1 (pass argmax to be able to tell).
 * The first call on a device sets it up (looks up the array's device
 * address and reads the SM count); make that first call before any stream
 * capture.  Every call makes sure the kernel's shared-memory limit covers
 * its size, through the same never-lowering registry as the context-based
 * calls, so the two kinds of call can be mixed in any order.  Every call
 * shares the array and clears the 16 bytes it uses on the caller's stream
 * before the kernel runs; calls that overlap on the GPU (another stream,
 * another host thread on the same device) race on it. */
LALB_API int lalb_lm_head_int8_range_noalloc(const int8_t *W, const float *sw, int K,
                                             int row_begin, int row_end, const float *x,
                                             float *logits, int32_t *argmax,
                                             lalb_stream stream);

/* ---- Qwen2.5-shape decode (one token) -----------------------------------
 * Per layer, with h the fp32 residual stream [hidden]:
 *   qkv  = Wqkv . Q8(rmsnorm(h, attn_norm))    rows q_rows + 2*kv_rows
 *   att  = attention(qkv, KV cache, pos)       (lalb_attention_decode; with
 *                                              head_dim = 0 there is no
 *                                              attention and att = q, the
 *                                              matmul set alone)
 *   h    = h + Wo . Q8(att)
 *   a    = silu(gate) * up, gate/up = Wgu . Q8(rmsnorm(h, ffn_norm))
 *   h    = h + Wdown . Q8(a)
 * then logits = LMhead . Q8(rmsnorm(h, output norm)) and argmax.
 * rmsnorm is rms_norm (runtime/lal_runtime.c:82-87): out = (x * s) * w with
 * s = 1/sqrt(mean(x^2) + rms_eps), s computed in double and rounded to
 * float once; a NULL weight vector means unit weights.  silu(g)*u is
 * evaluated in double and rounded once.  Wgu interleaves gate and up in
 * 32-row tiles: rows [64t, 64t+32) are gate rows [32t, 32t+32), rows
 * [64t+32, 64t+64) the up rows of the same range.  Weights are caller-owned
 * device buffers. */
typedef struct {
    int n_layer;
    int hidden;     /* K of qkv / gate-up, rows of o / down */
    int q_rows;     /* n_head * head_dim */
    int kv_rows;    /* n_kv_head * head_dim */
    int ffn;        /* intermediate size */
    int vocab;      /* LM-head rows */
    float rms_eps;  /* RMSNorm epsilon; 0 selects 1e-5 (the reference's rms_norm) */
    int head_dim;   /* 0: no attention; else 32, 64, 128 or 256, dividing q_rows and
                     * kv_rows (q_rows/head_dim heads over kv_rows/head_dim KV heads) */
    int max_ctx;    /* positions of every layer's KV cache (attention only) */
    float rope_theta; /* RoPE base; 0 selects 10000 (the reference's apply_rope) */
} lalb_decoder_cfg;

typedef struct {
    const void *wqkv;        /* Q4_K [q_rows + 2*kv_rows][hidden] */
    const void *wo;          /* Q4_K [hidden][q_rows] */
    const void *wgu;         /* Q4_K [2*ffn][hidden], 32-row gate/up tiles */
    const void *wdown;       /* Q4_K [hidden][ffn] */
    const float *attn_norm;  /* [hidden] RMSNorm weights before qkv; NULL: unit */
    const float *ffn_norm;   /* [hidden] RMSNorm weights before gate/up; NULL: unit */
} lalb_layer_weights;

typedef struct lalb_decoder lalb_decoder;

LALB_API int lalb_decoder_create(lalb_ctx *ctx, const lalb_decoder_cfg *cfg,
                                 lalb_decoder **out);
LALB_API int lalb_decoder_set_layer(lalb_decoder *dec, int layer,
                                    const lalb_layer_weights *w);
LALB_API int lalb_decoder_set_lm_head(lalb_decoder *dec, const int8_t *w,
                                      const float *sw);
/* RMSNorm weights [hidden] applied before the LM head (NULL: unit, the
 * default).  Every rank of a tensor-parallel decoder holds them whole. */
LALB_API int lalb_decoder_set_output_norm(lalb_decoder *dec, const float *w);
/* Attention only: layer `layer`'s KV cache, two caller-owned device buffers
 * of max_ctx * kv_rows fp32 (16-byte aligned; row p holds position p).
 * Every rank of a tensor-parallel decoder holds its own full cache (the
 * attention is computed whole on every rank, like q and o). */
LALB_API int lalb_decoder_set_kv_cache(lalb_decoder *dec, int layer, float *k_cache,
                                       float *v_cache);
/* Attention only: the position of the next token (0 at creation); every step
 * attends positions 0..pos, writes row pos of the caches and advances pos.
 * A step at pos >= max_ctx fails with LALB_ERR_INVALID.  Enqueued on the
 * stream (no synchronisation); set the same position on every rank. */
LALB_API int lalb_decoder_set_position(lalb_decoder *dec, int pos, lalb_stream stream);
LALB_API int lalb_decoder_position(const lalb_decoder *dec);
/* One token on device buffers: h_in [hidden] (read only), h_out [hidden]
 * (nullable: final residual stream), logits [vocab] (nullable), argmax
 * (device int32, nullable).  On a non-default stream the token is captured
 * into a CUDA graph on first use of a pointer set and replayed after. */
LALB_API int lalb_decoder_step(lalb_decoder *dec, const float *h_in, float *h_out,
                               float *logits, int32_t *argmax, lalb_stream stream);
/* One token from host memory: copies h_in_host (pinned recommended) to the
 * device, runs the step, copies the argmax back to *argmax_host and waits
 * for the stream. */
LALB_API int lalb_decoder_step_host(lalb_decoder *dec, const float *h_in_host,
                                    int32_t *argmax_host, lalb_stream stream);
/* One token on the per-phase kernel chain with a CUDA event between
 * consecutive kernels (no programmatic overlap): kernel_us (host,
 * P*n_layer + 1 floats, P = 5 with attention, else 4) receives each
 * kernel's duration in launch order -- per layer qkv, (attention,) o,
 * gate/up, down; then the LM head.  Synchronises the stream. */
LALB_API int lalb_decoder_profile_step(lalb_decoder *dec, const float *h_in,
                                       float *kernel_us, lalb_stream stream);
/* One token on the persistent path with a phase timeline: trace_host
 * (host, trace_len >= n_cta * (P*n_layer + 1) * 8 values, P as above) receives, for
 * each CTA and phase, six GPU global-timer figures (ns): [0] the CTA
 * finished the phase's work, [1] it left the grid barrier that ends the
 * phase, [2] its activation prologue was done, [3] the time its first
 * consumer warp waited for weights in the phase and [4] the time it spent
 * computing, [5] its producer had issued the phase's last copy; then two
 * counts: [6] the producer's and [7] the first consumer's mbarrier polls.
 * *n_cta is the number of CTAs (one per SM).  Synchronises the stream. */
LALB_API int lalb_decoder_trace_step(lalb_decoder *dec, const float *h_in,
                                     unsigned long long *trace_host, int trace_len,
                                     int *n_cta, lalb_stream stream);
/* ---- tensor parallelism ------------------------------------------------
 * A decoder may hold one rank of n_rank (one process or thread per GPU) or
 * every rank at once on one GPU (rank = -1: the ranks run as groups of CTAs
 * of one launch; for tests and for GPUs short of peers).  Rank r holds rows
 * lalb_tp_rows(cfg, n_rank, r, matrix) of every matrix: 0 qkv and 1 o in
 * full (every rank computes q and the residual update itself), 2 gate/up
 * (whole 64-row gate/up tiles), 3 down and 4 LM head split.  Each rank's
 * CTAs write their gate/up and down output rows into every rank's exchange
 * buffer over NVLink and wait on every rank's phase counters after those
 * phases (two cross-GPU exchanges per layer); the argmax is the first
 * maximum over all ranks' rows.  Steps run on the persistent path only. */
#define LALB_IPC_HANDLE_BYTES 64
LALB_API int lalb_tp_rows(const lalb_decoder_cfg *cfg, int n_rank, int rank, int matrix,
                          int *row0, int *row1);
LALB_API int lalb_decoder_create_tp(lalb_ctx *ctx, const lalb_decoder_cfg *cfg, int n_rank,
                                    int rank, lalb_decoder **out);
/* w: the rank's row shard of each matrix (rows lalb_tp_rows(...), Q4_K). */
LALB_API int lalb_decoder_set_layer_shard(lalb_decoder *dec, int rank, int layer,
                                          const lalb_layer_weights *w);
LALB_API int lalb_decoder_set_lm_head_shard(lalb_decoder *dec, int rank, const int8_t *w,
                                            const float *sw);
/* One rank per decoder: export this rank's exchange buffer (handle:
 * LALB_IPC_HANDLE_BYTES bytes), gather every rank's handle (rank order) by
 * any host means, then map the peers' buffers.  Every rank must connect
 * before the first step. */
LALB_API int lalb_decoder_ipc_handle(lalb_decoder *dec, void *handle);
LALB_API int lalb_decoder_connect(lalb_decoder *dec, const void *handles);
/* The same connection when every rank lives in one process (one host thread
 * per GPU, peer access enabled between the GPUs by the caller with
 * cudaDeviceEnablePeerAccess; or several ranks' decoders on one GPU, whose
 * steps must then never run at the same time): exchange_buffer gives this
 * rank's buffer (device address, 128-byte aligned), connect_local takes
 * every rank's, in rank order. */
LALB_API int lalb_decoder_exchange_buffer(lalb_decoder *dec, void **buf);
LALB_API int lalb_decoder_connect_local(lalb_decoder *dec, void *const *bufs);
/* Bound on every grid-wide and cross-GPU wait of the persistent kernel, in
 * seconds (default 10; accepted range [1e-4, 600]).  A wait that expires
 * raises the context's status word (lalb_device_status returns
 * LALB_STATUS_WAIT_TIMEOUT = 1), the rest of the token runs on whatever
 * data it has, and its argmax is -1.  Waits for the kernel's own copies are
 * bounded by four times this limit. */
LALB_API int lalb_decoder_set_wait_limit(lalb_decoder *dec, double seconds);
/* After a failed step: clears this rank's exchange buffer (phase counters,
 * token count, argmax keys).  Every rank resets, with a host barrier between
 * the ranks before (no step in flight anywhere) and after (no rank steps
 * before all have reset); then reset the context's status word with
 * lalb_device_status(ctx, 1). */
LALB_API int lalb_decoder_reset(lalb_decoder *dec, lalb_stream stream);

/* Execution path of lalb_decoder_step.  AUTO takes the persistent path
 * (the whole token in one cooperative kernel, one CTA per SM) when the
 * shapes fit it -- hidden <= 4096, q_rows <= 4096, ffn <= 20480, at most
 * 8 gate/up tiles of 64 rows per SM -- and the per-phase kernel chain
 * otherwise.  PERSISTENT fails with LALB_ERR_UNSUPPORTED when the shapes
 * do not fit. */
enum {
    LALB_DECODE_AUTO = 0,
    LALB_DECODE_KERNELS = 1,
    LALB_DECODE_PERSISTENT = 2
};
LALB_API int lalb_decoder_set_path(lalb_decoder *dec, int path);
/* The path lalb_decoder_step takes: LALB_DECODE_KERNELS or
 * LALB_DECODE_PERSISTENT. */
LALB_API int lalb_decoder_path(const lalb_decoder *dec);
/* Number of kernels one step launches. */
LALB_API int lalb_decoder_launches_per_step(const lalb_decoder *dec);
LALB_API int lalb_decoder_destroy(lalb_decoder *dec);

/* ---- prefill: the Q4_K x Q8 matmul for T tokens at once (tcgen05) --------
 * Y [T][rows] fp32 = lal_matmul_q4_k (README.md:130,210) applied to each of
 * the T rows of X [T][K] fp32, with the same per-32 activation quantizer,
 * straight from the Q4_K rows W (as for lalb_matmul_q4_k; 16-byte aligned).
 * On the tensor cores (tcgen05.mma kind::f16, fp32 accumulators in TMEM):
 * each row's 4-bit quants are decoded on chip into A = sc*q as fp16
 * (exact), B = xq*sx per token as two fp16 parts under a per-token power of
 * two, the min terms as bf16 parts; each 256-weight super-block is scaled
 * by d in the epilogue.  Every output is within 1e-5 of the exact value
 * relative to the sum of its term magnitudes.  `ws` (ws_bytes from
 * lalb_prefill_ws_bytes, 256-byte aligned) holds the prepared tokens and,
 * for calls with fewer 128 x 128 output tiles than SMs, the partial sums of
 * a split of K over several CTAs per tile (added in a fixed order: the
 * result does not depend on which CTA finishes last).  K % 256 == 0. */
LALB_API int lalb_prefill_ws_bytes(int rows, int K, int T, size_t *ws_bytes);
LALB_API int lalb_matmul_q4_k_prefill(lalb_ctx *ctx, const void *W, int rows, int K,
                                      const float *X, int T, void *ws, float *Y,
                                      lalb_stream stream);

/* Measured tensor-core throughput: back-to-back tcgen05.mma (M = 128,
 * N = 256) from shared memory on every SM for a few milliseconds; *tera_ops =
 * 2 M N K per instruction over the time, in units of 10^12 (TFLOP/s for
 * kind::f16, TOPS for kind::i8).  The dense peak at the clock the GPU holds
 * under that load: the denominator of the prefill kernel's tensor fractions. */
enum { LALB_MMA_F16 = 0, LALB_MMA_I8 = 1 };
LALB_API int lalb_measure_mma_peak(lalb_ctx *ctx, int kind, double *tera_ops);

/* ---- weight blobs: one file of named tensors, written and loaded here ----
 * The reference ships its 7B weights pre-converted in one file
 * (prebuilt/qwen7b_q4k_weights.bin from scripts/convert_qwen7b_q4k.py,
 * README.md:18-20,154; neither is in its snapshot) and loads fp32 tensor
 * files with tensor_load_all (runtime/lal_runtime.c:2798-2822).  This blob
 * format is our own, version 1: a 64-byte header ("LQ4K", version,
 * count, alignment 4096, table offset and size, file size), each tensor's
 * bytes on a 4096-byte boundary, and a table of 128-byte entries at the end
 * (key of at most 71 bytes, dtype, up to 3 dims, offset, size, FNV-1a-64
 * checksum).  A 2-D tensor is row-major, so a row range is one byte range.
 * Every call returns LALB_ERR_INVALID on a malformed file or argument. */
enum {
    LALB_DT_F32 = 0,
    LALB_DT_Q4K = 1,   /* dims [rows, K], K % 256 == 0: rows * K/256 * 144 bytes */
    LALB_DT_I8 = 2,
    LALB_DT_F16 = 3,
    LALB_DT_BF16 = 4
};
typedef struct {
    char key[72];
    int dtype;
    int ndim;
    uint64_t dims[3];
    uint64_t bytes;      /* whole tensor */
    uint64_t row_bytes;  /* bytes / dims[0] */
} lalb_blob_tensor;

typedef struct lalb_blob_writer lalb_blob_writer;
LALB_API int lalb_blob_writer_open(const char *path, lalb_blob_writer **out);
/* Host bytes of a tensor as they are (the key must be new). */
LALB_API int lalb_blob_writer_add(lalb_blob_writer *w, const char *key, int dtype, int ndim,
                                  const uint64_t *dims, const void *data);
/* The converter: host weights [rows][K] in src_dtype (LALB_DT_F32 or
 * LALB_DT_BF16) quantized on ctx's GPU by lalb_q4k_quantize (dtype
 * LALB_DT_Q4K) or lalb_q8_quantize_rows (dtype LALB_DT_I8: the int8 rows
 * under key, their fp32 scales under scale_key), then written. */
LALB_API int lalb_blob_writer_add_quantized(lalb_ctx *ctx, lalb_blob_writer *w, const char *key,
                                            const char *scale_key, int dtype, int src_dtype,
                                            const void *host, int rows, int K);
/* Writes the header and table; the file is complete only after this. */
LALB_API int lalb_blob_writer_close(lalb_blob_writer *w);

typedef struct lalb_blob lalb_blob;
LALB_API int lalb_blob_open(const char *path, lalb_blob **out);
LALB_API int lalb_blob_close(lalb_blob *b);
LALB_API int lalb_blob_count(const lalb_blob *b);
/* Index of the tensor named key, or LALB_ERR_INVALID. */
LALB_API int lalb_blob_find(const lalb_blob *b, const char *key);
LALB_API int lalb_blob_info(const lalb_blob *b, int index, lalb_blob_tensor *info);
/* Recomputes the tensor's checksum from the file: LALB_OK if it matches. */
LALB_API int lalb_blob_verify(const lalb_blob *b, int index);
/* Rows [row0, row1) of tensor `index` into host memory. */
LALB_API int lalb_blob_read_host(const lalb_blob *b, int index, uint64_t row0, uint64_t row1,
                                 void *dst);
/* Rows [row0, row1) of tensor `index` into caller-owned device memory dst
 * (a tensor-parallel rank loads its shard), through two 32 MB pinned
 * staging buffers that the blob allocates on its first load (one device per
 * blob): the file read of one chunk overlaps the copy of the previous one on
 * `stream`.  Returns when the last copy has finished. */
LALB_API int lalb_blob_load(lalb_ctx *ctx, lalb_blob *b, int index, uint64_t row0, uint64_t row1,
                            void *dst, lalb_stream stream);

/* ---- the seed STE model's forward matmuls (tensor cores) -----------------
 * A BinLayer (runtime/lal_runtime.h:171-197) with one CORE (0) / BINARY (1)
 * / PRUNE (2) state per output row.  Built like bin_layer_init_logic
 * (runtime/lal_runtime.c:1567-1676) from W [out][in] fp32 (row-major),
 * bias [out] (nullable) and mask [out], all device buffers; alpha_repack = 1
 * recomputes alpha as bin_layer_repack (:1703-1766) does.  max_rows bounds
 * the M of a forward (the layer owns its per-row scale buffer).
 * in_dim % 32 == 0. */
typedef struct lalb_binlayer lalb_binlayer;
LALB_API int lalb_binlayer_create(lalb_ctx *ctx, const float *W, const float *bias,
                                  const uint8_t *mask, int in_dim, int out_dim,
                                  int alpha_repack, float binary_scale, int max_rows,
                                  lalb_binlayer **out);
/* Y [M][out] = the layer over the M rows of X [M][in]: mode 0 bin_forward
 * (:1852-1938, logic-mask path), mode 1 bin_forward_pure_float (:543-582).
 * fp32 operands as sums of tf32 parts on tcgen05 (X is read once, its parts
 * formed on chip); within 1e-5 of the exact products.  X 16-byte
 * aligned (LALB_ERR_INVALID otherwise). */
LALB_API int lalb_binlayer_forward(lalb_binlayer *bl, const float *X, int M, float *Y,
                                   int mode, lalb_stream stream);
LALB_API int lalb_binlayer_alpha(lalb_binlayer *bl, float *alpha, lalb_stream stream);
LALB_API int lalb_binlayer_destroy(lalb_binlayer *bl);

/* Per-element states (state [rows][K]: 0 CORE, 1 BINARY, 2 PRUNE) packed as
 * int8 codes with one fp32 scale per row: CORE weights quantized to +-127,
 * BINARY weights +-(row's mean |w| in the same scale), PRUNE 0. */
LALB_API int lalb_logic_pack(lalb_ctx *ctx, const float *W, const uint8_t *state, int rows,
                             int K, int8_t *codes, float *srow, lalb_stream stream);
/* Y [M][rows] = srow * (X . codes^T) + bias; bias nullable.  The layer reads
 * codes, srow and bias in place (keep them alive while it exists): the codes
 * stay 1 byte per weight and are decoded on chip into exact fp16 for the
 * tcgen05 tensor cores, X goes in as two fp16 parts under a per-row power of
 * two (22 bits); within 1e-5 of the exact products.  codes and X 16-byte
 * aligned, K % 32 == 0, M <= max_rows. */
typedef struct lalb_logic_layer lalb_logic_layer;
LALB_API int lalb_logic_layer_create(lalb_ctx *ctx, const int8_t *codes, const float *srow,
                                     const float *bias, int rows, int K, int max_rows,
                                     lalb_logic_layer **out);
LALB_API int lalb_logic_layer_forward(lalb_logic_layer *L, const float *X, int M, float *Y,
                                      lalb_stream stream);
LALB_API int lalb_logic_layer_destroy(lalb_logic_layer *L);

#ifdef __cplusplus
}
#endif
#endif /* LALB_H */
