/*
 * lalb_oracle.h -- CPU restatement of LAL's quantized-matmul hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker: the pytest suite,
 * the smoke check and the CPU-baseline leg of the benchmark call it to produce
 * the expected answer or the CPU timing.  The product (liblalb.so, the sm_100a
 * kernels) never links or calls it.
 *
 * What it restates (the reference's kernel headers runtime/lal_q4k_kernel.h and
 * runtime/lal_q8_kernel.h are listed in the reference README.md:130-131 but are
 * absent from the reference snapshot):
 *   - the llama.cpp-compatible Q4_K super-block format (README.md:28, 284):
 *     144 bytes per 256 weights = fp16 d | fp16 dmin | 12 bytes of packed 6-bit
 *     scales/mins | 128 bytes of 4-bit quants, w = d*sc_j*q - dmin*m_j;
 *   - unpack_scales_6bit (README.md:212): 12 packed bytes -> 8 scales + 8 mins;
 *   - the "simple min-max" Q4_K weight quantizer (README.md:48, 154);
 *   - the per-32-block fp32 -> int8 activation quantizer (fp32 scale);
 *   - lal_matmul_q4_k (README.md:130, 210): Q4_K x Q8 dot, int32 per 32-wide
 *     sub-block, fp32 combine;
 *   - lal_lm_head_int8_range (README.md:131, 211, 285): int8 x int8 LM head
 *     over a row range (the "sign trick" |w|*sign(w)x is an identity for
 *     w != -128, which the quantizer never produces), plus first-max argmax
 *     (models/ste_train.c:1503-1509, sample_argmax);
 *   - the seed STE model's per-element CORE/BINARY/PRUNE int8 forward.
 *
 * Parity status: the Q4_K byte layout and dequantization are pinned against
 * gguf 0.19.0 (llama.cpp's Python package, gguf/quants.py Q4_K); the int8
 * activation quantizer is pinned against gguf's Q8_0 quantize_blocks.  The
 * Q4_K min-max weight quantizer itself has no third-party twin (the
 * reference's converter scripts/convert_qwen7b_q4k.py is absent).
 *
 * Quantizers use IEEE single precision with no contraction (-ffp-contract=
 * off); the matvec and LM-head outputs are the fp32 roundings of their exact
 * real values (integer sums exact, products and sums in binary128).
 */
#ifndef LALB_ORACLE_H
#define LALB_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LALB_O_QK 256          /* weights per Q4_K super-block */
#define LALB_O_QB 32           /* weights per sub-block / activation block */
#define LALB_O_Q4K_BYTES 144   /* bytes per Q4_K super-block */

/* --- seeded synthetic data ------------------------------------------------ */
/* Counter-based normal generator: element i of stream `seed` is
 *   u = mix64(seed * 0xD1B54A32D192ED03 + i), u1 = ((u>>40)+1)/2^24,
 *   u2 = ((u>>16)&0xFFFFFF)/2^24, z = sqrt(-2 ln u1) cos(2 pi u2)  (double),
 * out[k] = (float)(sigma * z) for i = offset + k.  mix64 is the SplitMix64
 * finalizer (Steele, Lea, Flood 2014). */
uint64_t lalb_o_mix64(uint64_t z);
void lalb_o_fill_normal(float *out, size_t n, uint64_t seed, uint64_t offset,
                        float sigma);

/* --- fp16 ---------------------------------------------------------------- */
uint16_t lalb_o_f32_to_f16(float f);   /* round to nearest even */
float    lalb_o_f16_to_f32(uint16_t h);

/* --- Q4_K format --------------------------------------------------------- */
void lalb_o_unpack_scales_6bit(const uint8_t scales12[12], uint8_t out16[16]);
void lalb_o_q4k_quantize(const float *w, int rows, int K, uint8_t *blocks);
void lalb_o_q4k_dequantize(const uint8_t *blocks, int rows, int K, float *w);

/* --- activation quantizer: per 32-block amax/127, roundf, clamp +-127 ----- */
void lalb_o_quantize_act(const float *x, int M, int K, int8_t *xq, float *sx,
                         int32_t *sumq);

/* --- Q4_K x Q8 matvec / matmul -------------------------------------------
 * y[m*rows + r] = the fp32 rounding of the exact real value
 *     sum over sub-blocks s of  sx[m][s] * (d*sc_s*isum_s - dmin*m_s*sumq[m][s])
 * (computed exactly in binary128, rounded once).  isum (nullable) receives
 * the exact int32 sub-block dot products, laid out [m][r][K/32]. */
void lalb_o_q4k_matmul(const uint8_t *W, int rows, int K, const int8_t *xq,
                       const float *sx, const int32_t *sumq, int M, float *y,
                       int32_t *isum);

/* --- Q8 (int8 per-row-scaled) LM head ----------------------------------- */
void lalb_o_q8_quantize_rows(const float *w, int rows, int K, int8_t *q,
                             float *s);
/* logits[r - r0] = fp32 rounding of the exact sw[r] * sum_b sx[b]*isum_b for r
 * in [r0, r1); isum (nullable) gets [r1-r0][K/32] int32 block dots.  Returns
 * the first index (absolute row number) of the maximum logit. */
int lalb_o_q8_lmhead_range(const int8_t *W, const float *sw, int K, int r0,
                           int r1, const int8_t *xq, const float *sx,
                           float *logits, int32_t *isum);
int lalb_o_argmax(const float *v, int n);

/* --- decode chain used by the Qwen-shape matmul set ----------------------- */
/* act[i] = (float)(g / (1 + exp(-g)) * up[i]) evaluated in double. */
void lalb_o_swiglu(const float *gate, const float *up, int n, float *act);

/* RMSNorm, after rms_norm (runtime/lal_runtime.c:82-87):
 *   s = (float)(1 / sqrt(sum x^2 / n + eps)), the sum and root in double;
 *   out[i] = (x[i] * s) * w[i], each product one IEEE float rounding.
 * w may be NULL (unit weights: out[i] = x[i] * s).  The reference sums the
 * squares in float; here the sum is in double, so s is the float rounding
 * of the (nearly) exact value and does not depend on summation order. */
void lalb_o_rms_norm(const float *x, const float *w, int n, float eps, float *out);

/* One decode step of causal attention for one layer, after apply_rope
 * (runtime/lal_runtime.c:137-153) and attention_forward (:833-882),
 * generalised to grouped KV heads.  qkv = q [n_head*hd] | k [n_kv*hd] |
 * v [n_kv*hd]; the caches are [max_ctx][n_kv*hd].
 *   RoPE at position pos on every q and k head, pairs (d, d + hd/2):
 *     a = pos * theta^(-2d/hd); (x0, x1) -> (x0 c - x1 s, x0 s + x1 c),
 *     in double, each result rounded to float once;
 *   k_cache[pos] = rotated k, v_cache[pos] = v;
 *   head h reads KV head g = h / (n_head / n_kv): for j = 0..pos
 *     s_j = (q_h . k_j) / sqrt(hd), w_j = exp(s_j - max s) / (sum + 1e-12),
 *     out_h = sum_j w_j v_j, everything in double, rounded to float once.
 * The reference computes the angle, cos/sin and sums in float. */
void lalb_o_attention_decode(const float *qkv, int n_head, int n_kv, int hd, int pos,
                             float theta, float *k_cache, float *v_cache, float *out);

/* Next-token sampling after the LM head, after generate_text
 * (models/ste_train.c:2229-2318) and sample_argmax (:1503-1509):
 *   adjusted = logits; ids < n_mask -> -1e30;
 *   every distinct token of history (once): adjusted /= rep if > 0, else *= rep;
 *   ngram >= 2: every token t such that history[-(ngram-1):] + [t] already
 *   occurs in history -> -1e30 (the reference: ngram = 3);
 *   temp <= 0.01: the first maximum (sample_argmax);
 *   else the top_k largest (value descending; ties: tie_rule 0 = lower index
 *   first, 1 = the reference's selection sort, :2286-2297), p_j =
 *   (float)exp((double)((a_j - a_0) / temp)) (float subtraction and
 *   division, the exponential rounded once), cumulative float sums: the
 *   nucleus ends at the first j whose running sum exceeds top_p * sum;
 *   r = u * (that running sum); the token is the first j of the nucleus with
 *   r < running sum (index 0 if none).
 * idx/prob (nullable, top_k entries) receive the ranked ids and p_j.
 * Returns the token. */
int lalb_o_sample(const float *logits, int vocab, const int32_t *history, int n_hist,
                  float temp, int top_k, float top_p, float rep, int ngram, int n_mask,
                  float u, int tie_rule, int32_t *idx, float *prob);

/* --- seed STE model, per-element CORE/BINARY/PRUNE int8 encoding --------- */
/* state[i] (0 CORE, 1 BINARY, 2 PRUNE) and w[i] (fp32) per weight, W [rows][K].
 * Per row j:  amax = max |w| over CORE entries, alpha = mean |w| over BINARY
 * entries, s_j = max(amax, alpha) / 127 (0 if both are 0);
 *   CORE   code = clamp(roundf(w / s_j), -127, 127)
 *   BINARY code = (w > 0 ? 1 : -1) * clamp(roundf(alpha / s_j), 1, 127)
 *   PRUNE  code = 0.
 * Forward (fp32 X [M][K]):  Y[m][j] = s_j * (float)(sum_i code*X) + bias[j],
 * the sum taken in double. */
void lalb_o_logic_state(uint64_t seed, size_t n, float p_core, float p_binary,
                        uint8_t *state);
void lalb_o_logic_pack(const float *w, const uint8_t *state, int rows, int K,
                       int8_t *codes, float *srow);
void lalb_o_logic_forward(const int8_t *codes, const float *srow,
                          const float *bias, int rows, int K, const float *X,
                          int M, float *Y);

/* The reference's logic-masked BinLayer over M input rows, computed in
 * double and rounded once per output: mode 0 bin_forward
 * (runtime/lal_runtime.c:1852-1938), mode 1 bin_forward_pure_float
 * (:543-582); alpha as bin_layer_init_logic (:1567-1676) leaves it, or, with
 * repack, as bin_layer_repack (:1703-1766) recomputes it.  W [out][in],
 * bias [out] (nullable), mask [out], X [M][in] -> Y [M][out]; alpha_out
 * [out] nullable. */
void lalb_o_binlayer_forward(const float *W, const float *bias,
                             const uint8_t *mask, int in_dim, int out_dim,
                             const float *X, int M, float *Y, int mode,
                             int repack, float binary_scale, float *alpha_out);

/* --- AVX2 + OpenMP CPU baseline (same integer results as the scalar code) - */
int  lalb_cpu_threads(void);
void lalb_cpu_set_threads(int n);
void lalb_cpu_quantize_act(const float *x, int M, int K, int8_t *xq, float *sx,
                           int32_t *sumq);
void lalb_cpu_q4k_gemv(const uint8_t *W, int rows, int K, const int8_t *xq,
                       const float *sx, const int32_t *sumq, float *y);
int  lalb_cpu_q8_lmhead(const int8_t *W, const float *sw, int rows, int K,
                        const int8_t *xq, const float *sx, float *logits);

#ifdef __cplusplus
}
#endif
#endif
