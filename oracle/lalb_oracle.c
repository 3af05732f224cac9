/*
 * lalb_oracle.c -- scalar C restatement of the quantized-matmul hot path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker).  Built with -ffp-contract=off so
 * every float operation below is one IEEE-rounded single-precision op.
 * Reference anchors (paths inside the reference project):
 *   README.md:28,284      Q4_K format, llama.cpp-compatible
 *   README.md:48,154      min-max quantization, no importance matrix
 *   README.md:130,210     lal_matmul_q4_k
 *   README.md:131,211,285 lal_lm_head_int8_range, sign trick
 *   README.md:212         unpack_scales_6bit (12 bytes -> 16 u8)
 *   models/ste_train.c:1503-1509  sample_argmax (first maximum wins)
 */
#include "lalb_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* seeded data                                                               */
/* ------------------------------------------------------------------------ */
uint64_t lalb_o_mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

void lalb_o_fill_normal(float *out, size_t n, uint64_t seed, uint64_t offset,
                        float sigma) {
    const uint64_t base = seed * 0xD1B54A32D192ED03ull;
    const double two_pi = 6.283185307179586476925286766559;
#pragma omp parallel for schedule(static)
    for (long long k = 0; k < (long long)n; k++) {
        uint64_t u = lalb_o_mix64(base + offset + (uint64_t)k);
        double u1 = (double)((u >> 40) + 1) * (1.0 / 16777216.0);
        double u2 = (double)((u >> 16) & 0xFFFFFFu) * (1.0 / 16777216.0);
        double z = sqrt(-2.0 * log(u1)) * cos(two_pi * u2);
        out[k] = (float)((double)sigma * z);
    }
}

/* ------------------------------------------------------------------------ */
/* fp16 <-> fp32 (IEEE binary16, round to nearest even)                      */
/* ------------------------------------------------------------------------ */
uint16_t lalb_o_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u)                      /* inf / nan */
        return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0));
    if (ax >= 0x477FF000u)                      /* rounds to >= 65520: inf */
        return (uint16_t)(sign | 0x7C00u);
    if (ax < 0x38800000u) {                     /* result is subnormal or 0 */
        if (ax < 0x33000000u) return (uint16_t)sign;   /* < 2^-25: to 0 */
        uint32_t mant = (ax & 0x7FFFFFu) | 0x800000u;
        int e = (int)(ax >> 23);                /* 102..112 */
        int shift = 126 - e;                    /* so that value = mant>>shift */
        uint32_t q = mant >> shift;
        uint32_t rem = mant & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t e = (ax >> 23) - 112u;             /* rebias 127 -> 15 */
    uint32_t mant = ax & 0x7FFFFFu;
    uint32_t h = (e << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;  /* may carry */
    return (uint16_t)(sign | h);
}

float lalb_o_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu;
    uint32_t m = h & 0x3FFu;
    uint32_t x;
    if (e == 0) {
        if (m == 0) {
            x = sign;
        } else {                                /* normalise a subnormal */
            int sh = 0;
            while (!(m & 0x400u)) { m <<= 1; sh++; }
            m &= 0x3FFu;
            x = sign | ((uint32_t)(113 - sh) << 23) | (m << 13);
        }
    } else if (e == 31) {
        x = sign | 0x7F800000u | (m << 13);
    } else {
        x = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

/* ------------------------------------------------------------------------ */
/* Q4_K format                                                               */
/* ------------------------------------------------------------------------ */
/* Byte j of the 12 packed bytes: j=0..3 low 6 bits = scale j, top 2 bits =
 * bits 4-5 of scale j+4;  j=4..7 low 6 bits = min j-4, top 2 bits = bits 4-5
 * of min j;  j=8..11 low nibble = bits 0-3 of scale j-4, high nibble = bits
 * 0-3 of min j-4.  out16[0..7] = scales, out16[8..15] = mins. */
void lalb_o_unpack_scales_6bit(const uint8_t s[12], uint8_t out[16]) {
    for (int j = 0; j < 4; j++) {
        out[j] = s[j] & 63;
        out[8 + j] = s[j + 4] & 63;
    }
    for (int j = 4; j < 8; j++) {
        out[j] = (uint8_t)((s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4));
        out[8 + j] = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
    }
}

static void pack_scales_6bit(const uint8_t sc[8], const uint8_t mn[8],
                             uint8_t s[12]) {
    memset(s, 0, 12);
    for (int j = 0; j < 4; j++) {
        s[j] = sc[j];
        s[j + 4] = mn[j];
    }
    for (int j = 4; j < 8; j++) {
        s[j + 4] = (uint8_t)((sc[j] & 0x0F) | ((mn[j] & 0x0F) << 4));
        s[j - 4] |= (uint8_t)((sc[j] >> 4) << 6);
        s[j] |= (uint8_t)((mn[j] >> 4) << 6);
    }
}

/* Min-max quantization of one 256-weight super-block:
 *   per 32 sub-block: mn = min(0, min x), mx = max x,
 *                     scale = (mx - mn) / 15, minv = -mn;
 *   d = max scale / 63, dmin = max minv / 63 (stored fp16);
 *   sc = min(63, rint(63/max_scale * scale)), m likewise (0 if max is 0);
 *   q = clamp(rint((x + fp16(dmin)*m) / (fp16(d)*sc)), 0, 15)  (0 if d*sc==0).
 * rint is round-half-even; the maxima start from +0. */
static void q4k_quantize_block(const float *x, uint8_t *blk) {
    float scale[8], minv[8];
    float max_scale = 0.0f, max_min = 0.0f;
    for (int j = 0; j < 8; j++) {
        const float *v = x + 32 * j;
        float mn = v[0], mx = v[0];
        for (int i = 1; i < 32; i++) {
            if (v[i] < mn) mn = v[i];
            if (v[i] > mx) mx = v[i];
        }
        if (mn > 0.0f) mn = 0.0f;
        scale[j] = (mx - mn) / 15.0f;
        minv[j] = -mn;
        if (scale[j] > max_scale) max_scale = scale[j];
        if (minv[j] > max_min) max_min = minv[j];
    }
    float inv_scale = max_scale > 0.0f ? 63.0f / max_scale : 0.0f;
    float inv_min = max_min > 0.0f ? 63.0f / max_min : 0.0f;
    uint8_t ls[8], lm[8];
    for (int j = 0; j < 8; j++) {
        float a = rintf(inv_scale * scale[j]);
        float b = rintf(inv_min * minv[j]);
        ls[j] = (uint8_t)(a > 63.0f ? 63 : (int)a);
        lm[j] = (uint8_t)(b > 63.0f ? 63 : (int)b);
    }
    uint16_t dh = lalb_o_f32_to_f16(max_scale / 63.0f);
    uint16_t mh = lalb_o_f32_to_f16(max_min / 63.0f);
    blk[0] = (uint8_t)(dh & 0xFF);
    blk[1] = (uint8_t)(dh >> 8);
    blk[2] = (uint8_t)(mh & 0xFF);
    blk[3] = (uint8_t)(mh >> 8);
    pack_scales_6bit(ls, lm, blk + 4);
    float d = lalb_o_f16_to_f32(dh), dmin = lalb_o_f16_to_f32(mh);
    uint8_t L[256];
    for (int j = 0; j < 8; j++) {
        float dj = d * (float)ls[j];
        float dmj = dmin * (float)lm[j];
        for (int i = 0; i < 32; i++) {
            int l = 0;
            if (dj != 0.0f) {
                float t = rintf((x[32 * j + i] + dmj) / dj);
                l = t < 0.0f ? 0 : (t > 15.0f ? 15 : (int)t);
            }
            L[32 * j + i] = (uint8_t)l;
        }
    }
    uint8_t *qs = blk + 16;
    for (int g = 0; g < 4; g++)
        for (int i = 0; i < 32; i++)
            qs[32 * g + i] = (uint8_t)(L[64 * g + i] | (L[64 * g + 32 + i] << 4));
}

void lalb_o_q4k_quantize(const float *w, int rows, int K, uint8_t *blocks) {
    const int nb = K / LALB_O_QK;
#pragma omp parallel for schedule(static)
    for (long long t = 0; t < (long long)rows * nb; t++)
        q4k_quantize_block(w + (size_t)t * LALB_O_QK,
                           blocks + (size_t)t * LALB_O_Q4K_BYTES);
}

void lalb_o_q4k_dequantize(const uint8_t *blocks, int rows, int K, float *w) {
    const int nb = K / LALB_O_QK;
    for (long long t = 0; t < (long long)rows * nb; t++) {
        const uint8_t *blk = blocks + (size_t)t * LALB_O_Q4K_BYTES;
        float d = lalb_o_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
        float dmin = lalb_o_f16_to_f32((uint16_t)(blk[2] | (blk[3] << 8)));
        uint8_t sm[16];
        lalb_o_unpack_scales_6bit(blk + 4, sm);
        const uint8_t *qs = blk + 16;
        float *o = w + (size_t)t * LALB_O_QK;
        for (int j = 0; j < 8; j++) {
            float dj = d * (float)sm[j];
            float mj = dmin * (float)sm[8 + j];
            for (int i = 0; i < 32; i++) {
                uint8_t byte = qs[32 * (j >> 1) + i];
                int q = (j & 1) ? (byte >> 4) : (byte & 0x0F);
                o[32 * j + i] = dj * (float)q - mj;
            }
        }
    }
}

/* ------------------------------------------------------------------------ */
/* activation quantizer                                                      */
/* ------------------------------------------------------------------------ */
void lalb_o_quantize_act(const float *x, int M, int K, int8_t *xq, float *sx,
                         int32_t *sumq) {
    const int nblk = K / LALB_O_QB;
    for (long long b = 0; b < (long long)M * nblk; b++) {
        const float *v = x + (size_t)b * LALB_O_QB;
        float amax = 0.0f;
        for (int i = 0; i < 32; i++) {
            float a = fabsf(v[i]);
            if (a > amax) amax = a;
        }
        float d = amax / 127.0f;
        float id = d != 0.0f ? 1.0f / d : 0.0f;
        int s = 0;
        for (int i = 0; i < 32; i++) {
            float r = roundf(v[i] * id);
            int q = r > 127.0f ? 127 : (r < -127.0f ? -127 : (int)r);
            xq[(size_t)b * 32 + i] = (int8_t)q;
            s += q;
        }
        sx[b] = d;
        if (sumq) sumq[b] = s;
    }
}

/* ------------------------------------------------------------------------ */
/* Q4_K x Q8                                                                 */
/* ------------------------------------------------------------------------ */
void lalb_o_q4k_matmul(const uint8_t *W, int rows, int K, const int8_t *xq,
                       const float *sx, const int32_t *sumq, int M, float *y,
                       int32_t *isum) {
    const int nb = K / LALB_O_QK, ns = K / LALB_O_QB;
#pragma omp parallel for schedule(static) collapse(2)
    for (int m = 0; m < M; m++) {
        for (int r = 0; r < rows; r++) {
            const int8_t *xm = xq + (size_t)m * K;
            const float *sxm = sx + (size_t)m * ns;
            const int32_t *sqm = sumq + (size_t)m * ns;
            /* every product below is exact in binary128 (at most 24 + 11 + 22
             * significant bits); the sum is rounded once, to fp32, at the end */
            __float128 acc = 0;
            for (int b = 0; b < nb; b++) {
                const uint8_t *blk = W + ((size_t)r * nb + b) * LALB_O_Q4K_BYTES;
                float d = lalb_o_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
                float dmin = lalb_o_f16_to_f32((uint16_t)(blk[2] | (blk[3] << 8)));
                uint8_t sm[16];
                lalb_o_unpack_scales_6bit(blk + 4, sm);
                const uint8_t *qs = blk + 16;
                for (int j = 0; j < 8; j++) {
                    const int8_t *xv = xm + 256 * b + 32 * j;
                    int32_t s = 0;
                    for (int i = 0; i < 32; i++) {
                        uint8_t byte = qs[32 * (j >> 1) + i];
                        int q = (j & 1) ? (byte >> 4) : (byte & 0x0F);
                        s += q * (int32_t)xv[i];
                    }
                    int sidx = 8 * b + j;
                    if (isum) isum[((size_t)m * rows + r) * ns + sidx] = s;
                    __float128 a = (__float128)d * (__float128)(sm[j] * s);
                    __float128 c = (__float128)dmin * (__float128)(sm[8 + j] * sqm[sidx]);
                    acc += (__float128)sxm[sidx] * (a - c);
                }
            }
            y[(size_t)m * rows + r] = (float)acc;
        }
    }
}

/* ------------------------------------------------------------------------ */
/* Q8 LM head                                                                */
/* ------------------------------------------------------------------------ */
void lalb_o_q8_quantize_rows(const float *w, int rows, int K, int8_t *q,
                             float *s) {
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; r++) {
        const float *v = w + (size_t)r * K;
        float amax = 0.0f;
        for (int i = 0; i < K; i++) {
            float a = fabsf(v[i]);
            if (a > amax) amax = a;
        }
        float d = amax / 127.0f;
        float id = d != 0.0f ? 1.0f / d : 0.0f;
        for (int i = 0; i < K; i++) {
            float t = roundf(v[i] * id);
            q[(size_t)r * K + i] =
                (int8_t)(t > 127.0f ? 127 : (t < -127.0f ? -127 : (int)t));
        }
        s[r] = d;
    }
}

int lalb_o_argmax(const float *v, int n) {
    int best = 0;
    for (int i = 1; i < n; i++)
        if (v[i] > v[best]) best = i;
    return best;
}

int lalb_o_q8_lmhead_range(const int8_t *W, const float *sw, int K, int r0,
                           int r1, const int8_t *xq, const float *sx,
                           float *logits, int32_t *isum) {
    const int nblk = K / LALB_O_QB;
#pragma omp parallel for schedule(static)
    for (int r = r0; r < r1; r++) {
        const int8_t *wr = W + (size_t)r * K;
        __float128 acc = 0;   /* exact: sx * isum has at most 24 + 20 bits */
        for (int b = 0; b < nblk; b++) {
            int32_t s = 0;
            for (int i = 0; i < 32; i++)
                s += (int32_t)wr[32 * b + i] * (int32_t)xq[32 * b + i];
            if (isum) isum[(size_t)(r - r0) * nblk + b] = s;
            acc += (__float128)sx[b] * (__float128)s;
        }
        logits[r - r0] = (float)((__float128)sw[r] * acc);
    }
    return r1 > r0 ? r0 + lalb_o_argmax(logits, r1 - r0) : -1;
}

void lalb_o_swiglu(const float *gate, const float *up, int n, float *act) {
    for (int i = 0; i < n; i++) {
        double g = gate[i];
        act[i] = (float)(g / (1.0 + exp(-g)) * (double)up[i]);
    }
}

/* apply_rope (runtime/lal_runtime.c:137-153) on one head, in double */
static void rope_head(float *x, int hd, int pos, double theta) {
    const int half = hd / 2;
    for (int d = 0; d < half; d++) {
        const double a = (double)pos * pow(theta, -(double)(2 * d) / (double)hd);
        const double c = cos(a), s = sin(a);
        const double x0 = x[d], x1 = x[d + half];
        x[d] = (float)(x0 * c - x1 * s);
        x[d + half] = (float)(x0 * s + x1 * c);
    }
}

/* attention_forward (runtime/lal_runtime.c:833-882) with RoPE and grouped
 * KV heads; see lalb_oracle.h. */
void lalb_o_attention_decode(const float *qkv, int n_head, int n_kv, int hd, int pos,
                             float theta, float *k_cache, float *v_cache, float *out) {
    const int qr = n_head * hd, kvr = n_kv * hd, group = n_head / n_kv;
    float *q = (float *)malloc(sizeof(float) * (size_t)qr);
    double *sc = (double *)malloc(sizeof(double) * (size_t)(pos + 1));
    memcpy(q, qkv, sizeof(float) * (size_t)qr);
    for (int h = 0; h < n_head; h++) rope_head(q + (size_t)h * hd, hd, pos, theta);
    float *krow = k_cache + (size_t)pos * kvr, *vrow = v_cache + (size_t)pos * kvr;
    memcpy(krow, qkv + qr, sizeof(float) * (size_t)kvr);
    memcpy(vrow, qkv + qr + kvr, sizeof(float) * (size_t)kvr);
    for (int g = 0; g < n_kv; g++) rope_head(krow + (size_t)g * hd, hd, pos, theta);
    const double scale = 1.0 / sqrt((double)hd);
    for (int h = 0; h < n_head; h++) {
        const int g = h / group;
        const float *qh = q + (size_t)h * hd;
        double mx = -INFINITY;
        for (int j = 0; j <= pos; j++) {
            const float *kj = k_cache + (size_t)j * kvr + (size_t)g * hd;
            double dot = 0.0;
            for (int d = 0; d < hd; d++) dot += (double)qh[d] * (double)kj[d];
            sc[j] = dot * scale;
            if (sc[j] > mx) mx = sc[j];
        }
        double sum = 0.0;
        for (int j = 0; j <= pos; j++) {
            sc[j] = exp(sc[j] - mx);
            sum += sc[j];
        }
        const double inv = 1.0 / (sum + 1e-12);
        for (int d = 0; d < hd; d++) {
            double acc = 0.0;
            for (int j = 0; j <= pos; j++)
                acc += sc[j] * (double)v_cache[(size_t)j * kvr + (size_t)g * hd + d];
            out[(size_t)h * hd + d] = (float)(acc * inv);
        }
    }
    free(q);
    free(sc);
}

/* generate_text's sampling (models/ste_train.c:2229-2318); see lalb_oracle.h */
int lalb_o_sample(const float *logits, int vocab, const int32_t *history, int n_hist,
                  float temp, int top_k, float top_p, float rep, int ngram, int n_mask,
                  float u, int tie_rule, int32_t *idx_out, float *prob_out) {
    float *adj = (float *)malloc(sizeof(float) * (size_t)vocab);
    char *seen = (char *)calloc((size_t)vocab, 1);
    memcpy(adj, logits, sizeof(float) * (size_t)vocab);
    for (int i = 0; i < n_mask && i < vocab; i++) adj[i] = -1e30f;
    for (int j = 0; j < n_hist; j++) {               /* :2254-2264, once per token */
        const int t = history[j];
        if (t >= 0 && t < vocab && !seen[t]) {
            volatile float a = adj[t];
            adj[t] = a > 0 ? a / rep : a * rep;
            seen[t] = 1;
        }
    }
    if (ngram >= 2 && n_hist >= ngram - 1) {          /* :2270-2281 for ngram = 3 */
        const int m = ngram - 1;
        for (int j = 0; j + m < n_hist; j++) {
            int match = 1;
            for (int q = 0; q < m && match; q++)
                match = history[j + q] == history[n_hist - m + q];
            if (match) {
                const int banned = history[j + m];
                if (banned >= 0 && banned < vocab) adj[banned] = -1e30f;
            }
        }
    }
    int token;
    if (temp <= 0.01f) {                              /* sample_argmax, :1503-1509 */
        token = 0;
        for (int i = 1; i < vocab; i++)
            if (adj[i] > adj[token]) token = i;
        if (idx_out) idx_out[0] = token;
        if (prob_out) prob_out[0] = 1.0f;
    } else {
        const int k = top_k < vocab ? top_k : vocab;
        int *ind = (int *)malloc(sizeof(int) * (size_t)vocab);
        float *pr = (float *)malloc(sizeof(float) * (size_t)k);
        for (int j = 0; j < vocab; j++) ind[j] = j;
        for (int j = 0; j < k; j++) {
            int best = j;
            for (int q = j + 1; q < vocab; q++) {
                const float a = adj[ind[q]], b = adj[ind[best]];
                if (a > b || (tie_rule == 0 && a == b && ind[q] < ind[best])) best = q;
            }
            const int tmp = ind[j];
            ind[j] = ind[best];
            ind[best] = tmp;
        }
        const float mx = adj[ind[0]];
        float sum = 0.0f;
        for (int j = 0; j < k; j++) {
            volatile float d = adj[ind[j]] - mx;
            volatile float x = d / temp;
            pr[j] = (float)exp((double)x);
            sum += pr[j];
        }
        const float thresh = top_p * sum;
        int p_limit = k;
        float cum = 0.0f;
        for (int j = 0; j < k; j++) {
            cum += pr[j];
            if (cum > thresh) {
                p_limit = j + 1;
                break;
            }
        }
        const float r = u * cum;
        token = ind[0];
        float c2 = 0.0f;
        for (int j = 0; j < p_limit; j++) {
            c2 += pr[j];
            if (r < c2) {
                token = ind[j];
                break;
            }
        }
        for (int j = 0; j < k; j++) {
            if (idx_out) idx_out[j] = ind[j];
            if (prob_out) prob_out[j] = pr[j];
        }
        free(ind);
        free(pr);
    }
    free(adj);
    free(seen);
    return token;
}

/* rms_norm, runtime/lal_runtime.c:82-87 (the scale's sum of squares in
 * double instead of float; see lalb_oracle.h). */
void lalb_o_rms_norm(const float *x, const float *w, int n, float eps, float *out) {
    double ss = 0.0;
    for (int i = 0; i < n; i++) ss += (double)x[i] * (double)x[i];
    const float s = (float)(1.0 / sqrt(ss / (double)n + (double)eps));
    for (int i = 0; i < n; i++) {
        volatile float t = x[i] * s;     /* one rounding per product */
        out[i] = w ? t * w[i] : t;
    }
}

/* ------------------------------------------------------------------------ */
/* seed STE model (per-element CORE/BINARY/PRUNE)                            */
/* ------------------------------------------------------------------------ */
void lalb_o_logic_state(uint64_t seed, size_t n, float p_core, float p_binary,
                        uint8_t *state) {
    const uint64_t base = seed * 0xD1B54A32D192ED03ull;
    const float t1 = p_core, t2 = p_core + p_binary;
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)n; i++) {
        float u = (float)(lalb_o_mix64(base + (uint64_t)i) >> 40) *
                  (1.0f / 16777216.0f);
        state[i] = (uint8_t)(u < t1 ? 0 : (u < t2 ? 1 : 2));
    }
}

void lalb_o_logic_pack(const float *w, const uint8_t *state, int rows, int K,
                       int8_t *codes, float *srow) {
#pragma omp parallel for schedule(static)
    for (int j = 0; j < rows; j++) {
        const float *v = w + (size_t)j * K;
        const uint8_t *st = state + (size_t)j * K;
        float amax = 0.0f;
        double asum = 0.0;
        int nbin = 0;
        for (int i = 0; i < K; i++) {
            float a = fabsf(v[i]);
            if (st[i] == 0 && a > amax) amax = a;
            if (st[i] == 1) { asum += a; nbin++; }
        }
        float alpha = nbin ? (float)(asum / nbin) : 0.0f;
        float s = (amax > alpha ? amax : alpha) / 127.0f;
        int b = 0;
        if (s != 0.0f) {
            float t = roundf(alpha / s);
            b = t < 1.0f ? 1 : (t > 127.0f ? 127 : (int)t);
        }
        for (int i = 0; i < K; i++) {
            int c = 0;
            if (s != 0.0f) {
                if (st[i] == 0) {
                    float t = roundf(v[i] / s);
                    c = t > 127.0f ? 127 : (t < -127.0f ? -127 : (int)t);
                } else if (st[i] == 1) {
                    c = v[i] > 0.0f ? b : -b;
                }
            }
            codes[(size_t)j * K + i] = (int8_t)c;
        }
        srow[j] = s;
    }
}

void lalb_o_logic_forward(const int8_t *codes, const float *srow,
                          const float *bias, int rows, int K, const float *X,
                          int M, float *Y) {
#pragma omp parallel for schedule(static) collapse(2)
    for (int m = 0; m < M; m++) {
        for (int j = 0; j < rows; j++) {
            const int8_t *c = codes + (size_t)j * K;
            const float *x = X + (size_t)m * K;
            double acc = 0.0;
            for (int i = 0; i < K; i++) acc += (double)c[i] * (double)x[i];
            Y[(size_t)m * rows + j] =
                srow[j] * (float)acc + (bias ? bias[j] : 0.0f);
        }
    }
}

/* bin_layer_init_logic (runtime/lal_runtime.c:1567-1676): alpha = mean |w|
 * for BINARY rows, 0 for CORE and PRUNE; PRUNE rows lose their bias.
 * bin_layer_repack (:1703-1766): alpha = mean |w| for every row.
 * bin_forward logic path (:1852-1938): K = mean |x|; CORE
 * (w.x) * min(1/(alpha+1e-8), 5) * K + b; BINARY (sign(w).x) * alpha * K *
 * binary_scale + b with sign(w) = +1 iff w > 0; PRUNE 0.
 * bin_forward_pure_float (:543-582): CORE w.x + b; BINARY
 * b + (w.x) * binary_scale; PRUNE 0. */
void lalb_o_binlayer_forward(const float *W, const float *bias,
                             const uint8_t *mask, int in_dim, int out_dim,
                             const float *X, int M, float *Y, int mode,
                             int repack, float binary_scale, float *alpha_out) {
    float *alpha = (float *)malloc(sizeof(float) * (size_t)out_dim);
    for (int j = 0; j < out_dim; j++) {
        const float *w = W + (size_t)j * in_dim;
        double s = 0.0;
        for (int i = 0; i < in_dim; i++) s += fabs((double)w[i]);
        alpha[j] = (mask[j] == 1 || repack) ? (float)(s / in_dim) : 0.0f;
        if (alpha_out) alpha_out[j] = alpha[j];
    }
#pragma omp parallel for schedule(static)
    for (int m = 0; m < M; m++) {
        const float *x = X + (size_t)m * in_dim;
        double ks = 0.0;
        for (int i = 0; i < in_dim; i++) ks += fabs((double)x[i]);
        const double K = ks / in_dim;
        for (int j = 0; j < out_dim; j++) {
            const float *w = W + (size_t)j * in_dim;
            const uint8_t st = mask[j];
            const double b = (bias && st != 2) ? (double)bias[j] : 0.0;
            double y = 0.0;
            if (st == 0) {
                double d = 0.0;
                for (int i = 0; i < in_dim; i++) d += (double)w[i] * (double)x[i];
                if (mode == 0) {
                    double gain = 1.0 / ((double)alpha[j] + 1e-8);
                    if (gain > 5.0) gain = 5.0;
                    y = d * gain * K + b;
                } else {
                    y = d + b;
                }
            } else if (st == 1) {
                double d = 0.0;
                if (mode == 0) {
                    for (int i = 0; i < in_dim; i++) d += (w[i] > 0.0f ? 1.0 : -1.0) * (double)x[i];
                    y = d * (double)alpha[j] * K * (double)binary_scale + b;
                } else {
                    for (int i = 0; i < in_dim; i++) d += (double)w[i] * (double)x[i];
                    y = b + d * (double)binary_scale;
                }
            }
            Y[(size_t)m * out_dim + j] = (float)y;
        }
    }
    free(alpha);
}
