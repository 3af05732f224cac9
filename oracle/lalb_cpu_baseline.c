/*
 * lalb_cpu_baseline.c -- AVX2 + OpenMP CPU kernels for the CPU baseline.
 *
 * TEST / BENCHMARK INFRASTRUCTURE ONLY: timed beside the GPU kernels as the
 * host-CPU baseline and checked against the scalar oracle.  It stands in for
 * the reference's AVX2 kernels (runtime/lal_q4k_kernel.h "256-bit maddubs,
 * 8-row parallel, prefetch", README.md:29,130; runtime/lal_q8_kernel.h
 * sign-trick int8 dot, README.md:131,285), which are absent from the
 * reference snapshot.  Integer sub-block dot products are exact (no int16
 * saturation is possible: |q*x| <= 15*127 and |w*x| <= 127*127 per lane, two
 * lanes per int16), so they equal the scalar oracle's; the fp32 combine is
 * vectorised and so differs from the oracle only by rounding.
 */
#include "lalb_oracle.h"

#include <immintrin.h>
#include <math.h>
#include <omp.h>
#include <string.h>

int lalb_cpu_threads(void) { return omp_get_max_threads(); }

/* The OpenMP team size of the baseline's parallel loops.  A launcher such as
 * torchrun exports OMP_NUM_THREADS=1 to every rank; the timed CPU baseline
 * sets its thread count explicitly instead of inheriting that. */
void lalb_cpu_set_threads(int n) {
    if (n > 0) omp_set_num_threads(n);
}

void lalb_cpu_quantize_act(const float *x, int M, int K, int8_t *xq, float *sx,
                           int32_t *sumq) {
    const int nblk = K / 32;
#pragma omp parallel for schedule(static) if (M > 1)
    for (int m = 0; m < M; m++)
        lalb_o_quantize_act(x + (size_t)m * K, 1, K, xq + (size_t)m * K,
                            sx + (size_t)m * nblk, sumq + (size_t)m * nblk);
}

static inline float hsum8(__m256 v) {
    __m128 lo = _mm256_castps256_ps128(v), hi = _mm256_extractf128_ps(v, 1);
    __m128 s = _mm_add_ps(lo, hi);
    s = _mm_add_ps(s, _mm_movehl_ps(s, s));
    s = _mm_add_ss(s, _mm_shuffle_ps(s, s, 1));
    return _mm_cvtss_f32(s);
}

/* One Q4_K row against a quantized activation vector. */
static inline float q4k_row(const uint8_t *row, int nb, const int8_t *xq,
                            const float *sx, const float *sxq) {
    const __m256i m4 = _mm256_set1_epi8(0x0F);
    const __m256i ones = _mm256_set1_epi16(1);
    __m256 acc = _mm256_setzero_ps();
    float minacc = 0.0f;
    for (int b = 0; b < nb; b++) {
        const uint8_t *blk = row + (size_t)b * 144;
        _mm_prefetch((const char *)(blk + 4 * 144), _MM_HINT_T0);
        _mm_prefetch((const char *)(blk + 4 * 144 + 64), _MM_HINT_T0);
        _mm_prefetch((const char *)(blk + 4 * 144 + 128), _MM_HINT_T0);
        uint16_t dh, mh;
        memcpy(&dh, blk, 2);
        memcpy(&mh, blk + 2, 2);
        float d = _cvtsh_ss(dh), dmin = _cvtsh_ss(mh);
        uint8_t sm[16];
        lalb_o_unpack_scales_6bit(blk + 4, sm);
        const int8_t *xb = xq + 256 * b;
        const float *sxb = sx + 8 * b;
        /* min term: dmin * sum_j m_j * sx_j * sumq_j */
        float mt = 0.0f;
        for (int j = 0; j < 8; j++) mt += (float)sm[8 + j] * sxq[8 * b + j];
        minacc += dmin * mt;
        for (int g = 0; g < 4; g++) {
            __m256i q = _mm256_loadu_si256((const __m256i *)(blk + 16 + 32 * g));
            __m256i lo = _mm256_and_si256(q, m4);
            __m256i hi = _mm256_and_si256(_mm256_srli_epi16(q, 4), m4);
            __m256i x0 = _mm256_loadu_si256((const __m256i *)(xb + 64 * g));
            __m256i x1 = _mm256_loadu_si256((const __m256i *)(xb + 64 * g + 32));
            __m256i p0 = _mm256_madd_epi16(_mm256_maddubs_epi16(lo, x0), ones);
            __m256i p1 = _mm256_madd_epi16(_mm256_maddubs_epi16(hi, x1), ones);
            float f0 = d * (float)sm[2 * g] * sxb[2 * g];
            float f1 = d * (float)sm[2 * g + 1] * sxb[2 * g + 1];
            acc = _mm256_fmadd_ps(_mm256_cvtepi32_ps(p0), _mm256_set1_ps(f0), acc);
            acc = _mm256_fmadd_ps(_mm256_cvtepi32_ps(p1), _mm256_set1_ps(f1), acc);
        }
    }
    return hsum8(acc) - minacc;
}

void lalb_cpu_q4k_gemv(const uint8_t *W, int rows, int K, const int8_t *xq,
                       const float *sx, const int32_t *sumq, float *y) {
    const int nb = K / 256, ns = K / 32;
    float sxq[ns > 0 ? ns : 1];
    for (int s = 0; s < ns; s++) sxq[s] = sx[s] * (float)sumq[s];
    /* 8 consecutive rows per scheduling unit (the reference's "8-row
     * parallel" structure); rows are independent. */
#pragma omp parallel for schedule(static)
    for (int r8 = 0; r8 < (rows + 7) / 8; r8++) {
        int r1 = r8 * 8 + 8 < rows ? r8 * 8 + 8 : rows;
        for (int r = r8 * 8; r < r1; r++)
            y[r] = q4k_row(W + (size_t)r * nb * 144, nb, xq, sx, sxq);
    }
}

int lalb_cpu_q8_lmhead(const int8_t *W, const float *sw, int rows, int K,
                       const int8_t *xq, const float *sx, float *logits) {
    const int nblk = K / 32;
    const __m256i ones = _mm256_set1_epi16(1);
    int nthr = omp_get_max_threads();
    float bestv[nthr > 0 ? nthr : 1];
    int besti[nthr > 0 ? nthr : 1];
    for (int t = 0; t < nthr; t++) besti[t] = -1;
#pragma omp parallel
    {
        int t = omp_get_thread_num();
        float bv = -INFINITY;
        int bi = -1;
#pragma omp for schedule(static)
        for (int r = 0; r < rows; r++) {
            const int8_t *wr = W + (size_t)r * K;
            __m256 acc = _mm256_setzero_ps();
            for (int b = 0; b < nblk; b++) {
                _mm_prefetch((const char *)(wr + 32 * b + 512), _MM_HINT_T0);
                __m256i w = _mm256_loadu_si256((const __m256i *)(wr + 32 * b));
                __m256i x = _mm256_loadu_si256((const __m256i *)(xq + 32 * b));
                /* sign trick: |w| (unsigned) x (sign(w) * x) (signed) */
                __m256i p = _mm256_maddubs_epi16(_mm256_sign_epi8(w, w),
                                                 _mm256_sign_epi8(x, w));
                p = _mm256_madd_epi16(p, ones);
                acc = _mm256_fmadd_ps(_mm256_cvtepi32_ps(p),
                                      _mm256_set1_ps(sx[b]), acc);
            }
            float v = sw[r] * hsum8(acc);
            logits[r] = v;
            if (v > bv) { bv = v; bi = r; }
        }
        bestv[t] = bv;
        besti[t] = bi;
    }
    int best = -1;
    float bv = -INFINITY;
    for (int t = 0; t < nthr; t++)      /* threads own increasing row ranges */
        if (besti[t] >= 0 && bestv[t] > bv) { bv = bestv[t]; best = besti[t]; }
    return best;
}
