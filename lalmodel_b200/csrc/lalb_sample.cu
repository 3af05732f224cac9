// lalb_sample.cu -- next-token sampling on the GPU after the LM head.
//
// The reference downloads the logits and samples on the host: generate_text
// (models/ste_train.c:2229-2318) masks the special ids, applies the
// repetition penalty once per distinct generated token, bans tokens that
// would repeat a trigram, and then takes the argmax (temperature <= 0.01,
// sample_argmax :1503-1509) or samples from the top-k / top-p nucleus.  Here
// the same steps run on the device, over logits that never leave HBM:
//
//   kernel 1 (one CTA per vocabulary slice of <= 8192 ids): marks the
//     slice's history tokens and n-gram bans in shared memory from the
//     history list, forms each id's adjusted logit and its 64-bit key
//     (ordered float << 32 | ~id: larger value first, then lower id),
//     bitonic-sorts the slice's keys and writes its best top_k;
//   kernel 2 (one CTA): bitonic-sorts the candidates of all slices, takes
//     the global top_k and one thread forms the probabilities, the nucleus
//     and the draw in the reference's float order.
//
// The exponential is exp() in double rounded to float once (the reference
// calls expf); ties in the top-k order go to the lower id (the reference's
// selection sort agrees with that whenever the top_k values are distinct).
#include <algorithm>

#include "lalb_internal.cuh"
#include "lalb_kernels.cuh"

using namespace lalb;

namespace {

constexpr int kT1 = 256;          // threads of a slice CTA
constexpr int kT2 = 1024;         // threads of the selection CTA
constexpr int kMaxSlice = 8192;   // ids per slice CTA (keys in shared memory)
constexpr int kMaxCand = 16384;   // candidates the selection CTA sorts
constexpr int kMaxTopK = 256;

__host__ __device__ inline int pow2_at_least(int n) {
    int p = 1;
    while (p < n) p <<= 1;
    return p;
}

struct SampleGeom {
    int k;        // top_k clipped to the vocabulary
    int G;        // slice CTAs
    int slice;    // ids per slice
    int nb;       // keys per slice CTA (power of two >= slice)
    int nc;       // candidates (power of two >= G * k)
};

bool sample_geom(int vocab, int top_k, SampleGeom *g) {
    if (vocab <= 0 || top_k < 1 || top_k > kMaxTopK) return false;
    g->k = std::min(top_k, vocab);
    int G = (vocab + 1023) / 1024;
    if (G * g->k > kMaxCand) G = kMaxCand / g->k;
    g->G = std::max(G, 1);
    g->slice = (vocab + g->G - 1) / g->G;
    if (g->slice > kMaxSlice) return false;
    g->nb = pow2_at_least(std::max(g->slice, g->k));
    g->nc = pow2_at_least(g->G * g->k);
    return g->nb <= kMaxSlice && g->nc <= kMaxCand;
}

__device__ __forceinline__ float key_value(unsigned long long key) {
    const uint32_t u = (uint32_t)(key >> 32);
    return __uint_as_float((u & 0x80000000u) ? (u & 0x7FFFFFFFu) : ~u);
}
__device__ __forceinline__ int key_id(unsigned long long key) {
    return (int)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull));
}

// Sorts n (a power of two) keys in shared memory into descending order.
__device__ void bitonic_desc(unsigned long long *keys, int n, int tid, int nthr) {
    for (int k = 2; k <= n; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = tid; i < n; i += nthr) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const unsigned long long a = keys[i], b = keys[ixj];
                    const bool desc = (i & k) == 0;
                    if (desc ? (a < b) : (a > b)) {
                        keys[i] = b;
                        keys[ixj] = a;
                    }
                }
            }
            __syncthreads();
        }
    }
}

struct SampleArgs {
    const float *logits;
    int vocab;
    const int32_t *history;
    int n_hist;
    lalb_sampling p;
    const float *u;
    unsigned long long *cand;   // [G][k]
    int32_t *token;
    int32_t *topk_id;           // nullable [k]
    float *topk_prob;           // nullable [k]
    SampleGeom g;
};

__global__ void __launch_bounds__(kT1) sample_slice_kernel(const SampleArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int nb = a.g.nb;
    unsigned long long *keys = reinterpret_cast<unsigned long long *>(smem);
    unsigned char *in_hist = smem + (size_t)nb * 8;
    unsigned char *banned = in_hist + nb;
    const int tid = threadIdx.x;
    const int v0 = blockIdx.x * a.g.slice;
    const int v1 = min(a.vocab, v0 + a.g.slice);
    for (int i = tid; i < nb; i += kT1) in_hist[i] = banned[i] = 0;
    __syncthreads();
    // the slice's history tokens (penalised once, however often they occur)
    for (int j = tid; j < a.n_hist; j += kT1) {
        const int t = a.history[j];
        if (t >= v0 && t < v1) in_hist[t - v0] = 1;
    }
    // n-gram bans: t completes an n-gram whose first n-1 tokens end the history
    const int m = a.p.no_repeat_ngram - 1;
    if (m >= 1 && a.n_hist >= m) {
        for (int j = tid; j + m < a.n_hist; j += kT1) {
            bool match = true;
            for (int q = 0; q < m && match; ++q) match = a.history[j + q] == a.history[a.n_hist - m + q];
            const int t = a.history[j + m];
            if (match && t >= v0 && t < v1) banned[t - v0] = 1;
        }
    }
    __syncthreads();
    for (int i = tid; i < nb; i += kT1) {
        const int t = v0 + i;
        unsigned long long key = 0;   // padding sorts last
        if (t < v1) {
            float v = a.logits[t];
            if (t < a.p.n_masked_low_ids) v = -1e30f;
            if (in_hist[i]) v = v > 0.0f ? __fdiv_rn(v, a.p.rep_penalty) : __fmul_rn(v, a.p.rep_penalty);
            if (banned[i]) v = -1e30f;
            key = ((unsigned long long)ordered_key(v) << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)t);
        }
        keys[i] = key;
    }
    __syncthreads();
    bitonic_desc(keys, nb, tid, kT1);
    for (int i = tid; i < a.g.k; i += kT1) a.cand[(size_t)blockIdx.x * a.g.k + i] = keys[i];
}

__global__ void __launch_bounds__(kT2) sample_select_kernel(const SampleArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    unsigned long long *keys = reinterpret_cast<unsigned long long *>(smem);
    const int tid = threadIdx.x, n = a.g.G * a.g.k;
    for (int i = tid; i < a.g.nc; i += kT2) keys[i] = i < n ? a.cand[i] : 0ull;
    __syncthreads();
    bitonic_desc(keys, a.g.nc, tid, kT2);
    if (tid != 0) return;
    const int k = a.g.k;
    const float temp = a.p.temperature;
    int token = key_id(keys[0]);
    if (temp <= 0.01f) {   // sample_argmax: the first maximum
        if (a.topk_id) a.topk_id[0] = token;
        if (a.topk_prob) a.topk_prob[0] = 1.0f;
    } else {
        const float mx = key_value(keys[0]);
        float sum = 0.0f;
        for (int j = 0; j < k; ++j) {
            const float x = __fdiv_rn(__fsub_rn(key_value(keys[j]), mx), temp);
            const float pj = (float)exp((double)x);
            sum = __fadd_rn(sum, pj);
            if (a.topk_id) a.topk_id[j] = key_id(keys[j]);
            if (a.topk_prob) a.topk_prob[j] = pj;
        }
        const float thresh = __fmul_rn(a.p.top_p, sum);
        int p_limit = k;
        float cum = 0.0f;
        for (int j = 0; j < k; ++j) {
            cum = __fadd_rn(cum, (float)exp((double)__fdiv_rn(__fsub_rn(key_value(keys[j]), mx), temp)));
            if (cum > thresh) {
                p_limit = j + 1;
                break;
            }
        }
        const float r = __fmul_rn(a.u ? *a.u : 0.0f, cum);
        float c2 = 0.0f;
        for (int j = 0; j < p_limit; ++j) {
            c2 = __fadd_rn(c2, (float)exp((double)__fdiv_rn(__fsub_rn(key_value(keys[j]), mx), temp)));
            if (r < c2) {
                token = key_id(keys[j]);
                break;
            }
        }
    }
    *a.token = token;
}

}  // namespace

extern "C" int lalb_sample_ws_bytes(int vocab, int top_k, size_t *bytes) {
    SampleGeom g;
    if (!bytes || !sample_geom(vocab, top_k, &g)) return LALB_ERR_INVALID;
    *bytes = (size_t)g.G * g.k * sizeof(unsigned long long);
    return LALB_OK;
}

extern "C" int lalb_sample(lalb_ctx *ctx, const float *logits, int vocab, const int32_t *history,
                           int n_history, const lalb_sampling *params, const float *u, void *ws,
                           int32_t *token, int32_t *topk_id, float *topk_prob,
                           lalb_stream stream) {
    if (!ctx) return LALB_ERR_INVALID;
    if (!logits || !params || !ws || !token || n_history < 0 || (n_history > 0 && !history))
        return lalb_fail(ctx, LALB_ERR_INVALID, "sample: null argument or negative history");
    const lalb_sampling &p = *params;
    SampleGeom g;
    if (!sample_geom(vocab, p.top_k, &g))
        return lalb_fail(ctx, LALB_ERR_INVALID, "sample: vocab %d / top_k %d outside the limits", vocab,
                         p.top_k);
    if (!(p.rep_penalty > 0.0f) || !(p.top_p > 0.0f && p.top_p <= 1.0f) || p.no_repeat_ngram < 0 ||
        p.n_masked_low_ids < 0 || p.temperature != p.temperature)
        return lalb_fail(ctx, LALB_ERR_INVALID, "sample: bad parameters");
    if (p.temperature > 0.01f && !u)
        return lalb_fail(ctx, LALB_ERR_INVALID, "sample: a draw u is needed above temperature 0.01");
    if ((uintptr_t)ws & 7u) return lalb_fail(ctx, LALB_ERR_INVALID, "sample: ws must be 8-byte aligned");
    SampleArgs a = {};
    a.logits = logits;
    a.vocab = vocab;
    a.history = history;
    a.n_hist = n_history;
    a.p = p;
    a.u = u;
    a.cand = static_cast<unsigned long long *>(ws);
    a.token = token;
    a.topk_id = topk_id;
    a.topk_prob = topk_prob;
    a.g = g;
    cudaStream_t s = (cudaStream_t)stream;
    const int smem1 = g.nb * 8 + 2 * g.nb, smem2 = g.nc * 8;
    if (int st = lalb_set_smem_attr(ctx, (const void *)sample_slice_kernel, smem1)) return st;
    if (int st = lalb_set_smem_attr(ctx, (const void *)sample_select_kernel, smem2)) return st;
    sample_slice_kernel<<<g.G, kT1, smem1, s>>>(a);
    LALB_LAUNCH_CHECK(ctx, "sample_slice_kernel");
    sample_select_kernel<<<1, kT2, smem2, s>>>(a);
    LALB_LAUNCH_CHECK(ctx, "sample_select_kernel");
    return LALB_OK;
}
