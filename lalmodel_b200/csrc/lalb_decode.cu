// lalb_decode.cu -- one-token decode over the Qwen2.5-shape Q4_K matmul set.
//
// The C host driver that the reference's (absent) tools/server/qwen7b_server.c
// would have been for the matmul part of a token (Makefile:165-170,
// README.md:14-15,130-131): per layer four fused Q4_K matvecs, then the Q8
// LM head with argmax.  Kernels are chained with programmatic dependent
// launch (each one starts streaming its weights while its predecessor is
// still finishing) and the whole token is captured once into a CUDA graph
// per set of buffer pointers, then replayed.
#include <cstring>
#include <map>
#include <tuple>
#include <vector>

#include "lalb_internal.cuh"
#include "lalb_kernels.cuh"

struct lalb_decoder {
    lalb_ctx *ctx;
    lalb_decoder_cfg cfg;
    // tensor parallelism: this decoder holds ranks [rank0, rank0 + ranks_here)
    // of n_rank (ranks_here is 1, or n_rank when one GPU runs every rank)
    int n_rank = 1, rank0 = 0, ranks_here = 1;
    std::vector<std::vector<lalb_layer_weights>> layers;   // [ranks_here][n_layer] row shards
    std::vector<const int8_t *> lm_w;                     // [ranks_here]
    std::vector<const float *> lm_s;
    const float *out_norm = nullptr;   // RMSNorm weights before the LM head (nullable)
    // attention (cfg.head_dim > 0): phases per layer, KV caches, position
    bool attn = false;
    int ppl = 4;
    std::vector<float *> kv_host;      // [n_layer][2] k, v cache pointers (caller-owned)
    float **kv_dev = nullptr;          // device copy for the persistent kernel
    bool kv_dirty = true;
    int pos = 0;                       // host mirror of the position word
    float *att = nullptr;              // chain: attention output [q_rows]
    // activations of the per-phase kernel chain (device, owned; one rank only)
    float *qkv = nullptr;     // [q_rows + 2*kv_rows]
    float *h_res = nullptr;   // [hidden] residual stream
    int8_t *aq = nullptr;     // [ffn] quantized SwiGLU product
    float *asx = nullptr;     // [ffn/32]
    int32_t *asumq = nullptr; // [ffn/32]
    float *h_in_dev = nullptr;
    int32_t *argmax_dev = nullptr;
    int32_t *argmax_host = nullptr;  // pinned
    // persistent path
    lalb_layer_weights *layers_dev = nullptr;  // [ranks_here][n_layer]
    unsigned char *xb_own = nullptr;           // exchange buffers of the held ranks
    size_t xb_bytes = 0;                       // one rank's exchange buffer
    unsigned char *xb[kPersistMaxRanks] = {};  // every rank's (peer mappings for others)
    bool xb_opened[kPersistMaxRanks] = {};     // mapped through CUDA IPC
    bool connected = false;
    bool layers_dirty = true;
    unsigned long long wait_ns = 10ull * 1000 * 1000 * 1000;   // bound on a grid / cross-GPU wait
    bool persist_fits = false;
    int path = LALB_DECODE_AUTO;
    bool use_graph = true;
    std::map<std::tuple<const void *, void *, void *, void *, void *>, cudaGraphExec_t> graphs;
};

namespace {

// Enqueues one token.  With `ev` (profiling), an event is recorded before
// every kernel and after the last one, and programmatic overlap is off so
// that each interval is one kernel.
int launch_token(lalb_decoder *d, const float *h_in, float *h_out, float *logits,
                 int32_t *argmax, cudaStream_t s, const std::vector<cudaEvent_t> *ev = nullptr) {
    lalb_ctx *ctx = d->ctx;
    const lalb_decoder_cfg &c = d->cfg;
    const int qkv_rows = c.q_rows + 2 * c.kv_rows;
    bool pdl = false;  // the first kernel of a token has no predecessor
    size_t mark_i = 0;
    auto mark = [&]() -> cudaError_t {
        if (!ev) return cudaSuccess;
        pdl = false;
        // external: inside stream capture this becomes a timestamp node
        return cudaEventRecordWithFlags((*ev)[mark_i++], s, cudaEventRecordExternal);
    };
    for (int l = 0; l < c.n_layer; ++l) {
        const lalb_layer_weights &w = d->layers[0][l];
        const float *resid = l == 0 ? h_in : d->h_res;
        int st;
        {
            Q4kGemvArgs a = {};
            a.W = static_cast<const uint8_t *>(w.wqkv);
            a.rows = qkv_rows;
            a.K = c.hidden;
            a.x = resid;
            a.gamma = w.attn_norm;
            a.eps = c.rms_eps;
            a.y = d->qkv;
            a.unit = 1;
            LALB_CUDA_TRY(ctx, mark());
            if ((st = lalb_launch_q4k_gemv(ctx, a, kInF32Rms, kEpiStore, s, pdl, 2))) return st;
            pdl = true;
        }
        if (d->attn) {
            const PersistXLayout L = lalb_persist_xlayout(c.n_layer, c.hidden, c.q_rows, c.kv_rows,
                                                          c.ffn, c.head_dim);
            lalb::AttnStep a = {};
            a.qkv = d->qkv;
            a.k_cache = d->kv_host[2 * l];
            a.v_cache = d->kv_host[2 * l + 1];
            a.out = d->att;
            a.part = reinterpret_cast<double *>(d->xb_own + L.att_part);
            a.cnt = reinterpret_cast<unsigned int *>(d->xb_own + L.att_cnt);
            a.n_head = c.q_rows / c.head_dim;
            a.n_kv = c.kv_rows / c.head_dim;
            a.hd = c.head_dim;
            a.theta = (double)c.rope_theta;
            LALB_CUDA_TRY(ctx, mark());
            const int ctas = a.n_head * lalb::attn_chunks(a.n_head, c.max_ctx - 1, ctx->sm_count);
            if ((st = lalb_launch_attention(ctx, a, reinterpret_cast<const int *>(d->xb_own + L.pos),
                                            c.max_ctx, ctas, s)))
                return st;
        }
        {
            Q4kGemvArgs a = {};
            a.W = static_cast<const uint8_t *>(w.wo);
            a.rows = c.hidden;
            a.K = c.q_rows;
            a.x = d->attn ? d->att : d->qkv;  // without attention q stands in
            a.y = d->h_res;
            a.resid = resid;
            a.unit = 1;
            LALB_CUDA_TRY(ctx, mark());
            if ((st = lalb_launch_q4k_gemv(ctx, a, kInF32, kEpiResid, s, pdl, 2))) return st;
        }
        {
            Q4kGemvArgs a = {};
            a.W = static_cast<const uint8_t *>(w.wgu);
            a.rows = 2 * c.ffn;
            a.K = c.hidden;
            a.x = d->h_res;
            a.gamma = w.ffn_norm;
            a.eps = c.rms_eps;
            a.aq = d->aq;
            a.asx = d->asx;
            a.asumq = d->asumq;
            a.unit = 64;
            LALB_CUDA_TRY(ctx, mark());
            if ((st = lalb_launch_q4k_gemv(ctx, a, kInF32Rms, kEpiSwiglu, s, pdl, 2))) return st;
        }
        {
            Q4kGemvArgs a = {};
            a.W = static_cast<const uint8_t *>(w.wdown);
            a.rows = c.hidden;
            a.K = c.ffn;
            a.xq = d->aq;
            a.sx = d->asx;
            a.sumq = d->asumq;
            a.y = d->h_res;
            a.resid = d->h_res;
            a.unit = 1;
            LALB_CUDA_TRY(ctx, mark());
            if ((st = lalb_launch_q4k_gemv(ctx, a, kInQ8, kEpiResid, s, pdl, 2))) return st;
        }
    }
    Q8HeadArgs a = {};
    a.W = d->lm_w[0];
    a.sw = d->lm_s[0];
    a.K = c.hidden;
    a.row_begin = 0;
    a.row_end = c.vocab;
    a.x = c.n_layer > 0 ? d->h_res : h_in;
    a.gamma = d->out_norm;
    a.eps = c.rms_eps;
    a.logits = logits;
    a.argmax = argmax;
    LALB_CUDA_TRY(ctx, mark());
    int st = lalb_launch_q8_head(ctx, a, kInF32Rms, s, pdl, 2);
    if (st) return st;
    LALB_CUDA_TRY(ctx, mark());
    if (d->attn) {
        const PersistXLayout L = lalb_persist_xlayout(c.n_layer, c.hidden, c.q_rows, c.kv_rows, c.ffn,
                                                      c.head_dim);
        if ((st = lalb_launch_advance_position(ctx, reinterpret_cast<int *>(d->xb_own + L.pos), s)))
            return st;
    }
    if (h_out)
        LALB_CUDA_TRY(ctx, cudaMemcpyAsync(h_out, c.n_layer > 0 ? d->h_res : h_in,
                                           sizeof(float) * c.hidden, cudaMemcpyDeviceToDevice, s));
    return LALB_OK;
}

bool use_persistent(const lalb_decoder *d) {
    return d->persist_fits && (d->n_rank > 1 || d->path != LALB_DECODE_KERNELS);
}

// The same token as launch_token, as one cooperative kernel (every held rank
// as one group of CTAs).
int launch_token_persistent(lalb_decoder *d, const float *h_in, float *h_out, float *logits,
                            int32_t *argmax, cudaStream_t s,
                            unsigned long long *trace = nullptr) {
    lalb_ctx *ctx = d->ctx;
    const lalb_decoder_cfg &c = d->cfg;
    if (d->layers_dirty) {
        for (int r = 0; r < d->ranks_here && c.n_layer > 0; ++r)
            LALB_CUDA_TRY(ctx, cudaMemcpyAsync(d->layers_dev + (size_t)r * c.n_layer,
                                               d->layers[r].data(),
                                               sizeof(lalb_layer_weights) * c.n_layer,
                                               cudaMemcpyHostToDevice, s));
        LALB_CUDA_TRY(ctx, cudaStreamSynchronize(s));  // the host vectors may change after
        d->layers_dirty = false;
    }
    if (d->attn && d->kv_dirty) {
        LALB_CUDA_TRY(ctx, cudaMemcpyAsync(d->kv_dev, d->kv_host.data(),
                                           sizeof(float *) * 2 * c.n_layer, cudaMemcpyHostToDevice, s));
        LALB_CUDA_TRY(ctx, cudaStreamSynchronize(s));
        d->kv_dirty = false;
    }
    PersistArgs a = {};
    a.n_layer = c.n_layer;
    a.hidden = c.hidden;
    a.q_rows = c.q_rows;
    a.kv_rows = c.kv_rows;
    a.ffn = c.ffn;
    a.vocab = c.vocab;
    a.ppl = d->ppl;
    a.norm = d->out_norm != nullptr;
    for (int r = 0; r < d->ranks_here; ++r)
        for (int l = 0; l < c.n_layer; ++l)
            if (d->layers[r][l].attn_norm || d->layers[r][l].ffn_norm) a.norm = 1;
    a.head_dim = c.head_dim;
    a.max_ctx = c.max_ctx;
    a.rope_theta = (double)c.rope_theta;
    a.kv_cache = d->kv_dev;
    a.n_rank = d->n_rank;
    a.rank0 = d->rank0;
    a.ranks_here = d->ranks_here;
    a.cta_per_rank = ctx->sm_count / d->ranks_here;
    a.remote = d->ranks_here < d->n_rank;
    for (int r = 0; r < d->ranks_here; ++r) {
        a.rk[r].layers = d->layers_dev + (size_t)r * c.n_layer;
        a.rk[r].lm_w = d->lm_w[r];
        a.rk[r].lm_s = d->lm_s[r];
    }
    for (int j = 0; j < d->n_rank; ++j) a.xb[j] = d->xb[j];
    a.h_in = h_in;
    a.rms_eps = c.rms_eps;
    a.out_norm = d->out_norm;
    a.logits = logits;
    a.argmax = argmax;
    a.status = &ctx->scratch->status;
    a.wait_ns = d->wait_ns;
    a.trace = trace;
    if (int st = lalb_launch_persist(ctx, a, s)) return st;
    if (h_out) {
        const PersistXLayout L = lalb_persist_xlayout(c.n_layer, c.hidden, c.q_rows, c.kv_rows, c.ffn,
                                                      c.head_dim);
        const float *hf = c.n_layer > 0 ? reinterpret_cast<const float *>(d->xb[d->rank0] + L.h) : h_in;
        LALB_CUDA_TRY(ctx, cudaMemcpyAsync(h_out, hf, sizeof(float) * c.hidden,
                                           cudaMemcpyDeviceToDevice, s));
    }
    return LALB_OK;
}

int enqueue_token(lalb_decoder *d, const float *h_in, float *h_out, float *logits,
                  int32_t *argmax, cudaStream_t s) {
    return use_persistent(d) ? launch_token_persistent(d, h_in, h_out, logits, argmax, s)
                             : launch_token(d, h_in, h_out, logits, argmax, s);
}

void drop_graphs(lalb_decoder *d) {
    for (auto &kv : d->graphs) cudaGraphExecDestroy(kv.second);
    d->graphs.clear();
}

void free_decoder(lalb_decoder *d) {
    drop_graphs(d);
    cudaFree(d->qkv);
    cudaFree(d->h_res);
    cudaFree(d->aq);
    cudaFree(d->asx);
    cudaFree(d->asumq);
    cudaFree(d->h_in_dev);
    cudaFree(d->argmax_dev);
    cudaFreeHost(d->argmax_host);
    cudaFree(d->layers_dev);
    cudaFree(d->kv_dev);
    cudaFree(d->att);
    for (int j = 0; j < kPersistMaxRanks; ++j)
        if (d->xb_opened[j]) cudaIpcCloseMemHandle(d->xb[j]);
    cudaFree(d->xb_own);
    delete d;
}

}  // namespace

extern "C" int lalb_tp_rows(const lalb_decoder_cfg *cfg, int n_rank, int rank, int matrix,
                            int *row0, int *row1) {
    if (!cfg || !row0 || !row1 || n_rank < 1 || n_rank > kPersistMaxRanks || rank < 0 ||
        rank >= n_rank || matrix < 0 || matrix > 4)
        return LALB_ERR_INVALID;
    lalb_tp_range(*cfg, matrix, n_rank, rank, row0, row1);
    return LALB_OK;
}

extern "C" int lalb_decoder_create_tp(lalb_ctx *ctx, const lalb_decoder_cfg *cfg, int n_rank,
                                      int rank, lalb_decoder **out) {
    if (!ctx) return LALB_ERR_INVALID;
    if (!cfg || !out) return lalb_fail(ctx, LALB_ERR_INVALID, "decoder_create: null");
    *out = nullptr;
    const lalb_decoder_cfg &c = *cfg;
    if (c.n_layer < 0 || c.hidden <= 0 || c.hidden % 256 || c.q_rows <= 0 || c.q_rows % 256 ||
        c.kv_rows < 0 || c.ffn <= 0 || c.ffn % 256 || c.vocab <= 0 || c.hidden > 4096)
        return lalb_fail(ctx, LALB_ERR_INVALID,
                         "decoder_create: hidden/q_rows/ffn must be multiples of 256, hidden <= 4096");
    if (c.vocab >= (1 << 24) || 2LL * c.ffn >= (1 << 24) || c.q_rows + 2LL * c.kv_rows >= (1 << 24))
        return lalb_fail(ctx, LALB_ERR_INVALID, "decoder_create: matrices must have < 2^24 rows");
    if (!(c.rms_eps >= 0.0f) || c.rms_eps > 1.0f)
        return lalb_fail(ctx, LALB_ERR_INVALID, "decoder_create: rms_eps %g outside [0, 1]",
                         (double)c.rms_eps);
    if (c.head_dim != 0) {
        if (c.head_dim < 0 || c.q_rows % c.head_dim || c.kv_rows <= 0 || c.kv_rows % c.head_dim ||
            lalb_attention_check(c.q_rows / c.head_dim, c.kv_rows / c.head_dim, c.head_dim))
            return lalb_fail(ctx, LALB_ERR_INVALID,
                             "decoder_create: head_dim %d (32, 64, 128 or 256, dividing q_rows and "
                             "kv_rows, KV heads dividing the heads)", c.head_dim);
        if (c.max_ctx <= 0 || (long long)c.max_ctx * c.kv_rows >= (1LL << 31))
            return lalb_fail(ctx, LALB_ERR_INVALID, "decoder_create: max_ctx %d", c.max_ctx);
        if (!(c.rope_theta == 0.0f || c.rope_theta > 1.0f))
            return lalb_fail(ctx, LALB_ERR_INVALID, "decoder_create: rope_theta %g",
                             (double)c.rope_theta);
    }
    if (n_rank < 1 || n_rank > kPersistMaxRanks || rank < -1 || rank >= n_rank)
        return lalb_fail(ctx, LALB_ERR_INVALID, "decoder_create: rank %d of %d", rank, n_rank);
    LALB_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    lalb_decoder *d = new (std::nothrow) lalb_decoder();
    if (!d) return LALB_ERR_NOMEM;
    d->ctx = ctx;
    d->cfg = c;
    if (d->cfg.rms_eps == 0.0f) d->cfg.rms_eps = 1e-5f;   // rms_norm's constant (lal_runtime.c:84)
    if (d->cfg.rope_theta == 0.0f) d->cfg.rope_theta = 10000.0f;   // apply_rope's base (:143)
    d->attn = c.head_dim > 0;
    d->ppl = d->attn ? 5 : 4;
    d->kv_host.assign(d->attn ? 2 * c.n_layer : 0, nullptr);
    d->n_rank = n_rank;
    d->rank0 = rank < 0 ? 0 : rank;
    d->ranks_here = rank < 0 ? n_rank : 1;
    d->layers.assign(d->ranks_here, std::vector<lalb_layer_weights>(c.n_layer, lalb_layer_weights{}));
    d->lm_w.assign(d->ranks_here, nullptr);
    d->lm_s.assign(d->ranks_here, nullptr);
    d->xb_bytes =
        lalb_persist_xlayout(c.n_layer, c.hidden, c.q_rows, c.kv_rows, c.ffn, c.head_dim).total;
    const bool chain = n_rank == 1;   // the per-phase kernel chain runs on one GPU only
    bool ok = (!chain || (cudaMalloc(&d->qkv, sizeof(float) * (c.q_rows + 2 * c.kv_rows)) == cudaSuccess &&
                          cudaMalloc(&d->h_res, sizeof(float) * c.hidden) == cudaSuccess &&
                          cudaMalloc(&d->aq, c.ffn) == cudaSuccess &&
                          cudaMalloc(&d->asx, sizeof(float) * (c.ffn / 32)) == cudaSuccess &&
                          cudaMalloc(&d->asumq, sizeof(int32_t) * (c.ffn / 32)) == cudaSuccess)) &&
              cudaMalloc(&d->h_in_dev, sizeof(float) * c.hidden) == cudaSuccess &&
              cudaMalloc(&d->argmax_dev, sizeof(int32_t)) == cudaSuccess &&
              cudaMallocHost(&d->argmax_host, sizeof(int32_t)) == cudaSuccess &&
              cudaMalloc(&d->layers_dev, sizeof(lalb_layer_weights) * (d->ranks_here * c.n_layer + 1)) ==
                  cudaSuccess &&
              (!d->attn || (cudaMalloc(&d->kv_dev, sizeof(float *) * (2 * c.n_layer + 1)) == cudaSuccess &&
                            (!chain || cudaMalloc(&d->att, sizeof(float) * c.q_rows) == cudaSuccess))) &&
              cudaMalloc(&d->xb_own, d->xb_bytes * d->ranks_here) == cudaSuccess &&
              cudaMemset(d->xb_own, 0, d->xb_bytes * d->ranks_here) == cudaSuccess &&
              cudaDeviceSynchronize() == cudaSuccess;
    if (!ok) {
        cudaGetLastError();
        free_decoder(d);
        return lalb_fail(ctx, LALB_ERR_NOMEM, "decoder_create: device buffers");
    }
    for (int r = 0; r < d->ranks_here; ++r) d->xb[d->rank0 + r] = d->xb_own + d->xb_bytes * r;
    d->connected = d->ranks_here == n_rank;
    // the persistent kernel's limits: activations in shared memory, gate/up
    // tiles per CTA, one resident CTA per SM (every rank of this GPU gets
    // sm_count / ranks_here of them)
    int coop = 0;
    cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, ctx->device);
    const int cta = ctx->sm_count / d->ranks_here;
    int g0, g1;
    lalb_tp_range(c, 2, n_rank, 0, &g0, &g1);
    const long long gu_units = (g1 - g0) / 64 + 1;   // the largest shard
    d->persist_fits = coop && cta >= 1 && c.hidden <= kPersistMaxHidden &&
                      c.q_rows <= kPersistMaxHidden && c.ffn <= kPersistMaxFfn && c.ffn % 32 == 0 &&
                      (gu_units + cta - 1) / cta <= lalb_persist_max_tiles() &&
                      (size_t)lalb_persist_smem_bytes() <= ctx->smem_optin;
    if (n_rank > 1 && !d->persist_fits) {
        free_decoder(d);
        return lalb_fail(ctx, LALB_ERR_UNSUPPORTED,
                         "decoder_create: tensor parallelism needs the persistent kernel's limits");
    }
    *out = d;
    return LALB_OK;
}

extern "C" int lalb_decoder_create(lalb_ctx *ctx, const lalb_decoder_cfg *cfg,
                                   lalb_decoder **out) {
    return lalb_decoder_create_tp(ctx, cfg, 1, 0, out);
}

static int held(lalb_decoder *d, int rank) {
    return rank >= d->rank0 && rank < d->rank0 + d->ranks_here;
}

extern "C" int lalb_decoder_set_layer_shard(lalb_decoder *d, int rank, int layer,
                                            const lalb_layer_weights *w) {
    if (!d) return LALB_ERR_INVALID;
    if (!held(d, rank))
        return lalb_fail(d->ctx, LALB_ERR_INVALID, "decoder_set_layer: rank %d not held here", rank);
    if (!w || layer < 0 || layer >= d->cfg.n_layer || !w->wqkv || !w->wo || !w->wgu || !w->wdown)
        return lalb_fail(d->ctx, LALB_ERR_INVALID, "decoder_set_layer: bad layer %d", layer);
    if (((uintptr_t)w->wqkv | (uintptr_t)w->wo | (uintptr_t)w->wgu | (uintptr_t)w->wdown |
         (uintptr_t)w->attn_norm | (uintptr_t)w->ffn_norm) & 15u)
        return lalb_fail(d->ctx, LALB_ERR_INVALID,
                         "decoder_set_layer: weights and norms must be 16-byte aligned");
    d->layers[rank - d->rank0][layer] = *w;
    d->layers_dirty = true;
    drop_graphs(d);
    return LALB_OK;
}

extern "C" int lalb_decoder_set_layer(lalb_decoder *d, int layer, const lalb_layer_weights *w) {
    if (!d) return LALB_ERR_INVALID;
    if (d->n_rank != 1)
        return lalb_fail(d->ctx, LALB_ERR_INVALID, "decoder_set_layer: use the shard call");
    return lalb_decoder_set_layer_shard(d, 0, layer, w);
}

extern "C" int lalb_decoder_set_lm_head_shard(lalb_decoder *d, int rank, const int8_t *w,
                                              const float *sw) {
    if (!d) return LALB_ERR_INVALID;
    if (!held(d, rank))
        return lalb_fail(d->ctx, LALB_ERR_INVALID, "decoder_set_lm_head: rank %d not held here", rank);
    if (!w || !sw) return lalb_fail(d->ctx, LALB_ERR_INVALID, "decoder_set_lm_head: null");
    if (((uintptr_t)w & 15u) || ((uintptr_t)sw & 3u))
        return lalb_fail(d->ctx, LALB_ERR_INVALID, "decoder_set_lm_head: misaligned");
    d->lm_w[rank - d->rank0] = w;
    d->lm_s[rank - d->rank0] = sw;
    drop_graphs(d);
    return LALB_OK;
}

extern "C" int lalb_decoder_set_lm_head(lalb_decoder *d, const int8_t *w, const float *sw) {
    if (!d) return LALB_ERR_INVALID;
    if (d->n_rank != 1)
        return lalb_fail(d->ctx, LALB_ERR_INVALID, "decoder_set_lm_head: use the shard call");
    return lalb_decoder_set_lm_head_shard(d, 0, w, sw);
}

extern "C" int lalb_decoder_set_output_norm(lalb_decoder *d, const float *w) {
    if (!d) return LALB_ERR_INVALID;
    if ((uintptr_t)w & 15u)
        return lalb_fail(d->ctx, LALB_ERR_INVALID, "decoder_set_output_norm: 16-byte alignment");
    d->out_norm = w;
    drop_graphs(d);
    return LALB_OK;
}

extern "C" int lalb_decoder_set_kv_cache(lalb_decoder *d, int layer, float *k_cache,
                                         float *v_cache) {
    if (!d) return LALB_ERR_INVALID;
    if (!d->attn)
        return lalb_fail(d->ctx, LALB_ERR_INVALID, "decoder_set_kv_cache: no attention (head_dim 0)");
    if (layer < 0 || layer >= d->cfg.n_layer || !k_cache || !v_cache ||
        (((uintptr_t)k_cache | (uintptr_t)v_cache) & 15u))
        return lalb_fail(d->ctx, LALB_ERR_INVALID,
                         "decoder_set_kv_cache: layer %d, caches non-null and 16-byte aligned", layer);
    d->kv_host[2 * layer] = k_cache;
    d->kv_host[2 * layer + 1] = v_cache;
    d->kv_dirty = true;
    drop_graphs(d);
    return LALB_OK;
}

extern "C" int lalb_decoder_set_position(lalb_decoder *d, int pos, lalb_stream stream) {
    if (!d) return LALB_ERR_INVALID;
    if (!d->attn)
        return lalb_fail(d->ctx, LALB_ERR_INVALID, "decoder_set_position: no attention (head_dim 0)");
    if (pos < 0 || pos > d->cfg.max_ctx)
        return lalb_fail(d->ctx, LALB_ERR_INVALID, "decoder_set_position: %d outside [0, %d]", pos,
                         d->cfg.max_ctx);
    LALB_CUDA_TRY(d->ctx, cudaSetDevice(d->ctx->device));
    const lalb_decoder_cfg &c = d->cfg;
    const PersistXLayout L =
        lalb_persist_xlayout(c.n_layer, c.hidden, c.q_rows, c.kv_rows, c.ffn, c.head_dim);
    for (int r = 0; r < d->ranks_here; ++r)
        if (int st = lalb_launch_set_position(
                d->ctx, reinterpret_cast<int *>(d->xb_own + d->xb_bytes * r + L.pos), pos,
                (cudaStream_t)stream))
            return st;
    d->pos = pos;
    return LALB_OK;
}

extern "C" int lalb_decoder_position(const lalb_decoder *d) {
    if (!d) return LALB_ERR_INVALID;
    return d->pos;
}

extern "C" int lalb_decoder_ipc_handle(lalb_decoder *d, void *handle) {
    if (!d) return LALB_ERR_INVALID;
    if (!handle || d->ranks_here != 1)
        return lalb_fail(d->ctx, LALB_ERR_INVALID, "decoder_ipc_handle: one rank per decoder");
    static_assert(sizeof(cudaIpcMemHandle_t) == LALB_IPC_HANDLE_BYTES, "IPC handle size");
    cudaIpcMemHandle_t h;
    LALB_CUDA_TRY(d->ctx, cudaIpcGetMemHandle(&h, d->xb_own));
    memcpy(handle, &h, sizeof(h));
    return LALB_OK;
}

extern "C" int lalb_decoder_connect(lalb_decoder *d, const void *handles) {
    if (!d) return LALB_ERR_INVALID;
    if (!handles || d->ranks_here != 1)
        return lalb_fail(d->ctx, LALB_ERR_INVALID, "decoder_connect: one rank per decoder");
    if (d->connected) return LALB_OK;
    LALB_CUDA_TRY(d->ctx, cudaSetDevice(d->ctx->device));
    for (int j = 0; j < d->n_rank; ++j) {
        if (j == d->rank0) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const unsigned char *>(handles) + (size_t)j * LALB_IPC_HANDLE_BYTES,
               sizeof(h));
        void *p = nullptr;
        LALB_CUDA_TRY(d->ctx, cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
        d->xb[j] = static_cast<unsigned char *>(p);
        d->xb_opened[j] = true;
    }
    d->connected = true;
    drop_graphs(d);
    return LALB_OK;
}

extern "C" int lalb_decoder_exchange_buffer(lalb_decoder *d, void **buf) {
    if (!d) return LALB_ERR_INVALID;
    if (!buf || d->ranks_here != 1)
        return lalb_fail(d->ctx, LALB_ERR_INVALID, "decoder_exchange_buffer: one rank per decoder");
    *buf = d->xb_own;
    return LALB_OK;
}

extern "C" int lalb_decoder_connect_local(lalb_decoder *d, void *const *bufs) {
    if (!d) return LALB_ERR_INVALID;
    if (!bufs || d->ranks_here != 1)
        return lalb_fail(d->ctx, LALB_ERR_INVALID, "decoder_connect_local: one rank per decoder");
    if (d->connected) return LALB_OK;
    for (int j = 0; j < d->n_rank; ++j) {
        if (!bufs[j] || ((uintptr_t)bufs[j] & 127u))
            return lalb_fail(d->ctx, LALB_ERR_INVALID,
                             "decoder_connect_local: exchange buffer %d null or misaligned", j);
        if (j == d->rank0 && bufs[j] != d->xb_own)
            return lalb_fail(d->ctx, LALB_ERR_INVALID,
                             "decoder_connect_local: entry %d is not this rank's buffer", j);
    }
    for (int j = 0; j < d->n_rank; ++j) d->xb[j] = static_cast<unsigned char *>(bufs[j]);
    d->connected = true;
    drop_graphs(d);
    return LALB_OK;
}

extern "C" int lalb_decoder_set_wait_limit(lalb_decoder *d, double seconds) {
    if (!d) return LALB_ERR_INVALID;
    if (!(seconds >= 1e-4 && seconds <= 600.0))
        return lalb_fail(d->ctx, LALB_ERR_INVALID, "decoder_set_wait_limit: %g s outside [1e-4, 600]",
                         seconds);
    d->wait_ns = (unsigned long long)(seconds * 1e9);
    drop_graphs(d);   // the limit is a kernel argument baked into captured graphs
    return LALB_OK;
}

extern "C" int lalb_decoder_reset(lalb_decoder *d, lalb_stream stream) {
    if (!d) return LALB_ERR_INVALID;
    LALB_CUDA_TRY(d->ctx, cudaSetDevice(d->ctx->device));
    LALB_CUDA_TRY(d->ctx, cudaMemsetAsync(d->xb_own, 0, d->xb_bytes * d->ranks_here,
                                          (cudaStream_t)stream));
    d->pos = 0;   // the position word is part of the buffer
    return LALB_OK;
}

static int check_ready(lalb_decoder *d) {
    for (int r = 0; r < d->ranks_here; ++r) {
        if (!d->lm_w[r])
            return lalb_fail(d->ctx, LALB_ERR_INVALID, "decoder: LM head of rank %d not set",
                             d->rank0 + r);
        for (int l = 0; l < d->cfg.n_layer; ++l)
            if (!d->layers[r][l].wqkv)
                return lalb_fail(d->ctx, LALB_ERR_INVALID, "decoder: layer %d of rank %d not set", l,
                                 d->rank0 + r);
    }
    if (!d->connected)
        return lalb_fail(d->ctx, LALB_ERR_INVALID, "decoder: peers not connected");
    if (d->attn) {
        for (int l = 0; l < d->cfg.n_layer; ++l)
            if (!d->kv_host[2 * l])
                return lalb_fail(d->ctx, LALB_ERR_INVALID, "decoder: KV cache of layer %d not set", l);
        if (d->pos >= d->cfg.max_ctx)
            return lalb_fail(d->ctx, LALB_ERR_INVALID, "decoder: position %d, the KV cache holds %d",
                             d->pos, d->cfg.max_ctx);
    }
    return LALB_OK;
}

static int step_impl(lalb_decoder *d, const float *h_in, float *h_out, float *logits,
                     int32_t *argmax, lalb_stream stream);

extern "C" int lalb_decoder_step(lalb_decoder *d, const float *h_in, float *h_out,
                                 float *logits, int32_t *argmax, lalb_stream stream) {
    if (!d) return LALB_ERR_INVALID;
    const int st = step_impl(d, h_in, h_out, logits, argmax, stream);
    if (st == LALB_OK && d->attn) ++d->pos;   // the token advances the device position word
    return st;
}

static int step_impl(lalb_decoder *d, const float *h_in, float *h_out, float *logits,
                     int32_t *argmax, lalb_stream stream) {
    lalb_ctx *ctx = d->ctx;
    if (!h_in) return lalb_fail(ctx, LALB_ERR_INVALID, "decoder_step: null h_in");
    if (int st = check_ready(d)) return st;
    cudaStream_t s = (cudaStream_t)stream;
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (s) LALB_CUDA_TRY(ctx, cudaStreamIsCapturing(s, &cap));
    if (d->layers_dirty && cap != cudaStreamCaptureStatusNone && use_persistent(d))
        return lalb_fail(ctx, LALB_ERR_INVALID,
                         "decoder_step: run one step outside stream capture after set_layer");
    if (!d->use_graph || !s || cap != cudaStreamCaptureStatusNone)
        return enqueue_token(d, h_in, h_out, logits, argmax, s);

    auto key = std::make_tuple((const void *)h_in, (void *)h_out, (void *)logits, (void *)argmax,
                               (void *)s);
    auto it = d->graphs.find(key);
    if (it == d->graphs.end()) {
        // first use of this pointer set: launch once directly (sets kernel
        // attributes outside capture), then capture the token into a graph
        int st = enqueue_token(d, h_in, h_out, logits, argmax, s);
        if (st) return st;
        cudaGraph_t g = nullptr;
        LALB_CUDA_TRY(ctx, cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
        st = enqueue_token(d, h_in, h_out, logits, argmax, s);
        cudaError_t e = cudaStreamEndCapture(s, &g);
        if (st) {
            if (g) cudaGraphDestroy(g);
            return st;
        }
        if (e != cudaSuccess) return lalb_cuda_fail(ctx, e, "cudaStreamEndCapture");
        cudaGraphExec_t ge = nullptr;
        e = cudaGraphInstantiate(&ge, g, 0);
        cudaGraphDestroy(g);
        if (e != cudaSuccess) return lalb_cuda_fail(ctx, e, "cudaGraphInstantiate");
        d->graphs[key] = ge;
        return LALB_OK;  // the direct launch above already produced this token
    }
    LALB_CUDA_TRY(ctx, cudaGraphLaunch(it->second, s));
    return LALB_OK;
}

extern "C" int lalb_decoder_step_host(lalb_decoder *d, const float *h_in_host,
                                      int32_t *argmax_host, lalb_stream stream) {
    if (!d) return LALB_ERR_INVALID;
    lalb_ctx *ctx = d->ctx;
    if (!h_in_host || !argmax_host)
        return lalb_fail(ctx, LALB_ERR_INVALID, "decoder_step_host: null host buffer");
    cudaStream_t s = (cudaStream_t)stream;
    LALB_CUDA_TRY(ctx, cudaMemcpyAsync(d->h_in_dev, h_in_host, sizeof(float) * d->cfg.hidden,
                                       cudaMemcpyHostToDevice, s));
    int st = lalb_decoder_step(d, d->h_in_dev, nullptr, nullptr, d->argmax_dev, stream);
    if (st) return st;
    LALB_CUDA_TRY(ctx, cudaMemcpyAsync(d->argmax_host, d->argmax_dev, sizeof(int32_t),
                                       cudaMemcpyDeviceToHost, s));
    LALB_CUDA_TRY(ctx, cudaStreamSynchronize(s));
    *argmax_host = *d->argmax_host;
    return LALB_OK;
}

extern "C" int lalb_decoder_profile_step(lalb_decoder *d, const float *h_in, float *kernel_us,
                                         lalb_stream stream) {
    if (!d) return LALB_ERR_INVALID;
    lalb_ctx *ctx = d->ctx;
    if (!h_in || !kernel_us)
        return lalb_fail(ctx, LALB_ERR_INVALID, "decoder_profile_step: null argument");
    if (d->n_rank != 1)
        return lalb_fail(ctx, LALB_ERR_UNSUPPORTED, "decoder_profile_step: one GPU only");
    if (int st = check_ready(d)) return st;
    // The instrumented token is captured into a graph and replayed, so the
    // intervals hold device time only (no host launch latency between them).
    cudaStream_t s = nullptr;
    LALB_CUDA_TRY(ctx, cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
    cudaEvent_t dep = nullptr;
    const int n = d->ppl * d->cfg.n_layer + 1;
    std::vector<cudaEvent_t> ev(n + 1, nullptr);
    int st = LALB_OK;
    for (auto &e : ev)
        if (cudaEventCreate(&e) != cudaSuccess) st = LALB_ERR_CUDA;
    // order the private stream after the caller's work
    if (!st && (cudaEventCreateWithFlags(&dep, cudaEventDisableTiming) != cudaSuccess ||
                cudaEventRecord(dep, (cudaStream_t)stream) != cudaSuccess ||
                cudaStreamWaitEvent(s, dep, 0) != cudaSuccess))
        st = LALB_ERR_CUDA;
    cudaGraph_t g = nullptr;
    cudaGraphExec_t ge = nullptr;
    if (!st && cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal) != cudaSuccess)
        st = LALB_ERR_CUDA;
    if (!st) {
        st = launch_token(d, h_in, nullptr, nullptr, d->argmax_dev, s, &ev);
        if (cudaStreamEndCapture(s, &g) != cudaSuccess && !st) st = LALB_ERR_CUDA;
    }
    if (!st && cudaGraphInstantiate(&ge, g, 0) != cudaSuccess) st = LALB_ERR_CUDA;
    if (!st && cudaGraphLaunch(ge, s) != cudaSuccess) st = LALB_ERR_CUDA;
    if (!st && cudaEventSynchronize(ev[n]) != cudaSuccess) st = LALB_ERR_CUDA;
    if (ge) cudaGraphExecDestroy(ge);
    if (g) cudaGraphDestroy(g);
    if (dep) cudaEventDestroy(dep);
    cudaStreamSynchronize(s);
    cudaStreamDestroy(s);
    for (int i = 0; !st && i < n; ++i) {
        float ms = 0.0f;
        if (cudaEventElapsedTime(&ms, ev[i], ev[i + 1]) != cudaSuccess) st = LALB_ERR_CUDA;
        kernel_us[i] = 1000.0f * ms;
    }
    for (auto &e : ev)
        if (e) cudaEventDestroy(e);
    if (st == LALB_ERR_CUDA)
        return lalb_fail(ctx, st, "decoder_profile_step: event timing failed (%s)",
                         cudaGetErrorString(cudaGetLastError()));
    if (st == LALB_OK && d->attn) ++d->pos;
    return st;
}

extern "C" int lalb_decoder_trace_step(lalb_decoder *d, const float *h_in,
                                       unsigned long long *trace_host, int trace_len,
                                       int *n_cta, lalb_stream stream) {
    if (!d) return LALB_ERR_INVALID;
    lalb_ctx *ctx = d->ctx;
    if (!h_in || !trace_host || !n_cta)
        return lalb_fail(ctx, LALB_ERR_INVALID, "decoder_trace_step: null argument");
    if (int st = check_ready(d)) return st;
    if (!use_persistent(d))
        return lalb_fail(ctx, LALB_ERR_INVALID, "decoder_trace_step: needs the persistent path");
    const size_t n = (size_t)ctx->sm_count * (d->ppl * d->cfg.n_layer + 1) * 8;
    if ((size_t)trace_len < n)
        return lalb_fail(ctx, LALB_ERR_INVALID, "decoder_trace_step: trace_len < %zu", n);
    cudaStream_t s = (cudaStream_t)stream;
    unsigned long long *tr = nullptr;
    LALB_CUDA_TRY(ctx, cudaMalloc(&tr, n * sizeof(unsigned long long)));
    int st = launch_token_persistent(d, h_in, nullptr, nullptr, d->argmax_dev, s, tr);
    if (!st && (cudaMemcpyAsync(trace_host, tr, n * sizeof(unsigned long long),
                                cudaMemcpyDeviceToHost, s) != cudaSuccess ||
                cudaStreamSynchronize(s) != cudaSuccess))
        st = lalb_cuda_fail(ctx, cudaGetLastError(), "decoder_trace_step: copy");
    cudaFree(tr);
    *n_cta = (ctx->sm_count / d->ranks_here) * d->ranks_here;
    if (st == LALB_OK && d->attn) ++d->pos;
    return st;
}

extern "C" int lalb_decoder_set_path(lalb_decoder *d, int path) {
    if (!d) return LALB_ERR_INVALID;
    if (path != LALB_DECODE_AUTO && path != LALB_DECODE_KERNELS && path != LALB_DECODE_PERSISTENT)
        return lalb_fail(d->ctx, LALB_ERR_INVALID, "decoder_set_path: unknown path %d", path);
    if (path == LALB_DECODE_PERSISTENT && !d->persist_fits)
        return lalb_fail(d->ctx, LALB_ERR_UNSUPPORTED,
                         "decoder_set_path: shapes outside the persistent kernel's limits");
    if (path == LALB_DECODE_KERNELS && d->n_rank != 1)
        return lalb_fail(d->ctx, LALB_ERR_UNSUPPORTED,
                         "decoder_set_path: the kernel chain runs on one GPU only");
    if (path != d->path) drop_graphs(d);
    d->path = path;
    return LALB_OK;
}

extern "C" int lalb_decoder_path(const lalb_decoder *d) {
    if (!d) return LALB_ERR_INVALID;
    return use_persistent(d) ? LALB_DECODE_PERSISTENT : LALB_DECODE_KERNELS;
}

extern "C" int lalb_decoder_launches_per_step(const lalb_decoder *d) {
    if (!d) return LALB_ERR_INVALID;
    // the chain: one kernel per phase, plus the position update with attention
    return use_persistent(d) ? 1 : d->ppl * d->cfg.n_layer + 1 + (d->attn ? 1 : 0);
}

extern "C" int lalb_decoder_destroy(lalb_decoder *d) {
    if (!d) return LALB_ERR_INVALID;
    cudaSetDevice(d->ctx->device);
    free_decoder(d);
    return LALB_OK;
}
