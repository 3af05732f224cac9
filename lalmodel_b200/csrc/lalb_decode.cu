// lalb_decode.cu -- one-token decode over the Qwen2.5-shape Q4_K matmul set.
//
// The C host driver that the reference's (absent) tools/server/qwen7b_server.c
// would have been for the matmul part of a token (Makefile:165-170,
// README.md:14-15,130-131): per layer four fused Q4_K matvecs, then the Q8
// LM head with argmax.  Kernels are chained with programmatic dependent
// launch (each one starts streaming its weights while its predecessor is
// still finishing) and the whole token is captured once into a CUDA graph
// per set of buffer pointers, then replayed.
#include <map>
#include <tuple>
#include <vector>

#include "lalb_internal.cuh"
#include "lalb_kernels.cuh"

struct lalb_decoder {
    lalb_ctx *ctx;
    lalb_decoder_cfg cfg;
    std::vector<lalb_layer_weights> layers;
    const int8_t *lm_w = nullptr;
    const float *lm_s = nullptr;
    // activations (device, owned)
    float *qkv = nullptr;     // [q_rows + 2*kv_rows]
    float *h_res = nullptr;   // [hidden] residual stream
    int8_t *aq = nullptr;     // [ffn] quantized SwiGLU product
    float *asx = nullptr;     // [ffn/32]
    int32_t *asumq = nullptr; // [ffn/32]
    float *h_in_dev = nullptr;
    int32_t *argmax_dev = nullptr;
    int32_t *argmax_host = nullptr;  // pinned
    // persistent path
    lalb_layer_weights *layers_dev = nullptr;  // [n_layer]
    unsigned int *pctr = nullptr;              // grid-barrier counters [4*n_layer], ticket
    unsigned long long *pbest = nullptr;       // argmax key
    bool layers_dirty = true;
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
        const lalb_layer_weights &w = d->layers[l];
        const float *resid = l == 0 ? h_in : d->h_res;
        int st;
        {
            Q4kGemvArgs a = {};
            a.W = static_cast<const uint8_t *>(w.wqkv);
            a.rows = qkv_rows;
            a.K = c.hidden;
            a.x = resid;
            a.y = d->qkv;
            a.unit = 1;
            LALB_CUDA_TRY(ctx, mark());
            if ((st = lalb_launch_q4k_gemv(ctx, a, kInF32Rms, kEpiStore, s, pdl, 2))) return st;
            pdl = true;
        }
        {
            Q4kGemvArgs a = {};
            a.W = static_cast<const uint8_t *>(w.wo);
            a.rows = c.hidden;
            a.K = c.q_rows;
            a.x = d->qkv;  // the attention output is out of scope: q stands in
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
    a.W = d->lm_w;
    a.sw = d->lm_s;
    a.K = c.hidden;
    a.row_begin = 0;
    a.row_end = c.vocab;
    a.x = c.n_layer > 0 ? d->h_res : h_in;
    a.logits = logits;
    a.argmax = argmax;
    LALB_CUDA_TRY(ctx, mark());
    int st = lalb_launch_q8_head(ctx, a, kInF32Rms, s, pdl, 2);
    if (st) return st;
    LALB_CUDA_TRY(ctx, mark());
    if (h_out)
        LALB_CUDA_TRY(ctx, cudaMemcpyAsync(h_out, c.n_layer > 0 ? d->h_res : h_in,
                                           sizeof(float) * c.hidden, cudaMemcpyDeviceToDevice, s));
    return LALB_OK;
}

bool use_persistent(const lalb_decoder *d) {
    return d->persist_fits && d->path != LALB_DECODE_KERNELS;
}

// The same token as launch_token, as one cooperative kernel.
int launch_token_persistent(lalb_decoder *d, const float *h_in, float *h_out, float *logits,
                            int32_t *argmax, cudaStream_t s,
                            unsigned long long *trace = nullptr) {
    lalb_ctx *ctx = d->ctx;
    const lalb_decoder_cfg &c = d->cfg;
    if (d->layers_dirty) {
        if (c.n_layer > 0)
            LALB_CUDA_TRY(ctx, cudaMemcpyAsync(d->layers_dev, d->layers.data(),
                                               sizeof(lalb_layer_weights) * c.n_layer,
                                               cudaMemcpyHostToDevice, s));
        LALB_CUDA_TRY(ctx, cudaStreamSynchronize(s));  // the host vector may change after
        d->layers_dirty = false;
    }
    PersistArgs a = {};
    a.n_layer = c.n_layer;
    a.hidden = c.hidden;
    a.q_rows = c.q_rows;
    a.kv_rows = c.kv_rows;
    a.ffn = c.ffn;
    a.vocab = c.vocab;
    a.layers = d->layers_dev;
    a.lm_w = d->lm_w;
    a.lm_s = d->lm_s;
    a.h_in = h_in;
    a.h = d->h_res;
    a.qkv = d->qkv;
    a.aq = d->aq;
    a.asx = d->asx;
    a.asumq = d->asumq;
    a.logits = logits;
    a.argmax = argmax;
    a.gbar = d->pctr;
    a.ticket = d->pctr + 4 * c.n_layer;
    a.best = d->pbest;
    a.status = &ctx->scratch->status;
    a.trace = trace;
    if (int st = lalb_launch_persist(ctx, a, s)) return st;
    if (h_out)
        LALB_CUDA_TRY(ctx, cudaMemcpyAsync(h_out, c.n_layer > 0 ? d->h_res : h_in,
                                           sizeof(float) * c.hidden, cudaMemcpyDeviceToDevice, s));
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
    cudaFree(d->pctr);
    cudaFree(d->pbest);
    delete d;
}

}  // namespace

extern "C" int lalb_decoder_create(lalb_ctx *ctx, const lalb_decoder_cfg *cfg,
                                   lalb_decoder **out) {
    if (!ctx) return LALB_ERR_INVALID;
    if (!cfg || !out) return lalb_fail(ctx, LALB_ERR_INVALID, "decoder_create: null");
    *out = nullptr;
    const lalb_decoder_cfg &c = *cfg;
    if (c.n_layer < 0 || c.hidden <= 0 || c.hidden % 256 || c.q_rows <= 0 || c.q_rows % 256 ||
        c.kv_rows < 0 || c.ffn <= 0 || c.ffn % 256 || c.vocab <= 0 || c.hidden > 4096)
        return lalb_fail(ctx, LALB_ERR_INVALID,
                         "decoder_create: hidden/q_rows/ffn must be multiples of 256, hidden <= 4096");
    LALB_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    lalb_decoder *d = new (std::nothrow) lalb_decoder();
    if (!d) return LALB_ERR_NOMEM;
    d->ctx = ctx;
    d->cfg = c;
    d->layers.assign(c.n_layer, lalb_layer_weights{nullptr, nullptr, nullptr, nullptr});
    bool ok = cudaMalloc(&d->qkv, sizeof(float) * (c.q_rows + 2 * c.kv_rows)) == cudaSuccess &&
              cudaMalloc(&d->h_res, sizeof(float) * c.hidden) == cudaSuccess &&
              cudaMalloc(&d->aq, c.ffn) == cudaSuccess &&
              cudaMalloc(&d->asx, sizeof(float) * (c.ffn / 32)) == cudaSuccess &&
              cudaMalloc(&d->asumq, sizeof(int32_t) * (c.ffn / 32)) == cudaSuccess &&
              cudaMalloc(&d->h_in_dev, sizeof(float) * c.hidden) == cudaSuccess &&
              cudaMalloc(&d->argmax_dev, sizeof(int32_t)) == cudaSuccess &&
              cudaMallocHost(&d->argmax_host, sizeof(int32_t)) == cudaSuccess &&
              cudaMalloc(&d->layers_dev, sizeof(lalb_layer_weights) * (c.n_layer + 1)) ==
                  cudaSuccess &&
              cudaMalloc(&d->pctr, sizeof(unsigned int) * (4 * c.n_layer + 1)) == cudaSuccess &&
              cudaMalloc(&d->pbest, sizeof(unsigned long long)) == cudaSuccess &&
              cudaMemset(d->pctr, 0, sizeof(unsigned int) * (4 * c.n_layer + 1)) == cudaSuccess &&
              cudaMemset(d->pbest, 0, sizeof(unsigned long long)) == cudaSuccess &&
              cudaDeviceSynchronize() == cudaSuccess;
    if (!ok) {
        cudaGetLastError();
        free_decoder(d);
        return lalb_fail(ctx, LALB_ERR_NOMEM, "decoder_create: activation buffers");
    }
    // the persistent kernel's limits: activations in shared memory, gate/up
    // tiles per CTA, one resident CTA per SM for the grid barriers
    int coop = 0;
    cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, ctx->device);
    const long long gu_units = 2LL * c.ffn / 64;
    d->persist_fits = coop && c.hidden <= kPersistMaxHidden && c.q_rows <= kPersistMaxHidden &&
                      c.ffn <= kPersistMaxFfn && c.ffn % 32 == 0 &&
                      (gu_units + ctx->sm_count - 1) / ctx->sm_count <= lalb_persist_max_tiles() &&
                      (size_t)lalb_persist_smem_bytes() <= ctx->smem_optin;
    *out = d;
    return LALB_OK;
}

extern "C" int lalb_decoder_set_layer(lalb_decoder *d, int layer, const lalb_layer_weights *w) {
    if (!d) return LALB_ERR_INVALID;
    if (!w || layer < 0 || layer >= d->cfg.n_layer || !w->wqkv || !w->wo || !w->wgu || !w->wdown)
        return lalb_fail(d->ctx, LALB_ERR_INVALID, "decoder_set_layer: bad layer %d", layer);
    if (((uintptr_t)w->wqkv | (uintptr_t)w->wo | (uintptr_t)w->wgu | (uintptr_t)w->wdown) & 15u)
        return lalb_fail(d->ctx, LALB_ERR_INVALID,
                         "decoder_set_layer: weights must be 16-byte aligned");
    d->layers[layer] = *w;
    d->layers_dirty = true;
    drop_graphs(d);
    return LALB_OK;
}

extern "C" int lalb_decoder_set_lm_head(lalb_decoder *d, const int8_t *w, const float *sw) {
    if (!d) return LALB_ERR_INVALID;
    if (!w || !sw) return lalb_fail(d->ctx, LALB_ERR_INVALID, "decoder_set_lm_head: null");
    if (((uintptr_t)w & 15u) || ((uintptr_t)sw & 3u))
        return lalb_fail(d->ctx, LALB_ERR_INVALID, "decoder_set_lm_head: misaligned");
    d->lm_w = w;
    d->lm_s = sw;
    drop_graphs(d);
    return LALB_OK;
}

static int check_ready(lalb_decoder *d) {
    if (!d->lm_w) return lalb_fail(d->ctx, LALB_ERR_INVALID, "decoder: LM head not set");
    for (int l = 0; l < d->cfg.n_layer; ++l)
        if (!d->layers[l].wqkv)
            return lalb_fail(d->ctx, LALB_ERR_INVALID, "decoder: layer %d not set", l);
    return LALB_OK;
}

extern "C" int lalb_decoder_step(lalb_decoder *d, const float *h_in, float *h_out,
                                 float *logits, int32_t *argmax, lalb_stream stream) {
    if (!d) return LALB_ERR_INVALID;
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
    if (int st = check_ready(d)) return st;
    // The instrumented token is captured into a graph and replayed, so the
    // intervals hold device time only (no host launch latency between them).
    cudaStream_t s = nullptr;
    LALB_CUDA_TRY(ctx, cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
    cudaEvent_t dep = nullptr;
    const int n = 4 * d->cfg.n_layer + 1;
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
    const size_t n = (size_t)ctx->sm_count * (4 * d->cfg.n_layer + 1) * 8;
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
    *n_cta = ctx->sm_count;
    return st;
}

extern "C" int lalb_decoder_set_path(lalb_decoder *d, int path) {
    if (!d) return LALB_ERR_INVALID;
    if (path != LALB_DECODE_AUTO && path != LALB_DECODE_KERNELS && path != LALB_DECODE_PERSISTENT)
        return lalb_fail(d->ctx, LALB_ERR_INVALID, "decoder_set_path: unknown path %d", path);
    if (path == LALB_DECODE_PERSISTENT && !d->persist_fits)
        return lalb_fail(d->ctx, LALB_ERR_UNSUPPORTED,
                         "decoder_set_path: shapes outside the persistent kernel's limits");
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
    return use_persistent(d) ? 1 : 4 * d->cfg.n_layer + 1;
}

extern "C" int lalb_decoder_destroy(lalb_decoder *d) {
    if (!d) return LALB_ERR_INVALID;
    cudaSetDevice(d->ctx->device);
    free_decoder(d);
    return LALB_OK;
}
