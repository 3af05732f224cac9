// lalb_attention.cu -- standalone decode attention kernel (one layer, one
// token) and its C ABI entry point lalb_attention_decode, the replacement of
// apply_rope + attention_forward (runtime/lal_runtime.c:137-153, 833-882)
// for grouped KV heads.  The per-item arithmetic lives in lalb_attention.cuh
// and is shared with the persistent decode kernel's attention phase.
#include "lalb_attention.cuh"
#include "lalb_internal.cuh"
#include "lalb_kernels.cuh"

using namespace lalb;

namespace {

struct SyncAll {
    __device__ void operator()() const { __syncthreads(); }
};

// One CTA per item (q head, position chunk).  The position is `pos`, or
// *pos_ptr when that is given (a decoder's position word, advanced by the
// decoder after every token, so that a captured graph replays correctly).
// With part/cnt (S > 1) the chunks of a head meet through the partial
// buffer; without them every head is one chunk.
__global__ void __launch_bounds__(32 * kAttnWarps) attention_decode_kernel(AttnStep a,
                                                                          const int *pos_ptr,
                                                                          int max_ctx,
                                                                          unsigned int *status) {
    extern __shared__ __align__(16) unsigned char smem[];
    if (pos_ptr) a.pos = *pos_ptr;
    if (a.pos < 0 || a.pos >= max_ctx) {
        // nothing is read or written outside the caches: report and stop
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(status, LALB_STATUS_BAD_POSITION);
        return;
    }
    a.S = (a.part && a.cnt) ? attn_chunks(a.n_head, a.pos, gridDim.x) : 1;
    attn_items(a, blockIdx.x, gridDim.x, threadIdx.x, smem, SyncAll());
}

__global__ void advance_position_kernel(int *pos) { *pos += 1; }

__global__ void set_position_kernel(int *pos, int value) { *pos = value; }

}  // namespace

int lalb_attention_check(int n_head, int n_kv, int hd) {
    if (n_head <= 0 || n_kv <= 0 || n_head % n_kv) return LALB_ERR_INVALID;
    if (hd != 32 && hd != 64 && hd != 128 && hd != 256) return LALB_ERR_UNSUPPORTED;
    return LALB_OK;
}

int lalb_launch_attention(lalb_ctx *ctx, const AttnStep &a, const int *pos_ptr, int max_ctx,
                          int ctas, cudaStream_t s) {
    const int grid = ctas < a.n_head ? a.n_head : ctas;
    attention_decode_kernel<<<grid, 32 * kAttnWarps, kAttnSmemBytes, s>>>(a, pos_ptr, max_ctx,
                                                                        &ctx->scratch->status);
    LALB_LAUNCH_CHECK(ctx, "attention_decode_kernel");
    return LALB_OK;
}

int lalb_launch_advance_position(lalb_ctx *ctx, int *pos, cudaStream_t s) {
    advance_position_kernel<<<1, 1, 0, s>>>(pos);
    LALB_LAUNCH_CHECK(ctx, "advance_position_kernel");
    return LALB_OK;
}

int lalb_launch_set_position(lalb_ctx *ctx, int *pos, int value, cudaStream_t s) {
    set_position_kernel<<<1, 1, 0, s>>>(pos, value);
    LALB_LAUNCH_CHECK(ctx, "set_position_kernel");
    return LALB_OK;
}

extern "C" int lalb_attention_decode(lalb_ctx *ctx, const float *qkv, int n_head, int n_kv_head,
                                     int head_dim, int pos, int max_ctx, float rope_theta,
                                     float *k_cache, float *v_cache, float *out,
                                     lalb_stream stream) {
    if (!ctx) return LALB_ERR_INVALID;
    if (!qkv || !k_cache || !v_cache || !out)
        return lalb_fail(ctx, LALB_ERR_INVALID, "attention_decode: null pointer");
    if (int st = lalb_attention_check(n_head, n_kv_head, head_dim))
        return lalb_fail(ctx, st, "attention_decode: n_head %d, n_kv_head %d, head_dim %d "
                                  "(n_kv_head must divide n_head; head_dim 32, 64, 128 or 256)",
                         n_head, n_kv_head, head_dim);
    if (pos < 0 || pos >= max_ctx)
        return lalb_fail(ctx, LALB_ERR_INVALID, "attention_decode: pos %d outside [0, %d)", pos,
                         max_ctx);
    if ((((uintptr_t)k_cache | (uintptr_t)v_cache) & 15u))
        return lalb_fail(ctx, LALB_ERR_INVALID, "attention_decode: caches must be 16-byte aligned");
    if (!(rope_theta > 1.0f))
        return lalb_fail(ctx, LALB_ERR_INVALID, "attention_decode: rope_theta must be > 1");
    AttnStep a = {};
    a.qkv = qkv;
    a.k_cache = k_cache;
    a.v_cache = v_cache;
    a.out = out;
    a.n_head = n_head;
    a.n_kv = n_kv_head;
    a.hd = head_dim;
    a.pos = pos;
    a.S = 1;
    a.theta = (double)rope_theta;
    return lalb_launch_attention(ctx, a, nullptr, max_ctx, n_head, (cudaStream_t)stream);
}
