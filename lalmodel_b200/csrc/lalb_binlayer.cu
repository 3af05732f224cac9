// lalb_binlayer.cu -- the seed STE model's logic-masked forward on tensor
// cores.
//
// A BinLayer (runtime/lal_runtime.h:171-197) has one CORE / BINARY / PRUNE
// state per output row.  The reference's forward, per input row x:
//   bin_forward (runtime/lal_runtime.c:1852-1938), K = mean |x|:
//     CORE    y = (w . x) * min(1 / (alpha + 1e-8), 5) * K + b
//     BINARY  y = (sign(w) . x) * alpha * K * binary_scale + b
//     PRUNE   y = 0
//   bin_forward_pure_float (:543-582):
//     CORE    y = w . x + b
//     BINARY  y = b + (w . x) * binary_scale
//     PRUNE   y = 0
// with sign(w) = +1 for w > 0, else -1, and alpha = mean |w| over the row
// for BINARY rows and 0 for CORE rows as bin_layer_init_logic (:1567-1676)
// leaves it, or mean |w| for every row after bin_layer_repack (:1703-1766).
//
// Both are Y = rowscale (X . B^T) colscale + bias with a per-mode B, so one
// tcgen05 GEMM serves them: lalb_binlayer_create builds B (fp32 weights, +-1
// or 0 per row, split into tf32 parts), the column scales and biases;
// lalb_binlayer_forward splits X and computes K.
//
// The per-element encoding (each weight CORE, BINARY or PRUNE, packed as
// int8 codes with a per-row scale: lalb_logic_pack / lalb_logic_layer_*)
// runs on its own tensor-core GEMM straight from the int8 codes
// (lalb_logic_gemm.cu).
#include <algorithm>

#include "lalb_internal.cuh"
#include "lalb_logic_gemm.cuh"
#include "lalb_tc_gemm.cuh"

struct lalb_binlayer {
    lalb_ctx *ctx;
    int in, out, max_rows;
    float *b0_hi, *b0_lo;   // bin_forward weights [out][in]
    float *b1_hi, *b1_lo;   // bin_forward_pure_float weights
    float *cs0, *bias0;     // [out]
    float *cs1, *bias1;
    float *alpha;           // [out]
    float *knorm;           // [max_rows]
};

struct lalb_logic_layer {
    lalb_ctx *ctx;
    int rows, K, max_rows;
    const int8_t *codes;    // [rows][K], the caller's (read in place)
    const float *srow, *bias;
    void *ws;               // token parts and split-K partial sums
    size_t ws_bytes;
};

namespace {

// sum over the block of a per-thread double (blockDim.x a multiple of 32, <= 1024)
__device__ __forceinline__ double block_sum_d(double v, double *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    double t = 0.0;
    for (int k = 0; k < (int)(blockDim.x >> 5); ++k) t += red[k];
    __syncthreads();
    return t;
}

// One CTA per output row: alpha, both modes' weights, scales and biases.
__global__ void binlayer_pack_kernel(const float *__restrict__ W, const float *__restrict__ bias,
                                     const uint8_t *__restrict__ mask, int in, int repack,
                                     float binary_scale, lalb_binlayer bl) {
    const int j = blockIdx.x;
    const float *w = W + (size_t)j * in;
    const uint8_t m = mask[j];
    __shared__ double red[32];
    double s = 0.0;
    for (int i = threadIdx.x; i < in; i += blockDim.x) s += fabs((double)w[i]);
    const double t = block_sum_d(s, red);
    const float mean_abs = (float)(t / in);
    const float alpha = (m == 1 || repack) ? mean_abs : 0.0f;
    const float b = bias && m != 2 ? bias[j] : 0.0f;
    for (int i = threadIdx.x; i < in; i += blockDim.x) {
        const float v = w[i];
        uint32_t h, l;
        asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(v));
        const float r = __fsub_rn(v, __uint_as_float(h));
        asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(l) : "f"(r));
        const float whi = __uint_as_float(h), wlo = __uint_as_float(l);
        const size_t o = (size_t)j * in + i;
        // bin_forward: CORE w, BINARY sign(w), PRUNE 0
        bl.b0_hi[o] = m == 0 ? whi : (m == 1 ? (v > 0.0f ? 1.0f : -1.0f) : 0.0f);
        bl.b0_lo[o] = m == 0 ? wlo : 0.0f;
        // bin_forward_pure_float: CORE and BINARY w, PRUNE 0
        bl.b1_hi[o] = m == 2 ? 0.0f : whi;
        bl.b1_lo[o] = m == 2 ? 0.0f : wlo;
    }
    if (threadIdx.x == 0) {
        bl.alpha[j] = alpha;
        float gain = 1.0f / (alpha + 1e-8f);
        if (gain > 5.0f) gain = 5.0f;
        bl.cs0[j] = m == 0 ? gain : (m == 1 ? alpha * binary_scale : 0.0f);
        bl.cs1[j] = m == 0 ? 1.0f : (m == 1 ? binary_scale : 0.0f);
        bl.bias0[j] = b;
        bl.bias1[j] = b;
    }
}

// K = mean |x| per input row (double sum, one rounding).
__global__ void knorm_kernel(const float *__restrict__ X, int in, float *__restrict__ k) {
    const float *x = X + (size_t)blockIdx.x * in;
    __shared__ double red[32];
    double s = 0.0;
    for (int i = threadIdx.x; i < in; i += blockDim.x) s += fabs((double)x[i]);
    const double t = block_sum_d(s, red);
    if (threadIdx.x == 0) k[blockIdx.x] = (float)(t / in);
}

// Per-element CORE/BINARY/PRUNE codes, as the oracle's lalb_o_logic_pack:
// per row, s = max(amax of CORE weights, alpha = mean |w| of BINARY weights)
// / 127; CORE -> round(w / s) clamped to +-127, BINARY -> +-round(alpha / s)
// (at least 1), PRUNE -> 0.
__global__ void logic_pack_kernel(const float *__restrict__ W, const uint8_t *__restrict__ state,
                                  int K, int8_t *__restrict__ codes, float *__restrict__ srow) {
    const int j = blockIdx.x;
    const float *v = W + (size_t)j * K;
    const uint8_t *st = state + (size_t)j * K;
    __shared__ double red[32];
    __shared__ unsigned int ramax;
    if (threadIdx.x == 0) ramax = 0;
    __syncthreads();
    double asum = 0.0, nbin = 0.0;
    uint32_t amax = 0;
    for (int i = threadIdx.x; i < K; i += blockDim.x) {
        const float a = fabsf(v[i]);
        if (st[i] == 0) amax = max(amax, __float_as_uint(a));
        if (st[i] == 1) {
            asum += a;
            nbin += 1.0;
        }
    }
    atomicMax(&ramax, amax);
    const double t = block_sum_d(asum, red);
    const double nb = block_sum_d(nbin, red);
    const float alpha = nb > 0.0 ? (float)(t / nb) : 0.0f;
    const float am = __uint_as_float(ramax);
    const float s = __fdiv_rn(am > alpha ? am : alpha, 127.0f);
    int b = 0;
    if (s != 0.0f) {
        const float tb = roundf(__fdiv_rn(alpha, s));
        b = tb < 1.0f ? 1 : (tb > 127.0f ? 127 : (int)tb);
    }
    for (int i = threadIdx.x; i < K; i += blockDim.x) {
        int c = 0;
        if (s != 0.0f) {
            if (st[i] == 0) {
                const float tq = roundf(__fdiv_rn(v[i], s));
                c = tq > 127.0f ? 127 : (tq < -127.0f ? -127 : (int)tq);
            } else if (st[i] == 1) {
                c = v[i] > 0.0f ? b : -b;
            }
        }
        codes[(size_t)j * K + i] = (int8_t)c;
    }
    if (threadIdx.x == 0) srow[j] = s;
}

void free_binlayer(lalb_binlayer *b) {
    for (float *p : {b->b0_hi, b->b0_lo, b->b1_hi, b->b1_lo, b->cs0, b->bias0, b->cs1, b->bias1,
                     b->alpha, b->knorm})
        cudaFree(p);
    delete b;
}

void free_logic(lalb_logic_layer *L) {
    cudaFree(L->ws);
    delete L;
}

}  // namespace

extern "C" int lalb_binlayer_create(lalb_ctx *ctx, const float *W, const float *bias,
                                    const uint8_t *mask, int in_dim, int out_dim, int alpha_repack,
                                    float binary_scale, int max_rows, lalb_binlayer **out) {
    if (!ctx) return LALB_ERR_INVALID;
    if (!W || !mask || !out || in_dim <= 0 || out_dim <= 0 || max_rows <= 0)
        return lalb_fail(ctx, LALB_ERR_INVALID, "binlayer_create: bad arguments");
    if (in_dim % 32)
        return lalb_fail(ctx, LALB_ERR_UNSUPPORTED, "binlayer_create: in_dim must be a multiple of 32");
    *out = nullptr;
    LALB_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    lalb_binlayer *b = new (std::nothrow) lalb_binlayer();
    if (!b) return LALB_ERR_NOMEM;
    b->ctx = ctx;
    b->in = in_dim;
    b->out = out_dim;
    b->max_rows = max_rows;
    const size_t wn = (size_t)in_dim * out_dim;
    bool ok = cudaMalloc(&b->b0_hi, 4 * wn) == cudaSuccess && cudaMalloc(&b->b0_lo, 4 * wn) == cudaSuccess &&
              cudaMalloc(&b->b1_hi, 4 * wn) == cudaSuccess && cudaMalloc(&b->b1_lo, 4 * wn) == cudaSuccess &&
              cudaMalloc(&b->cs0, 4 * out_dim) == cudaSuccess &&
              cudaMalloc(&b->bias0, 4 * out_dim) == cudaSuccess &&
              cudaMalloc(&b->cs1, 4 * out_dim) == cudaSuccess &&
              cudaMalloc(&b->bias1, 4 * out_dim) == cudaSuccess &&
              cudaMalloc(&b->alpha, 4 * out_dim) == cudaSuccess && cudaMalloc(&b->knorm, 4 * max_rows) == cudaSuccess;
    if (!ok) {
        cudaGetLastError();
        free_binlayer(b);
        return lalb_fail(ctx, LALB_ERR_NOMEM, "binlayer_create: device buffers");
    }
    binlayer_pack_kernel<<<out_dim, 256>>>(W, bias, mask, in_dim, alpha_repack, binary_scale, *b);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        free_binlayer(b);
        return lalb_cuda_fail(ctx, e, "binlayer_pack_kernel");
    }
    *out = b;
    return LALB_OK;
}

extern "C" int lalb_binlayer_forward(lalb_binlayer *b, const float *X, int M, float *Y, int mode,
                                     lalb_stream stream) {
    if (!b) return LALB_ERR_INVALID;
    lalb_ctx *ctx = b->ctx;
    if (!X || !Y || M <= 0 || M > b->max_rows || (mode != 0 && mode != 1))
        return lalb_fail(ctx, LALB_ERR_INVALID, "binlayer_forward: bad arguments (M <= %d, mode 0/1)",
                         b->max_rows);
    cudaStream_t s = (cudaStream_t)stream;
    if (mode == 0) {
        knorm_kernel<<<M, 128, 0, s>>>(X, b->in, b->knorm);
        LALB_LAUNCH_CHECK(ctx, "knorm_kernel");
    }
    TcGemmParts p = {};
    p.M = M;
    p.N = b->out;
    p.K = b->in;
    p.a_hi = X;   // the GEMM splits X into tf32 parts in shared memory
    p.split_a = 1;
    p.b_hi = mode == 0 ? b->b0_hi : b->b1_hi;
    p.b_lo = mode == 0 ? b->b0_lo : b->b1_lo;
    p.Y = Y;
    p.rowscale = mode == 0 ? b->knorm : nullptr;
    p.colscale = mode == 0 ? b->cs0 : b->cs1;
    p.bias = mode == 0 ? b->bias0 : b->bias1;
    return lalb_tc_gemm_tf32(ctx, p, s);
}

extern "C" int lalb_binlayer_alpha(lalb_binlayer *b, float *alpha, lalb_stream stream) {
    if (!b) return LALB_ERR_INVALID;
    if (!alpha) return lalb_fail(b->ctx, LALB_ERR_INVALID, "binlayer_alpha: null");
    LALB_CUDA_TRY(b->ctx, cudaMemcpyAsync(alpha, b->alpha, 4 * (size_t)b->out, cudaMemcpyDeviceToDevice,
                                          (cudaStream_t)stream));
    return LALB_OK;
}

extern "C" int lalb_binlayer_destroy(lalb_binlayer *b) {
    if (!b) return LALB_ERR_INVALID;
    cudaSetDevice(b->ctx->device);
    free_binlayer(b);
    return LALB_OK;
}

extern "C" int lalb_logic_pack(lalb_ctx *ctx, const float *W, const uint8_t *state, int rows, int K,
                               int8_t *codes, float *srow, lalb_stream stream) {
    if (!ctx) return LALB_ERR_INVALID;
    if (!W || !state || !codes || !srow || rows <= 0 || K <= 0)
        return lalb_fail(ctx, LALB_ERR_INVALID, "logic_pack: bad arguments");
    logic_pack_kernel<<<rows, 256, 0, (cudaStream_t)stream>>>(W, state, K, codes, srow);
    LALB_LAUNCH_CHECK(ctx, "logic_pack_kernel");
    return LALB_OK;
}

extern "C" int lalb_logic_layer_create(lalb_ctx *ctx, const int8_t *codes, const float *srow,
                                       const float *bias, int rows, int K, int max_rows,
                                       lalb_logic_layer **out) {
    if (!ctx) return LALB_ERR_INVALID;
    if (!codes || !srow || !out || rows <= 0 || K <= 0 || max_rows <= 0)
        return lalb_fail(ctx, LALB_ERR_INVALID, "logic_layer_create: bad arguments");
    if (K % 32)
        return lalb_fail(ctx, LALB_ERR_UNSUPPORTED, "logic_layer_create: K must be a multiple of 32");
    if ((uintptr_t)codes & 15u)
        return lalb_fail(ctx, LALB_ERR_INVALID, "logic_layer_create: codes must be 16-byte aligned");
    *out = nullptr;
    LALB_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    lalb_logic_layer *L = new (std::nothrow) lalb_logic_layer();
    if (!L) return LALB_ERR_NOMEM;
    L->ctx = ctx;
    L->rows = rows;
    L->K = K;
    L->max_rows = max_rows;
    L->codes = codes;
    L->srow = srow;
    L->bias = bias;
    L->ws_bytes = lalb_logic_gemm_ws_bytes(rows, K, max_rows);
    if (cudaMalloc(&L->ws, L->ws_bytes) != cudaSuccess) {
        cudaGetLastError();
        L->ws = nullptr;
        free_logic(L);
        return lalb_fail(ctx, LALB_ERR_NOMEM, "logic_layer_create: device buffers");
    }
    *out = L;
    return LALB_OK;
}

extern "C" int lalb_logic_layer_forward(lalb_logic_layer *L, const float *X, int M, float *Y,
                                        lalb_stream stream) {
    if (!L) return LALB_ERR_INVALID;
    lalb_ctx *ctx = L->ctx;
    if (!X || !Y || M <= 0 || M > L->max_rows)
        return lalb_fail(ctx, LALB_ERR_INVALID, "logic_layer_forward: bad arguments (M <= %d)",
                         L->max_rows);
    return lalb_logic_gemm(ctx, L->codes, L->srow, L->bias, L->rows, L->K, X, M, L->ws, L->ws_bytes, Y,
                           (cudaStream_t)stream);
}

extern "C" int lalb_logic_layer_destroy(lalb_logic_layer *L) {
    if (!L) return LALB_ERR_INVALID;
    cudaSetDevice(L->ctx->device);
    free_logic(L);
    return LALB_OK;
}
