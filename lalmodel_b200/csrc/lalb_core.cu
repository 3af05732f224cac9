// lalb_core.cu -- context, error reporting, seeded fill and the quantizers.
//
// Quantizers reproduce the CPU restatement bit for bit: they use only IEEE
// single-precision +, -, *, / (explicit __f*_rn intrinsics, so nothing can
// be contracted into an FMA), rintf/roundf and the round-to-nearest-even
// fp32 -> fp16 conversion.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <utility>

#include "lalb_internal.cuh"

using namespace lalb;

// ---------------------------------------------------------------------------
// errors
// ---------------------------------------------------------------------------
int lalb_fail(lalb_ctx *ctx, int status, const char *fmt, ...) {
    if (ctx) {
        char buf[512];
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(buf, sizeof(buf), fmt, ap);
        va_end(ap);
        ctx->last_error = buf;
    }
    return status;
}

int lalb_cuda_fail(lalb_ctx *ctx, cudaError_t e, const char *what) {
    return lalb_fail(ctx, LALB_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e),
                     cudaGetErrorName(e));
}

// Raises a kernel's dynamic shared-memory limit, per (device, kernel), to the
// largest size any caller has asked for; it is never lowered, so a launch
// sized for an earlier, larger request stays valid.  Every path that sets
// the attribute goes through this registry (the context-based launchers and
// the allocation-free LM head alike).  Later launches with a size already
// covered (including those recorded during stream capture) skip the call.
cudaError_t lalb_raise_smem_attr(int device, const void *fn, int bytes) {
    static std::mutex mu;
    static std::map<std::pair<int, const void *>, int> done;
    std::lock_guard<std::mutex> lock(mu);
    auto key = std::make_pair(device, fn);
    auto it = done.find(key);
    if (it != done.end() && it->second >= bytes) return cudaSuccess;
    const cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) done[key] = bytes;
    return e;
}

int lalb_set_smem_attr(lalb_ctx *ctx, const void *fn, int bytes) {
    LALB_CUDA_TRY(ctx, lalb_raise_smem_attr(ctx->device, fn, bytes));
    return LALB_OK;
}

extern "C" int lalb_abi_version(void) { return LALB_ABI_VERSION; }

extern "C" const char *lalb_status_string(int s) {
    switch (s) {
        case LALB_OK: return "ok";
        case LALB_ERR_INVALID: return "invalid argument";
        case LALB_ERR_CUDA: return "CUDA error";
        case LALB_ERR_NOMEM: return "out of memory";
        case LALB_ERR_UNSUPPORTED: return "unsupported shape";
        case LALB_ERR_TIMEOUT: return "bounded device wait expired";
        case LALB_ERR_COMM: return "communicator error";
        case LALB_ERR_DEVICE: return "device is not sm_100";
        default: return "unknown status";
    }
}

extern "C" int lalb_init(int device, lalb_ctx **out) {
    if (!out) return LALB_ERR_INVALID;
    *out = nullptr;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) {
        cudaGetLastError();
        return LALB_ERR_DEVICE;
    }
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return LALB_ERR_CUDA;
    if (prop.major != 10 || prop.minor != 0) return LALB_ERR_DEVICE;
    if (cudaSetDevice(device) != cudaSuccess) return LALB_ERR_CUDA;
    lalb_ctx *ctx = new (std::nothrow) lalb_ctx();
    if (!ctx) return LALB_ERR_NOMEM;
    ctx->device = device;
    ctx->sm_count = prop.multiProcessorCount;
    ctx->smem_optin = prop.sharedMemPerBlockOptin;
    if (cudaMalloc(&ctx->scratch, sizeof(lalb_scratch)) != cudaSuccess) {
        delete ctx;
        return LALB_ERR_NOMEM;
    }
    if (cudaMemset(ctx->scratch, 0, sizeof(lalb_scratch)) != cudaSuccess ||
        cudaDeviceSynchronize() != cudaSuccess) {
        cudaFree(ctx->scratch);
        delete ctx;
        return LALB_ERR_CUDA;
    }
    *out = ctx;
    return LALB_OK;
}

extern "C" int lalb_destroy(lalb_ctx *ctx) {
    if (!ctx) return LALB_ERR_INVALID;
    cudaSetDevice(ctx->device);
    cudaFree(ctx->scratch);
    delete ctx;
    return LALB_OK;
}

extern "C" const char *lalb_last_error(const lalb_ctx *ctx) {
    return ctx ? ctx->last_error.c_str() : "null context";
}

extern "C" int lalb_device_status(lalb_ctx *ctx, int reset) {
    if (!ctx) return LALB_ERR_INVALID;
    LALB_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    LALB_CUDA_TRY(ctx, cudaDeviceSynchronize());
    unsigned int st = 0;
    LALB_CUDA_TRY(ctx, cudaMemcpy(&st, &ctx->scratch->status, sizeof(st), cudaMemcpyDeviceToHost));
    if (reset) LALB_CUDA_TRY(ctx, cudaMemset(&ctx->scratch->status, 0, sizeof(st)));
    return static_cast<int>(st);
}

extern "C" int lalb_unpack_scales_6bit(const uint8_t *s, uint8_t *out) {
    if (!s || !out) return LALB_ERR_INVALID;
    for (int j = 0; j < 4; j++) {
        out[j] = s[j] & 63;
        out[8 + j] = s[j + 4] & 63;
    }
    for (int j = 4; j < 8; j++) {
        out[j] = static_cast<uint8_t>((s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4));
        out[8 + j] = static_cast<uint8_t>((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
    }
    return LALB_OK;
}

// ---------------------------------------------------------------------------
// seeded normal fill
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// Box-Muller on two 24-bit uniforms of one SplitMix64 output, in single
// precision (the CPU restatement evaluates the same formula in double; the
// two agree to a few float ulps, which is all a synthetic draw needs).
__global__ void fill_normal_kernel(float *out, size_t n, uint64_t base, uint64_t offset,
                                   float sigma) {
    const float two_pi = 6.28318530717958647692f;
    for (size_t k = blockIdx.x * (size_t)blockDim.x + threadIdx.x; k < n;
         k += (size_t)gridDim.x * blockDim.x) {
        uint64_t u = mix64(base + offset + k);
        float u1 = (float)((u >> 40) + 1) * (1.0f / 16777216.0f);
        float u2 = (float)((u >> 16) & 0xFFFFFFu) * (1.0f / 16777216.0f);
        float z = sqrtf(-2.0f * logf(u1)) * cosf(two_pi * u2);
        out[k] = sigma * z;
    }
}

extern "C" int lalb_fill_normal(lalb_ctx *ctx, float *out, size_t n, uint64_t seed,
                                uint64_t offset, float sigma, lalb_stream stream) {
    if (!ctx) return LALB_ERR_INVALID;
    if (!out && n) return lalb_fail(ctx, LALB_ERR_INVALID, "fill_normal: null output");
    if (n == 0) return LALB_OK;
    int grid = ctx->sm_count * 8;
    fill_normal_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(out, n, seed * 0xD1B54A32D192ED03ull,
                                                               offset, sigma);
    LALB_LAUNCH_CHECK(ctx, "fill_normal_kernel");
    return LALB_OK;
}

// ---------------------------------------------------------------------------
// Q4_K min-max quantizer: one warp per 256-weight super-block.  Lane l owns
// weights [8l, 8l+8) (sub-block l/4).  Same arithmetic as the restatement:
//   scale_j = (max - min(0,min)) / 15, minv_j = -min(0,min)
//   d = fp16(max scale / 63), dmin = fp16(max minv / 63)
//   sc_j = min(63, rint(63/maxscale * scale_j)), m_j likewise
//   q = clamp(rint((x + dmin*m_j) / (d*sc_j)), 0, 15)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) q4k_quantize_kernel(const float *w, long long nblocks,
                                                           uint8_t *out) {
    const int lane = threadIdx.x & 31;
    const long long warp0 = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
    const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
    for (long long blk = warp0; blk < nblocks; blk += nwarps) {
        const float4 *src = reinterpret_cast<const float4 *>(w + blk * 256 + 8 * lane);
        float4 a = src[0], b = src[1];
        float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        float mn = v[0], mx = v[0];
#pragma unroll
        for (int i = 1; i < 8; i++) {
            mn = v[i] < mn ? v[i] : mn;
            mx = v[i] > mx ? v[i] : mx;
        }
        // reduce within the 4 lanes of the sub-block
#pragma unroll
        for (int o = 1; o < 4; o <<= 1) {
            float omn = __shfl_xor_sync(0xffffffffu, mn, o);
            float omx = __shfl_xor_sync(0xffffffffu, mx, o);
            mn = omn < mn ? omn : mn;
            mx = omx > mx ? omx : mx;
        }
        if (mn > 0.0f) mn = 0.0f;
        const float scale = __fdiv_rn(__fsub_rn(mx, mn), 15.0f);
        const float minv = -mn;
        // the maxima start from +0 as in the restatement (minv of an all-zero
        // sub-block is -0, which must not reach the fp16 dmin as 0x8000)
        float max_scale = scale > 0.0f ? scale : 0.0f;
        float max_min = minv > 0.0f ? minv : 0.0f;
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
            float os = __shfl_xor_sync(0xffffffffu, max_scale, o);
            float om = __shfl_xor_sync(0xffffffffu, max_min, o);
            max_scale = os > max_scale ? os : max_scale;
            max_min = om > max_min ? om : max_min;
        }
        const float inv_scale = max_scale > 0.0f ? __fdiv_rn(63.0f, max_scale) : 0.0f;
        const float inv_min = max_min > 0.0f ? __fdiv_rn(63.0f, max_min) : 0.0f;
        float ta = rintf(__fmul_rn(inv_scale, scale));
        float tb = rintf(__fmul_rn(inv_min, minv));
        const int ls = ta > 63.0f ? 63 : (int)ta;
        const int lm = tb > 63.0f ? 63 : (int)tb;
        const __half dh = __float2half_rn(__fdiv_rn(max_scale, 63.0f));
        const __half mh = __float2half_rn(__fdiv_rn(max_min, 63.0f));
        const float dj = __fmul_rn(__half2float(dh), (float)ls);
        const float dmj = __fmul_rn(__half2float(mh), (float)lm);
        uint32_t nib = 0;  // 8 nibbles, element i in bits 4i..4i+3
#pragma unroll
        for (int i = 0; i < 8; i++) {
            int l = 0;
            if (dj != 0.0f) {
                float t = rintf(__fdiv_rn(__fadd_rn(v[i], dmj), dj));
                l = t < 0.0f ? 0 : (t > 15.0f ? 15 : (int)t);
            }
            nib |= (uint32_t)l << (4 * i);
        }
        // gather ls/lm of the 8 sub-blocks (lanes 0,4,...,28)
        uint8_t *ob = out + blk * 144;
        uint32_t lsj[8], lmj[8];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            lsj[j] = (uint32_t)__shfl_sync(0xffffffffu, ls, 4 * j);
            lmj[j] = (uint32_t)__shfl_sync(0xffffffffu, lm, 4 * j);
        }
        if (lane == 0) {
            uint8_t s[12];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                s[j] = (uint8_t)lsj[j];
                s[j + 4] = (uint8_t)lmj[j];
            }
#pragma unroll
            for (int j = 4; j < 8; j++) {
                s[j + 4] = (uint8_t)((lsj[j] & 0x0F) | ((lmj[j] & 0x0F) << 4));
                s[j - 4] |= (uint8_t)((lsj[j] >> 4) << 6);
                s[j] |= (uint8_t)((lmj[j] >> 4) << 6);
            }
            uint32_t hdr[4];
            hdr[0] = (uint32_t)__half_as_ushort(dh) | ((uint32_t)__half_as_ushort(mh) << 16);
            memcpy(&hdr[1], s, 12);
            *reinterpret_cast<uint4 *>(ob) = make_uint4(hdr[0], hdr[1], hdr[2], hdr[3]);
        }
        // qs byte 32g + i = L[64g+i] | L[64g+32+i] << 4.  Lane l = 8g + a
        // (a < 4) holds L[64g + 8a .. +8]; lane 8g+4+a holds the high halves.
        const uint32_t hi = __shfl_down_sync(0xffffffffu, nib, 4);
        if ((lane & 7) < 4) {
            const int g = lane >> 3, a4 = lane & 3;
            uint32_t lo_w = 0, hi_w = 0;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                lo_w |= (((nib >> (4 * i)) & 0xFu) | (((hi >> (4 * i)) & 0xFu) << 4)) << (8 * i);
                hi_w |= (((nib >> (4 * (i + 4))) & 0xFu) | (((hi >> (4 * (i + 4))) & 0xFu) << 4))
                        << (8 * i);
            }
            *reinterpret_cast<uint2 *>(ob + 16 + 32 * g + 8 * a4) = make_uint2(lo_w, hi_w);
        }
    }
}

extern "C" int lalb_q4k_quantize(lalb_ctx *ctx, const float *w, int rows, int K, void *blocks,
                                 lalb_stream stream) {
    if (!ctx) return LALB_ERR_INVALID;
    if (!w || !blocks || rows < 0 || K <= 0 || K % LALB_QK_K)
        return lalb_fail(ctx, LALB_ERR_INVALID, "q4k_quantize: bad arguments (rows=%d K=%d)", rows, K);
    if ((reinterpret_cast<uintptr_t>(w) & 15) || (reinterpret_cast<uintptr_t>(blocks) & 15))
        return lalb_fail(ctx, LALB_ERR_INVALID, "q4k_quantize: pointers must be 16-byte aligned");
    long long nblocks = (long long)rows * (K / LALB_QK_K);
    if (nblocks == 0) return LALB_OK;
    long long want = (nblocks + 7) / 8;
    int grid = (int)(want < (long long)ctx->sm_count * 16 ? want : (long long)ctx->sm_count * 16);
    q4k_quantize_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(w, nblocks,
                                                                static_cast<uint8_t *>(blocks));
    LALB_LAUNCH_CHECK(ctx, "q4k_quantize_kernel");
    return LALB_OK;
}

// ---------------------------------------------------------------------------
// per-row int8 quantizer (LM head weights): one warp per row
// ---------------------------------------------------------------------------
__global__ void q8_quantize_rows_kernel(const float *w, int rows, int K, int8_t *q, float *s) {
    const int lane = threadIdx.x & 31;
    const int warp0 = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    for (int r = warp0; r < rows; r += nwarps) {
        const float *v = w + (size_t)r * K;
        uint32_t amax = 0;
        for (int i = lane; i < K; i += 32) amax = max(amax, __float_as_uint(fabsf(v[i])));
        amax = __reduce_max_sync(0xffffffffu, amax);
        const float d = __fdiv_rn(__uint_as_float(amax), 127.0f);
        const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        for (int i = lane; i < K; i += 32) {
            float t = roundf(__fmul_rn(v[i], id));
            q[(size_t)r * K + i] = (int8_t)(t > 127.0f ? 127 : (t < -127.0f ? -127 : (int)t));
        }
        if (lane == 0) s[r] = d;
    }
}

extern "C" int lalb_q8_quantize_rows(lalb_ctx *ctx, const float *w, int rows, int K, int8_t *q,
                                     float *s, lalb_stream stream) {
    if (!ctx) return LALB_ERR_INVALID;
    if (!w || !q || !s || rows < 0 || K <= 0)
        return lalb_fail(ctx, LALB_ERR_INVALID, "q8_quantize_rows: bad arguments");
    if (rows == 0) return LALB_OK;
    int grid = (rows + 7) / 8;
    if (grid > ctx->sm_count * 16) grid = ctx->sm_count * 16;
    q8_quantize_rows_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(w, rows, K, q, s);
    LALB_LAUNCH_CHECK(ctx, "q8_quantize_rows_kernel");
    return LALB_OK;
}

// ---------------------------------------------------------------------------
// activation quantizer: one warp per 32-block
// ---------------------------------------------------------------------------
__global__ void quantize_act_kernel(const float *x, long long nblk, int8_t *xq, float *sx,
                                    int32_t *sumq) {
    const int lane = threadIdx.x & 31;
    const long long warp0 = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
    const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
    for (long long b = warp0; b < nblk; b += nwarps) {
        const float v = x[b * 32 + lane];
        const uint32_t amax = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(v)));
        const float d = __fdiv_rn(__uint_as_float(amax), 127.0f);
        const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        const float t = roundf(__fmul_rn(v, id));
        const int q = t > 127.0f ? 127 : (t < -127.0f ? -127 : (int)t);
        xq[b * 32 + lane] = (int8_t)q;
        const int s = __reduce_add_sync(0xffffffffu, q);
        if (lane == 0) {
            sx[b] = d;
            if (sumq) sumq[b] = s;
        }
    }
}

extern "C" int lalb_quantize_act(lalb_ctx *ctx, const float *x, int M, int K, int8_t *xq,
                                 float *sx, int32_t *sumq, lalb_stream stream) {
    if (!ctx) return LALB_ERR_INVALID;
    if (!x || !xq || !sx || M < 0 || K <= 0 || K % LALB_QB)
        return lalb_fail(ctx, LALB_ERR_INVALID, "quantize_act: bad arguments (M=%d K=%d)", M, K);
    long long nblk = (long long)M * (K / LALB_QB);
    if (nblk == 0) return LALB_OK;
    long long want = (nblk + 7) / 8;
    int grid = (int)(want < (long long)ctx->sm_count * 16 ? want : (long long)ctx->sm_count * 16);
    quantize_act_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(x, nblk, xq, sx, sumq);
    LALB_LAUNCH_CHECK(ctx, "quantize_act_kernel");
    return LALB_OK;
}
