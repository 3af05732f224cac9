// lalb_q8_head.cu -- int8 x int8 LM-head matvec with fused argmax (sm_100a).
//
// logits[r] = sw[r] * sum_b sx[b] * isum_b(r), isum_b = exact int32 dot of
// the 32-byte block b of row r with the int8 activation block b.  The
// reference does this on the CPU with the "sign trick" (maddubs needs an
// unsigned operand, so |w| x sign(w)*x; README.md:131,285); dp4a multiplies
// signed bytes directly, and both give the same int32 because the row
// quantizer never emits -128.
//
// Structure: identical streaming skeleton to the Q4_K matvec (contiguous
// row range per CTA, 1-D bulk copies into a ring of shared stages, one
// mbarrier per stage, activation quantized in the prologue, one warp per
// row).  Lane l owns 32-byte blocks c = l, l+32, l+64, l+96 and keeps their
// activations in registers; it reads the two 16-byte halves of each block
// in an order that alternates every 4 lanes, so a warp's shared loads hit
// all 32 banks once per 128 bytes.  The exact block products sx*isum are
// summed in double, scaled by the row scale and rounded to fp32 once.
// Argmax: per-warp running best (first maximum wins because each warp walks
// rows in increasing order), a CTA reduction,
// one 64-bit atomicMax of (ordered logit, ~row) per CTA, and the last CTA to
// arrive (ticket counter) publishes the row index and resets the scratch
// for the next call.
#include <algorithm>
#include <mutex>

#include "lalb_internal.cuh"
#include "lalb_kernels.cuh"

using namespace lalb;

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kRps = 8;      // rows per stage, one per warp
constexpr int kMaxGpl = 4;   // 32-byte blocks per lane -> K <= 4096

struct Layout {
    uint32_t off_xq, off_sx, off_red, off_stage, stage_bytes, total;
};

__host__ __device__ inline uint32_t align_up(uint32_t v, uint32_t a) {
    return (v + a - 1) / a * a;
}

__host__ __device__ inline Layout make_layout(int K, int nstages) {
    Layout L;
    L.off_xq = 128;
    L.off_sx = align_up(L.off_xq + K, 16);
    L.off_red = align_up(L.off_sx + 4 * (K / 32), 16);
    L.off_stage = align_up(L.off_red + 2 * kWarps * 8 + 64, 128);
    L.stage_bytes = kRps * (uint32_t)K;
    L.total = L.off_stage + nstages * L.stage_bytes;
    return L;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

template <int IN>
__global__ void __launch_bounds__(kThreads, 1) q8_head_kernel(const Q8HeadArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int K = a.K, NB = K >> 5;
    const Layout L = make_layout(K, a.nstages);
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem);
    int8_t *xq_s = reinterpret_cast<int8_t *>(smem + L.off_xq);
    float *sx_s = reinterpret_cast<float *>(smem + L.off_sx);
    float *redf = reinterpret_cast<float *>(smem + L.off_red);
    int *redi = reinterpret_cast<int *>(smem + L.off_red + kWarps * 4);
    uint8_t *stage_s = smem + L.off_stage;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nrows = a.row_end - a.row_begin;
    const int q0 = (int)((long long)blockIdx.x * nrows / gridDim.x);
    const int q1 = (int)((long long)(blockIdx.x + 1) * nrows / gridDim.x);
    const int r0 = a.row_begin + q0, r1 = a.row_begin + q1;
    const int nst = (r1 - r0 + kRps - 1) / kRps;
    const int nstages = a.nstages;

    uint64_t policy = 0;
    auto issue = [&](int i) {
        const int rs = r0 + i * kRps;
        const int nr = min(kRps, r1 - rs);
        const uint32_t bytes = (uint32_t)nr * (uint32_t)K;
        const int buf = i % nstages;
        mbar_arrive_expect_tx(&bar[buf], bytes);
        bulk_g2s(stage_s + (size_t)buf * L.stage_bytes, a.W + (size_t)rs * K, bytes, &bar[buf],
                 policy);
    };
    if (tid == 0) {
        for (int s = 0; s < nstages; ++s) mbar_init(&bar[s], 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (tid == 0) {
        policy = l2_evict_first_policy();
        const int pre = min(nstages, nst);
        for (int i = 0; i < pre; ++i) issue(i);
    }
    pdl_wait();

    // ---- activation prologue ------------------------------------------------
    if (IN == kInQ8) {
        const int4 *src = reinterpret_cast<const int4 *>(a.xq);
        int4 *dst = reinterpret_cast<int4 *>(xq_s);
        for (int i = tid; i < K / 16; i += kThreads) dst[i] = src[i];
        for (int i = tid; i < NB; i += kThreads) sx_s[i] = a.sx[i];
    } else {
        float scale = 1.0f;
        if (IN == kInF32Rms) scale = block_rms_scale(a.x, K, a.eps);
        for (int blk = warp; blk < NB; blk += kWarps) {
            float v = a.x[blk * 32 + lane];
            if (IN == kInF32Rms) {
                v = __fmul_rn(v, scale);
                if (a.gamma) v = __fmul_rn(v, a.gamma[blk * 32 + lane]);
            }
            const uint32_t amax = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(v)));
            const float dsc = __fdiv_rn(__uint_as_float(amax), 127.0f);
            const float id = dsc != 0.0f ? __fdiv_rn(1.0f, dsc) : 0.0f;
            const float t = roundf(__fmul_rn(v, id));
            const int q = t > 127.0f ? 127 : (t < -127.0f ? -127 : (int)t);
            xq_s[blk * 32 + lane] = (int8_t)q;
            if (lane == 0) sx_s[blk] = dsc;
        }
    }
    __syncthreads();
    pdl_launch_dependents();

    // ---- per-lane activation registers ---------------------------------------
    const int h0 = (lane >> 2) & 1;  // which 16-byte half this lane reads first
    int xv[kMaxGpl][8];
    double sxv[kMaxGpl];
#pragma unroll
    for (int k = 0; k < kMaxGpl; ++k) {
        const int c = lane + 32 * k;
        if (c < NB) {
            const int4 lo = *reinterpret_cast<const int4 *>(xq_s + 32 * c);
            const int4 hi = *reinterpret_cast<const int4 *>(xq_s + 32 * c + 16);
            xv[k][0] = lo.x; xv[k][1] = lo.y; xv[k][2] = lo.z; xv[k][3] = lo.w;
            xv[k][4] = hi.x; xv[k][5] = hi.y; xv[k][6] = hi.z; xv[k][7] = hi.w;
            sxv[k] = (double)sx_s[c];
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) xv[k][j] = 0;
            sxv[k] = 0.0;
        }
    }

    float best_v = 0.0f;
    int best_r = -1;
    int issued = min(nstages, nst);
    for (int i = 0; i < nst; ++i) {
        const int buf = i % nstages;
        const bool ok = mbar_wait_bounded(&bar[buf], (uint32_t)(i / nstages) & 1u, a.status);
        const int row = r0 + i * kRps + warp;
        double acc = 0.0;
        if (ok && row < r1) {
            const uint8_t *rowp = stage_s + (size_t)buf * L.stage_bytes + (size_t)warp * K;
            int32_t *isum_row = a.isum ? a.isum + (size_t)(row - a.row_begin) * NB : nullptr;
#pragma unroll
            for (int k = 0; k < kMaxGpl; ++k) {
                const int c = lane + 32 * k;
                if (c < NB) {
                    const uint4 A = *reinterpret_cast<const uint4 *>(rowp + 32 * c + 16 * h0);
                    const uint4 B = *reinterpret_cast<const uint4 *>(rowp + 32 * c + 16 * (1 - h0));
                    const uint4 lo = h0 ? B : A, hi = h0 ? A : B;
                    int s = 0;
                    s = dp4a((int)lo.x, xv[k][0], s);
                    s = dp4a((int)lo.y, xv[k][1], s);
                    s = dp4a((int)lo.z, xv[k][2], s);
                    s = dp4a((int)lo.w, xv[k][3], s);
                    s = dp4a((int)hi.x, xv[k][4], s);
                    s = dp4a((int)hi.y, xv[k][5], s);
                    s = dp4a((int)hi.z, xv[k][6], s);
                    s = dp4a((int)hi.w, xv[k][7], s);
                    if (isum_row) isum_row[c] = s;
                    acc = fma(sxv[k], (double)s, acc);   // sx*isum is exact in fp64
                }
            }
        }
        acc = warp_sum_d(acc);
        if (row < r1 && ok) {
            const float v = (float)((double)a.sw[row] * acc);
            if (lane == 0 && a.logits) a.logits[row - a.row_begin] = v;
            if (best_r < 0 || v > best_v) {
                best_v = v;
                best_r = row;
            }
        }
        const bool stop = __syncthreads_or(!ok);
        if (stop) break;
        if (tid == 0 && issued < nst) {
            issue(issued);
            ++issued;
        }
    }
    if (tid == 0) {
        for (int i = max(0, issued - nstages); i < issued; ++i)
            mbar_wait_bounded(&bar[i % nstages], (uint32_t)(i / nstages) & 1u, a.status);
    }

    // ---- argmax: CTA reduction, then one atomic per CTA ------------------------
    if (!a.argmax) return;
    if (lane == 0) {
        redf[warp] = best_v;
        redi[warp] = best_r;
    }
    __syncthreads();
    if (tid == 0) {
        float bv = 0.0f;
        int br = -1;
        for (int w = 0; w < kWarps; ++w) {
            const int r = redi[w];
            if (r < 0) continue;
            const float v = redf[w];
            if (br < 0 || v > bv || (v == bv && r < br)) {
                bv = v;
                br = r;
            }
        }
        if (br >= 0) {
            const unsigned long long key = ((unsigned long long)ordered_key(bv) << 32) |
                                           (unsigned long long)(0xFFFFFFFFu - (uint32_t)br);
            atomicMax(a.best, key);
        }
        __threadfence();
        const unsigned int t = atomicAdd(a.ticket, 1u);
        if (t == gridDim.x - 1) {
            const unsigned long long key = atomicExch(a.best, 0ull);
            int32_t row = (int32_t)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull));
            if (a.fail_argmax) {
                // every CTA raised the status word (if it failed) before its
                // ticket: a row over a partial range is never published
                __threadfence();
                if (*(volatile unsigned int *)a.status) row = -1;
            }
            *a.argmax = row;
            atomicExch(a.ticket, 0u);
        }
    }
}

}  // namespace

int lalb_launch_q8_head(lalb_ctx *ctx, const Q8HeadArgs &args_in, int in, cudaStream_t stream,
                        bool pdl, int ctas_per_sm) {
    Q8HeadArgs a = args_in;
    if (!a.W || !a.sw || a.K <= 0 || a.K % 32 || a.row_begin < 0 || a.row_end < a.row_begin)
        return lalb_fail(ctx, LALB_ERR_INVALID, "lm head: bad arguments (K=%d range=[%d,%d))", a.K,
                         a.row_begin, a.row_end);
    if (a.K > 32 * 32 * kMaxGpl)
        return lalb_fail(ctx, LALB_ERR_UNSUPPORTED, "lm head: K=%d > %d", a.K, 32 * 32 * kMaxGpl);
    if (reinterpret_cast<uintptr_t>(a.W) & 15)
        return lalb_fail(ctx, LALB_ERR_INVALID, "lm head: rows must start 16-byte aligned");
    if (in == kInQ8 && (!a.xq || !a.sx || (reinterpret_cast<uintptr_t>(a.xq) & 15)))
        return lalb_fail(ctx, LALB_ERR_INVALID, "lm head: xq must be non-null and 16-byte aligned");
    if (in != kInQ8 && !a.x) return lalb_fail(ctx, LALB_ERR_INVALID, "lm head: null x");
    const int nrows = a.row_end - a.row_begin;
    if (nrows == 0) {
        if (a.argmax) LALB_CUDA_TRY(ctx, cudaMemsetAsync(a.argmax, 0xFF, sizeof(int32_t), stream));
        return LALB_OK;
    }
    const size_t budget = ctas_per_sm >= 2 ? 110 * 1024 : ctx->smem_optin - 1024;
    const Layout base = make_layout(a.K, 0);
    int nst = (int)((budget - base.off_stage) / base.stage_bytes);
    if (nst > 8) nst = 8;
    if (nst < 2) nst = 2;
    a.nstages = nst;
    a.status = &ctx->scratch->status;
    a.best = &ctx->scratch->best;
    a.ticket = &ctx->scratch->ticket;
    const Layout L = make_layout(a.K, nst);
    void *fn = in == kInQ8 ? (void *)q8_head_kernel<kInQ8>
               : in == kInF32Rms ? (void *)q8_head_kernel<kInF32Rms>
                                 : (void *)q8_head_kernel<kInF32>;
    {
        const int st = lalb_set_smem_attr(ctx, fn, (int)L.total);
        if (st) return st;
    }
    int resident = 0;
    LALB_CUDA_TRY(ctx, cudaOccupancyMaxActiveBlocksPerMultiprocessor(&resident, (const void *)fn,
                                                                     kThreads, L.total));
    if (resident < 1) return lalb_fail(ctx, LALB_ERR_UNSUPPORTED, "lm head: CTA does not fit");
    if (ctas_per_sm > resident) ctas_per_sm = resident;
    int grid = ctx->sm_count * ctas_per_sm;
    const int units = (nrows + kRps - 1) / kRps;
    if (grid > units) grid = units;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = L.total;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void *params[] = {&a};
    LALB_CUDA_TRY(ctx, cudaLaunchKernelExC(&cfg, fn, params));
    return LALB_OK;
}

extern "C" int lalb_lm_head_int8_range(lalb_ctx *ctx, const int8_t *W, const float *sw, int K,
                                       int row_begin, int row_end, const float *x,
                                       float *logits, int32_t *argmax, lalb_stream stream) {
    if (!ctx) return LALB_ERR_INVALID;
    Q8HeadArgs a = {};
    a.W = W;
    a.sw = sw;
    a.K = K;
    a.row_begin = row_begin;
    a.row_end = row_end;
    a.x = x;
    a.logits = logits;
    a.argmax = argmax;
    return lalb_launch_q8_head(ctx, a, kInF32, (cudaStream_t)stream, false, 1);
}

extern "C" int lalb_lm_head_int8_q8(lalb_ctx *ctx, const int8_t *W, const float *sw, int K,
                                    int row_begin, int row_end, const int8_t *xq,
                                    const float *sx, float *logits, int32_t *isum,
                                    int32_t *argmax, lalb_stream stream) {
    if (!ctx) return LALB_ERR_INVALID;
    Q8HeadArgs a = {};
    a.W = W;
    a.sw = sw;
    a.K = K;
    a.row_begin = row_begin;
    a.row_end = row_end;
    a.xq = xq;
    a.sx = sx;
    a.logits = logits;
    a.isum = isum;
    a.argmax = argmax;
    return lalb_launch_q8_head(ctx, a, kInQ8, (cudaStream_t)stream, false, 1);
}

// ---------------------------------------------------------------------------
// Allocation-free LM head.
//
// Some callers cannot call cudaMalloc: an engine whose own caching pool owns
// every byte of device memory and forbids libraries from allocating behind
// its back (cudaMalloc also stalls the whole device while it runs), or code
// that must not create a lalb_ctx because creating one allocates.  For them
// the argmax reduction state lives in the file-scope array below instead of
// a context's scratch.  It needs no context: device properties come from
// cudaDeviceGetAttribute, and errors are reported only through the status.
// ---------------------------------------------------------------------------
namespace {

// 256 bytes, held by every GPU that loads the library until the process
// exits.  A call uses the first 16: the packed best key (8 bytes), the CTA
// ticket (4) and the bounded-wait status word (4).  That need does not grow
// with the row count or K.
constexpr int kNoAllocScratchBytes = 256;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kNoAllocMaxDevices = 64;
struct NoAllocDevice {
    unsigned char *scratch;   // device address of g_noalloc_scratch on this device
    int sm_count;
    int smem_budget;          // dynamic shared memory one CTA may use
    bool ready;
};
NoAllocDevice g_noalloc_dev[kNoAllocMaxDevices];
std::mutex g_noalloc_mu;

// Once per device, with that device current: the array's device address (the
// host-side name g_noalloc_scratch is only a stand-in and must never reach a
// kernel), the SM count and the shared-memory budget of one CTA.
int noalloc_setup(int dev, NoAllocDevice **out) {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    NoAllocDevice &d = g_noalloc_dev[dev];
    if (!d.ready) {
        void *ptr = nullptr;
        if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || !ptr) {
            cudaGetLastError();
            return LALB_ERR_CUDA;
        }
        int sm = 0, optin = 0;
        if (cudaDeviceGetAttribute(&sm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) !=
                cudaSuccess) {
            cudaGetLastError();
            return LALB_ERR_CUDA;
        }
        const int budget = optin - 1024;
        d.scratch = static_cast<unsigned char *>(ptr);
        d.sm_count = sm;
        d.smem_budget = budget;
        d.ready = true;
    }
    *out = &d;
    return LALB_OK;
}

}  // namespace

extern "C" int lalb_lm_head_int8_range_noalloc(const int8_t *W, const float *sw, int K,
                                               int row_begin, int row_end, const float *x,
                                               float *logits, int32_t *argmax,
                                               lalb_stream stream) {
    if (!W || !sw || !x || K <= 0 || K % 32 || row_begin < 0 || row_end < row_begin)
        return LALB_ERR_INVALID;
    if (K > 32 * 32 * kMaxGpl) return LALB_ERR_UNSUPPORTED;  // the kernel's K limit (4096)
    if (reinterpret_cast<uintptr_t>(W) & 15) return LALB_ERR_INVALID;
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return LALB_ERR_CUDA;
    }
    if (dev < 0 || dev >= kNoAllocMaxDevices) return LALB_ERR_UNSUPPORTED;
    NoAllocDevice *nd = nullptr;
    if (int st = noalloc_setup(dev, &nd)) return st;
    cudaStream_t s = (cudaStream_t)stream;
    const int nrows = row_end - row_begin;
    if (nrows == 0) {
        if (argmax && cudaMemsetAsync(argmax, 0xFF, sizeof(int32_t), s) != cudaSuccess)
            return LALB_ERR_CUDA;
        return LALB_OK;
    }
    const Layout base = make_layout(K, 0);
    int nst = (int)((nd->smem_budget - (int)base.off_stage) / (int)base.stage_bytes);
    if (nst > 8) nst = 8;
    if (nst < 2) return LALB_ERR_UNSUPPORTED;
    const Layout L = make_layout(K, nst);
    // The kernel's shared-memory limit goes through the same raise-only
    // registry as the context-based launches, so a later regular call with a
    // smaller K cannot lower it below what this launch needs.
    if (lalb_raise_smem_attr(dev, (const void *)q8_head_kernel<kInF32>, (int)L.total) !=
        cudaSuccess) {
        cudaGetLastError();
        return LALB_ERR_CUDA;
    }

    // the array keeps the previous call's contents: clear the key, ticket and
    // status word that this call's reduction starts from
    if (cudaMemsetAsync(nd->scratch, 0, 16, s) != cudaSuccess) return LALB_ERR_CUDA;

    Q8HeadArgs a = {};
    a.W = W;
    a.sw = sw;
    a.K = K;
    a.row_begin = row_begin;
    a.row_end = row_end;
    a.x = x;
    a.logits = logits;
    a.argmax = argmax;
    a.nstages = nst;
    a.best = reinterpret_cast<unsigned long long *>(nd->scratch);
    a.ticket = reinterpret_cast<unsigned int *>(nd->scratch + 8);
    a.status = reinterpret_cast<unsigned int *>(nd->scratch + 12);
    a.fail_argmax = 1;   // a bounded wait that expired publishes argmax = -1
    int grid = nd->sm_count;
    const int units = (nrows + kRps - 1) / kRps;
    if (grid > units) grid = units;
    // the launch's own result (cudaGetLastError would also report, and
    // clear, an earlier error of unrelated code)
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = L.total;
    cfg.stream = s;
    void *params[] = {&a};
    if (cudaLaunchKernelExC(&cfg, (const void *)q8_head_kernel<kInF32>, params) != cudaSuccess)
        return LALB_ERR_CUDA;
    return LALB_OK;
}
