// lalb_internal.cuh -- shared device helpers and the context definition.
//
// Device-side building blocks for the sm_100a kernels: mbarrier + bulk-copy
// (TMA 1-D) PTX wrappers with bounded waits, programmatic-dependent-launch
// controls, int8 dot helpers and the Q4_K scale unpacking.
#pragma once

#include <initializer_list>

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "lalb.h"

// ---------------------------------------------------------------------------
// context
// ---------------------------------------------------------------------------
struct lalb_scratch {            // device-resident, owned by the context
    unsigned long long best;     // packed (ordered logit, ~row) argmax key
    unsigned int ticket;         // CTAs that finished the LM-head reduction
    unsigned int status;         // nonzero: a bounded wait expired
    unsigned int pad[12];
};

struct lalb_ctx {
    int device;
    int sm_count;
    size_t smem_optin;
    lalb_scratch *scratch;       // device
    std::string last_error;
};

// Records an error message on the context and returns the status code.
int lalb_fail(lalb_ctx *ctx, int status, const char *fmt, ...);
// Raises cudaFuncAttributeMaxDynamicSharedMemorySize of a kernel on `device`
// (the current device) to at least `bytes`; never lowers it.
cudaError_t lalb_raise_smem_attr(int device, const void *fn, int bytes);
// The same for the context's device, with the error recorded on the context.
int lalb_set_smem_attr(lalb_ctx *ctx, const void *fn, int bytes);
// Converts a CUDA error into LALB_ERR_CUDA with the call site recorded.
int lalb_cuda_fail(lalb_ctx *ctx, cudaError_t e, const char *what);

#define LALB_CUDA_TRY(ctx, call)                                           \
    do {                                                                   \
        cudaError_t e_ = (call);                                           \
        if (e_ != cudaSuccess) return lalb_cuda_fail((ctx), e_, #call);    \
    } while (0)

#define LALB_LAUNCH_CHECK(ctx, what)                                       \
    do {                                                                   \
        cudaError_t e_ = cudaGetLastError();                               \
        if (e_ != cudaSuccess) return lalb_cuda_fail((ctx), e_, (what));   \
    } while (0)

// status word bits
#define LALB_STATUS_WAIT_TIMEOUT 1u
#define LALB_STATUS_BAD_POSITION 2u   // a decode position outside the KV cache

// Bound on every wait: LALB_SPIN_LIMIT tries.  An mbarrier try_wait sleeps
// until the phase completes or LALB_WAIT_HINT_NS passes, so a wait that can
// never complete gives up after at most ~0.4 s, and a waiting warp does not
// spin on the issue slots that the working warps need.
#define LALB_SPIN_LIMIT (1u << 14)
#define LALB_WAIT_HINT_NS 25000u

namespace lalb {

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier --------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar,
                                                      uint32_t bytes) {
    asm volatile(
        "mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
            smem_u32(bar)),
        "r"(bytes)
        : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ uint32_t mbar_try_wait(uint64_t *bar,
                                                  uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(LALB_WAIT_HINT_NS)
        : "memory");
    return ok;
}

// Non-blocking test of an mbarrier phase.  A try_wait on a phase that has
// already completed still costs on the order of a hundred cycles; most waits
// of a streaming pipeline find their phase complete.
__device__ __forceinline__ uint32_t mbar_test_wait(uint64_t *bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done;
}

// Bounded wait on an mbarrier phase.  Returns false (and raises the status
// word) when the spin limit is reached.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar,
                                                  uint32_t parity,
                                                  unsigned int *status) {
    if (mbar_test_wait(bar, parity)) return true;
    for (uint32_t i = 0; i < LALB_SPIN_LIMIT; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    if (status) atomicOr(status, LALB_STATUS_WAIT_TIMEOUT);
    return false;
}

// ---- bulk copy (TMA, 1-D): global -> shared, completion on an mbarrier -----
// Both addresses 16-byte aligned, bytes a multiple of 16.  The L2 policy
// marks the streamed weights evict-first so they do not displace the small
// activation vectors that every CTA re-reads.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;"
                 : "=l"(pol));
    return pol;
}

__device__ __forceinline__ void bulk_g2s(void *smem_dst, const void *gsrc,
                                         uint32_t bytes, uint64_t *bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::"
        "cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(smem_dst)),
        "l"(gsrc), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// Same copy without an L2 policy (activations, which should stay cached).
__device__ __forceinline__ void bulk_g2s_plain(void *smem_dst, const void *gsrc,
                                               uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(smem_dst)),
        "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Bulk prefetch of global memory into L2 (no shared-memory destination, no
// completion): address and size 16-byte aligned.
__device__ __forceinline__ void bulk_prefetch_l2(const void *gsrc, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(gsrc), "r"(bytes) : "memory");
}

// ---- programmatic dependent launch -----------------------------------------
// wait: block until the preceding kernel in the stream has completed and its
// writes are visible (no-op when the launch had no programmatic dependency).
__device__ __forceinline__ void pdl_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
// allow the next kernel in the stream to be scheduled early.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Launch with programmatic dependent launch allowed (the kernels call
// pdl_wait before reading what the previous kernel wrote).
inline int launch_pdl(lalb_ctx *ctx, const void *fn, dim3 grid, dim3 block, size_t smem, cudaStream_t s,
               std::initializer_list<void *> args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    constexpr size_t kMaxParams = 16;
    if (args.size() > kMaxParams) return lalb_fail(ctx, LALB_ERR_INVALID, "launch_pdl: more than 16 parameters");
    void *params[kMaxParams];
    size_t i = 0;
    for (void *p : args) params[i++] = p;
    LALB_CUDA_TRY(ctx, cudaLaunchKernelExC(&cfg, fn, params));
    return LALB_OK;
}

// ---- misc ------------------------------------------------------------------
__device__ __forceinline__ int dp4a(int a, int b, int c) {
    return __dp4a(a, b, c);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float f16_bits_to_f32(uint32_t bits16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16)));
}

// Q4_K 6-bit scales of one super-block, from the 12 packed bytes held in
// three 32-bit words (bytes 0-3, 4-7, 8-11).  Produces four words of four
// bytes each: scales 0-3, scales 4-7, mins 0-3, mins 4-7.
struct ScaleWords {
    uint32_t sc_lo, sc_hi, mn_lo, mn_hi;
};
__device__ __forceinline__ ScaleWords unpack_scale_words(uint32_t s0,
                                                         uint32_t s1,
                                                         uint32_t s2) {
    ScaleWords r;
    r.sc_lo = s0 & 0x3F3F3F3Fu;
    r.mn_lo = s1 & 0x3F3F3F3Fu;
    r.sc_hi = (s2 & 0x0F0F0F0Fu) | ((s0 >> 2) & 0x30303030u);
    r.mn_hi = ((s2 >> 4) & 0x0F0F0F0Fu) | ((s1 >> 2) & 0x30303030u);
    return r;
}

// RMS normalisation factor 1/sqrt(mean(x^2) + eps) of a K-vector, for the
// whole CTA.  The sum of squares is accumulated in double (each square is
// exact there), so the float result does not depend on the summation order
// except in the rare case of a double-rounding tie.
__device__ __forceinline__ float block_rms_scale(const float *x, int K, float eps) {
    __shared__ double red[32];
    __shared__ float result;
    double ss = 0.0;
    for (int i = threadIdx.x; i < K; i += blockDim.x) {
        const double v = x[i];
        ss += v * v;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        double t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        if (threadIdx.x == 0) result = (float)(1.0 / sqrt(t / (double)K + (double)eps));
    }
    __syncthreads();
    return result;
}

// silu(g) * u evaluated in double and rounded once to float.
__device__ __forceinline__ float silu_mul(float g, float u) {
    const double gd = g;
    return (float)(gd / (1.0 + exp(-gd)) * (double)u);
}

// Monotone map float -> uint32 (larger float, larger key; -0 < +0).
__device__ __forceinline__ uint32_t ordered_key(float f) {
    uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

}  // namespace lalb
