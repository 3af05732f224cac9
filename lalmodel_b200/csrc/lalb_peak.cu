// lalb_peak.cu -- measured tensor-core throughput: back-to-back tcgen05.mma on
// every SM, the denominators of the prefill kernel's tensor fractions.
//
// One CTA per SM (shared memory sized so no two fit), one warp issuing from an
// elected lane; each K-block is four M = 128, N = 256 MMAs (K = 16 for
// kind::f16, K = 32 for kind::i8) from zeroed 128-byte-swizzled shared-memory
// tiles into one TMEM accumulator.  The issuing thread runs ahead until the
// tensor pipe's queue pushes back, so the time is the pipe's: the result is the
// dense MMA rate at the clock the GPU holds under this load.
#include <cuda_runtime.h>

#include "lalb_internal.cuh"

using namespace lalb;

namespace {

constexpr int kPkSmem = 120 * 1024;   // one CTA per SM: the kernel takes all 512 TMEM columns
constexpr uint32_t kPkM = 128, kPkN = 256;
// f32 accumulator, fp16 A and B, K-major
constexpr uint32_t kIdescPkF16 = (1u << 4) | ((kPkN >> 3) << 17) | ((kPkM >> 4) << 24);
// s32 accumulator, signed 8-bit A and B, K-major
constexpr uint32_t kIdescPkI8 = (2u << 4) | (1u << 7) | (1u << 10) | ((kPkN >> 3) << 17) | ((kPkM >> 4) << 24);

__device__ __forceinline__ uint64_t pk_sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

template <int KIND>
__global__ void __launch_bounds__(128, 1) mma_peak_kernel(int iters, unsigned int *status) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *sm = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    __shared__ uint64_t done;
    __shared__ uint32_t tslot;
    for (int i = threadIdx.x; i < 48 * 1024 / 16; i += blockDim.x)   // A 16 KB, B 32 KB
        reinterpret_cast<uint4 *>(sm)[i] = make_uint4(0, 0, 0, 0);
    const int warp = threadIdx.x >> 5;
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(&tslot))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (threadIdx.x == 0) {
        mbar_init(&done, 1);
        fence_barrier_init();
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // the zeroed tiles, for the MMAs
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tslot;
    if (warp == 0) {
        const uint32_t a = smem_u32(sm), b = a + 16384;
        for (int it = 0; it < iters; ++it) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const uint64_t ad = pk_sw128_desc(a + kk * 32), bd = pk_sw128_desc(b + kk * 32);
                if (KIND == LALB_MMA_I8)
                    asm volatile(
                        "{\n\t.reg .pred e, p;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
                        "l"(ad), "l"(bd), "r"(kIdescPkI8), "r"(it | kk)
                        : "memory");
                else
                    asm volatile(
                        "{\n\t.reg .pred e, p;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
                        "l"(ad), "l"(bd), "r"(kIdescPkF16), "r"(it | kk)
                        : "memory");
            }
        }
        asm volatile(
            "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
            "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(
                smem_u32(&done))
            : "memory");
        // a wait that runs out raised the status word; one more bounded wait
        // gives the MMAs in flight their time before the columns are freed
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(&done, 0, status)))
            (void)__all_sync(0xffffffffu, mbar_wait_bounded(&done, 0, nullptr));
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
    }
}

}  // namespace

extern "C" int lalb_measure_mma_peak(lalb_ctx *ctx, int kind, double *tera_ops) {
    if (!ctx) return LALB_ERR_INVALID;
    if (!tera_ops || (kind != LALB_MMA_F16 && kind != LALB_MMA_I8))
        return lalb_fail(ctx, LALB_ERR_INVALID, "measure_mma_peak: kind LALB_MMA_F16 or LALB_MMA_I8");
    const void *fn = kind == LALB_MMA_I8 ? (const void *)mma_peak_kernel<LALB_MMA_I8>
                                         : (const void *)mma_peak_kernel<LALB_MMA_F16>;
    int st;
    if ((st = lalb_set_smem_attr(ctx, fn, kPkSmem))) return st;
    cudaStream_t s;
    LALB_CUDA_TRY(ctx, cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    const int iters = 20000;   // 80000 MMAs per SM: a few milliseconds
    unsigned int *status = &ctx->scratch->status;
    int err = 0;
    auto launch = [&](int n) {
        void *args[] = {(void *)&n, (void *)&status};
        return cudaLaunchKernel(fn, dim3(ctx->sm_count), dim3(128), args, kPkSmem, s);
    };
    float ms = 0.0f;
    if (launch(iters / 10) != cudaSuccess || cudaEventRecord(e0, s) != cudaSuccess || launch(iters) != cudaSuccess ||
        cudaEventRecord(e1, s) != cudaSuccess || cudaStreamSynchronize(s) != cudaSuccess ||
        cudaEventElapsedTime(&ms, e0, e1) != cudaSuccess)
        err = 1;
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaStreamDestroy(s);
    if (err) return lalb_fail(ctx, LALB_ERR_CUDA, "measure_mma_peak: %s", cudaGetErrorString(cudaGetLastError()));
    const double k_per_mma = kind == LALB_MMA_I8 ? 32.0 : 16.0;
    const double ops = 2.0 * kPkM * kPkN * k_per_mma * 4.0 * iters * ctx->sm_count;
    *tera_ops = ops / (ms * 1e-3) / 1e12;
    return LALB_OK;
}
