// lalb_tcgen05.cuh -- tcgen05 / TMA building blocks shared by the tensor-core
// kernels that decode their weight operand into TMEM (lalb_prefill.cu,
// lalb_logic_gemm.cu): shared-memory matrix descriptors, 2-D tiled TMA loads,
// TMEM loads and stores, MMAs with A in TMEM issued from one elected lane of a
// converged warp, and the host-side tensor-map encoder.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>

#include <mutex>

#include "lalb_internal.cuh"

namespace lalb {

// K-major, 128-byte swizzle (one 64-element fp16 K-block per row): 8-row atoms of 1 KB.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// K-major, 32-byte swizzle (one 16-element bf16 K-step per row): 8-row atoms of 256 B.
__device__ __forceinline__ uint64_t sw32_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(256 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)6 << 61);
}

// 2-D tiled TMA load into this CTA's shared memory, completion on `bar`.
__device__ __forceinline__ void tma2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 16 columns of the warp's 32 TMEM lanes into registers (lane i, column + j -> r[j]).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15}, [%16];"
        : "=f"(r[0]), "=f"(r[1]), "=f"(r[2]), "=f"(r[3]), "=f"(r[4]), "=f"(r[5]), "=f"(r[6]),
          "=f"(r[7]), "=f"(r[8]), "=f"(r[9]), "=f"(r[10]), "=f"(r[11]), "=f"(r[12]), "=f"(r[13]),
          "=f"(r[14]), "=f"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 8 (32) columns of the warp's 32 TMEM lanes: register j of lane i -> (lane i, column + j)
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
        : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
        "%13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(
            taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
        "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
        "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

// D (TMEM) += A (TMEM) x B (shared memory descriptor), issued by one elected
// lane of a converged warp: the whole warp runs the issue loop, so the
// operands are warp-uniform values.
__device__ __forceinline__ void mma_f16_ta(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// tcgen05.commit from one elected lane of a converged warp: `bar` gets one
// arrival once every MMA the thread issued before has completed.
__device__ __forceinline__ void commit_elect(uint64_t *bar) {
    asm volatile(
        "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(
            smem_u32(bar))
        : "memory");
}

// A bounded wait by every lane of a warp, which goes on only when all of them
// saw the phase complete: the .sync.aligned tcgen05 instructions and the
// __syncwarp calls after it need the whole warp on the same path, the
// timeout path included.
__device__ __forceinline__ bool warp_wait_fast(uint64_t *bar, uint32_t parity, unsigned int *status) {
    return __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity, status));
}

// ---- host: 2-D tensor maps -------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult qr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qr) == cudaSuccess &&
            qr == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// 2-D row-major map: dims {inner, outer} in elements of esize bytes, box
// {bi, bo}; rows and columns past the end read as zeros.
inline int map2d(lalb_ctx *ctx, CUtensorMap *m, const void *base, CUtensorMapDataType dt, int esize,
                 long long inner, long long outer, int bi, int bo, CUtensorMapSwizzle sw) {
    EncodeTiledFn fn = encode_tiled_fn();
    if (!fn) return lalb_fail(ctx, LALB_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
    const cuuint64_t strides[1] = {(cuuint64_t)inner * esize};
    const cuuint32_t box[2] = {(cuuint32_t)bi, (cuuint32_t)bo};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(m, dt, 2, const_cast<void *>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return lalb_fail(ctx, LALB_ERR_CUDA, "tensor map encode (%d)", (int)r);
    return LALB_OK;
}

}  // namespace lalb
