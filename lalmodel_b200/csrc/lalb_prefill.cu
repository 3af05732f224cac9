// lalb_prefill.cu -- batched (prefill) Q4_K x Q8 matmul on tcgen05 int8 MMA.
//
//   Y[t][r] = sum_j sx[t][j] * (d_r sc_rj * isum[t][r][j] - dmin_r m_rj * sumq[t][j])
//
// the same arithmetic as lal_matmul_q4_k (README.md:130,210) for T tokens at
// once: isum[t][r][j] is the exact int32 dot of weight row r's sub-block j
// (32 unsigned 4-bit quants) with token t's int8 activations.  Each
// tcgen05.mma.kind::i8 instruction (M = 128 weight rows, N = 64 tokens,
// K = 32 = one sub-block) produces exactly those int32 sums for one
// sub-block into its own TMEM slot; the epilogue warps promote every slot
// into fp32 register accumulators with the sub-block's scales (fp32 combine,
// within 1e-5 of the exact dot).
//
// Layouts (prepared once: lalb_q4k_prefill_pack for the weights, per call
// for the activations):
//   weights   q  int8 [rows][K] (the 4-bit quants 0..15), rs fp32 [rows][K/32][2]
//             = {d * sc_j, dmin * m_j}
//   tokens    xq int8 [T][K], ts fp32 [K/32][T][2] = {sx_j, sx_j * sumq_j}
//
// One CTA per 128-row x 64-token tile, 10 warps:
//   warp 0     TMA producer: per 128-wide K-block, the 128 x 128 q tile and the
//              64 x 128 xq tile (128-byte swizzle) and their scale tiles into a
//              4-stage ring;
//   warp 1     allocates 512 TMEM columns (8 slots of 64) and issues the MMAs:
//              sub-block g into slot g % 8, one commit per slot;
//   warps 2-9  epilogue, two groups of four (tokens 0-31 and 32-63), each warp
//              on its TMEM lane quarter (32 weight rows): per sub-block, read
//              the slot (tcgen05.ld 32x32b.x32), free it, promote.
// A stage is free when its MMAs completed (commit) and all 8 epilogue warps
// have read its scales.  Every wait is bounded.
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "lalb_internal.cuh"
#include "lalb_prefill.cuh"

using namespace lalb;

namespace {

constexpr int PM = 128, PN = 64, PK = 128;   // PK int8 = 128 B: one swizzle row = 4 sub-blocks
constexpr int kPStages = 4;
constexpr int kSlotsT = 8;                   // TMEM accumulator slots (PN columns each)
constexpr int kEpiWarps = 8;
constexpr int kPThreads = 32 * (2 + kEpiWarps);
constexpr uint32_t kPA = PM * PK;            // 16 KB
constexpr uint32_t kPB = PN * PK;            // 8 KB
constexpr uint32_t kPRS = PM * 8 * 4;        // 4 KB: 128 rows x 4 sub-blocks x {dsc, dmm}
constexpr uint32_t kPTS = 4 * PN * 2 * 4;    // 2 KB: 4 sub-blocks x 64 tokens x {sx, a}
constexpr uint32_t kPStage = kPA + kPB + kPRS + kPTS;   // 30 KB (1024-multiple)
constexpr uint32_t kPSmem = 1024 + kPStages * kPStage + 512;

// kind::i8: s32 accumulator, signed A and B, both K-major, M = 128, N = 64.
constexpr uint32_t kIdescI8 = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(PN >> 3) << 17) |
                              ((uint32_t)(PM >> 4) << 24);

__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void tma2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc) {
    // every sub-block starts its own slot: no accumulation across sub-blocks
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, 0, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(kIdescI8)
        : "memory");
}

__device__ __forceinline__ void commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld32_i(uint32_t taddr, int (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
        "%28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
          "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
          "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

struct PfArgs {
    int rows, K, T;
    float *Y;               // [T][rows]
    unsigned int *status;
};

__global__ void __launch_bounds__(kPThreads, 1)
    prefill_i8_kernel(const __grid_constant__ CUtensorMap mQ, const __grid_constant__ CUtensorMap mX,
                      const __grid_constant__ CUtensorMap mRS, const __grid_constant__ CUtensorMap mTS,
                      const PfArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + kPStages * kPStage);
    uint64_t *empty = full + kPStages;
    uint64_t *sfull = empty + kPStages;       // TMEM slot holds a sub-block's sums
    uint64_t *sempty = sfull + kSlotsT;       // the epilogue has read the slot
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sempty + kSlotsT);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r0 = blockIdx.y * PM, t0 = blockIdx.x * PN;
    const int nkb = a.K / PK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kPStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1 + kEpiWarps);   // the MMA commit and every epilogue warp
        }
        for (int s = 0; s < kSlotsT; ++s) {
            mbar_init(&sfull[s], 1);
            mbar_init(&sempty[s], kEpiWarps);
        }
        fence_barrier_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(kSlotsT * PN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    }
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            for (int kb = 0; kb < nkb; ++kb) {
                const int s = kb % kPStages;
                const uint32_t use = kb / kPStages;
                if (use > 0 && !mbar_wait_bounded(&empty[s], (use - 1) & 1u, a.status)) break;
                uint8_t *st = smem + (size_t)s * kPStage;
                mbar_arrive_expect_tx(&full[s], kPStage);
                tma2d(st, &mQ, kb * PK, r0, &full[s]);
                tma2d(st + kPA, &mX, kb * PK, t0, &full[s]);
                tma2d(st + kPA + kPB, &mRS, kb * 8, r0, &full[s]);
                tma2d(st + kPA + kPB + kPRS, &mTS, t0 * 2, kb * 4, &full[s]);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            for (int kb = 0; kb < nkb; ++kb) {
                const int s = kb % kPStages;
                if (!mbar_wait_bounded(&full[s], (uint32_t)(kb / kPStages) & 1u, a.status)) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t st = smem_u32(smem + (size_t)s * kPStage);
                bool ok = true;
#pragma unroll
                for (int j = 0; j < 4; ++j) {   // one sub-block (32 bytes of K) per instruction
                    const uint32_t g = kb * 4 + j;
                    const uint32_t slot = g % kSlotsT, use = g / kSlotsT;
                    if (use > 0 && !mbar_wait_bounded(&sempty[slot], (use - 1) & 1u, a.status)) {
                        ok = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    mma_i8(tmem + slot * PN, sw128_desc(st + j * 32), sw128_desc(st + kPA + j * 32));
                    commit(&sfull[slot]);
                }
                commit(&empty[s]);   // the stage's A/B tiles are read once these MMAs complete
                if (!ok) break;
            }
        }
    } else {
        // ---- epilogue: warp -> TMEM lane quarter (weight rows), group -> tokens ----
        const int ew = warp - 2;
        const int q = warp & 3;              // lane quarter
        const int grp = ew >> 2;             // tokens 32*grp .. 32*grp + 31
        const int row = q * 32 + lane;       // weight row within the tile
        float acc[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] = 0.0f;
        bool ok = true;
        for (int kb = 0; kb < nkb && ok; ++kb) {
            const int s = kb % kPStages;
            const uint8_t *st = smem + (size_t)s * kPStage;
            const float *rs = reinterpret_cast<const float *>(st + kPA + kPB);         // [128][8]
            const float *ts = reinterpret_cast<const float *>(st + kPA + kPB + kPRS);  // [4][64][2]
            // the scale tiles came in with the stage's TMA copies
            if (!mbar_wait_bounded(&full[s], (uint32_t)(kb / kPStages) & 1u, a.status)) break;
            for (int j = 0; j < 4; ++j) {
                const uint32_t g = kb * 4 + j;
                const uint32_t slot = g % kSlotsT;
                if (!mbar_wait_bounded(&sfull[slot], (g / kSlotsT) & 1u, a.status)) {
                    ok = false;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                int isum[32];
                tmem_ld32_i(tmem + ((uint32_t)(q * 32) << 16) + slot * PN + grp * 32, isum);
                asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(&sempty[slot]);
                const float dsc = rs[row * 8 + 2 * j], dmm = rs[row * 8 + 2 * j + 1];
                const float *tj = ts + (j * PN + grp * 32) * 2;
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const float sx = tj[2 * i], am = tj[2 * i + 1];
                    acc[i] = fmaf(sx * dsc, (float)isum[i], acc[i]);
                    acc[i] = fmaf(-am, dmm, acc[i]);
                }
            }
            // this warp is done with the stage's scales (its MMAs completed:
            // their sums were read above)
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        // rows are the fast dimension of Y: lane = row gives 128-byte stores
        const int r = r0 + row;
        if (r < a.rows)
            for (int i = 0; i < 32; ++i) {
                const int t = t0 + grp * 32 + i;
                if (t < a.T) a.Y[(size_t)t * a.rows + r] = acc[i];
            }
    }
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(kSlotsT * PN)
                     : "memory");
    }
}

// Q4_K rows -> int8 quants and per-(row, sub-block) {d*sc, dmin*m}: one
// warp per 256-weight super-block.
__global__ void prefill_pack_kernel(const uint8_t *__restrict__ W, long long nsb, int8_t *__restrict__ q,
                                    float *__restrict__ rs) {
    const int lane = threadIdx.x & 31;
    const long long w0 = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
    const long long nw = ((long long)gridDim.x * blockDim.x) >> 5;
    for (long long b = w0; b < nsb; b += nw) {
        const uint8_t *blk = W + b * 144;
        // lane handles quant bytes 4*lane .. 4*lane+3 of the 128: group g = lane / 8
        const uint32_t qs = *reinterpret_cast<const uint32_t *>(blk + 16 + 4 * lane);
        const int g = lane >> 3, off = (lane & 7) * 4;
        // low nibbles -> sub-block 2g, high nibbles -> sub-block 2g+1
        const uint32_t lo = qs & 0x0F0F0F0Fu, hi = (qs >> 4) & 0x0F0F0F0Fu;
        *reinterpret_cast<uint32_t *>(q + b * 256 + (2 * g) * 32 + off) = lo;
        *reinterpret_cast<uint32_t *>(q + b * 256 + (2 * g + 1) * 32 + off) = hi;
        if (lane < 8) {
            const uint32_t s0 = *reinterpret_cast<const uint32_t *>(blk + 4);
            const uint32_t s1 = *reinterpret_cast<const uint32_t *>(blk + 8);
            const uint32_t s2 = *reinterpret_cast<const uint32_t *>(blk + 12);
            const ScaleWords sw = unpack_scale_words(s0, s1, s2);
            const uint32_t scw = lane < 4 ? sw.sc_lo : sw.sc_hi, mnw = lane < 4 ? sw.mn_lo : sw.mn_hi;
            const int sc = (scw >> (8 * (lane & 3))) & 0xFF, mn = (mnw >> (8 * (lane & 3))) & 0xFF;
            const uint32_t dd = *reinterpret_cast<const uint32_t *>(blk);
            const float d = f16_bits_to_f32(dd & 0xFFFFu), dmin = f16_bits_to_f32(dd >> 16);
            rs[(b * 8 + lane) * 2] = __fmul_rn(d, (float)sc);
            rs[(b * 8 + lane) * 2 + 1] = __fmul_rn(dmin, (float)mn);
        }
    }
}

// Tokens: fp32 [T][K] -> xq int8 [T][K] and ts [K/32][Tp][2] = {sx, sx * sumq}
// (Tp = T rounded up to the token tile)
// (the activation quantizer of quantize_act_kernel, one warp per 32-block).
__global__ void prefill_act_kernel(const float *__restrict__ X, int T, int Tp, int K,
                                   int8_t *__restrict__ xq, float *__restrict__ ts) {
    const int lane = threadIdx.x & 31;
    const int nb = K / 32;
    const long long nblk = (long long)T * nb;
    const long long w0 = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
    const long long nw = ((long long)gridDim.x * blockDim.x) >> 5;
    for (long long b = w0; b < nblk; b += nw) {
        const long long t = b / nb, j = b % nb;
        const float v = X[b * 32 + lane];
        const uint32_t amax = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(v)));
        const float d = __fdiv_rn(__uint_as_float(amax), 127.0f);
        const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        const float tq = roundf(__fmul_rn(v, id));
        const int qv = tq > 127.0f ? 127 : (tq < -127.0f ? -127 : (int)tq);
        xq[b * 32 + lane] = (int8_t)qv;
        const int s = __reduce_add_sync(0xffffffffu, qv);
        if (lane == 0) {
            ts[(j * Tp + t) * 2] = d;
            ts[(j * Tp + t) * 2 + 1] = __fmul_rn(d, (float)s);
        }
    }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
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

// 2-D row-major map: dims {inner, outer}, box {bi, bo}; outer rows past the
// end (and inner columns past the end) read as zeros.
int map2d(lalb_ctx *ctx, CUtensorMap *m, const void *base, CUtensorMapDataType dt, int esize,
          long long inner, long long outer, int bi, int bo, CUtensorMapSwizzle sw) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return lalb_fail(ctx, LALB_ERR_CUDA, "prefill: cuTensorMapEncodeTiled unavailable");
    const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
    const cuuint64_t strides[1] = {(cuuint64_t)inner * esize};
    const cuuint32_t box[2] = {(cuuint32_t)bi, (cuuint32_t)bo};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(m, dt, 2, const_cast<void *>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return lalb_fail(ctx, LALB_ERR_CUDA, "prefill: tensor map encode (%d)", (int)r);
    return LALB_OK;
}

}  // namespace

size_t lalb_prefill_weight_bytes(int rows, int K) {
    return (size_t)rows * K + (size_t)rows * (K / 32) * 2 * sizeof(float);
}

static int tokens_padded(int T) { return (T + PN - 1) / PN * PN; }

size_t lalb_prefill_act_bytes(int T, int K) {
    return (size_t)T * K + 256 + (size_t)tokens_padded(T) * (K / 32) * 2 * sizeof(float);
}

int lalb_prefill_pack(lalb_ctx *ctx, const void *W, int rows, int K, void *packed, cudaStream_t s) {
    int8_t *q = static_cast<int8_t *>(packed);
    float *rs = reinterpret_cast<float *>(q + (size_t)rows * K);
    const long long nsb = (long long)rows * (K / 256);
    const int blocks = (int)std::min<long long>((nsb * 32 + 255) / 256, (long long)ctx->sm_count * 16);
    prefill_pack_kernel<<<blocks, 256, 0, s>>>(static_cast<const uint8_t *>(W), nsb, q, rs);
    LALB_LAUNCH_CHECK(ctx, "prefill_pack_kernel");
    return LALB_OK;
}

int lalb_prefill_matmul(lalb_ctx *ctx, const void *packed, int rows, int K, const float *X, int T,
                        void *ws, float *Y, cudaStream_t s) {
    const int8_t *q = static_cast<const int8_t *>(packed);
    const float *rs = reinterpret_cast<const float *>(q + (size_t)rows * K);
    int8_t *xq = static_cast<int8_t *>(ws);
    float *ts = reinterpret_cast<float *>(
        (reinterpret_cast<uintptr_t>(xq + (size_t)T * K) + 255) & ~(uintptr_t)255);
    {
        const long long nblk = (long long)T * (K / 32);
        const int blocks = (int)std::min<long long>((nblk * 32 + 255) / 256, (long long)ctx->sm_count * 16);
        prefill_act_kernel<<<blocks, 256, 0, s>>>(X, T, tokens_padded(T), K, xq, ts);
        LALB_LAUNCH_CHECK(ctx, "prefill_act_kernel");
    }
    CUtensorMap mQ, mX, mRS, mTS;
    int st;
    if ((st = map2d(ctx, &mQ, q, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, rows, PK, PM,
                    CU_TENSOR_MAP_SWIZZLE_128B)))
        return st;
    if ((st = map2d(ctx, &mX, xq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, T, PK, PN,
                    CU_TENSOR_MAP_SWIZZLE_128B)))
        return st;
    if ((st = map2d(ctx, &mRS, rs, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (long long)(K / 32) * 2, rows, 8,
                    PM, CU_TENSOR_MAP_SWIZZLE_NONE)))
        return st;
    if ((st = map2d(ctx, &mTS, ts, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (long long)tokens_padded(T) * 2,
                    K / 32, 2 * PN, 4, CU_TENSOR_MAP_SWIZZLE_NONE)))
        return st;
    if ((st = lalb_set_smem_attr(ctx, (const void *)prefill_i8_kernel, (int)kPSmem))) return st;
    PfArgs a;
    a.rows = rows;
    a.K = K;
    a.T = T;
    a.Y = Y;
    a.status = &ctx->scratch->status;
    const dim3 grid((T + PN - 1) / PN, (rows + PM - 1) / PM);
    prefill_i8_kernel<<<grid, kPThreads, kPSmem, s>>>(mQ, mX, mRS, mTS, a);
    LALB_LAUNCH_CHECK(ctx, "prefill_i8_kernel");
    return LALB_OK;
}

// ---- C ABI -------------------------------------------------------------------
extern "C" int lalb_prefill_sizes(int rows, int K, int T, size_t *weight_bytes, size_t *ws_bytes) {
    if (rows <= 0 || K <= 0 || K % 256 || T <= 0 || !weight_bytes || !ws_bytes) return LALB_ERR_INVALID;
    *weight_bytes = lalb_prefill_weight_bytes(rows, K);
    *ws_bytes = lalb_prefill_act_bytes(T, K);
    return LALB_OK;
}

extern "C" int lalb_q4k_prefill_pack(lalb_ctx *ctx, const void *W, int rows, int K, void *packed,
                                     lalb_stream stream) {
    if (!ctx) return LALB_ERR_INVALID;
    if (!W || !packed || rows <= 0 || K <= 0 || K % 256)
        return lalb_fail(ctx, LALB_ERR_INVALID, "q4k_prefill_pack: K a multiple of 256, non-null buffers");
    if (((uintptr_t)W & 3u) || ((uintptr_t)packed & 255u))
        return lalb_fail(ctx, LALB_ERR_INVALID, "q4k_prefill_pack: W 4-byte, packed 256-byte aligned");
    return lalb_prefill_pack(ctx, W, rows, K, packed, (cudaStream_t)stream);
}

extern "C" int lalb_matmul_q4_k_prefill(lalb_ctx *ctx, const void *packed, int rows, int K,
                                        const float *X, int T, void *ws, float *Y, lalb_stream stream) {
    if (!ctx) return LALB_ERR_INVALID;
    if (!packed || !X || !ws || !Y || rows <= 0 || K <= 0 || K % 256 || T <= 0)
        return lalb_fail(ctx, LALB_ERR_INVALID, "matmul_q4_k_prefill: bad arguments");
    if (((uintptr_t)packed | (uintptr_t)ws) & 255u || ((uintptr_t)X & 15u) || ((uintptr_t)Y & 3u))
        return lalb_fail(ctx, LALB_ERR_INVALID, "matmul_q4_k_prefill: misaligned buffer");
    return lalb_prefill_matmul(ctx, packed, rows, K, X, T, ws, Y, (cudaStream_t)stream);
}
