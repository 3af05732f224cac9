// lalb_prefill.cu -- batched (prefill) Q4_K x Q8 matmul on the tcgen05 tensor cores.
//
//   Y[t][r] = sum_j sx[t][j] * (d_r sc_rj * isum[t][r][j] - dmin_r m_rj * sumq[t][j])
//
// the arithmetic of lal_matmul_q4_k (README.md:130,210) for T tokens at once:
// isum[t][r][j] is the integer dot of weight row r's sub-block j (32 unsigned
// 4-bit quants) with token t's int8 activations xq, sumq[t][j] the sum of
// those activations, sx[t][j] their block scale.
//
// Rewritten per 256-weight super-block b (one d_r, dmin_r; sub-blocks j in b),
// with D = d (1 where d = 0: every sc, and so every A below, is then 0):
//
//   Y[t][r] = sum_b D_rb * S_b[t][r],
//   S_b[t][r] = sum_{i in b} (sc_rj q_ri) (xq_ti sx_tj) + sum_{j in b} c_rj a_tj,
//   c_rj = -dmin_rb m_rj / D_rb,   a_tj = sx_tj sumq_tj.
//
// S_b is one fp32 tensor-core accumulation in a TMEM slot:
//   sc * q            fp16, exact (integers <= 63 * 15 = 945);
//   xq * sx * 2^e_t   two fp16 parts (hi + lo, 22 significant bits), e_t a
//                     per-token power of two that puts the token's largest
//                     |xq sx| in [2^14, 2^15) (exact to apply and to undo);
//   c and a * 2^e_t   three bf16 parts each (24 bits, fp32 range); the six
//                     part products with weight >= 2^-16 of the whole, as one
//                     16-wide bf16 MMA per two sub-blocks;
// per 64 weights: 8 kind::f16 MMAs (4 K-steps x {B_hi, B_lo}) and one bf16 MMA
// for the two sub-blocks' min terms.  The epilogue only adds D * S_b (paired
// __ffma2_rn) and undoes 2^e_t.  Within 1e-5 of the exact dot.
//
// Layouts (the weights prepared once by lalb_q4k_prefill_pack, the tokens per
// call):
//   weights  A    fp16 [rows][K] = sc_j * q
//            Ax   bf16 [rows][K/4]: per 64 weights 16 values, for their two
//                 sub-blocks {c0 c0 c1 c0 c1 c2} each, then 4 zeros
//            rs   fp32 [K/256][rows128] = D
//   tokens   Bhi, Blo  fp16 [T][K]
//            Bx   bf16 [T][K/4]: per 64 weights, for their two sub-blocks
//                 {a0 a1 a0 a2 a1 a0} (parts of a 2^e_t) each, then 4 zeros
//            inv  fp32 [Tp] = 2^-e_t   (Tp = T rounded up to 128)
//
// One CTA per 128-row x 128-token tile, 18 warps:
//   warp 0     TMA producer: per 64-wide K-block the A, B_hi, B_lo (128-byte
//              swizzle), Ax and Bx (32-byte swizzle) tiles into a 4-stage
//              ring; per super-block the rows' D into a 2-slot ring;
//   warp 1     allocates 512 TMEM columns (4 super-block slots of 128) and
//              issues the MMAs, one commit per stage and one per super-block;
//   warps 2-17 epilogue, four groups of four (32 tokens each), each warp on its
//              TMEM lane quarter (32 weight rows): per super-block, read the
//              slot (tcgen05.ld 32x32b.x16 twice), free it, acc += D * S.
// Every wait is bounded.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <mutex>

#include "lalb_internal.cuh"
#include "lalb_prefill.cuh"

using namespace lalb;

namespace {

constexpr int PM = 128, PN = 128, PK = 64;   // PK fp16 = 128 B: one swizzle row
constexpr int kPStages = 4;
constexpr int kSlotsT = 2;                   // TMEM super-block slots
constexpr int kSlotW = 2 * PN;               // a slot: B_hi products (PN columns), then B_lo's
constexpr int kTmemCols = kSlotsT * kSlotW;
constexpr int kEpiWarps = 16;
constexpr int kPThreads = 32 * (2 + kEpiWarps);
constexpr uint32_t kPA = PM * PK * 2;        // 16 KB
constexpr uint32_t kPB = PN * PK * 2;        // 16 KB (each of B_hi, B_lo)
constexpr uint32_t kPAX = PM * 16 * 2;       // 4 KB: 128 rows x 16 bf16
constexpr uint32_t kPBX = PN * 16 * 2;       // 4 KB
constexpr uint32_t kOffBh = kPA, kOffBl = kPA + kPB, kOffAx = kPA + 2 * kPB, kOffBx = kOffAx + kPAX;
constexpr uint32_t kPStage = kOffBx + kPBX;  // 56 KB
constexpr uint32_t kSbBytes = PM * 4;        // the tile rows' D of one super-block
constexpr int kSbSlots = 2;
constexpr uint32_t kPSmem = 1024 + kPStages * kPStage + kSbSlots * kSbBytes + 512;
static_assert(kPStage % 1024 == 0, "stages keep the 1024-byte swizzle alignment");
static_assert(kPSmem <= 232448, "fits the 227 KB opt-in shared memory");
constexpr int kActThreads = 128;   // token preparation: 4 warps per token, 4 tokens per SM at once
constexpr int kActCache = 20;      // 128-element groups a warp keeps in registers between the passes
                                   // (K <= 4 x 20 x 128 = 10240 reads X once, longer rows
                                   // re-read the rest)

// kind::f16: f32 accumulator, fp16 A and B, both K-major, M = 128, N = 256:
// B is B_hi's 128 token rows followed by B_lo's (adjacent in the stage), so
// one MMA reads A once for both parts.
constexpr uint32_t kIdescF16 = (1u << 4) | ((uint32_t)(kSlotW >> 3) << 17) | ((uint32_t)(PM >> 4) << 24);
// bf16 A and B, N = 128 (the min-term MMA, into the B_hi half)
constexpr uint32_t kIdescBF16 =
    (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(PN >> 3) << 17) | ((uint32_t)(PM >> 4) << 24);
static_assert(kOffBl == kOffBh + PN * 128, "B_lo's rows follow B_hi's in the stage");

__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// K-major, 32-byte swizzle (one 16-element bf16 K-step per row): 8-row atoms of 256 B.
__device__ __forceinline__ uint64_t sw32_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(256 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)6 << 61);
}

__device__ __forceinline__ void tma2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

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


struct PfArgs {
    int rows, K, T;
    const float *inv;       // [Tp] 2^-e_t
    float *Y;               // [T][rows]
    unsigned int *status;
};

__global__ void __launch_bounds__(kPThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap mA, const __grid_constant__ CUtensorMap mBh,
                      const __grid_constant__ CUtensorMap mBl, const __grid_constant__ CUtensorMap mAx,
                      const __grid_constant__ CUtensorMap mBx, const __grid_constant__ CUtensorMap mRS,
                      const PfArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    float *sbring = reinterpret_cast<float *>(smem + kPStages * kPStage);   // [2][128] D
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + kPStages * kPStage + kSbSlots * kSbBytes);
    uint64_t *empty = full + kPStages;
    uint64_t *sbfull = empty + kPStages;      // a super-block's D arrived
    uint64_t *sbempty = sbfull + kSbSlots;    // every epilogue warp is done with it
    uint64_t *sfull = sbempty + kSbSlots;     // TMEM slot holds a super-block's sums
    uint64_t *sempty = sfull + kSlotsT;       // the epilogue has read the slot
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sempty + kSlotsT);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r0 = blockIdx.y * PM, t0 = blockIdx.x * PN;
    const int nkb = a.K / PK;
    const int nsb = a.K / 256;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kPStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);              // the MMA commit
        }
        for (int s = 0; s < kSbSlots; ++s) {
            mbar_init(&sbfull[s], 1);
            mbar_init(&sbempty[s], kEpiWarps);
        }
        for (int s = 0; s < kSlotsT; ++s) {
            mbar_init(&sfull[s], 1);
            mbar_init(&sempty[s], kEpiWarps);
        }
        fence_barrier_init();
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&mA)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&mBh)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&mBl)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&mAx)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&mBx)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&mRS)) : "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    }
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;
    // programmatic dependent launch: the setup above overlapped the previous
    // kernel's tail; the token parts it wrote are read only after it completes
    pdl_wait();
    pdl_launch_dependents();

    if (warp == 0) {
        if (lane == 0) {
            for (int kb = 0; kb < nkb; ++kb) {
                if ((kb & 3) == 0) {   // a new super-block: its rows' D
                    const int sb = kb >> 2, slot = sb & 1;
                    if (sb >= kSbSlots && !mbar_wait_bounded(&sbempty[slot], ((sb >> 1) - 1) & 1u, a.status))
                        break;
                    mbar_arrive_expect_tx(&sbfull[slot], kSbBytes);
                    tma2d(sbring + slot * PM, &mRS, r0, sb, &sbfull[slot]);
                }
                const int s = kb % kPStages;
                const uint32_t use = kb / kPStages;
                if (use > 0 && !mbar_wait_bounded(&empty[s], (use - 1) & 1u, a.status)) break;
                uint8_t *st = smem + (size_t)s * kPStage;
                mbar_arrive_expect_tx(&full[s], kPStage);
                tma2d(st, &mA, kb * PK, r0, &full[s]);
                tma2d(st + kOffBh, &mBh, kb * PK, t0, &full[s]);
                tma2d(st + kOffBl, &mBl, kb * PK, t0, &full[s]);
                tma2d(st + kOffAx, &mAx, kb * 16, r0, &full[s]);
                tma2d(st + kOffBx, &mBx, kb * 16, t0, &full[s]);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            for (int kb = 0; kb < nkb; ++kb) {
                const int s = kb % kPStages;
                const int sb = kb >> 2;
                const uint32_t slot = sb % kSlotsT;
                if ((kb & 3) == 0 && sb >= kSlotsT &&
                    !mbar_wait_bounded(&sempty[slot], (uint32_t)(sb / kSlotsT - 1) & 1u, a.status))
                    break;
                if (!mbar_wait_bounded(&full[s], (uint32_t)(kb / kPStages) & 1u, a.status)) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t st = smem_u32(smem + (size_t)s * kPStage);
                const uint32_t d = tmem + slot * kSlotW;
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {   // 16 weights per step, B_hi and B_lo at once
                    mma_f16(d, sw128_desc(st + kk * 32), sw128_desc(st + kOffBh + kk * 32), kIdescF16,
                            ((kb & 3) | kk) != 0 ? 1u : 0u);
                }
                // the two sub-blocks' min terms
                mma_f16(d, sw32_desc(st + kOffAx), sw32_desc(st + kOffBx), kIdescBF16, 1u);
                commit(&empty[s]);                         // the stage's tiles are read once these complete
                if ((kb & 3) == 3) commit(&sfull[slot]);   // the super-block's sums are complete
            }
        }
    } else {
        // ---- epilogue: warp -> TMEM lane quarter (weight rows), group -> tokens ----
        const int ew = warp - 2;
        const int q = warp & 3;              // lane quarter
        const int grp = ew >> 2;             // tokens 32*grp .. 32*grp + 31
        const int row = q * 32 + lane;       // weight row within the tile
        const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + grp * 32;
        float2 acc[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[i] = make_float2(0.0f, 0.0f);
        bool ok = true;
        for (int sb = 0; sb < nsb; ++sb) {
            const int sslot = sb & 1;
            const uint32_t slot = sb % kSlotsT;
            if (!mbar_wait_bounded(&sbfull[sslot], (uint32_t)(sb >> 1) & 1u, a.status) ||
                !mbar_wait_bounded(&sfull[slot], (uint32_t)(sb / kSlotsT) & 1u, a.status)) {
                ok = false;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const float D = sbring[sslot * PM + row];
            const float2 D2 = make_float2(D, D);
            float S[32], L[32];
            tmem_ld16(tbase + slot * kSlotW, *reinterpret_cast<float(*)[16]>(S));
            tmem_ld16(tbase + slot * kSlotW + 16, *reinterpret_cast<float(*)[16]>(S + 16));
            tmem_ld16(tbase + slot * kSlotW + PN, *reinterpret_cast<float(*)[16]>(L));
            tmem_ld16(tbase + slot * kSlotW + PN + 16, *reinterpret_cast<float(*)[16]>(L + 16));
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
#pragma unroll
            for (int i = 0; i < 32; ++i) S[i] = __fadd_rn(S[i], L[i]);   // B_hi + B_lo products
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&sempty[slot]);
                mbar_arrive(&sbempty[sslot]);
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) acc[i] = __ffma2_rn(make_float2(S[2 * i], S[2 * i + 1]), D2, acc[i]);
        }
        // undo 2^e_t; rows are the fast dimension of Y: lane = row gives 128-byte stores
        const int r = r0 + row;
        if (ok && r < a.rows) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const int t = t0 + grp * 32 + 2 * i;
                if (t < a.T) a.Y[(size_t)t * a.rows + r] = acc[i].x * __ldg(a.inv + t);
                if (t + 1 < a.T) a.Y[(size_t)(t + 1) * a.rows + r] = acc[i].y * __ldg(a.inv + t + 1);
            }
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    }
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(kTmemCols)
                     : "memory");
    }
}

// x = p0 + p1 + p2, three bf16 parts (each the round-to-nearest of what is left).
__device__ __forceinline__ void split3_bf16(float x, __nv_bfloat16 &p0, __nv_bfloat16 &p1, __nv_bfloat16 &p2) {
    p0 = __float2bfloat16_rn(x);
    const float r1 = x - __bfloat162float(p0);
    p1 = __float2bfloat16_rn(r1);
    p2 = __float2bfloat16_rn(r1 - __bfloat162float(p1));
}

// Q4_K rows -> fp16 A = sc_j * q, the min-term parts Ax and the rows' D:
// one warp per 256-weight super-block.
__global__ void prefill_pack_kernel(const uint8_t *__restrict__ W, int rows, int K, int rows128,
                                    __half *__restrict__ A, __nv_bfloat16 *__restrict__ Ax,
                                    float *__restrict__ rs) {
    const int lane = threadIdx.x & 31;
    const int nsr = K / 256;
    const long long nsb = (long long)rows * nsr;
    const long long w0 = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
    const long long nw = ((long long)gridDim.x * blockDim.x) >> 5;
    for (long long b = w0; b < nsb; b += nw) {
        const uint8_t *blk = W + b * 144;
        const uint32_t s0 = *reinterpret_cast<const uint32_t *>(blk + 4);
        const uint32_t s1 = *reinterpret_cast<const uint32_t *>(blk + 8);
        const uint32_t s2 = *reinterpret_cast<const uint32_t *>(blk + 12);
        const ScaleWords sw = unpack_scale_words(s0, s1, s2);
        // lane handles quant bytes 4*lane .. 4*lane+3 of the 128: group g = lane / 8;
        // low nibbles -> sub-block 2g, high nibbles -> sub-block 2g+1
        const int g = lane >> 3, off = (lane & 7) * 4;
        const uint32_t scw = g < 2 ? sw.sc_lo : sw.sc_hi;
        const int sc_lo = (scw >> (16 * (g & 1))) & 0xFF, sc_hi = (scw >> (16 * (g & 1) + 8)) & 0xFF;
        const uint32_t qs = *reinterpret_cast<const uint32_t *>(blk + 16 + 4 * lane);
        __align__(8) __half lo[4], hi[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            lo[i] = __int2half_rn(sc_lo * (int)((qs >> (8 * i)) & 0xF));
            hi[i] = __int2half_rn(sc_hi * (int)((qs >> (8 * i + 4)) & 0xF));
        }
        __half *dst = A + b * 256;
        *reinterpret_cast<uint2 *>(dst + (2 * g) * 32 + off) = *reinterpret_cast<const uint2 *>(lo);
        *reinterpret_cast<uint2 *>(dst + (2 * g + 1) * 32 + off) = *reinterpret_cast<const uint2 *>(hi);
        const uint32_t dd = *reinterpret_cast<const uint32_t *>(blk);
        float D = f16_bits_to_f32(dd & 0xFFFFu);
        if (D == 0.0f) D = 1.0f;   // every sc is 0: only the min terms count
        __nv_bfloat16 *ax = Ax + b * 64;
        if (lane < 8) {            // sub-block j = lane: c = -dmin m_j / D as three bf16 parts
            const uint32_t mnw = lane < 4 ? sw.mn_lo : sw.mn_hi;
            const int mn = (mnw >> (8 * (lane & 3))) & 0xFF;
            const float c = -__fdiv_rn(__fmul_rn(f16_bits_to_f32(dd >> 16), (float)mn), D);
            __nv_bfloat16 c0, c1, c2;
            split3_bf16(c, c0, c1, c2);
            __nv_bfloat16 *o = ax + (lane >> 1) * 16 + (lane & 1) * 6;
            o[0] = c0; o[1] = c0; o[2] = c1; o[3] = c0; o[4] = c1; o[5] = c2;
        } else if (lane < 24) {    // the four zeros after each pair of sub-blocks
            const int k = lane - 8;
            ax[(k >> 2) * 16 + 12 + (k & 3)] = __float2bfloat16_rn(0.0f);
        } else if (lane == 24) {
            const long long r = b / nsr, sbi = b % nsr;
            rs[sbi * rows128 + r] = D;
        }
    }
}

// Tokens: one CTA per token.  The activation quantizer of quantize_act_kernel
// per 32-block (sx = amax / 127, xq = round(x / sx)), then the token's power
// of two e (largest block amax * 2^e in [2^14, 2^15)), and
//   Bhi + Blo = xq * sx * 2^e (fp16 parts),  Bx = the parts of sx * sumq * 2^e,
//   inv[t] = 2^-e.
__global__ void __launch_bounds__(kActThreads, 4) prefill_act_kernel(const float *__restrict__ X, int T, int K, __half *__restrict__ Bh,
                                   __half *__restrict__ Bl, __nv_bfloat16 *__restrict__ Bx,
                                   float *__restrict__ inv) {
    __shared__ float s_amax[32];
    __shared__ float s_scale;
    const int t = blockIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarp = blockDim.x >> 5;
    const int nb = K / 32;
    const float *x = X + (size_t)t * K;
    // X may be the previous kernel's output, and the previous matmul reads the
    // workspace written here: wait for it before any global access
    pdl_wait();
    pdl_launch_dependents();
    // pass 1: the token's largest |x| (rows are 16-byte aligned: K % 256 == 0).
    // A warp takes the 128-element groups g = warp + i nwarp, a lane 4
    // consecutive elements of each; the first kActCache stay in registers
    // for pass 2.
    const int ngrp = nb / 4;                 // K % 256 == 0: whole groups
    float m = 0.0f;
    const float4 *x4 = reinterpret_cast<const float4 *>(x);
    float4 cache[kActCache];
#pragma unroll
    for (int i = 0; i < kActCache; ++i) {
        const int g = warp + i * nwarp;
        cache[i] = g < ngrp ? x4[g * 32 + lane] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        const float4 v = cache[i];
        m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
    for (int g = warp + kActCache * nwarp; g < ngrp; g += nwarp) {
        const float4 v = x4[g * 32 + lane];
        m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
    m = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(m)));
    if (lane == 0) s_amax[warp] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        float mm = 0.0f;
        for (int w = 0; w < nwarp; ++w) mm = fmaxf(mm, s_amax[w]);
        int e = 0;
        if (mm > 0.0f) {
            int ex;
            frexpf(mm, &ex);          // mm in [2^(ex-1), 2^ex)
            e = min(15 - ex, 126);    // mm * 2^e in [2^14, 2^15); 2^e and 2^-e stay normal
        }
        s_scale = ldexpf(1.0f, e);
        inv[t] = ldexpf(1.0f, -e);
    }
    __syncthreads();
    const float sc2 = s_scale;
    __nv_bfloat16 *bx = Bx + (size_t)t * (K / 4);
    // pass 2: a block is 8 lanes of a group
    const int sub = lane & 7;                // lane within its block
    auto group = [&](int g, const float4 v) {
        const int j = g * 4 + (lane >> 3);   // this lane's block
        float a = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
        const float d = __fdiv_rn(a, 127.0f);
        const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        const float vv[4] = {v.x, v.y, v.z, v.w};
        int qv[4], sq = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float tq = roundf(__fmul_rn(vv[e], id));
            qv[e] = tq > 127.0f ? 127 : (tq < -127.0f ? -127 : (int)tq);
            sq += qv[e];
        }
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
        __align__(8) __half hh[4], hl[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float b = __fmul_rn(__fmul_rn((float)qv[e], d), sc2);
            hh[e] = __float2half_rn(b);
            hl[e] = __float2half_rn(b - __half2float(hh[e]));
        }
        const size_t off = (size_t)t * K + (size_t)g * 128 + lane * 4;
        *reinterpret_cast<uint2 *>(Bh + off) = *reinterpret_cast<const uint2 *>(hh);
        *reinterpret_cast<uint2 *>(Bl + off) = *reinterpret_cast<const uint2 *>(hl);
        // the block's min-term parts: 16 values per pair of blocks
        __nv_bfloat16 *o = bx + (j >> 1) * 16;
        if (sub == 0) {
            __nv_bfloat16 a0, a1, a2;
            split3_bf16(__fmul_rn(__fmul_rn(d, (float)sq), sc2), a0, a1, a2);
            __nv_bfloat16 *p = o + (j & 1) * 6;
            p[0] = a0; p[1] = a1; p[2] = a0; p[3] = a2; p[4] = a1; p[5] = a0;
        } else if ((j & 1) == 0 && sub < 5) {
            o[12 + sub - 1] = __float2bfloat16_rn(0.0f);
        }
    };
#pragma unroll
    for (int i = 0; i < kActCache; ++i) {
        const int g = warp + i * nwarp;
        if (g < ngrp) group(g, cache[i]);
    }
    for (int g = warp + kActCache * nwarp; g < ngrp; g += nwarp) group(g, x4[g * 32 + lane]);
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

// 2-D row-major map: dims {inner, outer}, box {bi, bo}; rows and columns past
// the end read as zeros.
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

int rows_padded(int rows) { return (rows + PM - 1) / PM * PM; }
int tokens_padded(int T) { return (T + PN - 1) / PN * PN; }
size_t up256(size_t n) { return (n + 255) / 256 * 256; }

// packed weights: A | Ax | rs
size_t weight_a_bytes(int rows, int K) { return (size_t)rows * K * sizeof(__half); }
size_t weight_ax_bytes(int rows, int K) { return up256((size_t)rows * (K / 4) * sizeof(__nv_bfloat16)); }
// workspace: Bh | Bl | Bx | inv
size_t act_b_bytes(int T, int K) { return up256((size_t)T * K * sizeof(__half)); }
size_t act_bx_bytes(int T, int K) { return up256((size_t)T * (K / 4) * sizeof(__nv_bfloat16)); }

}  // namespace

size_t lalb_prefill_weight_bytes(int rows, int K) {
    return weight_a_bytes(rows, K) + weight_ax_bytes(rows, K) +
           (size_t)(K / 256) * rows_padded(rows) * sizeof(float);
}

size_t lalb_prefill_act_bytes(int T, int K) {
    return 2 * act_b_bytes(T, K) + act_bx_bytes(T, K) + (size_t)tokens_padded(T) * sizeof(float);
}

int lalb_prefill_pack(lalb_ctx *ctx, const void *W, int rows, int K, void *packed, cudaStream_t s) {
    uint8_t *p = static_cast<uint8_t *>(packed);
    __half *A = reinterpret_cast<__half *>(p);
    __nv_bfloat16 *Ax = reinterpret_cast<__nv_bfloat16 *>(p + weight_a_bytes(rows, K));
    float *rs = reinterpret_cast<float *>(p + weight_a_bytes(rows, K) + weight_ax_bytes(rows, K));
    LALB_CUDA_TRY(ctx, cudaMemsetAsync(rs, 0, (size_t)(K / 256) * rows_padded(rows) * sizeof(float), s));
    const long long nsb = (long long)rows * (K / 256);
    const int blocks = (int)std::min<long long>((nsb * 32 + 255) / 256, (long long)ctx->sm_count * 16);
    prefill_pack_kernel<<<blocks, 256, 0, s>>>(static_cast<const uint8_t *>(W), rows, K, rows_padded(rows),
                                                A, Ax, rs);
    LALB_LAUNCH_CHECK(ctx, "prefill_pack_kernel");
    return LALB_OK;
}

int lalb_prefill_matmul(lalb_ctx *ctx, const void *packed, int rows, int K, const float *X, int T,
                        void *ws, float *Y, cudaStream_t s) {
    const uint8_t *p = static_cast<const uint8_t *>(packed);
    const __half *A = reinterpret_cast<const __half *>(p);
    const __nv_bfloat16 *Ax = reinterpret_cast<const __nv_bfloat16 *>(p + weight_a_bytes(rows, K));
    const float *rs = reinterpret_cast<const float *>(p + weight_a_bytes(rows, K) + weight_ax_bytes(rows, K));
    uint8_t *w = static_cast<uint8_t *>(ws);
    __half *Bh = reinterpret_cast<__half *>(w);
    __half *Bl = reinterpret_cast<__half *>(w + act_b_bytes(T, K));
    __nv_bfloat16 *Bx = reinterpret_cast<__nv_bfloat16 *>(w + 2 * act_b_bytes(T, K));
    float *inv = reinterpret_cast<float *>(w + 2 * act_b_bytes(T, K) + act_bx_bytes(T, K));
    const int Tp = tokens_padded(T);
    int st;
    if ((st = launch_pdl(ctx, (const void *)prefill_act_kernel, dim3(T), dim3(kActThreads), 0, s,
                         {&X, &T, &K, &Bh, &Bl, &Bx, &inv})))
        return st;
    LALB_LAUNCH_CHECK(ctx, "prefill_act_kernel");
    CUtensorMap mA, mBh, mBl, mAx, mBx, mRS;
    if ((st = map2d(ctx, &mA, A, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, K, rows, PK, PM,
                    CU_TENSOR_MAP_SWIZZLE_128B)))
        return st;
    if ((st = map2d(ctx, &mBh, Bh, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, K, T, PK, PN,
                    CU_TENSOR_MAP_SWIZZLE_128B)))
        return st;
    if ((st = map2d(ctx, &mBl, Bl, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, K, T, PK, PN,
                    CU_TENSOR_MAP_SWIZZLE_128B)))
        return st;
    if ((st = map2d(ctx, &mAx, Ax, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K / 4, rows, 16, PM,
                    CU_TENSOR_MAP_SWIZZLE_32B)))
        return st;
    if ((st = map2d(ctx, &mBx, Bx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K / 4, T, 16, PN,
                    CU_TENSOR_MAP_SWIZZLE_32B)))
        return st;
    if ((st = map2d(ctx, &mRS, rs, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, rows_padded(rows), K / 256, PM, 1,
                    CU_TENSOR_MAP_SWIZZLE_NONE)))
        return st;
    if ((st = lalb_set_smem_attr(ctx, (const void *)prefill_tc_kernel, (int)kPSmem))) return st;
    PfArgs a = {};
    a.rows = rows;
    a.K = K;
    a.T = T;
    a.inv = inv;
    a.Y = Y;
    a.status = &ctx->scratch->status;
    const dim3 grid(Tp / PN, (rows + PM - 1) / PM);
    if ((st = launch_pdl(ctx, (const void *)prefill_tc_kernel, grid, dim3(kPThreads), kPSmem, s,
                         {&mA, &mBh, &mBl, &mAx, &mBx, &mRS, &a})))
        return st;
    LALB_LAUNCH_CHECK(ctx, "prefill_tc_kernel");
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
