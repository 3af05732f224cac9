// lalb_prefill.cu -- batched (prefill) Q4_K x Q8 matmul on the tcgen05 tensor cores,
// straight from the Q4_K bytes.
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
// The weights stay the caller's Q4_K rows (0.5625 bytes per weight in HBM):
// the 128-row x 256-weight tile of a super-block comes into shared memory as
// its raw 144-byte blocks (18 KB), and worker warps decode it in registers
// (row = TMEM lane) into the MMA's A operand, stored straight into TMEM with
// tcgen05.st: per 64-weight K-block the fp16 sc_j * q (32 columns) and the
// bf16 min-term parts (8 columns).  The MMAs read A from TMEM and only the
// token tiles from shared memory.
//
// Tokens, prepared per call (prefill_act_kernel) in the workspace:
//   Bhi, Blo  fp16 [T][K]
//   Bx        bf16 [T][K/4]: per 64 weights, for their two sub-blocks
//             {a0 a1 a0 a2 a1 a0} (parts of a 2^e_t) each, then 4 zeros
//   inv       fp32 [Tp] = 2^-e_t   (Tp = T rounded up to 128)
//
// TMEM (all 512 columns of the SM):
//   columns   0..255   two super-block accumulator slots of 128 (fp32): the
//                      B_hi and B_lo products of a K-step accumulate into the
//                      same slot (two N = 128 MMAs)
//   columns 256..511   four A stages of 64: sc * q (32), min-term parts (8)
// Every wait is bounded.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <mutex>

#include "lalb_internal.cuh"
#include "lalb_prefill.cuh"
#include "lalb_tcgen05.cuh"

using namespace lalb;

namespace {

constexpr int PM = 128, PN = 128, PK = 64;   // PK fp16 = 128 B: one swizzle row
constexpr int kSlotsT = 2;                   // TMEM super-block slots
constexpr int kTmemCols = 512;
constexpr int kEpiWarps = 16;
constexpr uint32_t kPB = PN * PK * 2;        // 16 KB (each of B_hi, B_lo)
constexpr uint32_t kPBX = PN * 16 * 2;       // 4 KB: 128 tokens x 16 bf16
constexpr int kRBStages = 4;                    // token tiles: B_hi, B_lo, Bx
constexpr uint32_t kRBStage = 2 * kPB + kPBX;   // 36 KB
constexpr uint32_t kRBOffBx = 2 * kPB;
constexpr int kRawSlots = 3;                    // raw super-block tiles
constexpr uint32_t kRawBytes = PM * 144;        // 18 KB
constexpr int kRThreads = 32 * (2 + kEpiWarps);   // producer, MMA, 16 workers
constexpr int kRAccW = PN;                      // accumulator slot: 128 columns
constexpr int kRAStages = 4;                    // A stages in TMEM
constexpr int kRAColW = 64;                     // columns per A stage
constexpr int kRAColBase = kSlotsT * kRAccW;    // 256
constexpr int kRAColX = 32;                     // min-term parts within the stage
static_assert(kRAColBase + kRAStages * kRAColW <= kTmemCols, "A stages fit the TMEM allocation");
constexpr uint32_t kRSmem = 1024 + kRBStages * kRBStage + kRawSlots * kRawBytes + 512;
static_assert(kRSmem <= 232448, "fits the 227 KB opt-in shared memory");
static_assert(kRBStage % 1024 == 0, "stages keep the 1024-byte swizzle alignment");
static_assert(kRawBytes % 128 == 0, "raw slots keep 128-byte alignment");
static_assert(kRAStages == kRBStages && kRAStages == 4, "A stage g holds K-block g of each super-block");
constexpr int kActThreads = 128;   // token preparation: 4 warps per token, 4 tokens per SM at once
constexpr int kActThreadsLong = 256;   // rows longer than 4 warps' caches: 8 warps, 2 tokens per SM
constexpr int kActCache = 20;      // 128-element groups a warp keeps in registers between the passes
                                   // (K <= 4 x 20 x 128 = 10240 reads X once with 4 warps, K <=
                                   // 20480 with 8; longer rows re-read the rest)

// kind::f16, f32 accumulator, fp16 A (TMEM) and B (shared memory), both
// K-major, M = 128, N = 128
constexpr uint32_t kIdescF16N128 = (1u << 4) | ((uint32_t)(PN >> 3) << 17) | ((uint32_t)(PM >> 4) << 24);
// bf16 A and B, N = 128 (the min-term MMA)
constexpr uint32_t kIdescBF16 =
    (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(PN >> 3) << 17) | ((uint32_t)(PM >> 4) << 24);

struct PfArgs {
    int rows, K, T;
    int splits, sb_per;     // K split over gridDim.z CTAs of sb_per super-blocks each (the last fewer)
    const float *inv;       // [Tp] 2^-e_t
    float *Y;               // [T][rows]
    float *part;            // splits > 1: [splits][T][rows] partial sums (prefill_split_sum_kernel adds them)
    unsigned int *status;
};

// x = p0 + p1 + p2, three bf16 parts (each the round-to-nearest of what is left).
__device__ __forceinline__ void split3_bf16(float x, __nv_bfloat16 &p0, __nv_bfloat16 &p1, __nv_bfloat16 &p2) {
    p0 = __float2bfloat16_rn(x);
    const float r1 = x - __bfloat162float(p0);
    p1 = __float2bfloat16_rn(r1);
    p2 = __float2bfloat16_rn(r1 - __bfloat162float(p1));
}

// The 64 fp16 values sc * q of one row's 64-weight K-block kbl, from its raw
// 144-byte block, as 32 half2 words in weight order: the 32 quant bytes of
// group kbl hold sub-block 2 kbl (weights 0..31) in their low and 2 kbl + 1
// (weights 32..63) in their high nibbles.  sc * q is an integer <= 945, exact
// in fp16: (1024 + q) as fp16 times sc minus 1024 sc, one fused rounding of
// an exact result.
__device__ __forceinline__ void conv_kblock(const uint8_t *blk, int kbl, uint32_t sc0, uint32_t sc1,
                                            uint32_t (&o)[32]) {
    const uint4 v0 = *reinterpret_cast<const uint4 *>(blk + 16 + 32 * kbl);
    const uint4 v1 = *reinterpret_cast<const uint4 *>(blk + 32 + 32 * kbl);
    const uint32_t w[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    const __half2 s0 = __half2half2(__uint2half_rn(sc0)), s1 = __half2half2(__uint2half_rn(sc1));
    const __half2 m0 = __hneg2(__half2half2(__uint2half_rn(1024u * sc0)));
    const __half2 m1 = __hneg2(__half2half2(__uint2half_rn(1024u * sc1)));
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const uint32_t l = w[k] & 0x0F0F0F0Fu, h = (w[k] >> 4) & 0x0F0F0F0Fu;
        const uint32_t l01 = __byte_perm(l, 0x64646464u, 0x5140), l23 = __byte_perm(l, 0x64646464u, 0x7362);
        const uint32_t h01 = __byte_perm(h, 0x64646464u, 0x5140), h23 = __byte_perm(h, 0x64646464u, 0x7362);
        const __half2 a = __hfma2(*reinterpret_cast<const __half2 *>(&l01), s0, m0);
        const __half2 b = __hfma2(*reinterpret_cast<const __half2 *>(&l23), s0, m0);
        const __half2 c = __hfma2(*reinterpret_cast<const __half2 *>(&h01), s1, m1);
        const __half2 d = __hfma2(*reinterpret_cast<const __half2 *>(&h23), s1, m1);
        o[2 * k] = *reinterpret_cast<const uint32_t *>(&a);
        o[2 * k + 1] = *reinterpret_cast<const uint32_t *>(&b);
        o[16 + 2 * k] = *reinterpret_cast<const uint32_t *>(&c);
        o[16 + 2 * k + 1] = *reinterpret_cast<const uint32_t *>(&d);
    }
}

__device__ __forceinline__ uint32_t pack_bf16(__nv_bfloat16 lo, __nv_bfloat16 hi) {
    return (uint32_t)__bfloat16_as_ushort(lo) | ((uint32_t)__bfloat16_as_ushort(hi) << 16);
}

// The 16 bf16 min-term values of one row's K-block (sub-blocks 2 kbl and
// 2 kbl + 1) as 8 words: {c0 c0 c1 c0 c1 c2} of each sub-block's
// c = -dmin m / D, then four zeros; against the token side's {a0 a1 a0 a2 a1
// a0} (prefill_act_kernel) the 16-wide bf16 MMA adds the six products
// c_i a_j with i + j <= 2.
__device__ __forceinline__ void conv_minparts(float dmin, float D, int m0, int m1, uint32_t (&o)[8]) {
    __nv_bfloat16 a0, a1, a2, b0, b1, b2;
    split3_bf16(-__fdiv_rn(__fmul_rn(dmin, (float)m0), D), a0, a1, a2);
    split3_bf16(-__fdiv_rn(__fmul_rn(dmin, (float)m1), D), b0, b1, b2);
    o[0] = pack_bf16(a0, a0);
    o[1] = pack_bf16(a1, a0);
    o[2] = pack_bf16(a1, a2);
    o[3] = pack_bf16(b0, b0);
    o[4] = pack_bf16(b1, b0);
    o[5] = pack_bf16(b1, b2);
    o[6] = 0u;
    o[7] = 0u;
}

// One CTA per 128-row x 128-token tile, 18 warps:
//   warp 0      TMA producer: the first three raw 128 x 144-byte super-block
//               tiles, then per K-block the B_hi, B_lo and Bx token tiles into
//               a 4-stage ring;
//   warp 1      the MMAs, the whole warp in the loop and one elected lane
//               issuing: per K-step A x B_hi and A x B_lo into the
//               super-block's slot, per K-block the min-term MMA, and one
//               commit that frees the K-block's token stage and A stage (the
//               two rings share their stage index kb % 4);
//   warps 2-17  workers, each on its TMEM lane quarter q = warp % 4 (rows
//               32 q .. 32 q + 31, lane = row) and group g = (warp - 2) / 4:
//               of every super-block, K-block g into A stage g (64 sc * q
//               values and the 16 min-term parts per row), then the epilogue
//               of the previous super-block (tokens 32 g .. 32 g + 31 of its
//               slot), whose D the thread kept from the row's header.  The
//               raw tiles have a 3-slot ring: once every worker has decoded
//               super-block sb, the first worker thread loads sb + 3 into its
//               slot, two super-blocks ahead of its use.
// TMEM: all 512 columns are allocated, so its base address is column 0 and
// the MMA warp's TMEM operands are constants plus the loop's offsets.
__global__ void __launch_bounds__(kRThreads, 1)
    prefill_q4k_kernel(const __grid_constant__ CUtensorMap mW, const __grid_constant__ CUtensorMap mBh,
                       const __grid_constant__ CUtensorMap mBl, const __grid_constant__ CUtensorMap mBx,
                       const PfArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    uint8_t *bring = smem;                                      // [4] B_hi | B_lo | Bx
    uint8_t *rawring = bring + kRBStages * kRBStage;            // [3] raw super-block tiles
    uint64_t *bfull = reinterpret_cast<uint64_t *>(rawring + kRawSlots * kRawBytes);
    uint64_t *afull = bfull + kRBStages;      // the four workers of the stage stored their rows
    uint64_t *kempty = afull + kRAStages;     // the K-block's MMAs completed: token and A stage free
    uint64_t *rfull = kempty + kRBStages;     // a raw super-block tile landed
    uint64_t *rempty = rfull + kRawSlots;     // every worker has decoded it
    uint64_t *sfull = rempty + kRawSlots;     // TMEM slot holds a super-block's sums
    uint64_t *sempty = sfull + kSlotsT;       // the epilogue has read the slot
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sempty + kSlotsT);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r0 = blockIdx.y * PM, t0 = blockIdx.x * PN;
    // this CTA's super-blocks: sb0 .. sb0 + nsb - 1 of the K / 256 (every
    // index below counts from sb0; the host makes every split non-empty)
    const int sb0 = blockIdx.z * a.sb_per;
    const int nsb = min(a.K / 256 - sb0, a.sb_per);
    const int nkb = nsb * 4;
    const int kb0 = sb0 * 4;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kRBStages; ++s) {
            mbar_init(&bfull[s], 1);
            mbar_init(&afull[s], 4);
            mbar_init(&kempty[s], 1);             // the MMA commit
        }
        for (int s = 0; s < kRawSlots; ++s) {
            mbar_init(&rfull[s], 1);
            mbar_init(&rempty[s], kEpiWarps);
        }
        for (int s = 0; s < kSlotsT; ++s) {
            mbar_init(&sfull[s], 1);
            mbar_init(&sempty[s], kEpiWarps);
        }
        fence_barrier_init();
        prefetch_tensormap(&mW);
        prefetch_tensormap(&mBh);
        prefetch_tensormap(&mBl);
        prefetch_tensormap(&mBx);
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
    // every role reads the same word; a base other than column 0 (impossible
    // with the whole of TMEM allocated) raises a status bit and skips the work
    const bool tmem_ok = tmem == 0;
    if (!tmem_ok && threadIdx.x == 0) atomicOr(a.status, LALB_STATUS_WAIT_TIMEOUT);

    if (warp == 0) {
        if (lane == 0 && tmem_ok) {
            // the weights are not written by the previous kernel (the token
            // preparation): their first tiles go out before the dependency wait
            for (int sb = 0; sb < kRawSlots && sb < nsb; ++sb) {
                mbar_arrive_expect_tx(&rfull[sb], kRawBytes);
                tma2d(rawring + sb * kRawBytes, &mW, (sb0 + sb) * 144, r0, &rfull[sb]);
            }
            pdl_wait();
            pdl_launch_dependents();
            for (int kb = 0; kb < nkb; ++kb) {
                const int s = kb % kRBStages;
                const uint32_t use = kb / kRBStages;
                if (use > 0 && !mbar_wait_bounded(&kempty[s], (use - 1) & 1u, a.status)) break;
                uint8_t *st = bring + (size_t)s * kRBStage;
                mbar_arrive_expect_tx(&bfull[s], kRBStage);
                tma2d(st, &mBh, (kb0 + kb) * PK, t0, &bfull[s]);
                tma2d(st + kPB, &mBl, (kb0 + kb) * PK, t0, &bfull[s]);
                tma2d(st + kRBOffBx, &mBx, (kb0 + kb) * 16, t0, &bfull[s]);
            }
        } else {
            pdl_wait();
        }
    } else if (warp == 1) {
        pdl_wait();
        const uint32_t bring_s = smem_u32(bring);
        for (int kb = 0; kb < nkb && tmem_ok; ++kb) {
            const int sb = kb >> 2;
            const uint32_t slot = sb % kSlotsT;
            if ((kb & 3) == 0 && sb >= kSlotsT &&
                !warp_wait_fast(&sempty[slot], (uint32_t)(sb / kSlotsT - 1) & 1u, a.status))
                break;
            const int s = kb % kRBStages;
            if (!warp_wait_fast(&bfull[s], (uint32_t)(kb / kRBStages) & 1u, a.status) ||
                !warp_wait_fast(&afull[s], (uint32_t)(kb / kRAStages) & 1u, a.status))
                break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t bst = bring_s + (uint32_t)s * kRBStage;
            const uint32_t ta = kRAColBase + s * kRAColW;
            const uint32_t d = slot * kRAccW;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {   // 16 weights (8 columns of A) per step
                mma_f16_ta(d, ta + kk * 8, sw128_desc(bst + kk * 32), kIdescF16N128,
                           ((kb & 3) | kk) != 0 ? 1u : 0u);
                mma_f16_ta(d, ta + kk * 8, sw128_desc(bst + kPB + kk * 32), kIdescF16N128, 1u);
            }
            mma_f16_ta(d, ta + kRAColX, sw32_desc(bst + kRBOffBx), kIdescBF16, 1u);   // min terms
            commit_elect(&kempty[s]);
            if ((kb & 3) == 3) commit_elect(&sfull[slot]);
        }
    } else {
        pdl_wait();
        const int q = warp & 3;             // TMEM lane quarter: rows 32 q .. 32 q + 31
        const int grp = (warp - 2) >> 2;    // K-block of each super-block; tokens 32 grp .. of the epilogue
        const int row = q * 32 + lane;
        const uint32_t lanes = (uint32_t)(q * 32) << 16;
        const uint32_t tacc = lanes + grp * 32;
        const uint32_t ta = lanes + kRAColBase + grp * kRAColW;   // A stage grp
        float2 acc[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[i] = make_float2(0.0f, 0.0f);
        bool ok = tmem_ok;
        auto epilogue = [&](int sb, float D) -> bool {
            const uint32_t slot = sb % kSlotsT;
            if (!warp_wait_fast(&sfull[slot], (uint32_t)(sb / kSlotsT) & 1u, a.status)) return false;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            float S[32];
            tmem_ld16(tacc + slot * kRAccW, *reinterpret_cast<float(*)[16]>(S));
            tmem_ld16(tacc + slot * kRAccW + 16, *reinterpret_cast<float(*)[16]>(S + 16));
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&sempty[slot]);
            const float2 D2 = make_float2(D, D);
#pragma unroll
            for (int i = 0; i < 16; ++i) acc[i] = __ffma2_rn(make_float2(S[2 * i], S[2 * i + 1]), D2, acc[i]);
            return true;
        };
        float Dprev = 1.0f;
        for (int sb = 0; sb < nsb && ok; ++sb) {
            const int rs = sb % kRawSlots;
            if (!warp_wait_fast(&rfull[rs], (uint32_t)(sb / kRawSlots) & 1u, a.status)) {
                ok = false;
                break;
            }
            const uint8_t *blk = rawring + rs * kRawBytes + row * 144;
            const uint4 hdr = *reinterpret_cast<const uint4 *>(blk);
            const ScaleWords sw = unpack_scale_words(hdr.y, hdr.z, hdr.w);
            float D = f16_bits_to_f32(hdr.x & 0xFFFFu);
            if (D == 0.0f) D = 1.0f;   // every sc is 0: only the min terms count
            const float dmin = f16_bits_to_f32(hdr.x >> 16);
            // K-block kb = 4 sb + grp into A stage grp, free once K-block kb - 4 completed
            if (sb > 0 && !warp_wait_fast(&kempty[grp], (uint32_t)(sb - 1) & 1u, a.status)) {
                ok = false;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t scw = grp < 2 ? sw.sc_lo : sw.sc_hi, mnw = grp < 2 ? sw.mn_lo : sw.mn_hi;
            const int sh = 16 * (grp & 1);
            {
                uint32_t v[32];
                conv_kblock(blk, grp, (scw >> sh) & 0xFF, (scw >> (sh + 8)) & 0xFF, v);
                tmem_st32(ta, v);
            }
            {
                uint32_t v[8];
                conv_minparts(dmin, D, (mnw >> sh) & 0xFF, (mnw >> (sh + 8)) & 0xFF, v);
                tmem_st8(ta + kRAColX, v);
            }
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&afull[grp]);
                mbar_arrive(&rempty[rs]);
                if (warp == 2 && sb + kRawSlots < nsb) {   // refill the raw slot
                    if (mbar_wait_bounded(&rempty[rs], (uint32_t)(sb / kRawSlots) & 1u, a.status)) {
                        mbar_arrive_expect_tx(&rfull[rs], kRawBytes);
                        tma2d(rawring + rs * kRawBytes, &mW, (sb0 + sb + kRawSlots) * 144, r0, &rfull[rs]);
                    }
                }
            }
            __syncwarp();
            if (sb > 0) ok = epilogue(sb - 1, Dprev);
            Dprev = D;
        }
        if (ok) ok = epilogue(nsb - 1, Dprev);
        // undo 2^e_t; rows are the fast dimension of Y: lane = row gives 128-byte stores
        const int r = r0 + row;
        float *out = a.splits == 1 ? a.Y : a.part + (size_t)blockIdx.z * a.T * a.rows;
        if (ok && r < a.rows) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const int t = t0 + grp * 32 + 2 * i;
                if (t < a.T) out[(size_t)t * a.rows + r] = acc[i].x * __ldg(a.inv + t);
                if (t + 1 < a.T) out[(size_t)(t + 1) * a.rows + r] = acc[i].y * __ldg(a.inv + t + 1);
            }
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    }
    __syncwarp();   // warp 0's lane 0 ran the producer loop alone: the barrier below is warp-aligned
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(kTmemCols)
                     : "memory");
    }
}

// Tokens: one CTA per token.  The activation quantizer of quantize_act_kernel
// per 32-block (sx = amax / 127, xq = round(x / sx)), then the token's power
// of two e (largest block amax * 2^e in [2^14, 2^15)), and
//   Bhi + Blo = xq * sx * 2^e (fp16 parts),  Bx = the parts of sx * sumq * 2^e,
//   inv[t] = 2^-e.
template <int NT>
__global__ void __launch_bounds__(NT, 512 / NT) prefill_act_kernel(const float *__restrict__ X, int T, int K, __half *__restrict__ Bh,
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

// The K splits of a call: Y = the partial sums part[z] added in split order
// z = 0, 1, .. (the same sum on every run).  4 consecutive outputs per thread
// when rows is a multiple of 4, else one.
__global__ void __launch_bounds__(256) prefill_split_sum_kernel(const float *__restrict__ part, int splits,
                                                               long long n, int vec4, float *__restrict__ Y) {
    // the partial sums are the matmul's output: wait for it to complete
    pdl_wait();
    pdl_launch_dependents();
    const long long stride = (long long)gridDim.x * blockDim.x;
    if (vec4) {
        const long long n4 = n >> 2;
        const float4 *p4 = reinterpret_cast<const float4 *>(part);
        for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += stride) {
            float4 v = __ldcg(p4 + i);
            for (int z = 1; z < splits; ++z) {
                const float4 u = __ldcg(p4 + z * n4 + i);
                v.x += u.x;
                v.y += u.y;
                v.z += u.z;
                v.w += u.w;
            }
            reinterpret_cast<float4 *>(Y)[i] = v;
        }
    } else {
        for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += stride) {
            float v = __ldcg(part + i);
            for (int z = 1; z < splits; ++z) v += __ldcg(part + z * n + i);
            Y[i] = v;
        }
    }
}

int tokens_padded(int T) { return (T + PN - 1) / PN * PN; }
size_t up256(size_t n) { return (n + 255) / 256 * 256; }

// workspace: Bh | Bl | Bx | inv | part
size_t act_b_bytes(int T, int K) { return up256((size_t)T * K * sizeof(__half)); }
size_t act_bx_bytes(int T, int K) { return up256((size_t)T * (K / 4) * sizeof(__nv_bfloat16)); }
size_t act_bytes(int T, int K) {
    return 2 * act_b_bytes(T, K) + act_bx_bytes(T, K) + up256((size_t)tokens_padded(T) * sizeof(float));
}
int n_tiles(int rows, int T) { return ((rows + PM - 1) / PM) * (tokens_padded(T) / PN); }

// The K split of a call: with fewer output tiles than the B200's 148 SMs,
// the K super-blocks are shared out over `splits` CTAs per tile, sb_per each.
// Cost model, in super-blocks of MMA work: waves x (sb_per + 1), the 1 being
// a CTA's fixed cost (set-up, pipeline fill, epilogue).
constexpr int kSplitSms = 148;
constexpr int kMaxSplits = 16;
void split_plan(int rows, int K, int T, int *splits, int *sb_per) {
    const int tiles = n_tiles(rows, T), nsb = K / 256;
    int best = 1, best_per = nsb;
    if (tiles < kSplitSms) {
        long long best_cost = (long long)nsb + 1;
        for (int s = 2; s <= std::min(nsb, kMaxSplits); ++s) {
            const int per = (nsb + s - 1) / s, se = (nsb + per - 1) / per;
            const long long waves = ((long long)tiles * se + kSplitSms - 1) / kSplitSms;
            const long long cost = waves * (per + 1);
            if (cost < best_cost) best_cost = cost, best = se, best_per = per;
        }
    }
    *splits = best;
    *sb_per = best_per;
}
size_t part_bytes(int rows, int K, int T) {
    int splits, per;
    split_plan(rows, K, T, &splits, &per);
    return splits > 1 ? up256((size_t)splits * T * rows * sizeof(float)) : 0;
}

}  // namespace

size_t lalb_prefill_ws_bytes(int rows, int K, int T) {
    return act_bytes(T, K) + part_bytes(rows, K, T);
}

// W: rows x K/256 Q4_K blocks of 144 bytes, 16-byte aligned; ws: the prepared
// tokens and the split-K partial sums (lalb_prefill_ws_bytes),
// 256-byte aligned.
int lalb_prefill_matmul(lalb_ctx *ctx, const void *W, int rows, int K, const float *X, int T, void *ws,
                        float *Y, cudaStream_t s) {
    uint8_t *w = static_cast<uint8_t *>(ws);
    __half *Bh = reinterpret_cast<__half *>(w);
    __half *Bl = reinterpret_cast<__half *>(w + act_b_bytes(T, K));
    __nv_bfloat16 *Bx = reinterpret_cast<__nv_bfloat16 *>(w + 2 * act_b_bytes(T, K));
    float *inv = reinterpret_cast<float *>(w + 2 * act_b_bytes(T, K) + act_bx_bytes(T, K));
    float *part = reinterpret_cast<float *>(w + act_bytes(T, K));
    int splits, sb_per;
    split_plan(rows, K, T, &splits, &sb_per);
    const int Tp = tokens_padded(T);
    int st;
    // 8 warps per token once 4 warps' register caches cannot hold the row: the
    // 18944-long rows of the down projection are then read once (measured:
    // 420.6-420.9 -> 424.0-425.5 TOPS per 7B prefill step)
    const bool long_k = K / 128 > 4 * kActCache;
    const void *act_fn = long_k ? (const void *)prefill_act_kernel<kActThreadsLong>
                                : (const void *)prefill_act_kernel<kActThreads>;
    if ((st = launch_pdl(ctx, act_fn, dim3(T), dim3(long_k ? kActThreadsLong : kActThreads), 0, s,
                         {&X, &T, &K, &Bh, &Bl, &Bx, &inv})))
        return st;
    LALB_LAUNCH_CHECK(ctx, "prefill_act_kernel");
    CUtensorMap mW, mBh, mBl, mBx;
    // a row's blocks as bytes: the box is one 144-byte block of 128 rows, its
    // x coordinate sb * 144 a multiple of 16
    if ((st = map2d(ctx, &mW, W, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (long long)(K / 256) * 144, rows, 144, PM,
                    CU_TENSOR_MAP_SWIZZLE_NONE)))
        return st;
    if ((st = map2d(ctx, &mBh, Bh, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, K, T, PK, PN,
                    CU_TENSOR_MAP_SWIZZLE_128B)))
        return st;
    if ((st = map2d(ctx, &mBl, Bl, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, K, T, PK, PN,
                    CU_TENSOR_MAP_SWIZZLE_128B)))
        return st;
    if ((st = map2d(ctx, &mBx, Bx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K / 4, T, 16, PN,
                    CU_TENSOR_MAP_SWIZZLE_32B)))
        return st;
    if ((st = lalb_set_smem_attr(ctx, (const void *)prefill_q4k_kernel, (int)kRSmem))) return st;
    PfArgs a = {};
    a.rows = rows;
    a.K = K;
    a.T = T;
    a.splits = splits;
    a.sb_per = sb_per;
    a.inv = inv;
    a.Y = Y;
    a.part = part;
    a.status = &ctx->scratch->status;
    const dim3 grid(Tp / PN, (rows + PM - 1) / PM, splits);
    if ((st = launch_pdl(ctx, (const void *)prefill_q4k_kernel, grid, dim3(kRThreads), kRSmem, s,
                         {&mW, &mBh, &mBl, &mBx, &a})))
        return st;
    LALB_LAUNCH_CHECK(ctx, "prefill_q4k_kernel");
    if (splits > 1) {
        long long n = (long long)T * rows;
        int vec4 = (rows % 4) == 0;
        const long long work = vec4 ? n / 4 : n;
        const int blocks = (int)std::min<long long>((work + 255) / 256, (long long)ctx->sm_count * 8);
        if ((st = launch_pdl(ctx, (const void *)prefill_split_sum_kernel, dim3(blocks), dim3(256), 0, s,
                             {&part, &splits, &n, &vec4, &Y})))
            return st;
        LALB_LAUNCH_CHECK(ctx, "prefill_split_sum_kernel");
    }
    return LALB_OK;
}

// ---- C ABI -------------------------------------------------------------------
extern "C" int lalb_prefill_ws_bytes(int rows, int K, int T, size_t *ws_bytes) {
    if (rows <= 0 || K <= 0 || K % 256 || T <= 0 || !ws_bytes) return LALB_ERR_INVALID;
    *ws_bytes = lalb_prefill_ws_bytes(rows, K, T);
    return LALB_OK;
}

extern "C" int lalb_matmul_q4_k_prefill(lalb_ctx *ctx, const void *W, int rows, int K, const float *X, int T,
                                        void *ws, float *Y, lalb_stream stream) {
    if (!ctx) return LALB_ERR_INVALID;
    if (!W || !X || !ws || !Y || rows <= 0 || K <= 0 || K % 256 || T <= 0)
        return lalb_fail(ctx, LALB_ERR_INVALID, "matmul_q4_k_prefill: bad arguments");
    if (((uintptr_t)W & 15u) || ((uintptr_t)ws & 255u) || ((uintptr_t)X & 15u) || ((uintptr_t)Y & 3u))
        return lalb_fail(ctx, LALB_ERR_INVALID, "matmul_q4_k_prefill: misaligned buffer");
    return lalb_prefill_matmul(ctx, W, rows, K, X, T, ws, Y, (cudaStream_t)stream);
}
