// lalb_logic_gemm.cu -- the seed STE model's logic layers on the tcgen05 tensor
// cores, straight from their int8 codes.
//
//   Y[t][n] = srow[n] * sum_k codes[n][k] * X[t][k] + bias[n]
//
// the per-element CORE / BINARY / PRUNE encoding of lalb_logic_pack (one int8
// code per weight, |code| <= 127, one scale per output row) applied to the
// T rows of X (bin_forward, runtime/lal_runtime.c:1852-1956, with the code
// and the row scale in place of the mode's weight).
//
// Exactness: every code is an integer exact in fp16; X goes in as two fp16
// parts under a per-token power of two (hi + lo: 22 significant bits, the
// token's largest |x| scaled into [2^14, 2^15), exact to apply and undo), so
// every product is exact in fp32 and the fp32 tensor-core sum is the only
// rounding.  srow and the bias are applied once, in fp32, at the end.
//
// The codes stay 1 byte per weight in HBM: each K-block's 128-row x 64-code
// tile comes into shared memory by TMA (64-byte swizzle) beside the token
// tiles, and worker warps decode it in registers (row = TMEM lane) into the
// MMA's fp16 A operand in TMEM (tcgen05.st).  The MMAs read A from TMEM and
// only the token tiles from shared memory.  There is no scale inside K, so a
// unit's whole K accumulates in one slot, B_hi and B_lo products together.
//
// TMEM (all 512 columns of the SM):
//   columns   0..255   two accumulator slots of 128 (fp32, tokens)
//   columns 256..383   four A stages of 32 (64 fp16 codes of a K-block per row)
//
// Persistent: at most one CTA per SM, each taking every gridDim.x-th unit of
// work (a 128-row x 128-token output tile, or one K split of it when the
// call has fewer tiles than SMs: their partial sums go through a workspace
// and a split-sum kernel that adds them in split order), 18 warps:
//   warp 0      TMA producer: per K-block the B_hi, B_lo and code tiles into a
//               4-stage ring (40 KB a stage), running ahead across units;
//   warp 1      the MMAs, the whole warp in the loop and one elected lane
//               issuing: per K-step one N = 128 MMA over B_hi and one over
//               B_lo into the unit's accumulator slot (two slots, so a unit's
//               epilogue overlaps the next unit's MMAs), one commit freeing the
//               K-block's stage, one per unit for its epilogue;
//   warps 2-17  warp (q, g) on TMEM lanes 32 q .. 32 q + 31 decodes the
//               K-blocks whose index across the CTA's units is g mod 4 into A
//               stage g, then does the previous unit's epilogue (tokens
//               32 g .. 32 g + 31 of its slot).
// Every wait is bounded.
#include <cuda.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "lalb_internal.cuh"
#include "lalb_logic_gemm.cuh"
#include "lalb_tcgen05.cuh"

using namespace lalb;

namespace {

constexpr int LM = 128, LN = 128, LK = 64;       // weight rows, tokens, K-block (64 fp16 = 128 B)
constexpr int kLStages = 4;
constexpr uint32_t kLB = LN * LK * 2;            // 16 KB: the B_hi or B_lo tile
constexpr uint32_t kLC = LM * LK;                // 8 KB: the code tile
constexpr uint32_t kLStage = 2 * kLB + kLC;      // 40 KB
constexpr int kLWorkers = 16;
constexpr int kLThreads = 32 * (2 + kLWorkers);
constexpr int kLTmemCols = 512;
constexpr int kLSlots = 2;                       // accumulator slots of LN columns
constexpr int kLAColBase = kLSlots * LN;         // 256
constexpr int kLAColW = LK / 2;                  // 32 columns: 64 fp16 per row
constexpr uint32_t kLSmem = 1024 + kLStages * kLStage + 256;
static_assert(kLStage % 1024 == 0, "stages keep the 1024-byte swizzle alignment");
static_assert(kLSmem <= 232448, "fits the 227 KB opt-in shared memory");
static_assert(kLAColBase + kLStages * kLAColW <= kLTmemCols, "A stages fit the TMEM allocation");
constexpr int kLActThreads = 128;
constexpr int kLMaxSplits = 16;
constexpr int kLSplitSms = 148;
constexpr int kLCtaCost = 6;                     // a CTA's fixed cost, in K-blocks of MMA work
constexpr int kLSumCost = 10;                    // the split-sum launch, in the same units

// kind::f16, f32 accumulator, fp16 A (TMEM) and B (shared memory), K-major,
// M = 128, N = 128: per K-step one MMA over B_hi and one over B_lo into the
// same slot
constexpr uint32_t kIdescLogic = (1u << 4) | ((uint32_t)(LN >> 3) << 17) | ((uint32_t)(LM >> 4) << 24);

// A unit of work is one 128-row x 128-token output tile and one K split of
// it; units are numbered token tile fastest, then row tile, then split.
struct LgArgs {
    int rows, K, M;          // layer rows (the output's columns), K, tokens
    int t_tiles, r_tiles;    // 128-token and 128-row tiles
    int splits, kb_per;      // K splits of kb_per K-blocks each (the last may have fewer)
    int units;               // t_tiles * r_tiles * splits; CTA b takes units b, b + gridDim.x, ...
    const float *inv;        // [Mp] 2^-e_t
    const float *srow, *bias;
    float *Y;                // [M][rows]
    float *part;             // splits > 1: [splits][M][rows] partial sums, before srow and bias
    unsigned int *status;
};

struct LgUnit {
    int t0, r0, z, kb0, nkb;
};

__device__ __forceinline__ LgUnit lg_unit(const LgArgs &a, int u) {
    LgUnit w;
    const int tt = u % a.t_tiles, rest = u / a.t_tiles;
    w.t0 = tt * LN;
    w.r0 = (rest % a.r_tiles) * LM;
    w.z = rest / a.r_tiles;
    w.kb0 = w.z * a.kb_per;
    w.nkb = min((a.K + LK - 1) / LK - w.kb0, a.kb_per);
    return w;
}

// 16 int8 codes -> 8 half2 words in order: the byte with its sign bit flipped
// is c + 128 in [1, 255]; as the low byte of 0x64xx it is the fp16 1152 + c,
// and one exact subtraction of 1152 leaves c.
__device__ __forceinline__ void codes16_to_half(const uint4 w, uint32_t *o) {
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
    const __half2 bias = __half2half2(__ushort_as_half((unsigned short)0x6480));   // 1152
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint32_t u = ww[k] ^ 0x80808080u;
        const uint32_t p01 = __byte_perm(u, 0x64646464u, 0x5140), p23 = __byte_perm(u, 0x64646464u, 0x7362);
        const __half2 a = __hsub2(*reinterpret_cast<const __half2 *>(&p01), bias);
        const __half2 b = __hsub2(*reinterpret_cast<const __half2 *>(&p23), bias);
        o[2 * k] = *reinterpret_cast<const uint32_t *>(&a);
        o[2 * k + 1] = *reinterpret_cast<const uint32_t *>(&b);
    }
}

__global__ void __launch_bounds__(kLThreads, 1)
    logic_gemm_kernel(const __grid_constant__ CUtensorMap mC, const __grid_constant__ CUtensorMap mBh,
                      const __grid_constant__ CUtensorMap mBl, const LgArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    uint64_t *bfull = reinterpret_cast<uint64_t *>(smem + kLStages * kLStage);   // token and code tiles landed
    uint64_t *afull = bfull + kLStages;      // the stage's four worker warps stored their A rows
    uint64_t *kempty = afull + kLStages;     // the K-block's MMAs completed: stage free
    uint64_t *sfull = kempty + kLStages;     // a slot holds a unit's complete sums
    uint64_t *sempty = sfull + kLSlots;      // the epilogue has read the slot
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sempty + kLSlots);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_my = a.units > (int)blockIdx.x ? (a.units - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kLStages; ++s) {
            mbar_init(&bfull[s], 1);
            mbar_init(&afull[s], 4);
            mbar_init(&kempty[s], 1);
        }
        for (int s = 0; s < kLSlots; ++s) {
            mbar_init(&sfull[s], 1);
            mbar_init(&sempty[s], kLWorkers);
        }
        fence_barrier_init();
        prefetch_tensormap(&mC);
        prefetch_tensormap(&mBh);
        prefetch_tensormap(&mBl);
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(kLTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    }
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;
    // every role reads the same word; with the whole of TMEM allocated the
    // base is column 0, and anything else raises a status bit and skips the work
    const bool tmem_ok = tmem == 0;
    if (!tmem_ok && threadIdx.x == 0) atomicOr(a.status, LALB_STATUS_WAIT_TIMEOUT);
    // K-blocks are numbered across this CTA's units (kbg): stage kbg % 4,
    // phase (kbg / 4) & 1
    if (warp == 0) {
        if (lane == 0 && tmem_ok) {
            // The codes are never the preceding kernel's output (it prepares
            // the tokens), so the code tiles of the first stages go out
            // before the dependency wait; each stage's one expect_tx covers
            // them and the token tiles that follow after it.
            int npre = 0;
            if (n_my > 0) {
                const LgUnit w0 = lg_unit(a, blockIdx.x);
                npre = min(w0.nkb, kLStages);
                for (int kb = 0; kb < npre; ++kb) {
                    mbar_arrive_expect_tx(&bfull[kb], kLStage);
                    tma2d(smem + (size_t)kb * kLStage + 2 * kLB, &mC, (w0.kb0 + kb) * LK, w0.r0, &bfull[kb]);
                }
            }
            pdl_wait();   // the token parts are the preceding kernel's output
            pdl_launch_dependents();
            int kbg = 0;
            bool ok = true;
            for (int j = 0; j < n_my && ok; ++j) {
                const LgUnit w = lg_unit(a, blockIdx.x + j * gridDim.x);
                for (int kb = 0; kb < w.nkb; ++kb, ++kbg) {
                    const int s = kbg % kLStages;
                    const uint32_t use = kbg / kLStages;
                    if (use > 0 && !mbar_wait_bounded(&kempty[s], (use - 1) & 1u, a.status)) {
                        ok = false;
                        break;
                    }
                    uint8_t *st = smem + (size_t)s * kLStage;
                    if (kbg >= npre) {
                        mbar_arrive_expect_tx(&bfull[s], kLStage);
                        tma2d(st + 2 * kLB, &mC, (w.kb0 + kb) * LK, w.r0, &bfull[s]);
                    }
                    tma2d(st, &mBh, (w.kb0 + kb) * LK, w.t0, &bfull[s]);
                    tma2d(st + kLB, &mBl, (w.kb0 + kb) * LK, w.t0, &bfull[s]);
                }
            }
        } else {
            pdl_wait();
            pdl_launch_dependents();
        }
    } else if (warp == 1) {
        pdl_wait();
        pdl_launch_dependents();
        const uint32_t stage0 = smem_u32(smem);
        bool ok = tmem_ok;
        int kbg = 0;
        for (int j = 0; j < n_my && ok; ++j) {
            const LgUnit w = lg_unit(a, blockIdx.x + j * gridDim.x);
            const int slot = j % kLSlots;
            if (j >= kLSlots && !warp_wait_fast(&sempty[slot], (uint32_t)(j / kLSlots - 1) & 1u, a.status)) {
                ok = false;
                break;
            }
            const uint32_t d = slot * LN;
            for (int kb = 0; kb < w.nkb; ++kb, ++kbg) {
                const int s = kbg % kLStages;
                const uint32_t ph = (uint32_t)(kbg / kLStages) & 1u;
                if (!warp_wait_fast(&bfull[s], ph, a.status) || !warp_wait_fast(&afull[s], ph, a.status)) {
                    ok = false;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t bst = stage0 + (uint32_t)s * kLStage;
                const uint32_t ta = kLAColBase + s * kLAColW;
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {   // 16 codes (8 columns of A) per step
                    mma_f16_ta(d, ta + kk * 8, sw128_desc(bst + kk * 32), kIdescLogic, (kb | kk) != 0 ? 1u : 0u);
                    mma_f16_ta(d, ta + kk * 8, sw128_desc(bst + kLB + kk * 32), kIdescLogic, 1u);
                }
                commit_elect(&kempty[s]);
            }
            if (ok) commit_elect(&sfull[slot]);
        }
    } else {
        pdl_wait();
        pdl_launch_dependents();
        const int q = warp & 3;             // TMEM lane quarter: rows 32 q .. 32 q + 31
        const int g = (warp - 2) >> 2;      // K-blocks with kbg % 4 == g; tokens 32 g .. of the epilogue
        const int row = q * 32 + lane;
        const uint32_t lanes = (uint32_t)(q * 32) << 16;
        bool ok = tmem_ok;
        auto epilogue = [&](int j) -> bool {
            const LgUnit w = lg_unit(a, blockIdx.x + j * gridDim.x);
            const int slot = j % kLSlots;
            if (!warp_wait_fast(&sfull[slot], (uint32_t)(j / kLSlots) & 1u, a.status)) return false;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            float S[32];
            const uint32_t tb = lanes + slot * LN + g * 32;
            tmem_ld16(tb, *reinterpret_cast<float(*)[16]>(S));
            tmem_ld16(tb + 16, *reinterpret_cast<float(*)[16]>(S + 16));
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&sempty[slot]);
            const int r = w.r0 + row;
            if (r < a.rows) {
                const bool whole = a.splits == 1;
                const float sr = whole ? __ldg(a.srow + r) : 1.0f;
                const float b = whole && a.bias ? __ldg(a.bias + r) : 0.0f;
                float *out = whole ? a.Y : a.part + (size_t)w.z * a.M * a.rows;
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const int t = w.t0 + g * 32 + i;
                    if (t < a.M) {
                        const float y = __fmul_rn(S[i], __ldg(a.inv + t));   // an exact power of two
                        out[(size_t)t * a.rows + r] = whole ? __fadd_rn(__fmul_rn(y, sr), b) : y;
                    }
                }
            }
            return true;
        };
        int kbg = 0;
        for (int j = 0; j < n_my && ok; ++j) {
            const LgUnit w = lg_unit(a, blockIdx.x + j * gridDim.x);
            for (int kb = 0; kb < w.nkb; ++kb, ++kbg) {
                if (kbg % kLStages != g) continue;
                // the stage's tiles landed (which also means that the MMAs of
                // K-block kbg - 4, the last readers of A stage g, completed)
                if (!warp_wait_fast(&bfull[g], (uint32_t)(kbg / kLStages) & 1u, a.status)) {
                    ok = false;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                // the code tile: 64-byte rows, chunk c of row r at chunk c ^ ((r >> 1) & 3)
                const uint8_t *crow = smem + (size_t)g * kLStage + 2 * kLB + row * 64;
                uint32_t v[32];
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const uint4 cw = *reinterpret_cast<const uint4 *>(crow + ((c ^ ((row >> 1) & 3)) << 4));
                    codes16_to_half(cw, v + 8 * c);
                }
                tmem_st32(lanes + kLAColBase + g * kLAColW, v);
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(&afull[g]);
            }
            // the previous unit's sums (its MMAs ran while this unit's codes were decoded)
            if (ok && j > 0) ok = epilogue(j - 1);
        }
        if (ok && n_my > 0) ok = epilogue(n_my - 1);
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    }
    __syncwarp();   // warp 0's lane 0 ran the producer loop alone: the barrier below is warp-aligned
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kLTmemCols)
                     : "memory");
    }
}

// Tokens: one CTA per row of X.  e = the power of two that puts the row's
// largest |x| in [2^14, 2^15) (0 for an all-zero row); Bhi = fp16(x 2^e),
// Blo = fp16(x 2^e - Bhi), inv = 2^-e.  K % 8 == 0, X rows 16-byte aligned.
__global__ void __launch_bounds__(kLActThreads) logic_act_kernel(const float *__restrict__ X, int K,
                                                                 __half *__restrict__ Bh,
                                                                 __half *__restrict__ Bl,
                                                                 float *__restrict__ inv) {
    __shared__ float s_amax[kLActThreads / 32];
    const int t = blockIdx.x;
    const float4 *x = reinterpret_cast<const float4 *>(X + (size_t)t * K);
    // X may be the preceding kernel's output, and the preceding GEMM reads
    // the token parts written here
    pdl_wait();
    pdl_launch_dependents();
    float m = 0.0f;
    for (int i = threadIdx.x; i < K / 4; i += blockDim.x) {
        const float4 v = x[i];
        m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) s_amax[threadIdx.x >> 5] = m;
    __syncthreads();
    m = 0.0f;
    for (int w = 0; w < kLActThreads / 32; ++w) m = fmaxf(m, s_amax[w]);
    int e = 0;
    if (m > 0.0f) {
        int ex;
        frexpf(m, &ex);   // m in [2^(ex-1), 2^ex)
        e = 15 - ex;
    }
    for (int i = threadIdx.x; i < K / 8; i += blockDim.x) {
        const float4 v0 = x[2 * i], v1 = x[2 * i + 1];
        const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        __align__(16) __half h[8], l[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float s = ldexpf(v[j], e);   // exact: a power-of-two scale, |s| < 2^15
            h[j] = __float2half_rn(s);
            l[j] = __float2half_rn(s - __half2float(h[j]));
        }
        reinterpret_cast<uint4 *>(Bh + (size_t)t * K)[i] = *reinterpret_cast<const uint4 *>(h);
        reinterpret_cast<uint4 *>(Bl + (size_t)t * K)[i] = *reinterpret_cast<const uint4 *>(l);
    }
    if (threadIdx.x == 0) inv[t] = ldexpf(1.0f, -e);
}

// The K splits: Y[t][n] = (sum over z in split order of part[z][t][n]) srow[n] + bias[n].
__global__ void __launch_bounds__(256) logic_split_sum_kernel(const float *__restrict__ part, int splits,
                                                             int M, int rows, const float *__restrict__ srow,
                                                             const float *__restrict__ bias,
                                                             float *__restrict__ Y) {
    pdl_wait();   // the partial sums are the GEMM's output
    pdl_launch_dependents();
    const long long n = (long long)M * rows;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        float v = __ldcg(part + i);
        for (int z = 1; z < splits; ++z) v = __fadd_rn(v, __ldcg(part + z * n + i));
        const int r = (int)(i % rows);
        Y[i] = __fadd_rn(__fmul_rn(v, srow[r]), bias ? bias[r] : 0.0f);
    }
}

int tokens_padded(int M) { return (M + LN - 1) / LN * LN; }
size_t up256(size_t n) { return (n + 255) / 256 * 256; }
size_t tok_bytes(int M, int K) { return up256((size_t)M * K * sizeof(__half)); }

// K split of a call with fewer output tiles than the B200's 148 SMs. Cost
// model, in K-blocks of MMA work: waves x (K-blocks per CTA + a CTA's fixed
// cost), plus the split-sum launch.
void split_plan(int rows, int K, int M, int *splits, int *kb_per) {
    const int tiles = ((rows + LM - 1) / LM) * (tokens_padded(M) / LN), nkb = (K + LK - 1) / LK;
    int best = 1, best_per = nkb;
    if (tiles < kLSplitSms) {
        long long best_cost = (long long)nkb + kLCtaCost;
        for (int s = 2; s <= std::min(nkb, kLMaxSplits); ++s) {
            const int per = (nkb + s - 1) / s, se = (nkb + per - 1) / per;
            const long long waves = ((long long)tiles * se + kLSplitSms - 1) / kLSplitSms;
            const long long cost = waves * (per + kLCtaCost) + kLSumCost;
            if (cost < best_cost) best_cost = cost, best = se, best_per = per;
        }
    }
    *splits = best;
    *kb_per = best_per;
}

size_t part_bytes(int rows, int K, int M) {
    int splits, per;
    split_plan(rows, K, M, &splits, &per);
    return splits > 1 ? up256((size_t)splits * M * rows * sizeof(float)) : 0;
}

}  // namespace

size_t lalb_logic_gemm_ws_bytes(int rows, int K, int max_M) {
    // the token parts for max_M rows, and the largest partial-sum buffer of
    // any M <= max_M (the split depends on the number of 128-token tiles)
    size_t part = 0;
    for (int tt = 1; tt <= tokens_padded(max_M) / LN; ++tt)
        part = std::max(part, part_bytes(rows, K, std::min(tt * LN, max_M)));
    return 2 * tok_bytes(max_M, K) + up256((size_t)tokens_padded(max_M) * sizeof(float)) + part;
}

int lalb_logic_gemm(lalb_ctx *ctx, const int8_t *codes, const float *srow, const float *bias, int rows, int K,
                    const float *X, int M, void *ws, size_t ws_bytes, float *Y, cudaStream_t s) {
    if (!codes || !srow || !X || !Y || !ws || rows <= 0 || K <= 0 || K % 32 || M <= 0)
        return lalb_fail(ctx, LALB_ERR_INVALID, "logic gemm: bad arguments");
    if (((uintptr_t)codes | (uintptr_t)X) & 15u)
        return lalb_fail(ctx, LALB_ERR_INVALID, "logic gemm: codes and X must be 16-byte aligned");
    int splits, kb_per;
    split_plan(rows, K, M, &splits, &kb_per);
    const size_t need = 2 * tok_bytes(M, K) + up256((size_t)tokens_padded(M) * sizeof(float)) + part_bytes(rows, K, M);
    if (need > ws_bytes) return lalb_fail(ctx, LALB_ERR_INVALID, "logic gemm: workspace too small");
    uint8_t *w = static_cast<uint8_t *>(ws);
    __half *Bh = reinterpret_cast<__half *>(w);
    __half *Bl = reinterpret_cast<__half *>(w + tok_bytes(M, K));
    float *inv = reinterpret_cast<float *>(w + 2 * tok_bytes(M, K));
    float *part = reinterpret_cast<float *>(w + 2 * tok_bytes(M, K) + up256((size_t)tokens_padded(M) * sizeof(float)));
    int st;
    if ((st = launch_pdl(ctx, (const void *)logic_act_kernel, dim3(M), dim3(kLActThreads), 0, s,
                         {&X, &K, &Bh, &Bl, &inv})))
        return st;
    LALB_LAUNCH_CHECK(ctx, "logic_act_kernel");
    CUtensorMap mC, mBh, mBl;
    if ((st = map2d(ctx, &mC, codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, rows, LK, LM, CU_TENSOR_MAP_SWIZZLE_64B)))
        return st;
    if ((st = map2d(ctx, &mBh, Bh, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, K, M, LK, LN, CU_TENSOR_MAP_SWIZZLE_128B)))
        return st;
    if ((st = map2d(ctx, &mBl, Bl, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, K, M, LK, LN, CU_TENSOR_MAP_SWIZZLE_128B)))
        return st;
    if ((st = lalb_set_smem_attr(ctx, (const void *)logic_gemm_kernel, (int)kLSmem))) return st;
    LgArgs a = {};
    a.rows = rows;
    a.K = K;
    a.M = M;
    a.t_tiles = tokens_padded(M) / LN;
    a.r_tiles = (rows + LM - 1) / LM;
    a.splits = splits;
    a.kb_per = kb_per;
    a.units = a.t_tiles * a.r_tiles * splits;
    a.inv = inv;
    a.srow = srow;
    a.bias = bias;
    a.Y = Y;
    a.part = part;
    a.status = &ctx->scratch->status;
    // persistent: at most one CTA per SM, each taking every gridDim.x-th unit
    const dim3 grid(std::min(a.units, ctx->sm_count));
    if ((st = launch_pdl(ctx, (const void *)logic_gemm_kernel, grid, dim3(kLThreads), kLSmem, s,
                         {&mC, &mBh, &mBl, &a})))
        return st;
    LALB_LAUNCH_CHECK(ctx, "logic_gemm_kernel");
    if (splits > 1) {
        const long long n = (long long)M * rows;
        const int blocks = (int)std::min<long long>((n + 255) / 256, (long long)ctx->sm_count * 8);
        if ((st = launch_pdl(ctx, (const void *)logic_split_sum_kernel, dim3(blocks), dim3(256), 0, s,
                             {&part, &splits, &M, &rows, &srow, &bias, &Y})))
            return st;
        LALB_LAUNCH_CHECK(ctx, "logic_split_sum_kernel");
    }
    return LALB_OK;
}
