// lalb_tc_gemm.cu -- tcgen05 (5th-generation tensor core) GEMM with fp32
// operands carried exactly as sums of tf32 parts.
//
//   Y[m][n] = rowscale[m] * colscale[n] * sum_k A[m][k] * B[n][k] + bias[n]
//
// A (activations, [M][K]) and B (weights, [N][K]) are row-major fp32 in HBM,
// both K-major.  B is given as one or two tf32 parts (x = hi + lo, each part
// exactly representable in tf32); A either the same way or raw (split_a),
// in which case the kernel forms its parts on chip: hi is the raw fp32 read
// by the tensor core as its tf32 truncation, lo = x - hi is written next to
// it by converter warps.  The kernel accumulates hi*hi + lo*hi (+ hi*lo when
// B has two parts) in fp32 in TMEM.  This is the seed STE model's forward
// (BinLayer) on tensor cores: the reference computes it in fp32 on the CPU
// (runtime/lal_runtime.c bin_forward :1852-1938, bin_forward_pure_float
// :543-582).
//
// tc_gemm_tf32_kernel, persistent: one CTA per SM walks the output tiles of
// 128 x bn (bn = 128, or 256 over many tiles; tile t, t + grid, ...), 10 warps:
//   warp 0     TMA producer: per 32-wide K-block, 2-D tiled copies
//              (128-byte swizzle) of the A and B parts into a ring of 4 slots
//              (3 when B has two parts), full mbarrier per slot;
//   warp 1     allocates all 512 TMEM columns and issues tcgen05.mma
//              (kind::tf32, M=128, N=bn, K=8 per instruction) from one lane.
//              K-block kb of a tile goes to accumulator kb % nacc of the
//              tile's accumulator group; with short K there are two groups,
//              so the next tile's MMAs run while the epilogue drains the
//              previous tile; long K uses one group of more accumulators
//              (shorter fp32 accumulation chains in the tensor core);
//   warps 2-5  epilogue: wait for the group (commit), read each warp's 32
//              TMEM lanes (= rows) 32 columns at a time from every
//              accumulator (tcgen05.ld 32x32b.x32), add them, free the group,
//              transpose through shared memory and write 128-byte row
//              segments with the scales and bias;
//   warps 6-9  converters (raw A only): A's lo part per slot.
// Rows-as-M (swap, 128-wide tiles with two A parts and one B part): the MMA
// takes B's 128 rows as M and A's hi and lo tiles, adjacent in the slot, as
// one N = 256 operand, so B is read once per step instead of twice; TMEM
// lanes are then output columns and the epilogue stores rows from registers.
// tc_gemm_tf32_splitk_kernel: outputs with few tiles; a cluster of S CTAs
// shares a tile along K and sums the partial tiles through distributed
// shared memory (its comment below).  The host picks the tile width and S.
// Every wait is bounded; on expiry the kernel raises the status word and
// still drains and frees its TMEM.
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "lalb_internal.cuh"
#include "lalb_tc_gemm.cuh"

using namespace lalb;

namespace {

constexpr int BM = 128, BN = 128, BK = 32;     // BK fp32 = 128 B: one 128-byte swizzle row
constexpr int kBNWide = 256;                    // wide tiles: A read once for 256 output columns
constexpr int kMaxStages = 4;                   // ring slots: 4 x 48 KB (one B part) or 3 x 64 KB
constexpr int kTmemCols = 512;                  // the whole TMEM of the SM: 4 accumulators of 128 columns
constexpr int kLongK = 16;                      // K-blocks above which one group of 4 accumulators is used
constexpr int kEpiWarpsTc = 4;
constexpr int kConvWarps = 4;                   // A given as raw fp32: its lo part formed in shared memory
constexpr int kConvWarp0 = 2 + kEpiWarpsTc;
constexpr int kTcThreads = 32 * (2 + kEpiWarpsTc + kConvWarps);
constexpr uint32_t kATile = BM * BK * 4;       // 16 KB
constexpr uint32_t kBTile = BN * BK * 4;       // 16 KB
// stage: A hi | A lo | B hi | B lo
constexpr uint32_t kStageBytes = 2 * kATile + 2 * kBTile;
constexpr uint32_t kRingBytes = 3 * kStageBytes;
constexpr uint32_t kEpiBytes = 4 * 32 * 33 * 4;             // per-warp 32x32 transpose
constexpr uint32_t kTcSmem = 1024 /* alignment slack */ + kRingBytes + kEpiBytes + 256;

// K-major operand tile with 128-byte swizzle (the TMA layout): rows of
// 128 bytes, 8-row groups 1024 bytes apart.  Descriptor fields: start
// address >> 4, leading byte offset 1 (unused for this layout), stride byte
// offset 1024 >> 4, version 1, layout type 2 (128-byte swizzle).
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// kind::tf32 instruction descriptor: fp32 accumulator, tf32 A and B, both
// K-major, M = 128, N = bn (128 or 256).
__host__ __device__ constexpr uint32_t idesc_tf32(int bn) {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(bn >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// 32 consecutive fp32 columns of this warp's 32 TMEM lanes (lane = row).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
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

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

// The low part of x below its tf32 truncation: x - (x with the low 13
// mantissa bits cleared), exact in fp32.  The tensor core reads the raw fp32
// x as its truncation (the low 13 bits are not used), so hi + lo = x up to
// the tf32 rounding of lo (2^-21 |x| at most).
__device__ __forceinline__ float tf32_trunc_lo(float x) {
    return __fsub_rn(x, __uint_as_float(__float_as_uint(x) & 0xFFFFE000u));
}

// One stage's A tile (raw fp32, 128 x 32) -> its lo part in the next 16 KB,
// same swizzled layout (element for element); 128 converter threads.  Then
// the writes are made visible to the tensor core (async proxy) and the warp
// arrives on conv.
__device__ __forceinline__ void convert_a_stage(uint8_t *stage, int ct, int lane, uint64_t *conv) {
    const float4 *src = reinterpret_cast<const float4 *>(stage);
    float4 *dst = reinterpret_cast<float4 *>(stage + BM * BK * 4);
#pragma unroll
    for (int i = 0; i < (BM * BK / 4) / (32 * kConvWarps); ++i) {
        const float4 x = src[ct + 32 * kConvWarps * i];
        dst[ct + 32 * kConvWarps * i] =
            make_float4(tf32_trunc_lo(x.x), tf32_trunc_lo(x.y), tf32_trunc_lo(x.z), tf32_trunc_lo(x.w));
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    if (lane == 0) mbar_arrive(conv);
}

struct TcArgs {
    int M, N, K;
    int a_parts, b_parts;       // parts multiplied: 1 or 2 each
    int a_loads;                // A parts loaded by TMA (1 when the kernel forms lo itself)
    int conv_a;                 // A is raw fp32: hi = its tf32 truncation, lo = A - hi
    int nstages;                // ring slots in use
    uint32_t stage_bytes;       // A hi | A lo | B hi (| B lo)
    int bn;                     // output tile width: 128 or 256
    int swap;                   // rows-as-M: B's tile is the MMA's M side, A's hi and lo
                                //   parts (adjacent in the slot) its N = 256 side, so one
                                //   MMA reads B once for both parts; TMEM lane = output
                                //   column, TMEM column = output row (hi, then lo at +128)
    int acc_cols;               // TMEM columns per accumulator
    uint32_t b_tile;            // bytes of one B part's tile: bn x BK fp32
    uint32_t idesc;             // MMA instruction descriptor for bn
    int tiles_n, tiles;         // output tiles along N, in all
    int nacc, ngroups;          // accumulators per tile, accumulator groups in TMEM
    int splits;                 // split-K kernel: CTAs of a cluster sharing a tile
    int y_vec4;                 // Y rows 16-byte aligned (N % 4 == 0, Y aligned)
    float *Y;                   // [M][N]
    const float *rowscale;      // [M] or null (1)
    const float *colscale;      // [N] or null (1)
    const float *bias;          // [N] or null (0)
    unsigned int *status;
};

__global__ void __launch_bounds__(kTcThreads, 1)
    tc_gemm_tf32_kernel(const __grid_constant__ CUtensorMap mA0, const __grid_constant__ CUtensorMap mA1,
                        const __grid_constant__ CUtensorMap mB0, const __grid_constant__ CUtensorMap mB1,
                        const TcArgs a) {
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte alignment for the swizzled tiles
    uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    uint8_t *stages = smem;
    float *epi = reinterpret_cast<float *>(smem + kRingBytes);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + kRingBytes + kEpiBytes);
    uint64_t *empty = full + kMaxStages;         // the stage's MMAs completed
    uint64_t *acc_full = empty + kMaxStages;     // [2] a tile's accumulators are complete
    uint64_t *acc_empty = acc_full + 2;         // [2] the epilogue has read them
    uint64_t *conv = acc_empty + 2;             // [stages] the stage's A lo part is formed
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(conv + kMaxStages);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nk = a.K / BK;

    if (threadIdx.x == 0) {
        // the TMA unit fetches the descriptors while the barriers and TMEM are set up
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&mA0)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&mA1)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&mB0)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&mB1)) : "memory");
        for (int s = 0; s < kMaxStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int g = 0; g < 2; ++g) {
            mbar_init(&acc_full[g], 1);
            mbar_init(&acc_empty[g], kEpiWarpsTc);
        }
        for (int st = 0; st < kMaxStages; ++st) mbar_init(&conv[st], kConvWarps);
        fence_barrier_init();
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
    // kernel's tail; its outputs (A) are read only after it completes
    pdl_wait();
    pdl_launch_dependents();

    const uint32_t stage_tx = (uint32_t)(a.a_loads * kATile + a.b_parts * a.b_tile);
    if (warp == 0) {
        if (lane == 0) {
            // ---- TMA producer ----
            uint32_t it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < a.tiles && ok; t += gridDim.x) {
                const int m0 = (t / a.tiles_n) * BM, n0 = (t % a.tiles_n) * a.bn;
                for (int kb = 0; kb < nk; ++kb, ++it) {
                    const int s = it % a.nstages;
                    const uint32_t use = it / a.nstages;
                    if (use > 0 && !mbar_wait_bounded(&empty[s], (use - 1) & 1u, a.status)) {
                        ok = false;
                        break;
                    }
                    uint8_t *st = stages + (size_t)s * a.stage_bytes;
                    mbar_arrive_expect_tx(&full[s], stage_tx);
                    tma_load_2d(st, &mA0, kb * BK, m0, &full[s]);
                    if (a.a_loads > 1) tma_load_2d(st + kATile, &mA1, kb * BK, m0, &full[s]);
                    tma_load_2d(st + 2 * kATile, &mB0, kb * BK, n0, &full[s]);
                    if (a.b_parts > 1) tma_load_2d(st + 2 * kATile + a.b_tile, &mB1, kb * BK, n0, &full[s]);
                }
            }
        }
    } else if (warp >= kConvWarp0) {
        // ---- A lo parts (raw fp32 A only) ----
        if (a.conv_a) {
            const int ct = threadIdx.x - 32 * kConvWarp0;
            uint32_t it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < a.tiles && ok; t += gridDim.x) {
                for (int kb = 0; kb < nk; ++kb, ++it) {
                    const int s = it % a.nstages;
                    ok = __all_sync(0xffffffffu, mbar_wait_bounded(&full[s], (it / a.nstages) & 1u, a.status));
                    if (!ok) break;
                    convert_a_stage(stages + (size_t)s * a.stage_bytes, ct, lane, &conv[s]);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---- MMA issuer ----
            uint32_t it = 0, ti = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < a.tiles && ok; t += gridDim.x, ++ti) {
                const int g = ti % a.ngroups;
                const uint32_t gu = ti / a.ngroups;
                if (gu > 0 && !mbar_wait_bounded(&acc_empty[g], (gu - 1) & 1u, a.status)) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                for (int kb = 0; kb < nk; ++kb, ++it) {
                    const int s = it % a.nstages;
                    // raw fp32 A: the converters' arrival implies the stage's TMA data too
                    if (!mbar_wait_bounded(a.conv_a ? &conv[s] : &full[s], (it / a.nstages) & 1u, a.status)) {
                        ok = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint32_t st = smem_u32(stages + (size_t)s * a.stage_bytes);
                    const uint32_t a0 = st, a1 = st + kATile, b0 = st + 2 * kATile, b1 = b0 + a.b_tile;
                    const uint32_t td = tmem + (uint32_t)((g * a.nacc + kb % a.nacc) * a.acc_cols);
                    uint32_t acc = kb >= a.nacc;   // the first block of an accumulator overwrites it
#pragma unroll
                    for (int k = 0; k < BK / 8; ++k) {   // 8 tf32 = 32 bytes per instruction
                        const uint32_t ko = k * 32;
                        if (a.swap) {   // B rows x (A hi rows ; A lo rows)
                            mma_tf32(td, sw128_kmajor_desc(b0 + ko), sw128_kmajor_desc(a0 + ko), a.idesc, acc);
                            acc = 1;
                            continue;
                        }
                        mma_tf32(td, sw128_kmajor_desc(a0 + ko), sw128_kmajor_desc(b0 + ko), a.idesc, acc);
                        acc = 1;
                        if (a.a_parts > 1)
                            mma_tf32(td, sw128_kmajor_desc(a1 + ko), sw128_kmajor_desc(b0 + ko), a.idesc, 1);
                        if (a.b_parts > 1)
                            mma_tf32(td, sw128_kmajor_desc(a0 + ko), sw128_kmajor_desc(b1 + ko), a.idesc, 1);
                    }
                    mma_commit(&empty[s]);   // the stage is free once these MMAs have read it
                }
                mma_commit(&acc_full[g]);    // arrives when every MMA of the tile has completed
            }
        }
    } else {
        // ---- epilogue: warps 2..5, TMEM lane quarter = warp % 4 ----
        const int q = warp & 3;
        float *st = epi + (size_t)(warp - 2) * 32 * 33;
        const int nacc = nk < a.nacc ? nk : a.nacc;
        uint32_t ti = 0;
        for (int t = blockIdx.x; t < a.tiles; t += gridDim.x, ++ti) {
            const int m0 = (t / a.tiles_n) * BM, n0 = (t % a.tiles_n) * a.bn;
            const int g = ti % a.ngroups;
            if (!mbar_wait_bounded(&acc_full[g], (ti / a.ngroups) & 1u, a.status)) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            if (a.swap) {
                // lane = output column n, TMEM columns = output rows: hi products
                // at c, lo products at c + 128; row stores are 128 bytes per warp
                const int n = n0 + q * 32 + lane;
                const bool ncol = n < a.N;
                const float cs = ncol && a.colscale ? a.colscale[n] : 1.0f;
                const float b = ncol && a.bias ? a.bias[n] : 0.0f;
                for (int c0 = 0; c0 < BM; c0 += 32) {
                    float sum[32];
#pragma unroll
                    for (int j = 0; j < 32; ++j) sum[j] = 0.0f;
                    for (int ai = 0; ai < nacc; ++ai) {
                        uint32_t r[32];
                        const uint32_t col = (uint32_t)((g * a.nacc + ai) * a.acc_cols + c0);
                        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + col, r);
#pragma unroll
                        for (int j = 0; j < 32; ++j) sum[j] = __fadd_rn(sum[j], __uint_as_float(r[j]));
                        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + col + BM, r);
#pragma unroll
                        for (int j = 0; j < 32; ++j) sum[j] = __fadd_rn(sum[j], __uint_as_float(r[j]));
                    }
                    if (c0 == BM - 32) {   // the group's last columns are in registers: free it
                        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&acc_empty[g]);
                    }
                    const int mrow = m0 + c0 + lane;
                    const float rs_lane = a.rowscale && mrow < a.M ? a.rowscale[mrow] : 1.0f;
                    float *yc = a.Y + (size_t)(m0 + c0) * a.N + n;
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const float rs = __shfl_sync(0xffffffffu, rs_lane, j);
                        if (m0 + c0 + j < a.M && ncol)
                            yc[(size_t)j * a.N] = __fadd_rn(__fmul_rn(__fmul_rn(sum[j], rs), cs), b);
                    }
                }
                continue;
            }
            for (int c0 = 0; c0 < a.bn; c0 += 32) {
                float sum[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) sum[j] = 0.0f;
                for (int ai = 0; ai < nacc; ++ai) {
                    uint32_t r[32];
                    tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)((g * a.nacc + ai) * a.bn + c0), r);
#pragma unroll
                    for (int j = 0; j < 32; ++j) sum[j] = __fadd_rn(sum[j], __uint_as_float(r[j]));
                }
                if (c0 == a.bn - 32) {   // the group's last columns are in registers: free it
                    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&acc_empty[g]);
                }
                // lane holds row q*32 + lane, columns c0..c0+31
#pragma unroll
                for (int j = 0; j < 32; ++j) st[lane * 33 + j] = sum[j];
                __syncwarp();
                const int n = n0 + c0 + lane;
                const bool ncol = n < a.N;
                const float cs = ncol && a.colscale ? a.colscale[n] : 1.0f;
                const float b = ncol && a.bias ? a.bias[n] : 0.0f;
                // lane's row scale, broadcast per row below; rows unrolled so
                // that the loads and stores of several rows are in flight
                const int mrow = m0 + q * 32 + lane;
                const float rs_lane = a.rowscale && mrow < a.M ? a.rowscale[mrow] : 1.0f;
                float *yc = a.Y + (size_t)(m0 + q * 32) * a.N + n;
#pragma unroll 8
                for (int j = 0; j < 32; ++j) {
                    const float rs = __shfl_sync(0xffffffffu, rs_lane, j);
                    if (m0 + q * 32 + j < a.M && ncol)
                        yc[(size_t)j * a.N] = __fadd_rn(__fmul_rn(__fmul_rn(st[j * 33 + lane], rs), cs), b);
                }
                __syncwarp();
            }
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    }
    __syncwarp();   // lane 0 of warps 0 and 1 ran their loops alone: the barrier below is warp-aligned
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(kTmemCols)
                     : "memory");
    }
}

__device__ __forceinline__ void cluster_sync_all() {
    __syncwarp();   // .aligned: the whole warp executes the barrier together (a lane may have looped alone)
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Split-K over a thread-block cluster, for outputs with few tiles (the seed
// model's o and down projections: 32 tiles of 128 x 128 on 148 SMs).  The
// S = a.splits CTAs of a cluster share one output tile: CTA r (its rank in
// the cluster) accumulates K-blocks [r nk / S, (r+1) nk / S) in TMEM, writes
// its fp32 partial tile into its own shared memory (the operand ring, idle by
// then), and after a cluster barrier sums rows [r BM / S, (r+1) BM / S) of
// all S partials through distributed shared memory, in rank order, applying
// the scales and bias.  A second cluster barrier keeps every partial alive
// until all readers are done.  Same warp roles as tc_gemm_tf32_kernel.
constexpr int kSplitAcc = 2;   // accumulators per split (K-blocks round-robin)

__global__ void __launch_bounds__(kTcThreads, 1)
    tc_gemm_tf32_splitk_kernel(const __grid_constant__ CUtensorMap mA0, const __grid_constant__ CUtensorMap mA1,
                               const __grid_constant__ CUtensorMap mB0, const __grid_constant__ CUtensorMap mB1,
                               const TcArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    uint8_t *stages = smem;
    float *part = reinterpret_cast<float *>(smem);   // [BM][bn] partial, reuses the ring
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + kRingBytes + kEpiBytes);
    uint64_t *empty = full + kMaxStages;
    uint64_t *acc_full = empty + kMaxStages;
    uint64_t *conv = acc_full + 2;              // [stages] the stage's A lo part is formed
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(conv + kMaxStages);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = a.splits;
    uint32_t rank;
    asm("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
    const int t = blockIdx.x / S;
    const int m0 = (t / a.tiles_n) * BM, n0 = (t % a.tiles_n) * a.bn;
    const int nk = a.K / BK;
    const int kb0 = (int)rank * nk / S, kb1 = ((int)rank + 1) * nk / S;

    if (threadIdx.x == 0) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&mA0)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&mA1)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&mB0)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&mB1)) : "memory");
        for (int st = 0; st < kMaxStages; ++st) {
            mbar_init(&full[st], 1);
            mbar_init(&empty[st], 1);
        }
        mbar_init(&acc_full[0], 1);
        for (int st = 0; st < kMaxStages; ++st) mbar_init(&conv[st], kConvWarps);
        fence_barrier_init();
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
    pdl_wait();
    pdl_launch_dependents();

    const uint32_t stage_tx = (uint32_t)(a.a_loads * kATile + a.b_parts * a.b_tile);
    if (warp == 0) {
        if (lane == 0) {
            for (int kb = kb0; kb < kb1; ++kb) {
                const uint32_t it = (uint32_t)(kb - kb0);
                const int st = it % a.nstages;
                const uint32_t use = it / a.nstages;
                if (use > 0 && !mbar_wait_bounded(&empty[st], (use - 1) & 1u, a.status)) break;
                uint8_t *sp = stages + (size_t)st * a.stage_bytes;
                mbar_arrive_expect_tx(&full[st], stage_tx);
                tma_load_2d(sp, &mA0, kb * BK, m0, &full[st]);
                if (a.a_loads > 1) tma_load_2d(sp + kATile, &mA1, kb * BK, m0, &full[st]);
                tma_load_2d(sp + 2 * kATile, &mB0, kb * BK, n0, &full[st]);
                if (a.b_parts > 1) tma_load_2d(sp + 2 * kATile + a.b_tile, &mB1, kb * BK, n0, &full[st]);
            }
        }
        __syncwarp();
    } else if (warp >= kConvWarp0) {
        if (a.conv_a) {
            const int ct = threadIdx.x - 32 * kConvWarp0;
            for (int kb = kb0; kb < kb1; ++kb) {
                const uint32_t it = (uint32_t)(kb - kb0);
                const int st = it % a.nstages;
                if (!__all_sync(0xffffffffu, mbar_wait_bounded(&full[st], (it / a.nstages) & 1u, a.status)))
                    break;
                convert_a_stage(stages + (size_t)st * a.stage_bytes, ct, lane, &conv[st]);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            for (int kb = kb0; kb < kb1; ++kb) {
                const uint32_t it = (uint32_t)(kb - kb0);
                const int st = it % a.nstages;
                if (!mbar_wait_bounded(a.conv_a ? &conv[st] : &full[st], (it / a.nstages) & 1u, a.status))
                    break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t sp = smem_u32(stages + (size_t)st * a.stage_bytes);
                const uint32_t a0 = sp, a1 = sp + kATile, b0 = sp + 2 * kATile, b1 = b0 + a.b_tile;
                const uint32_t td = tmem + (uint32_t)((it % kSplitAcc) * a.acc_cols);
                uint32_t acc = it >= (uint32_t)kSplitAcc;   // the first block of an accumulator overwrites it
#pragma unroll
                for (int k = 0; k < BK / 8; ++k) {
                    const uint32_t ko = k * 32;
                    if (a.swap) {   // B rows x (A hi rows ; A lo rows)
                        mma_tf32(td, sw128_kmajor_desc(b0 + ko), sw128_kmajor_desc(a0 + ko), a.idesc, acc);
                        acc = 1;
                        continue;
                    }
                    mma_tf32(td, sw128_kmajor_desc(a0 + ko), sw128_kmajor_desc(b0 + ko), a.idesc, acc);
                    acc = 1;
                    if (a.a_parts > 1) mma_tf32(td, sw128_kmajor_desc(a1 + ko), sw128_kmajor_desc(b0 + ko), a.idesc, 1);
                    if (a.b_parts > 1) mma_tf32(td, sw128_kmajor_desc(a0 + ko), sw128_kmajor_desc(b1 + ko), a.idesc, 1);
                }
                mma_commit(&empty[st]);
            }
            mma_commit(&acc_full[0]);   // every MMA above (and the stage reads) completed
        }
        __syncwarp();
    } else {
        // ---- the partial tile into shared memory: row R = q*32 + lane, its
        // 16-byte chunk c (of 32) at chunk c ^ (R & 31) ----
        const int q = warp & 3, R = q * 32 + lane;
        const int nacc = kb1 - kb0 < kSplitAcc ? kb1 - kb0 : kSplitAcc;
        // warp-uniform, so that the tcgen05.ld below stay converged
        const bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(&acc_full[0], 0, a.status));
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (a.swap) {
            // lane = output column R (of bn = 128), TMEM columns = output rows
            // (hi at c, lo at c + 128): element (row t, column R) goes to the
            // same swizzled place as above, t * bn + 4 ((R >> 2) ^ (t & 31)) + (R & 3)
            for (int c0 = 0; c0 < BM; c0 += 32) {
                float sum[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) sum[j] = 0.0f;
                for (int ai = 0; ai < nacc && ok; ++ai) {
                    uint32_t r[32];
                    const uint32_t col = (uint32_t)(ai * a.acc_cols + c0);
                    tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + col, r);
#pragma unroll
                    for (int j = 0; j < 32; ++j) sum[j] = __fadd_rn(sum[j], __uint_as_float(r[j]));
                    tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + col + BM, r);
#pragma unroll
                    for (int j = 0; j < 32; ++j) sum[j] = __fadd_rn(sum[j], __uint_as_float(r[j]));
                }
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int t = c0 + j;
                    part[(size_t)t * a.bn + 4 * ((R >> 2) ^ (t & 31)) + (R & 3)] = sum[j];
                }
            }
        }
        for (int c0 = 0; c0 < a.bn && !a.swap; c0 += 32) {
            float sum[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) sum[j] = 0.0f;
            for (int ai = 0; ai < nacc && ok; ++ai) {
                uint32_t r[32];
                tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(ai * a.acc_cols + c0), r);
#pragma unroll
                for (int j = 0; j < 32; ++j) sum[j] = __fadd_rn(sum[j], __uint_as_float(r[j]));
            }
            float4 *row = reinterpret_cast<float4 *>(part + (size_t)R * a.bn);
#pragma unroll
            for (int i = 0; i < 8; ++i)
                row[((c0 >> 2) + i) ^ (R & 31)] =
                    make_float4(sum[4 * i], sum[4 * i + 1], sum[4 * i + 2], sum[4 * i + 3]);
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    }
    cluster_sync_all();   // every CTA's partial is in its shared memory

    if (warp >= 2 && warp < kConvWarp0) {
        // ---- rows [rank BM/S, (rank+1) BM/S): sum the S partials, rank order ----
        const int r0 = (int)rank * BM / S, r1 = ((int)rank + 1) * BM / S, e = warp - 2;
        for (int c = lane; c < a.bn / 4; c += 32) {   // 16-byte chunk: columns 4c .. 4c+3
            const int n = n0 + 4 * c;
            float cs[4], bs[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const bool in = n + i < a.N;
                cs[i] = in && a.colscale ? a.colscale[n + i] : 1.0f;
                bs[i] = in && a.bias ? a.bias[n + i] : 0.0f;
            }
            for (int R = r0 + e; R < r1; R += kEpiWarpsTc) {
                const int m = m0 + R;
                const uint32_t off = smem_u32(part) + (uint32_t)((R * a.bn + 4 * (c ^ (R & 31))) * 4);
                // every partial's chunk in flight at once, then added in rank order
                float4 pj[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    if (j < S) {
                        uint32_t raddr;
                        asm("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(raddr) : "r"(off), "r"(j));
                        asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                                     : "=f"(pj[j].x), "=f"(pj[j].y), "=f"(pj[j].z), "=f"(pj[j].w)
                                     : "r"(raddr));
                    }
                }
                float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    if (j < S) {
                        v[0] = __fadd_rn(v[0], pj[j].x);
                        v[1] = __fadd_rn(v[1], pj[j].y);
                        v[2] = __fadd_rn(v[2], pj[j].z);
                        v[3] = __fadd_rn(v[3], pj[j].w);
                    }
                }
                if (m < a.M) {
                    const float rs = a.rowscale ? a.rowscale[m] : 1.0f;
                    float o[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) o[i] = __fadd_rn(__fmul_rn(__fmul_rn(v[i], rs), cs[i]), bs[i]);
                    float *yp = a.Y + (size_t)m * a.N + n;
                    if (a.y_vec4 && n + 3 < a.N) {
                        *reinterpret_cast<float4 *>(yp) = make_float4(o[0], o[1], o[2], o[3]);
                    } else {
#pragma unroll
                        for (int i = 0; i < 4; ++i)
                            if (n + i < a.N) yp[i] = o[i];
                    }
                }
            }
        }
    }
    cluster_sync_all();   // no CTA leaves while the others still read its partial
    if (warp == 1) {
        __syncwarp();
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(kTmemCols)
                     : "memory");
    }
}

// ---- tensor maps ----------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// Row-major fp32 [rows][K], box 32 (K) x box_rows, 128-byte swizzle; rows
// past the end read as zeros.
int make_map(lalb_ctx *ctx, CUtensorMap *m, const float *base, int rows, int K, int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return lalb_fail(ctx, LALB_ERR_CUDA, "tc_gemm: cuTensorMapEncodeTiled unavailable");
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)K * 4};
    const cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(base), dims, strides,
                          box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return lalb_fail(ctx, LALB_ERR_CUDA, "tc_gemm: tensor map encode (%d)", (int)r);
    return LALB_OK;
}

}  // namespace

namespace {

// Launch with a cluster of `cluster` CTAs along x and programmatic dependent
// launch allowed.
int launch_cluster_pdl(lalb_ctx *ctx, const void *fn, dim3 grid, dim3 block, size_t smem, int cluster,
                       cudaStream_t s, std::initializer_list<void *> args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)cluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    void *params[8];
    int i = 0;
    for (void *p : args) params[i++] = p;
    LALB_CUDA_TRY(ctx, cudaLaunchKernelExC(&cfg, fn, params));
    return LALB_OK;
}

// Clusters of S split-K CTAs that can be resident at once on this device
// (0 when the query fails), cached per device and S.
int splitk_clusters_fit(lalb_ctx *ctx, int S) {
    static std::mutex mu;
    static int cache[64][5];
    static bool have[64][5];
    std::lock_guard<std::mutex> lock(mu);
    const int dev = ctx->device & 63;
    if (!have[dev][S]) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)(S * 64));
        cfg.blockDim = dim3(kTcThreads);
        cfg.dynamicSmemBytes = kTcSmem;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = (unsigned)S;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, (const void *)tc_gemm_tf32_splitk_kernel, &cfg) != cudaSuccess) {
            cudaGetLastError();
            n = 0;
        }
        cache[dev][S] = n;
        have[dev][S] = true;
    }
    return cache[dev][S];
}

}  // namespace

int lalb_tc_gemm_tf32(lalb_ctx *ctx, const TcGemmParts &p, cudaStream_t s) {
    if (p.M <= 0 || p.N <= 0 || p.K <= 0 || p.K % BK || !p.a_hi || !p.b_hi || !p.Y)
        return lalb_fail(ctx, LALB_ERR_INVALID, "tc_gemm: M, N > 0, K a multiple of %d", BK);
    if (((uintptr_t)p.a_hi | (uintptr_t)p.a_lo | (uintptr_t)p.b_hi | (uintptr_t)p.b_lo) & 15u)
        return lalb_fail(ctx, LALB_ERR_INVALID, "tc_gemm: operands must be 16-byte aligned");
    TcArgs a = {};
    a.M = p.M;
    a.N = p.N;
    a.K = p.K;
    a.conv_a = p.split_a && !p.a_lo;
    a.a_parts = (p.a_lo || a.conv_a) ? 2 : 1;
    a.a_loads = p.a_lo ? 2 : 1;
    a.b_parts = p.b_lo ? 2 : 1;
    a.Y = p.Y;
    a.rowscale = p.rowscale;
    a.colscale = p.colscale;
    a.bias = p.bias;
    a.status = &ctx->scratch->status;
    a.y_vec4 = (p.N % 4 == 0) && ((uintptr_t)p.Y & 15u) == 0;
    int st;
    if ((st = lalb_set_smem_attr(ctx, (const void *)tc_gemm_tf32_kernel, (int)kTcSmem))) return st;
    if ((st = lalb_set_smem_attr(ctx, (const void *)tc_gemm_tf32_splitk_kernel, (int)kTcSmem))) return st;

    // Plan: tile width bn (256 only with one B part, its ring slot then 64 KB,
    // and only for many tiles) and split S (a cluster of S CTAs per tile when
    // one wave of them fits).  The K-loop is bound by the shared memory each SM
    // moves per K-block: TMA writes, the converters' reads and writes, and the
    // MMAs' operand reads; the plan with the fewest such bytes on the busiest
    // SM wins.
    const int nk = p.K / BK, tiles_m = (p.M + BM - 1) / BM;
    const int mmas_per_k8 = a.a_parts + (a.b_parts - 1);
    // rows-as-M (one MMA per step over A's adjacent hi and lo tiles) when A
    // has two parts and B one, with 128-wide tiles
    const bool can_swap = a.a_parts == 2 && a.b_parts == 1;
    int best_bn = BN, best_s = 1;
    double best_cost = 1e300;
    for (int bn : {BN, kBNWide}) {
        // 256-wide tiles only for the persistent kernel over many tiles: in one
        // wave (and with split-K) they measured slower than 128-wide ones
        if (bn == kBNWide && (a.b_parts > 1 || ((p.N + BN - 1) / BN) * tiles_m <= 2 * ctx->sm_count))
            continue;
        const int tiles = ((p.N + bn - 1) / bn) * tiles_m;
        const double mma_bytes = (bn == BN && can_swap)
                                     ? (double)(BK / 8) * (bn * 8 * 4 + 2 * BM * 8 * 4)
                                     : (double)(BK / 8) * mmas_per_k8 * (BM * 8 * 4 + bn * 8 * 4);
        const double kb_bytes = (double)a.a_loads * kATile + (double)a.b_parts * bn * BK * 4 +
                                (a.conv_a ? 2.0 * kATile : 0.0) + mma_bytes;
        for (int S = 1; S <= (bn == BN ? 4 : 1); ++S) {
            double cost;
            if (S == 1) {
                const double waves = tiles <= ctx->sm_count ? 1.0 : (double)tiles / ctx->sm_count;
                cost = waves * nk * kb_bytes;
            } else {
                if (tiles * S > ctx->sm_count || nk < 2 * S) continue;
                if (splitk_clusters_fit(ctx, S) < tiles) continue;   // one wave of clusters or nothing
                cost = (double)nk / S * kb_bytes + 2.0 * BM * bn * 4;   // + the partial's write and reads
            }
            if (cost < best_cost * 0.97) {   // ties go to the simpler plan
                best_cost = cost;
                best_bn = bn;
                best_s = S;
            }
        }
    }
    a.bn = best_bn;
    a.b_tile = (uint32_t)a.bn * BK * 4;
    a.swap = can_swap && a.bn == BN;
    a.acc_cols = a.swap ? 2 * BM : a.bn;   // swap: N = 256 (A hi rows, then A lo rows)
    a.idesc = idesc_tf32(a.swap ? 2 * BM : a.bn);
    // ring slot: A hi | A lo | B hi (| B lo), each 1024-byte aligned
    a.stage_bytes = 2 * kATile + (uint32_t)a.b_parts * a.b_tile;
    a.nstages = (int)std::min<uint32_t>(kMaxStages, kRingBytes / a.stage_bytes);
    if (a.nstages < 2 || (size_t)a.nstages * a.stage_bytes > kRingBytes)
        return lalb_fail(ctx, LALB_ERR_UNSUPPORTED, "tc_gemm: ring layout");
    a.tiles_n = (p.N + a.bn - 1) / a.bn;
    a.tiles = a.tiles_n * tiles_m;
    // accumulators: 512 TMEM columns hold nacc x ngroups tiles of bn columns;
    // short K: two groups (the epilogue of one tile overlaps the next tile's
    // MMAs), long K: one group of more accumulators (shorter fp32 chains)
    const bool long_k = nk > kLongK;
    a.nacc = (long_k ? 4 : 2) * BN / a.acc_cols;
    a.ngroups = long_k ? 1 : 2;
    a.splits = best_s;

    CUtensorMap mA0, mA1, mB0, mB1;
    if ((st = make_map(ctx, &mA0, p.a_hi, p.M, p.K, BM))) return st;
    if ((st = make_map(ctx, &mA1, p.a_lo ? p.a_lo : p.a_hi, p.M, p.K, BM))) return st;
    if ((st = make_map(ctx, &mB0, p.b_hi, p.N, p.K, a.bn))) return st;
    if ((st = make_map(ctx, &mB1, p.b_lo ? p.b_lo : p.b_hi, p.N, p.K, a.bn))) return st;
    if (a.splits > 1)
        return launch_cluster_pdl(ctx, (const void *)tc_gemm_tf32_splitk_kernel, dim3(a.tiles * a.splits),
                                  dim3(kTcThreads), kTcSmem, a.splits, s,
                                  {(void *)&mA0, (void *)&mA1, (void *)&mB0, (void *)&mB1, (void *)&a});
    const int grid = std::min(a.tiles, ctx->sm_count);
    return launch_pdl(ctx, (const void *)tc_gemm_tf32_kernel, dim3(grid), dim3(kTcThreads), kTcSmem, s,
                      {(void *)&mA0, (void *)&mA1, (void *)&mB0, (void *)&mB1, (void *)&a});
}
