// lalb_q4k_gemv.cu -- Q4_K x Q8 matvec for batch-1 decode on sm_100a.
//
// Memory-bound by design: the only bytes that must cross HBM are the Q4_K
// super-blocks (4.5 bits per weight).  One CTA owns a contiguous range of
// weight rows (one contiguous byte range of the row-major matrix) and is
// split into T independent teams of WR warps:
//
//   * a stage is kR = 4 consecutive rows.  Team t takes stages t, t+T, ...;
//     it owns kBufPerTeam shared-memory buffers and keeps them full itself:
//     after the team has read a buffer, one of its lanes refills it with a
//     1-D bulk copy (cp.async.bulk, the TMA engine) of the team's next stage,
//     completion tracked by one mbarrier per buffer.  No CTA-wide barrier in
//     the main loop; the weights stream with an L2 evict-first policy;
//   * the activation arrives after the dependency wait (bulk copy when it is
//     already quantized) and is quantized in the prologue one 32-block per
//     thread (fp32 -> int8 with an fp32 scale, optional RMS normalisation);
//   * warp k of a team owns the 128-weight half-blocks c = 32k + lane; the
//     lane keeps that half-block's int8 activations, scales and scale*sum
//     terms in registers for the whole kernel, so shared-memory traffic is
//     the weights only;
//   * per half-block and row: 5 x 16-byte shared loads (header, 64 bytes of
//     quants), 32 dp4a giving the four exact int32 sub-block sums, and the
//     exact fp64 products sx*sc*isum and sx*sumq*m, combined with d and dmin.
//     The 4 rows of a stage are 4 independent chains;
//   * a transposed shuffle reduction sums the 4 rows across the warp at once;
//     teams of several warps combine their partials through shared memory
//     (the last warp to arrive finishes the rows and refills the buffer);
//   * rows are summed in double and rounded to fp32 once, so the output is the
//     fp32 rounding of the exact dot product whatever the thread mapping;
//   * fused epilogues: store, residual add, SwiGLU + re-quantization of the
//     product for the next matvec (64-row tiles completed through a small
//     ring of shared-memory tiles with arrival counters).
//
// References (paths inside the reference project): lal_matmul_q4_k
// (runtime/lal_q4k_kernel.h, README.md:130,210), unpack_scales_6bit
// (README.md:212), Q4_K layout (README.md:28,284).
#include <algorithm>

#include "lalb_internal.cuh"
#include "lalb_kernels.cuh"
#include "lalb_q4k_common.cuh"

using namespace lalb;

namespace {

constexpr int kR = 4;            // rows per stage
constexpr int kBufPerTeam = 2;   // stage buffers owned by each team
constexpr int kTiles = 4;        // SwiGLU tile ring
constexpr int kMaxThreads = 512;
constexpr int kMaxK = 32768;     // two 4-row stages of this K fill one SM's shared memory

struct Layout {
    uint32_t off_xq, off_sx, off_sq, off_red, off_rcnt, off_issued, off_tile, off_tcnt, off_ttag;
    uint32_t off_stage, stage_bytes, total;
    int nstages;
};

__host__ __device__ inline uint32_t align_up(uint32_t v, uint32_t a) {
    return (v + a - 1) / a * a;
}

// Shared-memory layout shared by host (size) and device (pointers).  The
// first bytes hold the mbarriers: one per stage buffer + one for the
// activation copy.
__host__ __device__ inline Layout make_layout(int K, int wr, int teams) {
    Layout L;
    const uint32_t ns = K / 32;
    L.nstages = teams * kBufPerTeam;
    L.off_xq = align_up(8u * (L.nstages + 1), 128);
    L.off_sx = align_up(L.off_xq + K, 16);
    L.off_sq = L.off_sx + 4 * ns;
    L.off_red = align_up(L.off_sq + 4 * ns, 16);
    uint32_t nred = (uint32_t)L.nstages * wr * kR;
    if (nred < 40) nred = 40;                        // also the prologue's block reduction
    L.off_rcnt = L.off_red + 8 * nred;
    L.off_issued = L.off_rcnt + 4 * L.nstages;
    L.off_tile = align_up(L.off_issued + 4 * teams, 16);
    L.off_tcnt = L.off_tile + kTiles * 64 * 4;
    L.off_ttag = L.off_tcnt + 4 * kTiles;
    L.off_stage = align_up(L.off_ttag + 4 * kTiles, 128);
    L.stage_bytes = kR * (uint32_t)(K / 256) * 144u;
    L.total = L.off_stage + L.nstages * L.stage_bytes;
    return L;
}

template <int IN, int EPI>
__global__ void __launch_bounds__(kMaxThreads, 1) q4k_gemv_kernel(const Q4kGemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int WR = a.wr, T = a.teams;
    const int K = a.K;
    const int NH = K >> 7, NS = K >> 5;
    const uint32_t row_bytes = (uint32_t)(K >> 8) * 144u;
    const Layout L = make_layout(K, WR, T);
    const int nstages = L.nstages;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *act_bar = full + nstages;
    int8_t *xq_s = reinterpret_cast<int8_t *>(smem + L.off_xq);
    float *sx_s = reinterpret_cast<float *>(smem + L.off_sx);
    int *sq_s = reinterpret_cast<int *>(smem + L.off_sq);
    double *red_s = reinterpret_cast<double *>(smem + L.off_red);
    int *rcnt_s = reinterpret_cast<int *>(smem + L.off_rcnt);
    int *issued_s = reinterpret_cast<int *>(smem + L.off_issued);  // stages issued per team
    float *tile_s = reinterpret_cast<float *>(smem + L.off_tile);
    int *tcnt_s = reinterpret_cast<int *>(smem + L.off_tcnt);
    volatile int *ttag_s = reinterpret_cast<volatile int *>(smem + L.off_ttag);
    uint8_t *stage_s = smem + L.off_stage;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nthreads = blockDim.x;
    const int team = warp / WR, kw = warp % WR;
    const int c = kw * 32 + lane;  // this lane's half-block

    // contiguous row range of this CTA, in units of a.unit rows
    const int nunits = a.rows / a.unit;
    const int u0 = (int)((long long)blockIdx.x * nunits / gridDim.x);
    const int u1 = (int)((long long)(blockIdx.x + 1) * nunits / gridDim.x);
    const int r0 = u0 * a.unit, r1 = u1 * a.unit;
    const int nst = (r1 - r0 + kR - 1) / kR;
    const int my_stages = team < nst ? (nst - team + T - 1) / T : 0;

    // stage s of this team: buffer team*kBufPerTeam + (it % kBufPerTeam),
    // that buffer's (it / kBufPerTeam)-th use, it = s / T
    auto issue = [&](int it, uint64_t pol) {
        const int s = team + it * T;
        const int rs = r0 + s * kR;
        const int nr = min(kR, r1 - rs);
        const uint32_t bytes = (uint32_t)nr * row_bytes;
        const int buf = team * kBufPerTeam + it % kBufPerTeam;
        issued_s[team] = it + 1;
        mbar_arrive_expect_tx(&full[buf], bytes);
        bulk_g2s(stage_s + (size_t)buf * L.stage_bytes, a.W + (size_t)rs * row_bytes, bytes,
                 &full[buf], pol);
    };

    if (tid == 0) {
        for (int s = 0; s <= nstages; ++s) mbar_init(&full[s], 1);
        fence_barrier_init();
    }
    for (int i = tid; i < nstages; i += nthreads) rcnt_s[i] = 0;
    for (int i = tid; i < T; i += nthreads) issued_s[i] = 0;
    if (tid < kTiles) {
        tcnt_s[tid] = 0;
        ttag_s[tid] = tid;
    }
    __syncthreads();
    const uint64_t policy = l2_evict_first_policy();
    if (a.w_l2_first) {
        // The weights may be the preceding kernel's output: before the
        // dependency wait this CTA's rows are only prefetched into L2 (where
        // that kernel's writes land, so nothing stale is kept), and the
        // shared-memory stream starts after it.
        if (warp == 0) {
            const uint8_t *w0 = a.W + (size_t)r0 * row_bytes;
            const size_t bytes = (size_t)(r1 - r0) * row_bytes;   // a multiple of 16
            for (size_t off = (size_t)lane * 32768; off < bytes; off += 32 * 32768)
                bulk_prefetch_l2(w0 + off, (uint32_t)(bytes - off < 32768 ? bytes - off : 32768));
        }
        pdl_wait();
        // the shared-memory stream starts after the activation prologue: its
        // copies (a good part of the SM's L2 bandwidth for a microsecond or
        // two) would otherwise delay the activation loads queued behind them
    } else {
        // The weights are never written by the preceding kernel, so their
        // stream starts before the dependency wait; activations come after it.
        if (kw == 0 && lane == 0)
            for (int it = 0; it < kBufPerTeam && it < my_stages; ++it) issue(it, policy);
        pdl_wait();
    }

    // ---- activation prologue -------------------------------------------------
    if (IN == kInQ8) {
        // the int8 activation goes into the swizzled layout (xq_swz_chunk)
        if (a.act_bulk) {
            if (tid == 0) {
                mbar_arrive_expect_tx(act_bar, 8u * NS);
                bulk_g2s_plain(sx_s, a.sx, 4u * NS, act_bar);
                bulk_g2s_plain(sq_s, a.sumq, 4u * NS, act_bar);
            }
        } else {
            for (int i = tid; i < NS; i += nthreads) {
                sx_s[i] = a.sx[i];
                sq_s[i] = a.sumq[i];
            }
        }
        const int4 *src = reinterpret_cast<const int4 *>(a.xq);
        int4 *dst = reinterpret_cast<int4 *>(xq_s);
        for (int i = tid; i < K / 16; i += nthreads) dst[xq_swz_chunk(i >> 3, i & 7)] = src[i];
        if (a.act_bulk) mbar_wait_bounded(act_bar, 0, a.status);
    } else {
        const bool vec = a.act_bulk;  // x is 16-byte aligned
        // a quad of lanes per 32-block; whole warps per pass so the quad
        // shuffles always have all lanes present
        const int nquads = ((nthreads >> 5) << 5) >> 2;
        float scale = 1.0f;
        if (IN == kInF32Rms) {
            // sum of squares in double (each square is exact), then 1/rms
            double ss = 0.0;
            for (int e = tid * 8; e < K; e += nthreads * 8) {
                float v[8];
                load8(a.x + e, vec, v);
#pragma unroll
                for (int i = 0; i < 8; ++i) ss += (double)v[i] * (double)v[i];
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            if (lane == 0) red_s[warp] = ss;
            __syncthreads();
            if (warp == 0) {
                double t = lane < (nthreads >> 5) ? red_s[lane] : 0.0;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
                if (lane == 0) red_s[32] = (double)(float)(1.0 / sqrt(t / (double)K + (double)a.eps));
            }
            __syncthreads();
            scale = (float)red_s[32];
        }
        const int quad = tid >> 2, qi = tid & 3;
        if (IN == kInF32 && NS <= 2 * nquads) {
            // both passes' loads in flight at once (one L2 round trip), then
            // the weight stream, then the quantizer
            float v[2][8];
#pragma unroll
            for (int ps = 0; ps < 2; ++ps) {
                const int blk = ps * nquads + quad;
                if (blk < NS) load8(a.x + blk * 32 + 8 * qi, vec, v[ps]);
                else
#pragma unroll
                    for (int i = 0; i < 8; ++i) v[ps][i] = 0.0f;
            }
            if (a.w_l2_first && kw == 0 && lane == 0)
                for (int it = 0; it < kBufPerTeam && it < my_stages; ++it) issue(it, policy);
#pragma unroll
            for (int ps = 0; ps < 2; ++ps) {
                const int blk = ps * nquads + quad;
                if (ps * nquads + (tid & ~31) / 4 < NS)
                    quantize_block_quad_swz(v[ps], qi, blk < NS, xq_s, blk, sx_s + blk, sq_s + blk);
            }
        } else
        for (int blk0 = 0; blk0 < NS; blk0 += nquads) {
            const int blk = blk0 + quad;
            const bool have = blk < NS;
            float v[8];
            if (have) {
                load8(a.x + blk * 32 + 8 * qi, vec, v);
                if (IN == kInF32Rms) {
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        v[i] = __fmul_rn(v[i], scale);
                        if (a.gamma) v[i] = __fmul_rn(v[i], a.gamma[blk * 32 + 8 * qi + i]);
                    }
                }
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) v[i] = 0.0f;
            }
            // whole warps take part (the quad shuffles need every lane)
            if (blk0 + (tid & ~31) / 4 < NS)
                quantize_block_quad_swz(v, qi, have, xq_s, blk, sx_s + blk, sq_s + blk);
        }
    }
    __syncthreads();
    // (the one-round-trip fp32 prologue above has issued them already)
    if (a.w_l2_first && !(IN == kInF32 && NS <= 2 * (((nthreads >> 5) << 5) >> 2)) && kw == 0 &&
        lane == 0)
        for (int it = 0; it < kBufPerTeam && it < my_stages; ++it) issue(it, policy);
    pdl_launch_dependents();

    // ---- per-lane activation registers ------------------------------------
    int xv[32];
    double sxd[4], ad[4];
    if (c < NH) {
        const int4 *p = reinterpret_cast<const int4 *>(xq_s + 128 * c);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int4 v = p[j ^ (c & 7)];   // swizzled: conflict-free across lanes
            xv[4 * j + 0] = v.x;
            xv[4 * j + 1] = v.y;
            xv[4 * j + 2] = v.z;
            xv[4 * j + 3] = v.w;
        }
        const float4 sx4 = reinterpret_cast<const float4 *>(sx_s)[c];   // one 16-byte load each
        const int4 sq4 = reinterpret_cast<const int4 *>(sq_s)[c];
        const float sxa[4] = {sx4.x, sx4.y, sx4.z, sx4.w};
        const int sqa[4] = {sq4.x, sq4.y, sq4.z, sq4.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            sxd[j] = (double)sxa[j];
            ad[j] = sxd[j] * (double)sqa[j];
        }
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) xv[j] = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) sxd[j] = ad[j] = 0.0;
    }

    // ---- main loop: this team's stages --------------------------------------
    const int myrow = ((lane >> 4) & 1) * 2 + ((lane >> 3) & 1);  // row held after the reduction
    for (int it = 0; it < my_stages; ++it) {
        const int s = team + it * T;
        const int buf = team * kBufPerTeam + it % kBufPerTeam;
        const bool ok = mbar_wait_bounded(&full[buf], (uint32_t)(it / kBufPerTeam) & 1u, a.status);
        if (!ok) break;
        const int rs = r0 + s * kR;
        const uint8_t *sb = stage_s + (size_t)buf * L.stage_bytes;
        double acc[kR];
#pragma unroll
        for (int r = 0; r < kR; ++r) {
            acc[r] = 0.0;
            if (c < NH && rs + r < r1)
                acc[r] = q4k_half(sb + r * row_bytes, c, xv, sxd, ad,
                                  a.isum ? a.isum + (size_t)(rs + r) * NS + 4 * c : nullptr);
        }
        double v = warp_sum_rows4(acc, lane);
        bool finisher = true;   // this warp completes the stage's rows
        if (WR > 1) {
            if ((lane & 7) == 0) red_s[(buf * WR + kw) * kR + myrow] = v;
            __syncwarp();
            int last = 0;
            if (lane == 0) {
                __threadfence_block();
                last = atomicAdd(&rcnt_s[buf], 1) == WR - 1;
            }
            finisher = __shfl_sync(0xffffffffu, last, 0);
            if (finisher) {
                __threadfence_block();
                double sum = 0.0;
                for (int w2 = 0; w2 < WR; ++w2) sum += red_s[(buf * WR + w2) * kR + myrow];
                v = sum;
                if (lane == 0) rcnt_s[buf] = 0;
            }
        }
        if (finisher) {
            const int row = rs + myrow;
            if (EPI == kEpiSwiglu) {
                // 64-row tile t (32 gate + 32 up rows) of this CTA's range
                const int lrow = s * kR;
                const int t = lrow >> 6, jb = t % kTiles;
                if (lane == 0) {
                    for (uint32_t k = 0; ttag_s[jb] != t; ++k) {
                        if (k > LALB_SPIN_LIMIT) {
                            atomicOr(a.status, LALB_STATUS_WAIT_TIMEOUT);
                            break;
                        }
                        __nanosleep(32);
                    }
                }
                __syncwarp();
                if ((lane & 7) == 0) tile_s[jb * 64 + (lrow & 63) + myrow] = (float)v;
                __syncwarp();
                int last = 0;
                if (lane == 0) {
                    __threadfence_block();
                    last = atomicAdd(&tcnt_s[jb], kR) == 64 - kR;
                }
                if (__shfl_sync(0xffffffffu, last, 0)) {
                    __threadfence_block();
                    const float av = silu_mul(tile_s[jb * 64 + lane], tile_s[jb * 64 + 32 + lane]);
                    const int gt = (r0 >> 6) + t;  // 32-element block of the product
                    if (a.act_out) a.act_out[gt * 32 + lane] = av;
                    quantize_block32(av, lane, a.aq + gt * 32, a.asx + gt, a.asumq + gt);
                    __syncwarp();
                    if (lane == 0) {
                        tcnt_s[jb] = 0;
                        __threadfence_block();
                        ttag_s[jb] = t + kTiles;
                    }
                }
            } else if ((lane & 7) == 0 && row < r1) {
                const float f = (float)v;
                a.y[row] = EPI == kEpiResid ? __fadd_rn(a.resid[row], f) : f;
            }
            // every warp of the team is done with this buffer: refill it
            __syncwarp();
            if (lane == 0 && it + kBufPerTeam < my_stages) issue(it + kBufPerTeam, policy);
        }
    }
    // drain: a copy still in flight (only after an expired wait) must land
    // before the CTA's shared memory is released
    __syncthreads();
    if (kw == 0 && lane == 0) {
        const int n = issued_s[team];
        for (int j = 0; j < kBufPerTeam && j < n; ++j) {
            const int last_it = ((n - 1 - j) / kBufPerTeam) * kBufPerTeam + j;
            mbar_wait_bounded(&full[team * kBufPerTeam + j], (uint32_t)(last_it / kBufPerTeam) & 1u,
                              a.status);
        }
    }
    if (tid == 0 && IN == kInQ8 && a.act_bulk) mbar_wait_bounded(act_bar, 0, a.status);
}

template <int IN, int EPI>
void *kernel_ptr() {
    return (void *)q4k_gemv_kernel<IN, EPI>;
}

void *select_kernel(int in, int epi) {
#define LALB_SEL(I, E) \
    if (in == I && epi == E) return kernel_ptr<I, E>();
    LALB_SEL(kInF32, kEpiStore)
    LALB_SEL(kInF32Rms, kEpiStore)
    LALB_SEL(kInQ8, kEpiStore)
    LALB_SEL(kInF32, kEpiResid)
    LALB_SEL(kInQ8, kEpiResid)
    LALB_SEL(kInF32Rms, kEpiSwiglu)
#undef LALB_SEL
    return nullptr;
}

}  // namespace

// Launches one Q4_K matvec.  `unit` = row granularity of the CTA split (64
// for the SwiGLU epilogue).  ctas_per_sm: 1 or 2 (clamped to what fits).
int lalb_launch_q4k_gemv(lalb_ctx *ctx, const Q4kGemvArgs &args_in, int in, int epi,
                         cudaStream_t stream, bool pdl, int ctas_per_sm) {
    Q4kGemvArgs a = args_in;
    if (!a.W || a.rows <= 0 || a.K <= 0 || a.K % 256)
        return lalb_fail(ctx, LALB_ERR_INVALID, "q4k gemv: bad shape rows=%d K=%d", a.rows, a.K);
    if (reinterpret_cast<uintptr_t>(a.W) & 15)
        return lalb_fail(ctx, LALB_ERR_INVALID, "q4k gemv: W must be 16-byte aligned");
    if (a.unit <= 0 || a.rows % a.unit)
        return lalb_fail(ctx, LALB_ERR_INVALID, "q4k gemv: rows %% unit != 0");
    const int NH = a.K / 128;
    const int wr = (NH + 31) / 32;
    if (a.K > kMaxK)
        return lalb_fail(ctx, LALB_ERR_UNSUPPORTED, "q4k gemv: K=%d > %d", a.K, kMaxK);
    if (epi == kEpiSwiglu && (wr != 1 || a.unit % 64))
        return lalb_fail(ctx, LALB_ERR_UNSUPPORTED, "q4k gemv: SwiGLU epilogue needs K <= 4096");
    if (in == kInQ8 && (reinterpret_cast<uintptr_t>(a.xq) & 15))
        return lalb_fail(ctx, LALB_ERR_INVALID, "q4k gemv: xq must be 16-byte aligned");
    void *fn = select_kernel(in, epi);
    if (!fn) return lalb_fail(ctx, LALB_ERR_UNSUPPORTED, "q4k gemv: no variant in=%d epi=%d", in, epi);
    const auto al16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    a.act_bulk = in == kInQ8 ? (al16(a.xq) && al16(a.sx) && al16(a.sumq)) : al16(a.x);

    // teams: as many as fit the thread, register and shared-memory budget
    const size_t budget = ctas_per_sm >= 2 ? 110 * 1024 : ctx->smem_optin - 1024;
    int teams = std::max(1, std::min(12 / wr, kMaxThreads / (32 * wr)));
    while (teams > 1 && make_layout(a.K, wr, teams).total > budget) --teams;
    Layout L = make_layout(a.K, wr, teams);
    if (L.total > ctx->smem_optin - 1024)
        return lalb_fail(ctx, LALB_ERR_UNSUPPORTED, "q4k gemv: K=%d too large for smem", a.K);
    a.wr = wr;
    a.teams = teams;
    a.nstages = L.nstages;
    a.status = &ctx->scratch->status;
    {
        const int st = lalb_set_smem_attr(ctx, fn, (int)L.total);
        if (st) return st;
    }
    const int threads = 32 * wr * teams;
    int resident = 0;
    LALB_CUDA_TRY(ctx, cudaOccupancyMaxActiveBlocksPerMultiprocessor(&resident, (const void *)fn,
                                                                     threads, L.total));
    if (resident < 1) return lalb_fail(ctx, LALB_ERR_UNSUPPORTED, "q4k gemv: CTA does not fit");
    if (ctas_per_sm > resident) ctas_per_sm = resident;
    const int nunits = a.rows / a.unit;
    int grid = ctx->sm_count * ctas_per_sm;
    if (grid > nunits) grid = nunits;

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(threads);
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

extern "C" int lalb_matmul_q4_k(lalb_ctx *ctx, const void *W, int rows, int K, const float *x,
                                float *y, lalb_stream stream) {
    if (!ctx) return LALB_ERR_INVALID;
    if (!x || !y) return lalb_fail(ctx, LALB_ERR_INVALID, "matmul_q4_k: null x/y");
    Q4kGemvArgs a = {};
    a.W = static_cast<const uint8_t *>(W);
    a.rows = rows;
    a.K = K;
    a.x = x;
    a.y = y;
    a.unit = 1;
    a.w_l2_first = 1;   // W may be the output of the preceding kernel in the stream
    return lalb_launch_q4k_gemv(ctx, a, kInF32, kEpiStore, (cudaStream_t)stream, true, 1);
}

extern "C" int lalb_matmul_q4_k_q8(lalb_ctx *ctx, const void *W, int rows, int K,
                                   const int8_t *xq, const float *sx, const int32_t *sumq,
                                   float *y, int32_t *isum, lalb_stream stream) {
    if (!ctx) return LALB_ERR_INVALID;
    if (!xq || !sx || !sumq || !y)
        return lalb_fail(ctx, LALB_ERR_INVALID, "matmul_q4_k_q8: null argument");
    Q4kGemvArgs a = {};
    a.W = static_cast<const uint8_t *>(W);
    a.rows = rows;
    a.K = K;
    a.xq = xq;
    a.sx = sx;
    a.sumq = sumq;
    a.y = y;
    a.isum = isum;
    a.unit = 1;
    a.w_l2_first = 1;
    return lalb_launch_q4k_gemv(ctx, a, kInQ8, kEpiStore, (cudaStream_t)stream, true, 1);
}
