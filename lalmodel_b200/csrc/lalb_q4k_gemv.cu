// lalb_q4k_gemv.cu -- Q4_K x Q8 matvec for batch-1 decode on sm_100a.
//
// Memory-bound by design: the only bytes that must cross HBM are the Q4_K
// super-blocks (4.5 bits per weight).  Structure of one CTA (256 threads):
//
//   * it owns a contiguous range of weight rows, i.e. one contiguous byte
//     range of the row-major Q4_K matrix;
//   * thread 0 streams that range into a ring of shared-memory stages with
//     1-D bulk copies (cp.async.bulk, the TMA engine), completion tracked by
//     one mbarrier per stage, L2 policy evict-first;
//   * the activation arrives by one more bulk copy after the dependency wait
//     and is quantized (fp32 -> int8 per 32-block, optional RMS
//     normalisation) in shared memory by the whole CTA -- the quantizer is
//     fused, no separate launch;
//   * a "team" of WR warps owns one row of a stage; team lane t owns the
//     128-weight half-block c = t (sub-blocks 4(c&1)..4(c&1)+3 of super-block
//     c/2).  The lane keeps that half-block's int8 activations, scales and
//     scale*sum terms in registers for the whole kernel, so shared-memory
//     traffic is the weights only;
//   * per half-block: 5 x 16-byte shared loads (header, 64 bytes of quants),
//     32 dp4a giving the four exact int32 sub-block sums, and the exact fp64
//     products sx*sc*isum and sx*sumq*m, combined with d and dmin;
//   * the row is reduced in double (warp shuffles, then across the team) and
//     rounded to fp32 once, so the output is the fp32 rounding of the exact
//     dot product whatever the thread mapping;
//   * fused epilogues: store, residual add, SwiGLU + re-quantization of the
//     product for the next matvec.
//
// References (paths inside the reference project): lal_matmul_q4_k
// (runtime/lal_q4k_kernel.h, README.md:130,210), unpack_scales_6bit
// (README.md:212), Q4_K layout (README.md:28,284).
#include <algorithm>

#include "lalb_internal.cuh"
#include "lalb_kernels.cuh"

using namespace lalb;

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxStagedK = 4096;   // fp32 activations up to this K are bulk-copied to smem

struct Layout {
    uint32_t off_xq, off_sx, off_sq, off_xf, off_red, off_tile, off_stage;
    uint32_t stage_bytes, total;
};

__host__ __device__ inline uint32_t align_up(uint32_t v, uint32_t a) {
    return (v + a - 1) / a * a;
}

// Shared-memory layout shared by host (size) and device (pointers).  The
// first 128 bytes hold the mbarriers: one per weight stage + one for the
// activation copy.  xf_floats = K when the fp32 activation is staged.
__host__ __device__ inline Layout make_layout(int K, int wr, int nstages, int xf_floats) {
    Layout L;
    const uint32_t ns = K / 32;
    L.off_xq = 128;
    L.off_sx = align_up(L.off_xq + K, 16);
    L.off_sq = L.off_sx + 4 * ns;
    L.off_xf = align_up(L.off_sq + 4 * ns, 16);
    L.off_red = align_up(L.off_xf + 4 * xf_floats, 16);
    L.off_tile = L.off_red + 2 * kWarps * 8;         // double partials
    L.off_stage = align_up(L.off_tile + 2 * 64 * 4, 128);
    const uint32_t rps = kWarps / wr;
    L.stage_bytes = rps * (uint32_t)(K / 256) * 144u;
    L.total = L.off_stage + nstages * L.stage_bytes;
    return L;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// unsigned bytes of a times signed bytes of b, accumulated into c
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Quantizes one 32-element block held one element per lane: writes the int8
// codes, and (lane 0) the fp32 scale and the int32 sum.  Same operations as
// the CPU restatement.
__device__ __forceinline__ void quantize_block32(float v, int lane, int8_t *xq32, float *sx,
                                                 int *sumq) {
    const uint32_t amax = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(v)));
    const float dsc = __fdiv_rn(__uint_as_float(amax), 127.0f);
    const float id = dsc != 0.0f ? __fdiv_rn(1.0f, dsc) : 0.0f;
    const float t = roundf(__fmul_rn(v, id));
    const int q = t > 127.0f ? 127 : (t < -127.0f ? -127 : (int)t);
    xq32[lane] = (int8_t)q;
    const int s = __reduce_add_sync(0xffffffffu, q);
    if (lane == 0) {
        *sx = dsc;
        *sumq = s;
    }
}

// Activation state of GPL half-blocks of 128 weights, held in registers.
template <int GPL>
struct HalfBlockAct {
    int xv[GPL][32];       // 128 int8 codes each
    double sxd[GPL][4];    // per sub-block scale (exact as double)
    double ad[GPL][4];     // scale * sumq (exact as double)
};

// One half-block of one row: returns d*sum_j sx_j*sc_j*isum_j -
// dmin*sum_j sx_j*sumq_j*m_j in double; writes the four exact int32
// sub-block dot products to isum4 when non-null.
__device__ __forceinline__ double q4k_half(const uint8_t *__restrict__ rowp, int c,
                                           const int (&xv)[32], const double (&sxd)[4],
                                           const double (&ad)[4], int32_t *isum4) {
    const int b = c >> 1, hsel = c & 1;
    const uint8_t *bp = rowp + b * 144;
    const uint4 h = *reinterpret_cast<const uint4 *>(bp);
    const uint4 q0 = *reinterpret_cast<const uint4 *>(bp + 16 + 64 * hsel);
    const uint4 q1 = *reinterpret_cast<const uint4 *>(bp + 32 + 64 * hsel);
    const uint4 q2 = *reinterpret_cast<const uint4 *>(bp + 48 + 64 * hsel);
    const uint4 q3 = *reinterpret_cast<const uint4 *>(bp + 64 + 64 * hsel);
    // scales / mins of sub-blocks 4hsel..4hsel+3, byte j = sub-block 4hsel+j
    const uint32_t scw = hsel ? ((h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u))
                              : (h.y & 0x3F3F3F3Fu);
    const uint32_t mnw = hsel ? (((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u))
                              : (h.z & 0x3F3F3F3Fu);
    const uint32_t w[16] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w,
                            q2.x, q2.y, q2.z, q2.w, q3.x, q3.y, q3.z, q3.w};
    // sub-block 0: low nibbles of words 0-7; 1: high nibbles of words 0-7;
    // 2: low nibbles of words 8-15; 3: high nibbles of words 8-15.  A high
    // nibble masked in place is 16*q as an unsigned byte: the dot is 16x.
    int a0 = 0, b0 = 0, a1 = 0, b1 = 0, a2 = 0, b2 = 0, a3 = 0, b3 = 0;
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
        a0 = dp4a_us(w[i] & 0x0F0F0F0Fu, xv[i], a0);
        b0 = dp4a_us(w[i + 1] & 0x0F0F0F0Fu, xv[i + 1], b0);
        a1 = dp4a_us(w[i] & 0xF0F0F0F0u, xv[8 + i], a1);
        b1 = dp4a_us(w[i + 1] & 0xF0F0F0F0u, xv[9 + i], b1);
        a2 = dp4a_us(w[8 + i] & 0x0F0F0F0Fu, xv[16 + i], a2);
        b2 = dp4a_us(w[9 + i] & 0x0F0F0F0Fu, xv[17 + i], b2);
        a3 = dp4a_us(w[8 + i] & 0xF0F0F0F0u, xv[24 + i], a3);
        b3 = dp4a_us(w[9 + i] & 0xF0F0F0F0u, xv[25 + i], b3);
    }
    const int s0 = a0 + b0, s1 = (a1 + b1) >> 4, s2 = a2 + b2, s3 = (a3 + b3) >> 4;
    if (isum4) {
        isum4[0] = s0;
        isum4[1] = s1;
        isum4[2] = s2;
        isum4[3] = s3;
    }
    // sc*isum fits 22 bits, so sx*(sc*isum) and sx*sumq*m are exact in fp64
    double s1acc = sxd[0] * (double)((int)(scw & 0xFF) * s0);
    s1acc = fma(sxd[1], (double)((int)((scw >> 8) & 0xFF) * s1), s1acc);
    s1acc = fma(sxd[2], (double)((int)((scw >> 16) & 0xFF) * s2), s1acc);
    s1acc = fma(sxd[3], (double)((int)(scw >> 24) * s3), s1acc);
    double s2acc = ad[0] * (double)(mnw & 0xFF);
    s2acc = fma(ad[1], (double)((mnw >> 8) & 0xFF), s2acc);
    s2acc = fma(ad[2], (double)((mnw >> 16) & 0xFF), s2acc);
    s2acc = fma(ad[3], (double)(mnw >> 24), s2acc);
    const double d = (double)f16_bits_to_f32(h.x & 0xFFFFu);
    const double dmin = (double)f16_bits_to_f32(h.x >> 16);
    return fma(d, s1acc, -dmin * s2acc);
}

template <int WR, int GPL, int IN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    q4k_gemv_kernel(const Q4kGemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int RPS = kWarps / WR;  // rows per stage (one per team)
    const int K = a.K;
    const int NH = K >> 7, NS = K >> 5;
    const uint32_t row_bytes = (uint32_t)(K >> 8) * 144u;
    const bool staged = IN != kInQ8 && a.act_bulk;
    const Layout L = make_layout(K, WR, a.nstages, staged ? K : 0);
    const int nstages = a.nstages;
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem);
    uint64_t *act_bar = bar + nstages;
    int8_t *xq_s = reinterpret_cast<int8_t *>(smem + L.off_xq);
    float *sx_s = reinterpret_cast<float *>(smem + L.off_sx);
    int *sq_s = reinterpret_cast<int *>(smem + L.off_sq);
    float *xf_s = reinterpret_cast<float *>(smem + L.off_xf);
    double *red_s = reinterpret_cast<double *>(smem + L.off_red);
    float *tile_s = reinterpret_cast<float *>(smem + L.off_tile);
    uint8_t *stage_s = smem + L.off_stage;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int team = warp / WR, wit = warp % WR;
    const int tl = wit * 32 + lane;

    // contiguous row range of this CTA, in units of a.unit rows
    const int nunits = a.rows / a.unit;
    const int u0 = (int)((long long)blockIdx.x * nunits / gridDim.x);
    const int u1 = (int)((long long)(blockIdx.x + 1) * nunits / gridDim.x);
    const int r0 = u0 * a.unit, r1 = u1 * a.unit;
    const int nst = (r1 - r0 + RPS - 1) / RPS;

    uint64_t policy = 0;
    auto issue = [&](int i) {
        const int rs = r0 + i * RPS;
        const int nr = min(RPS, r1 - rs);
        const uint32_t bytes = (uint32_t)nr * row_bytes;
        const int buf = i % nstages;
        mbar_arrive_expect_tx(&bar[buf], bytes);
        bulk_g2s(stage_s + (size_t)buf * L.stage_bytes, a.W + (size_t)rs * row_bytes, bytes,
                 &bar[buf], policy);
    };

    if (tid == 0) {
        for (int s = 0; s <= nstages; ++s) mbar_init(&bar[s], 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (tid == 0) {
        policy = l2_evict_first_policy();
        const int pre = min(nstages, nst);
        for (int i = 0; i < pre; ++i) issue(i);
    }

    // The weights are never written by the preceding kernel, so their
    // stream starts before the dependency wait; activations come after it.
    pdl_wait();

    // ---- activation prologue -------------------------------------------------
    if (a.act_bulk) {
        // one bulk copy per array into shared memory, then everyone waits
        if (tid == 0) {
            if (IN == kInQ8) {
                mbar_arrive_expect_tx(act_bar, (uint32_t)K + 8u * NS);
                bulk_g2s_plain(xq_s, a.xq, (uint32_t)K, act_bar);
                bulk_g2s_plain(sx_s, a.sx, 4u * NS, act_bar);
                bulk_g2s_plain(sq_s, a.sumq, 4u * NS, act_bar);
            } else {
                mbar_arrive_expect_tx(act_bar, 4u * K);
                bulk_g2s_plain(xf_s, a.x, 4u * K, act_bar);
            }
        }
        mbar_wait_bounded(act_bar, 0, a.status);
    } else if (IN == kInQ8) {
        const int4 *src = reinterpret_cast<const int4 *>(a.xq);
        int4 *dst = reinterpret_cast<int4 *>(xq_s);
        for (int i = tid; i < K / 16; i += kThreads) dst[i] = src[i];
        for (int i = tid; i < NS; i += kThreads) {
            sx_s[i] = a.sx[i];
            sq_s[i] = a.sumq[i];
        }
    }
    if (IN != kInQ8) {
        const float *xsrc = staged ? xf_s : a.x;
        float scale = 1.0f;
        if (IN == kInF32Rms) scale = block_rms_scale(xsrc, K);
        // two blocks per warp per step, both loads issued before either is used
        for (int blk = warp; blk < NS; blk += 2 * kWarps) {
            const int blk2 = blk + kWarps;
            float v = xsrc[blk * 32 + lane];
            float v2 = blk2 < NS ? xsrc[blk2 * 32 + lane] : 0.0f;
            if (IN == kInF32Rms) {
                v = __fmul_rn(v, scale);
                v2 = __fmul_rn(v2, scale);
                if (a.gamma) {
                    v = __fmul_rn(v, a.gamma[blk * 32 + lane]);
                    if (blk2 < NS) v2 = __fmul_rn(v2, a.gamma[blk2 * 32 + lane]);
                }
            }
            quantize_block32(v, lane, xq_s + blk * 32, sx_s + blk, sq_s + blk);
            if (blk2 < NS) quantize_block32(v2, lane, xq_s + blk2 * 32, sx_s + blk2, sq_s + blk2);
        }
    }
    __syncthreads();
    pdl_launch_dependents();

    // ---- per-lane activation registers ------------------------------------
    HalfBlockAct<GPL> act;
#pragma unroll
    for (int k = 0; k < GPL; ++k) {
        const int c = tl + k * 32 * WR;
        if (c < NH) {
            const int4 *p = reinterpret_cast<const int4 *>(xq_s + 128 * c);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int4 v = p[j];
                act.xv[k][4 * j + 0] = v.x;
                act.xv[k][4 * j + 1] = v.y;
                act.xv[k][4 * j + 2] = v.z;
                act.xv[k][4 * j + 3] = v.w;
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const double sxv = (double)sx_s[4 * c + j];
                act.sxd[k][j] = sxv;
                act.ad[k][j] = sxv * (double)sq_s[4 * c + j];
            }
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) act.xv[k][j] = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) act.sxd[k][j] = act.ad[k][j] = 0.0;
        }
    }

    // ---- main loop over stages ---------------------------------------------
    int issued = min(nstages, nst);
    for (int i = 0; i < nst; ++i) {
        const int buf = i % nstages;
        const uint32_t parity = (uint32_t)(i / nstages) & 1u;
        const bool ok = mbar_wait_bounded(&bar[buf], parity, a.status);
        const int row = r0 + i * RPS + team;
        double acc = 0.0;
        if (ok && row < r1) {
            const uint8_t *rowp = stage_s + (size_t)buf * L.stage_bytes + team * row_bytes;
            int32_t *isum_row = a.isum ? a.isum + (size_t)row * NS : nullptr;
#pragma unroll
            for (int k = 0; k < GPL; ++k) {
                const int c = tl + k * 32 * WR;
                if (c < NH)
                    acc += q4k_half(rowp, c, act.xv[k], act.sxd[k], act.ad[k],
                                    isum_row ? isum_row + 4 * c : nullptr);
            }
        }
        acc = warp_sum_d(acc);
        if (WR == 1) {
            if (lane == 0 && row < r1) {
                const float v = (float)acc;
                if (EPI == kEpiSwiglu) {
                    tile_s[(((row - r0) >> 6) & 1) * 64 + ((row - r0) & 63)] = v;
                } else {
                    a.y[row] = EPI == kEpiResid ? __fadd_rn(a.resid[row], v) : v;
                }
            }
        } else if (lane == 0) {
            red_s[(i & 1) * kWarps + team * WR + wit] = acc;
        }
        const bool stop = __syncthreads_or(!ok);
        if (stop) break;
        if (tid == 0 && issued < nst) {
            issue(issued);
            ++issued;
        }
        if (WR > 1 && tid < RPS) {
            const int rw = r0 + i * RPS + tid;
            if (rw < r1) {
                double s = 0.0;
#pragma unroll
                for (int w = 0; w < WR; ++w) s += red_s[(i & 1) * kWarps + tid * WR + w];
                const float v = (float)s;
                if (EPI == kEpiSwiglu) {
                    tile_s[(((rw - r0) >> 6) & 1) * 64 + ((rw - r0) & 63)] = v;
                } else {
                    a.y[rw] = EPI == kEpiResid ? __fadd_rn(a.resid[rw], v) : v;
                }
            }
        }
        if (EPI == kEpiSwiglu) {
            // a 64-row tile (32 gate + 32 up rows) completes every 64/RPS stages
            const int done_rows = (i + 1) * RPS;
            if ((done_rows & 63) == 0) {
                if (WR > 1) __syncthreads();   // the tile entries written above
                const int tloc = (done_rows - 1) >> 6;
                if (warp == kWarps - 1) {
                    const float *tb = tile_s + (tloc & 1) * 64;
                    const float av = silu_mul(tb[lane], tb[32 + lane]);
                    const int gt = (r0 >> 6) + tloc;  // 32-element block of the product
                    if (a.act_out) a.act_out[gt * 32 + lane] = av;
                    quantize_block32(av, lane, a.aq + gt * 32, a.asx + gt, a.asumq + gt);
                }
            }
        }
    }
    // drain: every issued copy must land before the CTA's shared memory is
    // released (returns at once after a normal run; bounded otherwise)
    if (tid == 0) {
        for (int i = max(0, issued - nstages); i < issued; ++i) {
            const int buf = i % nstages;
            mbar_wait_bounded(&bar[buf], (uint32_t)(i / nstages) & 1u, a.status);
        }
        if (a.act_bulk) mbar_wait_bounded(act_bar, 0, a.status);
    }
}

struct Variant {
    int wr, gpl;
};

// Lanes per row = 32*WR, each owning GPL half-blocks of 128 weights.
Variant pick_variant(int NH) {
    if (NH <= 32) return {1, 1};
    if (NH <= 64) return {2, 1};
    if (NH <= 128) return {4, 1};
    if (NH <= 256) return {8, 1};
    if (NH <= 512) return {8, 2};
    return {0, 0};
}

template <int IN, int EPI>
void *kernel_ptr(int wr, int gpl) {
    if (wr == 1) return (void *)q4k_gemv_kernel<1, 1, IN, EPI>;
    if (wr == 2) return (void *)q4k_gemv_kernel<2, 1, IN, EPI>;
    if (wr == 4) return (void *)q4k_gemv_kernel<4, 1, IN, EPI>;
    if (wr == 8 && gpl == 1) return (void *)q4k_gemv_kernel<8, 1, IN, EPI>;
    if (wr == 8 && gpl == 2) return (void *)q4k_gemv_kernel<8, 2, IN, EPI>;
    return nullptr;
}

void *select_kernel(int in, int epi, int wr, int gpl) {
#define LALB_SEL(I, E) \
    if (in == I && epi == E) return kernel_ptr<I, E>(wr, gpl);
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
    const Variant v = pick_variant(a.K / 128);
    if (!v.wr) return lalb_fail(ctx, LALB_ERR_UNSUPPORTED, "q4k gemv: K=%d > 65536", a.K);
    if (in == kInQ8 && (reinterpret_cast<uintptr_t>(a.xq) & 15))
        return lalb_fail(ctx, LALB_ERR_INVALID, "q4k gemv: xq must be 16-byte aligned");
    void *fn = select_kernel(in, epi, v.wr, v.gpl);
    if (!fn) return lalb_fail(ctx, LALB_ERR_UNSUPPORTED, "q4k gemv: no variant in=%d epi=%d", in, epi);

    // activations arrive by bulk copy when aligned (and, for fp32, small
    // enough to stage in shared memory)
    const auto al16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    if (in == kInQ8)
        a.act_bulk = al16(a.xq) && al16(a.sx) && al16(a.sumq);
    else
        a.act_bulk = a.K <= kMaxStagedK && al16(a.x);
    const int xf = (in != kInQ8 && a.act_bulk) ? a.K : 0;

    // pipeline depth: fill the per-CTA shared-memory budget
    const size_t budget = ctas_per_sm >= 2 ? 110 * 1024 : ctx->smem_optin - 1024;
    const Layout base = make_layout(a.K, v.wr, 0, xf);
    int nst = (int)((budget - base.off_stage) / base.stage_bytes);
    if (nst > 12) nst = 12;
    if (nst < 2) {
        nst = (int)((ctx->smem_optin - 1024 - base.off_stage) / base.stage_bytes);
        ctas_per_sm = 1;
        if (nst < 2) return lalb_fail(ctx, LALB_ERR_UNSUPPORTED, "q4k gemv: K=%d too large for smem", a.K);
        if (nst > 12) nst = 12;
    }
    a.nstages = nst;
    a.status = &ctx->scratch->status;
    const Layout L = make_layout(a.K, v.wr, nst, xf);
    {
        const int st = lalb_set_smem_attr(ctx, fn, (int)L.total);
        if (st) return st;
    }
    int resident = 0;
    LALB_CUDA_TRY(ctx, cudaOccupancyMaxActiveBlocksPerMultiprocessor(&resident, (const void *)fn,
                                                                     kThreads, L.total));
    if (resident < 1) return lalb_fail(ctx, LALB_ERR_UNSUPPORTED, "q4k gemv: CTA does not fit");
    if (ctas_per_sm > resident) ctas_per_sm = resident;
    const int nunits = a.rows / a.unit;
    int grid = ctx->sm_count * ctas_per_sm;
    if (grid > nunits) grid = nunits;

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
    return lalb_launch_q4k_gemv(ctx, a, kInF32, kEpiStore, (cudaStream_t)stream, false, 1);
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
    return lalb_launch_q4k_gemv(ctx, a, kInQ8, kEpiStore, (cudaStream_t)stream, false, 1);
}
