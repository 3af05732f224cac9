// lalb_decode_persistent.cu -- a whole decode token in one persistent kernel.
//
// The token is a chain of 4*n_layer + 1 dependent matvec phases (per layer
// qkv, o, gate/up, down; then the LM head).  Launched as separate kernels,
// every phase pays a launch, a prologue and a tail in which the SMs stream
// nothing.  Here one cooperative launch of one CTA per SM runs the whole
// chain:
//
//   * warps 0..kNP-1 are producers: lane 0 of each walks this CTA's row
//     range of every phase in order and streams its share of the chunks
//     through a ring of kSlots shared-memory slots with 1-D bulk copies (TMA
//     engine), one full/empty mbarrier pair per slot, and prefetches the
//     chunks beyond the ring into L2.  Weights never depend on activations,
//     so the producers run ahead across phase boundaries: while the CTA
//     waits for the previous phase to finish everywhere, the next phase's
//     weights are already landing;
//   * the other kNC warps are consumers.  Between phases they meet at a named
//     barrier, one thread arrives at a global counter and waits (bounded)
//     until every CTA has arrived, then they rebuild the phase's quantized
//     activation in shared memory (RMS-normalised and quantized per 32-block
//     from the fp32 vector, or copied when already quantized);
//   * a consumer takes the phase's slots round-robin and computes exactly
//     the same per-half-block arithmetic as the standalone matvec (exact
//     int32 sub-block sums, exact fp64 products, one fp32 rounding per row);
//   * epilogues: qkv stored, o and down added to the residual stream,
//     gate/up finished per 64-row tile into the quantized SwiGLU product,
//     the LM head reduced to an argmax (one 64-bit atomicMax per CTA, the
//     last CTA publishes the row and resets the counters for the next token).
//
// Every wait is bounded; an expired wait raises the status word and lets the
// kernel run to completion with whatever data it has.
#include <algorithm>

#include "lalb_internal.cuh"
#include "lalb_kernels.cuh"
#include "lalb_q4k_common.cuh"

using namespace lalb;

namespace {

// Tuning knobs (compile-time): producer and consumer warps, ring slots and
// slot size, L2 prefetch distance in chunks.
#ifndef LALB_PERSIST_NP
#define LALB_PERSIST_NP 4
#endif
#ifndef LALB_PERSIST_NC
#define LALB_PERSIST_NC 8
#endif
#ifndef LALB_PERSIST_SLOTS
#define LALB_PERSIST_SLOTS 12
#endif
#ifndef LALB_PERSIST_SLOT_BYTES
#define LALB_PERSIST_SLOT_BYTES 16384
#endif
#ifndef LALB_PERSIST_PREFETCH
#define LALB_PERSIST_PREFETCH 32
#endif
constexpr int kNP = LALB_PERSIST_NP;         // producer warps
constexpr int kNC = LALB_PERSIST_NC;         // consumer warps
constexpr int kThreads = 32 * (kNP + kNC);
constexpr int kConsThreads = 32 * kNC;
constexpr int kSlots = LALB_PERSIST_SLOTS;
constexpr uint32_t kSlotBytes = LALB_PERSIST_SLOT_BYTES;
constexpr int kMaxTiles = 8;                 // gate/up 64-row tiles per CTA
constexpr int kMaxNS = kPersistMaxFfn / 32;
constexpr uint32_t kGridSpinLimit = 1u << 22;
constexpr int kTraceFields = 8;
constexpr int kPrefetchChunks = LALB_PERSIST_PREFETCH;   // L2 prefetch distance beyond the ring
constexpr int kQuads = kConsThreads / 4;     // quantizer quads per pass
constexpr int kPrepPasses = (kPersistMaxHidden / 32 + kQuads - 1) / kQuads;
static_assert(kNC < 24, "red_s holds kNC partial sums and the scale");
static_assert((2 * kSlots) % kNC == 0, "slot reuse two uses back must be the same consumer");
static_assert(kSlots % kNP == 0, "every slot is filled by one producer");

struct Layout {
    uint32_t off_bar, off_xq, off_sx, off_sq, off_red, off_bestv, off_besti, off_tile, off_tcnt,
        off_slot, total;
};

__host__ __device__ inline uint32_t align_up(uint32_t v, uint32_t a) {
    return (v + a - 1) / a * a;
}

__host__ __device__ inline Layout make_layout() {
    Layout L;
    L.off_bar = 0;                                        // full[kSlots], empty[kSlots]
    L.off_xq = align_up(16u * kSlots, 128);
    L.off_sx = align_up(L.off_xq + kPersistMaxFfn, 16);
    L.off_sq = L.off_sx + 4 * kMaxNS;
    L.off_red = align_up(L.off_sq + 4 * kMaxNS, 16);      // 24 doubles
    L.off_bestv = L.off_red + 8 * 24;
    L.off_besti = L.off_bestv + 4 * kNC;
    L.off_tile = align_up(L.off_besti + 4 * kNC, 16);
    L.off_tcnt = L.off_tile + 4 * 64 * kMaxTiles;
    L.off_slot = align_up(L.off_tcnt + 4 * (kMaxTiles + 1), 128);
    L.total = L.off_slot + kSlots * kSlotBytes;
    return L;
}

enum : int { kQkv = 0, kO = 1, kGu = 2, kDown = 3, kHead = 4 };

struct Phase {
    const uint8_t *W;
    int kind, layer, K, rows_total, unit, row_bytes, R;
    int r0, r1, nchunks;
};

__device__ __forceinline__ Phase phase_desc(const PersistArgs &a, int p) {
    Phase d;
    d.layer = p >> 2;
    if (p == 4 * a.n_layer) {
        d.kind = kHead;
        d.W = reinterpret_cast<const uint8_t *>(a.lm_w);
        d.K = a.hidden;
        d.rows_total = a.vocab;
        d.unit = 1;
        d.row_bytes = a.hidden;
    } else {
        const lalb_layer_weights lw = a.layers[d.layer];
        d.kind = p & 3;
        switch (d.kind) {
            case kQkv:
                d.W = static_cast<const uint8_t *>(lw.wqkv);
                d.K = a.hidden;
                d.rows_total = a.q_rows + 2 * a.kv_rows;
                break;
            case kO:
                d.W = static_cast<const uint8_t *>(lw.wo);
                d.K = a.q_rows;
                d.rows_total = a.hidden;
                break;
            case kGu:
                d.W = static_cast<const uint8_t *>(lw.wgu);
                d.K = a.hidden;
                d.rows_total = 2 * a.ffn;
                break;
            default:
                d.W = static_cast<const uint8_t *>(lw.wdown);
                d.K = a.ffn;
                d.rows_total = a.hidden;
                break;
        }
        d.unit = d.kind == kGu ? 64 : 1;
        d.row_bytes = (d.K >> 8) * 144;
    }
    d.R = min(8, (int)(kSlotBytes / (uint32_t)d.row_bytes));
    if (d.kind == kGu) d.R = 1 << (31 - __clz(d.R));   // chunks never straddle a 64-row tile
    if (d.kind == kQkv || d.kind == kO) d.R = min(d.R, 4);   // small phases: every consumer gets rows
    const int units = d.rows_total / d.unit;
    d.r0 = (int)((long long)blockIdx.x * units / gridDim.x) * d.unit;
    d.r1 = (int)((long long)(blockIdx.x + 1) * units / gridDim.x) * d.unit;
    d.nchunks = (d.r1 - d.r0 + d.R - 1) / d.R;
    return d;
}

// Activations written by other CTAs in the previous phase: read at L2.
__device__ __forceinline__ void load8_cg(const float *x, float (&v)[8]) {
    const float4 a = __ldcg(reinterpret_cast<const float4 *>(x));
    const float4 b = __ldcg(reinterpret_cast<const float4 *>(x) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

__device__ __forceinline__ void cons_bar() {
    asm volatile("bar.sync 1, %0;" ::"r"(kConsThreads) : "memory");
}

// Arrives at a grid-barrier counter and waits until `target` CTAs have.
// Gives up at the spin limit or as soon as any CTA has raised the status
// word (then every later wait of the token is skipped: a failed token ends
// in seconds, not after one time-out per wait).  Returns false on failure.
__device__ __forceinline__ bool grid_arrive_wait(unsigned int *ctr, unsigned int target,
                                                 unsigned int *status) {
    // the named barrier before this call orders the CTA's writes before the
    // release; the acquire below orders every CTA's writes before the reads
    // that follow the next named barrier
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(ctr) : "memory");
    bool ok = true;
    for (uint32_t k = 0;; ++k) {
        unsigned int v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
        if (v >= target) break;
        if ((k & 15) == 15 && *(volatile unsigned int *)status) {
            ok = false;
            break;
        }
        if (k > kGridSpinLimit) {
            atomicOr(status, LALB_STATUS_WAIT_TIMEOUT);
            ok = false;
            break;
        }
        if (k > 64) __nanosleep(32);
    }
    return ok;
}

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded mbarrier wait that is skipped once this thread has seen a failure.
// Adds the number of polls to `polls`.
__device__ __forceinline__ void pwait(uint64_t *bar, uint32_t parity, unsigned int *status,
                                      bool &dead, unsigned long long &polls) {
    if (dead) return;
    for (uint32_t i = 0; i < LALB_SPIN_LIMIT; ++i) {
        ++polls;
        if (mbar_try_wait(bar, parity)) return;
    }
    if (status) atomicOr(status, LALB_STATUS_WAIT_TIMEOUT);
    dead = true;
}

// State of one consumer warp that the per-phase chunk loops share.
struct Cons {
    uint64_t *full, *empty;
    const uint8_t *slot_s;
    const int8_t *xq_s;
    const float *sx_s;
    const int *sq_s;
    float *tile_s;
    int *tcnt_s;
    int ci, lane;
    bool dead, tracing;
    float best_v;                       // LM head: this lane's best logit so far
    int best_r;                         //          and its row (-1: none)
    unsigned long long wait_ns, busy_ns, polls;   // trace only
};

// One phase's chunks for one consumer warp, specialised per phase kind so
// that each kind's loop is scheduled on its own.  Chunk g (numbered over
// the whole token) belongs to consumer g % kNC.  Before waiting for use u
// of a slot the consumer waits until use u-1 has been consumed: use u-2 was
// its own chunk (2*kSlots is a multiple of kNC), so both barriers are at
// most one phase behind and the parity waits cannot match a stale phase.
template <int KIND>
__device__ __forceinline__ void consume_phase(const PersistArgs &a, const Phase &d,
                                              uint32_t g_base, Cons &cs) {
    const int lane = cs.lane;
    const int NS = d.K >> 5, NH = d.K >> 7;
    const int myrow = ((lane >> 4) & 1) * 2 + ((lane >> 3) & 1);

    // per-lane activation registers
    int xv[32];
    double sxd[4], ad[4];
#pragma unroll
    for (int j = 0; j < 32; ++j) xv[j] = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) sxd[j] = ad[j] = 0.0;
    if (KIND == kHead) {
        // lane owns the 32-byte blocks lane + 32k, k < 4
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int c = lane + 32 * k;
            if (c < NS) {
                const int4 lo = *reinterpret_cast<const int4 *>(cs.xq_s + 32 * c);
                const int4 hi = *reinterpret_cast<const int4 *>(cs.xq_s + 32 * c + 16);
                xv[8 * k + 0] = lo.x; xv[8 * k + 1] = lo.y;
                xv[8 * k + 2] = lo.z; xv[8 * k + 3] = lo.w;
                xv[8 * k + 4] = hi.x; xv[8 * k + 5] = hi.y;
                xv[8 * k + 6] = hi.z; xv[8 * k + 7] = hi.w;
                sxd[k] = (double)cs.sx_s[c];
            }
        }
    } else if (KIND != kDown) {
        // lane owns half-block min(lane, NH-1); lanes >= NH compute a copy
        // of the last one and drop it
        const int c = min(lane, NH - 1);
        const int4 *pp = reinterpret_cast<const int4 *>(cs.xq_s + 128 * c);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int4 v = pp[j];
            xv[4 * j] = v.x;
            xv[4 * j + 1] = v.y;
            xv[4 * j + 2] = v.z;
            xv[4 * j + 3] = v.w;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            sxd[j] = (double)cs.sx_s[4 * c + j];
            ad[j] = sxd[j] * (double)cs.sq_s[4 * c + j];
        }
    }
    const int cc = min(lane, NH - 1);
    const bool lane_on = lane < NH;

    const int j0 = (int)((cs.ci + kNC - (int)(g_base % kNC)) % kNC);
    for (int j = j0; j < d.nchunks; j += kNC) {
        const uint32_t g = g_base + j;
        const int slot = g % kSlots;
        const uint32_t use = g / kSlots;
        const unsigned long long tw0 = cs.tracing ? global_ns() : 0;
        if (use > 0) pwait(&cs.empty[slot], (use - 1) & 1u, a.status, cs.dead, cs.polls);
        pwait(&cs.full[slot], use & 1u, a.status, cs.dead, cs.polls);
        const unsigned long long tw1 = cs.tracing ? global_ns() : 0;
        cs.wait_ns += tw1 - tw0;
        const uint8_t *sp = cs.slot_s + (size_t)slot * kSlotBytes;
        const int rs = d.r0 + j * d.R;
        const int nr = min(d.R, d.r1 - rs);
        // per-row values needed by the epilogue, fetched before the math
        float pre = 0.0f;
        if (lane < nr) {
            if (KIND == kO) pre = __ldcg((d.layer == 0 ? a.h_in : a.h) + rs + lane);
            if (KIND == kDown) pre = __ldcg(a.h + rs + lane);
            if (KIND == kHead) pre = a.lm_s[rs + lane];
        }
        if (KIND == kDown) {
            // K > 4096: activations from shared memory, one row at a time
            for (int r = 0; r < nr; ++r) {
                const uint8_t *rowp = sp + (size_t)r * d.row_bytes;
                double acc = 0.0;
                for (int c = lane; c < NH; c += 32) {
                    int xw[32];
                    const int4 *pp = reinterpret_cast<const int4 *>(cs.xq_s + 128 * c);
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        const int4 v = pp[q ^ (c & 7)];
                        xw[4 * q] = v.x;
                        xw[4 * q + 1] = v.y;
                        xw[4 * q + 2] = v.z;
                        xw[4 * q + 3] = v.w;
                    }
                    const float4 sx4 = reinterpret_cast<const float4 *>(cs.sx_s)[c];
                    const int4 sq4 = reinterpret_cast<const int4 *>(cs.sq_s)[c];
                    const double s4[4] = {(double)sx4.x, (double)sx4.y, (double)sx4.z,
                                          (double)sx4.w};
                    const double a4[4] = {s4[0] * (double)sq4.x, s4[1] * (double)sq4.y,
                                          s4[2] * (double)sq4.z, s4[3] * (double)sq4.w};
                    acc += q4k_half(rowp, c, xw, s4, a4, nullptr);
                }
                acc = warp_sum_d(acc);
                const float hv = __shfl_sync(0xffffffffu, pre, r);
                if (lane == 0) a.h[rs + r] = __fadd_rn(hv, (float)acc);
            }
        } else if (KIND == kHead) {
            const int h0 = (lane >> 2) & 1;
            for (int r4 = 0; r4 < nr; r4 += 4) {
                double acc[4];
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const uint8_t *rowp = sp + (size_t)min(r4 + r, nr - 1) * d.row_bytes;
                    double t = 0.0;
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const int c = lane + 32 * k;
                        if (c < NS) {
                            const uint4 A = *reinterpret_cast<const uint4 *>(rowp + 32 * c + 16 * h0);
                            const uint4 B =
                                *reinterpret_cast<const uint4 *>(rowp + 32 * c + 16 * (1 - h0));
                            const uint4 lo = h0 ? B : A, hi = h0 ? A : B;
                            int sdot = 0;
                            sdot = dp4a((int)lo.x, xv[8 * k + 0], sdot);
                            sdot = dp4a((int)lo.y, xv[8 * k + 1], sdot);
                            sdot = dp4a((int)lo.z, xv[8 * k + 2], sdot);
                            sdot = dp4a((int)lo.w, xv[8 * k + 3], sdot);
                            sdot = dp4a((int)hi.x, xv[8 * k + 4], sdot);
                            sdot = dp4a((int)hi.y, xv[8 * k + 5], sdot);
                            sdot = dp4a((int)hi.z, xv[8 * k + 6], sdot);
                            sdot = dp4a((int)hi.w, xv[8 * k + 7], sdot);
                            t = fma(sxd[k], (double)sdot, t);
                        }
                    }
                    acc[r] = r4 + r < nr ? t : 0.0;
                }
                const double v = warp_sum_rows4(acc, lane);
                const float swr = __shfl_sync(0xffffffffu, pre, (r4 + myrow) & 31);
                const int row = rs + r4 + myrow;
                if ((lane & 7) == 0 && r4 + myrow < nr) {
                    const float logit = (float)((double)swr * v);
                    if (a.logits) a.logits[row] = logit;
                    if (cs.best_r < 0 || logit > cs.best_v) {
                        cs.best_v = logit;
                        cs.best_r = row;
                    }
                }
            }
        } else {
            // K <= 4096: activations in registers, 4 rows at a time
            for (int r4 = 0; r4 < nr; r4 += 4) {
                double acc[4];
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const double v = q4k_half(sp + (size_t)min(r4 + r, nr - 1) * d.row_bytes, cc,
                                              xv, sxd, ad, nullptr);
                    acc[r] = (lane_on && r4 + r < nr) ? v : 0.0;
                }
                const double v = warp_sum_rows4(acc, lane);
                const float prev = __shfl_sync(0xffffffffu, pre, (r4 + myrow) & 31);
                const int lr = r4 + myrow, row = rs + lr;
                if ((lane & 7) == 0 && lr < nr) {
                    if (KIND == kQkv) a.qkv[row] = (float)v;
                    if (KIND == kO) a.h[row] = __fadd_rn(prev, (float)v);
                    if (KIND == kGu) cs.tile_s[row - d.r0] = (float)v;   // gate/up tile entry
                }
            }
            if (KIND == kGu) {
                // 64-row tiles: the warp that completes one finishes it
                const int t = (rs - d.r0) >> 6;
                __syncwarp();
                int last = 0;
                if (lane == 0) {
                    __threadfence_block();
                    last = atomicAdd(&cs.tcnt_s[t], nr) + nr == 64;
                }
                if (__shfl_sync(0xffffffffu, last, 0)) {
                    __threadfence_block();
                    const float av = silu_mul(cs.tile_s[t * 64 + lane], cs.tile_s[t * 64 + 32 + lane]);
                    const int gt = (d.r0 >> 6) + t;
                    quantize_block32(av, lane, a.aq + gt * 32, a.asx + gt, a.asumq + gt);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&cs.empty[slot]);
        if (cs.tracing) cs.busy_ns += global_ns() - tw1;
    }
}

__global__ void __launch_bounds__(kThreads, 1) decode_persistent_kernel(const PersistArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const Layout L = make_layout();
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.off_bar);
    uint64_t *empty = full + kSlots;
    int8_t *xq_s = reinterpret_cast<int8_t *>(smem + L.off_xq);
    float *sx_s = reinterpret_cast<float *>(smem + L.off_sx);
    int *sq_s = reinterpret_cast<int *>(smem + L.off_sq);
    double *red_s = reinterpret_cast<double *>(smem + L.off_red);
    float *bestv_s = reinterpret_cast<float *>(smem + L.off_bestv);
    int *besti_s = reinterpret_cast<int *>(smem + L.off_besti);
    float *tile_s = reinterpret_cast<float *>(smem + L.off_tile);
    int *tcnt_s = reinterpret_cast<int *>(smem + L.off_tcnt);
    uint8_t *slot_s = smem + L.off_slot;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int NP = 4 * a.n_layer + 1;

    if (tid == 0) {
        for (int s = 0; s < kSlots; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        fence_barrier_init();
    }
    __syncthreads();

    // ===================== producers ========================================
    // Producer warp w (lane 0) issues the chunks g with g % kNP == w, so each
    // slot (g % kSlots) is always filled by the same producer, in order.
    if (warp < kNP) {
        if (lane == 0) {
            const uint64_t policy = l2_evict_first_policy();
            bool dead = false;
            unsigned long long polls = 0;
            // A second cursor walks the same chunks kPrefetchChunks ahead and
            // pulls this producer's share into L2, so that HBM keeps
            // streaming while the ring is full across a phase boundary.
            int pf_p = 0, pf_j = 0;
            uint32_t pf_g = 0;
            Phase pf_d = phase_desc(a, 0);
            auto prefetch_to = [&](uint32_t g_end) {
                for (; pf_g < g_end; ++pf_g, ++pf_j) {
                    while (pf_p < NP && pf_j >= pf_d.nchunks) {
                        if (++pf_p < NP) pf_d = phase_desc(a, pf_p);
                        pf_j = 0;
                    }
                    if (pf_p >= NP) return;
                    if (pf_g % kNP != (uint32_t)warp) continue;
                    const int rs = pf_d.r0 + pf_j * pf_d.R;
                    const int nr = min(pf_d.R, pf_d.r1 - rs);
                    bulk_prefetch_l2(pf_d.W + (size_t)rs * pf_d.row_bytes,
                                     (uint32_t)(nr * pf_d.row_bytes));
                }
            };
            prefetch_to(kPrefetchChunks);
            uint32_t g = 0;
            for (int p = 0; p < NP && !dead; ++p) {
                const Phase d = phase_desc(a, p);
                for (int j = 0; j < d.nchunks; ++j, ++g) {
                    if (g % kNP != (uint32_t)warp) continue;
                    const int slot = g % kSlots;
                    const uint32_t use = g / kSlots;
                    if (use > 0) pwait(&empty[slot], (use - 1) & 1u, a.status, dead, polls);
                    if (dead) break;   // stop issuing: consumers time out once and skip
                    const int rs = d.r0 + j * d.R;
                    const int nr = min(d.R, d.r1 - rs);
                    const uint32_t bytes = (uint32_t)(nr * d.row_bytes);
                    mbar_arrive_expect_tx(&full[slot], bytes);
                    bulk_g2s(slot_s + (size_t)slot * kSlotBytes,
                             d.W + (size_t)rs * d.row_bytes, bytes, &full[slot], policy);
                    prefetch_to(g + 1 + kPrefetchChunks);
                }
                if (a.trace && warp == 0) {
                    a.trace[((size_t)blockIdx.x * NP + p) * kTraceFields + 5] = global_ns();
                    a.trace[((size_t)blockIdx.x * NP + p) * kTraceFields + 6] = polls;
                    polls = 0;
                }
            }
        }
        return;
    }

    // ===================== consumers ========================================
    const int ci = warp - kNP;        // consumer index 0..kNC-1
    const int ct = tid - 32 * kNP;    // consumer thread 0..kConsThreads-1
    uint32_t g_base = 0;
    int *abort_s = tcnt_s + kMaxTiles;   // CTA-wide: a grid barrier failed
    Cons cs;
    cs.full = full;
    cs.empty = empty;
    cs.slot_s = slot_s;
    cs.xq_s = xq_s;
    cs.sx_s = sx_s;
    cs.sq_s = sq_s;
    cs.tile_s = tile_s;
    cs.tcnt_s = tcnt_s;
    cs.ci = ci;
    cs.lane = lane;
    cs.dead = false;
    cs.tracing = a.trace != nullptr && ct == 0;
    cs.best_v = 0.0f;
    cs.best_r = -1;
    cs.wait_ns = cs.busy_ns = cs.polls = 0;

    for (int p = 0; p < NP; ++p) {
        const Phase d = phase_desc(a, p);
        const int NS = d.K >> 5;

        // ---- every CTA must have finished phase p-1 --------------------------
        if (p > 0) {
            cons_bar();
            if (ct == 0) {
                unsigned long long *tr =
                    a.trace ? a.trace + ((size_t)blockIdx.x * NP + p - 1) * kTraceFields : nullptr;
                if (tr) {
                    tr[0] = global_ns();
                    tr[3] = cs.wait_ns;
                    tr[4] = cs.busy_ns;
                    tr[7] = cs.polls;
                    cs.wait_ns = cs.busy_ns = cs.polls = 0;
                }
                *abort_s = !grid_arrive_wait(&a.gbar[p - 1], gridDim.x, a.status);
                if (tr) tr[1] = global_ns();
            }
            cons_bar();
            if (*abort_s) cs.dead = true;
        }

        // ---- the phase's activation in shared memory -------------------------
        if (d.kind == kDown) {
            // 16-byte chunk q of half-block c is stored at chunk q ^ (c & 7):
            // the eight lanes of a 128-bit load phase then hit distinct banks
            const int4 *src = reinterpret_cast<const int4 *>(a.aq);
            int4 *dst = reinterpret_cast<int4 *>(xq_s);
#pragma unroll 4
            for (int i = ct; i < d.K / 16; i += kConsThreads) {
                const int c = i >> 3;
                dst[(c << 3) | ((i & 7) ^ (c & 7))] = __ldcg(src + i);
            }
            for (int i = ct; i < NS; i += kConsThreads) {
                sx_s[i] = __ldcg(a.asx + i);
                sq_s[i] = __ldcg(a.asumq + i);
            }
        } else {
            // one round trip to L2: every thread loads its quads' elements,
            // then the RMS scale (sum of squares in double) and the quantizer
            // work from registers
            const float *src = d.kind == kO ? a.qkv : ((p == 0) ? a.h_in : a.h);
            const int quad = ct >> 2, qi = ct & 3;
            float v[kPrepPasses][8];
            double ss = 0.0;
#pragma unroll
            for (int ps = 0; ps < kPrepPasses; ++ps) {
                const int blk = ps * kQuads + quad;
                if (blk < NS) {
                    load8_cg(src + blk * 32 + 8 * qi, v[ps]);
#pragma unroll
                    for (int i = 0; i < 8; ++i) ss += (double)v[ps][i] * (double)v[ps][i];
                } else {
#pragma unroll
                    for (int i = 0; i < 8; ++i) v[ps][i] = 0.0f;
                }
            }
            if (d.kind != kO) {
                ss = warp_sum_d(ss);
                if (lane == 0) red_s[ci] = ss;
                cons_bar();
                if (ct == 0) {
                    double t = 0.0;
                    for (int w = 0; w < kNC; ++w) t += red_s[w];
                    red_s[kNC] = (double)(float)(1.0 / sqrt(t / (double)d.K + 1e-6));
                }
                cons_bar();
                const float scale = (float)red_s[kNC];
#pragma unroll
                for (int ps = 0; ps < kPrepPasses; ++ps)
#pragma unroll
                    for (int i = 0; i < 8; ++i) v[ps][i] = __fmul_rn(v[ps][i], scale);
            }
#pragma unroll
            for (int ps = 0; ps < kPrepPasses; ++ps) {
                const int blk = ps * kQuads + quad;
                // whole warps take part (the quad shuffles need every lane)
                if (ps * kQuads + (ct & ~31) / 4 < NS)
                    quantize_block_quad(v[ps], qi, blk < NS, xq_s + blk * 32, sx_s + blk, sq_s + blk);
            }
        }
        if (d.kind == kGu && ct < kMaxTiles) tcnt_s[ct] = 0;
        cons_bar();
        if (ct == 0 && a.trace) a.trace[((size_t)blockIdx.x * NP + p) * kTraceFields + 2] = global_ns();

        switch (d.kind) {
            case kQkv: consume_phase<kQkv>(a, d, g_base, cs); break;
            case kO: consume_phase<kO>(a, d, g_base, cs); break;
            case kGu: consume_phase<kGu>(a, d, g_base, cs); break;
            case kDown: consume_phase<kDown>(a, d, g_base, cs); break;
            default: consume_phase<kHead>(a, d, g_base, cs); break;
        }
        g_base += d.nchunks;
    }

    // Every issued copy has been waited for above unless a wait expired; in
    // that case wait (bounded) for the last copy of every slot so that none
    // lands after the CTA has exited.
    if (ct == 0 && *(volatile unsigned int *)a.status) {
        for (uint32_t g = g_base > kSlots ? g_base - kSlots : 0; g < g_base; ++g)
            mbar_wait_bounded(&full[g % kSlots], (g / kSlots) & 1u, nullptr);
    }

    // ---- LM head argmax: CTA best, one atomic, last CTA publishes ----------------
    {
        // reduce the warp's candidates (lanes 0, 8, 16, 24), first maximum wins
        float best_v = cs.best_v;
        int best_r = cs.best_r;
#pragma unroll
        for (int o = 8; o < 32; o <<= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
            const int orr = __shfl_xor_sync(0xffffffffu, best_r, o);
            if (orr >= 0 && (best_r < 0 || ov > best_v || (ov == best_v && orr < best_r))) {
                best_v = ov;
                best_r = orr;
            }
        }
        if (lane == 0) {
            bestv_s[ci] = best_v;
            besti_s[ci] = best_r;
        }
        cons_bar();
        if (ct == 0 && a.trace) {
            unsigned long long *tr = a.trace + ((size_t)blockIdx.x * NP + NP - 1) * kTraceFields;
            tr[0] = tr[1] = global_ns();
            tr[3] = cs.wait_ns;
            tr[4] = cs.busy_ns;
            tr[7] = cs.polls;
        }
        if (ct == 0) {
            float bv = 0.0f;
            int br = -1;
            for (int w = 0; w < kNC; ++w) {
                const int r = besti_s[w];
                if (r < 0) continue;
                const float v = bestv_s[w];
                if (br < 0 || v > bv || (v == bv && r < br)) {
                    bv = v;
                    br = r;
                }
            }
            if (br >= 0) {
                const unsigned long long key = ((unsigned long long)ordered_key(bv) << 32) |
                                               (unsigned long long)(0xFFFFFFFFu - (uint32_t)br);
                atomicMax(a.best, key);
            }
            __threadfence();
            const unsigned int t = atomicAdd(a.ticket, 1u);
            if (t == gridDim.x - 1) {
                // every CTA is past every barrier: publish and reset for the next token
                const unsigned long long key = atomicExch(a.best, 0ull);
                if (a.argmax) *a.argmax = (int32_t)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull));
                for (int q = 0; q < NP - 1; ++q) a.gbar[q] = 0;
                __threadfence();
                atomicExch(a.ticket, 0u);
            }
        }
    }
}

}  // namespace

int lalb_persist_smem_bytes() { return (int)make_layout().total; }
int lalb_persist_max_tiles() { return kMaxTiles; }

int lalb_launch_persist(lalb_ctx *ctx, const PersistArgs &a, cudaStream_t stream) {
    const Layout L = make_layout();
    {
        const int st = lalb_set_smem_attr(ctx, (const void *)decode_persistent_kernel, (int)L.total);
        if (st) return st;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ctx->sm_count);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = L.total;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;   // all CTAs resident: grid barriers are safe
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    PersistArgs args = a;
    void *params[] = {&args};
    LALB_CUDA_TRY(ctx, cudaLaunchKernelExC(&cfg, (const void *)decode_persistent_kernel, params));
    return LALB_OK;
}
