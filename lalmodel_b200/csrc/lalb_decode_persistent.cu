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
//     so the L2 prefetch runs ahead across phase boundaries and HBM keeps
//     streaming while the CTA waits for the previous phase to finish
//     everywhere; a phase's shared-memory copies start once this CTA has
//     arrived at that wait (copies in flight would hold up its release
//     fence), and they hit L2;
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
#include <atomic>

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
constexpr uint32_t kWaitIterCap = 1u << 28;   // safety net beside the time limit
constexpr int kTraceFields = 8;
constexpr uint32_t kGoSpinCap = 1u << 22;      // producer's pause at a phase start, bounded
constexpr int kPrefetchChunks = LALB_PERSIST_PREFETCH;   // L2 prefetch distance beyond the ring
constexpr int kQuads = kConsThreads / 4;     // quantizer quads per pass
// Register split (setmaxnreg): the producer warps, in which one lane issues
// the copies, give up registers to the consumer warps, whose exact Q4_K/Q8
// arithmetic is latency-bound at two warps per SM sub-partition and
// schedules better with more registers (measured, the matmul-only token on
// one box: 813-815 tok/s without the split, 820-821 with 56/224, 821-825
// with 40/232).  The block is launched with kThreads x 168 registers (ptxas
// reports 168 for every instantiation, and the launcher checks it); each
// split adds up to exactly that: 4 x 32 x 40 + 8 x 32 x 232 = 4 x 32 x 56 +
// 8 x 32 x 224 = 384 x 168.  The kernel with the attention phase keeps 56
// for its producers, whose phase descriptions need them.
constexpr int kLaunchRegs = 168;
constexpr int kProdRegs(int ppl) { return ppl == 4 ? 40 : 56; }
constexpr int kConsRegs(int ppl) { return ppl == 4 ? 232 : 224; }
static_assert(kNP * 32 * kProdRegs(4) + kNC * 32 * kConsRegs(4) <= kThreads * kLaunchRegs &&
                  kNP * 32 * kProdRegs(5) + kNC * 32 * kConsRegs(5) <= kThreads * kLaunchRegs,
              "the register split must fit the block's launch allocation");
static_assert(kNP == 4 && kNC % 4 == 0, "setmaxnreg works on whole warpgroups");
constexpr int kPrepPasses = (kPersistMaxHidden / 32 + kQuads - 1) / kQuads;
static_assert(kNC < 24, "red_s holds kNC partial sums and the scale");
static_assert((2 * kSlots) % kNC == 0, "slot reuse two uses back must be the same consumer");
static_assert(kSlots % kNP == 0, "every slot is filled by one producer");
static_assert(kNC == kAttnWarps, "the attention items run on the consumer warps");
static_assert(kPersistMaxFfn >= (int)kAttnSmemBytes, "attention scratch lives in the xq area");

struct Layout {
    uint32_t off_bar, off_xq, off_sx, off_sq, off_red, off_bestv, off_besti, off_tile, off_tcnt,
        off_go, off_slot, total;
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
    L.off_go = L.off_tcnt + 4 * (kMaxTiles + 1);            // last phase arrived for
    L.off_slot = align_up(L.off_go + 4, 128);
    L.total = L.off_slot + kSlots * kSlotBytes;
    return L;
}

enum : int { kQkv = 0, kAttn = 1, kO = 2, kGu = 3, kDown = 4, kHead = 5, kSmall = 6 };

// Kind of phase p: per layer qkv, (attention,) o, gate/up, down; then the head.
template <int PPL>
__device__ __forceinline__ int phase_kind(const PersistArgs &a, int p) {
    if (p == PPL * a.n_layer) return kHead;
    const int k = p % PPL;
    return PPL == 5 ? k : (k == 0 ? kQkv : k + 1);
}

struct Phase {
    const uint8_t *W;                   // this rank's row shard
    int kind, layer, K, rows_total, unit, row_bytes, R;
    int goff;                           // global index of the shard's first row
    int r0, r1, nchunks;                // this CTA's rows, relative to the shard
};

// Where this CTA sits: its rank (group of cta_per_rank CTAs) and its index
// within the rank's CTAs.
struct Where {
    int rl;        // rank - rank0
    int rank;
    int cb;        // CTA index within the rank
};

template <int PPL>
__device__ __forceinline__ Phase phase_desc(const PersistArgs &a, int p, const Where &w) {
    Phase d;
    d.layer = p / PPL;
    const PersistRank &rk = a.rk[w.rl];
    lalb_decoder_cfg c;
    c.n_layer = a.n_layer;
    c.hidden = a.hidden;
    c.q_rows = a.q_rows;
    c.kv_rows = a.kv_rows;
    c.ffn = a.ffn;
    c.vocab = a.vocab;
    int g0, g1;
    d.kind = phase_kind<PPL>(a, p);
    if (d.kind == kAttn) {
        // no weights: the producers skip the phase (their L2 prefetch runs
        // on into o's rows), the consumers run the attention items
        d.W = nullptr;
        d.K = a.q_rows;
        d.unit = 1;
        d.row_bytes = 0;
        d.goff = d.rows_total = d.r0 = d.r1 = d.nchunks = 0;
        d.R = 1;
        return d;
    }
    if (d.kind == kHead) {
        d.W = reinterpret_cast<const uint8_t *>(rk.lm_w);
        d.K = a.hidden;
        d.unit = 1;
        d.row_bytes = a.hidden;
        lalb_tp_range(c, 4, a.n_rank, w.rank, &g0, &g1);
    } else {
        const lalb_layer_weights lw = rk.layers[d.layer];
        switch (d.kind) {
            case kQkv:
                d.W = static_cast<const uint8_t *>(lw.wqkv);
                d.K = a.hidden;
                break;
            case kO:
                d.W = static_cast<const uint8_t *>(lw.wo);
                d.K = a.q_rows;
                break;
            case kGu:
                d.W = static_cast<const uint8_t *>(lw.wgu);
                d.K = a.hidden;
                break;
            default:
                d.W = static_cast<const uint8_t *>(lw.wdown);
                d.K = a.ffn;
                break;
        }
        d.unit = d.kind == kGu ? 64 : 1;
        d.row_bytes = (d.K >> 8) * 144;
        // matrix numbers of lalb_tp_range: 0 qkv, 1 o, 2 gate/up, 3 down
        const int matrix = d.kind == kQkv ? 0 : d.kind == kO ? 1 : d.kind == kGu ? 2 : 3;
        lalb_tp_range(c, matrix, a.n_rank, w.rank, &g0, &g1);
    }
    d.goff = g0;
    d.rows_total = g1 - g0;
    d.R = min(8, (int)(kSlotBytes / (uint32_t)d.row_bytes));
    if (d.kind == kGu) d.R = 1 << (31 - __clz(d.R));   // chunks never straddle a 64-row tile
    if (d.kind == kQkv || d.kind == kO) d.R = min(d.R, 4);   // small phases: every consumer gets rows
    const int units = d.rows_total / d.unit;
    const int G = a.cta_per_rank;
    // 32-bit: units < 2^24 and cb < 256
    d.r0 = (int)((unsigned)w.cb * (unsigned)units / (unsigned)G) * d.unit;
    d.r1 = (int)((unsigned)(w.cb + 1) * (unsigned)units / (unsigned)G) * d.unit;
    d.nchunks = (d.r1 - d.r0 + d.R - 1) / d.R;
    return d;
}

// Views of one rank's exchange buffer.
struct XView {
    unsigned int *gbar, *seq, *ticket;
    int *pos;
    unsigned long long *best, *keys;
    float *h, *q, *att;
    unsigned int *att_cnt;
    double *att_part;
    int8_t *aq;
    float *asx;
    int *asumq;
};
template <int PPL>
__device__ __forceinline__ PersistXLayout xlayout(const PersistArgs &a) {
    return lalb_persist_xlayout(a.n_layer, a.hidden, a.q_rows, a.kv_rows, a.ffn,
                                PPL == 5 ? a.head_dim : 0);
}
template <int PPL>
__device__ __forceinline__ XView xview(const PersistArgs &a, int rank) {
    const PersistXLayout L = xlayout<PPL>(a);
    unsigned char *b = a.xb[rank];
    XView v;
    v.gbar = reinterpret_cast<unsigned int *>(b + L.gbar);
    v.seq = reinterpret_cast<unsigned int *>(b + L.seq);
    v.ticket = reinterpret_cast<unsigned int *>(b + L.ticket);
    v.pos = reinterpret_cast<int *>(b + L.pos);
    v.att = reinterpret_cast<float *>(b + L.att);
    v.att_cnt = reinterpret_cast<unsigned int *>(b + L.att_cnt);
    v.att_part = reinterpret_cast<double *>(b + L.att_part);
    v.best = reinterpret_cast<unsigned long long *>(b + L.best);
    v.keys = reinterpret_cast<unsigned long long *>(b + L.keys);
    v.h = reinterpret_cast<float *>(b + L.h);
    v.q = reinterpret_cast<float *>(b + L.q);
    v.aq = reinterpret_cast<int8_t *>(b + L.aq);
    v.asx = reinterpret_cast<float *>(b + L.asx);
    v.asumq = reinterpret_cast<int *>(b + L.asumq);
    return v;
}

// Activations written by other CTAs in the previous phase: read at L2.
__device__ __forceinline__ void load8_cg(const float *x, float (&v)[8]) {
    const float4 a = __ldcg(reinterpret_cast<const float4 *>(x));
    const float4 b = __ldcg(reinterpret_cast<const float4 *>(x) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void cons_bar() {
    asm volatile("bar.sync 1, %0;" ::"r"(kConsThreads) : "memory");
}

struct ConsBar {
    __device__ void operator()() const { cons_bar(); }
};

// Two-level phase barrier.  Every CTA arrives on its own rank's counter
// lbar[ph] (GPU scope, release); the CTA whose arrival completes the rank
// (it sees the count reach its target) acquires and then adds one to rbar[ph] of
// every other rank with a system-scope release when ranks live on other
// GPUs.  Its acquire saw every CTA of its rank, so the release also carries
// their stores into the other ranks' buffers.  A CTA then waits until its
// rank's lbar[ph] has all local CTAs and rbar[ph] all other ranks.  Both
// counters grow across tokens (targets from the token count `seq`; the
// comparisons survive wrap-around).  Gives up after a.wait_ns, or as soon
// as this rank's status word is raised (then every later grid wait of the
// token gives up at once: a failed token ends after one time-out, not one
// per wait).  Returns false on failure.
// Phases whose outputs go to other ranks (gate/up, down): their barrier waits
// for every rank; after qkv and o (computed whole on every rank) a rank only
// waits for its own CTAs.
template <int PPL>
__device__ __forceinline__ bool cross_phase(const PersistArgs &a, int ph) {
    const int k = phase_kind<PPL>(a, ph);
    return k == kGu || k == kDown;
}

// Called by the 32 threads of the CTA's first consumer warp (lane = 0..31).
// The rank's last arrival signals the other ranks from one warp instruction:
// lane j adds to rank j's counter, so the system-scope releases to the peers
// are issued together rather than one after another (n_rank <= 8 <= 32).
template <int PPL>
__device__ __forceinline__ void grid_arrive(const PersistArgs &a, const XView &own, int rank,
                                            int ph, unsigned int seq, int lane) {
    const unsigned int nl = a.cta_per_rank, nr = cross_phase<PPL>(a, ph) ? a.n_rank - 1 : 0;
    const unsigned int t_local = (seq + 1u) * nl;
    unsigned int *lbar = own.gbar + ph;
    if (nr == 0) {
        if (lane == 0) {
            asm volatile("fence.acq_rel.gpu;" ::: "memory");
            asm volatile("red.relaxed.gpu.global.add.u32 [%0], 1;" ::"l"(lbar) : "memory");
        }
        return;
    }
    unsigned int last = 0;
    if (lane == 0) {
        unsigned int old;
        asm volatile("atom.release.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(lbar) : "memory");
        last = old + 1u == t_local;
        // the rank's last arrival: acquire every other CTA's release first
        if (last) asm volatile("fence.acq_rel.gpu;" ::: "memory");
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    __syncwarp();   // lane 0's acquire happens before the other lanes' releases
    if (last && lane < a.n_rank && lane != rank) {
        unsigned int *ctr = xview<PPL>(a, lane).gbar + PPL * a.n_layer + ph;
        if (a.remote)
            asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(ctr) : "memory");
        else
            asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(ctr) : "memory");
    }
}

template <int PPL>
__device__ __forceinline__ bool grid_wait(const PersistArgs &a, const XView &own, int ph,
                                          unsigned int seq) {
    const unsigned int nl = a.cta_per_rank, nr = cross_phase<PPL>(a, ph) ? a.n_rank - 1 : 0;
    const unsigned int t_local = (seq + 1u) * nl, t_remote = (seq + 1u) * nr;
    unsigned int *lbar = own.gbar + ph;
    unsigned int *rbar = own.gbar + PPL * a.n_layer + ph;
    bool ok = true;
    unsigned long long t0 = 0;
    bool local_done = false;
    for (uint32_t k = 0;; ++k) {
        unsigned int v;
        if (!local_done) {
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(lbar) : "memory");
            local_done = (int)(v - t_local) >= 0;
        }
        if (local_done) {
            if (nr == 0) break;
            if (a.remote)
                asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(rbar) : "memory");
            else
                asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(rbar) : "memory");
            if ((int)(v - t_remote) >= 0) break;
        }
        if ((k & 15) == 15 && *(volatile unsigned int *)a.status) {
            ok = false;
            break;
        }
        if ((k & 255) == 255) {
            const unsigned long long t = global_ns();
            if (t0 == 0) t0 = t;
            else if (t - t0 > a.wait_ns) k = kWaitIterCap;
        }
        if (k >= kWaitIterCap) {
            atomicOr(a.status, LALB_STATUS_WAIT_TIMEOUT);
            ok = false;
            break;
        }
        if (k > 64) __nanosleep(32);
    }
    return ok;
}

// The ranks' LM-head keys: each rank's last CTA stored its key into every
// rank's buffer, then arrives here once per rank (the counter after the
// phase counters) and waits for all n_rank arrivals of this token.
template <int PPL>
__device__ __forceinline__ bool keys_arrive_wait(const PersistArgs &a, const XView &own,
                                                 unsigned int seq) {
    for (int j = 0; j < a.n_rank; ++j) {
        unsigned int *ctr = xview<PPL>(a, j).gbar + 2 * PPL * a.n_layer;
        if (a.remote)
            asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(ctr) : "memory");
        else
            asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(ctr) : "memory");
    }
    const unsigned int target = (seq + 1u) * (unsigned int)a.n_rank;
    unsigned int *kb = own.gbar + 2 * PPL * a.n_layer;
    unsigned long long t0 = 0;
    for (uint32_t k = 0;; ++k) {
        unsigned int v;
        if (a.remote)
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(kb) : "memory");
        else
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(kb) : "memory");
        if ((int)(v - target) >= 0) return true;
        if ((k & 15) == 15 && *(volatile unsigned int *)a.status) return false;
        if ((k & 255) == 255) {
            const unsigned long long t = global_ns();
            if (t0 == 0) t0 = t;
            else if (t - t0 > a.wait_ns) k = kWaitIterCap;
        }
        if (k >= kWaitIterCap) {
            atomicOr(a.status, LALB_STATUS_WAIT_TIMEOUT);
            return false;
        }
        if (k > 64) __nanosleep(32);
    }
}

// Bounded mbarrier wait that is skipped once this thread has seen an
// mbarrier wait expire.  Adds the number of polls to `polls`.
// The limit is time-based (4 x a.wait_ns on the global timer, with an
// iteration cap as well): a producer waiting for a free slot legitimately
// waits as long as its consumers wait at a grid barrier (up to a.wait_ns,
// on other GPUs whose launches can lag), so its own limit is longer.  A
// grid barrier that gave up does NOT make the CTA skip mbarrier waits: the
// producers keep issuing and the consumers keep waiting for every copy, so
// no copy is ever in flight when a slot is refilled or the CTA exits.
__device__ __forceinline__ void pwait(const PersistArgs &a, uint64_t *bar, uint32_t parity,
                                      bool &dead, unsigned long long &polls) {
    if (dead || mbar_test_wait(bar, parity)) return;
    const unsigned long long limit = 4ull * a.wait_ns;
    unsigned long long t0 = 0;
    for (uint32_t i = 0; i < kWaitIterCap; ++i) {
        ++polls;
        if (mbar_try_wait(bar, parity)) return;
        if ((i & 63) == 63) {
            const unsigned long long t = global_ns();
            if (t0 == 0) t0 = t;
            else if (t - t0 > limit) break;
        }
    }
    atomicOr(a.status, LALB_STATUS_WAIT_TIMEOUT);
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
template <int KIND, int PPL>
__device__ __forceinline__ void consume_phase(const PersistArgs &a, const Phase &d,
                                              uint32_t g_base, const PersistXLayout &XL,
                                              const XView &own, const PersistRank &rk, Cons &cs) {
    const int lane = cs.lane;
    const int NS = d.K >> 5, NH = d.K >> 7;
    // kSmall: one instantiation for qkv, o and gate/up, the kind read at run time
    const int kind = KIND == kSmall ? d.kind : KIND;
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
                // block c = chunks 2(c%4), 2(c%4)+1 of half-block c/4 (swizzled layout)
                const int4 *xs = reinterpret_cast<const int4 *>(cs.xq_s);
                const int4 lo = xs[xq_swz_chunk(c >> 2, 2 * (c & 3))];
                const int4 hi = xs[xq_swz_chunk(c >> 2, 2 * (c & 3) + 1)];
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
            const int4 v = pp[j ^ (c & 7)];   // swizzled: conflict-free across lanes
            xv[4 * j] = v.x;
            xv[4 * j + 1] = v.y;
            xv[4 * j + 2] = v.z;
            xv[4 * j + 3] = v.w;
        }
        const float4 sx4 = reinterpret_cast<const float4 *>(cs.sx_s)[c];   // one 16-byte load each
        const int4 sq4 = reinterpret_cast<const int4 *>(cs.sq_s)[c];
        const float sxa[4] = {sx4.x, sx4.y, sx4.z, sx4.w};
        const int sqa[4] = {sq4.x, sq4.y, sq4.z, sq4.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            sxd[j] = (double)sxa[j];
            ad[j] = sxd[j] * (double)sqa[j];
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
        if (use > 0) pwait(a, &cs.empty[slot], (use - 1) & 1u, cs.dead, cs.polls);
        pwait(a, &cs.full[slot], use & 1u, cs.dead, cs.polls);
        const unsigned long long tw1 = cs.tracing ? global_ns() : 0;
        cs.wait_ns += tw1 - tw0;
        const uint8_t *sp = cs.slot_s + (size_t)slot * kSlotBytes;
        const int rs = d.r0 + j * d.R;
        const int nr = min(d.R, d.r1 - rs);
        // per-row values needed by the epilogue, fetched before the math
        // (the residual rows of o and down are this rank's own rows)
        float pre = 0.0f;
        if (lane < nr) {
            const int grow = d.goff + rs + lane;
            if (kind == kO) pre = __ldcg((d.layer == 0 ? a.h_in : own.h) + grow);
            if (KIND == kDown) pre = __ldcg(own.h + grow);
            if (KIND == kHead) pre = rk.lm_s[rs + lane];
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
                // the new residual row goes to every rank
                if (lane == 0) {
                    const float hn = __fadd_rn(hv, (float)acc);
                    for (int j = 0; j < a.n_rank; ++j)
                        reinterpret_cast<float *>(a.xb[j] + XL.h)[d.goff + rs + r] = hn;
                }
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
                const int row = d.goff + rs + r4 + myrow;   // global vocabulary row
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
                const int lr = r4 + myrow, row = rs + lr, grow = d.goff + row;
                if ((lane & 7) == 0 && lr < nr) {
                    // every rank computes all of qkv and of the residual update, so
                    // they stay in its own buffer (k and v are read by the
                    // attention phase, when there is one)
                    if (kind == kQkv && (PPL == 5 || grow < a.q_rows)) own.q[grow] = (float)v;
                    if (kind == kO) own.h[grow] = __fadd_rn(prev, (float)v);
                    if (kind == kGu) cs.tile_s[row - d.r0] = (float)v;   // gate/up tile entry
                }
            }
            if (kind == kGu) {
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
                    const int gt = ((d.goff + d.r0) >> 6) + t;   // global 32-block of the product
                    // quantized once (same operations as quantize_block32), stored to every rank
                    const uint32_t amax = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(av)));
                    const float dsc = __fdiv_rn(__uint_as_float(amax), 127.0f);
                    const float id = dsc != 0.0f ? __fdiv_rn(1.0f, dsc) : 0.0f;
                    const float tq = roundf(__fmul_rn(av, id));
                    const int q = tq > 127.0f ? 127 : (tq < -127.0f ? -127 : (int)tq);
                    const int qsum = __reduce_add_sync(0xffffffffu, q);
                    for (int j = 0; j < a.n_rank; ++j) {
                        (reinterpret_cast<int8_t *>(a.xb[j] + XL.aq) + gt * 32)[lane] = (int8_t)q;
                        if (lane == 0) {
                            reinterpret_cast<float *>(a.xb[j] + XL.asx)[gt] = dsc;
                            reinterpret_cast<int *>(a.xb[j] + XL.asumq)[gt] = qsum;
                        }
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&cs.empty[slot]);
        if (cs.tracing) cs.busy_ns += global_ns() - tw1;
    }
}

// PPL (phases per layer) is 4 for the matmul set and 5 with the attention
// phase; NORM is whether any RMSNorm weight vector is set.  Each combination
// is its own instantiation, so that the matmul-only kernel with unit norms
// carries neither the attention code nor the norm weights' registers in its
// activation prologue (measured: 2-3 % of the token with them).
template <int PPL, bool NORM>
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
    volatile int *go_s = reinterpret_cast<volatile int *>(smem + L.off_go);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int NP = PPL * a.n_layer + 1;
    Where w;
    w.rl = blockIdx.x / a.cta_per_rank;
    w.rank = a.rank0 + w.rl;
    w.cb = blockIdx.x % a.cta_per_rank;
    const PersistXLayout XL = xlayout<PPL>(a);
    const XView own = xview<PPL>(a, w.rank);
    const PersistRank &rk = a.rk[w.rl];

    if (tid == 0) {
        for (int s = 0; s < kSlots; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        fence_barrier_init();
        *go_s = 0;
    }
    __syncthreads();

    // ===================== producers ========================================
    // Producer warp w (lane 0) issues the chunks g with g % kNP == w, so each
    // slot (g % kSlots) is always filled by the same producer, in order.
    if (warp < kNP) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kProdRegs(PPL)) : "memory");
        if (lane == 0) {
            const uint64_t policy = l2_evict_first_policy();
            bool dead = false;
            unsigned long long polls = 0;
            // A second cursor walks the same chunks kPrefetchChunks ahead and
            // pulls this producer's share into L2, so that HBM keeps
            // streaming while the ring is full across a phase boundary.
            int pf_p = 0, pf_j = 0;
            uint32_t pf_g = 0;
            Phase pf_d = phase_desc<PPL>(a, 0, w);
            auto prefetch_to = [&](uint32_t g_end) {
                for (; pf_g < g_end; ++pf_g, ++pf_j) {
                    while (pf_p < NP && pf_j >= pf_d.nchunks) {
                        if (++pf_p < NP) pf_d = phase_desc<PPL>(a, pf_p, w);
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
                const Phase d = phase_desc<PPL>(a, p, w);
                // Phase p's copies wait until this CTA has arrived at the
                // barrier after phase p-1.  The arrival's release fence waits
                // for every copy the SM still has in flight (measured: 0.5 us
                // with none, 0.7-1.7 us with the next phase's copies landing),
                // and the last CTA's fence is on every CTA's critical path.
                // The L2 prefetch keeps running ahead meanwhile, so HBM stays
                // busy and the copies issued after the arrival hit L2.  Not
                // before gate/up: its 16 KB chunks landing during its RMS
                // prologue cost more than the fence after o saves (measured:
                // 813 against 799 tok/s with the pause at every phase).  The
                // pause is bounded: it only orders work, nothing depends on it.
                if (p > 0 && d.kind != kGu)
                    for (uint32_t it = 0; it < kGoSpinCap && *go_s < p; ++it) __nanosleep(32);
                for (int j = 0; j < d.nchunks; ++j, ++g) {
                    if (g % kNP != (uint32_t)warp) continue;
                    const int slot = g % kSlots;
                    const uint32_t use = g / kSlots;
                    if (use > 0) pwait(a, &empty[slot], (use - 1) & 1u, dead, polls);
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
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kConsRegs(PPL)) : "memory");
    const int ci = warp - kNP;        // consumer index 0..kNC-1
    const int ct = tid - 32 * kNP;    // consumer thread 0..kConsThreads-1
    uint32_t g_base = 0;
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

    // the phase counters grow across tokens: their targets derive from seq
    const unsigned int seq = *(volatile unsigned int *)own.seq;
    // the decode position of this token (attention); advanced by the rank's
    // last CTA after every CTA of the rank has read it
    const int pos = PPL == 5 ? *(volatile int *)own.pos : 0;

    for (int p = 0; p < NP; ++p) {
        Phase d;

        // ---- every CTA must have finished phase p-1 --------------------------
        if (p > 0) {
            cons_bar();
            unsigned long long *tr =
                a.trace && ct == 0 ? a.trace + ((size_t)blockIdx.x * NP + p - 1) * kTraceFields
                                   : nullptr;
            if (tr) {
                tr[0] = global_ns();
                tr[3] = cs.wait_ns;
                tr[4] = cs.busy_ns;
                tr[7] = cs.polls;
                cs.wait_ns = cs.busy_ns = cs.polls = 0;
            }
            if (ct < 32) grid_arrive<PPL>(a, own, w.rank, p - 1, seq, ct);
            if (ct == 0) *go_s = p;   // this CTA has arrived: the producers may go on
            if (ct == 0) {
                d = phase_desc<PPL>(a, p, w);   // while the arrivals propagate
                // a grid barrier that gives up leaves the rest of the token
                // to run on whatever data it has: later grid waits give up
                // at once (the status word is raised), mbarrier waits stay
                grid_wait<PPL>(a, own, p - 1, seq);
                if (tr) tr[1] = global_ns();
            } else {
                d = phase_desc<PPL>(a, p, w);
            }
            cons_bar();
        } else {
            d = phase_desc<PPL>(a, p, w);
        }
        const int NS = d.K >> 5;

        if (PPL == 5 && d.kind == kAttn) {
            // ---- attention over the KV cache: items (q head, position chunk)
            // over this rank's CTAs; output to own.att ----------------------------
            if (pos >= 0 && pos < a.max_ctx) {
                AttnStep st;
                st.qkv = own.q;
                st.k_cache = a.kv_cache[2 * d.layer];
                st.v_cache = a.kv_cache[2 * d.layer + 1];
                st.out = own.att;
                st.part = own.att_part;
                st.cnt = own.att_cnt;
                st.n_head = a.q_rows / a.head_dim;
                st.n_kv = a.kv_rows / a.head_dim;
                st.hd = a.head_dim;
                st.pos = pos;
                st.S = attn_chunks(st.n_head, pos, a.cta_per_rank);
                st.theta = a.rope_theta;
                attn_items(st, w.cb, a.cta_per_rank, ct, reinterpret_cast<unsigned char *>(xq_s),
                           ConsBar());
            } else {
                // outside the cache: nothing is read or written there
                if (ct == 0 && w.cb == 0) atomicOr(a.status, LALB_STATUS_BAD_POSITION);
                for (int i = w.cb * kConsThreads + ct; i < a.q_rows; i += a.cta_per_rank * kConsThreads)
                    own.att[i] = 0.0f;
            }
            if (ct == 0 && a.trace)
                a.trace[((size_t)blockIdx.x * NP + p) * kTraceFields + 2] = global_ns();
            continue;
        }

        // ---- the phase's activation in shared memory -------------------------
        if (d.kind == kDown) {
            // 16-byte chunk q of half-block c is stored at chunk q ^ (c & 7):
            // the eight lanes of a 128-bit load phase then hit distinct banks
            const int4 *src = reinterpret_cast<const int4 *>(own.aq);
            int4 *dst = reinterpret_cast<int4 *>(xq_s);
#pragma unroll 4
            for (int i = ct; i < d.K / 16; i += kConsThreads) {
                const int c = i >> 3;
                dst[(c << 3) | ((i & 7) ^ (c & 7))] = __ldcg(src + i);
            }
            for (int i = ct; i < NS; i += kConsThreads) {
                sx_s[i] = __ldcg(own.asx + i);
                sq_s[i] = __ldcg(own.asumq + i);
            }
        } else {
            // one round trip to L2: every thread loads its quads' elements
            // (and their RMSNorm weights), then the RMS scale (sum of squares
            // in double) and the quantizer work from registers
            const float *src = d.kind == kO ? (PPL == 5 ? own.att : own.q)
                                            : ((p == 0) ? a.h_in : own.h);
            // the prologue's RMSNorm weights (nullable: unit), looked up here
            // rather than carried through the phase's matvec loops
            const float *gamma = !NORM ? nullptr
                                 : d.kind == kQkv ? rk.layers[d.layer].attn_norm
                                 : d.kind == kGu ? rk.layers[d.layer].ffn_norm
                                 : d.kind == kHead ? a.out_norm : nullptr;
            const int quad = ct >> 2, qi = ct & 3;
            float v[kPrepPasses][8], gv[kPrepPasses][8];
            double ss = 0.0;
#pragma unroll
            for (int ps = 0; ps < kPrepPasses; ++ps) {
                const int blk = ps * kQuads + quad;
                if (blk < NS) {
                    load8_cg(src + blk * 32 + 8 * qi, v[ps]);
                    if (NORM && gamma) load8_cg(gamma + blk * 32 + 8 * qi, gv[ps]);
#pragma unroll
                    for (int i = 0; i < 8; ++i) ss += (double)v[ps][i] * (double)v[ps][i];
                } else {
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        v[ps][i] = 0.0f;
                        if (NORM) gv[ps][i] = 0.0f;
                    }
                }
            }
            if (d.kind != kO) {
                ss = warp_sum_d(ss);
                if (lane == 0) red_s[ci] = ss;
                cons_bar();
                // every thread adds the warps' partial sums in the same order:
                // the same scale everywhere, with one barrier fewer
                double t = 0.0;
#pragma unroll
                for (int cw = 0; cw < kNC; ++cw) t += red_s[cw];
                const float scale = (float)(1.0 / sqrt(t / (double)d.K + (double)a.rms_eps));
                // (x * s) * w, one rounding per product (rms_norm's order)
#pragma unroll
                for (int ps = 0; ps < kPrepPasses; ++ps)
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        v[ps][i] = __fmul_rn(v[ps][i], scale);
                        if (NORM && gamma) v[ps][i] = __fmul_rn(v[ps][i], gv[ps][i]);
                    }
            }
#pragma unroll
            for (int ps = 0; ps < kPrepPasses; ++ps) {
                const int blk = ps * kQuads + quad;
                // whole warps take part (the quad shuffles need every lane)
                if (ps * kQuads + (ct & ~31) / 4 < NS)
                    quantize_block_quad_swz(v[ps], qi, blk < NS, xq_s, blk, sx_s + blk, sq_s + blk);
            }
        }
        if (d.kind == kGu && ct < kMaxTiles) tcnt_s[ct] = 0;
        cons_bar();
        if (ct == 0 && a.trace) a.trace[((size_t)blockIdx.x * NP + p) * kTraceFields + 2] = global_ns();

        if constexpr (PPL == 5) {
            // With the attention phase the per-layer code no longer fits the
            // instruction cache (ncu, 2-layer token: no_instruction stalls
            // 2.09 per issue against 1.48 without attention), so qkv, o and
            // gate/up share one inlined copy of the matvec loop (one call
            // site) and the kind is read at run time.  Without attention the
            // loops specialised per kind are faster (812 against 796 tok/s).
            switch (d.kind) {
                case kQkv:
                case kO:
                case kGu: consume_phase<kSmall, PPL>(a, d, g_base, XL, own, rk, cs); break;
                case kDown: consume_phase<kDown, PPL>(a, d, g_base, XL, own, rk, cs); break;
                default: consume_phase<kHead, PPL>(a, d, g_base, XL, own, rk, cs); break;
            }
        } else {
            switch (d.kind) {
                case kQkv: consume_phase<kQkv, PPL>(a, d, g_base, XL, own, rk, cs); break;
                case kO: consume_phase<kO, PPL>(a, d, g_base, XL, own, rk, cs); break;
                case kGu: consume_phase<kGu, PPL>(a, d, g_base, XL, own, rk, cs); break;
                case kDown: consume_phase<kDown, PPL>(a, d, g_base, XL, own, rk, cs); break;
                default: consume_phase<kHead, PPL>(a, d, g_base, XL, own, rk, cs); break;
            }
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
            for (int cw = 0; cw < kNC; ++cw) {
                const int r = besti_s[cw];
                if (r < 0) continue;
                const float v = bestv_s[cw];
                if (br < 0 || v > bv || (v == bv && r < br)) {
                    bv = v;
                    br = r;
                }
            }
            if (br >= 0) {
                const unsigned long long key = ((unsigned long long)ordered_key(bv) << 32) |
                                               (unsigned long long)(0xFFFFFFFFu - (uint32_t)br);
                atomicMax(own.best, key);
            }
            __threadfence();
            const unsigned int t = atomicAdd(own.ticket, 1u);
            if (t == (unsigned int)a.cta_per_rank - 1) {
                // this rank's CTAs are all done: its key goes to every rank,
                // then the ranks' keys meet (first maximum wins: the key holds
                // ~row, so equal logits prefer the lower global row)
                const unsigned long long key = atomicExch(own.best, 0ull);
                unsigned long long kmax = key;
                bool ok = true;
                if (a.n_rank > 1) {
                    for (int j = 0; j < a.n_rank; ++j) xview<PPL>(a, j).keys[w.rank] = key;
                    __threadfence_system();
                    ok = keys_arrive_wait<PPL>(a, own, seq);
                    kmax = 0;
                    for (int j = 0; j < a.n_rank; ++j) {
                        const unsigned long long kj = __ldcg(own.keys + j);
                        kmax = kj > kmax ? kj : kmax;
                    }
                }
                if (a.argmax && w.rl == 0)
                    *a.argmax = ok && kmax ? (int32_t)(0xFFFFFFFFu - (uint32_t)(kmax & 0xFFFFFFFFull)) : -1;
                *own.ticket = 0u;
                if (PPL == 5) *own.pos = pos + 1;   // every CTA of the rank read pos
                __threadfence();
                atomicAdd(own.seq, 1u);   // the next token's counter targets
            }
        }
    }
}

}  // namespace

int lalb_persist_smem_bytes() { return (int)make_layout().total; }
int lalb_persist_max_tiles() { return kMaxTiles; }

int lalb_launch_persist(lalb_ctx *ctx, const PersistArgs &a, cudaStream_t stream) {
    const Layout L = make_layout();
    const void *fn = a.ppl == 5 ? (a.norm ? (const void *)decode_persistent_kernel<5, true>
                                          : (const void *)decode_persistent_kernel<5, false>)
                                : (a.norm ? (const void *)decode_persistent_kernel<4, true>
                                          : (const void *)decode_persistent_kernel<4, false>);
    {
        const int st = lalb_set_smem_attr(ctx, fn, (int)L.total);
        if (st) return st;
    }
    {
        // the consumers' setmaxnreg.inc waits until the producers' released
        // registers cover it: the split is sized for exactly kLaunchRegs per
        // thread at launch, so refuse any other count rather than launch a
        // kernel whose consumers could wait forever
        static std::atomic<int> regs[2][2];   // per instantiation, 0 until read
        std::atomic<int> &slot = regs[a.ppl == 5][a.norm ? 1 : 0];
        int r = slot.load(std::memory_order_relaxed);
        if (r == 0) {
            cudaFuncAttributes fa;
            LALB_CUDA_TRY(ctx, cudaFuncGetAttributes(&fa, fn));
            r = fa.numRegs;
            slot.store(r, std::memory_order_relaxed);
        }
        if (r != kLaunchRegs)
            return lalb_fail(ctx, LALB_ERR_UNSUPPORTED,
                             "decode_persistent_kernel: %d registers per thread, the register split "
                             "needs %d", r, kLaunchRegs);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.cta_per_rank * a.ranks_here);
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
    LALB_CUDA_TRY(ctx, cudaLaunchKernelExC(&cfg, fn, params));
    return LALB_OK;
}
