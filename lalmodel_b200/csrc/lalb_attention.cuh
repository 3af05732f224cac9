// lalb_attention.cuh -- one decode step of causal attention over an fp32 KV
// cache, shared by the standalone kernel (lalb_attention.cu) and the
// attention phase of the persistent decode kernel.
//
// The arithmetic is attention_forward (runtime/lal_runtime.c:833-882) after
// apply_rope (:137-153), generalised to grouped KV heads, carried out in
// double and rounded to float once per output:
//   * RoPE at position pos on every q head and k head, pairs (d, d + hd/2),
//     angle pos * theta^(-2d/hd); the rotated values are rounded to float
//     (the KV cache holds float, as in the reference);
//   * the rotated k and the v of this token go to row pos of the caches;
//   * head h attends KV head g = h / (n_head / n_kv) over positions 0..pos:
//     s_j = (q_h . k_j) / sqrt(hd), out_h = sum_j exp(s_j - max) v_j /
//     (sum_j exp(s_j - max) + 1e-12).
//
// Work unit ("item"): one q head h and one contiguous chunk c of the
// positions 0..pos (S chunks per head).  A CTA's consumer threads (8 warps)
// take an item; warp w walks positions j0 + w, j0 + w + 8, ... four at a
// time (eight row loads in flight per lane), keeping an online softmax state
// (max, sum, the head_dim accumulators spread over the lanes) in double.  The
// warps' states are merged in warp order; with S > 1 the item's state goes to
// a global partial buffer and the CTA that completes a head (arrival counter)
// merges the S partials in chunk order.  The position-pos rows are read from
// the token's own k and v (rotated in shared memory), never from the cache,
// so the cache write of this step races with nothing.
#pragma once

#include <math.h>
#include <stdint.h>

namespace lalb {

struct AttnStep {
    const float *qkv;       // this token: q [n_head*hd] | k [n_kv*hd] | v [n_kv*hd]
    float *k_cache;         // [max_ctx][n_kv*hd]
    float *v_cache;
    float *out;             // [n_head*hd]
    double *part;           // S > 1: [n_head][S][hd + 2] (max, sum, accumulators)
    unsigned int *cnt;      // S > 1: [n_head] arrival counters, 0 between steps
    int n_head, n_kv, hd, pos, S;
    double theta;
};

constexpr int kAttnWarps = 8;
constexpr int kAttnMaxHd = 256;
constexpr int kAttnMaxS = 8;    // position chunks per head at most (attn_chunks)

// Shared memory of one item (bytes): rotated q and k of the head, and the
// warps' softmax states.
constexpr uint32_t kAttnSmemBytes = 2 * kAttnMaxHd * 4 + 2 * kAttnWarps * 8 +
                                    kAttnWarps * kAttnMaxHd * 8 + 16;
// the last chunk's merge reuses the warps' states for the S partials
static_assert(kAttnMaxS * (kAttnMaxHd + 2) <= 2 * kAttnWarps + kAttnWarps * kAttnMaxHd,
              "the partials of a head fit where the warps' states were");

// Chunks per head: as many as the CTAs allow (at most 8), never more than
// the positions.
__host__ __device__ inline int attn_chunks(int n_head, int pos, int ctas) {
    int S = ctas / n_head;
    if (S > kAttnMaxS) S = kAttnMaxS;
    if (S > pos + 1) S = pos + 1;
    return S < 1 ? 1 : S;
}

// Sums U per-lane values (U = 2 or 4) over the warp at once and returns every
// total on every lane: the first exchange levels halve the values a lane
// carries (lane L ends with total ((L >> 4) & 1) * 2 + ((L >> 3) & 1) for
// U = 4, (L >> 4) & 1 for U = 2), the last ones add plainly, then each total
// is read from a lane that holds it.  10 double shuffles for U = 4 instead of
// 20 for four separate reductions.
template <int U>
__device__ __forceinline__ void attn_warp_sums(double (&v)[U], int lane) {
    static_assert(U == 2 || U == 4, "two or four values");
    const bool b4 = lane & 16;
    double x;
    if constexpr (U == 4) {
        const double w0 = (b4 ? v[2] : v[0]) + __shfl_xor_sync(0xffffffffu, b4 ? v[0] : v[2], 16);
        const double w1 = (b4 ? v[3] : v[1]) + __shfl_xor_sync(0xffffffffu, b4 ? v[1] : v[3], 16);
        const bool b3 = lane & 8;
        x = (b3 ? w1 : w0) + __shfl_xor_sync(0xffffffffu, b3 ? w0 : w1, 8);
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
#pragma unroll
        for (int u = 0; u < 4; ++u) v[u] = __shfl_sync(0xffffffffu, x, (u >> 1) * 16 + (u & 1) * 8);
    } else {
        x = (b4 ? v[1] : v[0]) + __shfl_xor_sync(0xffffffffu, b4 ? v[0] : v[1], 16);
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
#pragma unroll
        for (int u = 0; u < 2; ++u) v[u] = __shfl_sync(0xffffffffu, x, u * 16);
    }
}

// Rotates the pair (x0, x1) of dimension d of a head by the angle at pos.
__device__ __forceinline__ void attn_rope_pair(float &x0, float &x1, int d, int hd, int pos,
                                               double theta) {
    const double a = (double)pos * pow(theta, -(double)(2 * d) / (double)hd);
    double sn, cs;
    sincos(a, &sn, &cs);
    const double y0 = (double)x0 * cs - (double)x1 * sn;
    const double y1 = (double)x0 * sn + (double)x1 * cs;
    x0 = (float)y0;
    x1 = (float)y1;
}

template <int DPL>
__device__ __forceinline__ void attn_load_row(const float *p, float (&v)[DPL]) {
    if constexpr (DPL == 1) {
        v[0] = __ldcg(p);
    } else if constexpr (DPL == 2) {
        const float2 a = __ldcg(reinterpret_cast<const float2 *>(p));
        v[0] = a.x;
        v[1] = a.y;
    } else {
#pragma unroll
        for (int i = 0; i < DPL; i += 4) {
            const float4 a = __ldcg(reinterpret_cast<const float4 *>(p + i));
            v[i] = a.x;
            v[i + 1] = a.y;
            v[i + 2] = a.z;
            v[i + 3] = a.w;
        }
    }
}

// One item on the calling CTA's consumer threads (thread t of nthr = 256,
// 8 warps).  BAR synchronises exactly those threads.  smem: kAttnSmemBytes,
// 16-byte aligned.
// Not inlined: the persistent kernel's matvec loops keep their own register
// allocation.
template <int DPL, class BAR>
__device__ __noinline__ void attn_item(const AttnStep &a, int h, int c, int t, unsigned char *smem,
                                       BAR bar) {
    const int hd = a.hd, half = hd >> 1;
    const int group = a.n_head / a.n_kv, g = h / group;
    const int qr = a.n_head * hd, kvr = a.n_kv * hd;
    const int P = a.pos + 1;
    const int j0 = (int)((long long)c * P / a.S), j1 = (int)((long long)(c + 1) * P / a.S);
    float *q_s = reinterpret_cast<float *>(smem);
    float *k_s = q_s + kAttnMaxHd;
    double *m_s = reinterpret_cast<double *>(k_s + kAttnMaxHd);
    double *l_s = m_s + kAttnWarps;
    double *acc_s = l_s + kAttnWarps;                       // [kAttnWarps][hd]
    int *flag_s = reinterpret_cast<int *>(acc_s + kAttnWarps * kAttnMaxHd);
    const float *vcur = a.qkv + qr + kvr + (size_t)g * hd;
    // the designated item of each KV head stores this step's cache rows
    const bool writer = (h % group == 0) && c == a.S - 1;

    // ---- the warp's first batch of cached rows goes out first ----------------------
    // (the cache rows only; their latency overlaps the RoPE section below)
    const int w = t >> 5, lane = t & 31;
    const int d0 = lane * DPL;
    const float *kbase = a.k_cache + (size_t)g * hd + d0;
    const float *vbase = a.v_cache + (size_t)g * hd + d0;
    constexpr int U = DPL >= 8 ? 2 : 4;   // row loads in flight per lane: 2 * U * DPL / 4
    // Batch j: positions j + u * kAttnWarps, u < U.  Rows past the chunk are
    // zero (and masked); row pos is this token's, filled in from shared memory.
    float kv[U][DPL], vv[U][DPL];
    auto load_batch = [&](int j) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int jj = j + u * kAttnWarps;
            if (jj < j1 && jj != a.pos) {
                attn_load_row<DPL>(kbase + (size_t)jj * kvr, kv[u]);
                attn_load_row<DPL>(vbase + (size_t)jj * kvr, vv[u]);
            } else {
#pragma unroll
                for (int i = 0; i < DPL; ++i) kv[u][i] = vv[u][i] = 0.0f;
            }
        }
    };
    auto fill_pos = [&](int j) {
#pragma unroll
        for (int u = 0; u < U; ++u)
            if (j + u * kAttnWarps == a.pos) {
#pragma unroll
                for (int i = 0; i < DPL; ++i) {
                    kv[u][i] = k_s[d0 + i];
                    vv[u][i] = vcur[d0 + i];
                }
            }
    };
    if (j0 + w < j1) load_batch(j0 + w);

    // ---- rotated q of head h and k of KV head g ---------------------------------
    if (t < half) {
        float q0 = a.qkv[(size_t)h * hd + t], q1 = a.qkv[(size_t)h * hd + t + half];
        float k0 = a.qkv[qr + (size_t)g * hd + t], k1 = a.qkv[qr + (size_t)g * hd + t + half];
        attn_rope_pair(q0, q1, t, hd, a.pos, a.theta);
        attn_rope_pair(k0, k1, t, hd, a.pos, a.theta);
        q_s[t] = q0;
        q_s[t + half] = q1;
        k_s[t] = k0;
        k_s[t + half] = k1;
        if (writer) {
            float *kr = a.k_cache + (size_t)a.pos * kvr + (size_t)g * hd;
            kr[t] = k0;
            kr[t + half] = k1;
        }
    }
    if (writer && t < hd) a.v_cache[(size_t)a.pos * kvr + (size_t)g * hd + t] = vcur[t];
    bar();

    // ---- per warp: online softmax over positions j0 + w + 8i ----------------------
    double qd[DPL], acc[DPL];
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
        qd[i] = (double)q_s[d0 + i];
        acc[i] = 0.0;
    }
    const double scale = 1.0 / sqrt((double)hd);
    double m = -INFINITY, l = 0.0;
    for (int j = j0 + w; j < j1; j += U * kAttnWarps) {
        if (j != j0 + w) load_batch(j);
        fill_pos(j);
        double s[U];
        double mx = m;
#pragma unroll
        for (int u = 0; u < U; ++u) {
            double dot = 0.0;
#pragma unroll
            for (int i = 0; i < DPL; ++i) dot = fma(qd[i], (double)kv[u][i], dot);
            s[u] = dot;
        }
        attn_warp_sums<U>(s, lane);
#pragma unroll
        for (int u = 0; u < U; ++u) {
            s[u] = (j + u * kAttnWarps < j1) ? s[u] * scale : -INFINITY;
            mx = fmax(mx, s[u]);
        }
        const double corr = exp(m - mx);   // m = -inf on the first batch: 0
        l *= corr;
#pragma unroll
        for (int i = 0; i < DPL; ++i) acc[i] *= corr;
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const double p = exp(s[u] - mx);   // 0 for positions past the chunk
            l += p;
#pragma unroll
            for (int i = 0; i < DPL; ++i) acc[i] = fma(p, (double)vv[u][i], acc[i]);
        }
        m = mx;
    }
    if (lane == 0) {
        m_s[w] = m;
        l_s[w] = l;
    }
#pragma unroll
    for (int i = 0; i < DPL; ++i) acc_s[w * kAttnMaxHd + d0 + i] = acc[i];
    bar();

    // ---- merge the warps in order ------------------------------------------------------
    double M = -INFINITY;
#pragma unroll
    for (int ww = 0; ww < kAttnWarps; ++ww) M = fmax(M, m_s[ww]);
    double L = 0.0, A = 0.0;
#pragma unroll
    for (int ww = 0; ww < kAttnWarps; ++ww) {
        const double f = exp(m_s[ww] - M);   // warps without positions: exp(-inf) = 0
        L += l_s[ww] * f;
        if (t < hd) A += acc_s[ww * kAttnMaxHd + t] * f;
    }
    if (a.S == 1) {
        if (t < hd) a.out[(size_t)h * hd + t] = (float)(A * (1.0 / (L + 1e-12)));
        bar();   // the shared state is free for the next item
        return;
    }
    double *pp = a.part + ((size_t)h * a.S + c) * (hd + 2);
    if (t == 0) {
        pp[0] = M;
        pp[1] = L;
    }
    if (t < hd) pp[2 + t] = A;
    __threadfence();
    bar();
    if (t == 0) flag_s[0] = atomicAdd(a.cnt + h, 1u) == (unsigned)(a.S - 1);
    bar();
    if (flag_s[0]) {
        // the last chunk of head h to finish merges all S in chunk order.
        // The S partials come into shared memory first, every load of a
        // thread in flight at once (one memory round trip on the phase's
        // critical path instead of one per dependent load); they take the
        // place of the warps' states (m_s, l_s, acc_s: S (hd + 2) <= 8 x 258
        // doubles, exactly that area), which every thread has finished
        // reading at the barriers above.
        __threadfence();
        const double *ph = a.part + (size_t)h * a.S * (hd + 2);
        double *ps = m_s;
        const int np = a.S * (hd + 2);
        constexpr int kNT = 32 * kAttnWarps;
        for (int i0 = t; i0 < np; i0 += 4 * kNT) {
            double v[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) v[k] = i0 + k * kNT < np ? __ldcg(ph + i0 + k * kNT) : 0.0;
#pragma unroll
            for (int k = 0; k < 4; ++k)
                if (i0 + k * kNT < np) ps[i0 + k * kNT] = v[k];
        }
        bar();
        double MM = -INFINITY;
        for (int cc = 0; cc < a.S; ++cc) MM = fmax(MM, ps[cc * (hd + 2)]);
        double LL = 0.0, AA = 0.0;
        for (int cc = 0; cc < a.S; ++cc) {
            const double f = exp(ps[cc * (hd + 2)] - MM);
            LL += ps[cc * (hd + 2) + 1] * f;
            if (t < hd) AA += ps[cc * (hd + 2) + 2 + t] * f;
        }
        if (t < hd) a.out[(size_t)h * hd + t] = (float)(AA * (1.0 / (LL + 1e-12)));
        if (t == 0) atomicExch(a.cnt + h, 0u);
    }
    bar();
}

// Items are numbered h * S + c; the caller's CTA cb of G takes items cb,
// cb + G, ...
template <class BAR>
__device__ void attn_items(const AttnStep &a, int cb, int G, int t, unsigned char *smem, BAR bar) {
    const int n = a.n_head * a.S;
    for (int it = cb; it < n; it += G) {
        const int h = it / a.S, c = it % a.S;
        switch (a.hd >> 5) {
            case 1: attn_item<1>(a, h, c, t, smem, bar); break;
            case 2: attn_item<2>(a, h, c, t, smem, bar); break;
            case 4: attn_item<4>(a, h, c, t, smem, bar); break;
            default: attn_item<8>(a, h, c, t, smem, bar); break;
        }
    }
}

}  // namespace lalb
