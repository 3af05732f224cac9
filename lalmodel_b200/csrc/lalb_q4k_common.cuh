// lalb_q4k_common.cuh -- device building blocks shared by the Q4_K matvec
// kernels: the exact half-block dot product, the activation quantizers and
// the warp reductions.
#pragma once

#include "lalb_internal.cuh"

namespace lalb {

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

// Quantizes one 32-block held by a quad of lanes (8 elements each, quad
// lane qi owns elements 8qi..8qi+7).  Same operations as the restatement.
__device__ __forceinline__ void quantize_block_quad(const float (&v)[8], int qi, bool store,
                                                    int8_t *xq32, float *sx, int *sumq) {
    uint32_t amax = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = max(amax, __float_as_uint(fabsf(v[i])));
    amax = max(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = max(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const float dsc = __fdiv_rn(__uint_as_float(amax), 127.0f);
    const float id = dsc != 0.0f ? __fdiv_rn(1.0f, dsc) : 0.0f;
    int s = 0;
    uint32_t packed[2];
#pragma unroll
    for (int w = 0; w < 2; ++w) {
        uint32_t word = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float t = roundf(__fmul_rn(v[4 * w + i], id));
            const int q = t > 127.0f ? 127 : (t < -127.0f ? -127 : (int)t);
            s += q;
            word |= ((uint32_t)q & 0xFFu) << (8 * i);
        }
        packed[w] = word;
    }
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    if (!store) return;
    *reinterpret_cast<uint2 *>(xq32 + 8 * qi) = make_uint2(packed[0], packed[1]);
    if (qi == 0) {
        *sx = dsc;
        *sumq = s;
    }
}

// Shared-memory layout of a quantized activation read back per 128-element
// half-block (one lane's 8 x 16-byte loads): 16-byte chunk q of half-block c
// is stored at chunk q ^ (c & 7) of that half-block, so that the lanes of a
// 128-bit load phase (consecutive c) hit distinct banks.
__device__ __forceinline__ int xq_swz_chunk(int c, int q) { return (c << 3) | (q ^ (c & 7)); }

// quantize_block_quad writing block blk of the swizzled layout at xq_s.
__device__ __forceinline__ void quantize_block_quad_swz(const float (&v)[8], int qi, bool store,
                                                        int8_t *xq_s, int blk, float *sx, int *sumq) {
    // this thread's 8 bytes: byte 8*qi of block blk = half-block blk/4, chunk
    // 2*(blk%4) + qi/2, offset 8*(qi%2); quantize_block_quad adds 8*qi itself
    int8_t *dst = xq_s + 16 * xq_swz_chunk(blk >> 2, 2 * (blk & 3) + (qi >> 1)) + 8 * (qi & 1) - 8 * qi;
    quantize_block_quad(v, qi, store, dst, sx, sumq);
}

__device__ __forceinline__ void load8(const float *x, bool vec, float (&v)[8]) {
    if (vec) {
        const float4 a = reinterpret_cast<const float4 *>(x)[0];
        const float4 b = reinterpret_cast<const float4 *>(x)[1];
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = x[i];
    }
}

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

// Sums v[0..3] (one value per row) over the 32 lanes.  On return lane L holds
// the total of row ((L >> 4) & 1) * 2 + ((L >> 3) & 1).
__device__ __forceinline__ double warp_sum_rows4(const double (&v)[4], int lane) {
    const bool hi16 = lane & 16;
    const double send0 = hi16 ? v[0] : v[2], send1 = hi16 ? v[1] : v[3];
    const double keep0 = hi16 ? v[2] : v[0], keep1 = hi16 ? v[3] : v[1];
    const double w0 = keep0 + __shfl_xor_sync(0xffffffffu, send0, 16);
    const double w1 = keep1 + __shfl_xor_sync(0xffffffffu, send1, 16);
    const bool hi8 = lane & 8;
    double u = (hi8 ? w1 : w0) + __shfl_xor_sync(0xffffffffu, hi8 ? w0 : w1, 8);
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) u += __shfl_xor_sync(0xffffffffu, u, o);
    return u;
}


__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace lalb
