// kq_imma.cuh -- one-row decode on the integer tensor cores (mma.sync
// m16n8k32, u8 weights x s8 activations, s32 accumulate).
//
// The activation row is quantized once to int16 per 32 values (scale
// dx = max|x| / 32512) and split EXACTLY into two signed bytes,
// q = 256 * hi + lo (hi = (q + 128) >> 8 in [-127, 127], lo in [-128, 127]).
// lo and hi are two columns of the MMA's B operand, so one MMA gives, per
// weight row, D_lo and D_hi with 256 * D_hi + D_lo = sum(q_w * q_x) exactly:
// the same integer dot as a 16-bit multiply, at 512 weights per instruction.
// Weights stay in their wire form: 4-bit (Q4_K) or 6-bit (Q6_K) unsigned
// values become u8 A fragments with a mask or two, and each sub-block's
// scale is applied to its int32 result in f32.
//
// Activation block layout (640 bytes per 256 values), written by
// imma_quantize and read by the B-fragment loads:
//   bytes [64 j, 64 j + 64): sub-block j (32 values) as [g = lo/hi][tq][8 B]
//     where the 8 bytes are values 4tq..4tq+3 and 16+4tq..16+4tq+3
//     (exactly the b0 / b1 registers of thread (g, tq) of an m16n8k32 B
//     fragment whose column g is this sub-block's lo or hi bytes);
//   floats at byte 512: [0..7] dx_j, [8..15] dx_j * sum_j(q),
//     [16..31] dx * sum(q) over each 16 values.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "kq_formats.cuh"

namespace kq {
namespace {

constexpr int IMMA_XB = 640;  // activation bytes per 256-value block

__device__ __forceinline__ void imma16832(int d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
}

// One warp quantizes one 256-value activation block (8 values per lane in
// `v`, values 8*lane .. 8*lane+7) into the layout above.
template <bool F16>
__device__ __forceinline__ void imma_quantize(const uint4 v, uint8_t *xb) {
    const int lane = threadIdx.x & 31, j = lane >> 2, part = lane & 3;  // sub-block j, values 8*part.. of it
    const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
    float f[8];
#pragma unroll
    for (int e = 0; e < 4; e++) {
        if constexpr (F16) {
            const float2 h = __half22float2(*reinterpret_cast<const __half2 *>(&w4[e]));
            f[2 * e] = h.x;
            f[2 * e + 1] = h.y;
        } else {
            f[2 * e] = __uint_as_float(w4[e] << 16);
            f[2 * e + 1] = __uint_as_float(w4[e] & 0xffff0000u);
        }
    }
    float am = 0.f;
#pragma unroll
    for (int e = 0; e < 8; e++) am = fmaxf(am, fabsf(f[e]));
    am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
    am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
    const float dx = am * (1.0f / 32512.0f), inv = am > 0.f ? 32512.0f / am : 0.f;
    int qs = 0;
    uint32_t lo[2] = {0, 0}, hi[2] = {0, 0};
#pragma unroll
    for (int e = 0; e < 8; e++) {
        const int q = __float2int_rn(f[e] * inv);
        qs += q;
        const int h = (q + 128) >> 8, l = q - 256 * h;
        lo[e >> 2] |= (uint32_t)(l & 255) << (8 * (e & 3));
        hi[e >> 2] |= (uint32_t)(h & 255) << (8 * (e & 3));
    }
    // values 8*part + 4*u .. +3 form quad m = 2*part + u: thread tq = m & 3, word m >> 2
    uint32_t *sb = reinterpret_cast<uint32_t *>(xb + 64 * j);
#pragma unroll
    for (int u = 0; u < 2; u++) {
        const int m = 2 * part + u, tq = m & 3, wd = m >> 2;
        sb[(0 * 32 + tq * 8) / 4 + wd] = lo[u];
        sb[(1 * 32 + tq * 8) / 4 + wd] = hi[u];
    }
    const int q16 = qs + __shfl_xor_sync(0xffffffffu, qs, 1);
    const int q32 = q16 + __shfl_xor_sync(0xffffffffu, q16, 2);
    float *xf = reinterpret_cast<float *>(xb + 512);
    if (part == 0) {
        xf[j] = dx;
        xf[8 + j] = dx * (float)q32;
    }
    if ((part & 1) == 0) xf[16 + (lane >> 1)] = dx * (float)q16;
}

__device__ __forceinline__ uint32_t lds32(const uint8_t *p) { return *reinterpret_cast<const uint32_t *>(p); }
// 32 bits at a 2-byte aligned shared address (two aligned loads + funnel shift)
__device__ __forceinline__ uint32_t lds32_a2(const uint8_t *p) {
    const uintptr_t a = (uintptr_t)p;
    const uint32_t *q = reinterpret_cast<const uint32_t *>(a & ~(uintptr_t)3);
    return __funnelshift_r(q[0], q[1], (uint32_t)(a & 3) * 8);
}

// m16n8k32 MMA accumulating into c.
__device__ __forceinline__ void imma16832_acc(int c[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Column placement: the four sub-blocks of a group go to B column pairs
// (0,1), (2,3), (4,5), (6,7) -- lo bytes in the even column, hi bytes in the
// odd one -- and the group's MMAs chain into ONE accumulator.  A column pair
// is zero in every other MMA of the group, so thread (g, tq) ends with the
// lo / hi sums of sub-block tq of the group for rows g and g + 8: each lane
// applies the scales of one sub-block instead of all four lanes repeating
// the same work.  The caller adds the four lanes of a row (tq) at the end.

// Q4_K: 16 weight rows (thread rows g and g+8: blocks bg / bg8 in shared
// memory, 16-byte aligned) x one 256-value block; acc0 / acc1 gather this
// lane's share of rows g / g+8.
__device__ __forceinline__ void imma_q4k(const uint8_t *bg, const uint8_t *bg8, const uint8_t *xb, int g, int tq,
                                         float &acc0, float &acc1) {
    const float *xf = reinterpret_cast<const float *>(xb + 512);
    const int pair = g >> 1, gq = g & 1;  // this thread's B column pair and lo / hi byte column
    int d[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};  // group 0: sub-blocks 0-3, group 1: 4-7
#pragma unroll
    for (int c = 0; c < 4; c++) {
        const uint32_t wa = lds32(bg + 16 + 32 * c + 4 * tq), wb = lds32(bg + 32 + 32 * c + 4 * tq);
        const uint32_t va = lds32(bg8 + 16 + 32 * c + 4 * tq), vb = lds32(bg8 + 32 + 32 * c + 4 * tq);
#pragma unroll
        for (int hh = 0; hh < 2; hh++) {  // sub-block j = 2c (low nibbles) and 2c + 1 (high nibbles)
            const int j = 2 * c + hh;
            const uint32_t a[4] = {(wa >> (4 * hh)) & 0x0f0f0f0fu, (va >> (4 * hh)) & 0x0f0f0f0fu,
                                   (wb >> (4 * hh)) & 0x0f0f0f0fu, (vb >> (4 * hh)) & 0x0f0f0f0fu};
            uint2 bb = make_uint2(0u, 0u);
            if (pair == (j & 3)) bb = *reinterpret_cast<const uint2 *>(xb + 64 * j + 32 * gq + 8 * tq);
            imma16832_acc(d[j >> 2], a, bb.x, bb.y);
        }
    }
    // this lane's sub-blocks: j = tq (group 0) and 4 + tq (group 1)
    const uint4 h0 = *reinterpret_cast<const uint4 *>(bg), h1 = *reinterpret_cast<const uint4 *>(bg8);
    uint32_t sc03a, sc47a, m03a, m47a, sc03b, sc47b, m03b, m47b;
    q4k_unpack_scales(h0.y, h0.z, h0.w, sc03a, sc47a, m03a, m47a);
    q4k_unpack_scales(h1.y, h1.z, h1.w, sc03b, sc47b, m03b, m47b);
    const int sh = 8 * tq;
    float s0 = 0.f, s1 = 0.f, m0 = 0.f, m1 = 0.f;
#pragma unroll
    for (int grp = 0; grp < 2; grp++) {
        const int j = 4 * grp + tq;
        const float dxj = xf[j], sxj = xf[8 + j];
        const uint32_t sw0 = grp ? sc47a : sc03a, mw0 = grp ? m47a : m03a;
        const uint32_t sw1 = grp ? sc47b : sc03b, mw1 = grp ? m47b : m03b;
        s0 = fmaf((float)((sw0 >> sh) & 63u) * dxj, (float)(d[grp][1] * 256 + d[grp][0]), s0);
        s1 = fmaf((float)((sw1 >> sh) & 63u) * dxj, (float)(d[grp][3] * 256 + d[grp][2]), s1);
        m0 = fmaf((float)((mw0 >> sh) & 63u), sxj, m0);
        m1 = fmaf((float)((mw1 >> sh) & 63u), sxj, m1);
    }
    const float d0 = half_bits_to_float(h0.x & 0xffffu), dm0 = half_bits_to_float(h0.x >> 16);
    const float d1 = half_bits_to_float(h1.x & 0xffffu), dm1 = half_bits_to_float(h1.x >> 16);
    acc0 += fmaf(d0, s0, -dm0 * m0);
    acc1 += fmaf(d1, s1, -dm1 * m1);
}

// Q6_K: 16 weight rows x one 128-value half (hf) of a 256-value block
// (blocks bg / bg8, 2-byte aligned).  Each k32 MMA spans two 16-value
// sub-blocks (one per column pair); two MMAs (quarters qd, qd + 1) chain into
// one accumulator holding four sub-blocks, 16-value sub-block 8 hf + 2 qd0 + tq
// in lane tq.
__device__ __forceinline__ void imma_q6k(const uint8_t *bg, const uint8_t *bg8, int hf, const uint8_t *xb, int g,
                                         int tq, float &acc0, float &acc1) {
    const float *xf = reinterpret_cast<const float *>(xb + 512);
    const int mm = g >> 2, part = g & 3;  // B columns 4mm .. 4mm+3: (first 16 lo, hi), (second 16 lo, hi)
    // quarter qd of the half: values l = 0..31 of ql[64 hf + 32 (qd & 1) + l] nibble (qd >> 1)
    // and qh[32 hf + l] bits 2 qd.  Thread tq: a0/a1 = l 4tq..4tq+3 (rows g, g+8), a2/a3 = l 16+4tq..
    const uint32_t ha0 = lds32_a2(bg + 128 + 32 * hf + 4 * tq), hb0 = lds32_a2(bg + 128 + 32 * hf + 16 + 4 * tq);
    const uint32_t ha1 = lds32_a2(bg8 + 128 + 32 * hf + 4 * tq), hb1 = lds32_a2(bg8 + 128 + 32 * hf + 16 + 4 * tq);
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int q2 = 0; q2 < 2; q2++) {  // quarters 2 q2, 2 q2 + 1
        int d[4] = {0, 0, 0, 0};
#pragma unroll
        for (int m = 0; m < 2; m++) {
            const int qd = 2 * q2 + m;
            const int qo = 64 * hf + 32 * (qd & 1), ns = 4 * (qd >> 1), hs = 2 * qd;
            const uint32_t la0 = lds32_a2(bg + qo + 4 * tq), lb0 = lds32_a2(bg + qo + 16 + 4 * tq);
            const uint32_t la1 = lds32_a2(bg8 + qo + 4 * tq), lb1 = lds32_a2(bg8 + qo + 16 + 4 * tq);
            const uint32_t a[4] = {((la0 >> ns) & 0x0f0f0f0fu) | (((ha0 >> hs) & 0x03030303u) << 4),
                                   ((la1 >> ns) & 0x0f0f0f0fu) | (((ha1 >> hs) & 0x03030303u) << 4),
                                   ((lb0 >> ns) & 0x0f0f0f0fu) | (((hb0 >> hs) & 0x03030303u) << 4),
                                   ((lb1 >> ns) & 0x0f0f0f0fu) | (((hb1 >> hs) & 0x03030303u) << 4)};
            const int j = 4 * hf + qd;  // 32-value activation sub-block
            uint32_t b0 = 0u, b1 = 0u;
            if (mm == m) {
                const uint2 bb = *reinterpret_cast<const uint2 *>(xb + 64 * j + 32 * (part & 1) + 8 * tq);
                b0 = part < 2 ? bb.x : 0u;   // columns 4m, 4m+1: the first 16 values
                b1 = part >= 2 ? bb.y : 0u;  // columns 4m+2, 4m+3: the second 16
            }
            imma16832_acc(d, a, b0, b1);
        }
        // lane tq: 16-value sub-block s = 2 (4 hf + 2 q2) + tq, of 32-value sub-block j = 4 hf + 2 q2 + (tq >> 1)
        const int j = 4 * hf + 2 * q2 + (tq >> 1), s = 2 * j + (tq & 1);
        const float sc0 = (float)(int8_t)bg[192 + s], sc1 = (float)(int8_t)bg8[192 + s];
        const float dxj = xf[j], sx16 = xf[16 + s];
        s0 = fmaf(sc0, fmaf(dxj, (float)(d[1] * 256 + d[0]), -32.f * sx16), s0);
        s1 = fmaf(sc1, fmaf(dxj, (float)(d[3] * 256 + d[2]), -32.f * sx16), s1);
    }
    acc0 = fmaf(half_bits_to_float(lds32_a2(bg + 208) & 0xffffu), s0, acc0);
    acc1 = fmaf(half_bits_to_float(lds32_a2(bg8 + 208) & 0xffffu), s1, acc1);
}

}  // namespace
}  // namespace kq
