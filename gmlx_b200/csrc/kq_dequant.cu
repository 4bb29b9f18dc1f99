// kq_dequant.cu -- block dequantization (the kq.dequantize op).
//
// Replaces mlx-kquant's dequantize as called from gmlx/modules.py:1461,
// gmlx/loader.py:3046-3048 and gmlx/dsv32_patches.py:229.  f32 output is
// bit-identical to gguf-py's dequantize (see kq_formats.cuh for why any
// evaluation order gives the same bits); f16/bf16 outputs are the f32 value
// rounded to nearest even.
//
// Memory-bound: each warp owns one super-block, each lane 8 consecutive
// weights (one 32-byte f32 store or one 16-byte f16/bf16 store).
#include <algorithm>

#include "kq_internal.cuh"
#include "kq_ptx.cuh"

namespace kq {

template <int C>
__device__ __forceinline__ void deq8(const uint8_t *b, int lane, float o[8]) {
    if constexpr (C == Q4_K) {
        const int j = lane >> 2, i0 = 8 * (lane & 3), c = j >> 1, h = j & 1;
        const float d = half_bits_to_float(ld_u16(b));
        const float dmin = half_bits_to_float(ld_u16(b + 2));
        const uint32_t s0 = ld_u32_unaligned(b + 4), s1 = ld_u32_unaligned(b + 8), s2 = ld_u32_unaligned(b + 12);
        uint32_t sc03, sc47, m03, m47;
        q4k_unpack_scales(s0, s1, s2, sc03, sc47, m03, m47);
        const uint32_t scw = j < 4 ? sc03 : sc47, mw = j < 4 ? m03 : m47;
        const float dl = d * byte_f(scw, j & 3), ml = dmin * byte_f(mw, j & 3);
        const uint8_t *q = b + 16 + 32 * c + i0;
#pragma unroll
        for (int i = 0; i < 8; i++) o[i] = dl * (float)((q[i] >> (4 * h)) & 15) - ml;
    } else if constexpr (C == Q5_K) {  // Q4_K layout + 32 bytes of fifth bits (bit j of qh[l]: sub-block j)
        const int j = lane >> 2, i0 = 8 * (lane & 3), c = j >> 1, h = j & 1;
        const float d = half_bits_to_float(ld_u16(b));
        const float dmin = half_bits_to_float(ld_u16(b + 2));
        const uint32_t s0 = ld_u32_unaligned(b + 4), s1 = ld_u32_unaligned(b + 8), s2 = ld_u32_unaligned(b + 12);
        uint32_t sc03, sc47, m03, m47;
        q4k_unpack_scales(s0, s1, s2, sc03, sc47, m03, m47);
        const uint32_t scw = j < 4 ? sc03 : sc47, mw = j < 4 ? m03 : m47;
        const float dl = d * byte_f(scw, j & 3), ml = dmin * byte_f(mw, j & 3);
        const uint8_t *q = b + 48 + 32 * c + i0, *qh = b + 16 + i0;
#pragma unroll
        for (int i = 0; i < 8; i++)
            o[i] = dl * (float)(((q[i] >> (4 * h)) & 15) | (((qh[i] >> j) & 1) << 4)) - ml;
    } else if constexpr (C == IQ2_XS || C == IQ2_S) {  // lane: grid entry lane (8 weights)
        const int e = lane;
        const float d = half_bits_to_float(ld_u16(b));
        uint32_t sg;
        uint64_t g;
        int s;
        if constexpr (C == IQ2_XS) {
            const uint32_t v = ld_u16(b + 2 + 2 * e);
            sg = ksigns(v >> 9);
            g = c_iq2xs_grid[v & 511];
            s = (b[66 + (e >> 2)] >> (4 * ((e >> 1) & 1))) & 15;
        } else {
            const uint32_t idx = b[2 + e] | (((b[66 + (e >> 2)] >> (2 * (e & 3))) & 3u) << 8);
            sg = b[34 + e];
            g = c_iq2s_grid[idx];
            s = (b[74 + (e >> 2)] >> (4 * ((e >> 1) & 1))) & 15;
        }
        const float db = d * (0.5f + (float)s) * 0.25f;
#pragma unroll
        for (int i = 0; i < 8; i++) o[i] = db * (float)((g >> (8 * i)) & 255u) * (((sg >> i) & 1u) ? -1.0f : 1.0f);
    } else if constexpr (C == IQ1_S || C == IQ1_M) {  // lane: grid entry lane (8 weights)
        const int e = lane;
        float dl, delta;
        uint32_t idx;
        if constexpr (C == IQ1_S) {
            const uint32_t qh = ld_u16(b + 34 + 2 * (e >> 2));
            dl = half_bits_to_float(ld_u16(b)) * (float)(2 * ((qh >> 12) & 7) + 1);
            delta = (qh & 0x8000u) ? -0.125f : 0.125f;
            idx = b[2 + e] | (((qh >> (3 * (e & 3))) & 7u) << 8);
        } else {
            const uint32_t s0 = ld_u16(b + 48), s1 = ld_u16(b + 50), s2 = ld_u16(b + 52), s3 = ld_u16(b + 54);
            const float d = half_bits_to_float((s0 >> 12) | ((s1 >> 8) & 0xf0u) | ((s2 >> 4) & 0xf00u) | (s3 & 0xf000u));
            const int k = e >> 1;
            const uint32_t sk = ld_u16(b + 48 + 2 * (k >> 2));
            dl = d * (float)(2 * ((sk >> (3 * (k & 3))) & 7) + 1);
            const uint32_t nib = (b[32 + (e >> 1)] >> (4 * (e & 1))) & 15u;
            delta = (nib & 8u) ? -0.125f : 0.125f;
            idx = b[e] | ((nib & 7u) << 8);
        }
        const uint64_t g = c_iq1s_grid[idx];
#pragma unroll
        for (int i = 0; i < 8; i++) o[i] = dl * ((float)(int8_t)((g >> (8 * i)) & 255u) + delta);
    } else if constexpr (C == IQ3_S) {  // lane: grid entries 2 lane, 2 lane + 1 (8 weights)
        const float d = half_bits_to_float(ld_u16(b));
        const int s = (b[106 + (lane >> 3)] >> (4 * ((lane >> 2) & 1))) & 15;
        const float db = d * (float)(1 + 2 * s);
        const uint32_t sg = b[74 + lane];
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int e = 2 * lane + h;
            const uint32_t g = c_iq3s_grid[b[2 + e] | (((b[66 + (e >> 3)] >> (e & 7)) & 1u) << 8)];
#pragma unroll
            for (int i = 0; i < 4; i++)
                o[4 * h + i] = db * (float)((g >> (8 * i)) & 255u) * (((sg >> (4 * h + i)) & 1u) ? -1.0f : 1.0f);
        }
    } else if constexpr (C == NVFP4) {  // lane: weights 8 lane .. +7 (one nibble half of 8 bytes)
        const uint8_t *blk = b + 36 * (lane >> 3);
        const int j = (lane >> 1) & 3, h = lane & 1;
        const float d = ue4m3_half(blk[j]);
        const uint8_t *q = blk + 4 + 8 * j;
#pragma unroll
        for (int i = 0; i < 8; i++) o[i] = d * (float)c_mxfp4_values[(q[i] >> (4 * h)) & 15];
    } else if constexpr (C == TQ1_0) {  // lane: weights 8 lane .. +7 (one digit position of 8 bytes)
        const int w0 = 8 * lane;
        const uint8_t *src;
        uint32_t pw;
        if (w0 < 160) {
            src = b + (w0 & 31);
            pw = 1u;
            for (int k = 0; k < (w0 >> 5); k++) pw *= 3u;
        } else if (w0 < 240) {
            src = b + 32 + ((w0 - 160) & 15);
            pw = 1u;
            for (int k = 0; k < ((w0 - 160) >> 4); k++) pw *= 3u;
        } else {  // weights 240 + 4k + l: two digit positions of the last 4 bytes
            src = nullptr;
            pw = 0u;
        }
        const float d = half_bits_to_float(ld_u16(b + 52));
#pragma unroll
        for (int i = 0; i < 8; i++) {
            uint32_t v, p;
            if (src) {
                v = src[i];
                p = pw;
            } else {
                const int w = w0 + i - 240;
                v = b[48 + (w & 3)];
                p = 1u;
                for (int k = 0; k < (w >> 2); k++) p *= 3u;
            }
            const int t = (int)((((v * p) & 255u) * 3u) >> 8);
            o[i] = d * (float)(t - 1);
        }
    } else if constexpr (C == TQ2_0) {  // lane: weights 8 lane .. +7
        const int w0 = 8 * lane, h = w0 >> 7, k = (w0 >> 5) & 3, l0 = w0 & 31;
        const float d = half_bits_to_float(ld_u16(b + 64));
#pragma unroll
        for (int i = 0; i < 8; i++) o[i] = d * (float)(((b[32 * h + l0 + i] >> (2 * k)) & 3) - 1);
    } else if constexpr (C == Q2_K || C == Q3_K) {  // lane: weights 8 lane .. +7 (one 16-weight sub-block)
        const int w0 = 8 * lane, h = w0 >> 7, k = (w0 >> 5) & 3, l0 = w0 & 31, j = w0 >> 4;
        float dl, ml = 0.f;
        const uint8_t *qs = b + (C == Q2_K ? 16 : 32) + 32 * h + l0;
        if constexpr (C == Q2_K) {
            dl = half_bits_to_float(ld_u16(b + 80)) * (float)(b[j] & 15);
            ml = half_bits_to_float(ld_u16(b + 82)) * (float)(b[j] >> 4);
        } else {
            const int lo = j < 8 ? (b[96 + j] & 15) : (b[88 + j] >> 4);
            const int hi = (b[104 + (j & 3)] >> (2 * (j >> 2))) & 3;
            dl = half_bits_to_float(ld_u16(b + 108)) * (float)((lo | (hi << 4)) - 32);
        }
#pragma unroll
        for (int i = 0; i < 8; i++) {
            int q = (qs[i] >> (2 * k)) & 3;
            if constexpr (C == Q3_K) q -= ((b[l0 + i] >> (4 * h + k)) & 1) ? 0 : 4;
            o[i] = C == Q2_K ? dl * (float)q - ml : dl * (float)q;
        }
    } else if constexpr (Legacy<C>::IS) {  // lane: 8 weights of ggml block lane / 4
        using LG = Legacy<C>;
        const uint8_t *blk = b + LG::BB * (lane >> 2);
        const float d = LG::MX ? e8m0_half(blk[0]) : half_bits_to_float(ld_u16(blk));
        const float m = LG::HASM ? half_bits_to_float(ld_u16(blk + 2)) : 0.f;
        const uint32_t qh = LG::HASH ? ld_u32_unaligned(blk + LG::HOFF) : 0u;
        const int i0 = 8 * (lane & 3), h = i0 >> 4;
        const uint8_t *q = blk + LG::QOFF + (i0 & 15);
#pragma unroll
        for (int i = 0; i < 8; i++) {
            int v = (q[i] >> (4 * h)) & 15;
            if constexpr (LG::HASH) v |= (int)((qh >> (i0 + i)) & 1u) << 4;
            if constexpr (LG::MX) o[i] = d * (float)c_mxfp4_values[v];
            else if constexpr (LG::NL) o[i] = d * (float)c_iq4nl_values[v];
            else if constexpr (LG::HASM) o[i] = __fadd_rn(__fmul_rn(d, (float)v), m);  // gguf order: d*q + m
            else o[i] = d * (float)(v - LG::OFF);
        }
    } else if constexpr (C == Q8_0) {  // lane: 8 weights of ggml block lane / 4
        const uint8_t *blk = b + 34 * (lane >> 2);
        const float d = half_bits_to_float(ld_u16(blk));
        const uint8_t *q = blk + 2 + 8 * (lane & 3);
#pragma unroll
        for (int i = 0; i < 8; i++) o[i] = (float)(int8_t)q[i] * d;
    } else if constexpr (C == Q6_K) {
        const int i0 = 8 * lane, hf = i0 >> 7, s = (i0 & 127) >> 5, lo = i0 & 31;
        const float d = half_bits_to_float(ld_u16(b + 208));
        const float dl = d * (float)(int8_t)b[192 + (i0 >> 4)];
        const uint8_t *ql = b + 64 * hf + 32 * (s & 1) + lo, *qh = b + 128 + 32 * hf + lo;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int q = (((ql[i] >> (4 * (s >> 1))) & 15) | (((qh[i] >> (2 * s)) & 3) << 4)) - 32;
            o[i] = dl * (float)q;
        }
    } else if constexpr (C == IQ3_XXS) {  // lane: sign group lane & 3 of sub-block lane >> 2
        const int j = lane >> 2, l = lane & 3;
        const float d = half_bits_to_float(ld_u16(b));
        const uint32_t aux = ld_u32_unaligned(b + 66 + 4 * j);
        const float db = d * (0.5f + (float)(aux >> 28)) * 0.5f;
        const uint32_t sg = ksigns((aux >> (7 * l)) & 127u);
        const uint32_t e0 = c_iq3xxs_grid[b[2 + 8 * j + 2 * l]], e1 = c_iq3xxs_grid[b[3 + 8 * j + 2 * l]];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const float gv = (float)(((i < 4 ? e0 : e1) >> (8 * (i & 3))) & 255u);
            o[i] = db * gv * (((sg >> i) & 1u) ? -1.0f : 1.0f);
        }
    } else if constexpr (C == IQ4_XS) {  // lane: weights 8 (lane & 3) .. +7 of sub-block lane >> 2
        const int j = lane >> 2, i0 = 8 * (lane & 3), h = i0 >> 4;
        const float d = half_bits_to_float(ld_u16(b));
        const int ls = ((b[4 + (j >> 1)] >> (4 * (j & 1))) & 15) | (((ld_u16(b + 2) >> (2 * j)) & 3) << 4);
        const float dl = d * (float)(ls - 32);
        const uint8_t *q = b + 8 + 16 * j + (i0 & 15);
#pragma unroll
        for (int i = 0; i < 8; i++) o[i] = dl * (float)c_iq4nl_values[(q[i] >> (4 * h)) & 15];
    } else {
        const int g = lane >> 2, s = lane & 3;
        const float d = half_bits_to_float(ld_u16(b));
        const uint32_t a0 = ld_u32_unaligned(b + 2 + 8 * g), a1 = ld_u32_unaligned(b + 6 + 8 * g);
        const float db = d * (0.5f + (float)(a1 >> 28)) * 0.25f;
        const uint32_t sg = ksigns((a1 >> (7 * s)) & 127u);
        const uint64_t e = c_iq2xxs_grid[(a0 >> (8 * s)) & 255u];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const float gv = (float)((e >> (8 * i)) & 255u);
            o[i] = db * gv * (((sg >> i) & 1u) ? -1.0f : 1.0f);
        }
    }
}

template <int C, int OUT>
__global__ void __launch_bounds__(256) dequant_kernel(const uint8_t *__restrict__ w, int64_t rows, int64_t nb,
                                                      int64_t row_stride, void *__restrict__ out, int64_t out_k,
                                                      int tail) {
    // nb groups per row, then (tail > 0) a partial last group of `tail`
    // weights: its lanes past the tail read and write nothing
    const int lane = threadIdx.x & 31;
    const int64_t gpr = nb + (tail > 0);
    const int64_t blk = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (blk >= rows * gpr) return;
    const int64_t r = blk / gpr, b = blk - r * gpr;
    if (b == nb && 8 * lane >= tail) return;
    float o[8];
    deq8<C>(w + r * row_stride + b * Fmt<C>::bpb, lane, o);
    const int64_t e0 = r * out_k + b * QK + 8 * lane;
    if constexpr (OUT == F32) {
        float4 *p = reinterpret_cast<float4 *>(reinterpret_cast<float *>(out) + e0);
        p[0] = make_float4(o[0], o[1], o[2], o[3]);
        p[1] = make_float4(o[4], o[5], o[6], o[7]);
    } else if constexpr (OUT == BF16) {
        uint4 v;
        uint32_t *u = reinterpret_cast<uint32_t *>(&v);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            __nv_bfloat162 h = __floats2bfloat162_rn(o[2 * i], o[2 * i + 1]);
            u[i] = *reinterpret_cast<uint32_t *>(&h);
        }
        *reinterpret_cast<uint4 *>(reinterpret_cast<__nv_bfloat16 *>(out) + e0) = v;
    } else {
        uint4 v;
        uint32_t *u = reinterpret_cast<uint32_t *>(&v);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            __half2 h = __floats2half2_rn(o[2 * i], o[2 * i + 1]);
            u[i] = *reinterpret_cast<uint32_t *>(&h);
        }
        *reinterpret_cast<uint4 *>(reinterpret_cast<__half *>(out) + e0) = v;
    }
}

// Contiguous rows (row stride == row bytes): the raw blocks form one byte range.
// A persistent CTA bulk-copies chunks of DQ_CHUNK blocks into a two-slot shared
// ring (one 1-D cp.async.bulk per chunk, mbarrier completion) and its 8 warps
// decode them from shared memory, so ~2 chunks per CTA are in flight instead of
// one block per warp.  Waits are bounded (~2 s; on expiry the CTA stops).
constexpr int DQ_CHUNK = 128;

__device__ __forceinline__ uint64_t dq_timer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

template <int C, int OUT>
__device__ __forceinline__ void store8(void *out, int64_t e0, const float o[8]) {
    if constexpr (OUT == F32) {
        float4 *p = reinterpret_cast<float4 *>(reinterpret_cast<float *>(out) + e0);
        p[0] = make_float4(o[0], o[1], o[2], o[3]);
        p[1] = make_float4(o[4], o[5], o[6], o[7]);
    } else {
        uint4 v;
        uint32_t *u = reinterpret_cast<uint32_t *>(&v);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            if constexpr (OUT == BF16) {
                __nv_bfloat162 h = __floats2bfloat162_rn(o[2 * i], o[2 * i + 1]);
                u[i] = *reinterpret_cast<uint32_t *>(&h);
            } else {
                __half2 h = __floats2half2_rn(o[2 * i], o[2 * i + 1]);
                u[i] = *reinterpret_cast<uint32_t *>(&h);
            }
        }
        *reinterpret_cast<uint4 *>(reinterpret_cast<uint16_t *>(out) + e0) = v;
    }
}

template <int C, int OUT>
__global__ void __launch_bounds__(256) dequant_bulk_kernel(const uint8_t *__restrict__ w, int64_t nblk,
                                                           void *__restrict__ out) {
    constexpr int bpb = Fmt<C>::bpb, CB = DQ_CHUNK * bpb + 16;
    extern __shared__ __align__(128) uint8_t sm[];
    uint64_t *bar = reinterpret_cast<uint64_t *>(sm);
    uint8_t *buf = sm + 128;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t nchunks = (nblk + DQ_CHUNK - 1) / DQ_CHUNK;
    if (threadIdx.x == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        fence_mbar_init();
    }
    __syncthreads();
    auto issue = [&](int64_t c, int slot) {  // thread 0: chunk c -> slot
        const int64_t b0 = c * DQ_CHUNK, nb = min((int64_t)DQ_CHUNK, nblk - b0);
        const uintptr_t src = (uintptr_t)(w + b0 * bpb);
        const uint32_t off = (uint32_t)(src & 15);
        const uint32_t bytes = (off + (uint32_t)nb * bpb + 15) & ~15u;
        mbar_arrive_expect_tx(&bar[slot], bytes);
        bulk_g2s(buf + slot * CB, (const void *)(src - off), bytes, &bar[slot], policy_evict_first());
    };
    int64_t c = blockIdx.x;
    int iss[2] = {0, 0};  // copies issued into each slot (thread 0)
    if (threadIdx.x == 0 && c < nchunks) {
        issue(c, 0);
        iss[0]++;
    }
    for (uint32_t it = 0; c < nchunks; c += gridDim.x, it++) {
        const int slot = it & 1;
        const int64_t cn = c + gridDim.x;
        if (threadIdx.x == 0 && cn < nchunks) {  // the other slot was freed by the last barrier
            issue(cn, slot ^ 1);
            iss[slot ^ 1]++;
        }
        // bounded wait for this chunk; the decision to go on is CTA-uniform
        bool ok = true;
        const uint64_t t0 = dq_timer();
        for (uint32_t i = 0; !mbar_try_wait(&bar[slot], (it >> 1) & 1); i++)
            if ((i & 1023) == 1023 && dq_timer() - t0 > 2000000000ull) {
                ok = false;
                break;
            }
        if (__syncthreads_or(!ok)) break;
        const int64_t b0 = c * DQ_CHUNK, nb = min((int64_t)DQ_CHUNK, nblk - b0);
        const uint8_t *base = buf + slot * CB + ((uintptr_t)(w + b0 * bpb) & 15);
        for (int b = warp; b < nb; b += 8) {
            float o[8];
            deq8<C>(base + b * bpb, lane, o);
            store8<C, OUT>(out, (b0 + b) * QK + 8 * lane, o);
        }
        __syncthreads();  // slot free before it is refilled
    }
    // after an early exit a copy may still be in flight: wait (bounded) for the
    // last one issued into each slot before the CTA's shared memory is released
    if (threadIdx.x == 0) {
        for (int sl = 0; sl < 2; sl++) {
            if (!iss[sl]) continue;
            const uint64_t t0 = dq_timer();
            while (!mbar_try_wait(&bar[sl], (uint32_t)(iss[sl] - 1) & 1u) && dq_timer() - t0 < 2000000000ull) {
            }
        }
    }
}

template <int C>
static cudaError_t launch_deq(const uint8_t *w, int64_t rows, int64_t nb, int64_t stride, void *out, int dtype,
                              cudaStream_t st, int64_t out_k, int tail) {
    const int64_t nblk = rows * nb;
    if (tail == 0 && stride == nb * Fmt<C>::bpb && nblk >= 8 * DQ_CHUNK) {
        constexpr int smem = 128 + 2 * (DQ_CHUNK * Fmt<C>::bpb + 16);
        const int nsm = num_sms();
        const int64_t nchunks = (nblk + DQ_CHUNK - 1) / DQ_CHUNK;
        const unsigned g = (unsigned)std::min<int64_t>(nchunks, (int64_t)nsm * 3);
        cudaError_t e;
        if (dtype == F32) {
            if ((e = cudaFuncSetAttribute(dequant_bulk_kernel<C, F32>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)))
                return e;
            dequant_bulk_kernel<C, F32><<<g, 256, smem, st>>>(w, nblk, out);
        } else if (dtype == BF16) {
            if ((e = cudaFuncSetAttribute(dequant_bulk_kernel<C, BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)))
                return e;
            dequant_bulk_kernel<C, BF16><<<g, 256, smem, st>>>(w, nblk, out);
        } else {
            if ((e = cudaFuncSetAttribute(dequant_bulk_kernel<C, F16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)))
                return e;
            dequant_bulk_kernel<C, F16><<<g, 256, smem, st>>>(w, nblk, out);
        }
        return cudaGetLastError();
    }
    const unsigned grid = (unsigned)((rows * (nb + (tail > 0)) + 7) / 8);
    if (dtype == F32) dequant_kernel<C, F32><<<grid, 256, 0, st>>>(w, rows, nb, stride, out, out_k, tail);
    else if (dtype == BF16) dequant_kernel<C, BF16><<<grid, 256, 0, st>>>(w, rows, nb, stride, out, out_k, tail);
    else dequant_kernel<C, F16><<<grid, 256, 0, st>>>(w, rows, nb, stride, out, out_k, tail);
    return cudaGetLastError();
}

cudaError_t launch_dequantize(int codec, const uint8_t *w, int64_t rows, int64_t k, int64_t row_stride, void *out,
                              int dtype, cudaStream_t st) {
    // whole 256-weight groups, then a partial last group (32/64-weight codecs)
    const int64_t nb = k / QK;
    const int tail = (int)(k % QK);
    if (rows == 0 || k == 0) return cudaSuccess;
    switch (codec) {
    case Q4_K: return launch_deq<Q4_K>(w, rows, nb, row_stride, out, dtype, st, k, tail);
    case Q5_K: return launch_deq<Q5_K>(w, rows, nb, row_stride, out, dtype, st, k, tail);
    case Q8_0: return launch_deq<Q8_0>(w, rows, nb, row_stride, out, dtype, st, k, tail);
    case Q4_0: return launch_deq<Q4_0>(w, rows, nb, row_stride, out, dtype, st, k, tail);
    case Q4_1: return launch_deq<Q4_1>(w, rows, nb, row_stride, out, dtype, st, k, tail);
    case MXFP4: return launch_deq<MXFP4>(w, rows, nb, row_stride, out, dtype, st, k, tail);
    case TQ2_0: return launch_deq<TQ2_0>(w, rows, nb, row_stride, out, dtype, st, k, tail);
    case TQ1_0: return launch_deq<TQ1_0>(w, rows, nb, row_stride, out, dtype, st, k, tail);
    case NVFP4: return launch_deq<NVFP4>(w, rows, nb, row_stride, out, dtype, st, k, tail);
    case IQ2_XS: return launch_deq<IQ2_XS>(w, rows, nb, row_stride, out, dtype, st, k, tail);
    case IQ2_S: return launch_deq<IQ2_S>(w, rows, nb, row_stride, out, dtype, st, k, tail);
    case IQ3_S: return launch_deq<IQ3_S>(w, rows, nb, row_stride, out, dtype, st, k, tail);
    case IQ1_S: return launch_deq<IQ1_S>(w, rows, nb, row_stride, out, dtype, st, k, tail);
    case IQ1_M: return launch_deq<IQ1_M>(w, rows, nb, row_stride, out, dtype, st, k, tail);
    case Q5_0: return launch_deq<Q5_0>(w, rows, nb, row_stride, out, dtype, st, k, tail);
    case Q5_1: return launch_deq<Q5_1>(w, rows, nb, row_stride, out, dtype, st, k, tail);
    case Q2_K: return launch_deq<Q2_K>(w, rows, nb, row_stride, out, dtype, st, k, tail);
    case Q3_K: return launch_deq<Q3_K>(w, rows, nb, row_stride, out, dtype, st, k, tail);
    case IQ4_NL: return launch_deq<IQ4_NL>(w, rows, nb, row_stride, out, dtype, st, k, tail);
    case Q6_K: return launch_deq<Q6_K>(w, rows, nb, row_stride, out, dtype, st, k, tail);
    case IQ3_XXS: return launch_deq<IQ3_XXS>(w, rows, nb, row_stride, out, dtype, st, k, tail);
    case IQ4_XS: return launch_deq<IQ4_XS>(w, rows, nb, row_stride, out, dtype, st, k, tail);
    default: return launch_deq<IQ2_XXS>(w, rows, nb, row_stride, out, dtype, st, k, tail);
    }
}

}  // namespace kq
