// kq_gemv.cu -- fused dequantize x GEMV for decode (M <= 32 activation rows
// per weight matrix).  Replaces mlx-kquant's quantized_matmul small-M route
// (called from KQuantLinear, gmlx/modules.py:1535-1539, and directly at
// gmlx/occupancy_fuse.py:284-287), the MoE decode gathers moe_glu_gather_kq /
// gather_qmv_kq (gmlx/modules.py:585-598) and their row-concat callers.
//
// Design (B200, HBM-bound):
//  * Persistent CTAs: 1 producer warp + 4 consumer warps.  A work unit is
//    (group, 32-row tile, K split).  The producer streams each row's raw
//    super-blocks (144/210/66 B, never repacked) into a shared-memory ring with
//    1-D bulk async copies (cp.async.bulk, completion on an mbarrier, L2
//    evict-first).  Copies start at the 16-byte granule holding the row's first
//    byte, so unaligned Q6_K/IQ2_XXS rows stream the same way as Q4_K.
//  * Each consumer warp owns one super-block per stage and turns the packed
//    bits straight into mma.sync m16n8k16 A fragments: quant values become
//    exact small-integer bf16 (or f16) by OR-ing them into the mantissa of a
//    magic constant, so the tensor-core products q*x are exact and the
//    per-sub-block scale is applied once per sub-block to the f32 partial:
//      Q4_K : sum (d sc)*q*x - (dmin m)*sum x  via  T = sum (128+q) x
//             acc += dsc*T - (128 dsc + dmin m) * S_j   (S_j = sub-block sum of x)
//      Q6_K : A = (128 + q) - 160 = q - 32 (exact packed subtract), acc += dsc*T
//      IQ2  : A = +-grid (table of exact bf16, sign bit xor), acc += db*T
//  * Tokens (activation rows) are the MMA N dimension (8 per n-tile, up to 4).
//  * Split-K partials (f32) are combined deterministically (fixed split order)
//    by the last CTA to finish a tile; the tile counters reset themselves.
//  * Fused GLU: a 32-row tile holds 16 gate rows and the same 16 up rows, so
//    act(gate)*up is formed in the epilogue without a second pass.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "kq_internal.cuh"
#include "kq_ptx.cuh"

namespace kq {
namespace {

constexpr int CW = 4;             // consumer warps
constexpr int NTHREADS = 32 * (CW + 1);
constexpr int TROWS = 32;         // weight rows per tile
constexpr int RED_TS = 36;        // token stride (floats) of the reduction buffer
constexpr int S_FLOATS = 4096;    // Q4_K sub-block sums capacity (16 KB)

template <int C> struct GCfg;
template <> struct GCfg<Q4_K> { static constexpr int NS = 3, SUBS = 8, SCW = 16; };
template <> struct GCfg<Q6_K> { static constexpr int NS = 3, SUBS = 16, SCW = 16; };
template <> struct GCfg<IQ2_XXS> { static constexpr int NS = 6, SUBS = 8, SCW = 8; };

__host__ __device__ constexpr int spitch_of(int bpb) {
    // one row of a stage: CW blocks + 16 B slack for the granule offset;
    // pitch == 32 (mod 128) spreads 8 rows x 32 B over all banks.
    return ((((CW * bpb + 16 + 15) / 16 * 16) - 32 + 127) / 128) * 128 + 32;
}

template <int C> struct GLayout {
    static constexpr int bpb = Fmt<C>::bpb;
    static constexpr int SP = spitch_of(bpb);
    static constexpr int NS = GCfg<C>::NS;
    static constexpr int STAGE = TROWS * SP;
    static constexpr int OFF_BAR = 0;                              // 2*NS mbarriers
    static constexpr int OFF_ROWOFF = 128;                         // NS x 32 bytes
    static constexpr int OFF_MISC = OFF_ROWOFF + 32 * 8;           // flags
    static constexpr int OFF_GRID = 512;                           // IQ2 grid: 256 x 16 B
    static constexpr int OFF_RING = OFF_GRID + (C == IQ2_XXS ? 4096 : 0);
    static constexpr int OFF_SCALE = OFF_RING + NS * STAGE;        // CW x 32 x SCW floats
    static constexpr int OFF_S = OFF_SCALE + CW * 32 * GCfg<C>::SCW * 4;
    static constexpr int OFF_RED = OFF_S + (C == Q4_K ? S_FLOATS * 4 : 0);
    static constexpr int BYTES = OFF_RED + CW * 32 * RED_TS * 4;
};

struct Unit {
    int g, s, tile, m, e;
    int b0, b1;
};

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Bounded mbarrier wait shared by all warps of the CTA: gives up after ~2 s or
// as soon as another warp gave up, records the error once and returns false.
__device__ __forceinline__ bool wait_bounded(uint64_t *bar, uint32_t parity, volatile int *abort, int *err,
                                             int code) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t i = 1;; i++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255) == 0) {
            if (*abort) return false;
            if (globaltimer() - t0 > 2000000000ull) {
                *abort = 1;
                atomicCAS(err, 0, code);
                return false;
            }
        }
    }
}

template <bool F16> __device__ __forceinline__ uint32_t magic2() { return F16 ? 0x64006400u : 0x43004300u; }
template <bool F16> __device__ __forceinline__ float magic_f() { return F16 ? 1024.f : 128.f; }

template <bool F16> __device__ __forceinline__ uint32_t sub2(uint32_t a, float v) {
    if constexpr (F16) {
        __half2 h = *reinterpret_cast<__half2 *>(&a);
        h = __hsub2(h, __float2half2_rn(v));
        return *reinterpret_cast<uint32_t *>(&h);
    } else {
        __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162 *>(&a);
        h = __hsub2(h, __float2bfloat162_rn(v));
        return *reinterpret_cast<uint32_t *>(&h);
    }
}

__device__ __forceinline__ float bytef(uint32_t w, int i) {  // exact byte -> float via the 2^23 magic
    return __uint_as_float(prmt(w, 0x4b000000u, 0x7650u | (uint32_t)i)) - 8388608.f;
}

template <bool F16> __device__ __forceinline__ float act_to_f(const void *x, int64_t i) {
    if constexpr (F16) return __half2float(reinterpret_cast<const __half *>(x)[i]);
    else return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(x)[i]);
}

__device__ __forceinline__ void store_out(void *y, int dtype, int64_t i, float v) {
    if (dtype == F32) reinterpret_cast<float *>(y)[i] = v;
    else if (dtype == BF16) reinterpret_cast<__nv_bfloat16 *>(y)[i] = __float2bfloat16_rn(v);
    else reinterpret_cast<__half *>(y)[i] = __float2half_rn(v);
}

__device__ __forceinline__ float apply_act(int act, float g) {
    if (act == ACT_SILU) return g / (1.0f + expf(-g));
    if (act == ACT_GELU) return 0.5f * g * (1.0f + erff(g * 0.70710678118654752f));
    // tanh approximation
    const float c = 0.7978845608028654f;
    return 0.5f * g * (1.0f + tanhf(c * (g + 0.044715f * g * g * g)));
}

template <bool F16> __device__ __forceinline__ uint4 ldx16(const void *x, int64_t i) {
    return __ldg(reinterpret_cast<const uint4 *>(reinterpret_cast<const uint16_t *>(x) + i));
}
template <bool F16> __device__ __forceinline__ uint2 ldx8(const void *x, int64_t i) {
    return __ldg(reinterpret_cast<const uint2 *>(reinterpret_cast<const uint16_t *>(x) + i));
}

template <int NT, bool GLU>
__device__ __forceinline__ bool decode_unit(const GemvArgs &a, int u, int tiles, int n_groups, int nb, Unit &U) {
    const int per_g = a.splits * tiles;
    U.g = u / per_g;
    if (U.g >= n_groups) return false;
    const int r = u - U.g * per_g;
    U.s = r / tiles;
    U.tile = r - U.s * tiles;
    const int bps = (nb + a.splits - 1) / a.splits;
    U.b0 = U.s * bps;
    U.b1 = min(nb, U.b0 + bps);
    if (a.dense_m > 0) {
        U.m = min(32, a.dense_m - 32 * U.g);
        U.e = 0;
    } else {
        U.m = __ldg(a.grp_count + U.g);
        U.e = __ldg(a.grp_expert + U.g);
    }
    return true;
}

__device__ __forceinline__ int xrow_of(const GemvArgs &a, const Unit &U, int tok) {
    return a.dense_m > 0 ? 32 * U.g + tok : __ldg(a.grp_xrow + 32 * U.g + tok);
}
__device__ __forceinline__ int orow_of(const GemvArgs &a, const Unit &U, int tok) {
    return a.dense_m > 0 ? 32 * U.g + tok : __ldg(a.grp_orow + 32 * U.g + tok);
}

// -------------------------------------------------------------------------
// per-codec consumer work on one super-block of 32 rows

template <int C, int NT, bool F16>
struct Block;

// Q4_K --------------------------------------------------------------------
template <int NT, bool F16>
struct Block<Q4_K, NT, F16> {
    static __device__ __forceinline__ void run(const uint8_t *sb, const uint8_t *roff, int col, float *stab,
                                               const float *Ssm, int jbase, const GemvArgs &a, const Unit &U,
                                               int64_t k0, float acc[2][NT][4]) {
        const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
        constexpr int bpb = 144, SP = GLayout<Q4_K>::SP;
        // header of row `lane`: 8 x (d*sc, 128*d*sc + dmin*m)
        {
            const uint8_t *h = sb + lane * SP + roff[lane] + col * bpb;
            const uint32_t h0 = lds_u32_a2(h), s0 = lds_u32_a2(h + 4), s1 = lds_u32_a2(h + 8), s2 = lds_u32_a2(h + 12);
            const float d = half_bits_to_float(h0 & 0xffffu), dmin = half_bits_to_float(h0 >> 16);
            uint32_t sc03, sc47, m03, m47;
            q4k_unpack_scales(s0, s1, s2, sc03, sc47, m03, m47);
            float4 *o = reinterpret_cast<float4 *>(stab + lane * 16);
#pragma unroll
            for (int j = 0; j < 8; j += 2) {
                const uint32_t sw = j < 4 ? sc03 : sc47, mw = j < 4 ? m03 : m47;
                const float ds0 = d * bytef(sw, j & 3), ds1 = d * bytef(sw, (j & 3) + 1);
                const float mt0 = fmaf(magic_f<F16>(), ds0, dmin * bytef(mw, j & 3));
                const float mt1 = fmaf(magic_f<F16>(), ds1, dmin * bytef(mw, (j & 3) + 1));
                o[j >> 1] = make_float4(ds0, mt0, ds1, mt1);
            }
        }
        __syncwarp();
#pragma unroll
        for (int c = 0; c < 4; c++) {
            // B fragments: sub 2c (low nibbles) at k0+64c, sub 2c+1 (high) at +32
            uint32_t B[2][NT][2][2];
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                const int tok = 8 * nt + g;
                uint4 xl = make_uint4(0, 0, 0, 0), xh = xl;
                if (tok < U.m) {
                    const int64_t base = (int64_t)xrow_of(a, U, tok) * a.x_row_stride + k0 + 64 * c + 8 * t;
                    xl = ldx16<F16>(a.x, base);
                    xh = ldx16<F16>(a.x, base + 32);
                }
                B[0][nt][0][0] = prmt(xl.x, xl.y, 0x5410);
                B[0][nt][0][1] = prmt(xl.x, xl.y, 0x7632);
                B[0][nt][1][0] = prmt(xl.z, xl.w, 0x5410);
                B[0][nt][1][1] = prmt(xl.z, xl.w, 0x7632);
                B[1][nt][0][0] = prmt(xh.x, xh.y, 0x5410);
                B[1][nt][0][1] = prmt(xh.x, xh.y, 0x7632);
                B[1][nt][1][0] = prmt(xh.z, xh.w, 0x5410);
                B[1][nt][1][1] = prmt(xh.z, xh.w, 0x7632);
            }
#pragma unroll
            for (int mt = 0; mt < 2; mt++) {
                const int ra = 16 * mt + g, rb = ra + 8;
                const uint2 wa = *reinterpret_cast<const uint2 *>(sb + ra * SP + roff[ra] + col * bpb + 16 + 32 * c + 8 * t);
                const uint2 wb = *reinterpret_cast<const uint2 *>(sb + rb * SP + roff[rb] + col * bpb + 16 + 32 * c + 8 * t);
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    float T[NT][4];
#pragma unroll
                    for (int nt = 0; nt < NT; nt++) T[nt][0] = T[nt][1] = T[nt][2] = T[nt][3] = 0.f;
#pragma unroll
                    for (int s = 0; s < 2; s++) {
                        const uint32_t xa = s ? wa.y : wa.x, xb = s ? wb.y : wb.x;
                        uint32_t A[4];
                        A[0] = lop_and_or(xa >> (4 * h), 0x000f000fu, magic2<F16>());
                        A[1] = lop_and_or(xb >> (4 * h), 0x000f000fu, magic2<F16>());
                        A[2] = lop_and_or(xa >> (8 + 4 * h), 0x000f000fu, magic2<F16>());
                        A[3] = lop_and_or(xb >> (8 + 4 * h), 0x000f000fu, magic2<F16>());
#pragma unroll
                        for (int nt = 0; nt < NT; nt++) mma16816<F16>(T[nt], A, B[h][nt][s][0], B[h][nt][s][1], T[nt]);
                    }
                    const int j = 2 * c + h;
                    const float2 sa = *reinterpret_cast<const float2 *>(stab + ra * 16 + 2 * j);
                    const float2 sbv = *reinterpret_cast<const float2 *>(stab + rb * 16 + 2 * j);
#pragma unroll
                    for (int nt = 0; nt < NT; nt++) {
                        const float2 S2 = *reinterpret_cast<const float2 *>(Ssm + (jbase + j) * (8 * NT) + 8 * nt + 2 * t);
                        acc[mt][nt][0] += fmaf(sa.x, T[nt][0], -sa.y * S2.x);
                        acc[mt][nt][1] += fmaf(sa.x, T[nt][1], -sa.y * S2.y);
                        acc[mt][nt][2] += fmaf(sbv.x, T[nt][2], -sbv.y * S2.x);
                        acc[mt][nt][3] += fmaf(sbv.x, T[nt][3], -sbv.y * S2.y);
                    }
                }
            }
        }
    }
};

// Q6_K --------------------------------------------------------------------
template <int NT, bool F16>
struct Block<Q6_K, NT, F16> {
    static __device__ __forceinline__ uint32_t qh_shift(uint32_t q, int s) {
        return s == 0 ? (q << 4) : s == 1 ? (q << 2) : s == 2 ? q : (q >> 2);
    }
    static __device__ __forceinline__ void run(const uint8_t *sb, const uint8_t *roff, int col, float *stab,
                                               const float *, int, const GemvArgs &a, const Unit &U, int64_t k0,
                                               float acc[2][NT][4]) {
        const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
        constexpr int bpb = 210, SP = GLayout<Q6_K>::SP;
        {
            const uint8_t *h = sb + lane * SP + roff[lane] + col * bpb;
            const float d = half_bits_to_float(*reinterpret_cast<const uint16_t *>(h + 208));
            float4 *o = reinterpret_cast<float4 *>(stab + lane * 16);
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const uint32_t w = lds_u32_a2(h + 192 + 4 * q) ^ 0x80808080u;  // int8 -> biased byte
                o[q] = make_float4(d * (bytef(w, 0) - 128.f), d * (bytef(w, 1) - 128.f), d * (bytef(w, 2) - 128.f),
                                   d * (bytef(w, 3) - 128.f));
            }
        }
        __syncwarp();
#pragma unroll
        for (int hf = 0; hf < 2; hf++) {
#pragma unroll
            for (int lh = 0; lh < 2; lh++) {
                // logical weights 128hf + 32s + 16lh + 4t + {0..3}, s = 0..3
                uint32_t B[NT][4][2];
#pragma unroll
                for (int nt = 0; nt < NT; nt++) {
                    const int tok = 8 * nt + g;
#pragma unroll
                    for (int s = 0; s < 4; s++) {
                        uint2 xv = make_uint2(0, 0);
                        if (tok < U.m)
                            xv = ldx8<F16>(a.x, (int64_t)xrow_of(a, U, tok) * a.x_row_stride + k0 + 128 * hf + 32 * s +
                                                    16 * lh + 4 * t);
                        B[nt][s][0] = prmt(xv.x, xv.y, 0x5410);
                        B[nt][s][1] = prmt(xv.x, xv.y, 0x7632);
                    }
                }
#pragma unroll
                for (int mt = 0; mt < 2; mt++) {
                    const int ra = 16 * mt + g, rb = ra + 8;
                    const uint8_t *pa = sb + ra * SP + roff[ra] + col * bpb;
                    const uint8_t *pb = sb + rb * SP + roff[rb] + col * bpb;
                    const int lo = 64 * hf + 16 * lh + 4 * t, ho = 128 + 32 * hf + 16 * lh + 4 * t;
                    const uint32_t qla[2] = {lds_u32_a2(pa + lo), lds_u32_a2(pa + lo + 32)};
                    const uint32_t qlb[2] = {lds_u32_a2(pb + lo), lds_u32_a2(pb + lo + 32)};
                    const uint32_t qha = lds_u32_a2(pa + ho), qhb = lds_u32_a2(pb + ho);
#pragma unroll
                    for (int s = 0; s < 4; s++) {
                        const int ns = 4 * (s >> 1);
                        const uint32_t la = qla[s & 1] >> ns, lb = qlb[s & 1] >> ns;
                        const uint32_t ha = qh_shift(qha, s), hb = qh_shift(qhb, s);
                        uint32_t A[4];
                        A[0] = sub2<F16>(lop_and_or(ha, 0x00300030u, lop_and_or(la, 0x000f000fu, magic2<F16>())), magic_f<F16>() + 32.f);
                        A[1] = sub2<F16>(lop_and_or(hb, 0x00300030u, lop_and_or(lb, 0x000f000fu, magic2<F16>())), magic_f<F16>() + 32.f);
                        A[2] = sub2<F16>(lop_and_or(ha >> 8, 0x00300030u, lop_and_or(la >> 8, 0x000f000fu, magic2<F16>())), magic_f<F16>() + 32.f);
                        A[3] = sub2<F16>(lop_and_or(hb >> 8, 0x00300030u, lop_and_or(lb >> 8, 0x000f000fu, magic2<F16>())), magic_f<F16>() + 32.f);
                        const int j = 8 * hf + 2 * s + lh;
                        const float sa = stab[ra * 16 + j], sbv = stab[rb * 16 + j];
#pragma unroll
                        for (int nt = 0; nt < NT; nt++) {
                            float T[4] = {0.f, 0.f, 0.f, 0.f};
                            mma16816<F16>(T, A, B[nt][s][0], B[nt][s][1], T);
                            acc[mt][nt][0] = fmaf(sa, T[0], acc[mt][nt][0]);
                            acc[mt][nt][1] = fmaf(sa, T[1], acc[mt][nt][1]);
                            acc[mt][nt][2] = fmaf(sbv, T[2], acc[mt][nt][2]);
                            acc[mt][nt][3] = fmaf(sbv, T[3], acc[mt][nt][3]);
                        }
                    }
                }
            }
        }
    }
};

// IQ2_XXS -----------------------------------------------------------------
template <int NT, bool F16>
struct Block<IQ2_XXS, NT, F16> {
    static __device__ __forceinline__ void run(const uint8_t *sb, const uint8_t *roff, int col, float *stab,
                                               const float *, int, const GemvArgs &a, const Unit &U, int64_t k0,
                                               float acc[2][NT][4], const uint4 *gridtab) {
        const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
        constexpr int bpb = 66, SP = GLayout<IQ2_XXS>::SP;
        {
            const uint8_t *h = sb + lane * SP + roff[lane] + col * bpb;
            const float d = half_bits_to_float(*reinterpret_cast<const uint16_t *>(h));
            float v[8];
#pragma unroll
            for (int s = 0; s < 8; s++) {
                const uint32_t a1 = lds_u32_a2(h + 6 + 8 * s);
                v[s] = d * (0.5f + (float)(a1 >> 28)) * 0.25f;
            }
            float4 *o = reinterpret_cast<float4 *>(stab + lane * 8);
            o[0] = make_float4(v[0], v[1], v[2], v[3]);
            o[1] = make_float4(v[4], v[5], v[6], v[7]);
        }
        __syncwarp();
#pragma unroll 2
        for (int sbk = 0; sbk < 8; sbk++) {
            uint32_t B[NT][4];
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                const int tok = 8 * nt + g;
                uint4 xv = make_uint4(0, 0, 0, 0);
                if (tok < U.m) xv = ldx16<F16>(a.x, (int64_t)xrow_of(a, U, tok) * a.x_row_stride + k0 + 32 * sbk + 8 * t);
                B[nt][0] = xv.x;
                B[nt][1] = xv.y;
                B[nt][2] = xv.z;
                B[nt][3] = xv.w;
            }
#pragma unroll
            for (int mt = 0; mt < 2; mt++) {
                const int ra = 16 * mt + g, rb = ra + 8;
                uint32_t Av[2][4];  // [row a/b][4 bf16 pairs]
#pragma unroll
                for (int rr = 0; rr < 2; rr++) {
                    const int row = rr ? rb : ra;
                    const uint8_t *p = sb + row * SP + roff[row] + col * bpb + 2 + 8 * sbk;
                    const uint32_t a0 = lds_u32_a2(p), a1 = lds_u32_a2(p + 4);
                    const uint32_t gi = (a0 >> (8 * t)) & 255u;
                    const uint32_t sg = ksigns((a1 >> (7 * t)) & 127u);
                    const uint4 G = gridtab[gi];
                    const uint32_t plo = (sg & 15u) * 0x10204080u, phi = (sg >> 4) * 0x10204080u;
                    Av[rr][0] = lop_xor_and(G.x, prmt(plo, 0, 0x9484), 0x80008000u);
                    Av[rr][1] = lop_xor_and(G.y, prmt(plo, 0, 0xB4A4), 0x80008000u);
                    Av[rr][2] = lop_xor_and(G.z, prmt(phi, 0, 0x9484), 0x80008000u);
                    Av[rr][3] = lop_xor_and(G.w, prmt(phi, 0, 0xB4A4), 0x80008000u);
                }
                float T[NT][4];
#pragma unroll
                for (int nt = 0; nt < NT; nt++) T[nt][0] = T[nt][1] = T[nt][2] = T[nt][3] = 0.f;
#pragma unroll
                for (int s = 0; s < 2; s++) {
                    const uint32_t A[4] = {Av[0][2 * s], Av[1][2 * s], Av[0][2 * s + 1], Av[1][2 * s + 1]};
#pragma unroll
                    for (int nt = 0; nt < NT; nt++) mma16816<F16>(T[nt], A, B[nt][2 * s], B[nt][2 * s + 1], T[nt]);
                }
                const float sa = stab[ra * 8 + sbk], sbv = stab[rb * 8 + sbk];
#pragma unroll
                for (int nt = 0; nt < NT; nt++) {
                    acc[mt][nt][0] = fmaf(sa, T[nt][0], acc[mt][nt][0]);
                    acc[mt][nt][1] = fmaf(sa, T[nt][1], acc[mt][nt][1]);
                    acc[mt][nt][2] = fmaf(sbv, T[nt][2], acc[mt][nt][2]);
                    acc[mt][nt][3] = fmaf(sbv, T[nt][3], acc[mt][nt][3]);
                }
            }
        }
    }
};

// -------------------------------------------------------------------------

template <int C, int NT, bool F16, bool GLU>
__global__ void __launch_bounds__(NTHREADS) gemv_kernel(const GemvArgs a) {
    using L = GLayout<C>;
    constexpr int bpb = Fmt<C>::bpb, NS = L::NS;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L::OFF_BAR);
    uint64_t *empty = full + NS;
    uint8_t *rowoff = smem + L::OFF_ROWOFF;
    volatile int *s_abort = reinterpret_cast<volatile int *>(smem + L::OFF_MISC);
    int *s_last = reinterpret_cast<int *>(smem + L::OFF_MISC + 4);
    uint4 *gridtab = reinterpret_cast<uint4 *>(smem + L::OFF_GRID);
    uint8_t *ring = smem + L::OFF_RING;
    float *Ssm = reinterpret_cast<float *>(smem + L::OFF_S);
    float *red = reinterpret_cast<float *>(smem + L::OFF_RED);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nb = a.K / QK;
    const int rows_out = GLU ? 16 : 32;
    const int tiles = (a.N + rows_out - 1) / rows_out;
    const int n_groups = a.dense_m > 0 ? (a.dense_m + 31) / 32 : min(*a.n_groups, a.max_groups);
    const int units = n_groups * a.splits * tiles;

    if (threadIdx.x == 0) {
        for (int i = 0; i < NS; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], CW);
        }
        *s_abort = 0;
        fence_mbar_init();
    }
    if constexpr (C == IQ2_XXS) {
        for (int e = threadIdx.x; e < 256; e += NTHREADS) {
            const uint64_t v = c_iq2xxs_grid[e];
            uint32_t w[4];
#pragma unroll
            for (int p = 0; p < 4; p++) {
                const float v0 = (float)((v >> (16 * p)) & 255u), v1 = (float)((v >> (16 * p + 8)) & 255u);
                if constexpr (F16) {
                    __half2 h = __floats2half2_rn(v0, v1);
                    w[p] = *reinterpret_cast<uint32_t *>(&h);
                } else {
                    __nv_bfloat162 h = __floats2bfloat162_rn(v0, v1);
                    w[p] = *reinterpret_cast<uint32_t *>(&h);
                }
            }
            gridtab[e] = make_uint4(w[0], w[1], w[2], w[3]);
        }
    }
    __syncthreads();

    if (warp == CW) {
        // ---------------- producer warp ----------------
        const uint64_t pol = policy_evict_first();
        uint32_t it = 0;
        for (int u = blockIdx.x; u < units; u += gridDim.x) {
            Unit U;
            decode_unit<NT, GLU>(a, u, tiles, n_groups, nb, U);
            const int orow = U.tile * rows_out + (GLU ? (lane & 15) : lane);
            const bool up = GLU && lane >= 16;
            const bool valid = orow < a.N;
            const uint8_t *base = up ? a.w2 + (int64_t)U.e * a.w2_expert_stride + (int64_t)orow * a.w2_row_stride
                                     : a.w + (int64_t)U.e * a.w_expert_stride + (int64_t)orow * a.w_row_stride;
            const int nst = (U.b1 - U.b0 + CW - 1) / CW;
            for (int st = 0; st < nst; st++, it++) {
                const int slot = it % NS;
                if (!wait_bounded(&empty[slot], ((it / NS) & 1) ^ 1, s_abort, a.err, 1)) { /* abort: keep flowing */ }
                const int bs = U.b0 + st * CW, nbk = min(CW, U.b1 - bs);
                const uintptr_t src = (uintptr_t)(base + (int64_t)bs * bpb);
                const uint32_t off = (uint32_t)(src & 15);
                const uint32_t bytes = valid ? ((off + nbk * bpb + 15) & ~15u) : 0u;
                rowoff[slot * 32 + lane] = (uint8_t)off;
                uint32_t total = bytes;
#pragma unroll
                for (int o = 16; o; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
                if (lane == 0) mbar_arrive_expect_tx(&full[slot], total);
                __syncwarp();
                if (bytes && !*s_abort)
                    bulk_g2s(ring + slot * L::STAGE + lane * L::SP, (const void *)(src - off), bytes, &full[slot], pol);
            }
        }
        return;
    }

    // ---------------- consumer warps ----------------
    float *stab = reinterpret_cast<float *>(smem + L::OFF_SCALE) + warp * 32 * GCfg<C>::SCW;
    const int ctid = threadIdx.x;  // 0 .. CW*32-1
    uint32_t it = 0;
    int s_key_g = -1, s_key_s = -1;
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
        Unit U;
        decode_unit<NT, GLU>(a, u, tiles, n_groups, nb, U);
        if constexpr (C == Q4_K) {
            if (U.g != s_key_g || U.s != s_key_s) {
                // sub-block sums of x for this group and K split: Ssm[sub][tok]
                named_bar_sync(1, CW * 32);
                const int nsub = (U.b1 - U.b0) * 8;
                for (int i = ctid; i < nsub * 8 * NT; i += CW * 32) {
                    const int sub = i / (8 * NT), tok = i - sub * (8 * NT);
                    float sacc = 0.f;
                    if (tok < U.m) {
                        const int64_t base = (int64_t)xrow_of(a, U, tok) * a.x_row_stride + (int64_t)U.b0 * QK + 32 * sub;
#pragma unroll
                        for (int q = 0; q < 4; q++) {
                            const uint4 v = ldx16<F16>(a.x, base + 8 * q);
                            const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                            for (int e = 0; e < 4; e++) {
                                float lo, hi;
                                if constexpr (F16) {
                                    const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w4[e]));
                                    lo = f.x; hi = f.y;
                                } else {
                                    lo = __uint_as_float(w4[e] << 16);
                                    hi = __uint_as_float(w4[e] & 0xffff0000u);
                                }
                                sacc += lo + hi;
                            }
                        }
                    }
                    Ssm[i] = sacc;
                }
                named_bar_sync(1, CW * 32);
                s_key_g = U.g;
                s_key_s = U.s;
            }
        }
        float acc[2][NT][4];
#pragma unroll
        for (int mt = 0; mt < 2; mt++)
#pragma unroll
            for (int nt = 0; nt < NT; nt++) acc[mt][nt][0] = acc[mt][nt][1] = acc[mt][nt][2] = acc[mt][nt][3] = 0.f;

        const int nst = (U.b1 - U.b0 + CW - 1) / CW;
        for (int st = 0; st < nst; st++, it++) {
            const int slot = it % NS;
            wait_bounded(&full[slot], (it / NS) & 1, s_abort, a.err, 2);
            const int b = U.b0 + st * CW + warp;
            if (b < U.b1 && !*s_abort) {
                const uint8_t *sb = ring + slot * L::STAGE;
                const int64_t k0 = (int64_t)b * QK;
                if constexpr (C == IQ2_XXS)
                    Block<C, NT, F16>::run(sb, rowoff + slot * 32, warp, stab, Ssm, (b - U.b0) * 8, a, U, k0, acc, gridtab);
                else
                    Block<C, NT, F16>::run(sb, rowoff + slot * 32, warp, stab, Ssm, (b - U.b0) * 8, a, U, k0, acc);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        }

        // ---- cross-warp reduction: red[w][tok][row]
        {
            const int g = lane >> 2, t = lane & 3;
            float *r = red + warp * 32 * RED_TS;
#pragma unroll
            for (int mt = 0; mt < 2; mt++)
#pragma unroll
                for (int nt = 0; nt < NT; nt++) {
                    const int row = 16 * mt + g, tok = 8 * nt + 2 * t;
                    r[tok * RED_TS + row] = acc[mt][nt][0];
                    r[(tok + 1) * RED_TS + row] = acc[mt][nt][1];
                    r[tok * RED_TS + row + 8] = acc[mt][nt][2];
                    r[(tok + 1) * RED_TS + row + 8] = acc[mt][nt][3];
                }
        }
        named_bar_sync(1, CW * 32);
        const int m = U.m;
        if (a.splits == 1) {
            for (int i = ctid; i < rows_out * m; i += CW * 32) {
                const int row = i % rows_out, tok = i / rows_out;
                const int n = U.tile * rows_out + row;
                if (n >= a.N) continue;
                float v = 0.f, v2 = 0.f;
#pragma unroll
                for (int w = 0; w < CW; w++) {
                    v += red[w * 32 * RED_TS + tok * RED_TS + row];
                    if (GLU) v2 += red[w * 32 * RED_TS + tok * RED_TS + row + 16];
                }
                if (GLU) v = apply_act(a.act, v) * v2;
                store_out(a.y, a.y_dtype, (int64_t)orow_of(a, U, tok) * a.y_row_stride + n, v);
            }
        } else {
            const int slot_id = (U.g * tiles + U.tile) * a.splits + U.s;
            float *part = a.partial + (int64_t)slot_id * 1024;
            for (int i = ctid; i < 32 * m; i += CW * 32) {
                const int row = i & 31, tok = i >> 5;
                float v = 0.f;
#pragma unroll
                for (int w = 0; w < CW; w++) v += red[w * 32 * RED_TS + tok * RED_TS + row];
                __stcg(part + tok * 32 + row, v);
            }
            __threadfence();
            named_bar_sync(1, CW * 32);
            if (ctid == 0) {
                const int old = atomicAdd(a.counters + U.g * tiles + U.tile, 1);
                *s_last = (old == a.splits - 1);
            }
            named_bar_sync(1, CW * 32);
            if (*s_last) {
                __threadfence();
                const float *p0 = a.partial + (int64_t)(U.g * tiles + U.tile) * a.splits * 1024;
                for (int i = ctid; i < rows_out * m; i += CW * 32) {
                    const int row = i % rows_out, tok = i / rows_out;
                    const int n = U.tile * rows_out + row;
                    if (n >= a.N) continue;
                    float v = 0.f, v2 = 0.f;
                    for (int s = 0; s < a.splits; s++) {
                        v += __ldcg(p0 + s * 1024 + tok * 32 + row);
                        if (GLU) v2 += __ldcg(p0 + s * 1024 + tok * 32 + row + 16);
                    }
                    if (GLU) v = apply_act(a.act, v) * v2;
                    store_out(a.y, a.y_dtype, (int64_t)orow_of(a, U, tok) * a.y_row_stride + n, v);
                }
                if (ctid == 0) a.counters[U.g * tiles + U.tile] = 0;
            }
        }
        named_bar_sync(1, CW * 32);
    }
}

template <int C, int NT, bool F16, bool GLU>
cudaError_t launch_t(const GemvArgs &a, cudaStream_t st) {
    using L = GLayout<C>;
    auto kern = gemv_kernel<C, NT, F16, GLU>;
    static bool configured = false;  // per instantiation; attribute set is idempotent
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::BYTES);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    const int rows_out = GLU ? 16 : 32;
    const int tiles = (a.N + rows_out - 1) / rows_out;
    const int groups = a.dense_m > 0 ? (a.dense_m + 31) / 32 : a.max_groups;
    const long units = (long)groups * a.splits * tiles;
    int per_sm = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, NTHREADS, L::BYTES);
    if (per_sm < 1) per_sm = 1;
    const long cap = (long)num_sms() * per_sm;
    const int grid = (int)(units < cap ? units : cap);
    if (grid <= 0) return cudaSuccess;
    kern<<<grid, NTHREADS, L::BYTES, st>>>(a);
    return cudaGetLastError();
}

template <int C, bool F16, bool GLU>
cudaError_t launch_nt(const GemvArgs &a, cudaStream_t st) {
    const int nt = (a.max_tokens + 7) / 8;
    switch (nt) {
    case 1: return launch_t<C, 1, F16, GLU>(a, st);
    case 2: return launch_t<C, 2, F16, GLU>(a, st);
    case 3: return launch_t<C, 3, F16, GLU>(a, st);
    default: return launch_t<C, 4, F16, GLU>(a, st);
    }
}

template <int C>
cudaError_t launch_c(const GemvArgs &a, cudaStream_t st) {
    const bool f16 = a.x_dtype == F16, glu = a.act != ACT_NONE;
    if (f16) return glu ? launch_nt<C, true, true>(a, st) : launch_nt<C, true, false>(a, st);
    return glu ? launch_nt<C, false, true>(a, st) : launch_nt<C, false, false>(a, st);
}

}  // namespace

int gemv_choose_splits(int codec, int N, int K, int max_groups, int max_tokens, bool glu, int nsm) {
    const int nb = K / QK;
    const int rows_out = glu ? 16 : 32;
    const long base = (long)max_groups * ((N + rows_out - 1) / rows_out);
    const int nt = (max_tokens + 7) / 8;
    int s = 1;
    // enough units for ~2 per SM, keeping >= 2 stages (8 blocks) per split
    while (s < 8 && base * s < 2L * nsm && (nb + 2 * s - 1) / (2 * s) >= 2 * CW) s *= 2;
    if (codec == Q4_K)  // sub-block sums of one split must fit the 16 KB table
        while (((nb + s - 1) / s) * 8 * 8 * nt > S_FLOATS && s < nb) s *= 2;
    return s < 1 ? 1 : s;
}

void gemv_scratch_need(const GemvArgs &a, size_t *partial_bytes, size_t *counter_bytes) {
    const int rows_out = a.act != ACT_NONE ? 16 : 32;
    const long tiles = (a.N + rows_out - 1) / rows_out;
    const long groups = a.dense_m > 0 ? (a.dense_m + 31) / 32 : a.max_groups;
    if (a.splits <= 1) {
        *partial_bytes = 0;
        *counter_bytes = 0;
        return;
    }
    *partial_bytes = (size_t)(groups * tiles * a.splits) * 1024 * sizeof(float);
    *counter_bytes = (size_t)(groups * tiles) * sizeof(int);
}

cudaError_t launch_gemv(const GemvArgs &a, cudaStream_t st) {
    switch (a.codec) {
    case Q4_K: return launch_c<Q4_K>(a, st);
    case Q6_K: return launch_c<Q6_K>(a, st);
    default: return launch_c<IQ2_XXS>(a, st);
    }
}

}  // namespace kq
