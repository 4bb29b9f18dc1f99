// kq_gemv_dev.cuh -- device building blocks of the decode GEMV kernels
// (kq_gemv.cu: the per-launch GEMV; kq_chain.cu: the persistent chain of
// GEMVs): tile geometry, bounded waits, the mma.sync block decoders and the
// lane-per-row integer dot products of every codec.  Everything sits in an
// unnamed namespace, so each including translation unit gets its own copy.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "kq_internal.cuh"
#include "kq_ptx.cuh"

namespace kq {
namespace {

constexpr int CW = 8;             // consumer warps: 2 row halves x 4 block columns
constexpr int NCOL = 4;           // block columns (consumer warps per row half)
constexpr int NTHREADS = 32 * (CW + 1);
constexpr int TROWS = 32;         // weight rows per tile
constexpr int RED_TS = 36;        // token stride (floats) of the reduction buffer

// NS: ring stages; TABW: floats of the per-warp scale table.  Tables are laid
// out [sub-block][g][..] so lane (g, t) reads the values of both its rows
// (g and g+8) with one 16- or 8-byte load, conflict-free.
// BPW: super-blocks each consumer warp decodes per stage, so one row's copy
// per stage is KB = 4*BPW blocks (>= ~1 KB: smaller bulk copies are
// request-rate bound on the TMA engine).
template <int C> struct GCfg;
template <> struct GCfg<Q4_K> { static constexpr int TABW = 8 * 8 * 4, BPW = 2; };     // (dsc, -mt) x 2 rows
template <> struct GCfg<Q5_K> { static constexpr int TABW = 8 * 8 * 4, BPW = 2; };     // lane-per-row path only
template <> struct GCfg<Q8_0> { static constexpr int TABW = 8 * 8 * 4, BPW = 1; };     // lane-per-row path only
template <> struct GCfg<Q2_K> { static constexpr int TABW = 8 * 8 * 4, BPW = 2; };     // lane-per-row path only
template <> struct GCfg<Q3_K> { static constexpr int TABW = 8 * 8 * 4, BPW = 2; };     // lane-per-row path only
template <> struct GCfg<IQ1_S> { static constexpr int TABW = 8 * 8 * 4, BPW = 2; };    // lane-per-row path only
template <> struct GCfg<IQ1_M> { static constexpr int TABW = 8 * 8 * 4, BPW = 2; };    // lane-per-row path only
template <> struct GCfg<IQ2_XS> { static constexpr int TABW = 8 * 8 * 4, BPW = 2; };   // lane-per-row path only
template <> struct GCfg<IQ2_S> { static constexpr int TABW = 8 * 8 * 4, BPW = 2; };    // lane-per-row path only
template <> struct GCfg<IQ3_S> { static constexpr int TABW = 8 * 8 * 4, BPW = 2; };    // lane-per-row path only
template <> struct GCfg<MXFP4> { static constexpr int TABW = 8 * 8 * 4, BPW = 2; };    // lane-per-row path only
template <> struct GCfg<NVFP4> { static constexpr int TABW = 8 * 8 * 4, BPW = 2; };    // lane-per-row path only
template <> struct GCfg<TQ1_0> { static constexpr int TABW = 8 * 8 * 4, BPW = 2; };    // lane-per-row path only
template <> struct GCfg<TQ2_0> { static constexpr int TABW = 8 * 8 * 4, BPW = 2; };    // lane-per-row path only
template <> struct GCfg<Q4_1> { static constexpr int TABW = 8 * 8 * 4, BPW = 2; };     // lane-per-row path only
template <> struct GCfg<Q5_0> { static constexpr int TABW = 8 * 8 * 4, BPW = 2; };     // lane-per-row path only
template <> struct GCfg<Q5_1> { static constexpr int TABW = 8 * 8 * 4, BPW = 1; };     // lane-per-row path only
template <> struct GCfg<Q4_0> { static constexpr int TABW = 8 * 8 * 4, BPW = 2; };     // lane-per-row path only
template <> struct GCfg<IQ4_NL> { static constexpr int TABW = 8 * 8 * 4, BPW = 2; };   // lane-per-row path only
template <> struct GCfg<Q6_K> { static constexpr int TABW = 16 * 8 * 2, BPW = 1; };    // dsc x 2 rows
template <> struct GCfg<IQ2_XXS> { static constexpr int TABW = 8 * 8 * 2, BPW = 2; };  // db x 2 rows
template <> struct GCfg<IQ3_XXS> { static constexpr int TABW = 8 * 8 * 4, BPW = 2; };  // lane-per-row path only
template <> struct GCfg<IQ4_XS> { static constexpr int TABW = 8 * 8 * 4, BPW = 2; };   // lane-per-row path only
// shared-memory lattice table: IQ2_XXS 256 x 16 B (MMA path) or 8 B; IQ3_XXS 256 x 4 B;
// IQ2_XS 512 x 8 B; IQ2_S 1024 x 8 B; IQ3_S 512 x 4 B; IQ1_S / IQ1_M 2048 x 8 B
template <int C> constexpr int GRIDB = C == IQ2_XXS ? 4096 : C == IQ3_XXS ? 1024 : C == IQ2_XS ? 4096 : C == IQ2_S ? 8192
                                     : C == IQ3_S ? 2048 : (C == IQ1_S || C == IQ1_M) ? 16384 : 0;
template <int C> constexpr int KB_OF = NCOL * GCfg<C>::BPW;
template <int C> constexpr int XSTR_OF = KB_OF<C> * QK * 2 + 64;  // staged activation row stride (bytes)
constexpr int SMEM_BUDGET = 112 * 1024;  // per CTA: two CTAs per SM
// 17-32 activation rows of Q4_K/Q6_K: one CTA per SM (registers for the MMA
// fragments of 3-4 n-tiles without spills) with the ring twice as deep;
// measured slower for 9-16 rows and for IQ2_XXS
template <int C, int NT, int XR> constexpr int CTAS_PER_SM = (XR == 0 && NT >= 3 && C != IQ2_XXS) ? 1 : 2;
constexpr int S_MAX = 2048;              // Q4_K one-row sub-block sums table: K <= 65536

template <int C, bool DPL = false> __host__ __device__ constexpr int spitch_of() {
    // one row of a stage: KB blocks + 16 B slack for the granule offset;
    // pitch == 32 (mod 128) spreads 8 rows x 32 B over all banks (MMA path);
    // pitch == 16 (mod 128) spreads 8 lanes x 16 B of 8 rows (lane-per-row path).
    return ((((KB_OF<C> * Fmt<C>::bpb + 16 + 15) / 16 * 16) - (DPL ? 16 : 32) + 127) / 128) * 128 + (DPL ? 16 : 32);
}

// XR: activation rows staged per stage with the weights (0 = read from global)
template <int C, int NT, int XR> struct GLayout {
    static constexpr bool XS = XR > 0;
    // lane-per-row integer dot-product path: XR activation rows staged with the
    // weights (1: every codec; up to 4 rows per group: IQ2_XXS)
    static constexpr bool DP = XR >= 1;
    static constexpr int bpb = Fmt<C>::bpb;
    static constexpr int KB = KB_OF<C>;
    static constexpr int XSTR = XSTR_OF<C>;
    static constexpr int SP = spitch_of<C, DP>();
    static constexpr int WBYTES = TROWS * SP;
    // a stage starts on 128 bytes on the lane-per-row path: tensor copies (the
    // Q4_K one-row weights) need a 128-byte aligned shared destination
    static constexpr int STAGE = DP ? (WBYTES + XR * XSTR + 127) / 128 * 128 : WBYTES + XR * XSTR;
    // scale tables (MMA path) or per-warp quantized activations (lane-per-row path)
    static constexpr int TABS = DP ? CW * 640 * XR : CW * GCfg<C>::TABW * GCfg<C>::BPW * 4;  // per warp: 160 / TABW*BPW floats
    // rotating row-partial buffers (NS + 1 <= 4; NS + 1 <= 3 with several rows), one row x XR tokens per warp
    static constexpr int DPB = DP ? (XR > 1 ? 3 : 4) * CW * 32 * 4 * XR : 0;
    static constexpr bool SX = false;  // Q4_K one-row sums table (off: its per-launch prologue costs more than it saves)
    static constexpr int SBYTES = SX ? S_MAX * 4 : 0;
    // one reduction buffer (two, alternating): [column][token][row]; the
    // lane-per-row path keeps one token per warp
    // (several staged rows run only on the dynamic schedule, which needs none)
    static constexpr int REDB = DP ? (XR > 1 ? 0 : CW * RED_TS * 4) : NCOL * 8 * NT * RED_TS * 4;
    static constexpr int FIXED = 512 + GRIDB<C> + TABS + SBYTES + 2 * REDB + DPB;
    static constexpr int NS_FIT = (SMEM_BUDGET * 2 / CTAS_PER_SM<C, NT, XR> - FIXED) / STAGE;
    // ring depth (<= 8: rowoff table; <= 3 on the lane-per-row path, whose
    // partial buffers rotate over NS + 1 <= 4 tiles)
    static constexpr int NS_MAX = DP ? (XR > 1 ? 2 : 3) : 8;
    static constexpr int NS = NS_FIT > NS_MAX ? NS_MAX : (NS_FIT < 2 ? 2 : NS_FIT);
    static constexpr int OFF_BAR = 0;                              // 2*NS mbarriers
    static constexpr int OFF_ROWOFF = 128;                         // NS x 32 bytes
    static constexpr int OFF_MISC = OFF_ROWOFF + 32 * 8;           // flags
    static constexpr int OFF_UNIT = 512;                           // dynamic mode: tile id per ring slot
    static constexpr int OFF_GRID = 640;                           // lattice table (GRIDB bytes)
    static constexpr int OFF_RING = OFF_GRID + GRIDB<C>;
    static constexpr int OFF_SCALE = OFF_RING + NS * STAGE;        // CW x TABW floats
    static constexpr int OFF_S = OFF_SCALE + TABS;
    static constexpr int OFF_RED = OFF_S + SBYTES;
    static constexpr int OFF_DPB = OFF_RED + 2 * REDB;
    static constexpr int BYTES = OFF_DPB + DPB;
    static_assert(!DP || NS <= 3, "lane-per-row path sizes its partial buffers for NS <= 3");
    static_assert(XR <= 1 || NS <= 2, "several staged rows size their partial buffers for NS <= 2");
    static_assert(!DP || CTAS_PER_SM<C, NT, XR> != 2 || BYTES <= 113 * 1024, "two CTAs per SM must fit");
};

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Bounded mbarrier wait shared by all warps of the CTA: gives up after ~2 s or
// as soon as another warp gave up, records the error once and returns false.
__device__ __forceinline__ bool wait_bounded(uint64_t *bar, uint32_t parity, volatile int *abort, int *err,
                                             int code, bool spin = false) {
    // the timer is read only every 1024 polls: a %globaltimer read is slow
    // enough to delay the wake-up of a wait that would otherwise end at once
    uint64_t t0 = 0;
    for (uint32_t i = 1;; i++) {
        if (spin ? mbar_test_wait(bar, parity) : mbar_try_wait(bar, parity)) return true;
        if ((i & 1023) == 0) {
            if (*abort) return false;
            const uint64_t now = globaltimer();
            if (t0 == 0) t0 = now;
            if (now - t0 > 2000000000ull) {
                *abort = 1;
                atomicCAS(err, 0, code);
                return false;
            }
        }
    }
}

template <bool F16> __device__ __forceinline__ uint32_t magic2() { return F16 ? 0x64006400u : 0x43004300u; }
template <bool F16> __device__ __forceinline__ float magic_f() { return F16 ? 1024.f : 128.f; }
template <bool F16> __device__ __forceinline__ uint32_t ones2() { return F16 ? 0x3c003c00u : 0x3f803f80u; }

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

// d += a * b on a pair of f32 (one packed FFMA2 on sm_100).
__device__ __forceinline__ void ffma2(float &d0, float &d1, float a0, float a1, float b0, float b1) {
    asm("{\n .reg .b64 ra, rb, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n mov.b64 rd, {%0, %1};\n"
        " fma.rn.f32x2 rd, ra, rb, rd;\n mov.b64 {%0, %1}, rd;\n}\n"
        : "+f"(d0), "+f"(d1)
        : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

// Activation fragment loads: from the staged slice (shared) or from global.
template <bool XS> __device__ __forceinline__ uint4 ldx16(const uint16_t *p) {
    if constexpr (XS) {
        uint4 v;
        asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                     : "r"(smem_u32(p)));
        return v;
    } else {
        return __ldg(reinterpret_cast<const uint4 *>(p));
    }
}
template <bool XS> __device__ __forceinline__ uint2 ldx8(const uint16_t *p) {
    if constexpr (XS) {
        uint2 v;
        asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(smem_u32(p)));
        return v;
    } else {
        return __ldg(reinterpret_cast<const uint2 *>(p));
    }
}

// optional per-output bias (dense, non-GLU): added once to each final value
__device__ __forceinline__ float bias_of(const GemvArgs &a, int n) {
    if (!a.bias) return 0.f;
    if (a.bias_dtype == F32) return reinterpret_cast<const float *>(a.bias)[n];
    if (a.bias_dtype == BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(a.bias)[n]);
    return __half2float(reinterpret_cast<const __half *>(a.bias)[n]);
}

struct Tile {
    int g, tile, m, e;
};

__device__ __forceinline__ void tile_of(const GemvArgs &a, int64_t gt, int tiles, Tile &T) {
    const int g32 = (int)gt;  // tile index fits 32 bits (checked on the host); 64-bit division is slow
    T.g = g32 / tiles;
    T.tile = g32 - T.g * tiles;
    if (a.dense_m > 0) {
        T.m = min(32, a.dense_m - 32 * T.g);
        T.e = 0;
    } else {
        T.m = __ldg(a.grp_count + T.g);
        T.e = __ldg(a.grp_expert + T.g);
    }
}

__device__ __forceinline__ int xrow_of(const GemvArgs &a, const Tile &T, int tok) {
    return a.dense_m > 0 ? 32 * T.g + tok : __ldg(a.grp_xrow + 32 * T.g + tok);
}
__device__ __forceinline__ int orow_of(const GemvArgs &a, const Tile &T, int tok) {
    return a.dense_m > 0 ? 32 * T.g + tok : __ldg(a.grp_orow + 32 * T.g + tok);
}

// stream-K partition: CTA c owns iterations [lo(c), lo(c+1))
__device__ __forceinline__ int64_t part_lo(int64_t c, int64_t I, int64_t P) { return c * I / P; }
__device__ __forceinline__ int64_t cta_of(int64_t i, int64_t I, int64_t P) { return ((i + 1) * P - 1) / I; }

// -------------------------------------------------------------------------
// per-codec consumer work: one super-block of one 16-row warp tile
// (rows 16*mt .. 16*mt+15 of the stage, block column `col`).  xr[nt] points at
// the activation row of lane g's token of n-tile nt, positioned at this
// block's first element (shared memory when XS, else global).

template <int C, int NT, bool F16, bool XS>
struct Block;

// Each run() decodes NB consecutive super-blocks (block columns col0 ..
// col0+NB-1 of the stage) for the warp's 16 rows; the NB blocks are
// independent work interleaved for instruction-level parallelism.  xr[nt]
// points at block col0's first activation element; block bb is at +bb*256.

// Q4_K --------------------------------------------------------------------
template <int NT, bool F16, bool XS>
struct Block<Q4_K, NT, F16, XS> {
    // Sx (one activation row): sub-block sums of x for block col0 from a shared
    // table; otherwise they come from an extra MMA with an all-ones A operand.
    template <int NB>
    static __device__ __forceinline__ void run(const uint8_t *sb, const uint8_t *roff, int col0, int mt, float *stab,
                                               const uint16_t *const xr[NT], float acc[NT][4], const uint4 *,
                                               const float *Sx = nullptr) {
        const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
        constexpr int bpb = 144, SP = spitch_of<Q4_K>();
        constexpr int TW = GCfg<Q4_K>::TABW;
        // header: lane -> (row lane&15, sub-blocks 4*(lane>>4) .. +3): (d*sc, -(128*d*sc + dmin*m))
#pragma unroll
        for (int bb = 0; bb < NB; bb++) {
            const int rr = lane & 15, r = 16 * mt + rr, hh = lane >> 4;
            const uint8_t *h = sb + r * SP + roff[r] + (col0 + bb) * bpb;
            const uint4 hv = *reinterpret_cast<const uint4 *>(h);
            const float d = half_bits_to_float(hv.x & 0xffffu), dmin = half_bits_to_float(hv.x >> 16);
            uint32_t sc03, sc47, m03, m47;
            q4k_unpack_scales(hv.y, hv.z, hv.w, sc03, sc47, m03, m47);
            const uint32_t sw = hh ? sc47 : sc03, mw = hh ? m47 : m03;
            float *o = stab + bb * TW + (rr & 7) * 4 + (rr >> 3) * 2;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const float ds = d * bytef(sw, j);
                *reinterpret_cast<float2 *>(o + (4 * hh + j) * 32) =
                    make_float2(ds, -fmaf(magic_f<F16>(), ds, dmin * bytef(mw, j)));
            }
        }
        __syncwarp();
        const int ra = 16 * mt + g, rb = ra + 8;
        const uint8_t *pa = sb + ra * SP + roff[ra] + col0 * bpb + 16 + 8 * t;
        const uint8_t *pb = sb + rb * SP + roff[rb] + col0 * bpb + 16 + 8 * t;
        const uint32_t ONES[4] = {ones2<F16>(), ones2<F16>(), ones2<F16>(), ones2<F16>()};
#pragma unroll
        for (int c = 0; c < 4; c++) {
#pragma unroll
            for (int bb = 0; bb < NB; bb++) {
                // B fragments: sub 2c (low nibbles) at 64c, sub 2c+1 (high) at 64c+32;
                // thread t holds logical weights 8t..8t+7 of each sub-block
                uint32_t B[2][NT][2][2];
#pragma unroll
                for (int nt = 0; nt < NT; nt++) {
                    const uint4 xl = ldx16<XS>(xr[nt] + bb * QK + 64 * c + 8 * t);
                    const uint4 xh = ldx16<XS>(xr[nt] + bb * QK + 64 * c + 32 + 8 * t);
                    B[0][nt][0][0] = prmt(xl.x, xl.y, 0x5410);
                    B[0][nt][0][1] = prmt(xl.x, xl.y, 0x7632);
                    B[0][nt][1][0] = prmt(xl.z, xl.w, 0x5410);
                    B[0][nt][1][1] = prmt(xl.z, xl.w, 0x7632);
                    B[1][nt][0][0] = prmt(xh.x, xh.y, 0x5410);
                    B[1][nt][0][1] = prmt(xh.x, xh.y, 0x7632);
                    B[1][nt][1][0] = prmt(xh.z, xh.w, 0x5410);
                    B[1][nt][1][1] = prmt(xh.z, xh.w, 0x7632);
                }
                const uint2 wa = *reinterpret_cast<const uint2 *>(pa + bb * bpb + 32 * c);
                const uint2 wb = *reinterpret_cast<const uint2 *>(pb + bb * bpb + 32 * c);
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    float T[NT][4], S[NT][4];
#pragma unroll
                    for (int nt = 0; nt < NT; nt++)
#pragma unroll
                        for (int q = 0; q < 4; q++) T[nt][q] = S[nt][q] = 0.f;
#pragma unroll
                    for (int s = 0; s < 2; s++) {
                        const uint32_t xa = s ? wa.y : wa.x, xb = s ? wb.y : wb.x;
                        uint32_t A[4];
                        A[0] = lop_and_or(xa >> (4 * h), 0x000f000fu, magic2<F16>());
                        A[1] = lop_and_or(xb >> (4 * h), 0x000f000fu, magic2<F16>());
                        A[2] = lop_and_or(xa >> (8 + 4 * h), 0x000f000fu, magic2<F16>());
                        A[3] = lop_and_or(xb >> (8 + 4 * h), 0x000f000fu, magic2<F16>());
#pragma unroll
                        for (int nt = 0; nt < NT; nt++) {
                            mma16816<F16>(T[nt], A, B[h][nt][s][0], B[h][nt][s][1], T[nt]);
                            mma16816<F16>(S[nt], ONES, B[h][nt][s][0], B[h][nt][s][1], S[nt]);
                        }
                    }
                    const float4 sc = *reinterpret_cast<const float4 *>(stab + bb * TW + (2 * c + h) * 32 + g * 4);
#pragma unroll
                    for (int nt = 0; nt < NT; nt++) {
                        ffma2(acc[nt][0], acc[nt][1], sc.x, sc.x, T[nt][0], T[nt][1]);
                        ffma2(acc[nt][0], acc[nt][1], sc.y, sc.y, S[nt][0], S[nt][1]);
                        ffma2(acc[nt][2], acc[nt][3], sc.z, sc.z, T[nt][2], T[nt][3]);
                        ffma2(acc[nt][2], acc[nt][3], sc.w, sc.w, S[nt][2], S[nt][3]);
                    }
                }
            }
        }
    }
};

// Q6_K --------------------------------------------------------------------
template <int NT, bool F16, bool XS>
struct Block<Q6_K, NT, F16, XS> {
    static __device__ __forceinline__ uint32_t qh_shift(uint32_t q, int s) {
        return s == 0 ? (q << 4) : s == 1 ? (q << 2) : s == 2 ? q : (q >> 2);
    }
    template <int NB>
    static __device__ __forceinline__ void run(const uint8_t *sb, const uint8_t *roff, int col0, int mt, float *stab,
                                               const uint16_t *const xr[NT], float acc[NT][4], const uint4 *,
                                               const float * = nullptr) {
        const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
        constexpr int bpb = 210, SP = spitch_of<Q6_K>();
        constexpr int TW = GCfg<Q6_K>::TABW;
#pragma unroll
        for (int bb = 0; bb < NB; bb++) {
            // header: lane -> (row lane&15, scales 8*(lane>>4) .. +7): d * sc
            const int rr = lane & 15, r = 16 * mt + rr, hh = lane >> 4;
            const uint8_t *h = sb + r * SP + roff[r] + (col0 + bb) * bpb;
            const float d = half_bits_to_float(*reinterpret_cast<const uint16_t *>(h + 208));
            float *o = stab + bb * TW + (rr & 7) * 2 + (rr >> 3);
#pragma unroll
            for (int q = 0; q < 2; q++) {
                const uint32_t w = lds_u32_a2(h + 192 + 8 * hh + 4 * q) ^ 0x80808080u;  // int8 -> biased byte
#pragma unroll
                for (int i = 0; i < 4; i++) o[(8 * hh + 4 * q + i) * 16] = d * (bytef(w, i) - 128.f);
            }
        }
        __syncwarp();
        const int ra = 16 * mt + g, rb = ra + 8;
#pragma unroll
        for (int hf = 0; hf < 2; hf++) {
#pragma unroll
            for (int lh = 0; lh < 2; lh++) {
#pragma unroll
                for (int bb = 0; bb < NB; bb++) {
                    const uint8_t *pa = sb + ra * SP + roff[ra] + (col0 + bb) * bpb;
                    const uint8_t *pb = sb + rb * SP + roff[rb] + (col0 + bb) * bpb;
                    // logical weights 128hf + 32s + 16lh + 4t + {0..3}, s = 0..3
                    uint32_t B[NT][4][2];
#pragma unroll
                    for (int nt = 0; nt < NT; nt++) {
#pragma unroll
                        for (int s = 0; s < 4; s++) {
                            const uint2 xv = ldx8<XS>(xr[nt] + bb * QK + 128 * hf + 32 * s + 16 * lh + 4 * t);
                            B[nt][s][0] = prmt(xv.x, xv.y, 0x5410);
                            B[nt][s][1] = prmt(xv.x, xv.y, 0x7632);
                        }
                    }
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
                        const float2 sc = *reinterpret_cast<const float2 *>(stab + bb * TW + j * 16 + g * 2);
#pragma unroll
                        for (int nt = 0; nt < NT; nt++) {
                            float T[4] = {0.f, 0.f, 0.f, 0.f};
                            mma16816<F16>(T, A, B[nt][s][0], B[nt][s][1], T);
                            ffma2(acc[nt][0], acc[nt][1], sc.x, sc.x, T[0], T[1]);
                            ffma2(acc[nt][2], acc[nt][3], sc.y, sc.y, T[2], T[3]);
                        }
                    }
                }
            }
        }
    }
};

// IQ2_XXS -----------------------------------------------------------------
template <int NT, bool F16, bool XS>
struct Block<IQ2_XXS, NT, F16, XS> {
    template <int NB>
    static __device__ __forceinline__ void run(const uint8_t *sb, const uint8_t *roff, int col0, int mt, float *stab,
                                               const uint16_t *const xr[NT], float acc[NT][4],
                                               const uint4 *gridtab, const float * = nullptr) {
        const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
        constexpr int bpb = 66, SP = spitch_of<IQ2_XXS>();
        constexpr int TW = GCfg<IQ2_XXS>::TABW;
#pragma unroll
        for (int bb = 0; bb < NB; bb++) {
            // header: lane -> (row lane&15, sub-blocks 4*(lane>>4) .. +3): d*(0.5+ls)*0.25
            const int rr = lane & 15, r = 16 * mt + rr, hh = lane >> 4;
            const uint8_t *h = sb + r * SP + roff[r] + (col0 + bb) * bpb;
            const float d = half_bits_to_float(*reinterpret_cast<const uint16_t *>(h));
            float *o = stab + bb * TW + (rr & 7) * 2 + (rr >> 3);
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const uint32_t a1 = lds_u32_a2(h + 6 + 8 * (4 * hh + q));
                o[(4 * hh + q) * 16] = d * (0.5f + (float)(a1 >> 28)) * 0.25f;
            }
        }
        __syncwarp();
        const int ra = 16 * mt + g, rb = ra + 8;
#pragma unroll 2
        for (int sbk = 0; sbk < 8; sbk++) {
#pragma unroll
            for (int bb = 0; bb < NB; bb++) {
                const uint8_t *pa = sb + ra * SP + roff[ra] + (col0 + bb) * bpb + 2;
                const uint8_t *pb = sb + rb * SP + roff[rb] + (col0 + bb) * bpb + 2;
                uint32_t B[NT][4];
#pragma unroll
                for (int nt = 0; nt < NT; nt++) {
                    const uint4 xv = ldx16<XS>(xr[nt] + bb * QK + 32 * sbk + 8 * t);
                    B[nt][0] = xv.x;
                    B[nt][1] = xv.y;
                    B[nt][2] = xv.z;
                    B[nt][3] = xv.w;
                }
                uint32_t Av[2][4];  // [row a/b][4 bf16 pairs of this thread's 8 weights]
#pragma unroll
                for (int rr = 0; rr < 2; rr++) {
                    const uint8_t *p = (rr ? pb : pa) + 8 * sbk;
                    const uint32_t a0 = lds_u32_a2(p), a1 = lds_u32_a2(p + 4);
                    const uint32_t gi = (a0 >> (8 * t)) & 255u;
                    const uint32_t sg = ksigns((a1 >> (7 * t)) & 127u);
                    const uint4 G = gridtab[gi];
                    // byte i of plo/phi carries the sign of weight i (lo) / 4+i (hi) in bit 7
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
                const float2 sc = *reinterpret_cast<const float2 *>(stab + bb * TW + sbk * 16 + g * 2);
#pragma unroll
                for (int nt = 0; nt < NT; nt++) {
                    ffma2(acc[nt][0], acc[nt][1], sc.x, sc.x, T[nt][0], T[nt][1]);
                    ffma2(acc[nt][2], acc[nt][3], sc.y, sc.y, T[nt][2], T[nt][3]);
                }
            }
        }
    }
};

// -------------------------------------------------------------------------
// Lane-per-row Q4_K path for one activation row.  Each consumer warp owns one
// super-block column of the stage; lane r owns tile row r.  The warp first
// quantizes its 256 activation values to int16 with one f32 scale per 32
// (relative error ~2^-16), then every lane dots its row's nibbles (as bytes)
// against them with dp2a into int32, one sum per 32-weight sub-block, and
// applies the block scales once per sub-block:
//     acc += (d sc_j dx_j) * sum_j(q x_q) - (dmin m_j) * (dx_j * sum_j x_q).
// Quantize the warp's 256 activations: xq = int16 values, one f32 scale per
// 32 (xsc[0..7]), dx*sum per 32 (xsc[8..15]) and per 16 (xsc[16..31]).
template <bool F16>
__device__ __forceinline__ void dp_quantize(const uint16_t *xs, uint32_t *xq, float *xsc) {
    const int lane = threadIdx.x & 31, j = lane >> 2;
    {
        const uint4 v = *reinterpret_cast<const uint4 *>(xs + 8 * lane);
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
        const float dx = am * (1.0f / 32767.0f), inv = am > 0.f ? 32767.0f / am : 0.f;
        int qs = 0;
        uint32_t pk[4];
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const int q0 = __float2int_rn(f[2 * e] * inv), q1 = __float2int_rn(f[2 * e + 1] * inv);
            qs += q0 + q1;
            pk[e] = (uint32_t)(q0 & 0xffff) | ((uint32_t)q1 << 16);
        }
        const int q16 = qs + __shfl_xor_sync(0xffffffffu, qs, 1);
        const int q32 = q16 + __shfl_xor_sync(0xffffffffu, q16, 2);
        *reinterpret_cast<uint4 *>(xq + 4 * lane) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        if ((lane & 3) == 0) {
            xsc[j] = dx;
            xsc[8 + j] = dx * (float)q32;
        }
        if ((lane & 1) == 0) xsc[16 + (lane >> 1)] = dx * (float)q16;
    }
    __syncwarp();
}

// Lane-per-row Q4_K in two steps: dp_q4k_load pulls the lane's 144-byte block
// (and the warp's quantized activations) out of the ring, so the stage can be
// released to the producer before dp_q4k_dot does the arithmetic.
struct Q4Regs {
    uint4 h, w[8];
};

__device__ __forceinline__ void dp_q4k_load(const uint8_t *row, Q4Regs &r) {
    r.h = *reinterpret_cast<const uint4 *>(row);
#pragma unroll
    for (int i = 0; i < 8; i++) r.w[i] = *reinterpret_cast<const uint4 *>(row + 16 + 16 * i);
}

__device__ __forceinline__ float dp_q4k_dot(const Q4Regs &r, const uint32_t *xq, const float *xsc) {
    const float d = half_bits_to_float(r.h.x & 0xffffu), dmin = half_bits_to_float(r.h.x >> 16);
    uint32_t sc03, sc47, m03, m47;
    q4k_unpack_scales(r.h.y, r.h.z, r.h.w, sc03, sc47, m03, m47);
    float acc = 0.f;
#pragma unroll
    for (int c = 0; c < 4; c++) {
        const uint4 wa = r.w[2 * c], wb = r.w[2 * c + 1];
        const uint32_t w8[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
        // four independent dp2a chains (two per sub-block) halve the dependent depth
        int sl = 0, sh = 0, sl2 = 0, sh2 = 0;
#pragma unroll
        for (int h4 = 0; h4 < 2; h4++) {
            // x values of sub 2c (k = 64c + 16*h4 .. +15) and sub 2c+1 (+32)
            const uint4 xl0 = *reinterpret_cast<const uint4 *>(xq + 32 * c + 8 * h4);
            const uint4 xl1 = *reinterpret_cast<const uint4 *>(xq + 32 * c + 8 * h4 + 4);
            const uint4 xh0 = *reinterpret_cast<const uint4 *>(xq + 32 * c + 16 + 8 * h4);
            const uint4 xh1 = *reinterpret_cast<const uint4 *>(xq + 32 * c + 16 + 8 * h4 + 4);
            const uint32_t xl[8] = {xl0.x, xl0.y, xl0.z, xl0.w, xl1.x, xl1.y, xl1.z, xl1.w};
            const uint32_t xh[8] = {xh0.x, xh0.y, xh0.z, xh0.w, xh1.x, xh1.y, xh1.z, xh1.w};
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const uint32_t w = w8[4 * h4 + i];
                const int lo = (int)(w & 0x0f0f0f0fu), hi = (int)((w >> 4) & 0x0f0f0f0fu);
                sl = __dp2a_lo((int)xl[2 * i], lo, sl);
                sl2 = __dp2a_hi((int)xl[2 * i + 1], lo, sl2);
                sh = __dp2a_lo((int)xh[2 * i], hi, sh);
                sh2 = __dp2a_hi((int)xh[2 * i + 1], hi, sh2);
            }
        }
        sl += sl2;
        sh += sh2;
        const int j0 = 2 * c, j1 = 2 * c + 1;
        const uint32_t scw = j0 < 4 ? sc03 : sc47, mw = j0 < 4 ? m03 : m47;
        const float sc0 = (float)((scw >> (8 * (j0 & 3))) & 63u), sc1 = (float)((scw >> (8 * (j1 & 3))) & 63u);
        const float m0 = (float)((mw >> (8 * (j0 & 3))) & 63u), m1 = (float)((mw >> (8 * (j1 & 3))) & 63u);
        acc = fmaf(d * sc0 * xsc[j0], (float)sl, acc);
        acc = fmaf(d * sc1 * xsc[j1], (float)sh, acc);
        acc = fmaf(-dmin * m0, xsc[8 + j0], acc);
        acc = fmaf(-dmin * m1, xsc[8 + j1], acc);
    }
    __syncwarp();  // xq is rewritten for the next block
    return acc;
}

// Lane-per-row Q5_K: the Q4_K dot with the fifth bit of every weight OR-ed in
// from the 32 qh bytes (bit j of qh[l] is weight l of sub-block j).
struct Q5Regs {
    uint4 h, qh[2], w[8];
};

__device__ __forceinline__ void dp_q5k_load(const uint8_t *row, Q5Regs &r) {
    r.h = *reinterpret_cast<const uint4 *>(row);
    r.qh[0] = *reinterpret_cast<const uint4 *>(row + 16);
    r.qh[1] = *reinterpret_cast<const uint4 *>(row + 32);
#pragma unroll
    for (int i = 0; i < 8; i++) r.w[i] = *reinterpret_cast<const uint4 *>(row + 48 + 16 * i);
}

__device__ __forceinline__ float dp_q5k_dot(const Q5Regs &r, const uint32_t *xq, const float *xsc) {
    const float d = half_bits_to_float(r.h.x & 0xffffu), dmin = half_bits_to_float(r.h.x >> 16);
    uint32_t sc03, sc47, m03, m47;
    q4k_unpack_scales(r.h.y, r.h.z, r.h.w, sc03, sc47, m03, m47);
    const uint32_t qh8[8] = {r.qh[0].x, r.qh[0].y, r.qh[0].z, r.qh[0].w, r.qh[1].x, r.qh[1].y, r.qh[1].z, r.qh[1].w};
    float acc = 0.f;
#pragma unroll
    for (int c = 0; c < 4; c++) {
        const uint4 wa = r.w[2 * c], wb = r.w[2 * c + 1];
        const uint32_t w8[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
        // four independent dp2a chains (two per sub-block) halve the dependent depth
        int sl = 0, sh = 0, sl2 = 0, sh2 = 0;
#pragma unroll
        for (int h4 = 0; h4 < 2; h4++) {
            const uint4 xl0 = *reinterpret_cast<const uint4 *>(xq + 32 * c + 8 * h4);
            const uint4 xl1 = *reinterpret_cast<const uint4 *>(xq + 32 * c + 8 * h4 + 4);
            const uint4 xh0 = *reinterpret_cast<const uint4 *>(xq + 32 * c + 16 + 8 * h4);
            const uint4 xh1 = *reinterpret_cast<const uint4 *>(xq + 32 * c + 16 + 8 * h4 + 4);
            const uint32_t xl[8] = {xl0.x, xl0.y, xl0.z, xl0.w, xl1.x, xl1.y, xl1.z, xl1.w};
            const uint32_t xh[8] = {xh0.x, xh0.y, xh0.z, xh0.w, xh1.x, xh1.y, xh1.z, xh1.w};
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const uint32_t w = w8[4 * h4 + i], q5 = qh8[4 * h4 + i];
                const int lo = (int)((w & 0x0f0f0f0fu) | (((q5 >> (2 * c)) & 0x01010101u) << 4));
                const int hi = (int)(((w >> 4) & 0x0f0f0f0fu) | (((q5 >> (2 * c + 1)) & 0x01010101u) << 4));
                sl = __dp2a_lo((int)xl[2 * i], lo, sl);
                sl = __dp2a_hi((int)xl[2 * i + 1], lo, sl);
                sh = __dp2a_lo((int)xh[2 * i], hi, sh);
                sh = __dp2a_hi((int)xh[2 * i + 1], hi, sh);
            }
        }
        const int j0 = 2 * c, j1 = 2 * c + 1;
        const uint32_t scw = j0 < 4 ? sc03 : sc47, mw = j0 < 4 ? m03 : m47;
        const float sc0 = (float)((scw >> (8 * (j0 & 3))) & 63u), sc1 = (float)((scw >> (8 * (j1 & 3))) & 63u);
        const float m0 = (float)((mw >> (8 * (j0 & 3))) & 63u), m1 = (float)((mw >> (8 * (j1 & 3))) & 63u);
        acc = fmaf(d * sc0 * xsc[j0], (float)sl, acc);
        acc = fmaf(d * sc1 * xsc[j1], (float)sh, acc);
        acc = fmaf(-dmin * m0, xsc[8 + j0], acc);
        acc = fmaf(-dmin * m1, xsc[8 + j1], acc);
    }
    __syncwarp();  // xq is rewritten for the next block
    return acc;
}

// Lane-per-row Q8_0: a lane takes four consecutive 34-byte ggml blocks (half a
// 272-byte group); int8 quants dot the int16 activations with dp2a and each
// block's fp16 d scales its 32-weight sum.  Blocks are only 2-byte aligned.
__device__ __forceinline__ uint32_t lds_w2(const uint32_t *base, int i, uint32_t sh) {
    return __funnelshift_r(base[i], base[i + 1], sh);
}

struct Q8Regs {
    uint32_t q[4][8];
    float d[4];
};

__device__ __forceinline__ void dp_q80_load(const uint8_t *half_blk, Q8Regs &r) {
#pragma unroll
    for (int s = 0; s < 4; s++) {
        const uint8_t *blk = half_blk + 34 * s;
        r.d[s] = half_bits_to_float(*reinterpret_cast<const uint16_t *>(blk));
        const uintptr_t qb = (uintptr_t)(blk + 2);
        const uint32_t *aw = reinterpret_cast<const uint32_t *>(qb & ~(uintptr_t)3);
        const uint32_t sh = (uint32_t)(qb & 3) * 8;
#pragma unroll
        for (int i = 0; i < 8; i++) r.q[s][i] = lds_w2(aw, i, sh);
    }
}

__device__ __forceinline__ float dp_q80_dot(const Q8Regs &r, int hf, const uint32_t *xq, const float *xsc) {
    float acc = 0.f;
#pragma unroll
    for (int s = 0; s < 4; s++) {
        int sum = 0;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const uint2 xv = *reinterpret_cast<const uint2 *>(xq + 64 * hf + 16 * s + 2 * i);
            sum = __dp2a_lo((int)xv.x, (int)r.q[s][i], sum);
            sum = __dp2a_hi((int)xv.y, (int)r.q[s][i], sum);
        }
        acc = fmaf(r.d[s] * xsc[4 * hf + s], (float)sum, acc);
    }
    __syncwarp();  // xq is rewritten for the next block
    return acc;
}

// Lane-per-row Q6_K: lanes 0-15 / 16-31 of a warp take the two 128-weight
// halves of rows row0..row0+15 of one block.  q6 = ql nibble | qh pair << 4 is
// dotted unsigned with dp2a; the -32 offset is applied as -32 * sum(x) per
// 16-weight sub-block.  Rows are only 2-byte aligned (210-byte blocks), so
// words are assembled from aligned loads with funnel shifts.

struct Q6Regs {
    uint32_t ql[16], qh[8], scw0, scw1;
    float d;
};

__device__ __forceinline__ void dp_q6k_load(const uint8_t *blk, int hf, Q6Regs &r) {
    const uintptr_t ab = (uintptr_t)blk;
    const uint32_t *aw = reinterpret_cast<const uint32_t *>(ab & ~(uintptr_t)3);
    const uint32_t sh = (uint32_t)(ab & 3) * 8;  // 0 or 16
#pragma unroll
    for (int i = 0; i < 16; i++) r.ql[i] = lds_w2(aw, 16 * hf + i, sh);     // bytes 64hf .. 64hf+63
#pragma unroll
    for (int i = 0; i < 8; i++) r.qh[i] = lds_w2(aw, 32 + 8 * hf + i, sh);  // bytes 128+32hf ..
    r.scw0 = lds_w2(aw, 48 + 2 * hf, sh);                                   // int8 scales 8hf..8hf+7
    r.scw1 = lds_w2(aw, 49 + 2 * hf, sh);
    r.d = half_bits_to_float(lds_w2(aw, 52, sh) & 0xffffu);                 // bytes 208-209
}

// Half-block loader for the row-per-lane mapping: 32 lanes read 32 rows at the
// same column, so when the rows' offsets agree (rows at a 16-byte multiple
// stride: every contiguous matrix) the half-block is read with 16-byte loads
// (conflict-free at the ring's row pitch) and realigned with funnel shifts by
// a warp-uniform amount; otherwise the word-by-word loader.
template <int Q>
__device__ __forceinline__ void q6_realign(const uint32_t (&cl)[20], const uint32_t (&ch)[12], uint32_t sh, Q6Regs &r) {
#pragma unroll
    for (int i = 0; i < 16; i++) r.ql[i] = __funnelshift_r(cl[Q + i], cl[Q + i + 1], sh);
#pragma unroll
    for (int i = 0; i < 8; i++) r.qh[i] = __funnelshift_r(ch[Q + i], ch[Q + i + 1], sh);
}

__device__ __forceinline__ void dp_q6k_load_rows(const uint8_t *blk, int hf, Q6Regs &r) {
    const uint32_t o = (uint32_t)(uintptr_t)blk & 15u;
    const uint32_t o0 = __shfl_sync(0xffffffffu, o, 0);
    if (!__all_sync(0xffffffffu, o == o0)) {
        dp_q6k_load(blk, hf, r);
        return;
    }
    const uint4 *bl = reinterpret_cast<const uint4 *>(((uintptr_t)blk + 64 * hf) & ~(uintptr_t)15);
    const uint4 *bh = reinterpret_cast<const uint4 *>(((uintptr_t)blk + 128 + 32 * hf) & ~(uintptr_t)15);
    uint32_t cl[20], ch[12];
#pragma unroll
    for (int i = 0; i < 5; i++) {
        const uint4 v = bl[i];
        cl[4 * i] = v.x, cl[4 * i + 1] = v.y, cl[4 * i + 2] = v.z, cl[4 * i + 3] = v.w;
    }
#pragma unroll
    for (int i = 0; i < 3; i++) {
        const uint4 v = bh[i];
        ch[4 * i] = v.x, ch[4 * i + 1] = v.y, ch[4 * i + 2] = v.z, ch[4 * i + 3] = v.w;
    }
    const uint32_t sh = (o & 3u) * 8u;
    switch (o >> 2) {  // warp-uniform
    case 0: q6_realign<0>(cl, ch, sh, r); break;
    case 1: q6_realign<1>(cl, ch, sh, r); break;
    case 2: q6_realign<2>(cl, ch, sh, r); break;
    default: q6_realign<3>(cl, ch, sh, r); break;
    }
    const uintptr_t ab = (uintptr_t)blk;
    const uint32_t *aw = reinterpret_cast<const uint32_t *>(ab & ~(uintptr_t)3);
    const uint32_t s2 = (uint32_t)(ab & 3) * 8;
    r.scw0 = lds_w2(aw, 48 + 2 * hf, s2);  // int8 scales 8hf..8hf+7
    r.scw1 = lds_w2(aw, 49 + 2 * hf, s2);
    r.d = half_bits_to_float(*reinterpret_cast<const uint16_t *>(blk + 208));
}

__device__ __forceinline__ float dp_q6k_dot(const Q6Regs &r, int hf, const uint32_t *xq, const float *xsc) {
    float acc = 0.f;
#pragma unroll
    for (int s4 = 0; s4 < 4; s4++) {
        const int ns = 4 * (s4 >> 1);
        int sm[2] = {0, 0}, sm2[2] = {0, 0};  // the two 16-weight sub-blocks of this 32-weight group (2 chains each)
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const uint32_t lw = r.ql[8 * (s4 & 1) + i] >> ns;
            const uint32_t hw = s4 == 0 ? (r.qh[i] << 4) : s4 == 1 ? (r.qh[i] << 2) : s4 == 2 ? r.qh[i] : (r.qh[i] >> 2);
            const int q6 = (int)lop_and_or(hw, 0x30303030u, lw & 0x0f0f0f0fu);
            // weights 128hf + 32 s4 + 4i .. +3  <-> x words (64 s4 + 8i)/2 of the block-half
            const uint2 xv = *reinterpret_cast<const uint2 *>(xq + 64 * hf + 16 * s4 + 2 * i);
            sm[i >> 2] = __dp2a_lo((int)xv.x, q6, sm[i >> 2]);
            sm2[i >> 2] = __dp2a_hi((int)xv.y, q6, sm2[i >> 2]);
        }
        sm[0] += sm2[0];
        sm[1] += sm2[1];
        const int g32 = 4 * hf + s4;  // x quantization group of these 32 weights
#pragma unroll
        for (int u = 0; u < 2; u++) {
            const int j = 2 * s4 + u;  // sub-block within the half (scale 8hf + j)
            const uint32_t scw = j < 4 ? r.scw0 : r.scw1;
            const float sc = (float)(int)(int8_t)((scw >> (8 * (j & 3))) & 255u);
            acc = fmaf(r.d * sc, fmaf(xsc[g32], (float)sm[u], -32.f * xsc[16 + 2 * g32 + u]), acc);
        }
    }
    __syncwarp();  // xq is rewritten for the next block
    return acc;
}

// Lane-per-row IQ2_XXS: the lane's 66-byte block (2-byte aligned) is read as
// words with funnel shifts; each group of 8 weights becomes two words of
// signed int8 (grid magnitude bytes, replaced by their negation where the
// sign bit is set) dotted against the int16 activations with dp2a.  Per
// 32-weight sub-block:
//     acc += d (0.5 + ls) / 4 * dx_j * sum_j(signed grid * x_q).
struct IQ2Regs {
    uint32_t q[16];
    float d;
};

__device__ __forceinline__ void dp_iq2_load(const uint8_t *blk, IQ2Regs &r) {
    const uintptr_t ab = (uintptr_t)blk;
    const uint32_t *aw = reinterpret_cast<const uint32_t *>(ab & ~(uintptr_t)3);
    const uint32_t sh = (uint32_t)(ab & 3) * 8;  // 0 or 16
    uint32_t w[17];
#pragma unroll
    for (int i = 0; i < 17; i++) w[i] = aw[i];  // up to 2 bytes past the block: the ring row has slack
    r.d = half_bits_to_float(__funnelshift_r(w[0], w[1], sh) & 0xffffu);
    // qs word j = block bytes 2+4j .. 5+4j
#pragma unroll
    for (int j = 0; j < 16; j++) r.q[j] = sh ? w[j + 1] : __funnelshift_r(w[j], w[j + 1], 16);
}

// Lane-per-row IQ2_XXS against R activation rows (row t's int16 table of
// dp_quantize at xq + 160 t, its scales at xsc + 160 t).  Each group of 8 weights is decoded
// once for all rows: sign bit i of the group lands in bit 7 of byte i
// (multiply by 0x10204080 spreads a nibble's bits to bytes), a byte permute
// replicates it into a 0x00 / 0xff mask, and the mask selects between the
// grid bytes g and their negations 0x01010100 - g (bytewise 256 - g: no
// borrows, as 1 <= g < 128).
template <int R>
__device__ __forceinline__ void dp_iq2_dot_r(const IQ2Regs &r, const uint32_t *xq, const float *xsc, const uint2 *grid,
                                            float *acc) {
#pragma unroll
    for (int sb = 0; sb < 8; sb++) {
        const uint32_t a0 = r.q[2 * sb], a1 = r.q[2 * sb + 1];
        int sum[R];
#pragma unroll
        for (int t = 0; t < R; t++) sum[t] = 0;
#pragma unroll
        for (int l = 0; l < 4; l++) {
            const uint2 g = grid[(a0 >> (8 * l)) & 255u];
            const uint32_t s7 = (a1 >> (7 * l)) & 127u;
            const uint32_t nlo = s7 & 15u, nhi = (s7 >> 4) | ((__popc(s7) & 1u) << 3);
            const uint32_t mlo = prmt(nlo * 0x10204080u, 0u, 0xBA98u), mhi = prmt(nhi * 0x10204080u, 0u, 0xBA98u);
            const int s0 = (int)((g.x & ~mlo) | ((0x01010100u - g.x) & mlo));
            const int s1 = (int)((g.y & ~mhi) | ((0x01010100u - g.y) & mhi));
#pragma unroll
            for (int t = 0; t < R; t++) {
                const uint4 xv = *reinterpret_cast<const uint4 *>(xq + 160 * t + 16 * sb + 4 * l);
                sum[t] = __dp2a_lo((int)xv.x, s0, sum[t]);
                sum[t] = __dp2a_hi((int)xv.y, s0, sum[t]);
                sum[t] = __dp2a_lo((int)xv.z, s1, sum[t]);
                sum[t] = __dp2a_hi((int)xv.w, s1, sum[t]);
            }
        }
        const float db = r.d * (0.5f + (float)(a1 >> 28)) * 0.25f;
#pragma unroll
        for (int t = 0; t < R; t++) acc[t] = fmaf(db * xsc[160 * t + sb], (float)sum[t], acc[t]);
    }
    __syncwarp();  // xq is rewritten for the next block
}

// The same dot read straight from the ring stage (the caller releases the
// stage afterwards), with the sub-block loop kept rolled: a kernel that holds
// all four row counts then stays within the instruction cache (the unrolled,
// register-held form is used for one row).  The 66-byte block is 2-byte
// aligned; qs word j is bytes 2 + 4j .. 5 + 4j.
template <int R>
__device__ __forceinline__ void dp_iq2_dot_smem(const uint8_t *blk, const uint32_t *xq, const float *xsc,
                                                const uint2 *grid, float *acc) {
    const uintptr_t ab = (uintptr_t)blk;
    const uint32_t *aw = reinterpret_cast<const uint32_t *>(ab & ~(uintptr_t)3);
    const uint32_t sh = (uint32_t)(ab & 3) * 8;  // 0 or 16
    const float dq = half_bits_to_float(__funnelshift_r(aw[0], aw[1], sh) & 0xffffu) * 0.25f;
    const uint32_t *bw = aw + (sh ? 1 : 0);
    const uint32_t s2 = 16u - sh;
#pragma unroll 1
    for (int sb = 0; sb < 8; sb++) {
        const uint32_t w0 = bw[2 * sb], w1 = bw[2 * sb + 1], w2 = bw[2 * sb + 2];
        const uint32_t a0 = __funnelshift_r(w0, w1, s2), a1 = __funnelshift_r(w1, w2, s2);
        int sum[R];
#pragma unroll
        for (int t = 0; t < R; t++) sum[t] = 0;
#pragma unroll
        for (int l = 0; l < 4; l++) {
            const uint2 g = grid[(a0 >> (8 * l)) & 255u];
            const uint32_t s7 = (a1 >> (7 * l)) & 127u;
            const uint32_t nlo = s7 & 15u, nhi = (s7 >> 4) | ((__popc(s7) & 1u) << 3);
            const uint32_t mlo = prmt(nlo * 0x10204080u, 0u, 0xBA98u), mhi = prmt(nhi * 0x10204080u, 0u, 0xBA98u);
            const int s0 = (int)((g.x & ~mlo) | ((0x01010100u - g.x) & mlo));
            const int s1 = (int)((g.y & ~mhi) | ((0x01010100u - g.y) & mhi));
#pragma unroll
            for (int t = 0; t < R; t++) {
                const uint4 xv = *reinterpret_cast<const uint4 *>(xq + 160 * t + 16 * sb + 4 * l);
                sum[t] = __dp2a_lo((int)xv.x, s0, sum[t]);
                sum[t] = __dp2a_hi((int)xv.y, s0, sum[t]);
                sum[t] = __dp2a_lo((int)xv.z, s1, sum[t]);
                sum[t] = __dp2a_hi((int)xv.w, s1, sum[t]);
            }
        }
        const float db = dq * (0.5f + (float)(a1 >> 28));
#pragma unroll
        for (int t = 0; t < R; t++) acc[t] = fmaf(db * xsc[160 * t + sb], (float)sum[t], acc[t]);
    }
    __syncwarp();  // xq is rewritten for the next block
}

// Lane-per-row IQ3_XXS: as IQ2_XXS with one grid byte index per 4 weights.
// The 98-byte block (2-byte aligned) is read as 25 words: 16 words of grid
// indices then 8 words of (four 7-bit sign indices, ls << 28), one per
// 32-weight sub-block.  Per sub-block:
//     acc += d (0.5 + ls) / 2 * dx_j * sum_j(signed grid * x_q).
struct IQ3Regs {
    uint32_t q[24];
    float d;
};

__device__ __forceinline__ void dp_iq3_load(const uint8_t *blk, IQ3Regs &r) {
    const uintptr_t ab = (uintptr_t)blk;
    const uint32_t *aw = reinterpret_cast<const uint32_t *>(ab & ~(uintptr_t)3);
    const uint32_t sh = (uint32_t)(ab & 3) * 8;  // 0 or 16
    uint32_t w[25];
#pragma unroll
    for (int i = 0; i < 25; i++) w[i] = aw[i];  // up to 2 bytes past the block: the ring row has slack
    r.d = half_bits_to_float(__funnelshift_r(w[0], w[1], sh) & 0xffffu);
#pragma unroll
    for (int j = 0; j < 24; j++) r.q[j] = sh ? w[j + 1] : __funnelshift_r(w[j], w[j + 1], 16);
}

__device__ __forceinline__ float dp_iq3_dot(const IQ3Regs &r, const uint32_t *xq, const float *xsc,
                                           const uint32_t *grid) {
    float acc = 0.f;
#pragma unroll
    for (int sb = 0; sb < 8; sb++) {
        const uint32_t aux = r.q[16 + sb];
        int sum = 0;
#pragma unroll
        for (int l = 0; l < 4; l++) {
            const uint32_t gw = r.q[2 * sb + (l >> 1)] >> (16 * (l & 1));
            const uint32_t g0 = grid[gw & 255u], g1 = grid[(gw >> 8) & 255u];
            const uint32_t sg = ksigns((aux >> (7 * l)) & 127u);
            const uint32_t f0 = ((sg & 15u) * 0x00204081u) & 0x01010101u, f1 = ((sg >> 4) * 0x00204081u) & 0x01010101u;
            const int s0 = (int)((g0 ^ (f0 * 0xffu)) + f0), s1 = (int)((g1 ^ (f1 * 0xffu)) + f1);
            const uint4 xv = *reinterpret_cast<const uint4 *>(xq + 16 * sb + 4 * l);
            sum = __dp2a_lo((int)xv.x, s0, sum);
            sum = __dp2a_hi((int)xv.y, s0, sum);
            sum = __dp2a_lo((int)xv.z, s1, sum);
            sum = __dp2a_hi((int)xv.w, s1, sum);
        }
        acc = fmaf(r.d * (0.5f + (float)(aux >> 28)) * 0.5f * xsc[sb], (float)sum, acc);
    }
    __syncwarp();  // xq is rewritten for the next block
    return acc;
}

// Lane-per-row IQ4_XS: every nibble selects one of sixteen signed bytes (the
// IQ4_NL values, held in four registers) by two byte permutes (low three bits)
// and a per-byte select on bit 3; the signed bytes dot the int16 activations
// with dp2a.  Blocks are 136 bytes, so rows at 8-byte aligned addresses keep
// every block 8-byte aligned (the entry points require it).  Per sub-block:
//     acc += d (ls - 32) * dx_j * sum_j(value[q] * x_q).
struct IQ4Regs {
    uint2 h;
    uint32_t q[32];
};

__device__ __forceinline__ void dp_iq4xs_load(const uint8_t *blk, IQ4Regs &r) {
    r.h = *reinterpret_cast<const uint2 *>(blk);
#pragma unroll
    for (int i = 0; i < 16; i++) {
        const uint2 v = *reinterpret_cast<const uint2 *>(blk + 8 + 8 * i);
        r.q[2 * i] = v.x;
        r.q[2 * i + 1] = v.y;
    }
}

// four nibbles (one per byte, bits 0-3) -> four signed table bytes
__device__ __forceinline__ int iq4_lookup4(uint32_t n, const uint32_t (&tv)[4]) {
    const uint32_t t = n & 0x07070707u;
    const uint32_t sel = prmt(t | (t >> 4), 0, 0x0020);  // nibble k = low 3 bits of byte k
    const uint32_t lo = prmt(tv[0], tv[1], sel), hi = prmt(tv[2], tv[3], sel);
    const uint32_t m = ((n >> 3) & 0x01010101u) * 0xffu;
    return (int)((lo & ~m) | (hi & m));
}

__device__ __forceinline__ float dp_iq4xs_dot(const IQ4Regs &r, const uint32_t *xq, const float *xsc) {
    const uint32_t *tw = reinterpret_cast<const uint32_t *>(c_iq4nl_values);
    const uint32_t tv[4] = {tw[0], tw[1], tw[2], tw[3]};
    const float d = half_bits_to_float(r.h.x & 0xffffu);
    const uint32_t sh = r.h.x >> 16, sl = r.h.y;
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        int sum = 0;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t w = r.q[4 * j + i];
            const int vlo = iq4_lookup4(w & 0x0f0f0f0fu, tv), vhi = iq4_lookup4((w >> 4) & 0x0f0f0f0fu, tv);
            const uint2 xl = *reinterpret_cast<const uint2 *>(xq + 16 * j + 2 * i);
            const uint2 xh = *reinterpret_cast<const uint2 *>(xq + 16 * j + 8 + 2 * i);
            sum = __dp2a_lo((int)xl.x, vlo, sum);
            sum = __dp2a_hi((int)xl.y, vlo, sum);
            sum = __dp2a_lo((int)xh.x, vhi, sum);
            sum = __dp2a_hi((int)xh.y, vhi, sum);
        }
        const int ls = (int)(((sl >> (4 * j)) & 15u) | (((sh >> (2 * j)) & 3u) << 4));
        acc = fmaf(d * (float)(ls - 32) * xsc[j], (float)sum, acc);
    }
    __syncwarp();  // xq is rewritten for the next block
    return acc;
}

// Lane-per-row legacy 32-weight codecs (Q4_0, Q4_1, Q5_0, Q5_1, IQ4_NL): a
// lane takes a whole group of eight blocks (144-176 bytes, 2-byte aligned),
// as Q4_K takes its 144-byte block, so stage rows are 8 groups long; Q5_1's
// 192-byte groups would not fit two CTAs per SM that way, so a Q5_1 lane takes
// half a group (NB = 4 blocks, warp = (group column, half)) as Q8_0 does.  Nibble
// j < 16 of a block is the low half of byte j, j >= 16 the high half of byte
// j - 16; Q5 fifth bits are OR-ed in from the block's u32.  Unsigned values
// are dotted against the int16 activations, per block g of 32 weights:
//     Q4_0 / Q5_0: acc += d (dx S_g - OFF dx sum_g(x_q))
//     Q4_1 / Q5_1: acc += d dx S_g + m dx sum_g(x_q)
//     IQ4_NL: values mapped to the sixteen signed bytes first, acc += d dx S_g.
template <int C> constexpr int LEG_NB = C == Q5_1 ? 4 : 8;  // blocks per lane
template <int C> struct LegRegs {
    static constexpr int NB = LEG_NB<C>;
    uint32_t q[NB][4];
    uint32_t qh[Legacy<C>::HASH ? NB : 1];
    float d[NB], m[Legacy<C>::HASM ? NB : 1];
};

template <int C> __device__ __forceinline__ void dp_leg_load(const uint8_t *grp, LegRegs<C> &r) {
    using LG = Legacy<C>;
#pragma unroll
    for (int s = 0; s < LEG_NB<C>; s++) {
        const uint8_t *blk = grp + LG::BB * s;
        if constexpr (LG::MX)
            r.d[s] = e8m0_half(blk[0]);
        else
            r.d[s] = half_bits_to_float(*reinterpret_cast<const uint16_t *>(blk));
        if constexpr (LG::HASM) r.m[s] = half_bits_to_float(*reinterpret_cast<const uint16_t *>(blk + 2));
        const uintptr_t hb = (uintptr_t)(blk + (LG::HASH ? LG::HOFF : LG::QOFF));
        const uint32_t *aw = reinterpret_cast<const uint32_t *>(hb & ~(uintptr_t)3);
        const uint32_t sh = (uint32_t)(hb & 3) * 8;
        if constexpr (LG::HASH) {
            r.qh[s] = lds_w2(aw, 0, sh);
#pragma unroll
            for (int i = 0; i < 4; i++) r.q[s][i] = lds_w2(aw, 1 + i, sh);
        } else {
#pragma unroll
            for (int i = 0; i < 4; i++) r.q[s][i] = lds_w2(aw, i, sh);
        }
    }
}

// four bits (bits 0-3 of v) -> bit 4 of each byte
__device__ __forceinline__ uint32_t bits_to_b4(uint32_t v) { return ((v & 15u) * 0x00204081u & 0x01010101u) << 4; }

// g0: 32-weight group index of the lane's first block (0, or 4 for the second half)
template <int C>
__device__ __forceinline__ float dp_leg_dot(const LegRegs<C> &r, const uint32_t *xq, const float *xsc, int g0) {
    using LG = Legacy<C>;
    uint32_t tv[4] = {0u, 0u, 0u, 0u};
    if constexpr (LG::NL) {
        const uint32_t *tw = reinterpret_cast<const uint32_t *>(LG::MX ? c_mxfp4_values : c_iq4nl_values);
        tv[0] = tw[0], tv[1] = tw[1], tv[2] = tw[2], tv[3] = tw[3];
    }
    float acc = 0.f;
#pragma unroll
    for (int s = 0; s < LEG_NB<C>; s++) {
        const int g = g0 + s;
        int sum = 0;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t w = r.q[s][i];
            uint32_t lo = w & 0x0f0f0f0fu, hi = (w >> 4) & 0x0f0f0f0fu;
            if constexpr (LG::HASH) {
                lo |= bits_to_b4(r.qh[s] >> (4 * i));
                hi |= bits_to_b4(r.qh[s] >> (16 + 4 * i));
            }
            if constexpr (LG::NL) {
                lo = (uint32_t)iq4_lookup4(lo, tv);
                hi = (uint32_t)iq4_lookup4(hi, tv);
            }
            const uint2 xl = *reinterpret_cast<const uint2 *>(xq + 16 * g + 2 * i);
            const uint2 xh = *reinterpret_cast<const uint2 *>(xq + 16 * g + 8 + 2 * i);
            sum = __dp2a_lo((int)xl.x, (int)lo, sum);
            sum = __dp2a_hi((int)xl.y, (int)lo, sum);
            sum = __dp2a_lo((int)xh.x, (int)hi, sum);
            sum = __dp2a_hi((int)xh.y, (int)hi, sum);
        }
        if constexpr (LG::NL)
            acc = fmaf(r.d[s] * xsc[g], (float)sum, acc);
        else if constexpr (LG::HASM)
            acc = fmaf(r.d[s] * xsc[g], (float)sum, fmaf(r.m[s], xsc[8 + g], acc));
        else
            acc = fmaf(r.d[s], fmaf(xsc[g], (float)sum, -(float)LG::OFF * xsc[8 + g]), acc);
    }
    __syncwarp();  // xq is rewritten for the next block
    return acc;
}

// Lane-per-row Q2_K / Q3_K: a lane takes a whole super-block.  Weight
// 128h + 32k + l is bits 2k of quant byte 32h + l, so quant word 8h + i
// shifted by 2k gives weights 128h + 32k + 4i .. +3 (sub-block 8h + 2k + i/4).
// The unsigned values (Q2_K: q in 0..3; Q3_K: q + 4 * hbit in 0..7) are dotted
// against the int16 activations; per 16-weight sub-block j:
//     Q2_K: acc += d sc_j dx S_j - dmin m_j dx sum16_j(x_q)
//     Q3_K: acc += d (s_j - 32) (dx S_j - 4 dx sum16_j(x_q)).
struct Q2Regs {
    uint32_t sc[4], q[16];
    float d, dmin;
};

__device__ __forceinline__ void dp_q2k_load(const uint8_t *blk, Q2Regs &r) {  // 4-byte aligned
    const uint32_t *w = reinterpret_cast<const uint32_t *>(blk);
#pragma unroll
    for (int i = 0; i < 4; i++) r.sc[i] = w[i];
#pragma unroll
    for (int i = 0; i < 16; i++) r.q[i] = w[4 + i];
    r.d = half_bits_to_float(w[20] & 0xffffu);
    r.dmin = half_bits_to_float(w[20] >> 16);
}

__device__ __forceinline__ float dp_q2k_dot(const Q2Regs &r, const uint32_t *xq, const float *xsc) {
    float acc = 0.f;
#pragma unroll
    for (int h = 0; h < 2; h++)
#pragma unroll
        for (int k = 0; k < 4; k++) {
            int s0 = 0, s1 = 0;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int q = (int)((r.q[8 * h + i] >> (2 * k)) & 0x03030303u);
                const uint2 xv = *reinterpret_cast<const uint2 *>(xq + 64 * h + 16 * k + 2 * i);
                int &sm = i < 4 ? s0 : s1;
                sm = __dp2a_lo((int)xv.x, q, sm);
                sm = __dp2a_hi((int)xv.y, q, sm);
            }
            const int g = 4 * h + k, j = 2 * g;  // 32-weight group, first 16-weight sub-block
            const uint32_t scw = r.sc[j >> 2];
            const float sc0 = (float)((scw >> (8 * (j & 3))) & 15u), m0 = (float)((scw >> (8 * (j & 3) + 4)) & 15u);
            const float sc1 = (float)((scw >> (8 * (j & 3) + 8)) & 15u), m1 = (float)((scw >> (8 * (j & 3) + 12)) & 15u);
            acc = fmaf(r.d * xsc[g], sc0 * (float)s0 + sc1 * (float)s1, acc);
            acc = fmaf(-r.dmin, fmaf(m0, xsc[16 + j], m1 * xsc[17 + j]), acc);
        }
    __syncwarp();  // xq is rewritten for the next block
    return acc;
}

// Lane-per-row IQ2_XS / IQ2_S / IQ3_S: as IQ2_XXS, the lane's block (2-byte
// aligned) is realigned into IQS_NW words of block bytes 2 + 4j; each group of
// 8 weights becomes two words of signed grid bytes dotted against the int16
// activations, and each scale is applied once per 16 (IQ2_XS / IQ2_S) or 32
// (IQ3_S) weights.  Word map (block byte 2 + 4j):
//   IQ2_XS: j 0-15 u16 entries, 16-17 scales
//   IQ2_S:  j 0-7 index low bytes, 8-15 sign bytes, 16-17 index high bits, 18-19 scales
//   IQ3_S:  j 0-15 index low bytes, 16-17 index high bits, 18-25 sign bytes, 26 scales
template <int C> constexpr int IQS_NW = C == IQ3_S ? 27 : C == IQ2_S ? 20 : C == IQ1_S ? 12 : 18;
template <int C> struct IQSRegs {
    uint32_t q[IQS_NW<C>];
    float d;
};

template <int C> __device__ __forceinline__ void dp_iqs_load(const uint8_t *blk, IQSRegs<C> &r) {
    constexpr int NW = IQS_NW<C>;
    const uintptr_t ab = (uintptr_t)blk;
    const uint32_t *aw = reinterpret_cast<const uint32_t *>(ab & ~(uintptr_t)3);
    const uint32_t sh = (uint32_t)(ab & 3) * 8;  // 0 or 16
    uint32_t w[NW + 1];
#pragma unroll
    for (int i = 0; i < NW + 1; i++) w[i] = aw[i];  // up to 2 bytes past the block: the ring row has slack
    r.d = half_bits_to_float(__funnelshift_r(w[0], w[1], sh) & 0xffffu);
#pragma unroll
    for (int j = 0; j < NW; j++) r.q[j] = sh ? w[j + 1] : __funnelshift_r(w[j], w[j + 1], 16);
}

// signed grid bytes of 4 weights: magnitudes g (each < 128), sign bits sb (bits 0-3)
__device__ __forceinline__ int signed4(uint32_t g, uint32_t sb) {
    const uint32_t f = ((sb & 15u) * 0x00204081u) & 0x01010101u;
    return (int)((g ^ (f * 0xffu)) + f);
}

template <int C>
__device__ __forceinline__ float dp_iqs_dot(const IQSRegs<C> &r, const uint32_t *xq, const float *xsc,
                                           const uint2 *grid8, const uint32_t *grid4) {
    float acc = 0.f;
#pragma unroll
    for (int g = 0; g < 8; g++) {  // 32-weight group
        int sm[2] = {0, 0};
#pragma unroll
        for (int l = 0; l < 4; l++) {  // 8 weights
            int s0, s1;
            if constexpr (C == IQ3_S) {
                const int e0 = 8 * g + 2 * l;  // two 4-weight entries
                const uint32_t lo = r.q[e0 >> 2] >> (8 * (e0 & 3));
                const uint32_t hb = r.q[16 + (g >> 2)] >> (8 * (g & 3) + 2 * l);
                const uint32_t g0 = grid4[(lo & 255u) | ((hb & 1u) << 8)];
                const uint32_t g1 = grid4[((lo >> 8) & 255u) | ((hb & 2u) << 7)];
                const uint32_t sbyte = (r.q[18 + g] >> (8 * l)) & 255u;
                s0 = signed4(g0, sbyte);
                s1 = signed4(g1, sbyte >> 4);
            } else {
                const int e = 4 * g + l;  // 8-weight entry
                uint32_t idx, sbyte;
                if constexpr (C == IQ2_XS) {
                    const uint32_t v = (r.q[e >> 1] >> (16 * (e & 1))) & 0xffffu;
                    idx = v & 511u;
                    sbyte = ksigns(v >> 9);
                } else {
                    idx = ((r.q[e >> 2] >> (8 * (e & 3))) & 255u) | (((r.q[16 + (e >> 4)] >> (2 * (e & 15))) & 3u) << 8);
                    sbyte = (r.q[8 + (e >> 2)] >> (8 * (e & 3))) & 255u;
                }
                const uint2 gv = grid8[idx];
                s0 = signed4(gv.x, sbyte);
                s1 = signed4(gv.y, sbyte >> 4);
            }
            const uint4 xv = *reinterpret_cast<const uint4 *>(xq + 16 * g + 4 * l);
            int &sum = sm[C == IQ3_S ? 0 : (l >> 1)];
            sum = __dp2a_lo((int)xv.x, s0, sum);
            sum = __dp2a_hi((int)xv.y, s0, sum);
            sum = __dp2a_lo((int)xv.z, s1, sum);
            sum = __dp2a_hi((int)xv.w, s1, sum);
        }
        if constexpr (C == IQ3_S) {
            const int s = (int)((r.q[26] >> (4 * g)) & 15u);
            acc = fmaf(r.d * (float)(1 + 2 * s) * xsc[g], (float)sm[0], acc);
        } else {
            const uint32_t scw = r.q[(C == IQ2_XS ? 16 : 18) + (g >> 2)];  // byte g: two 4-bit scales
            const float s0 = (float)((scw >> (8 * (g & 3))) & 15u), s1 = (float)((scw >> (8 * (g & 3) + 4)) & 15u);
            acc = fmaf(r.d * 0.25f * xsc[g], (0.5f + s0) * (float)sm[0] + (0.5f + s1) * (float)sm[1], acc);
        }
    }
    __syncwarp();  // xq is rewritten for the next block
    return acc;
}

// Lane-per-row IQ1_S / IQ1_M: grid values g in {-1, 0, 1} plus a delta of
// +-1/8 become the integers 8g +- 1 (per byte: (g << 3) masked, then a
// carry-free byte add of +-1), dotted against the int16 activations; the 1/8
// rides on the scale d (2s + 1) / 8.  IQ1_S is realigned at block byte 2
// (IQS_NW = 12 words: index bytes, then the 8 u16), IQ1_M at byte 0 (14 words:
// index bytes, nibbles, scales).
struct IQ1MRegs {
    uint32_t q[14];
};

__device__ __forceinline__ void dp_iq1m_load(const uint8_t *blk, IQ1MRegs &r) {
    const uintptr_t ab = (uintptr_t)blk;
    const uint32_t *aw = reinterpret_cast<const uint32_t *>(ab & ~(uintptr_t)3);
    const uint32_t sh = (uint32_t)(ab & 3) * 8;
    uint32_t w[15];
#pragma unroll
    for (int i = 0; i < 15; i++) w[i] = aw[i];  // up to 4 bytes past the block: the ring row has slack
#pragma unroll
    for (int j = 0; j < 14; j++) r.q[j] = __funnelshift_r(w[j], w[j + 1], sh);
}

__device__ __forceinline__ int iq1_vals(uint32_t g, bool neg) {
    return (int)__vadd4((g << 3) & 0xf8f8f8f8u, neg ? 0xffffffffu : 0x01010101u);
}

template <int C>
__device__ __forceinline__ float dp_iq1_dot(const uint32_t *q, float d_iq1s, const uint32_t *xq, const float *xsc,
                                           const uint2 *grid8) {
    float acc = 0.f, d = d_iq1s;
    if constexpr (C == IQ1_M)
        d = half_bits_to_float((q[12] >> 12 & 0xfu) | ((q[12] >> 24) & 0xf0u) | ((q[13] >> 4) & 0xf00u) |
                               ((q[13] >> 16) & 0xf000u));
#pragma unroll
    for (int g = 0; g < 8; g++) {  // 32-weight group
        int sm[2] = {0, 0};
        uint32_t qh = 0;
        if constexpr (C == IQ1_S) qh = (q[8 + (g >> 1)] >> (16 * (g & 1))) & 0xffffu;
#pragma unroll
        for (int l = 0; l < 4; l++) {
            const int e = 4 * g + l;
            uint32_t idx;
            bool neg;
            if constexpr (C == IQ1_S) {
                idx = ((q[e >> 2] >> (8 * (e & 3))) & 255u) | (((qh >> (3 * l)) & 7u) << 8);
                neg = (qh & 0x8000u) != 0;
            } else {
                const uint32_t nib = (q[8 + (e >> 3)] >> (4 * (e & 7))) & 15u;
                idx = ((q[e >> 2] >> (8 * (e & 3))) & 255u) | ((nib & 7u) << 8);
                neg = (nib & 8u) != 0;
            }
            const uint2 gv = grid8[idx];
            const int s0 = iq1_vals(gv.x, neg), s1 = iq1_vals(gv.y, neg);
            const uint4 xv = *reinterpret_cast<const uint4 *>(xq + 16 * g + 4 * l);
            int &sum = sm[C == IQ1_S ? 0 : (l >> 1)];
            sum = __dp2a_lo((int)xv.x, s0, sum);
            sum = __dp2a_hi((int)xv.y, s0, sum);
            sum = __dp2a_lo((int)xv.z, s1, sum);
            sum = __dp2a_hi((int)xv.w, s1, sum);
        }
        if constexpr (C == IQ1_S) {
            acc = fmaf(d * 0.125f * (float)(2 * ((qh >> 12) & 7) + 1) * xsc[g], (float)sm[0], acc);
        } else {
#pragma unroll
            for (int u = 0; u < 2; u++) {
                const int k = 2 * g + u;  // 16-weight sub-block: u16 k >> 2 of the scales
                const uint32_t sk = (q[12 + (k >> 3)] >> (16 * ((k >> 2) & 1))) & 0xffffu;
                acc = fmaf(d * 0.125f * (float)(2 * ((sk >> (3 * (k & 3))) & 7) + 1) * xsc[g], (float)sm[u], acc);
            }
        }
    }
    __syncwarp();  // xq is rewritten for the next block
    return acc;
}

// Lane-per-row TQ2_0: Q2_K's quant layout with one fp16 d per block (66 bytes,
// 2-byte aligned); per 32-weight group g: acc += d (dx S_g - dx sum_g(x_q)).
struct TQ2Regs {
    uint32_t q[16];
    float d;
};

__device__ __forceinline__ void dp_tq2_load(const uint8_t *blk, TQ2Regs &r) {
    const uintptr_t ab = (uintptr_t)blk;
    const uint32_t *aw = reinterpret_cast<const uint32_t *>(ab & ~(uintptr_t)3);
    const uint32_t sh = (uint32_t)(ab & 3) * 8;  // 0 or 16
    uint32_t w[18];
#pragma unroll
    for (int i = 0; i < 18; i++) w[i] = aw[i];  // up to 6 bytes past the block: the ring row has slack
#pragma unroll
    for (int i = 0; i < 16; i++) r.q[i] = __funnelshift_r(w[i], w[i + 1], sh);
    r.d = half_bits_to_float(__funnelshift_r(w[16], w[17], sh) & 0xffffu);
}

__device__ __forceinline__ float dp_tq2_dot(const TQ2Regs &r, const uint32_t *xq, const float *xsc) {
    float acc = 0.f;
#pragma unroll
    for (int h = 0; h < 2; h++)
#pragma unroll
        for (int k = 0; k < 4; k++) {
            int sum = 0;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int q = (int)((r.q[8 * h + i] >> (2 * k)) & 0x03030303u);
                const uint2 xv = *reinterpret_cast<const uint2 *>(xq + 64 * h + 16 * k + 2 * i);
                sum = __dp2a_lo((int)xv.x, q, sum);
                sum = __dp2a_hi((int)xv.y, q, sum);
            }
            const int g = 4 * h + k;
            acc = fmaf(xsc[g], (float)sum, acc - xsc[8 + g]);
        }
    __syncwarp();  // xq is rewritten for the next block
    return r.d * acc;
}

// Lane-per-row TQ1_0: four base-3 digits at a time.  For a word of four
// bytes and a power m = 3^k, the even and odd bytes sit in 16-bit lanes, so
// (v * m) mod 256 and then ((.) * 3) >> 8 run per lane without carries; the
// digits t in {0, 1, 2} are dotted against the int16 activations and the -1
// rides on the per-32 activation sums.  Digit position k of bytes 0-31 is the
// 32-weight group k; of bytes 32-47 half of group 5 + k/2; bytes 48-51 the
// second half of group 7.
struct TQ1Regs {
    uint32_t q[13];
    float d;
};

__device__ __forceinline__ void dp_tq1_load(const uint8_t *blk, TQ1Regs &r) {
    const uintptr_t ab = (uintptr_t)blk;
    const uint32_t *aw = reinterpret_cast<const uint32_t *>(ab & ~(uintptr_t)3);
    const uint32_t sh = (uint32_t)(ab & 3) * 8;  // 0 or 16
    uint32_t w[15];
#pragma unroll
    for (int i = 0; i < 15; i++) w[i] = aw[i];  // up to 6 bytes past the block: the ring row has slack
#pragma unroll
    for (int i = 0; i < 13; i++) r.q[i] = __funnelshift_r(w[i], w[i + 1], sh);
    r.d = half_bits_to_float(__funnelshift_r(w[13], w[14], sh) & 0xffffu);
}

__device__ __forceinline__ int tq1_digits(uint32_t w, uint32_t m) {
    const uint32_t lo = ((w & 0x00ff00ffu) * m) & 0x00ff00ffu, hi = (((w >> 8) & 0x00ff00ffu) * m) & 0x00ff00ffu;
    return (int)((((lo * 3u) >> 8) & 0x00030003u) | ((((hi * 3u) >> 8) & 0x00030003u) << 8));
}

__device__ __forceinline__ float dp_tq1_dot(const TQ1Regs &r, const uint32_t *xq, const float *xsc) {
    int S[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
    for (int k = 0; k < 5; k++) {
        const uint32_t m = k == 0 ? 1u : k == 1 ? 3u : k == 2 ? 9u : k == 3 ? 27u : 81u;
#pragma unroll
        for (int i = 0; i < 8; i++) {  // bytes 4i .. 4i + 3: weights 32k + 4i .. +3
            const int t = tq1_digits(r.q[i], m);
            const uint2 xv = *reinterpret_cast<const uint2 *>(xq + 16 * k + 2 * i);
            S[k] = __dp2a_lo((int)xv.x, t, S[k]);
            S[k] = __dp2a_hi((int)xv.y, t, S[k]);
        }
#pragma unroll
        for (int i = 0; i < 4; i++) {  // bytes 32 + 4i .. : weights 160 + 16k + 4i .. +3
            const int t = tq1_digits(r.q[8 + i], m);
            const uint2 xv = *reinterpret_cast<const uint2 *>(xq + 80 + 8 * k + 2 * i);
            int &s = S[5 + (k >> 1)];
            s = __dp2a_lo((int)xv.x, t, s);
            s = __dp2a_hi((int)xv.y, t, s);
        }
        if (k < 4) {  // bytes 48 .. 51: weights 240 + 4k .. +3
            const int t = tq1_digits(r.q[12], m);
            const uint2 xv = *reinterpret_cast<const uint2 *>(xq + 120 + 2 * k);
            S[7] = __dp2a_lo((int)xv.x, t, S[7]);
            S[7] = __dp2a_hi((int)xv.y, t, S[7]);
        }
    }
    float acc = 0.f;
#pragma unroll
    for (int g = 0; g < 8; g++) acc = fmaf(xsc[g], (float)S[g], acc - xsc[8 + g]);
    __syncwarp();  // xq is rewritten for the next block
    return r.d * acc;
}

// Lane-per-row NVFP4: a lane takes a whole 144-byte group (four 36-byte
// blocks, realigned into 36 words: block s = word 9s of scales, then 8 words
// of nibbles); nibbles map to the doubled e2m1 bytes by two byte permutes and
// a select (as IQ4_NL), each 16-weight sub-block J is one dot and one scale:
//     acc += ue4m3(s_J)/2 * dx_(J/2) * S_J.
struct NVRegs {
    uint32_t q[36];
};

__device__ __forceinline__ void dp_nv_load(const uint8_t *grp, NVRegs &r) {
    const uintptr_t ab = (uintptr_t)grp;
    const uint32_t *aw = reinterpret_cast<const uint32_t *>(ab & ~(uintptr_t)3);
    const uint32_t sh = (uint32_t)(ab & 3) * 8;
    uint32_t w[37];
#pragma unroll
    for (int i = 0; i < 37; i++) w[i] = aw[i];  // up to 4 bytes past the group: the ring row has slack
#pragma unroll
    for (int j = 0; j < 36; j++) r.q[j] = __funnelshift_r(w[j], w[j + 1], sh);
}

__device__ __forceinline__ float dp_nv_dot(const NVRegs &r, const uint32_t *xq, const float *xsc) {
    const uint32_t *tw = reinterpret_cast<const uint32_t *>(c_mxfp4_values);
    const uint32_t tv[4] = {tw[0], tw[1], tw[2], tw[3]};
    float acc = 0.f;
#pragma unroll
    for (int s = 0; s < 4; s++)
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int J = 4 * s + j;  // 16-weight sub-block of the 256
            int sum = 0;
#pragma unroll
            for (int u = 0; u < 2; u++) {  // bytes 4u .. 4u + 3 of the sub-block's 8
                const uint32_t w = r.q[9 * s + 1 + 2 * j + u];
                const int lo = iq4_lookup4(w & 0x0f0f0f0fu, tv), hi = iq4_lookup4((w >> 4) & 0x0f0f0f0fu, tv);
                const uint2 xl = *reinterpret_cast<const uint2 *>(xq + 8 * J + 2 * u);
                const uint2 xh = *reinterpret_cast<const uint2 *>(xq + 8 * J + 4 + 2 * u);
                sum = __dp2a_lo((int)xl.x, lo, sum);
                sum = __dp2a_hi((int)xl.y, lo, sum);
                sum = __dp2a_lo((int)xh.x, hi, sum);
                sum = __dp2a_hi((int)xh.y, hi, sum);
            }
            const float d = ue4m3_half((r.q[9 * s] >> (8 * j)) & 255u);
            acc = fmaf(d * xsc[J >> 1], (float)sum, acc);
        }
    __syncwarp();  // xq is rewritten for the next block
    return acc;
}

struct Q3Regs {
    uint32_t hm[8], q[16], s[3];
    float d;
};

__device__ __forceinline__ void dp_q3k_load(const uint8_t *blk, Q3Regs &r) {  // 2-byte aligned
    const uintptr_t ab = (uintptr_t)blk;
    const uint32_t *aw = reinterpret_cast<const uint32_t *>(ab & ~(uintptr_t)3);
    const uint32_t sh = (uint32_t)(ab & 3) * 8;  // 0 or 16
    uint32_t w[29];
#pragma unroll
    for (int i = 0; i < 29; i++) w[i] = aw[i];  // up to 6 bytes past the block: the ring row has slack
#pragma unroll
    for (int i = 0; i < 8; i++) r.hm[i] = __funnelshift_r(w[i], w[i + 1], sh);
#pragma unroll
    for (int i = 0; i < 16; i++) r.q[i] = __funnelshift_r(w[8 + i], w[9 + i], sh);
#pragma unroll
    for (int i = 0; i < 3; i++) r.s[i] = __funnelshift_r(w[24 + i], w[25 + i], sh);
    r.d = half_bits_to_float(__funnelshift_r(w[27], w[28], sh) & 0xffffu);
}

__device__ __forceinline__ float dp_q3k_dot(const Q3Regs &r, const uint32_t *xq, const float *xsc) {
    float acc = 0.f;
#pragma unroll
    for (int h = 0; h < 2; h++)
#pragma unroll
        for (int k = 0; k < 4; k++) {
            int s0 = 0, s1 = 0;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const uint32_t hb = (r.hm[i] >> (4 * h + k)) & 0x01010101u;
                const int q = (int)(((r.q[8 * h + i] >> (2 * k)) & 0x03030303u) | (hb << 2));
                const uint2 xv = *reinterpret_cast<const uint2 *>(xq + 64 * h + 16 * k + 2 * i);
                int &sm = i < 4 ? s0 : s1;
                sm = __dp2a_lo((int)xv.x, q, sm);
                sm = __dp2a_hi((int)xv.y, q, sm);
            }
            const int g = 4 * h + k;
#pragma unroll
            for (int u = 0; u < 2; u++) {
                const int j = 2 * g + u;  // 16-weight sub-block
                const uint32_t lw = r.s[(j & 7) >> 2];
                const int lo = (int)((lw >> (8 * (j & 3) + 4 * (j >> 3))) & 15u);
                const int hi = (int)((r.s[2] >> (8 * (j & 3) + 2 * (j >> 2))) & 3u);
                const float sc = (float)((lo | (hi << 4)) - 32);
                acc = fmaf(r.d * sc, fmaf(xsc[g], (float)(u ? s1 : s0), -4.f * xsc[16 + j]), acc);
            }
        }
    __syncwarp();  // xq is rewritten for the next block
    return acc;
}

}  // namespace
}  // namespace kq
