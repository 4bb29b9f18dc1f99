// kq_formats.cuh -- GGUF K-quant / IQ-quant super-block formats on sm_100a.
//
// Block layouts (256 weights per super-block), as decoded by gguf-py 0.19.0
// gguf/quants.py, the restatement of ggml's formats that gmlx depends on
// (gmlx pyproject.toml:62; the kernels gmlx calls live in the external
// mlx-kquant, gmlx/modules.py:35-40):
//
//   Q4_K  144 B  d f16 | dmin f16 | 12 B packed 6-bit (sc, m) x 8 | 128 B nibbles
//                w = (d*sc_j)*q - (dmin*m_j)              quants.py:475-522
//   Q6_K  210 B  128 B ql | 64 B qh | 16 x int8 sc | d f16
//                w = (d*sc_j)*(q - 32)                    quants.py:552-572
//   IQ2_XXS 66 B d f16 | 8 x (u32 grid indices, u32 signs+scale)
//                w = d*(0.5+ls)*0.25 * grid * sign        quants.py:766-829
//   Q5_K  176 B  d f16 | dmin f16 | 12 B scales | 32 B qh | 128 B nibbles
//                w = (d*sc_j)*(q | qh_bit << 4) - (dmin*m_j)  quants.py:525-549
//   Q8_0  8 x 34 B  (d f16 | 32 x int8), w = q*d       quants.py:378-402
//   IQ3_XXS 98 B d f16 | 64 B grid indices | 8 x u32 (4 x 7-bit signs, ls)
//                w = d*(0.5+ls)*0.5 * grid * sign         quants.py:1005-1054
//   IQ4_XS 136 B d f16 | u16 scales_h | 4 B scales_l | 128 B nibbles
//                w = (d*(ls-32)) * kvalues[q]             quants.py:1351-1377
//   Q4_0  8 x 18 B  (d f16 | 16 B nibbles), w = d*(q-8)  quants.py:241-251
//   IQ4_NL 8 x 18 B (d f16 | 16 B nibbles), w = d*kvalues[q]  quants.py:1333-1348
//         (32-weight blocks: nibble j < 16 low of byte j, else high of byte j-16)
//   Q4_1  8 x 20 B  (d | m | 16 B nibbles), w = d*q + m   quants.py:254-276
//   Q5_0  8 x 22 B  (d | u32 qh | 16 B), w = d*(q-16)     quants.py:279-305
//   Q5_1  8 x 24 B  (d | m | u32 qh | 16 B), w = d*q + m  quants.py:308-336
//         (Q5: q = nibble | (qh bit j) << 4 for weight j)
//   MXFP4 8 x 17 B  (e8m0 e | 16 B nibbles), w = 2^(e-128) * kvalues[q]
//                (kvalues: doubled e2m1; MXFP4.dequantize_blocks)
//   TQ2_0 66 B   64 B 2-bit q (Q2_K's layout) | d f16, w = d*(q-1)
//   NVFP4 4 x 36 B (4 UE4M3 scales, one per 16 | 4 x 8 B nibbles: low = weights
//                0-7, high = 8-15 of each 16), w = ue4m3(s)/2 * kvalues[q]
//                (MXFP4's doubled e2m1 values)   quants.py:707-763
//   TQ1_0 54 B   48 B of five base-3 digits | 4 B of four | d f16, w = d*(t-1);
//                digit k of byte v = ((v*3^k mod 256)*3) >> 8   quants.py:602-620
//   IQ2_XS 74 B  d | 32 x u16 (9-bit grid index, 7-bit sign index) | 8 B scales
//                w = d*(0.5+s)*0.25 * grid * sign (s per 16 weights)
//   IQ2_S 82 B   d | 32 B index lo | 32 B signs | 8 B index hi (2 bits) | 8 B scales
//   IQ3_S 110 B  d | 64 B index lo | 8 B index hi (1 bit) | 32 B signs | 4 B scales
//                w = d*(1+2s) * grid * sign (s per 32 weights)
//   IQ1_S 50 B   d | 32 B index lo | 8 x u16 (3 index bits x 4, s in 12-14, delta sign 15)
//                w = d*(2s+1) * (grid + delta), grid in {-1,0,1}, delta = +-1/8 (per 32)
//   IQ1_M 56 B   32 B index lo | 16 B nibbles (3 index bits, delta sign) | 4 x u16
//                (3-bit s per 16 weights; top nibbles = fp16 d); delta per 8 weights
//   Q2_K  84 B   16 x (sc | m << 4) | 64 B 2-bit q | d f16 | dmin f16
//                w = (d*sc_j)*q - (dmin*m_j), 16-weight j   quants.py:404-428
//   Q3_K  110 B  32 B high bits | 64 B 2-bit q | 12 B 6-bit scales | d f16
//                w = (d*(s_j-32))*(q - 4*(1-hbit))          quants.py:431-472
//         (both: weight 128h + 32k + l = bits 2k of quant byte 32h + l)
//
// Exactness: every product above is exact in f32 (fp16 d has 11 significant
// bits; d*sc <= 17 bits, d*sc*q <= 21 bits; Q6_K d*sc*(q-32) <= 24 bits;
// IQ2_XXS d*(0.5+ls)*0.25*grid <= 22 bits; IQ3_XXS d*(0.5+ls)*0.5*grid <= 22
// bits; IQ4_XS d*(ls-32)*kvalue <= 24 bits), so a dequantized weight is
// bit-identical to gguf-py whether or not the compiler contracts to FMA: only
// the final Q4_K subtraction rounds, once, in either form.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "_gen/kq_tables.h"

namespace kq {

enum Codec : int {
    Q4_0 = 2, Q4_1 = 3, Q5_0 = 6, Q5_1 = 7, Q8_0 = 8, TQ2_0 = 35, MXFP4 = 39, Q2_K = 10, Q3_K = 11, Q4_K = 12, Q5_K = 13, Q6_K = 14, IQ2_XXS = 16, IQ2_XS = 17, IQ3_XXS = 18, IQ4_NL = 20,
    IQ1_S = 19, IQ3_S = 21, IQ2_S = 22, IQ4_XS = 23, IQ1_M = 29, TQ1_0 = 34, NVFP4 = 40
};
enum DType : int { F32 = 0, F16 = 1, BF16 = 2 };

constexpr int QK = 256;

template <int C> struct Fmt;
template <> struct Fmt<Q4_K> { static constexpr int bpb = 144; static constexpr int sub = 32; };
template <> struct Fmt<Q5_K> { static constexpr int bpb = 176; static constexpr int sub = 32; };
// Q8_0: ggml blocks of 32 weights (fp16 d + 32 int8); eight of them (272 bytes)
// are handled as one 256-weight group
template <> struct Fmt<Q8_0> { static constexpr int bpb = 272; static constexpr int sub = 32; };
// Q4_0 / IQ4_NL: ggml blocks of 32 weights (fp16 d + 16 nibble bytes); eight
// of them (144 bytes) are handled as one 256-weight group
template <> struct Fmt<Q4_0> { static constexpr int bpb = 144; static constexpr int sub = 32; };
template <> struct Fmt<IQ4_NL> { static constexpr int bpb = 144; static constexpr int sub = 32; };
template <> struct Fmt<Q4_1> { static constexpr int bpb = 160; static constexpr int sub = 32; };
template <> struct Fmt<Q5_0> { static constexpr int bpb = 176; static constexpr int sub = 32; };
template <> struct Fmt<Q5_1> { static constexpr int bpb = 192; static constexpr int sub = 32; };
template <> struct Fmt<MXFP4> { static constexpr int bpb = 136; static constexpr int sub = 32; };
template <> struct Fmt<TQ2_0> { static constexpr int bpb = 66; static constexpr int sub = 32; };
template <> struct Fmt<IQ2_XS> { static constexpr int bpb = 74; static constexpr int sub = 16; };
template <> struct Fmt<IQ2_S> { static constexpr int bpb = 82; static constexpr int sub = 16; };
template <> struct Fmt<IQ3_S> { static constexpr int bpb = 110; static constexpr int sub = 32; };
template <> struct Fmt<IQ1_S> { static constexpr int bpb = 50; static constexpr int sub = 32; };
template <> struct Fmt<IQ1_M> { static constexpr int bpb = 56; static constexpr int sub = 16; };
template <> struct Fmt<TQ1_0> { static constexpr int bpb = 54; static constexpr int sub = 32; };
template <> struct Fmt<NVFP4> { static constexpr int bpb = 144; static constexpr int sub = 16; };

// The 32-weight legacy blocks: d (fp16; MXFP4: one e8m0 byte), m (fp16;
// HASM), a u32 of fifth bits (HASH), then 16 nibble bytes; BB bytes per
// block, OFF subtracted from q; NL / MX: nibbles index a value table.
template <int C> struct Legacy {
    static constexpr bool IS = C == Q4_0 || C == Q4_1 || C == Q5_0 || C == Q5_1 || C == IQ4_NL || C == MXFP4;
    static constexpr bool HASM = C == Q4_1 || C == Q5_1, HASH = C == Q5_0 || C == Q5_1;
    static constexpr bool MX = C == MXFP4, NL = C == IQ4_NL || C == MXFP4;
    static constexpr int BB = (MX ? 17 : 18) + (HASM ? 2 : 0) + (HASH ? 4 : 0);
    static constexpr int HOFF = HASM ? 4 : 2;  // fifth bits
    static constexpr int QOFF = BB - 16;       // nibble bytes
    static constexpr int OFF = C == Q4_0 ? 8 : C == Q5_0 ? 16 : 0;
};

// NVFP4's scale: unsigned E4M3 (bias 7) times 0.5, 0 and 0x7F decoding to 0;
// normal values are placed straight into f32 bits ((1 + m/8) 2^(e-8))
__device__ __forceinline__ float ue4m3_half(uint32_t x) {
    const uint32_t e = (x >> 3) & 15u, m = x & 7u;
    if (x == 0u || x == 0x7Fu) return 0.f;
    if (e == 0u) return (float)m * 0.0009765625f;  // m 2^-9 / 2
    return __uint_as_float(((e + 119u) << 23) | (m << 20));
}

// ggml's e8m0 "half" scale: 2^(e-128) as f32 bits (e < 2: subnormal)
__device__ __forceinline__ float e8m0_half(uint32_t e) {
    return __uint_as_float(e < 2 ? (0x00200000u << e) : ((e - 1) << 23));
}
template <> struct Fmt<Q2_K> { static constexpr int bpb = 84; static constexpr int sub = 16; };
template <> struct Fmt<Q3_K> { static constexpr int bpb = 110; static constexpr int sub = 16; };
template <> struct Fmt<Q6_K> { static constexpr int bpb = 210; static constexpr int sub = 16; };
template <> struct Fmt<IQ2_XXS> { static constexpr int bpb = 66; static constexpr int sub = 32; };
template <> struct Fmt<IQ3_XXS> { static constexpr int bpb = 98; static constexpr int sub = 32; };
template <> struct Fmt<IQ4_XS> { static constexpr int bpb = 136; static constexpr int sub = 32; };

// Weights per ggml block of the codecs that are handled in 256-weight groups
// of smaller blocks (a row may end in a partial group: K need only be a whole
// number of these blocks); 256 for every super-block codec.
__host__ __device__ inline int sub_block_weights(int codec) {
    switch (codec) {
    case Q8_0: case Q4_0: case Q4_1: case Q5_0: case Q5_1: case IQ4_NL: case MXFP4: return 32;
    case NVFP4: return 64;
    default: return 256;
    }
}

__host__ __device__ inline int block_bytes(int codec);
// Wire bytes of a row of k weights.
__host__ __device__ inline int64_t wire_row_bytes(int codec, int64_t k) {
    const int sw = sub_block_weights(codec);
    return k / sw * (block_bytes(codec) / (256 / sw));
}

__host__ __device__ inline int block_bytes(int codec) {
    return codec == Q4_K ? 144 : codec == Q5_K ? 176 : codec == Q6_K ? 210 : codec == IQ2_XXS ? 66
         : codec == Q8_0 ? 272 : codec == IQ3_XXS ? 98 : codec == IQ4_XS ? 136 : (codec == Q4_0 || codec == IQ4_NL) ? 144
         : codec == Q4_1 ? 160 : codec == Q5_0 ? 176 : codec == Q5_1 ? 192 : codec == MXFP4 ? 136 : codec == TQ2_0 ? 66
         : codec == IQ2_XS ? 74 : codec == IQ2_S ? 82 : codec == IQ3_S ? 110 : codec == IQ1_S ? 50 : codec == IQ1_M ? 56
         : codec == TQ1_0 ? 54 : codec == NVFP4 ? 144
         : codec == Q2_K ? 84 : codec == Q3_K ? 110 : -1;
}

// 256-entry IQ2_XXS grid, byte i of entry e = |w_i| in {8, 25, 43}.
static __device__ __constant__ uint64_t c_iq2xxs_grid[256] = KQ_IQ2XXS_GRID_INIT;
// 256-entry IQ3_XXS grid, byte i of entry e = |w_i| in {4, 12, ..., 62}.
static __device__ __constant__ uint32_t c_iq3xxs_grid[256] = KQ_IQ3XXS_GRID_INIT;
// The sixteen IQ4_NL values an IQ4_XS nibble selects, as bytes of four words.
static __device__ __constant__ __align__(16) int8_t c_iq4nl_values[16] = KQ_IQ4NL_VALUES_INIT;
// IQ2_XS (512 x 8), IQ2_S (1024 x 8) and IQ3_S (512 x 4) grids, byte i = |w_i|.
static __device__ __constant__ uint64_t c_iq2xs_grid[512] = KQ_IQ2XS_GRID_INIT;
static __device__ __constant__ uint64_t c_iq2s_grid[1024] = KQ_IQ2S_GRID_INIT;
static __device__ __constant__ uint32_t c_iq3s_grid[512] = KQ_IQ3S_GRID_INIT;
// IQ1_S / IQ1_M grid: 2048 x 8 values in {-1, 0, 1} as two's-complement bytes.
static __device__ __constant__ uint64_t c_iq1s_grid[2048] = KQ_IQ1S_GRID_INIT;
// MXFP4's doubled e2m1 values, as bytes of four words.
static __device__ __constant__ __align__(16) int8_t c_mxfp4_values[16] = KQ_MXFP4_VALUES_INIT;

// ggml's 7-bit -> 8-bit sign expansion: bit 7 restores even parity.
__device__ __forceinline__ uint32_t ksigns(uint32_t i7) {
    return i7 | ((__popc(i7) & 1u) << 7);
}

__device__ __forceinline__ float half_bits_to_float(uint32_t h16) {
    return __half2float(__ushort_as_half((unsigned short)h16));
}

__device__ __forceinline__ uint16_t ld_u16(const uint8_t *p) {
    return (uint16_t)p[0] | ((uint16_t)p[1] << 8);
}
__device__ __forceinline__ uint32_t ld_u32_unaligned(const uint8_t *p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

// Q4_K 12-byte scale/min unpack (gguf-py Q4_K.get_scale_min, quants.py:479-501)
// done four lanes at a time on 32-bit words: s0 = bytes 0-3, s1 = 4-7, s2 = 8-11.
__device__ __forceinline__ void q4k_unpack_scales(uint32_t s0, uint32_t s1, uint32_t s2,
                                                  uint32_t &sc03, uint32_t &sc47,
                                                  uint32_t &m03, uint32_t &m47) {
    sc03 = s0 & 0x3f3f3f3fu;
    m03 = s1 & 0x3f3f3f3fu;
    sc47 = (s2 & 0x0f0f0f0fu) | ((s0 >> 2) & 0x30303030u);
    m47 = ((s2 >> 4) & 0x0f0f0f0fu) | ((s1 >> 2) & 0x30303030u);
}

__device__ __forceinline__ float byte_f(uint32_t w, int i) { return (float)((w >> (8 * i)) & 0xffu); }

// Bounded spin limits for every device-side wait (mbarrier and flags).  A
// wait that runs out sets the kernel's error word and abandons the unit.
constexpr uint32_t kSpinLimit = 1u << 26;

}  // namespace kq
