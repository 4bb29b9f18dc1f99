/*
 * kq_oracle.c -- CPU restatement of the GGUF K-quant / IQ-quant block formats
 * on the fused dequantize-and-multiply path.  TEST INFRASTRUCTURE ONLY: this
 * file is the checker the CUDA kernels are compared against, and the timed
 * CPU baseline.  The product library (libkq_cuda.so) never links or calls it.
 *
 * The reference (gmlx) reaches these formats through the external mlx-kquant
 * library (gmlx/modules.py:35-40, pinned at pyproject.toml:33), whose source is
 * not available.  The published block semantics it implements are those of
 * ggml; the runnable restatement in this environment is gguf-py 0.19.0
 * (gguf/quants.py), a declared gmlx dependency (pyproject.toml:62).  Each
 * decoder below cites the gguf-py function it follows; the Python tests pin
 * this file bit-for-bit against gguf-py on seeded blocks and edge cases.
 *
 * Arithmetic order matches gguf-py exactly (all f32):
 *   Q4_K   (quants.py:504-522): dl = d*sc, ml = dmin*m, w = dl*q - ml
 *   Q5_K   (quants.py:525-549): as Q4_K with q = nibble | (qh bit j) << 4
 *   Q8_0   (Q8_0.dequantize_blocks): w = q * d per 32-weight block
 *   Q6_K   (quants.py:554-572): dl = d*sc, w = dl*(q-32)
 *   IQ2_XXS(quants.py:802-829): db = d*(0.5+ls)*0.25, w = db*grid*sign
 *   IQ3_XXS(quants.py:1027-1054): db = d*(0.5+ls)*0.5, w = db*grid*sign
 *   IQ4_XS (quants.py:1351-1377): dl = d*(ls-32), w = dl*kvalues[q]
 *   Q4_0   (quants.py:241-251): w = d*(q-8) per 32-weight block
 *   Q2_K   (quants.py:404-428): dl = d*sc, ml = dmin*m, w = dl*q - ml (16-weight sub-blocks)
 *   Q3_K   (quants.py:431-472): dl = d*(s-32), w = dl*(q2 - 4*(1-hbit))
 *   IQ4_NL (quants.py:1333-1348): w = d*kvalues[q] per 32-weight block
 *   Q4_1   (quants.py:254-276): w = d*q + m;  Q5_0 (:279-305): w = d*(q-16);
 *   Q5_1   (:308-336): w = d*q + m  (Q5: q = nibble | qh bit << 4)
 *   MXFP4  (MXFP4.dequantize_blocks): w = e8m0_half(e) * kvalues[q] per 32 weights
 *   TQ2_0  (TQ2_0.dequantize_blocks): w = d*(q-1), q 2-bit, Q2_K's quant layout
 *   NVFP4  (quants.py:707-763): w = ue4m3_half(s_j) * kvalues[q], s_j per 16 weights
 *   TQ1_0  (quants.py:602-620): trit k of byte b = ((b*3^k mod 256)*3) >> 8, w = d*(t-1)
 *   IQ1_S  (quants.py:1267-1288): dl = d*(2s+1) per 32, w = dl*(grid + delta), delta = +-0.125
 *   IQ1_M  (quants.py:1300-1327): the same with s per 16, delta per 8, d packed in the scales
 *   IQ2_XS (quants.py:872-898), IQ2_S (:974-1002): db = d*(0.5+s)*0.25 per 16
 *          weights, w = db*grid*sign;  IQ3_S (:1096-1125): db = d*(1+2s) per 32
 * Every product above is exact in f32 (see the kernels' header), so results
 * are independent of FMA contraction; the file is still built with
 * -ffp-contract=off to keep the statement literal.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#include "kq_tables.h"

#define QK 256
enum { KQO_Q8_0 = 8, KQO_Q4_K = 12, KQO_Q5_K = 13, KQO_Q6_K = 14, KQO_IQ2_XXS = 16, KQO_IQ3_XXS = 18, KQO_IQ4_XS = 23,
       KQO_Q4_0 = 2, KQO_IQ4_NL = 20, KQO_Q2_K = 10, KQO_Q3_K = 11,
       KQO_Q4_1 = 3, KQO_Q5_0 = 6, KQO_Q5_1 = 7, KQO_TQ2_0 = 35, KQO_MXFP4 = 39,
       KQO_IQ2_XS = 17, KQO_IQ3_S = 21, KQO_IQ2_S = 22, KQO_IQ1_S = 19, KQO_IQ1_M = 29, KQO_TQ1_0 = 34, KQO_NVFP4 = 40 };

static const uint64_t kqo_grid[256] = KQ_IQ2XXS_GRID_INIT;
static const uint32_t kqo_grid3[256] = KQ_IQ3XXS_GRID_INIT;
static const int8_t kqo_iq4nl[16] = KQ_IQ4NL_VALUES_INIT;
static const int8_t kqo_mxfp4[16] = KQ_MXFP4_VALUES_INIT;
static const uint64_t kqo_grid2xs[512] = KQ_IQ2XS_GRID_INIT;
static const uint64_t kqo_grid2s[1024] = KQ_IQ2S_GRID_INIT;
static const uint32_t kqo_grid3s[512] = KQ_IQ3S_GRID_INIT;
static const uint64_t kqo_grid1s[2048] = KQ_IQ1S_GRID_INIT;

/* IEEE binary16 -> f32, exact (gguf-py: view(np.float16).astype(np.float32)). */
static float kqo_half(uint16_t h) {
    uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 0x1f, m = h & 0x3ff, u;
    if (e == 0) {
        if (m == 0) { u = s; }
        else { /* subnormal: renormalise */
            e = 113;
            while (!(m & 0x400)) { m <<= 1; e--; }
            u = s | (e << 23) | ((m & 0x3ff) << 13);
        }
    } else if (e == 31) {
        u = s | 0x7f800000u | (m << 13);
    } else {
        u = s | ((e + 112) << 23) | (m << 13);
    }
    float f; memcpy(&f, &u, 4); return f;
}

static float kqo_bf16(uint16_t b) { uint32_t u = (uint32_t)b << 16; float f; memcpy(&f, &u, 4); return f; }

int kqo_block_bytes(int codec) {
    switch (codec) {
    case KQO_Q4_K: return 144; case KQO_Q5_K: return 176; case KQO_Q6_K: return 210; case KQO_IQ2_XXS: return 66;
    case KQO_Q8_0: return 272; /* eight 34-byte blocks per 256 weights */
    case KQO_IQ3_XXS: return 98; case KQO_IQ4_XS: return 136;
    case KQO_Q4_0: case KQO_IQ4_NL: return 144; /* eight 18-byte blocks per 256 weights */
    case KQO_Q2_K: return 84; case KQO_Q3_K: return 110;
    case KQO_Q4_1: return 160; case KQO_Q5_0: return 176; case KQO_Q5_1: return 192; /* eight blocks */
    case KQO_MXFP4: return 136; /* eight 17-byte blocks */
    case KQO_TQ2_0: return 66;
    case KQO_IQ2_XS: return 74; case KQO_IQ2_S: return 82; case KQO_IQ3_S: return 110;
    case KQO_IQ1_S: return 50; case KQO_IQ1_M: return 56; case KQO_TQ1_0: return 54;
    case KQO_NVFP4: return 144; /* four 36-byte blocks of 64 weights */
    }
    return -1;
}

/* gguf-py Q4_K.get_scale_min (quants.py:479-501): 12 packed bytes -> 8 x (sc, m). */
static void q4k_scale_min(const uint8_t *s, uint8_t sc[8], uint8_t mn[8]) {
    for (int j = 0; j < 4; j++) {
        sc[j] = s[j] & 0x3f;
        mn[j] = s[j + 4] & 0x3f;
        sc[j + 4] = (s[j + 8] & 0x0f) | ((s[j] >> 2) & 0x30);
        mn[j + 4] = (s[j + 8] >> 4) | ((s[j + 4] >> 2) & 0x30);
    }
}

/* gguf-py Q4_K.dequantize_blocks (quants.py:504-522). */
static void deq_q4k(const uint8_t *b, float *o) {
    float d = kqo_half((uint16_t)(b[0] | b[1] << 8));
    float dmin = kqo_half((uint16_t)(b[2] | b[3] << 8));
    uint8_t sc[8], mn[8];
    q4k_scale_min(b + 4, sc, mn);
    const uint8_t *q = b + 16;
    for (int c = 0; c < 4; c++) {          /* 32-byte chunk c -> sub-blocks 2c, 2c+1 */
        for (int h = 0; h < 2; h++) {      /* low nibble, then high nibble */
            int j = 2 * c + h;
            float dl = d * (float)sc[j], ml = dmin * (float)mn[j];
            for (int l = 0; l < 32; l++) {
                float qv = (float)((q[32 * c + l] >> (4 * h)) & 0x0f);
                o[32 * j + l] = dl * qv - ml;
            }
        }
    }
}

/* gguf-py Q5_K.dequantize_blocks (quants.py:525-549): d, dmin, the Q4_K
 * scale/min packing, 32 bytes of fifth bits (bit j of qh[l] belongs to weight
 * l of sub-block j) and 128 bytes of low nibbles (Q4_K order). */
static void deq_q5k(const uint8_t *b, float *o) {
    float d = kqo_half((uint16_t)(b[0] | b[1] << 8));
    float dmin = kqo_half((uint16_t)(b[2] | b[3] << 8));
    uint8_t sc[8], mn[8];
    q4k_scale_min(b + 4, sc, mn);
    const uint8_t *qh = b + 16, *qs = b + 48;
    for (int j = 0; j < 8; j++) {
        float dl = d * (float)sc[j], ml = dmin * (float)mn[j];
        for (int l = 0; l < 32; l++) {
            int lo = (qs[32 * (j >> 1) + l] >> (4 * (j & 1))) & 0x0f;
            int hi = (qh[l] >> j) & 1;
            o[32 * j + l] = dl * (float)(lo | (hi << 4)) - ml;
        }
    }
}

/* gguf-py Q8_0.dequantize_blocks: eight (fp16 d, 32 x int8 q) blocks, w = q * d. */
static void deq_q80(const uint8_t *b, float *o) {
    for (int j = 0; j < 8; j++) {
        const uint8_t *blk = b + 34 * j;
        float d = kqo_half((uint16_t)(blk[0] | blk[1] << 8));
        for (int l = 0; l < 32; l++) o[32 * j + l] = (float)(int8_t)blk[2 + l] * d;
    }
}

/* gguf-py Q6_K.dequantize_blocks (quants.py:554-572). */
static void deq_q6k(const uint8_t *b, float *o) {
    const uint8_t *ql = b, *qh = b + 128;
    const int8_t *sc = (const int8_t *)(b + 192);
    float d = kqo_half((uint16_t)(b[208] | b[209] << 8));
    for (int hf = 0; hf < 2; hf++) {       /* two 128-weight halves */
        for (int s = 0; s < 4; s++) {      /* 32-weight group s of the half */
            for (int l = 0; l < 32; l++) {
                int i = 128 * hf + 32 * s + l;
                int lo = (ql[64 * hf + 32 * (s & 1) + l] >> (4 * (s >> 1))) & 0x0f;
                int hi = (qh[32 * hf + l] >> (2 * s)) & 0x03;
                int q = (lo | (hi << 4)) - 32;
                float dl = d * (float)sc[i / 16];
                o[i] = dl * (float)q;
            }
        }
    }
}

/* ggml's ksigns table: 7-bit index plus an even-parity top bit
 * (gguf-py IQ2_XXS.ksigns, quants.py:767-776, is this table written out). */
static uint8_t kqo_ksigns(unsigned i) {
    unsigned p = i ^ (i >> 4); p ^= p >> 2; p ^= p >> 1;
    return (uint8_t)(i | ((p & 1) << 7));
}

/* gguf-py IQ2_XXS.dequantize_blocks (quants.py:802-829). */
static void deq_iq2xxs(const uint8_t *b, float *o) {
    float d = kqo_half((uint16_t)(b[0] | b[1] << 8));
    for (int g = 0; g < 8; g++) {
        uint32_t a0, a1;
        memcpy(&a0, b + 2 + 8 * g, 4);
        memcpy(&a1, b + 6 + 8 * g, 4);
        float db = d * (0.5f + (float)(a1 >> 28)) * 0.25f;
        for (int s = 0; s < 4; s++) {
            uint8_t sg = kqo_ksigns((a1 >> (7 * s)) & 0x7f);
            uint64_t e = kqo_grid[(a0 >> (8 * s)) & 0xff];
            for (int i = 0; i < 8; i++) {
                float gv = (float)((e >> (8 * i)) & 0xff);
                float sv = ((sg >> i) & 1) ? -1.0f : 1.0f;
                o[32 * g + 8 * s + i] = db * gv * sv;
            }
        }
    }
}

/* gguf-py IQ3_XXS.dequantize_blocks (quants.py:1027-1054): d, 64 grid-index
 * bytes (one per 4 weights), then 8 words of (4 x 7-bit sign indices, ls << 28),
 * one word per 32-weight sub-block. */
static void deq_iq3xxs(const uint8_t *b, float *o) {
    float d = kqo_half((uint16_t)(b[0] | b[1] << 8));
    const uint8_t *qs = b + 2, *ss = b + 66;
    for (int j = 0; j < 8; j++) {
        uint32_t aux;
        memcpy(&aux, ss + 4 * j, 4);
        float db = d * (0.5f + (float)(aux >> 28)) * 0.5f;
        for (int l = 0; l < 4; l++) {
            uint8_t sg = kqo_ksigns((aux >> (7 * l)) & 0x7f);
            for (int i = 0; i < 8; i++) {
                uint32_t e = kqo_grid3[qs[8 * j + 2 * l + (i >> 2)]];
                float gv = (float)((e >> (8 * (i & 3))) & 0xff);
                float sv = ((sg >> i) & 1) ? -1.0f : 1.0f;
                o[32 * j + 8 * l + i] = db * gv * sv;
            }
        }
    }
}

/* gguf-py IQ4_XS.dequantize_blocks (quants.py:1351-1377): d, 16 bits of
 * high scale pairs, 4 bytes of low scale nibbles, then 16 bytes per sub-block
 * (low nibbles: weights 0-15, high nibbles: 16-31) indexing IQ4_NL.kvalues. */
static void deq_iq4xs(const uint8_t *b, float *o) {
    float d = kqo_half((uint16_t)(b[0] | b[1] << 8));
    unsigned sh = (unsigned)(b[2] | b[3] << 8);
    const uint8_t *sl = b + 4, *qs = b + 8;
    for (int j = 0; j < 8; j++) {
        int ls = ((sl[j >> 1] >> (4 * (j & 1))) & 0x0f) | (((sh >> (2 * j)) & 3) << 4);
        float dl = d * (float)(ls - 32);
        for (int l = 0; l < 16; l++) {
            o[32 * j + l] = dl * (float)kqo_iq4nl[qs[16 * j + l] & 0x0f];
            o[32 * j + 16 + l] = dl * (float)kqo_iq4nl[qs[16 * j + l] >> 4];
        }
    }
}

/* The 32-weight legacy blocks over eight blocks (one 256-weight group):
 * gguf-py Q4_0 (quants.py:241-251), Q4_1 (:254-276), Q5_0 (:279-305), Q5_1
 * (:308-336) and IQ4_NL (:1333-1348).  A block is d (fp16), then m (fp16;
 * Q4_1 / Q5_1), then a little-endian u32 of fifth bits (Q5_0 / Q5_1; bit j
 * belongs to weight j), then 16 bytes whose low nibbles are weights 0-15 and
 * high nibbles 16-31. */
static void deq_legacy(int codec, const uint8_t *b, float *o) {
    const int has_m = codec == KQO_Q4_1 || codec == KQO_Q5_1, has_h = codec == KQO_Q5_0 || codec == KQO_Q5_1;
    const int bb = 18 + 2 * has_m + 4 * has_h;
    for (int j = 0; j < 8; j++) {
        const uint8_t *blk = b + bb * j;
        float d = kqo_half((uint16_t)(blk[0] | blk[1] << 8));
        float m = has_m ? kqo_half((uint16_t)(blk[2] | blk[3] << 8)) : 0.0f;
        uint32_t qh = 0;
        if (has_h) memcpy(&qh, blk + 2 + 2 * has_m, 4);
        const uint8_t *qs = blk + bb - 16;
        for (int l = 0; l < 32; l++) {
            int v = (qs[l & 15] >> (4 * (l >> 4))) & 0x0f;
            if (has_h) v |= (int)((qh >> l) & 1) << 4;
            float w;
            switch (codec) {
            case KQO_IQ4_NL: w = d * (float)kqo_iq4nl[v]; break;
            case KQO_Q4_0: w = d * (float)(v - 8); break;
            case KQO_Q5_0: w = d * (float)(v - 16); break;
            default: w = d * (float)v + m; break; /* Q4_1, Q5_1 */
            }
            o[32 * j + l] = w;
        }
    }
}

/* gguf-py Q2_K.dequantize_blocks (quants.py:404-428): 16 scale bytes (low
 * nibble sc, high nibble m, one per 16 weights), 64 bytes of 2-bit quants
 * (weight 128h + 32k + l = bits 2k of byte 32h + l), d, dmin. */
static void deq_q2k(const uint8_t *b, float *o) {
    const uint8_t *sc = b, *qs = b + 16;
    float d = kqo_half((uint16_t)(b[80] | b[81] << 8)), dmin = kqo_half((uint16_t)(b[82] | b[83] << 8));
    for (int w = 0; w < 256; w++) {
        int h = w >> 7, k = (w >> 5) & 3, l = w & 31, j = w >> 4;
        float dl = d * (float)(sc[j] & 0x0f), ml = dmin * (float)(sc[j] >> 4);
        o[w] = dl * (float)((qs[32 * h + l] >> (2 * k)) & 3) - ml;
    }
}

/* gguf-py Q3_K.dequantize_blocks (quants.py:431-472): 32 bytes of high bits
 * (bit 4h + k of byte l, set meaning "no -4"), 64 bytes of 2-bit quants laid
 * out as Q2_K's, 12 bytes of sixteen 6-bit scales (low nibbles in bytes 0-7,
 * high pairs in bytes 8-11), d. */
static void deq_q3k(const uint8_t *b, float *o) {
    const uint8_t *hm = b, *qs = b + 32, *s = b + 96;
    float d = kqo_half((uint16_t)(b[108] | b[109] << 8));
    for (int w = 0; w < 256; w++) {
        int h = w >> 7, k = (w >> 5) & 3, l = w & 31, j = w >> 4;
        int lo = j < 8 ? (s[j] & 0x0f) : (s[j - 8] >> 4);
        int hi = (s[8 + (j & 3)] >> (2 * (j >> 2))) & 3;
        float dl = d * (float)((lo | (hi << 4)) - 32);
        int q = ((qs[32 * h + l] >> (2 * k)) & 3) - (((hm[l] >> (4 * h + k)) & 1) ? 0 : 4);
        o[w] = dl * (float)q;
    }
}

/* ggml's e8m0 -> f32 "half" scale (gguf-py MXFP4.e8m0_to_fp32_half): 2^(e-128)
 * as bits, with e < 2 as subnormals. */
static float kqo_e8m0_half(uint8_t e) {
    uint32_t u = e < 2 ? (0x00200000u << e) : ((uint32_t)(e - 1) << 23);
    float f; memcpy(&f, &u, 4); return f;
}

/* gguf-py MXFP4.dequantize_blocks over eight 17-byte blocks: e, then 16 bytes
 * (low nibbles weights 0-15, high 16-31) indexing the doubled e2m1 values. */
static void deq_mxfp4(const uint8_t *b, float *o) {
    for (int j = 0; j < 8; j++) {
        const uint8_t *blk = b + 17 * j;
        float d = kqo_e8m0_half(blk[0]);
        for (int l = 0; l < 32; l++) o[32 * j + l] = d * (float)kqo_mxfp4[(blk[1 + (l & 15)] >> (4 * (l >> 4))) & 15];
    }
}

/* gguf-py TQ2_0.dequantize_blocks: 64 bytes of 2-bit values laid out as
 * Q2_K's quants, then d; w = d * (q - 1). */
static void deq_tq20(const uint8_t *b, float *o) {
    float d = kqo_half((uint16_t)(b[64] | b[65] << 8));
    for (int w = 0; w < 256; w++) {
        int h = w >> 7, k = (w >> 5) & 3, l = w & 31;
        o[w] = d * (float)(((b[32 * h + l] >> (2 * k)) & 3) - 1);
    }
}

/* gguf-py IQ2_XS.dequantize_blocks: d, 32 u16 entries (9-bit grid index,
 * 7-bit sign index) of 8 weights, 8 bytes of 4-bit scales (one per 16
 * weights, low nibble first). */
static void deq_iq2xs(const uint8_t *b, float *o) {
    float d = kqo_half((uint16_t)(b[0] | b[1] << 8));
    for (int e = 0; e < 32; e++) {
        unsigned v = b[2 + 2 * e] | (b[3 + 2 * e] << 8);
        int s = (b[66 + (e >> 2)] >> (4 * ((e >> 1) & 1))) & 15;
        float db = d * (0.5f + (float)s) * 0.25f;
        uint8_t sg = kqo_ksigns(v >> 9);
        uint64_t g = kqo_grid2xs[v & 511];
        for (int i = 0; i < 8; i++)
            o[8 * e + i] = db * (float)((g >> (8 * i)) & 0xff) * (((sg >> i) & 1) ? -1.0f : 1.0f);
    }
}

/* gguf-py IQ2_S.dequantize_blocks: d, 32 low index bytes, 32 sign bytes,
 * 8 bytes of 2-bit high index parts (entry 4b + k: bits 2k of byte b), 8
 * bytes of 4-bit scales (one per 16 weights). */
static void deq_iq2s(const uint8_t *b, float *o) {
    float d = kqo_half((uint16_t)(b[0] | b[1] << 8));
    for (int e = 0; e < 32; e++) {
        unsigned idx = b[2 + e] | (((b[66 + (e >> 2)] >> (2 * (e & 3))) & 3u) << 8);
        int s = (b[74 + (e >> 2)] >> (4 * ((e >> 1) & 1))) & 15;
        float db = d * (0.5f + (float)s) * 0.25f;
        uint8_t sg = b[34 + e];
        uint64_t g = kqo_grid2s[idx];
        for (int i = 0; i < 8; i++)
            o[8 * e + i] = db * (float)((g >> (8 * i)) & 0xff) * (((sg >> i) & 1) ? -1.0f : 1.0f);
    }
}

/* gguf-py IQ3_S.dequantize_blocks: d, 64 low index bytes (4 weights each),
 * 8 bytes of high index bits (entry 8b + i: bit i of byte b), 32 sign bytes
 * (8 weights each), 4 bytes of 4-bit scales (one per 32 weights). */
static void deq_iq3s(const uint8_t *b, float *o) {
    float d = kqo_half((uint16_t)(b[0] | b[1] << 8));
    for (int e = 0; e < 64; e++) {
        unsigned idx = b[2 + e] | (((b[66 + (e >> 3)] >> (e & 7)) & 1u) << 8);
        int s = (b[106 + (e >> 4)] >> (4 * ((e >> 3) & 1))) & 15;
        float db = d * (float)(1 + 2 * s);
        uint8_t sg = b[74 + (e >> 1)];
        uint32_t g = kqo_grid3s[idx];
        for (int i = 0; i < 4; i++)
            o[4 * e + i] = db * (float)((g >> (8 * i)) & 0xff) * (((sg >> (4 * (e & 1) + i)) & 1) ? -1.0f : 1.0f);
    }
}

static float kqo_grid1(unsigned idx, int i) { return (float)(int8_t)((kqo_grid1s[idx] >> (8 * i)) & 0xff); }

/* gguf-py IQ1_S.dequantize_blocks: d, 32 low index bytes (8 weights each),
 * 8 u16 (one per 32 weights: 3 high index bits per entry, scale in bits
 * 12-14, delta sign in bit 15). */
static void deq_iq1s(const uint8_t *b, float *o) {
    float d = kqo_half((uint16_t)(b[0] | b[1] << 8));
    for (int e = 0; e < 32; e++) {
        int g = e >> 2;
        unsigned qh = b[34 + 2 * g] | (b[35 + 2 * g] << 8);
        float dl = d * (float)(2 * ((qh >> 12) & 7) + 1);
        float delta = (qh & 0x8000) ? -0.125f : 0.125f;
        unsigned idx = b[2 + e] | (((qh >> (3 * (e & 3))) & 7) << 8);
        for (int i = 0; i < 8; i++) o[8 * e + i] = dl * (kqo_grid1(idx, i) + delta);
    }
}

/* gguf-py IQ1_M.dequantize_blocks: 32 low index bytes, 16 bytes of one nibble
 * per entry (3 high index bits, delta sign in bit 3), 4 u16 of 3-bit scales
 * (one per 16 weights) whose top nibbles together hold the fp16 d. */
static void deq_iq1m(const uint8_t *b, float *o) {
    unsigned s[4];
    for (int t = 0; t < 4; t++) s[t] = b[48 + 2 * t] | (b[49 + 2 * t] << 8);
    float d = kqo_half((uint16_t)((s[0] >> 12) | ((s[1] >> 8) & 0xf0) | ((s[2] >> 4) & 0xf00) | (s[3] & 0xf000)));
    for (int e = 0; e < 32; e++) {
        int k = e >> 1;
        float dl = d * (float)(2 * ((s[k >> 2] >> (3 * (k & 3))) & 7) + 1);
        unsigned nib = (b[32 + (e >> 1)] >> (4 * (e & 1))) & 15;
        float delta = (nib & 8) ? -0.125f : 0.125f;
        unsigned idx = b[e] | ((nib & 7) << 8);
        for (int i = 0; i < 8; i++) o[8 * e + i] = dl * (kqo_grid1(idx, i) + delta);
    }
}

/* gguf-py TQ1_0.dequantize_blocks: 48 bytes of five base-3 digits each
 * (bytes 0-31: weight 32k + l; bytes 32-47: weight 160 + 16k + l), 4 bytes of
 * four digits (weight 240 + 4k + l), d.  Digit k of byte v is
 * ((v * 3^k mod 256) * 3) >> 8. */
static void deq_tq10(const uint8_t *b, float *o) {
    static const unsigned pw[5] = {1, 3, 9, 27, 81};
    float d = kqo_half((uint16_t)(b[52] | b[53] << 8));
    for (int w = 0; w < 256; w++) {
        unsigned v, k;
        if (w < 160) { v = b[w & 31]; k = w >> 5; }
        else if (w < 240) { v = b[32 + ((w - 160) & 15)]; k = (w - 160) >> 4; }
        else { v = b[48 + ((w - 240) & 3)]; k = (w - 240) >> 2; }
        int t = (int)((((v * pw[k]) & 255u) * 3u) >> 8);
        o[w] = d * (float)(t - 1);
    }
}

/* gguf-py NVFP4.ue4m3_to_fp32: unsigned E4M3 (bias 7) times 0.5; 0 and 0x7F
 * decode to 0. */
static float kqo_ue4m3_half(uint8_t x) {
    int e = (x >> 3) & 15, m = x & 7;
    if (x == 0 || x == 0x7F) return 0.0f;
    float raw = e == 0 ? (float)m * 0.001953125f : (1.0f + (float)m / 8.0f) * ldexpf(1.0f, e - 7);
    return raw * 0.5f;
}

/* gguf-py NVFP4.dequantize_blocks over four 36-byte blocks: four scale bytes
 * (one per 16 weights), then 4 x 8 bytes (low nibbles weights 0-7, high
 * nibbles 8-15 of each 16) indexing the doubled e2m1 values. */
static void deq_nvfp4(const uint8_t *b, float *o) {
    for (int s = 0; s < 4; s++) {
        const uint8_t *blk = b + 36 * s;
        for (int j = 0; j < 4; j++) {
            float d = kqo_ue4m3_half(blk[j]);
            for (int l = 0; l < 16; l++)
                o[64 * s + 16 * j + l] = d * (float)kqo_mxfp4[(blk[4 + 8 * j + (l & 7)] >> (4 * (l >> 3))) & 15];
        }
    }
}

static int deq_block(int codec, const uint8_t *b, float *o) {
    switch (codec) {
    case KQO_Q4_K: deq_q4k(b, o); return 0;
    case KQO_Q5_K: deq_q5k(b, o); return 0;
    case KQO_Q8_0: deq_q80(b, o); return 0;
    case KQO_Q6_K: deq_q6k(b, o); return 0;
    case KQO_IQ2_XXS: deq_iq2xxs(b, o); return 0;
    case KQO_IQ3_XXS: deq_iq3xxs(b, o); return 0;
    case KQO_IQ4_XS: deq_iq4xs(b, o); return 0;
    case KQO_Q4_0: case KQO_Q4_1: case KQO_Q5_0: case KQO_Q5_1: case KQO_IQ4_NL: deq_legacy(codec, b, o); return 0;
    case KQO_Q2_K: deq_q2k(b, o); return 0;
    case KQO_MXFP4: deq_mxfp4(b, o); return 0;
    case KQO_TQ2_0: deq_tq20(b, o); return 0;
    case KQO_IQ2_XS: deq_iq2xs(b, o); return 0;
    case KQO_IQ2_S: deq_iq2s(b, o); return 0;
    case KQO_IQ3_S: deq_iq3s(b, o); return 0;
    case KQO_IQ1_S: deq_iq1s(b, o); return 0;
    case KQO_TQ1_0: deq_tq10(b, o); return 0;
    case KQO_NVFP4: deq_nvfp4(b, o); return 0;
    case KQO_IQ1_M: deq_iq1m(b, o); return 0;
    case KQO_Q3_K: deq_q3k(b, o); return 0;
    }
    return -1;
}

/* Dequantize rows x k weights; row r starts at w + r*row_stride bytes. */
int kqo_dequantize(int codec, const uint8_t *w, int64_t rows, int64_t k, int64_t row_stride,
                   float *out, int threads) {
    int bpb = kqo_block_bytes(codec);
    if (bpb < 0 || k % QK) return -1;
    int64_t nb = k / QK;
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel for schedule(static)
#endif
    for (int64_t r = 0; r < rows; r++)
        for (int64_t b = 0; b < nb; b++)
            deq_block(codec, w + r * row_stride + b * bpb, out + r * k + b * QK);
    return 0;
}

/* Reference matmul y[m][n] = sum_k x[m][k] * dequant(W)[n][k], f32 accumulate
 * in index order, x given as bf16 bits (x_bf16 != 0) or f32.  Dequantizes one
 * row at a time (the reference's CPU dequantize-then-matmul arm). */
int kqo_matmul(int codec, const void *x, int x_bf16, int64_t m, int64_t k,
               const uint8_t *w, int64_t n, int64_t row_stride, float *y, int threads) {
    int bpb = kqo_block_bytes(codec);
    if (bpb < 0 || k % QK) return -1;
    int64_t nb = k / QK;
    float *xf = (float *)malloc(sizeof(float) * (size_t)(m * k));
    if (!xf) return -2;
    for (int64_t i = 0; i < m * k; i++)
        xf[i] = x_bf16 ? kqo_bf16(((const uint16_t *)x)[i]) : ((const float *)x)[i];
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel
#endif
    {
        float *wr = (float *)malloc(sizeof(float) * (size_t)k);
#ifdef _OPENMP
#pragma omp for schedule(static)
#endif
        for (int64_t r = 0; r < n; r++) {
            for (int64_t b = 0; b < nb; b++) deq_block(codec, w + r * row_stride + b * bpb, wr + b * QK);
            for (int64_t i = 0; i < m; i++) {
                /* eight interleaved f32 partial sums (vectorisable without
                 * reassociation flags), combined pairwise at the end */
                const float *xr = xf + i * k;
                float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
                for (int64_t j = 0; j < k; j += 8)
                    for (int u = 0; u < 8; u++) acc[u] += xr[j + u] * wr[j + u];
                y[i * n + r] = ((acc[0] + acc[4]) + (acc[2] + acc[6])) + ((acc[1] + acc[5]) + (acc[3] + acc[7]));
            }
        }
        free(wr);
    }
    free(xf);
    return 0;
}

/* MoE router (gmlx/moe_experts.py:226-240): softmax over E logits (f32,
 * max-subtracted), top-k by probability (ties -> lower expert id), optional
 * renormalisation of the k scores.  Output order: descending probability. */
int kqo_router_topk(const float *logits, int64_t t, int64_t e, int k, int norm,
                    int32_t *idx, float *scores) {
    if (k <= 0 || k > e) return -1;
    float *p = (float *)malloc(sizeof(float) * (size_t)e);
    for (int64_t r = 0; r < t; r++) {
        const float *l = logits + r * e;
        float mx = -INFINITY, s = 0.f;
        for (int64_t j = 0; j < e; j++) mx = l[j] > mx ? l[j] : mx;
        for (int64_t j = 0; j < e; j++) { p[j] = expf(l[j] - mx); s += p[j]; }
        for (int64_t j = 0; j < e; j++) p[j] = p[j] / s;
        float tot = 0.f;
        for (int c = 0; c < k; c++) {
            int64_t best = -1;
            for (int64_t j = 0; j < e; j++) {
                int taken = 0;
                for (int q = 0; q < c; q++) taken |= idx[r * k + q] == (int32_t)j;
                if (taken) continue;
                if (best < 0 || p[j] > p[best]) best = j;
            }
            idx[r * k + c] = (int32_t)best;
            scores[r * k + c] = p[best];
            tot += p[best];
        }
        if (norm)
            for (int c = 0; c < k; c++) scores[r * k + c] /= tot;
    }
    free(p);
    return 0;
}
