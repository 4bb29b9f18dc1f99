// kq_gemm_sm100.cu -- prefill-shaped fused dequantize x GEMM on the 5th-gen
// tensor cores (tcgen05, TMEM accumulators).  Replaces mlx-kquant's M-banded
// qmm route of quantized_matmul (KQuantLinear, gmlx/modules.py:1535-1539;
// "M-banded qmm tiles" CHANGELOG.md:599-600) for large M.
//
//   y[M_tok, N_w] = x[M_tok, K] . dequant(W[N_w, K])^T
//
// Tile: 128 activation rows (MMA M) x 256 weight rows (MMA N) x K, K staged
// 64 at a time (one 128-byte swizzle atom of bf16/f16).  Warp roles (320 thr):
//   warp 0      TMA producer: activation tile (and, for dense B, the B tile)
//               into a 4-stage ring, SWIZZLE_128B, no cluster multicast;
//   warp 1      allocates 256 TMEM columns; one elected lane issues
//               tcgen05.mma (kind::f16, f32 accumulate) and tcgen05.commit;
//   warps 2-9   Q4_K: each thread owns one weight row, takes its raw 144-byte
//               blocks (16-byte header once per block, 32 bytes per stage) and
//               writes the dequantized bf16/f16 row of the stage straight into
//               the UMMA K-major SWIZZLE_128B layout; then the epilogue
//               (tcgen05.ld 32x32b, convert, 16-byte stores);
//   warp 10     Q4_K with contiguous weight rows: TMA of the raw bytes (the
//               stage's 32-byte quant chunk of 256 rows, the 16-byte block
//               headers once per block) into shared rings several stages
//               ahead, so the dequantizing warps never wait on global loads.
// Weights are rounded to the activation type before the MMA (the tolerance of
// the matmul outputs covers it; the exact dequantization is kq_dequantize).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "kq_internal.cuh"
#include "kq_ptx.cuh"

namespace kq {
namespace {

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int GT = 352;  // threads (11 warps)
constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2;

// raw Q4_K rings of the TMA-fed mode: RS stages of 32-byte quant chunks and
// HS blocks of 16-byte headers, 256 rows each
constexpr int RS = 3, HS = 2, QS_BYTES = BN * 32, HDR_BYTES = BN * 16;

// MT activation-row tiles of 128 per CTA (MT accumulators of 256 TMEM columns
// each): with MT = 2 every dequantized weight tile feeds twice the MMA work.
template <int MT, bool RAW = false> struct GL {
    static constexpr int NSTAGE = MT == 1 ? 4 : 3;
    static constexpr int STAGE_A = MT * A_BYTES;
    static constexpr int OFF_A = 0, OFF_B = NSTAGE * STAGE_A, OFF_RAW = OFF_B + NSTAGE * B_BYTES;
    static constexpr int OFF_HDR = OFF_RAW + RS * QS_BYTES;
    static constexpr int OFF_BAR = OFF_RAW + (RAW ? RS * QS_BYTES + HS * HDR_BYTES : 0);
    static constexpr int SMEM = OFF_BAR + 256 + 1024;  // + 1 KB for base alignment
    static constexpr int TMEM_COLS = MT * BN;
    static_assert(SMEM <= 232448, "shared memory per CTA");
};

// B_Q4K: Q4_K dequantized from global loads; B_TMA: dequantized copy by TMA;
// B_Q4KT: Q4_K dequantized from raw bytes brought in by TMA
enum BMode : int { B_Q4K = 0, B_TMA = 1, B_Q4KT = 2 };

__device__ __forceinline__ uint64_t gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ bool wait_b(uint64_t *bar, uint32_t par, volatile int *abort, int *err, int code) {
    uint64_t t0 = 0;  // timer read every 1024 polls only (a %globaltimer read is slow)
    for (uint32_t i = 1;; i++) {
        if (mbar_try_wait(bar, par)) return true;
        if ((i & 1023) == 0) {
            if (*abort) return false;
            const uint64_t now = gtimer();
            if (t0 == 0) t0 = now;
            if (now - t0 > 2000000000ull) {
                *abort = 1;
                atomicCAS(err, 0, code);
                return false;
            }
        }
    }
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int c0, int c1, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}

// UMMA shared-memory descriptor: K-major, SWIZZLE_128B, 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFF) >> 4) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

template <bool F16> __device__ __forceinline__ uint32_t idesc() {
    const uint32_t fmt = F16 ? 0u : 1u;
    return (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void umma(uint32_t tmem, uint64_t da, uint64_t db, uint32_t id, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
        "l"(da), "l"(db), "r"(id), "r"(acc)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void fence_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t r[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%"
        "19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

template <bool F16> __device__ __forceinline__ uint32_t pack2(float a, float b) {
    if constexpr (F16) {
        __half2 h = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t *>(&h);
    } else {
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t *>(&h);
    }
}

// (q pair as magic-offset 16-bit floats) -> d*q - m, one rounding (packed FMA)
template <bool F16> __device__ __forceinline__ uint32_t q4_pair(uint32_t nib2, uint32_t dsc2, uint32_t ndm2) {
    uint32_t r;
    if constexpr (F16) {
        __half2 q = __hsub2(*reinterpret_cast<__half2 *>(&nib2), __float2half2_rn(1024.f));
        __half2 o = __hfma2(q, *reinterpret_cast<__half2 *>(&dsc2), *reinterpret_cast<__half2 *>(&ndm2));
        r = *reinterpret_cast<uint32_t *>(&o);
    } else {
        __nv_bfloat162 q = __hsub2(*reinterpret_cast<__nv_bfloat162 *>(&nib2), __float2bfloat162_rn(128.f));
        __nv_bfloat162 o =
            __hfma2(q, *reinterpret_cast<__nv_bfloat162 *>(&dsc2), *reinterpret_cast<__nv_bfloat162 *>(&ndm2));
        r = *reinterpret_cast<uint32_t *>(&o);
    }
    return r;
}

// GLU: the 256-row weight tile is 128 gate rows over 128 up rows of the same
// output columns; accumulator columns [0,128) hold x.Wg, [128,256) x.Wu and the
// epilogue writes act(g) * u for 128 output columns.
template <bool F16, int BMODE, int MT, bool GLU, bool SPLIT = false>
__global__ void __launch_bounds__(GT, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmH,
                const __grid_constant__ CUtensorMap tmQ2, const __grid_constant__ CUtensorMap tmH2, const GemmArgs a) {
    using L = GL<MT, BMODE == B_Q4KT>;
    constexpr int NSTAGE = L::NSTAGE, OFF_A = L::OFF_A, OFF_B = L::OFF_B, OFF_BAR = L::OFF_BAR;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t *fullA = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
    uint64_t *fullB = fullA + NSTAGE;
    uint64_t *empty = fullB + NSTAGE;
    uint64_t *accbar = empty + NSTAGE;
    uint64_t *rawFull = accbar + 1, *rawEmpty = rawFull + RS, *hdrFull = rawEmpty + RS, *hdrEmpty = hdrFull + HS;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(hdrEmpty + HS);
    volatile int *s_abort = reinterpret_cast<volatile int *>(tmem_slot + 1);
    volatile int *s_last = reinterpret_cast<volatile int *>(tmem_slot + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int NOUT = GLU ? BN / 2 : BN;  // output columns per CTA
    const int n0 = blockIdx.y * NOUT;
    const int nk = a.K / BK;
    // split-K (dense plain GEMM only, its own instantiation so the other
    // kernels compile without it): this CTA covers stages [ks0, ks0 + nkl)
    static_assert(!SPLIT || !GLU, "split-K is for plain GEMMs");
    const int nsplit = SPLIT ? 2 : 1;
    const int nkl = SPLIT ? nk / 2 : nk, ks0 = SPLIT ? (int)blockIdx.z * nkl : 0;
    int m0 = blockIdx.x * BM * MT, mend = a.M, ex = 0;
    if (a.n_tiles) {  // grouped: this CTA's (expert, row range) from the device tile table
        if ((int)blockIdx.x >= *a.n_tiles) return;
        ex = a.tile_e[blockIdx.x];
        if (ex < a.ex_lo || ex >= a.ex_hi) return;
        m0 = a.tile_row0[blockIdx.x];
        mend = a.tile_rowend[blockIdx.x];
    }
    // row tiles with rows to compute (a grouped tile's second half may be empty)
    const int mt_live = (MT == 1 || m0 + BM < mend) ? MT : 1;

    if (threadIdx.x == 0) {
        for (int i = 0; i < NSTAGE; i++) {
            mbar_init(&fullA[i], 1);
            mbar_init(&fullB[i], 8);
            mbar_init(&empty[i], 1);
        }
        mbar_init(accbar, 1);
        for (int i = 0; i < RS; i++) {
            mbar_init(&rawFull[i], 1);
            mbar_init(&rawEmpty[i], 8);
        }
        for (int i = 0; i < HS; i++) {
            mbar_init(&hdrFull[i], 1);
            mbar_init(&hdrEmpty[i], 8);
        }
        *s_abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(L::TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            const uint32_t tx = mt_live * A_BYTES + (BMODE == B_TMA ? B_BYTES : 0);
            for (int s = 0; s < nkl; s++) {
                const int slot = s % NSTAGE, kx = (ks0 + s) * BK;
                wait_b(&empty[slot], ((s / NSTAGE) & 1) ^ 1, s_abort, a.err, 11);
                mbar_arrive_expect_tx(&fullA[slot], tx);
                if (*s_abort) continue;
#pragma unroll
                for (int t = 0; t < MT; t++)
                    if (t < mt_live)
                        tma_load_2d(smem + OFF_A + slot * L::STAGE_A + t * A_BYTES, &tmA, kx, m0 + t * BM,
                                    &fullA[slot]);
                if (BMODE == B_TMA) {
                    const int rb = (ex - a.ex_lo) * a.n_per_expert + n0;
                    tma_load_2d(smem + OFF_B + slot * B_BYTES, &tmB, kx, rb, &fullA[slot]);
                    if (GLU)  // up rows: second half of the dequantized scratch
                        tma_load_2d(smem + OFF_B + slot * B_BYTES + B_BYTES / 2, &tmB, kx,
                                    rb + (a.ex_hi - a.ex_lo) * a.n_per_expert, &fullA[slot]);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t id = idesc<F16>();
            for (int s = 0; s < nkl; s++) {
                const int slot = s % NSTAGE, par = (s / NSTAGE) & 1;
                wait_b(&fullA[slot], par, s_abort, a.err, 12);
                if (BMODE != B_TMA) wait_b(&fullB[slot], par, s_abort, a.err, 13);
                tc_fence_after();
                const uint32_t sa = smem_u32(smem + OFF_A + slot * L::STAGE_A);
                const uint32_t sb = smem_u32(smem + OFF_B + slot * B_BYTES);
#pragma unroll
                for (int t = 0; t < MT; t++)
#pragma unroll
                    for (int kk = 0; kk < BK / 16; kk++)
                        if (t < mt_live && !*s_abort)
                            umma(tmem + t * BN, umma_desc(sa + t * A_BYTES + kk * 32), umma_desc(sb + kk * 32), id,
                                 (s | kk) ? 1u : 0u);
                umma_commit(&empty[slot]);
            }
            umma_commit(accbar);
        }
    } else if (warp == 10) {
        if constexpr (BMODE == B_Q4KT) {
            if (lane == 0) {  // raw Q4_K bytes: rows [rb, rb + 256) (GLU: 128 gate rows over 128 up rows)
                const int rb = ex * a.n_per_expert + n0;
                for (int s = 0; s < nkl; s++) {
                    const int r = s % RS, b = (ks0 + s) >> 2, q = s & 3, bl = s >> 2;  // ks0 % 4 == 0
                    if (q == 0) {
                        const int h = bl % HS;
                        wait_b(&hdrEmpty[h], ((bl / HS) & 1) ^ 1, s_abort, a.err, 16);
                        mbar_arrive_expect_tx(&hdrFull[h], HDR_BYTES);
                        if (!*s_abort) {
                            uint8_t *dst = smem + L::OFF_HDR + h * HDR_BYTES;
                            tma_load_2d(dst, &tmH, b * 144, rb, &hdrFull[h]);
                            tma_load_2d(dst + HDR_BYTES / 2, GLU ? &tmH2 : &tmH, b * 144, GLU ? rb : rb + 128,
                                        &hdrFull[h]);
                        }
                    }
                    wait_b(&rawEmpty[r], ((s / RS) & 1) ^ 1, s_abort, a.err, 17);
                    mbar_arrive_expect_tx(&rawFull[r], QS_BYTES);
                    if (!*s_abort) {
                        uint8_t *dst = smem + L::OFF_RAW + r * QS_BYTES;
                        tma_load_2d(dst, &tmQ, b * 144 + 16 + 32 * q, rb, &rawFull[r]);
                        tma_load_2d(dst + QS_BYTES / 2, GLU ? &tmQ2 : &tmQ, b * 144 + 16 + 32 * q, GLU ? rb : rb + 128,
                                    &rawFull[r]);
                    }
                }
            }
        }
    } else {
        const int i = threadIdx.x - 64;  // 0..255: weight row of the tile
        if constexpr (BMODE == B_Q4KT) {
            uint32_t dsc2[8], ndm2[8];
            for (int s0 = 0; s0 < nkl; s0 += 4)  // nkl is a multiple of 4 (K % 256 == 0)
#pragma unroll
            for (int q = 0; q < 4; q++) {  // static q: dsc2[] / ndm2[] stay in registers
                const int s = s0 + q, slot = s % NSTAGE, r = s % RS;
                if (q == 0) {  // new super-block: 8 x (d*sc, -dmin*m) as packed 16-bit pairs
                    const int b = s >> 2, h = b % HS;
                    wait_b(&hdrFull[h], (b / HS) & 1, s_abort, a.err, 18);
                    const uint4 hv = *reinterpret_cast<const uint4 *>(smem + L::OFF_HDR + h * HDR_BYTES + i * 16);
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&hdrEmpty[h]);
                    const float d = half_bits_to_float(hv.x & 0xffffu), dmin = half_bits_to_float(hv.x >> 16);
                    uint32_t sc03, sc47, m03, m47;
                    q4k_unpack_scales(hv.y, hv.z, hv.w, sc03, sc47, m03, m47);
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        const float ds = d * (float)((((j < 4) ? sc03 : sc47) >> (8 * (j & 3))) & 63u);
                        const float dm = dmin * (float)((((j < 4) ? m03 : m47) >> (8 * (j & 3))) & 63u);
                        dsc2[j] = pack2<F16>(ds, ds);
                        ndm2[j] = pack2<F16>(-dm, -dm);
                    }
                }
                wait_b(&rawFull[r], (s / RS) & 1, s_abort, a.err, 19);
                const uint8_t *src = smem + L::OFF_RAW + r * QS_BYTES + i * 32;
                const uint4 c0 = *reinterpret_cast<const uint4 *>(src), c1 = *reinterpret_cast<const uint4 *>(src + 16);
                __syncwarp();
                if (lane == 0) mbar_arrive(&rawEmpty[r]);
                const uint32_t wds[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
                wait_b(&empty[slot], ((s / NSTAGE) & 1) ^ 1, s_abort, a.err, 14);
                uint8_t *dst = smem + OFF_B + slot * B_BYTES + (i >> 3) * 1024 + (i & 7) * 128;
                const uint32_t magic = F16 ? 0x64006400u : 0x43004300u;
#ifdef KQ_DEVELOPMENT
                if (a.debug & 4) {  // development: no stores
                } else if (a.debug & 1) {  // development: store without decoding
#pragma unroll
                    for (int c = 0; c < 8; c++)
                        *reinterpret_cast<uint4 *>(dst + ((c ^ (i & 7)) << 4)) = make_uint4(wds[c], wds[c], 0, 0);
                } else
#endif
#pragma unroll
                for (int c = 0; c < 8; c++) {  // 16-byte chunk c = k 8c..8c+7 of the stage
                    const int hh = c >> 2, j = 2 * q + hh;
                    const uint32_t w0 = wds[2 * (c & 3)] >> (4 * hh), w1 = wds[2 * (c & 3) + 1] >> (4 * hh);
                    uint4 o;
                    o.x = q4_pair<F16>(lop_and_or(prmt(w0, 0, 0x4140), 0x000f000fu, magic), dsc2[j], ndm2[j]);
                    o.y = q4_pair<F16>(lop_and_or(prmt(w0, 0, 0x4342), 0x000f000fu, magic), dsc2[j], ndm2[j]);
                    o.z = q4_pair<F16>(lop_and_or(prmt(w1, 0, 0x4140), 0x000f000fu, magic), dsc2[j], ndm2[j]);
                    o.w = q4_pair<F16>(lop_and_or(prmt(w1, 0, 0x4342), 0x000f000fu, magic), dsc2[j], ndm2[j]);
                    *reinterpret_cast<uint4 *>(dst + ((c ^ (i & 7)) << 4)) = o;
                }
#ifdef KQ_DEVELOPMENT
                if (!(a.debug & 2))  // development: no proxy fence
#endif
                    fence_async_shared();
                __syncwarp();
                if (lane == 0) mbar_arrive(&fullB[slot]);
            }
        }
        if constexpr (BMODE == B_Q4K) {
            const int n = n0 + (GLU ? (i & 127) : i);
            const bool valid = n < a.N;
            const uint8_t *wb = (GLU && i >= 128) ? a.w2 : a.w;
            const uint8_t *row = wb + (int64_t)ex * a.w_expert_stride + (int64_t)(valid ? n : 0) * a.w_row_stride +
                                 (int64_t)(ks0 >> 2) * 144;
            uint32_t dsc2[8], ndm2[8];
            // loads run one stage ahead of the decode (header of the next block, next chunk)
            uint4 nh = __ldg(reinterpret_cast<const uint4 *>(row));
            uint4 n0c = __ldg(reinterpret_cast<const uint4 *>(row + 16));
            uint4 n1c = __ldg(reinterpret_cast<const uint4 *>(row + 32));
            for (int s0 = 0; s0 < nkl; s0 += 4)  // nkl is a multiple of 4 (K % 256 == 0)
#pragma unroll
            for (int q = 0; q < 4; q++) {  // static q: dsc2[] / ndm2[] stay in registers
                const int s = s0 + q, slot = s % NSTAGE;
                const uint4 hcur = nh, c0 = n0c, c1 = n1c;
                if (s + 1 < nkl) {
                    const int b1 = (s + 1) >> 2, q1 = (s + 1) & 3;
                    if (q1 == 0) nh = __ldg(reinterpret_cast<const uint4 *>(row + (int64_t)b1 * 144));
                    n0c = __ldg(reinterpret_cast<const uint4 *>(row + (int64_t)b1 * 144 + 16 + 32 * q1));
                    n1c = __ldg(reinterpret_cast<const uint4 *>(row + (int64_t)b1 * 144 + 32 + 32 * q1));
                }
                if (q == 0) {  // new super-block: 8 x (d*sc, -dmin*m) as packed 16-bit pairs
                    const uint4 hv = hcur;
                    const float d = half_bits_to_float(hv.x & 0xffffu), dmin = half_bits_to_float(hv.x >> 16);
                    uint32_t sc03, sc47, m03, m47;
                    q4k_unpack_scales(hv.y, hv.z, hv.w, sc03, sc47, m03, m47);
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        const float ds = d * (float)((((j < 4) ? sc03 : sc47) >> (8 * (j & 3))) & 63u);
                        const float dm = dmin * (float)((((j < 4) ? m03 : m47) >> (8 * (j & 3))) & 63u);
                        dsc2[j] = pack2<F16>(ds, ds);
                        ndm2[j] = pack2<F16>(-dm, -dm);
                    }
                }
                const uint32_t wds[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
                wait_b(&empty[slot], ((s / NSTAGE) & 1) ^ 1, s_abort, a.err, 14);
                uint8_t *dst = smem + OFF_B + slot * B_BYTES + (i >> 3) * 1024 + (i & 7) * 128;
                const uint32_t magic = F16 ? 0x64006400u : 0x43004300u;
#pragma unroll
                for (int c = 0; c < 8; c++) {  // 16-byte chunk c = k 8c..8c+7 of the stage
                    const int h = c >> 2, j = 2 * q + h;
                    const uint32_t w0 = wds[2 * (c & 3)] >> (4 * h), w1 = wds[2 * (c & 3) + 1] >> (4 * h);
                    uint4 o;
                    o.x = q4_pair<F16>(lop_and_or(prmt(w0, 0, 0x4140), 0x000f000fu, magic), dsc2[j], ndm2[j]);
                    o.y = q4_pair<F16>(lop_and_or(prmt(w0, 0, 0x4342), 0x000f000fu, magic), dsc2[j], ndm2[j]);
                    o.z = q4_pair<F16>(lop_and_or(prmt(w1, 0, 0x4140), 0x000f000fu, magic), dsc2[j], ndm2[j]);
                    o.w = q4_pair<F16>(lop_and_or(prmt(w1, 0, 0x4342), 0x000f000fu, magic), dsc2[j], ndm2[j]);
                    if (!valid) o = make_uint4(0, 0, 0, 0);
                    *reinterpret_cast<uint4 *>(dst + ((c ^ (i & 7)) << 4)) = o;
                }
                fence_async_shared();
                __syncwarp();
                if (lane == 0) mbar_arrive(&fullB[slot]);
            }
        }
        // ---- epilogue: TMEM lane quarter = warp % 4; two warps per quarter split the columns
        wait_b(accbar, 0, s_abort, a.err, 15);
        tc_fence_after();
        const int quarter = warp & 3, chalf = (warp - 2) >> 2;
        if constexpr (SPLIT) {
            // split-K: post this split's f32 partial tile; the last split of the
            // tile to finish adds the other one (a + b == b + a: deterministic)
            float *mine = a.part + (int64_t)blockIdx.z * a.M * a.N;
#pragma unroll 1
            for (int q32 = 0; q32 < mt_live * (NOUT / 2); q32 += 32) {
                const int t = q32 / (NOUT / 2), cc = q32 % (NOUT / 2);
                const int tok = m0 + t * BM + quarter * 32 + lane;
                const int col = chalf * (NOUT / 2) + cc;
                uint32_t r[32];
                tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(t * BN + col), r);
                if (tok >= mend || *s_abort) continue;
                const int nb = n0 + col;
                float *pp = mine + (int64_t)tok * a.N + nb;
                if (nb + 32 <= a.N && ((uintptr_t)pp & 15) == 0) {
#pragma unroll
                    for (int v = 0; v < 8; v++)
                        reinterpret_cast<float4 *>(pp)[v] =
                            make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                        __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
                } else {
#pragma unroll
                    for (int v = 0; v < 32; v++)
                        if (nb + v < a.N) pp[v] = __uint_as_float(r[v]);
                }
            }
            named_bar_sync(1, 256);
            if (threadIdx.x == 64) {
                __threadfence();
                int *cnt = a.tile_cnt + blockIdx.y * gridDim.x + blockIdx.x;
                const int last = atomicAdd(cnt, 1) == nsplit - 1;
                if (last) *cnt = 0;  // counters are left zero
                *s_last = last;
            }
            named_bar_sync(1, 256);
            __threadfence();
            const float *other = a.part + (int64_t)(1 - (int)blockIdx.z) * a.M * a.N;
#pragma unroll 1
            for (int q32 = 0; q32 < (*s_last ? mt_live * (NOUT / 2) : 0); q32 += 32) {
                const int t = q32 / (NOUT / 2), cc = q32 % (NOUT / 2);
                const int tok = m0 + t * BM + quarter * 32 + lane;
                const int col = chalf * (NOUT / 2) + cc;
                uint32_t r[32];
                tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(t * BN + col), r);
                if (tok >= mend || *s_abort) continue;
                const int nb = n0 + col;
                const float *op = other + (int64_t)tok * a.N + nb;
                float v[32];
#pragma unroll
                for (int j = 0; j < 32; j++) v[j] = __uint_as_float(r[j]) + (nb + j < a.N ? __ldcg(op + j) : 0.f);
                if (a.y_dtype == F32) {
                    float *yp = reinterpret_cast<float *>(a.y) + (int64_t)tok * a.y_row_stride + nb;
#pragma unroll
                    for (int j = 0; j < 32; j++)
                        if (nb + j < a.N) yp[j] = v[j];
                } else {
                    const bool of16 = a.y_dtype == F16;
                    uint16_t *yp = reinterpret_cast<uint16_t *>(a.y) + (int64_t)tok * a.y_row_stride + nb;
                    uint32_t pk[16];
#pragma unroll
                    for (int j = 0; j < 16; j++) pk[j] = of16 ? pack2<true>(v[2 * j], v[2 * j + 1]) : pack2<false>(v[2 * j], v[2 * j + 1]);
                    if (nb + 32 <= a.N && ((uintptr_t)yp & 15) == 0) {
#pragma unroll
                        for (int j = 0; j < 4; j++)
                            reinterpret_cast<uint4 *>(yp)[j] = make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; j++)
                            if (nb + j < a.N) yp[j] = (uint16_t)(pk[j >> 1] >> (16 * (j & 1)));
                    }
                }
            }
        }
#pragma unroll 1
        for (int q32 = 0; q32 < (SPLIT ? 0 : mt_live * (NOUT / 2)); q32 += 32) {
            const int t = q32 / (NOUT / 2), cc = q32 % (NOUT / 2);
            const int tok = m0 + t * BM + quarter * 32 + lane;
            const int col = chalf * (NOUT / 2) + cc;
            uint32_t r[32];
            tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(t * BN + col), r);
            if constexpr (GLU) {
                uint32_t u[32];
                tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(t * BN + BN / 2 + col), u);
#pragma unroll
                for (int v = 0; v < 32; v++)
                    r[v] = __float_as_uint(apply_act(a.act, __uint_as_float(r[v])) * __uint_as_float(u[v]));
            }
            if (tok >= mend || *s_abort) continue;
            const int64_t orow = a.out_row ? (int64_t)a.out_row[tok] : (int64_t)tok;
            const int nb = n0 + col;
            if (a.row_scale) {  // y[out_row] += scale * row (f32; several rows add into one output row)
                const float sc = a.row_scale[tok];
                float *yp = reinterpret_cast<float *>(a.y) + orow * a.y_row_stride + nb;
                if (nb + 32 <= a.N && ((uintptr_t)yp & 15) == 0) {
#pragma unroll
                    for (int v = 0; v < 8; v++)
                        atomicAdd(reinterpret_cast<float4 *>(yp) + v,
                                  make_float4(sc * __uint_as_float(r[4 * v]), sc * __uint_as_float(r[4 * v + 1]),
                                              sc * __uint_as_float(r[4 * v + 2]), sc * __uint_as_float(r[4 * v + 3])));
                } else {
#pragma unroll
                    for (int v = 0; v < 32; v++)
                        if (nb + v < a.N) atomicAdd(yp + v, sc * __uint_as_float(r[v]));
                }
            } else if (a.y_dtype == F32) {
                float *yp = reinterpret_cast<float *>(a.y) + orow * a.y_row_stride + nb;
                if (nb + 32 <= a.N && ((uintptr_t)yp & 15) == 0) {
#pragma unroll
                    for (int v = 0; v < 8; v++)
                        reinterpret_cast<float4 *>(yp)[v] =
                            make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                        __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
                } else {  // ragged edge (static indices keep r[] in registers)
#pragma unroll
                    for (int v = 0; v < 32; v++)
                        if (nb + v < a.N) yp[v] = __uint_as_float(r[v]);
                }
            } else {
                const bool of16 = a.y_dtype == F16;
                uint16_t *yp = reinterpret_cast<uint16_t *>(a.y) + orow * a.y_row_stride + nb;
                uint32_t pk[16];
#pragma unroll
                for (int v = 0; v < 16; v++) {
                    const float f0 = __uint_as_float(r[2 * v]), f1 = __uint_as_float(r[2 * v + 1]);
                    pk[v] = of16 ? pack2<true>(f0, f1) : pack2<false>(f0, f1);
                }
                if (nb + 32 <= a.N && ((uintptr_t)yp & 15) == 0) {
#pragma unroll
                    for (int v = 0; v < 4; v++)
                        reinterpret_cast<uint4 *>(yp)[v] = make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
                } else {  // ragged edge (static indices keep pk[] in registers)
#pragma unroll
                    for (int v = 0; v < 32; v++)
                        if (nb + v < a.N) yp[v] = (uint16_t)(pk[v >> 1] >> (16 * (v & 1)));
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(L::TMEM_COLS));
    }
}

// ---------------------------------------------------------------------------
// host: tensor maps through the driver entry point (no -lcuda link needed)

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

bool make_map(CUtensorMap *m, const void *base, bool f16, int64_t rows, int64_t cols, int64_t row_stride_elems,
              int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)row_stride_elems * 2};
    const cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
    const cuuint32_t es[2] = {1, 1};
    return fn(m, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base),
              dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Raw Q4_K weight bytes as 2-D uint8 tensors [rows, row bytes] (row stride a
// multiple of 16, base 16-byte aligned): boxes of 32 (quant chunk) and 16
// (block header) bytes x 128 rows; rows past the end read as zeros.
bool make_raw_map(CUtensorMap *m, const void *base, int64_t rows, int64_t row_bytes, int64_t row_stride, int box_bytes) {
    EncodeTiledFn fn = encode_fn();
    if (!fn || ((uintptr_t)base & 15) || (row_stride & 15)) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)row_stride};
    const cuuint32_t box[2] = {(cuuint32_t)box_bytes, 128u};
    const cuuint32_t es[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// the four raw maps (gate/plain quant + header, up quant + header) over `rows` weight rows
bool make_raw_maps(const GemmArgs &a, int64_t rows, CUtensorMap *q, CUtensorMap *h, CUtensorMap *q2, CUtensorMap *h2) {
    const int64_t rb = (int64_t)a.K / QK * 144;
    if (!make_raw_map(q, a.w, rows, rb, a.w_row_stride, 32) || !make_raw_map(h, a.w, rows, rb, a.w_row_stride, 16))
        return false;
    if (!a.w2) {
        *q2 = *q;
        *h2 = *h;
        return true;
    }
    return make_raw_map(q2, a.w2, rows, rb, a.w_row_stride, 32) && make_raw_map(h2, a.w2, rows, rb, a.w_row_stride, 16);
}

// TMA-fed Q4_K needs 16-byte aligned weight bases and row strides (Q4_K rows
// are 144-byte multiples, so every contiguous Q4_K tensor qualifies) and, for
// expert stacks, rows of all experts equally spaced
static bool raw_tma_ok(const GemmArgs &a, bool contiguous_experts) {
    if (dev_env("KQ_GEMM_NO_RAW_TMA")) return false;  // development switch
    return contiguous_experts && !(((uintptr_t)a.w | (uintptr_t)(a.w2 ? a.w2 : a.w) | (uintptr_t)a.w_row_stride) & 15);
}

template <bool F16, int BMODE, int MT, bool GLU = false, bool SPLIT = false>
cudaError_t launch_gemm_t(const GemmArgs &a, const void *bdense, cudaStream_t st) {
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(gemm_kernel<F16, BMODE, MT, GLU, SPLIT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             GL<MT, BMODE == B_Q4KT>::SMEM);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    CUtensorMap ta, tb, tq, th, tq2, th2;
    if (!make_map(&ta, a.x, F16, a.M, a.K, a.x_row_stride, BM)) return cudaErrorInvalidValue;
    if (BMODE == B_TMA) {
        if (!make_map(&tb, bdense, F16, (int64_t)a.N * (GLU ? 2 : 1), a.K, a.K, GLU ? BN / 2 : BN))
            return cudaErrorInvalidValue;
    } else {
        tb = ta;
    }
    if (BMODE == B_Q4KT) {
        if (!make_raw_maps(a, a.N, &tq, &th, &tq2, &th2)) return cudaErrorInvalidValue;
    } else {
        tq = th = tq2 = th2 = ta;
    }
    constexpr int NOUT = GLU ? BN / 2 : BN;
    dim3 grid((a.M + BM * MT - 1) / (BM * MT), (a.N + NOUT - 1) / NOUT, SPLIT ? 2 : 1);
    gemm_kernel<F16, BMODE, MT, GLU, SPLIT><<<grid, GT, GL<MT, BMODE == B_Q4KT>::SMEM, st>>>(ta, tb, tq, th, tq2, th2, a);
    return cudaGetLastError();
}

template <bool F16, int BMODE, bool GLU = false>
cudaError_t launch_gemm_mt(const GemmArgs &a, const void *bdense, cudaStream_t st) {
    // two activation-row tiles per CTA once there are enough CTAs to fill the GPU
    constexpr int NOUT = GLU ? BN / 2 : BN;
    const long ctas2 = (long)((a.M + 2 * BM - 1) / (2 * BM)) * ((a.N + NOUT - 1) / NOUT);
    if constexpr (!GLU && BMODE == B_TMA)  // split-K: the dequantized-copy path only
        if (a.ksplit == 2) return launch_gemm_t<F16, BMODE, 1, false, true>(a, bdense, st);
    if (ctas2 >= num_sms()) return launch_gemm_t<F16, BMODE, 2, GLU>(a, bdense, st);
    return launch_gemm_t<F16, BMODE, 1, GLU>(a, bdense, st);
}

template <bool F16, int BMODE, int MT, bool GLU>
cudaError_t launch_grouped_t(const GemmArgs &a, int max_tiles, const void *bdense, cudaStream_t st) {
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(gemm_kernel<F16, BMODE, MT, GLU>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             GL<MT, BMODE == B_Q4KT>::SMEM);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    CUtensorMap ta, tb, tq, th, tq2, th2;
    if (!make_map(&ta, a.x, F16, a.M, a.K, a.x_row_stride, BM)) return cudaErrorInvalidValue;
    if (BMODE == B_TMA) {
        const int64_t brows = (int64_t)(a.ex_hi - a.ex_lo) * a.n_per_expert * (GLU ? 2 : 1);
        if (!make_map(&tb, bdense, F16, brows, a.K, a.K, GLU ? BN / 2 : BN)) return cudaErrorInvalidValue;
    } else {
        tb = ta;
    }
    if (BMODE == B_Q4KT) {  // expert stacks of contiguous rows: one [experts * N, row bytes] tensor
        if (!make_raw_maps(a, (int64_t)a.ex_hi * a.n_per_expert, &tq, &th, &tq2, &th2)) return cudaErrorInvalidValue;
    } else {
        tq = th = tq2 = th2 = ta;
    }
    if (max_tiles <= 0) return cudaSuccess;
    const int nout = GLU ? BN / 2 : BN;
    dim3 grid(max_tiles, (a.N + nout - 1) / nout);
    gemm_kernel<F16, BMODE, MT, GLU><<<grid, GT, GL<MT, BMODE == B_Q4KT>::SMEM, st>>>(ta, tb, tq, th, tq2, th2, a);
    return cudaGetLastError();
}

template <bool F16, int BMODE, bool GLU>
cudaError_t launch_grouped_mt(const GemmArgs &a, int mt, int max_tiles, const void *bdense, cudaStream_t st) {
    return mt == 2 ? launch_grouped_t<F16, BMODE, 2, GLU>(a, max_tiles, bdense, st)
                   : launch_grouped_t<F16, BMODE, 1, GLU>(a, max_tiles, bdense, st);
}

template <bool F16, int BMODE>
cudaError_t launch_grouped_glu(const GemmArgs &a, int mt, int max_tiles, const void *bdense, cudaStream_t st) {
    return a.w2 || (BMODE == B_TMA && a.act != ACT_NONE) ? launch_grouped_mt<F16, BMODE, true>(a, mt, max_tiles, bdense, st)
                                                           : launch_grouped_mt<F16, BMODE, false>(a, mt, max_tiles, bdense, st);
}

// ---- MoE routing helpers for the grouped path (three parallel passes)

// pass 1: rank of every local slot within its expert (order within an expert
// is arbitrary; each output row depends only on its own slot)
__global__ void rank_kernel(const int32_t *__restrict__ idx, int S, int ebase, int ecount, int etotal,
                            int *__restrict__ cnt, int *__restrict__ rank, int *err) {
    const int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= S) return;
    const int g = idx[s];
    if (g < 0 || g >= etotal) atomicCAS(err, 0, 3);  // expert id out of range (as the GEMV grouping)
    const int e = g - ebase;
    rank[s] = (e >= 0 && e < ecount) ? atomicAdd(&cnt[e], 1) : -1;
}

// pass 2 (one CTA): expert offsets and the (expert, row tile) table; resets
// the counts so the counter region is left zero
__global__ void table_kernel(int ecount, int tile_rows, int *__restrict__ cnt, int *__restrict__ off,
                             int *__restrict__ total, int *__restrict__ n_tiles, int *__restrict__ tile_e,
                             int *__restrict__ tile_row0, int *__restrict__ tile_rowend, int max_tiles, int *err) {
    __shared__ int s_wsum[2][32];
    const int e = threadIdx.x, lane = e & 31, w = e >> 5;
    const int c = e < ecount ? cnt[e] : 0;
    if (e < ecount) cnt[e] = 0;
    const int nt = (c + tile_rows - 1) / tile_rows;
    // block-wide inclusive scans of rows and tiles
    int rc = c, rt = nt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int a = __shfl_up_sync(0xffffffffu, rc, o), b = __shfl_up_sync(0xffffffffu, rt, o);
        if (lane >= o) rc += a, rt += b;
    }
    if (lane == 31) s_wsum[0][w] = rc, s_wsum[1][w] = rt;
    __syncthreads();
    if (w == 0) {
        int a = s_wsum[0][lane], b = s_wsum[1][lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int x = __shfl_up_sync(0xffffffffu, a, o), y = __shfl_up_sync(0xffffffffu, b, o);
            if (lane >= o) a += x, b += y;
        }
        s_wsum[0][lane] = a, s_wsum[1][lane] = b;
    }
    __syncthreads();
    const int r0 = rc - c + (w ? s_wsum[0][w - 1] : 0), t0 = rt - nt + (w ? s_wsum[1][w - 1] : 0);
    if (e < ecount) {
        off[e] = r0;
        for (int j = 0; j < nt; j++)
            if (t0 + j < max_tiles) {
                tile_e[t0 + j] = e;
                tile_row0[t0 + j] = r0 + j * tile_rows;
                tile_rowend[t0 + j] = r0 + c;
            }
    }
    if (e == blockDim.x - 1) {
        const int all_t = t0 + nt;
        if (all_t > max_tiles) atomicCAS(err, 0, 6);
        *n_tiles = all_t < max_tiles ? all_t : max_tiles;
        *total = r0 + c;
    }
}

// pass 3: slot -> sorted row; copy the slot's activation row there
__global__ void scatter_rows_kernel(const int32_t *__restrict__ idx, const int *__restrict__ rank,
                                    const int *__restrict__ off, int ebase, int k, int xrow_is_slot,
                                    const int32_t *__restrict__ xidx, const uint16_t *__restrict__ x, int64_t xs_stride,
                                    int K, int *__restrict__ perm, uint16_t *__restrict__ out,
                                    const float *__restrict__ scores, int *__restrict__ tok_of,
                                    float *__restrict__ scale_of) {
    const int s = blockIdx.x;
    const int r = rank[s];
    if (r < 0) return;
    const int p = off[idx[s] - ebase] + r;
    if (threadIdx.x == 0) {
        perm[p] = s;
        if (scores) {  // mixed output: sorted row p adds score * row into token s / k
            tok_of[p] = s / k;
            scale_of[p] = scores[s];
        }
    }
    const int xr = xidx ? xidx[s] : xrow_is_slot ? s : s / k;
    const uint4 *src = reinterpret_cast<const uint4 *>(x + (int64_t)xr * xs_stride);
    uint4 *dst = reinterpret_cast<uint4 *>(out + (int64_t)p * K);
    for (int i = threadIdx.x; i < K / 8; i += blockDim.x) dst[i] = src[i];
}

}  // namespace

cudaError_t launch_gemm_grouped(const GemmArgs &a, int mt, int max_tiles, const void *b_dense, cudaStream_t st) {
    const bool f16 = a.x_dtype == F16;
    if (!b_dense && raw_tma_ok(a, a.w_expert_stride == (int64_t)a.n_per_expert * a.w_row_stride))
        return f16 ? launch_grouped_glu<true, B_Q4KT>(a, mt, max_tiles, nullptr, st)
                   : launch_grouped_glu<false, B_Q4KT>(a, mt, max_tiles, nullptr, st);
    if (!b_dense)
        return f16 ? launch_grouped_glu<true, B_Q4K>(a, mt, max_tiles, nullptr, st)
                   : launch_grouped_glu<false, B_Q4K>(a, mt, max_tiles, nullptr, st);
    return f16 ? launch_grouped_glu<true, B_TMA>(a, mt, max_tiles, b_dense, st)
               : launch_grouped_glu<false, B_TMA>(a, mt, max_tiles, b_dense, st);
}

cudaError_t launch_moe_sort(const int32_t *idx, int S, int k, int ebase, int ecount, int etotal, int xrow_is_slot,
                            const int32_t *xidx, const void *x, int64_t x_row_stride, int K, void *xs, int tile_rows,
                            int *cnt, int *scratch, int *perm, int *counts, int *n_tiles, int *tile_e, int *tile_row0,
                            int *tile_rowend, int max_tiles, int *err, const float *scores, int *tok_of,
                            float *scale_of, cudaStream_t st) {
    if (ecount > 1024) return cudaErrorInvalidValue;
    int *rank = scratch, *off = scratch + S;
    rank_kernel<<<(S + 255) / 256, 256, 0, st>>>(idx, S, ebase, ecount, etotal, cnt, rank, err);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    table_kernel<<<1, 1024, 0, st>>>(ecount, tile_rows, cnt, off, counts, n_tiles, tile_e, tile_row0, tile_rowend,
                                     max_tiles, err);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    scatter_rows_kernel<<<S, 128, 0, st>>>(idx, rank, off, ebase, k, xrow_is_slot, xidx,
                                           reinterpret_cast<const uint16_t *>(x), x_row_stride, K, perm,
                                           reinterpret_cast<uint16_t *>(xs), scores, tok_of, scale_of);
    return cudaGetLastError();
}

bool gemm_supported(int codec, int64_t m, int64_t n, int64_t k, int x_dtype, int64_t x_row_stride) {
    (void)codec;
    (void)n;
    return m >= 1 && k % BK == 0 && (x_row_stride * 2) % 16 == 0 && (x_dtype == F16 || x_dtype == BF16) &&
           encode_fn() != nullptr;
}

// Q4_K is dequantized inside the GEMM up to this many activation rows; above
// it, one dequantized copy plus B by TMA is faster.  The copy costs ~N*K*2.6
// bytes of traffic once; the in-kernel path repeats the dequantization for
// every row tile and holds the tensor pipe near 45 % busy.  Measured on the
// Llama-3-8B layer shapes: fused wins at M = 512, the copy from M = 1024 on
// (layer 593 vs 646 us at M = 1024, 950 vs 1094 us at M = 2048).
constexpr int64_t Q4K_FUSED_MAX_M = 768;

static bool fused_q4k(int codec, int64_t m) {
    const char *e = dev_env("KQ_Q4K_FUSED_MAX_M");
    return codec == Q4_K && m <= (e ? atol(e) : Q4K_FUSED_MAX_M);
}

// Plain dense GEMMs on the dequantized-copy path that would fill at most half
// of the SMs with 128-row tiles split K in two (K % 512 == 0 keeps each half a
// whole number of super-blocks).  The in-kernel Q4_K path does not split: with
// half of K per CTA its per-tile dequantization overheads cost more than the
// idle SMs (M = 512 o projection: 43 -> 52 us).
int gemm_ksplit(int codec, int64_t m, int64_t n, int64_t k, bool glu) {
    if (glu || k % 512 || fused_q4k(codec, m) || dev_env("KQ_GEMM_NO_SPLIT")) return 1;
    const int64_t nt = (n + BN - 1) / BN;
    if (((m + 2 * BM - 1) / (2 * BM)) * nt >= num_sms()) return 1;  // two row tiles per CTA fill the GPU
    return ((m + BM - 1) / BM) * nt * 2 <= num_sms() ? 2 : 1;
}

static size_t deq_scratch_bytes(int codec, int64_t m, int64_t n, int64_t k, bool glu) {
    return fused_q4k(codec, m) ? 0 : ((size_t)n * k * 2 * (glu ? 2 : 1) + 255) & ~(size_t)255;
}

size_t gemm_scratch_bytes(int codec, int64_t m, int64_t n, int64_t k, bool glu) {
    // dequantized copy for the B-by-TMA path, then the split-K partial tiles
    const int ks = gemm_ksplit(codec, m, n, k, glu);
    return deq_scratch_bytes(codec, m, n, k, glu) + (ks > 1 ? (size_t)ks * m * n * sizeof(float) : 0);
}

cudaError_t launch_gemm(const GemmArgs &a0, void *scratch, cudaStream_t st) {
    const bool f16 = a0.x_dtype == F16;
    if (a0.act != ACT_NONE) {  // fused GLU: gate rows then up rows of the dequantized copy
        GemmArgs a = a0;
        a.ex_lo = 0;
        a.ex_hi = 1;
        a.n_per_expert = a.N;
        if (fused_q4k(a.codec, a.M) && raw_tma_ok(a, true))
            return f16 ? launch_gemm_mt<true, B_Q4KT, true>(a, nullptr, st)
                       : launch_gemm_mt<false, B_Q4KT, true>(a, nullptr, st);
        if (fused_q4k(a.codec, a.M))
            return f16 ? launch_gemm_mt<true, B_Q4K, true>(a, nullptr, st) : launch_gemm_mt<false, B_Q4K, true>(a, nullptr, st);
        cudaError_t e = launch_dequantize(a.codec, a.w, a.N, a.K, a.w_row_stride, scratch, a.x_dtype, st);
        if (e == cudaSuccess)
            e = launch_dequantize(a.codec, a.w2, a.N, a.K, a.w_row_stride, (char *)scratch + (size_t)a.N * a.K * 2,
                                  a.x_dtype, st);
        if (e != cudaSuccess) return e;
        return f16 ? launch_gemm_mt<true, B_TMA, true>(a, scratch, st) : launch_gemm_mt<false, B_TMA, true>(a, scratch, st);
    }
    GemmArgs a = a0;
    a.ksplit = gemm_ksplit(a.codec, a.M, a.N, a.K, false);
    a.part = reinterpret_cast<float *>((char *)scratch + deq_scratch_bytes(a.codec, a.M, a.N, a.K, false));
    a.tile_cnt = reinterpret_cast<int *>(reinterpret_cast<char *>(a.err) + 256);  // workspace counter region
    if (fused_q4k(a.codec, a.M) && raw_tma_ok(a, true))
        return f16 ? launch_gemm_mt<true, B_Q4KT>(a, nullptr, st) : launch_gemm_mt<false, B_Q4KT>(a, nullptr, st);
    if (fused_q4k(a.codec, a.M))
        return f16 ? launch_gemm_mt<true, B_Q4K>(a, nullptr, st) : launch_gemm_mt<false, B_Q4K>(a, nullptr, st);
    // other codecs and large batches: dequantize once into scratch (activation dtype), then B by TMA
    cudaError_t e = launch_dequantize(a.codec, a.w, a.N, a.K, a.w_row_stride, scratch, a.x_dtype, st);
    if (e != cudaSuccess) return e;
    return f16 ? launch_gemm_mt<true, B_TMA>(a, scratch, st) : launch_gemm_mt<false, B_TMA>(a, scratch, st);
}

}  // namespace kq
