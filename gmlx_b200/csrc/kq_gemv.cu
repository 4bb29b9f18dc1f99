// kq_gemv.cu -- fused dequantize x GEMV for decode (M <= 32 activation rows
// per weight matrix).  Replaces mlx-kquant's quantized_matmul small-M route
// (called from KQuantLinear, gmlx/modules.py:1535-1539, and directly at
// gmlx/occupancy_fuse.py:284-287), the MoE decode gathers moe_glu_gather_kq /
// gather_qmv_kq (gmlx/modules.py:585-598) and their row-concat callers.
//
// Design (B200, HBM-bound):
//  * Work = (group, 32-row tile, stage) iterations, a stage being 4 super-
//    blocks of every row of the tile.  Persistent CTAs (every CTA resident)
//    each take an equal contiguous range of iterations ("stream-K"), so the
//    whole GPU streams evenly whatever the tile count; a tile split between
//    CTAs is finished by whichever contributor arrives last, which sums the
//    f32 partials in CTA order (deterministic) and resets the tile counter.
//  * 1 producer warp + 8 consumer warps per CTA.  The producer streams each
//    row's raw super-blocks (144/210/66 B, never repacked) into a shared-memory
//    ring with 1-D bulk async copies (cp.async.bulk, mbarrier completion, L2
//    evict-first).  Copies start at the 16-byte granule holding the first
//    byte, so unaligned Q6_K/IQ2_XXS rows stream the same way as Q4_K.  Each
//    row copy is >= ~1 KB (smaller bulk copies are request-rate bound).  For
//    one activation row its matching slice rides in the same stage, so the
//    MMA B operands come from shared memory too.
//  * Consumer warp = 16 rows x one super-block per stage.  Packed bits become
//    mma.sync m16n8k16 A fragments directly: quant values turn into exact
//    small-integer bf16 (or f16) by OR-ing them into the mantissa of a magic
//    constant, so the tensor-core products q*x are exact and each sub-block's
//    scale is applied once to the f32 partial:
//      Q4_K : T = sum (128+q) x,  S = sum x (an MMA with an all-ones A)
//             acc += (d sc) T - (128 d sc + dmin m) S
//      Q6_K : A = (128 + q) - 160 = q - 32 (exact packed subtract), acc += (d sc) T
//      IQ2  : A = +-grid (exact bf16 table, sign-bit xor), acc += d (0.5+ls)/4 T
//  * Activation rows are the MMA N dimension (8 per n-tile, up to 4 n-tiles).
//  * Fused GLU: a 32-row tile holds 16 gate rows and the same 16 up rows, so
//    act(gate)*up is formed in the epilogue without a second pass.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdlib.h>

#include <algorithm>

#include "kq_internal.cuh"
#include "kq_ptx.cuh"

#include "kq_gemv_dev.cuh"

namespace kq {
namespace {

// -------------------------------------------------------------------------

// Weight rows of a dense one-row Q4_K problem as a 2-D tensor of uint64
// [N][row bytes / 8] (the whole-SM copy engine streams one box per stage far
// faster than 32 row copies).  use == 0: the per-row bulk copies.
struct GemvMaps {
    CUtensorMap w, w2;
    int use;
};

__device__ __forceinline__ void tma_box_g(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar,
                                          uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

template <int C, int NT, bool F16, bool GLU, int XR>
__global__ void __launch_bounds__(NTHREADS, CTAS_PER_SM<C, NT, XR>) gemv_kernel(const GemvArgs a,
                                                                             const __grid_constant__ GemvMaps mp) {
    using L = GLayout<C, NT, XR>;
    constexpr bool XS = L::XS;
    constexpr int bpb = Fmt<C>::bpb, NS = L::NS, KB = L::KB, XSTR = L::XSTR, BPW = GCfg<C>::BPW;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L::OFF_BAR);
    uint64_t *empty = full + NS;
    uint8_t *rowoff = smem + L::OFF_ROWOFF;
    volatile int *s_abort = reinterpret_cast<volatile int *>(smem + L::OFF_MISC);
    int *s_last = reinterpret_cast<int *>(smem + L::OFF_MISC + 4);
    int *s_unit = reinterpret_cast<int *>(smem + L::OFF_UNIT);  // NS <= 8 ints
    int *s_npub = s_unit + 8, *s_pub = s_unit + 9;               // deferred K-chunk publishes
    constexpr int MAXPUB = 23;
    uint4 *gridtab = reinterpret_cast<uint4 *>(smem + L::OFF_GRID);
    uint8_t *ring = smem + L::OFF_RING;
    float *red0 = reinterpret_cast<float *>(smem + L::OFF_RED);
    float *Ssm = reinterpret_cast<float *>(smem + L::OFF_S);

    const long long c_entry = clock64();  // development timing (debug bit 128)
    const uint32_t g_entry = (uint32_t)globaltimer();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nb = a.K / QK;
    const int nst = (nb + KB - 1) / KB;  // stages per tile
    const int rows_out = GLU ? 16 : 32;
    const int tiles = (a.N + rows_out - 1) / rows_out;
    const int n_groups = a.dense_m > 0 ? (a.dense_m + 31) / 32 : min(*a.n_groups, a.max_groups);
    const int64_t I = (int64_t)n_groups * tiles * nst;  // total stage iterations
    const int64_t P = gridDim.x;
    const int64_t lo = part_lo(blockIdx.x, I, P), hi = part_lo(blockIdx.x + 1, I, P);

    if (threadIdx.x == 0) {
        for (int i = 0; i < NS; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], CW);
        }
        *s_abort = 0;
        *s_npub = 0;
        for (int b = 0; b <= NS; b++) reinterpret_cast<int *>(smem + L::OFF_MISC + 16)[b] = 0;
        fence_mbar_init();
    }
    if constexpr (C == IQ3_XXS) {
        for (int e = threadIdx.x; e < 256; e += NTHREADS) reinterpret_cast<uint32_t *>(gridtab)[e] = c_iq3xxs_grid[e];
    } else if constexpr (C == IQ3_S) {
        for (int e = threadIdx.x; e < 512; e += NTHREADS) reinterpret_cast<uint32_t *>(gridtab)[e] = c_iq3s_grid[e];
    } else if constexpr (C == IQ1_S || C == IQ1_M) {
        for (int e = threadIdx.x; e < 2048; e += NTHREADS) {
            const uint64_t v = c_iq1s_grid[e];
            reinterpret_cast<uint2 *>(gridtab)[e] = make_uint2((uint32_t)v, (uint32_t)(v >> 32));
        }
    } else if constexpr (C == IQ2_XS || C == IQ2_S) {
        for (int e = threadIdx.x; e < (C == IQ2_XS ? 512 : 1024); e += NTHREADS) {
            const uint64_t v = C == IQ2_XS ? c_iq2xs_grid[e] : c_iq2s_grid[e];
            reinterpret_cast<uint2 *>(gridtab)[e] = make_uint2((uint32_t)v, (uint32_t)(v >> 32));
        }
    }
    if constexpr (C == IQ2_XXS && L::DP) {
        // lane-per-row path: the raw magnitude bytes (256 x 8 B)
        for (int e = threadIdx.x; e < 256; e += NTHREADS) {
            const uint64_t v = c_iq2xxs_grid[e];
            reinterpret_cast<uint2 *>(gridtab)[e] = make_uint2((uint32_t)v, (uint32_t)(v >> 32));
        }
    } else if constexpr (C == IQ2_XXS) {
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
    // programmatic dependent launch: let the next kernel on the stream start
    // its prologue now; weights are read-only, so only activation reads and
    // global writes below wait for the previous kernel (griddepcontrol.wait)
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if ((lo >= hi && !(L::DP && a.dyn)) || (a.debug & 64)) return;  // 64: development, prologue only
    unsigned *stamps = reinterpret_cast<unsigned *>(smem + L::OFF_MISC + 64);  // development timing (16 words)
    if ((a.debug & 128) && threadIdx.x == 0) stamps[0] = (unsigned)(clock64() - c_entry);

    if (warp == CW) {
        // ---------------- producer warp: lane r streams tile row r (+ activation row r) ----------------
        const uint64_t pol = policy_evict_first(), pol_x = policy_evict_last();
        if (L::DP && a.dyn) {
            // dynamic whole tiles: the first tile of a CTA is its index, later ones
            // come from a work counter (read only after griddepcontrol.wait, so a
            // previous kernel has reset it), so CTAs that start late take fewer
            const int S = a.ksplit, chunk = (nst + S - 1) / S;
            const int units = n_groups * tiles * S;
            uint32_t it = 0;
            bool dep_done = false;
            for (int unit = blockIdx.x;;) {
                const int slot0 = it % NS;
                if (unit >= units || *s_abort) {  // end marker: an empty stage with a negative tile id
                    wait_bounded(&empty[slot0], ((it / NS) & 1) ^ 1, s_abort, a.err, 1);
                    if (lane == 0) {
                        s_unit[slot0] = -1;
                        mbar_arrive(&full[slot0]);
                    }
                    break;
                }
                Tile T;
                tile_of(a, unit / S, tiles, T);
                const int s0 = (unit % S) * chunk, s1 = min(nst, s0 + chunk);
                const int orow = T.tile * rows_out + (GLU ? (lane & 15) : lane);
                const bool up = GLU && lane >= 16;
                const bool valid = orow < a.N;
                const uint8_t *base = up ? a.w2 + (int64_t)T.e * a.w2_expert_stride + (int64_t)orow * a.w2_row_stride
                                         : a.w + (int64_t)T.e * a.w_expert_stride + (int64_t)orow * a.w_row_stride;
                // lane t < m stages activation row t of the group (m <= XR)
                const int xm = min(T.m, XR);
                const uint8_t *xsrc = reinterpret_cast<const uint8_t *>(a.x) +
                                      (int64_t)xrow_of(a, T, lane < xm ? lane : 0) * a.x_row_stride * 2;
                for (int st = s0; st < s1; st++, it++) {
                    const int slot = it % NS;
                    wait_bounded(&empty[slot], ((it / NS) & 1) ^ 1, s_abort, a.err, 1);
                    const int bs = st * KB, nbk = min(KB, nb - bs);
                    const uintptr_t src = (uintptr_t)(base + (int64_t)bs * bpb);
                    const uint32_t off = (uint32_t)(src & 15);
                    // tensor-map path (mp.use): the stage's 32 rows arrive as one 2-D box
                    // (two 16-row boxes for the fused GLU) instead of 32 row copies
                    const uint32_t bytes = mp.use ? (lane == 0 ? (uint32_t)(TROWS * L::SP) : 0u)
                                                  : (valid && !(a.debug & 2)) ? ((off + nbk * bpb + 15) & ~15u) : 0u;
                    const uint32_t xbytes = (lane < xm && !(a.debug & 8)) ? (uint32_t)nbk * QK * 2 : 0u;
                    // tensor boxes start at the 16-byte granule holding the stage's first
                    // byte (rows are 16-byte aligned, so the offset is the same in every row)
                    const uint32_t boff = (uint32_t)(bs * bpb) & 15u;
                    rowoff[slot * 32 + lane] = mp.use ? (uint8_t)boff : (uint8_t)off;
                    uint32_t total = bytes + xbytes;
#pragma unroll
                    for (int o = 16; o; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
                    if (lane == 0) {
                        s_unit[slot] = unit;
                        mbar_arrive_expect_tx(&full[slot], total);
                    }
                    __syncwarp();
                    if (!*s_abort) {
                        uint8_t *stg = ring + slot * L::STAGE;
                        if (mp.use) {
                            if (lane == 0) {
                                const int x = (bs * bpb >> 4) << 1;  // uint64 units, even: 16-byte aligned
                                if (GLU) {
                                    tma_box_g(stg, &mp.w, x, T.tile * 16, &full[slot], pol);
                                    tma_box_g(stg + 16 * L::SP, &mp.w2, x, T.tile * 16, &full[slot], pol);
                                } else {
                                    tma_box_g(stg, &mp.w, x, T.tile * 32, &full[slot], pol);
                                }
                            }
                        } else if (bytes) {
                            bulk_g2s(stg + lane * L::SP, (const void *)(src - off), bytes, &full[slot], pol);
                        }
                        if (!dep_done) {
                            asm volatile("griddepcontrol.wait;" ::: "memory");
                            dep_done = true;
                        }
                        if (xbytes)
                            bulk_g2s(stg + L::WBYTES + lane * XSTR, xsrc + (int64_t)bs * QK * 2, xbytes, &full[slot], pol_x);
                    }
                }
                int nu = 0;
                if (lane == 0) nu = (int)gridDim.x + atomicAdd(a.counters, 1);
                unit = __shfl_sync(0xffffffffu, nu, 0);
            }
            return;
        }
        uint32_t it = 0;
        int64_t cur = -1;
        Tile T{};
        const uint8_t *base = nullptr;
        bool valid = false;
        const uint8_t *xsrc = nullptr;
        bool dep_done = false;
        int64_t gt = lo / nst;
        int st = (int)(lo - gt * nst);
        for (int64_t i = lo; i < hi; i++, it++, st++) {
            if (st == nst) {  // next tile (indices advance incrementally: no 64-bit division per stage)
                st = 0;
                gt++;
            }
            if (gt != cur) {
                cur = gt;
                tile_of(a, gt, tiles, T);
                const int orow = T.tile * rows_out + (GLU ? (lane & 15) : lane);
                const bool up = GLU && lane >= 16;
                valid = orow < a.N;
                base = up ? a.w2 + (int64_t)T.e * a.w2_expert_stride + (int64_t)orow * a.w2_row_stride
                          : a.w + (int64_t)T.e * a.w_expert_stride + (int64_t)orow * a.w_row_stride;
                if (XS && lane < T.m)
                    xsrc = reinterpret_cast<const uint8_t *>(a.x) + (int64_t)xrow_of(a, T, lane) * a.x_row_stride * 2;
            }
            const int slot = it % NS;
            wait_bounded(&empty[slot], ((it / NS) & 1) ^ 1, s_abort, a.err, 1, (a.debug & 256) != 0);
            if ((a.debug & 128) && lane == 0 && it < 6) stamps[10 + it] = (unsigned)(clock64() - c_entry);
            const int bs = st * KB, nbk = min(KB, nb - bs);
            const uintptr_t src = (uintptr_t)(base + (int64_t)bs * bpb);
            const uint32_t off = (uint32_t)(src & 15);
            const uint32_t bytes = mp.use ? (lane == 0 ? (uint32_t)(TROWS * L::SP) : 0u)
                                          : (valid && !(a.debug & 2)) ? ((off + nbk * bpb + 15) & ~15u) : 0u;
            const uint32_t xbytes = (XS && lane < T.m && !(a.debug & 8)) ? (uint32_t)nbk * QK * 2 : 0u;
            rowoff[slot * 32 + lane] = mp.use ? (uint8_t)((uint32_t)(bs * bpb) & 15u) : (uint8_t)off;
            uint32_t total = bytes + xbytes;
#pragma unroll
            for (int o = 16; o; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
            if (lane == 0) mbar_arrive_expect_tx(&full[slot], total);
            __syncwarp();
            if ((a.debug & 128) && lane == 0 && it < 6) stamps[4 + it] = (unsigned)(clock64() - c_entry);
            if (!*s_abort) {
                uint8_t *stg = ring + slot * L::STAGE;
                if (mp.use) {
                    if (lane == 0) {
                        const int x = (bs * bpb >> 4) << 1;
                        if (GLU) {
                            tma_box_g(stg, &mp.w, x, T.tile * 16, &full[slot], pol);
                            tma_box_g(stg + 16 * L::SP, &mp.w2, x, T.tile * 16, &full[slot], pol);
                        } else {
                            tma_box_g(stg, &mp.w, x, T.tile * 32, &full[slot], pol);
                        }
                    }
                } else if (bytes) {
                    if (a.debug & 4)
                        asm volatile(
                            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                                smem_u32(stg + lane * L::SP)),
                            "l"((const void *)(src - off)), "r"(bytes), "r"(smem_u32(&full[slot]))
                            : "memory");
                    else
                        bulk_g2s(stg + lane * L::SP, (const void *)(src - off), bytes, &full[slot], pol);
                }
                if (!dep_done) {  // the first weight copies are in flight; activations may be the
                    asm volatile("griddepcontrol.wait;" ::: "memory");  // previous kernel's output
                    dep_done = true;
                }
                if (xbytes)
                    bulk_g2s(stg + L::WBYTES + lane * XSTR, xsrc + (int64_t)bs * QK * 2, xbytes, &full[slot], pol_x);
            }
        }
        if ((a.debug & 128) && lane == 0) stamps[1] = (unsigned)(clock64() - c_entry);
        return;
    }

    // ---------------- consumer warps: warp -> (16-row half mt, block column col) ----------------
    // (lane-per-row path: warp -> block column, lane -> row)
    constexpr bool DP = L::DP;
    constexpr int RCOLS = DP ? CW : NCOL;                    // partial sums per row to reduce
    constexpr int RCS = DP ? RED_TS : 8 * NT * RED_TS;       // their stride in the reduction buffer
    // Q4_K lane-per-row: warp = block column, lane = row.  Q6_K: warp =
    // (block column warp&3, 16-row half warp>>2), half-warp = block half.
    // lane-per-row codecs with 4 block columns per stage (Q6_K, Q8_0): warp =
    // (block column, block half); the others: warp = block column
    constexpr bool HALVES = C == Q6_K || C == Q8_0 || C == Q5_1;
    const int mt = (DP && !HALVES) ? 0 : (warp & 1), col = (DP && !HALVES) ? warp : (DP ? (warp & 3) : (warp >> 1));
    // per-warp table: scales (MMA path) or quantized activations + their
    // scales (lane-per-row path: 128 words + 32 floats = 640 bytes, as TABS)
    float *stab = reinterpret_cast<float *>(smem + L::OFF_SCALE) + warp * (DP ? 160 * XR : GCfg<C>::TABW * BPW);
    const int ctid = threadIdx.x;  // 0 .. CW*32-1
    // Consumers block here until the previous kernel on the stream has finished
    // (they need its activations anyway).  Polling the ring instead would burn
    // the issue slots of the previous kernel's CTAs still running on this SM.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    uint32_t it = 0;
    int64_t i = lo;
    int rp = 0, s_group = -1, tix = 0;
    int *dcnt = const_cast<int *>(reinterpret_cast<volatile int *>(smem + L::OFF_MISC + 16));  // NS+1 tile counters
    // lane-per-row path: one stage of one block column (operands to registers,
    // release the stage, then the arithmetic)
    auto dp_stage = [&](int slot, int b, float *acc, int m) {
        uint32_t *xq = reinterpret_cast<uint32_t *>(stab);
        float *xsc = stab + 128;
        const bool run = b < nb && !*s_abort && !(a.debug & 1);
        const uint8_t *stg = ring + slot * L::STAGE;
        if constexpr (C == Q4_K) {
            Q4Regs r;
            if (run) {
                dp_quantize<F16>(reinterpret_cast<const uint16_t *>(stg + L::WBYTES) + col * QK, xq, xsc);
                dp_q4k_load(stg + lane * L::SP + rowoff[slot * 32 + lane] + col * bpb, r);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (run) acc[0] += dp_q4k_dot(r, xq, xsc);
        } else if constexpr (C == Q5_K) {
            Q5Regs r;
            if (run) {
                dp_quantize<F16>(reinterpret_cast<const uint16_t *>(stg + L::WBYTES) + col * QK, xq, xsc);
                dp_q5k_load(stg + lane * L::SP + rowoff[slot * 32 + lane] + col * bpb, r);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (run) acc[0] += dp_q5k_dot(r, xq, xsc);
        } else if constexpr (C == Q8_0) {
            // lane = row, warp = (group column warp&3, half warp>>2 = four 34-byte blocks)
            const int hf = warp >> 2;
            Q8Regs r;
            if (run) {
                dp_quantize<F16>(reinterpret_cast<const uint16_t *>(stg + L::WBYTES) + col * QK, xq, xsc);
                dp_q80_load(stg + lane * L::SP + rowoff[slot * 32 + lane] + col * bpb + 136 * hf, r);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (run) acc[0] += dp_q80_dot(r, hf, xq, xsc);
        } else if constexpr (C == Q2_K) {
            Q2Regs r;
            if (run) {
                dp_quantize<F16>(reinterpret_cast<const uint16_t *>(stg + L::WBYTES) + col * QK, xq, xsc);
                dp_q2k_load(stg + lane * L::SP + rowoff[slot * 32 + lane] + col * bpb, r);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (run) acc[0] += dp_q2k_dot(r, xq, xsc);
        } else if constexpr (C == IQ1_S) {
            IQSRegs<C> r;
            if (run) {
                dp_quantize<F16>(reinterpret_cast<const uint16_t *>(stg + L::WBYTES) + col * QK, xq, xsc);
                dp_iqs_load<C>(stg + lane * L::SP + rowoff[slot * 32 + lane] + col * bpb, r);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (run) acc[0] += dp_iq1_dot<C>(r.q, r.d, xq, xsc, reinterpret_cast<const uint2 *>(gridtab));
        } else if constexpr (C == IQ1_M) {
            IQ1MRegs r;
            if (run) {
                dp_quantize<F16>(reinterpret_cast<const uint16_t *>(stg + L::WBYTES) + col * QK, xq, xsc);
                dp_iq1m_load(stg + lane * L::SP + rowoff[slot * 32 + lane] + col * bpb, r);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (run) acc[0] += dp_iq1_dot<C>(r.q, 0.f, xq, xsc, reinterpret_cast<const uint2 *>(gridtab));
        } else if constexpr (C == IQ2_XS || C == IQ2_S || C == IQ3_S) {
            IQSRegs<C> r;
            if (run) {
                dp_quantize<F16>(reinterpret_cast<const uint16_t *>(stg + L::WBYTES) + col * QK, xq, xsc);
                dp_iqs_load<C>(stg + lane * L::SP + rowoff[slot * 32 + lane] + col * bpb, r);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (run)
                acc[0] += dp_iqs_dot<C>(r, xq, xsc, reinterpret_cast<const uint2 *>(gridtab),
                                     reinterpret_cast<const uint32_t *>(gridtab));
        } else if constexpr (C == NVFP4) {
            NVRegs r;
            if (run) {
                dp_quantize<F16>(reinterpret_cast<const uint16_t *>(stg + L::WBYTES) + col * QK, xq, xsc);
                dp_nv_load(stg + lane * L::SP + rowoff[slot * 32 + lane] + col * bpb, r);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (run) acc[0] += dp_nv_dot(r, xq, xsc);
        } else if constexpr (C == TQ1_0) {
            TQ1Regs r;
            if (run) {
                dp_quantize<F16>(reinterpret_cast<const uint16_t *>(stg + L::WBYTES) + col * QK, xq, xsc);
                dp_tq1_load(stg + lane * L::SP + rowoff[slot * 32 + lane] + col * bpb, r);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (run) acc[0] += dp_tq1_dot(r, xq, xsc);
        } else if constexpr (C == TQ2_0) {
            TQ2Regs r;
            if (run) {
                dp_quantize<F16>(reinterpret_cast<const uint16_t *>(stg + L::WBYTES) + col * QK, xq, xsc);
                dp_tq2_load(stg + lane * L::SP + rowoff[slot * 32 + lane] + col * bpb, r);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (run) acc[0] += dp_tq2_dot(r, xq, xsc);
        } else if constexpr (C == Q3_K) {
            Q3Regs r;
            if (run) {
                dp_quantize<F16>(reinterpret_cast<const uint16_t *>(stg + L::WBYTES) + col * QK, xq, xsc);
                dp_q3k_load(stg + lane * L::SP + rowoff[slot * 32 + lane] + col * bpb, r);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (run) acc[0] += dp_q3k_dot(r, xq, xsc);
        } else if constexpr (Legacy<C>::IS) {
            // warp = group column, lane = row (a whole group of eight blocks;
            // Q5_1: warp = (group column, half), four blocks)
            const int hf = LEG_NB<C> == 8 ? 0 : warp >> 2;
            LegRegs<C> r;
            if (run) {
                dp_quantize<F16>(reinterpret_cast<const uint16_t *>(stg + L::WBYTES) + col * QK, xq, xsc);
                dp_leg_load<C>(stg + lane * L::SP + rowoff[slot * 32 + lane] + col * bpb + hf * 4 * Legacy<C>::BB, r);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (run) acc[0] += dp_leg_dot<C>(r, xq, xsc, 4 * hf);
        } else if constexpr (C == Q6_K) {
            // lane = row, warp = (block column warp&3, block half warp>>2)
            const int hf = warp >> 2;
            Q6Regs r;
            if (run) {
                dp_quantize<F16>(reinterpret_cast<const uint16_t *>(stg + L::WBYTES) + col * QK, xq, xsc);
                dp_q6k_load_rows(stg + lane * L::SP + rowoff[slot * 32 + lane] + col * bpb, hf, r);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (run) acc[0] += dp_q6k_dot(r, hf, xq, xsc);
        } else if constexpr (C == IQ3_XXS) {
            IQ3Regs r;
            if (run) {
                dp_quantize<F16>(reinterpret_cast<const uint16_t *>(stg + L::WBYTES) + col * QK, xq, xsc);
                dp_iq3_load(stg + lane * L::SP + rowoff[slot * 32 + lane] + col * bpb, r);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (run) acc[0] += dp_iq3_dot(r, xq, xsc, reinterpret_cast<const uint32_t *>(gridtab));
        } else if constexpr (C == IQ4_XS) {
            IQ4Regs r;
            if (run) {
                dp_quantize<F16>(reinterpret_cast<const uint16_t *>(stg + L::WBYTES) + col * QK, xq, xsc);
                dp_iq4xs_load(stg + lane * L::SP + rowoff[slot * 32 + lane] + col * bpb, r);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (run) acc[0] += dp_iq4xs_dot(r, xq, xsc);
        } else if constexpr (XR > 1) {
            // IQ2_XXS, 1-4 staged rows: the dot reads the stage, then releases it
            if (run) {
#pragma unroll
                for (int t = 0; t < XR; t++)
                    if (t < m)
                        dp_quantize<F16>(reinterpret_cast<const uint16_t *>(stg + L::WBYTES + t * XSTR) + col * QK,
                                         xq + 160 * t, xsc + 160 * t);
                const uint8_t *blk = stg + lane * L::SP + rowoff[slot * 32 + lane] + col * bpb;
                const uint2 *gt = reinterpret_cast<const uint2 *>(gridtab);
                if (m == 1) dp_iq2_dot_smem<1>(blk, xq, xsc, gt, acc);  // m is warp-uniform
                else if (m == 2) dp_iq2_dot_smem<2>(blk, xq, xsc, gt, acc);
                else if (m == 3) dp_iq2_dot_smem<3>(blk, xq, xsc, gt, acc);
                else dp_iq2_dot_smem<4>(blk, xq, xsc, gt, acc);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        } else {
            IQ2Regs r;
            if (run) {
                dp_quantize<F16>(reinterpret_cast<const uint16_t *>(stg + L::WBYTES) + col * QK, xq, xsc);
                dp_iq2_load(stg + lane * L::SP + rowoff[slot * 32 + lane] + col * bpb, r);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (run) dp_iq2_dot_r<1>(r, xq, xsc, reinterpret_cast<const uint2 *>(gridtab), acc);
        }
    };
    // final value of output n of tile T: to y, or (fused all-reduce) as this
    // rank's f32 partial into every rank's communication buffer
    const unsigned ar_epoch = a.ar_world ? *reinterpret_cast<volatile unsigned *>(a.ar_bufs[a.ar_rank]) : 0u;
    const int ar_par = (int)(ar_epoch & 1u);
    auto emit = [&](const Tile &T, int tok, int n, float v) {
        if (a.ar_world == 0) {
            store_out(a.y, a.y_dtype, (int64_t)orow_of(a, T, tok) * a.y_row_stride + n, v + bias_of(a, n));
            return;
        }
        const int64_t off = ((int64_t)(ar_par * a.ar_world + a.ar_rank)) * a.N + n;
        for (int p = 0; p < a.ar_world; p++)
            reinterpret_cast<float *>(a.ar_bufs[p] + AR_HDR)[off] = v;
    };
    // lane-per-row path, whole tile: barrier-free store.  Each warp posts its 32
    // row partials; the last of the KB warps to arrive sums them in column order
    // and stores.  Buffers rotate over NS+1 tiles, which the ring keeps apart.
    auto dp_store = [&](const Tile &T, const float *acc, int m, int tix, int split_tile = -1, int chunk_id = 0) {
        const int bi = tix % (NS + 1);
        float *rb = reinterpret_cast<float *>(smem + L::OFF_DPB) + bi * (CW * 32 * XR);
#pragma unroll
        for (int t = 0; t < XR; t++) rb[(warp * XR + t) * 32 + lane] = acc[t];
        __syncwarp();
        int old = 0;
        if (lane == 0) {
            __threadfence_block();
            old = atomicAdd(dcnt + bi, 1);
        }
        old = __shfl_sync(0xffffffffu, old, 0);
        if (old == CW - 1) {
            __threadfence_block();
            const int row = GLU ? (lane & 15) : lane;
            const int n = T.tile * rows_out + row;
            if constexpr (XR > 1) {  // several rows: whole tiles only (no K split)
                for (int t = 0; t < m; t++) {
                    float v = 0.f, v2 = 0.f;
#pragma unroll
                    for (int w = 0; w < CW; w++) {
                        v += rb[(w * XR + t) * 32 + row];
                        if (GLU) v2 += rb[(w * XR + t) * 32 + row + 16];
                    }
                    if (GLU) v = apply_act(a.act, v) * v2;
                    if (n < a.N && (!GLU || lane < 16)) emit(T, t, n, v);
                }
                __syncwarp();
                if (lane == 0) dcnt[bi] = 0;
                return;
            }
            float v = 0.f, v2 = 0.f;
            if (split_tile < 0) {
#pragma unroll
                for (int w = 0; w < CW; w++) {
                    v += rb[w * 32 + row];
                    if (GLU) v2 += rb[w * 32 + row + 16];
                }
            } else {
                // K split over ksplit units: post this unit's 32 row sums, the
                // last unit of the tile adds them in chunk order and stores
                float u = 0.f;
#pragma unroll
                for (int w = 0; w < CW; w++) u += rb[w * 32 + lane];
                __stcg(a.partial + ((int64_t)split_tile * a.ksplit + chunk_id) * 32 + lane, u);
                __syncwarp();
                // defer the publish to the CTA's end (one fence for all its
                // chunks, off the ring's critical path); immediate if the list is full
                int k = 0;
                if (lane == 0) {
                    k = atomicAdd(s_npub, 1);
                    if (k < MAXPUB) s_pub[k] = split_tile;
                }
                k = __shfl_sync(0xffffffffu, k, 0);
                if (k < MAXPUB) split_tile = -2;
                int prev = 0;
                if (split_tile >= 0 && lane == 0) {
                    __threadfence();
                    prev = atomicAdd(a.counters + 2 + split_tile, 1);
                    if (prev == a.ksplit - 1) __threadfence();
                }
                prev = __shfl_sync(0xffffffffu, prev, 0);
                if (split_tile >= 0 && prev == a.ksplit - 1) {
                    for (int c = 0; c < a.ksplit; c++) {
                        const float *pp = a.partial + ((int64_t)split_tile * a.ksplit + c) * 32;
                        v += __ldcg(pp + row);
                        if (GLU) v2 += __ldcg(pp + row + 16);
                    }
                    if (lane == 0) a.counters[2 + split_tile] = 0;
                } else {
                    split_tile = -2;  // not the last: nothing to store
                }
            }
            if (GLU) v = apply_act(a.act, v) * v2;
            if (split_tile != -2 && n < a.N && (!GLU || lane < 16)) emit(T, 0, n, v);
            __syncwarp();
            if (lane == 0) dcnt[bi] = 0;
        }
    };
    if constexpr (DP) {
        if (a.dyn) {
            // dynamic whole tiles: the producer names each stage's tile in
            // s_unit[slot]; a negative id ends the work
            for (;;) {
                int slot = it % NS;
                wait_bounded(&full[slot], (it / NS) & 1, s_abort, a.err, 2, (a.debug & 256) != 0);
                const int unit = s_unit[slot];
                if (unit < 0 || *s_abort) break;
                const int S = a.ksplit, chunk = (nst + S - 1) / S;
                const int tile = unit / S, s0 = (unit % S) * chunk, s1 = min(nst, s0 + chunk);
                Tile T;
                tile_of(a, tile, tiles, T);
                float acc[XR];
#pragma unroll
                for (int t = 0; t < XR; t++) acc[t] = 0.f;
                const int m = min(T.m, XR);
                for (int st = s0; st < s1; st++, it++) {
                    slot = it % NS;
                    if (st > s0) wait_bounded(&full[slot], (it / NS) & 1, s_abort, a.err, 2, (a.debug & 256) != 0);
                    dp_stage(slot, st * KB + col, acc, m);
                }
                if (!(a.debug & 32)) dp_store(T, acc, m, tix, S > 1 ? tile : -1, unit % S);
                tix++;
            }
            // publish the deferred K-chunk partials: each warp fences its own
            // partial stores, then the chunks' tile counters are bumped; the
            // last chunk of a tile sums the partials in chunk order and stores
            __threadfence();
            named_bar_sync(1, CW * 32);
            const int npub = min(*s_npub, MAXPUB);
            for (int q = warp; q < npub; q += CW) {
                const int t = s_pub[q];
                int prev = 0;
                if (lane == 0) {
                    prev = atomicAdd(a.counters + 2 + t, 1);
                    if (prev == a.ksplit - 1) __threadfence();
                }
                prev = __shfl_sync(0xffffffffu, prev, 0);
                if (prev != a.ksplit - 1) continue;
                Tile T;
                tile_of(a, t, tiles, T);
                const int row = GLU ? (lane & 15) : lane;
                const int n = T.tile * rows_out + row;
                float v = 0.f, v2 = 0.f;
                for (int c = 0; c < a.ksplit; c++) {
                    const float *pp = a.partial + ((int64_t)t * a.ksplit + c) * 32;
                    v += __ldcg(pp + row);
                    if (GLU) v2 += __ldcg(pp + row + 16);
                }
                if (GLU) v = apply_act(a.act, v) * v2;
                if (n < a.N && (!GLU || lane < 16)) emit(T, 0, n, v);
                if (lane == 0) a.counters[2 + t] = 0;
            }
            if ((a.debug & 128) && ctid == 0) {  // development timing: per-CTA entry / end / tiles
                unsigned *o = reinterpret_cast<unsigned *>(a.y) + a.y_row_stride + 32 * blockIdx.x;
                o[0] = g_entry;
                o[1] = stamps[0];
                o[4] = (unsigned)(clock64() - c_entry);
                o[5] = (unsigned)tix;
                o[6] = (unsigned)globaltimer();
            }
            // the last CTA out resets the work counters (zero on entry, left zero).
            // Fused all-reduce: it also raises this rank's flag on every peer, waits
            // (bounded) for every rank's flag of this call and writes the rank-order
            // sum of all partials.  Only that CTA waits, and only on other GPUs, so
            // no CTA of this kernel depends on another being resident.  The other
            // CTAs' partial stores reach it through gpu-scope fence + counter; its
            // system-scope fence then orders them before the flag stores.
            named_bar_sync(1, CW * 32);
            if (ctid == 0) {
                __threadfence();
                const int last = atomicAdd(a.counters + 1, 1) == (int)gridDim.x - 1;
                if (last) {
                    a.counters[0] = 0;
                    a.counters[1] = 0;
                    if (a.ar_world) {
                        __threadfence_system();
                        const unsigned next = ar_epoch + 1u;
                        for (int p = 0; p < a.ar_world; p++) {
                            unsigned *f = reinterpret_cast<unsigned *>(a.ar_bufs[p] + 64) + ar_par * a.ar_world + a.ar_rank;
                            asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(next) : "memory");
                        }
                        *reinterpret_cast<volatile unsigned *>(a.ar_bufs[a.ar_rank]) = next;  // own epoch
                    }
                }
                *s_last = last;
            }
            if (a.ar_world) {
                named_bar_sync(1, CW * 32);
                if (!*s_last) return;
                if (ctid < a.ar_world) {
                    const unsigned *f = reinterpret_cast<const unsigned *>(a.ar_bufs[a.ar_rank] + 64) + ar_par * a.ar_world + ctid;
                    const uint64_t t0 = globaltimer();
                    for (uint32_t it2 = 0;; it2++) {
                        unsigned v;
                        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
                        if (v == ar_epoch + 1u) break;
                        if ((it2 & 255) == 255 && globaltimer() - t0 > 2000000000ull) {
                            atomicCAS(a.err, 0, 7);  // a peer never signalled
                            *s_abort = 1;
                            break;
                        }
                    }
                }
                named_bar_sync(1, CW * 32);
                if (*s_abort) return;
                const float *slots = reinterpret_cast<const float *>(a.ar_bufs[a.ar_rank] + AR_HDR) +
                                     (int64_t)ar_par * a.ar_world * a.N;
                for (int n = ctid; n < a.N; n += CW * 32) {
                    float v = 0.f;
                    for (int r = 0; r < a.ar_world; r++) v += __ldcv(slots + (int64_t)r * a.N + n);
                    store_out(a.y, a.y_dtype, n, v + bias_of(a, n));
                }
            }
            return;
        }
    }
    int64_t gt_next = lo / nst;
    while (i < hi) {
        const int64_t gt = gt_next++;
        const int st0 = (int)(i - gt * nst);
        const int64_t tile_lo = gt * nst, tile_hi = tile_lo + nst;
        const int64_t end = min(hi, tile_hi);
        Tile T;
        tile_of(a, gt, tiles, T);
        float *red = red0 + rp * (L::REDB / 4);
        rp ^= 1;
        if constexpr (L::SX) {
            if (T.g != s_group) {  // sub-block sums of this group's one activation row
                s_group = T.g;
                named_bar_sync(1, CW * 32);
                const uint16_t *xs = reinterpret_cast<const uint16_t *>(a.x) + (int64_t)xrow_of(a, T, 0) * a.x_row_stride;
                for (int q = ctid; q < nb * 8; q += CW * 32) {
                    float sacc = 0.f;
#pragma unroll
                    for (int v = 0; v < 4; v++) {
                        const uint4 u = __ldg(reinterpret_cast<const uint4 *>(xs + 32 * q + 8 * v));
                        const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                        for (int e = 0; e < 4; e++) {
                            if constexpr (F16) {
                                const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w4[e]));
                                sacc += f.x + f.y;
                            } else {
                                sacc += __uint_as_float(w4[e] << 16) + __uint_as_float(w4[e] & 0xffff0000u);
                            }
                        }
                    }
                    Ssm[q] = sacc;
                }
                named_bar_sync(1, CW * 32);
            }
        }
        float acc[NT][4];
        const uint16_t *xg[NT];  // global activation rows (non-staged path)
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
            // lane g of n-tile nt reads token 8nt+g; absent tokens read a valid
            // row (their output columns are never stored)
            const int tok = min(8 * nt + (lane >> 2), T.m - 1);
            xg[nt] = reinterpret_cast<const uint16_t *>(a.x) + (int64_t)xrow_of(a, T, tok) * a.x_row_stride;
        }
        const int xtok = min(lane >> 2, T.m - 1);
        for (int st = st0; i < end; st++, i++, it++) {
            const int slot = it % NS;
            wait_bounded(&full[slot], (it / NS) & 1, s_abort, a.err, 2, (a.debug & 256) != 0);
            if ((a.debug & 128) && ctid == 0 && i == lo) stamps[2] = (unsigned)(clock64() - c_entry);
            const int col0 = DP ? col : col * BPW, b = st * KB + col0;
            if constexpr (DP) {
                dp_stage(slot, b, &acc[0][0], 1);
                continue;
            } else if (b < nb && !*s_abort && !(a.debug & 1)) {
                const uint8_t *stg = ring + slot * L::STAGE;
                const uint16_t *xr[NT];
#pragma unroll
                for (int nt = 0; nt < NT; nt++)
                    xr[nt] = XS ? reinterpret_cast<const uint16_t *>(stg + L::WBYTES + xtok * XSTR) + col0 * QK
                                : xg[nt] + (int64_t)b * QK;
                if (b + BPW <= nb) {
                    Block<C, NT, F16, XS>::template run<BPW>(stg, rowoff + slot * 32, col0, mt, stab, xr, acc, gridtab,
                                                             Ssm + b * 8);
                } else {  // ragged last stage of a row: one block at a time
                    for (int bb = 0; b + bb < nb; bb++) {
                        const uint16_t *xb[NT];
#pragma unroll
                        for (int nt = 0; nt < NT; nt++) xb[nt] = xr[nt] + bb * QK;
                        Block<C, NT, F16, XS>::template run<1>(stg, rowoff + slot * 32, col0 + bb, mt, stab, xb, acc,
                                                               gridtab, Ssm + (b + bb) * 8);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        }

        if (a.debug & 32) continue;  // development: skip the epilogue
        const bool whole = tile_lo >= lo && tile_hi <= hi;
        if constexpr (DP) {
            if (whole) {
                dp_store(T, &acc[0][0], 1, tix);
                tix++;
                continue;
            }
            tix++;
        }
        // ---- reduce the block columns: red[col][tok][row]
        if constexpr (DP) {
            red[warp * RCS + lane] = acc[0][0];
        } else {
            const int g = lane >> 2, t = lane & 3;
            float *r = red + col * 8 * NT * RED_TS;
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                const int row = 16 * mt + g, tok = 8 * nt + 2 * t;
                r[tok * RED_TS + row] = acc[nt][0];
                r[(tok + 1) * RED_TS + row] = acc[nt][1];
                r[tok * RED_TS + row + 8] = acc[nt][2];
                r[(tok + 1) * RED_TS + row + 8] = acc[nt][3];
            }
        }
        named_bar_sync(1, CW * 32);
        const int m = T.m;
        if (whole) {
            for (int q = ctid; q < rows_out * m; q += CW * 32) {
                const int row = q % rows_out, tok = q / rows_out;
                const int n = T.tile * rows_out + row;
                if (n >= a.N) continue;
                float v = 0.f, v2 = 0.f;
#pragma unroll
                for (int w = 0; w < RCOLS; w++) {
                    v += red[w * RCS + tok * RED_TS + row];
                    if (GLU) v2 += red[w * RCS + tok * RED_TS + row + 16];
                }
                if (GLU) v = apply_act(a.act, v) * v2;
                store_out(a.y, a.y_dtype, (int64_t)orow_of(a, T, tok) * a.y_row_stride + n, v + bias_of(a, n));
            }
        } else {
            // partial tile: slot 2c for the CTA's first tile, 2c+1 for its last
            const int64_t pslot = 2 * (int64_t)blockIdx.x + (tile_lo < lo ? 0 : 1);
            float *part = a.partial + pslot * 1024;
            for (int q = ctid; q < 32 * m; q += CW * 32) {
                const int row = q & 31, tok = q >> 5;
                float v = 0.f;
#pragma unroll
                for (int w = 0; w < RCOLS; w++) v += red[w * RCS + tok * RED_TS + row];
                __stcg(part + tok * 32 + row, v);
            }
            // publish: CTA barrier, then one thread orders the CTA's partial
            // stores before its counter increment (gpu-scope fence)
            named_bar_sync(1, CW * 32);
            const int64_t c0 = cta_of(tile_lo, I, P), c1 = cta_of(tile_hi - 1, I, P);
            if (ctid == 0) {
                __threadfence();
                const int old = atomicAdd(a.counters + gt, 1);
                const int last = (old == (int)(c1 - c0));
                if (last) __threadfence();  // acquire the other contributors' partials
                *s_last = last;
            }
            named_bar_sync(1, CW * 32);
            if (*s_last) {
                for (int q = ctid; q < rows_out * m; q += CW * 32) {
                    const int row = q % rows_out, tok = q / rows_out;
                    const int n = T.tile * rows_out + row;
                    if (n >= a.N) continue;
                    float v = 0.f, v2 = 0.f;
                    for (int64_t c = c0; c <= c1; c++) {
                        const int64_t ps = 2 * c + (tile_lo < part_lo(c, I, P) ? 0 : 1);
                        const float *pp = a.partial + ps * 1024 + tok * 32 + row;
                        v += __ldcg(pp);
                        if (GLU) v2 += __ldcg(pp + 16);
                    }
                    if (GLU) v = apply_act(a.act, v) * v2;
                    store_out(a.y, a.y_dtype, (int64_t)orow_of(a, T, tok) * a.y_row_stride + n, v + bias_of(a, n));
                }
                if (ctid == 0) a.counters[gt] = 0;
            }
        }
        // no trailing barrier: the next tile reduces into the other buffer, and
        // the tile after that passes this tile's reads at its own barrier
    }
    if ((a.debug & 128) && ctid == 0) {  // development timing: per-CTA stamps into y (f32 output)
        unsigned *o = reinterpret_cast<unsigned *>(a.y) + a.y_row_stride + 32 * blockIdx.x;  // row 1 of a 2-row f32 buffer
        for (int q = 4; q < 16; q++) o[8 + q] = stamps[q];
        o[0] = g_entry;
        o[1] = stamps[0];
        o[2] = stamps[1];
        o[3] = stamps[2];
        o[4] = (unsigned)(clock64() - c_entry);
        o[5] = (unsigned)(hi - lo);
        o[6] = (unsigned)globaltimer();
    }
}

// host: encoded tensor maps, cached by (base, rows, row bytes, stride, box rows)
typedef CUresult (*GemvEncodeFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
bool gemv_map(CUtensorMap *m, const void *w, int64_t n, int64_t row_bytes, int64_t stride, int box_rows, int box_w) {
    static GemvEncodeFn fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return false;
        fn = reinterpret_cast<GemvEncodeFn>(p);
    }
    if (((uintptr_t)w & 15) || (stride & 15) || (row_bytes & 15) || (box_w & 1) || box_w > 256) return false;
    struct Entry {
        const void *w;
        int64_t n, rb, stride;
        int box, bw;
        CUtensorMap m;
    };
    static thread_local Entry cache[16];
    static thread_local int next = 0;
    for (const Entry &e : cache)
        if (e.w == w && e.n == n && e.rb == row_bytes && e.stride == stride && e.box == box_rows && e.bw == box_w) {
            *m = e.m;
            return true;
        }
    const cuuint64_t dims[2] = {(cuuint64_t)(row_bytes / 8), (cuuint64_t)n};
    const cuuint64_t strides[1] = {(cuuint64_t)stride};
    const cuuint32_t box[2] = {(cuuint32_t)box_w, (cuuint32_t)box_rows};  // the stage row pitch in uint64
    const cuuint32_t es[2] = {1, 1};
    if (fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void *>(w), dims, strides, box, es,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    Entry &e = cache[next];
    next = (next + 1) % 16;
    e = Entry{w, n, row_bytes, stride, box_rows, box_w, *m};
    return true;
}

template <int C, int NT, bool F16, bool GLU, int XR>
cudaError_t configure() {
    static bool done = false;  // per instantiation; the attribute set is idempotent
    if (done) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(gemv_kernel<C, NT, F16, GLU, XR>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, GLayout<C, NT, XR>::BYTES);
    if (e == cudaSuccess) done = true;
    return e;
}

// Grid size and schedule.  Lane-per-row (one activation row) problems hand out
// whole tiles dynamically when there are >= 2 per CTA, or give one whole tile
// to each CTA when the tiles fit the GPU and a tile's stages fit the ring (no
// split-K fixup).  Otherwise stream-K over (tile, stage) iterations.
template <int C, int NT, bool F16, bool GLU, int XR>
int grid_for(const GemvArgs &a, int *dyn = nullptr, int *ksplit = nullptr) {
    using L = GLayout<C, NT, XR>;
    configure<C, NT, F16, GLU, XR>();
    int per_sm = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemv_kernel<C, NT, F16, GLU, XR>, NTHREADS, L::BYTES);
    if (per_sm < 1) per_sm = 1;
    const int rows_out = GLU ? 16 : 32;
    const long tiles = (a.N + rows_out - 1) / rows_out;
    const long groups = a.dense_m > 0 ? (a.dense_m + 31) / 32 : a.max_groups;
    const long nst = (a.K / QK + L::KB - 1) / L::KB;
    const long iters = groups * tiles * nst, units = groups * tiles;
    long cap = (long)num_sms() * per_sm;
    if (const char *g = dev_env("KQ_GEMV_GRID")) cap = atol(g);  // development override
    int d = 0, S = 1;
    if (L::DP && XR == 1 && !dev_env("KQ_GEMV_STATIC")) {
        if (units >= 2 * cap) {
            d = 1;
        } else if (units <= cap && nst <= L::NS) {
            d = 1;
            cap = units;
        } else if (getenv("KQ_GEMV_KSPLIT") || a.ar_world) {  // a supported run-time switch, read per launch
            // split K into chunks so there are >= 2 units per CTA (off by default:
            // each chunk's partial publish stalls its CTA on a gpu-scope fence,
            // slower than stream-K's at most two partial tiles per CTA)
            const long want = (2 * cap + units - 1) / units;
            const long chunk = (nst + (want < nst ? want : nst) - 1) / (want < nst ? want : nst);
            S = (int)((nst + chunk - 1) / chunk);
            d = 1;
        }
    }
    if (XR > 1 && !d) {  // several staged rows: whole tiles handed out dynamically (no K split)
        d = 1;
        if (units < cap) cap = units;
    }
    if (d && L::DP && !a.ar_world && XR == 1)
        if (const char *f = dev_env("KQ_GEMV_FORCE_S")) S = (int)std::min<long>(nst, std::max(1, atoi(f)));  // development
    if (dyn) *dyn = d;
    if (ksplit) *ksplit = S;
    if (!d && iters > cap && !dev_env("KQ_GEMV_GRID")) {
        // stream-K: prefer a grid that gives every CTA the same whole number of
        // stages of one tile (tiles x a divisor of the stages per tile), so no
        // CTA carries an extra stage or two partial tiles; keep >= 70 % of the slots
        for (long sd = nst; sd >= 1; sd--)
            if (nst % sd == 0 && units * sd <= cap) {
                if (units * sd * 10 >= cap * 7) cap = units * sd;
                break;
            }
    }
    return (int)(iters < cap ? iters : cap);
}

template <int C, int NT, bool F16, bool GLU, int XR>
cudaError_t launch_t(const GemvArgs &a, cudaStream_t st, int *grid_out) {
    using L = GLayout<C, NT, XR>;
    cudaError_t e = configure<C, NT, F16, GLU, XR>();
    if (e != cudaSuccess) return e;
    int dyn = 0, ksplit = 1;
    const int grid = grid_for<C, NT, F16, GLU, XR>(a, &dyn, &ksplit);
    if (grid_out) {  // grid size query only: sizes the stream-K partial scratch
        *grid_out = grid;
        return cudaSuccess;
    }
    if (grid <= 0) return cudaSuccess;
    {
        const long tiles = (a.N + (GLU ? 16 : 32) - 1) / (GLU ? 16 : 32);
        const long groups = a.dense_m > 0 ? (a.dense_m + 31) / 32 : a.max_groups;
        if (groups * tiles > 0x7fffffffL) return cudaErrorInvalidValue;  // tile indices are 32-bit in the kernel
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(NTHREADS);
    cfg.dynamicSmemBytes = L::BYTES;
    cfg.stream = st;
    if (a.ar_world && (!L::DP || !dyn)) return cudaErrorInvalidValue;  // fused all-reduce: one-row dynamic schedule
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = dev_env("KQ_GEMV_NOPDL") ? 0 : 1;  // development switch
    GemvArgs b = a;
    b.dyn = dyn;
    b.ksplit = ksplit;
    GemvMaps mp{};
    {
        // dense problems whose wire rows are 16-byte aligned: each stage's
        // rows arrive as one 2-D tensor box (two 16-row boxes for the fused GLU),
        // one copy per stage instead of one per row (per-row copies of ~1 KB
        // leave one SM's copy engine request-bound well below its share of HBM)
        const int64_t rb = (int64_t)a.K / QK * Fmt<C>::bpb;
        if (a.dense_m > 0 && !a.ar_world && !dev_env("KQ_GEMV_NO_TMAP") && L::SP % 16 == 0 &&
            L::STAGE % 128 == 0 && L::OFF_RING % 128 == 0 && (16 * L::SP) % 128 == 0 &&
            gemv_map(&mp.w, a.w, a.N, rb, a.w_row_stride, GLU ? 16 : 32, L::SP / 8) &&
            (!GLU || gemv_map(&mp.w2, a.w2, a.N, rb, a.w2_row_stride, 16, L::SP / 8)))
            mp.use = 1;
    }
    return cudaLaunchKernelEx(&cfg, gemv_kernel<C, NT, F16, GLU, XR>, b, mp);
}

template <int C, bool F16, bool GLU>
cudaError_t launch_nt(const GemvArgs &a, cudaStream_t st, int *grid_out) {
    // one activation row: its slice is staged in the ring with the weights;
    // more rows: MMA B fragments read from global / L1
    // IQ2_XXS groups of 2-4 rows (sparse MoE decode): the lane-per-row integer
    // path with every row staged, each weight decoded once for all rows
    if constexpr (C == IQ2_XXS)
        if (a.max_tokens >= 2 && a.max_tokens <= 4 && a.K <= 32 * S_MAX) return launch_t<C, 1, F16, GLU, 4>(a, st, grid_out);
    switch ((a.max_tokens + 7) / 8) {
    case 1:
        return (a.max_tokens == 1 && a.K <= 32 * S_MAX) ? launch_t<C, 1, F16, GLU, 1>(a, st, grid_out)
                                 : launch_t<C, 1, F16, GLU, 0>(a, st, grid_out);
    case 2: return launch_t<C, 2, F16, GLU, 0>(a, st, grid_out);
    case 3: return launch_t<C, 3, F16, GLU, 0>(a, st, grid_out);
    default: return launch_t<C, 4, F16, GLU, 0>(a, st, grid_out);
    }
}

template <int C>
cudaError_t launch_c(const GemvArgs &a, cudaStream_t st, int *grid_out) {
    const bool f16 = a.x_dtype == F16, glu = a.act != ACT_NONE;
    if (f16) return glu ? launch_nt<C, true, true>(a, st, grid_out) : launch_nt<C, true, false>(a, st, grid_out);
    return glu ? launch_nt<C, false, true>(a, st, grid_out) : launch_nt<C, false, false>(a, st, grid_out);
}

// Q5_K, Q8_0, IQ3_XXS, IQ4_XS, Q2_K, Q3_K and the legacy 32-weight codecs have the lane-per-row path only (one activation row per
// group); the callers route every other shape to the tcgen05 GEMM
template <int C, bool F16, bool GLU>
cudaError_t launch_onerow(const GemvArgs &a, cudaStream_t st, int *grid_out) {
    if (a.max_tokens != 1) return cudaErrorNotSupported;
    return launch_t<C, 1, F16, GLU, 1>(a, st, grid_out);
}

template <int C>
cudaError_t launch_onerow_c(const GemvArgs &a, cudaStream_t st, int *grid_out) {
    const bool f16 = a.x_dtype == F16, glu = a.act != ACT_NONE;
    if (f16) return glu ? launch_onerow<C, true, true>(a, st, grid_out) : launch_onerow<C, true, false>(a, st, grid_out);
    return glu ? launch_onerow<C, false, true>(a, st, grid_out) : launch_onerow<C, false, false>(a, st, grid_out);
}

cudaError_t dispatch(const GemvArgs &a, cudaStream_t st, int *grid_out) {
    if (a.codec == Q5_K) return launch_onerow_c<Q5_K>(a, st, grid_out);
    if (a.codec == Q8_0) return launch_onerow_c<Q8_0>(a, st, grid_out);
    if (a.codec == Q4_0) return launch_onerow_c<Q4_0>(a, st, grid_out);
    if (a.codec == Q4_1) return launch_onerow_c<Q4_1>(a, st, grid_out);
    if (a.codec == MXFP4) return launch_onerow_c<MXFP4>(a, st, grid_out);
    if (a.codec == IQ2_XS) return launch_onerow_c<IQ2_XS>(a, st, grid_out);
    if (a.codec == IQ2_S) return launch_onerow_c<IQ2_S>(a, st, grid_out);
    if (a.codec == IQ3_S) return launch_onerow_c<IQ3_S>(a, st, grid_out);
    if (a.codec == IQ1_S) return launch_onerow_c<IQ1_S>(a, st, grid_out);
    if (a.codec == IQ1_M) return launch_onerow_c<IQ1_M>(a, st, grid_out);
    if (a.codec == TQ2_0) return launch_onerow_c<TQ2_0>(a, st, grid_out);
    if (a.codec == TQ1_0) return launch_onerow_c<TQ1_0>(a, st, grid_out);
    if (a.codec == NVFP4) return launch_onerow_c<NVFP4>(a, st, grid_out);
    if (a.codec == Q5_0) return launch_onerow_c<Q5_0>(a, st, grid_out);
    if (a.codec == Q5_1) return launch_onerow_c<Q5_1>(a, st, grid_out);
    if (a.codec == Q2_K) return launch_onerow_c<Q2_K>(a, st, grid_out);
    if (a.codec == Q3_K) return launch_onerow_c<Q3_K>(a, st, grid_out);
    if (a.codec == IQ4_NL) return launch_onerow_c<IQ4_NL>(a, st, grid_out);
    if (a.codec == IQ3_XXS) return launch_onerow_c<IQ3_XXS>(a, st, grid_out);
    if (a.codec == IQ4_XS) return launch_onerow_c<IQ4_XS>(a, st, grid_out);
    switch (a.codec) {
    case Q4_K: return launch_c<Q4_K>(a, st, grid_out);
    case Q6_K: return launch_c<Q6_K>(a, st, grid_out);
    default: return launch_c<IQ2_XXS>(a, st, grid_out);
    }
}

}  // namespace

void gemv_scratch_need(const GemvArgs &a, size_t *partial_bytes, size_t *counter_bytes) {
    int grid = 0;
    dispatch(a, nullptr, &grid);
    const int rows_out = a.act != ACT_NONE ? 16 : 32;
    const long tiles = (a.N + rows_out - 1) / rows_out;
    const long groups = a.dense_m > 0 ? (a.dense_m + 31) / 32 : a.max_groups;
    *partial_bytes = (size_t)(2 * (long)(grid > 0 ? grid : 1)) * 1024 * sizeof(float);
    *counter_bytes = (size_t)(groups * tiles + 2) * sizeof(int);  // + the dynamic-schedule work counters
}

cudaError_t launch_gemv(const GemvArgs &a, cudaStream_t st) { return dispatch(a, st, nullptr); }

}  // namespace kq
