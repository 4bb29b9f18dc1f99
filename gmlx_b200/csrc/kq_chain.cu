// kq_chain.cu -- a chain of one-row decode GEMVs in ONE persistent launch.
//
// A decoder layer at decode time is a short sequence of quantized matmuls on
// one activation row (q|k|v, o, gate+up, down).  gmlx shrinks the launch
// count by row-concatenating projections that share an input
// (gmlx/occupancy_fuse.py:141-200 q|k|v, :272-330 gate+up and split-K down);
// this kernel streams every projection of a list in one launch:
//
//  * Work units (32-row tile x K chunk) of all problems form one ordered list;
//    CTAs claim them in order (the first by CTA index, then from a counter),
//    so the GPU flows from one projection into the next with no drain.
//  * A problem may read an earlier problem's output (depends_on).  Its tile
//    stores raise that problem's completion counter; the consumers of a CTA
//    reaching a dependent problem wait for the counter while the producer
//    keeps streaming the problem's weights into the ring (weights never
//    depend on anything), so HBM keeps streaming through the hand-off.
//    Deadlock-free: units are claimed in list order and a problem only waits
//    on earlier ones, whose units are all held by running CTAs that wait on
//    nothing later.  Every wait is bounded (~2 s, then an error code in the
//    workspace's first word and the kernel winds down).
//  * One CTA per SM: a producer warp streams each stage -- 32 weight rows x
//    8 super-blocks of wire bytes -- into a ring with ONE 2-D TMA tensor copy
//    (two 16-row boxes for a fused gate/up).  Per-row 1-D bulk copies of
//    ~1 KB cap the SM's copy engine near 20 GB/s; one box per stage streams
//    at full HBM rate.  16 consumer warps (2 row halves x 8 block columns)
//    run the integer tensor-core dot of kq_imma.cuh on each stage.
//  * Each problem's activation row is quantized ONCE per CTA (int16 split
//    into two exact bytes, one f32 scale per 32 values, plus the sums the
//    codecs' offset terms need) into shared memory, when the CTA reaches the
//    problem's first unit -- after its dependency is complete.
//  * K-split units (long rows such as Q6_K down, 14336 inputs) post f32
//    partial rows; the last chunk of a tile to arrive sums them in chunk
//    order (deterministic) and stores.
//  * The last CTA to finish resets the work and completion counters, so the
//    workspace is left zeroed for the next call (as every kq workspace).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "../../include/kq_cuda.h"
#include "kq_gemv_dev.cuh"
#include "kq_imma.cuh"

namespace kq {
namespace {

constexpr int CH_MAX = KQ_CHAIN_MAX;
#ifndef KQ_CHAIN_CW
#define KQ_CHAIN_CW 8
#endif
constexpr int CH_CW = KQ_CHAIN_CW;            // consumer warps: 2 row halves x CH_NBC block columns
constexpr int CH_NBC = CH_CW / 2;             // block columns; each takes 8 / CH_NBC of a stage's 8 blocks
constexpr int CH_PW = CH_CW;                  // producer warp
constexpr int CH_THREADS = 32 * (CH_CW + 2);  // + producer + epilogue
constexpr int CH_EQ = 8;                      // finished-tile queue entries
constexpr int CH_KMAX = 16384;                // activation row length held quantized in shared memory
constexpr int CH_XQB = 101 * IMMA_XB;          // quantized activation rows of a chain (deduplicated)
constexpr int CH_SMEM = 232448;               // one CTA per SM

struct alignas(64) ChainProb {
    CUtensorMap tmw, tmw2;  // weight rows as [rows][row bytes / 8] uint64 tensors (w2: fused gate/up's up)
    const uint8_t *w, *w2;
    int64_t w_row_stride;
    const uint8_t *x;  // one activation row (f16 / bf16)
    void *y;
    const void *bias;
    int y_dtype, bias_dtype;
    int N, K, codec, act, dep;
    int counted;       // a later problem depends on this one: count finished tiles
    int tiles, nst, S, chunk;
    int unit_base, split_base;
    int xreg, xoff;    // activation region (rows shared by several problems share one) and its byte offset
    int cmajor;        // units ordered chunk-major (a K-split problem reading another's output)
    int rows_out;      // output rows per tile (32, or 16 for a fused gate/up)
};

// Completion is counted per slab of 4096 output rows (one K chunk of two
// 8-block stages of a problem that reads this output), so a dependent chunk
// waits only for the tiles that produce its inputs.
constexpr int CH_SLAB = 4096;
constexpr int CH_SLABS = 4;  // K <= 16384

struct ChainArgs {
    ChainProb p[CH_MAX];
    int count, total_units, nreg;
    int *err;
    int *ctl;         // [0] work counter, [1] finished CTAs, [16 + 4 p + s] finished tiles of slab s of problem p
    int *tcnt;        // K-split tile counters
    float *partial;   // K-split partial rows [split tile][S][32]
    int debug;        // development builds only: 1 = consumers skip the arithmetic, 2 = no weight copies,
                      // 4 = no activation quantization, 8 = no consumer barriers, 16 = no dependency wait,
                      // 32 = epilogue without fences (wrong results; timing only),
                      // 64 = CTA 0 records stage timestamps into dbg
    unsigned long long *dbg;  // development: [0,256) issue, [256,512) full seen, [512,768) slot free
};

// a stage: 8 super-blocks of 32 rows; the box row pitch is == 16 (mod 128)
// bytes, so the 8 rows x 4 words of an MMA fragment load hit 32 banks
// (Q4_K: 1152 bytes + 16 bytes of the next block; Q6_K: exactly 1680)
template <int C> constexpr int ch_kb() { return 8; }
template <int C> constexpr int ch_boxw() { return C == Q4_K ? 146 : 210; }  // uint64 elements per box row
template <int C> constexpr int ch_sp() { return 8 * ch_boxw<C>(); }
template <int C> constexpr int ch_wbytes() { return 32 * ch_sp<C>(); }
constexpr int cmax(int a, int b) { return a > b ? a : b; }

template <int CA, int CB> struct ChainLayout {
    static constexpr int SLOT = cmax(ch_wbytes<CA>(), ch_wbytes<CB>());  // one stage: 32 weight rows
    static constexpr int OFF_BAR = 0;       // full[NS], empty[NS]
    static constexpr int OFF_UNIT = 128;    // s_unit[8]
    static constexpr int OFF_MISC = 512;    // abort flag, sync counter, partial-buffer counters
    static constexpr int OFF_EBAR = 576;    // tile-queue mbarriers: efull[EQ], eempty[EQ]
    static constexpr int OFF_EQ = 768;      // tile queue: [EQ] x (q, tile, chunk, pad, 32 f32 row sums)
    static constexpr int EQ_ENTRY = 144;
    static constexpr int OFF_XQ = OFF_EQ + CH_EQ * EQ_ENTRY;  // the chain's quantized activation rows
    static constexpr int RB_ONE = 8 * 32 * 4;  // [block column][tile row] partials
    static constexpr int OFF_RB = OFF_XQ + CH_XQB;
    static constexpr int NS_FIT = (CH_SMEM - OFF_RB - RB_ONE - 128) / (SLOT + RB_ONE);  // NS + 1 partial buffers
    static constexpr int NS = NS_FIT > 6 ? 6 : NS_FIT;
    static constexpr int OFF_RING = (OFF_RB + (NS + 1) * RB_ONE + 127) / 128 * 128;
    static constexpr int BYTES = OFF_RING + NS * SLOT + 16;  // + the tail the 2-byte-aligned Q6_K reads may touch
    static_assert(NS >= 3, "ring must hold three stages");
    static_assert(OFF_RING % 128 == 0 && SLOT % 128 == 0, "TMA destinations");
    static_assert(BYTES <= CH_SMEM, "shared memory");
};

__device__ __forceinline__ void tma_box(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar,
                                        uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// Bring a box into L2 ahead of its shared-memory copy (no completion to wait on).
__device__ __forceinline__ void tma_prefetch_l2(const CUtensorMap *map, int x, int y) {
    asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(map), "r"(x), "r"(y)
                 : "memory");
}

__device__ __forceinline__ int ld_acquire(const int *p) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ int prob_of(const ChainArgs &a, int unit) {
    int p = 0;
#pragma unroll 1
    while (p + 1 < a.count && unit >= a.p[p + 1].unit_base) p++;
    return p;
}

// Bounded mbarrier wait that sleeps between checks (see mbar_try_wait_sleep):
// gives up after ~2 s or when another warp gave up, records `code` once.
__device__ int g_chain_wait_mode;  // development: 0 sleeping try_wait, 1 try_wait, 2 test_wait spin

__device__ __forceinline__ bool ch_wait(uint64_t *bar, uint32_t parity, volatile int *abort, int *err, int code) {
    uint64_t t0 = 0;
    const int mode = g_chain_wait_mode;
    for (;;) {
        for (int i = 0; i < 64; i++)
            if (mode == 0 ? mbar_try_wait_sleep(bar, parity, 20000)
                          : mode == 1 ? mbar_try_wait(bar, parity) : mbar_test_wait(bar, parity))
                return true;
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

// the stages [s0, s1) of a unit's tile
__device__ __forceinline__ void unit_stages(const ChainProb &P, int unit, int &tile, int &chunk, int &s0, int &s1) {
    const int lu = unit - P.unit_base;
    if (P.cmajor) {  // chunk 0 of every tile first: its inputs are the first to be ready
        chunk = lu / P.tiles;
        tile = lu - chunk * P.tiles;
    } else {
        tile = lu / P.S;
        chunk = lu - tile * P.S;
    }
    s0 = chunk * P.chunk;
    s1 = min(P.nst, s0 + P.chunk);
}

// Bounded barrier of the consumer warps (a monotonic shared counter): false
// when the kernel is aborting or ~2 s passed.
__device__ __forceinline__ bool consumers_sync(int *ctr, int target, volatile int *abort, int *err) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) {
        __threadfence_block();
        atomicAdd(ctr, 1);
    }
    uint64_t t0 = 0;
    for (uint32_t i = 1;; i++) {
        if (*reinterpret_cast<volatile int *>(ctr) >= target) break;
        if (*abort) return false;
        __nanosleep(64);
        if ((i & 255) == 0) {
            const uint64_t now = globaltimer();
            if (t0 == 0) t0 = now;
            if (now - t0 > 2000000000ull) {
                *abort = 1;
                atomicCAS(err, 0, 4);
                return false;
            }
        }
    }
    __threadfence_block();
    __syncwarp();
    return true;
}

template <int CA, int CB, bool F16>
__global__ void __launch_bounds__(CH_THREADS, 1) chain_kernel(const __grid_constant__ ChainArgs a) {
    using L = ChainLayout<CA, CB>;
    constexpr int NS = L::NS;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L::OFF_BAR);
    uint64_t *empty = full + NS;
    int *s_unit = reinterpret_cast<int *>(smem + L::OFF_UNIT);
    volatile int *s_abort = reinterpret_cast<volatile int *>(smem + L::OFF_MISC);
    int *s_sync = reinterpret_cast<int *>(smem + L::OFF_MISC + 4);
    int *dcnt = reinterpret_cast<int *>(smem + L::OFF_MISC + 16);  // NS + 1 partial-buffer counters
    uint8_t *xq8 = smem + L::OFF_XQ;
    uint8_t *ring = smem + L::OFF_RING;
    uint64_t *efull = reinterpret_cast<uint64_t *>(smem + L::OFF_EBAR);
    uint64_t *eempty = efull + CH_EQ;
    uint8_t *equeue = smem + L::OFF_EQ;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if ((a.debug & 128) && threadIdx.x == 0 && blockIdx.x < 256) a.dbg[1024 + 4 * blockIdx.x] = globaltimer();

    if (threadIdx.x == 0) {
        for (int i = 0; i < NS; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], CH_CW);
        }
        for (int i = 0; i < CH_EQ; i++) {
            mbar_init(&efull[i], 1);
            mbar_init(&eempty[i], 1);
        }
        *s_abort = 0;
        *s_sync = 0;
        for (int b = 0; b <= NS; b++) dcnt[b] = 0;
        fence_mbar_init();
    }
    __syncthreads();
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    if (warp == CH_PW) {
        // ---------------- producer: lane r streams tile row r of every stage ----------------
        const uint64_t pol = policy_evict_first();
        uint32_t it = 0;
        bool dep_done = false;
        // lane 0 claims units two ahead (pend: the next unit, nn: the one after),
        // so a claim's round trip hides behind a whole unit of copies
        int unit = blockIdx.x, pend = -1, nn = -1, n3 = -1;  // claims: next, after next, third
        bool first_unit = true;
        while (!*s_abort) {
            if (unit >= a.total_units) {  // end marker: a stage with a negative unit id
                const int slot = it % NS;
                if (ch_wait(&empty[slot], ((it / NS) & 1) ^ 1, s_abort, a.err, 1) && lane == 0) {
                    s_unit[slot] = -1;
                    mbar_arrive(&full[slot]);
                }
                it++;
                break;
            }
            const int p = prob_of(a, unit);
            const ChainProb &P = a.p[p];
            int tile, chunk, s0, s1;
            unit_stages(P, unit, tile, chunk, s0, s1);
            const bool glu = P.act != ACT_NONE;
            const bool ca = P.codec == CA;
            const int boxw = ca ? ch_boxw<CA>() : ch_boxw<CB>(), xstep = ca ? Fmt<CA>::bpb : Fmt<CB>::bpb;
            // the next claimed unit's weights to L2 now: its stage copies a unit from now then
            // come from L2, so more bytes are in flight than the ring holds
            if (!first_unit && lane == 0 && nn >= 0 && nn < a.total_units && !(a.debug & 2) &&
                !(a.debug & 512)) {  // the unit after next (its claim is a unit old)
                const int pq = prob_of(a, nn);
                const ChainProb &Q = a.p[pq];
                int qt, qc, q0, q1;
                unit_stages(Q, nn, qt, qc, q0, q1);
                const int qstep = Q.codec == CA ? Fmt<CA>::bpb : Fmt<CB>::bpb;
                for (int qs = q0; qs < q1; qs++) {
                    if (Q.act != ACT_NONE) {
                        tma_prefetch_l2(&Q.tmw, qs * qstep, qt * 16);
                        tma_prefetch_l2(&Q.tmw2, qs * qstep, qt * 16);
                    } else {
                        tma_prefetch_l2(&Q.tmw, qs * qstep, qt * 32);
                    }
                }
            }
            const uint32_t stage_bytes = 32u * 8u * (uint32_t)boxw;
            for (int st = s0; st < s1; st++, it++) {
                const int slot = it % NS;
                if (!ch_wait(&empty[slot], ((it / NS) & 1) ^ 1, s_abort, a.err, 1)) break;
                if ((a.debug & 64) && blockIdx.x == 0 && lane == 0 && it < 256) a.dbg[512 + it] = globaltimer();
                if (lane == 0) {
                    s_unit[slot] = unit;
                    uint8_t *dst = ring + slot * L::SLOT;
                    const int x = st * xstep;  // 8 blocks of bpb bytes = bpb uint64 elements
                    if (a.debug & 2) {
                        mbar_arrive(&full[slot]);
                    } else {
                        mbar_arrive_expect_tx(&full[slot], stage_bytes);
                        if (glu) {  // 16 gate rows over the same 16 up rows
                            tma_box(dst, &P.tmw, x, tile * 16, &full[slot], pol);
                            tma_box(dst + 16 * 8 * boxw, &P.tmw2, x, tile * 16, &full[slot], pol);
                        } else {
                            tma_box(dst, &P.tmw, x, tile * 32, &full[slot], pol);
                        }
                    }
                }
                __syncwarp();
                if ((a.debug & 64) && blockIdx.x == 0 && lane == 0 && it < 256) a.dbg[it] = globaltimer();
                if (!dep_done) {  // first weights in flight; the work counter is the previous kernel's
                    asm volatile("griddepcontrol.wait;" ::: "memory");
                    dep_done = true;
                }
                if (st == s0 && lane == 0) {
                    if (first_unit) {
                        pend = (int)gridDim.x + atomicAdd(a.ctl, 1);
                        nn = (int)gridDim.x + atomicAdd(a.ctl, 1);
                    }
                    n3 = (int)gridDim.x + atomicAdd(a.ctl, 1);
                }
            }
            first_unit = false;
            unit = __shfl_sync(0xffffffffu, pend, 0);
            pend = nn;
            nn = n3;
        }
        if (*s_abort) {
            // gave up: wait (bounded) until the copies this CTA issued last have
            // landed, so none writes shared memory after the CTA is gone
            const uint64_t t0 = globaltimer();
            for (uint32_t i = it > (uint32_t)NS ? it - NS : 0; i < it; i++)
                while (!mbar_try_wait(&full[i % NS], (i / NS) & 1) && globaltimer() - t0 < 500000000ull) {
                }
        }
    } else if (warp < CH_CW) {
        // ---------------- consumers: warp = (row half, block column) ----------------
        // thread (g, tq) of the m16n8k32 fragments holds rows g and g + 8 of
        // its warp's 16-row half of the tile
        const int rh = warp & 1, bc = warp >> 1, g = lane >> 2, tq = lane & 3;
        const int r0 = 16 * rh + g, r1 = r0 + 8;
        asm volatile("griddepcontrol.wait;" ::: "memory");
        // quantize one activation row into its region; warps take blocks in turn
        auto quantize_row = [&](const ChainProb &P, int bb0, int bb1) {
            const int nb = (a.debug & 4) ? bb0 : bb1;
            const uint16_t *xs = reinterpret_cast<const uint16_t *>(P.x);
            uint8_t *dst = xq8 + P.xoff;
            for (int b0 = bb0 + warp; b0 < nb; b0 += 4 * CH_CW) {
                uint4 v[4];
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const int b = b0 + u * CH_CW;
                    if (b < nb) v[u] = __ldcg(reinterpret_cast<const uint4 *>(xs + (int64_t)b * QK + 8 * lane));
                }
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const int b = b0 + u * CH_CW;
                    if (b < nb) imma_quantize<F16>(v[u], dst + b * IMMA_XB);
                }
            }
        };
        // rows that depend on nothing (the chain's inputs) are quantized up front
        unsigned ready = 0;
        int sync_target = 0;
        for (int q = 0; q < a.count; q++) {
            const ChainProb &P = a.p[q];
            const unsigned all = ((1u << CH_SLABS) - 1) << (P.xreg * CH_SLABS);
            if (P.dep < 0 && (ready & all) != all) {
                quantize_row(P, 0, P.K / QK);
                ready |= all;
            }
        }
        sync_target += CH_CW;
        consumers_sync(s_sync, sync_target, s_abort, a.err);
        if ((a.debug & 128) && warp == 0 && lane == 0 && blockIdx.x < 256) a.dbg[1025 + 4 * blockIdx.x] = globaltimer();
        uint32_t it = 0;
        int tix = 0;
        const bool tr = (a.debug & 64) && blockIdx.x == 0;  // development: time accounting, every consumer warp
        uint64_t t_wait = 0, t_comp = 0, t_store = 0, t_switch = 0, tm = tr ? globaltimer() : 0;
        auto lap = [&](uint64_t &acc) {
            if (tr) {
                const uint64_t n = globaltimer();
                acc += n - tm;
                tm = n;
            }
        };
        for (;;) {
            const int slot = it % NS;
            lap(t_store);
            if (!ch_wait(&full[slot], (it / NS) & 1, s_abort, a.err, 2)) break;
            lap(t_wait);
            const int unit = s_unit[slot];
            if (unit < 0 || *s_abort) break;
            const int q = prob_of(a, unit);
            const ChainProb &P = a.p[q];
            int tile, chunk, s0, s1;
            unit_stages(P, unit, tile, chunk, s0, s1);
            if (P.dep >= 0) {
                // this unit's inputs: activation blocks [8 s0, 8 s1) of a row that is
                // problem P.dep's output.  Slabs of 16 blocks (4096 values) are made
                // ready once per CTA: each warp waits for the slab's completion count,
                // quantizes its blocks, then all consumers meet once.
                const int sl0 = (8 * s0 * QK) / CH_SLAB, sl1 = min(CH_SLABS, (min(8 * s1 * QK, P.K) + CH_SLAB - 1) / CH_SLAB);
                const ChainProb &D = a.p[P.dep];
                bool fresh = false;
                for (int sl = sl0; sl < sl1; sl++) {
                    const unsigned bit = 1u << (P.xreg * CH_SLABS + sl);
                    if (ready & bit) continue;
                    fresh = true;
                    if (lane == 0 && !(a.debug & 16)) {
                        const int t0s = sl * CH_SLAB / D.rows_out;
                        const int need = min(D.tiles, (sl + 1) * CH_SLAB / D.rows_out) - t0s;
                        const uint64_t t0 = globaltimer();
                        while (ld_acquire(a.ctl + 16 + 4 * P.dep + sl) < need) {
                            if (*s_abort) break;
                            __nanosleep(128);
                            if (globaltimer() - t0 > 2000000000ull) {
                                *s_abort = 1;
                                atomicCAS(a.err, 0, 3);
                                break;
                            }
                        }
                    }
                    __syncwarp();
                    quantize_row(P, sl * (CH_SLAB / QK), min(P.K / QK, (sl + 1) * (CH_SLAB / QK)));
                    ready |= bit;
                }
                if (fresh) {
                    sync_target += CH_CW;
                    if (!(a.debug & 8) && !consumers_sync(s_sync, sync_target, s_abort, a.err)) break;
                }
                lap(t_switch);
            }
            const int nb = P.K / QK;
            const bool q6 = P.codec == Q6_K;
            float acc0 = 0.f, acc1 = 0.f;
            bool ok = true;
            for (int st = s0; st < s1; st++, it++) {
                const int sl = it % NS;
                lap(t_comp);
                if (st > s0 && !ch_wait(&full[sl], (it / NS) & 1, s_abort, a.err, 2)) {
                    ok = false;
                    break;
                }
                lap(t_wait);
                if ((a.debug & 64) && blockIdx.x == 0 && warp == 0 && lane == 0 && it < 256)
                    a.dbg[256 + it] = globaltimer();  // (warp 0: when it saw the stage full)
                const uint8_t *stg = ring + sl * L::SLOT;
                if (!*s_abort && !(a.debug & 1)) {
#pragma unroll
                    for (int i = 0; i < 8 / CH_NBC; i++) {  // independent blocks: their latencies overlap
                        const int bi = bc + CH_NBC * i, b = st * 8 + bi;
                        if (b < nb) {
                            if (!q6) {
                                imma_q4k(stg + r0 * ch_sp<Q4_K>() + bi * 144, stg + r1 * ch_sp<Q4_K>() + bi * 144,
                                         xq8 + P.xoff + b * IMMA_XB, g, tq, acc0, acc1);
                            } else {  // Q6_K: both 128-value halves of the block
                                const uint8_t *b0 = stg + r0 * ch_sp<Q6_K>() + bi * 210,
                                              *b1 = stg + r1 * ch_sp<Q6_K>() + bi * 210;
                                imma_q6k(b0, b1, 0, xq8 + P.xoff + b * IMMA_XB, g, tq, acc0, acc1);
                                imma_q6k(b0, b1, 1, xq8 + P.xoff + b * IMMA_XB, g, tq, acc0, acc1);
                            }
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[sl]);
            }
            lap(t_comp);
            if (!ok || *s_abort) break;
            // the four lanes of a row (tq) each hold a quarter of its sub-blocks
            acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
            acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
            acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
            acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
            // tile store: each warp posts its 16 row partials (lanes tq == 0);
            // the last of the 16 warps to arrive sums the 8 block columns of
            // every row in column order (and K chunks in chunk order through
            // the partial buffer) and stores
            const int bi = tix % (NS + 1);
            float *rb = reinterpret_cast<float *>(smem + L::OFF_RB) + bi * (8 * 32);
            if (tq == 0) {
                rb[bc * 32 + r0] = acc0;
                rb[bc * 32 + r1] = acc1;
            }
            __syncwarp();
            int old = 0;
            if (lane == 0) {
                __threadfence_block();
                old = atomicAdd(dcnt + bi, 1);
            }
            old = __shfl_sync(0xffffffffu, old, 0);
            tix++;
            if (old != CH_CW - 1) continue;
            // the last warp of the unit hands the tile's 32 row sums to the
            // epilogue warp through the queue (entry = the unit's sequence
            // number, the same in every warp), so no consumer waits on a fence
            __threadfence_block();
            float u = 0.f;
#pragma unroll
            for (int c = 0; c < CH_NBC; c++) u += rb[c * 32 + lane];
            const int e = (tix - 1) % CH_EQ;
            if (!ch_wait(&eempty[e], (((tix - 1) / CH_EQ) & 1) ^ 1, s_abort, a.err, 5)) break;
            int *ent = reinterpret_cast<int *>(equeue + e * L::EQ_ENTRY);
            reinterpret_cast<float *>(ent + 4)[lane] = u;
            if (lane == 0) {
                ent[0] = q;
                ent[1] = tile;
                ent[2] = chunk;
            }
            __syncwarp();
            if (lane == 0) {
                dcnt[bi] = 0;
                mbar_arrive(&efull[e]);
            }
        }
        if ((a.debug & 128) && warp == 0 && lane == 0 && blockIdx.x < 256) a.dbg[1026 + 4 * blockIdx.x] = globaltimer();
        if (tr && lane == 0) {
            a.dbg[768 + 8 * warp] = t_wait;
            a.dbg[769 + 8 * warp] = t_comp;
            a.dbg[770 + 8 * warp] = t_store;
            a.dbg[771 + 8 * warp] = t_switch;
            a.dbg[772 + 8 * warp] = (unsigned long long)tix;
        }
        // end of work: one warp queues the end marker for the epilogue warp
        if (warp == 0 && !*s_abort) {
            const int e = tix % CH_EQ;
            if (ch_wait(&eempty[e], ((tix / CH_EQ) & 1) ^ 1, s_abort, a.err, 5) && lane == 0) {
                reinterpret_cast<int *>(equeue + e * L::EQ_ENTRY)[0] = -1;
                mbar_arrive(&efull[e]);
            }
        }
    } else {
        // ---------------- epilogue: finished tiles, in unit order ----------------
        for (uint32_t n = 0;; n++) {
            const int e = n % CH_EQ;
            if (!ch_wait(&efull[e], (n / CH_EQ) & 1, s_abort, a.err, 6)) break;
            const int *ent = reinterpret_cast<const int *>(equeue + e * L::EQ_ENTRY);
            const int q = ent[0], tile = ent[1], chunk = ent[2];
            if (q < 0) break;
            const float u = reinterpret_cast<const float *>(ent + 4)[lane];
            __syncwarp();
            if (lane == 0) mbar_arrive(&eempty[e]);
            const ChainProb &P = a.p[q];
            const bool glu = P.act != ACT_NONE;
            const int row = glu ? (lane & 15) : lane;
            bool store = true;
            float v = 0.f, v2 = 0.f;
            if (P.S > 1) {  // K-split: the last chunk of the tile to arrive sums them in chunk order
                const int stile = P.split_base + tile;
                __stcg(a.partial + ((int64_t)stile * P.S + chunk) * 32 + lane, u);
                if (!(a.debug & 32)) __threadfence();
                __syncwarp();
                int prev = 0;
                if (lane == 0) {
                    prev = atomicAdd(a.tcnt + stile, 1);
                    if (prev == P.S - 1 && !(a.debug & 32)) __threadfence();
                }
                prev = __shfl_sync(0xffffffffu, prev, 0);
                store = prev == P.S - 1;
                if (store) {
                    for (int c = 0; c < P.S; c++) {
                        const float *pp = a.partial + ((int64_t)stile * P.S + c) * 32;
                        v += __ldcg(pp + row);
                        if (glu) v2 += __ldcg(pp + row + 16);
                    }
                    if (lane == 0) a.tcnt[stile] = 0;
                }
            } else {
                v = __shfl_sync(0xffffffffu, u, row);
                v2 = __shfl_sync(0xffffffffu, u, (row + 16) & 31);
            }
            if (store) {
                if (glu) v = apply_act(P.act, v) * v2;
                const int nn = tile * (glu ? 16 : 32) + row;
                if (nn < P.N && (!glu || lane < 16)) {
                    float bv = 0.f;
                    if (P.bias) {
                        if (P.bias_dtype == F32) bv = reinterpret_cast<const float *>(P.bias)[nn];
                        else if (P.bias_dtype == BF16)
                            bv = __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(P.bias)[nn]);
                        else bv = __half2float(reinterpret_cast<const __half *>(P.bias)[nn]);
                    }
                    store_out(P.y, P.y_dtype, nn, v + bv);
                }
                if (P.counted) {  // publish the finished tile to dependent problems (its slab's count)
                    if (!(a.debug & 32)) __threadfence();
                    __syncwarp();
                    if (lane == 0) atomicAdd(a.ctl + 16 + 4 * q + tile * P.rows_out / CH_SLAB, 1);
                }
            }
        }
    }
    // the last CTA out resets the work and completion counters
    __syncthreads();
    if ((a.debug & 128) && threadIdx.x == 0 && blockIdx.x < 256) a.dbg[1027 + 4 * blockIdx.x] = globaltimer();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(a.ctl + 1, 1) == (int)gridDim.x - 1) {
            __threadfence();
            a.ctl[0] = 0;
            for (int q = 0; q < 4 * CH_MAX; q++) a.ctl[16 + q] = 0;
            __threadfence();
            a.ctl[1] = 0;
        }
    }
}

template <int CA, int CB, bool F16>
cudaError_t launch_chain_t(const ChainArgs &a, cudaStream_t st) {
    using L = ChainLayout<CA, CB>;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(chain_kernel<CA, CB, F16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             L::BYTES);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    int per_sm = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, chain_kernel<CA, CB, F16>, CH_THREADS, L::BYTES);
    if (per_sm < 1) return cudaErrorInvalidConfiguration;  // the kernel needs one whole SM
    int grid = num_sms() * per_sm;
    if (const char *g = dev_env("KQ_CHAIN_GRID")) grid = atoi(g);  // development override
    grid = std::min(grid, a.total_units);
    if (grid <= 0) return cudaSuccess;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(CH_THREADS);
    cfg.dynamicSmemBytes = L::BYTES;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, chain_kernel<CA, CB, F16>, a);
}

int chain_kb(int codec) { return codec == Q4_K ? ch_kb<Q4_K>() : ch_kb<Q6_K>(); }

// host: tensor maps through the driver entry point
typedef CUresult (*ChainEncodeFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
ChainEncodeFn chain_encode() {
    static ChainEncodeFn fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<ChainEncodeFn>(p);
    }
    return fn;
}

// A weight matrix's wire rows as a 2-D tensor of uint64 elements [n][row
// bytes / 8]; boxes of `box_rows` rows x one stage (plus the pitch pad).  Rows
// past n and bytes past the row read as zeros.
bool chain_map(CUtensorMap *m, const void *w, int64_t n, int64_t row_bytes, int64_t row_stride, int boxw,
               int box_rows) {
    ChainEncodeFn fn = chain_encode();
    if (!fn) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)(row_bytes / 8), (cuuint64_t)n};
    const cuuint64_t strides[1] = {(cuuint64_t)row_stride};
    const cuuint32_t box[2] = {(cuuint32_t)boxw, (cuuint32_t)box_rows};
    const cuuint32_t es[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void *>(w), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

// Host plan: units and K chunks per problem, scratch sizes.  The fused kernel
// takes Q4_K and Q6_K problems (the Q4_K_M mix) with K <= 16384.
bool chain_plan(const ChainProblemDesc *pd, int count, ChainPlan *out) {
    if (count < 1 || count > CH_MAX) return false;
    for (int q = 0; q < count; q++) {
        const ChainProblemDesc &d = pd[q];
        if (d.codec != Q4_K && d.codec != Q6_K) return false;
        if (d.k > CH_KMAX) return false;  // the activation row must fit in shared memory
        // the weights must be describable as a TMA tensor: 16-byte aligned base
        // and row stride, rows a whole number of 8-byte elements
        const int64_t row_bytes = d.k / QK * (d.codec == Q4_K ? 144 : 210);
        if (row_bytes % 8 || d.w_row_stride % 16 || (uintptr_t)d.w % 16 || (d.w2 && (uintptr_t)d.w2 % 16))
            return false;
        if (d.n > (1 << 30)) return false;
    }
    int chunk_stages = 2;
    if (const char *e = dev_env("KQ_CHAIN_CHUNK")) chunk_stages = std::max(1, atoi(e));  // development override
    ChainPlan pl{};
    pl.pair = 0;
    long units = 0, split_tiles = 0, partial_floats = 0;
    for (int q = 0; q < count; q++) {
        const ChainProblemDesc &d = pd[q];
        const int kb = chain_kb(d.codec);
        const long rows_out = d.act != ACT_NONE ? 16 : 32;
        const long tiles = (d.n + rows_out - 1) / rows_out;
        const long nst = (d.k / QK + kb - 1) / kb;
        const long chunk = std::min<long>(nst, chunk_stages);
        const long S = (nst + chunk - 1) / chunk;
        pl.tiles[q] = (int)tiles;
        pl.nst[q] = (int)nst;
        pl.S[q] = (int)S;
        pl.chunk[q] = (int)chunk;
        pl.unit_base[q] = (int)units;
        pl.split_base[q] = (int)split_tiles;
        units += tiles * S;
        if (S > 1) {
            split_tiles += tiles;
            partial_floats += tiles * S * 32;
        }
    }
    // activation regions: one per distinct row (pointer, length), packed
    int nreg = 0;
    long xbytes = 0;
    for (int q = 0; q < count; q++) {
        int r = -1;
        for (int p = 0; p < q && r < 0; p++)
            if (pd[p].x == pd[q].x && pd[p].k == pd[q].k) r = pl.xreg[p];
        if (r < 0) {
            r = nreg++;
            pl.xoff[q] = (int)xbytes;
            xbytes += pd[q].k / QK * IMMA_XB;
        } else {
            for (int p = 0; p < q; p++)
                if (pl.xreg[p] == r) {
                    pl.xoff[q] = pl.xoff[p];
                    break;
                }
        }
        pl.xreg[q] = r;
    }
    if (xbytes > CH_XQB) return false;  // the chain's activation rows must fit in shared memory
    pl.nreg = nreg;
    if (units > 0x3fffffffL) return false;
    pl.total_units = (int)units;
    pl.split_tiles = split_tiles;
    pl.partial_floats = partial_floats;
    *out = pl;
    return true;
}

cudaError_t launch_chain(const ChainProblemDesc *pd, int count, const ChainPlan &pl, int x_dtype, int *err, int *ctl,
                         int *tcnt, float *partial, cudaStream_t st) {
    ChainArgs a{};
    a.count = count;
    a.nreg = pl.nreg;
    a.total_units = pl.total_units;
    a.err = err;
    a.ctl = ctl;
    a.tcnt = tcnt;
    a.partial = partial;
    if (const char *e = dev_env("KQ_CHAIN_DEBUG")) a.debug = atoi(e);  // development switch
    if (const char *e = dev_env("KQ_CHAIN_WAIT")) {                    // development switch
        const int m = atoi(e);
        cudaMemcpyToSymbolAsync(g_chain_wait_mode, &m, sizeof(int), 0, cudaMemcpyHostToDevice, st);
    }
    a.dbg = reinterpret_cast<unsigned long long *>(reinterpret_cast<char *>(partial) + (1 << 20));
    for (int q = 0; q < count; q++) {
        ChainProb &P = a.p[q];
        const ChainProblemDesc &d = pd[q];
        P.w = (const uint8_t *)d.w;
        P.w2 = (const uint8_t *)d.w2;
        P.w_row_stride = d.w_row_stride;
        P.x = (const uint8_t *)d.x;
        P.y = d.y;
        P.bias = d.bias;
        P.y_dtype = d.y_dtype;
        P.bias_dtype = d.bias_dtype;
        P.N = (int)d.n;
        P.K = (int)d.k;
        P.codec = d.codec;
        P.act = d.act;
        P.dep = d.dep;
        P.counted = 0;
        for (int r = q + 1; r < count; r++) P.counted |= pd[r].dep == q;
        P.rows_out = d.act != ACT_NONE ? 16 : 32;
        P.cmajor = d.dep >= 0 && P.S > 1;
        P.tiles = pl.tiles[q];
        P.nst = pl.nst[q];
        P.S = pl.S[q];
        P.chunk = pl.chunk[q];
        P.unit_base = pl.unit_base[q];
        P.split_base = pl.split_base[q];
        P.xreg = pl.xreg[q];
        P.xoff = pl.xoff[q];
        const bool q4 = d.codec == Q4_K;
        const int64_t row_bytes = d.k / QK * (q4 ? 144 : 210);
        const int boxw = q4 ? ch_boxw<Q4_K>() : ch_boxw<Q6_K>(), rows = d.act != ACT_NONE ? 16 : 32;
        if (!chain_map(&P.tmw, d.w, d.n, row_bytes, d.w_row_stride, boxw, rows)) return cudaErrorInvalidValue;
        if (d.act != ACT_NONE && !chain_map(&P.tmw2, d.w2, d.n, row_bytes, d.w_row_stride, boxw, rows))
            return cudaErrorInvalidValue;
    }
    return x_dtype == F16 ? launch_chain_t<Q4_K, Q6_K, true>(a, st) : launch_chain_t<Q4_K, Q6_K, false>(a, st);
}

}  // namespace kq
