// kq_capi.cu -- the extern "C" entry points declared in include/kq_cuda.h.
//
// Host-side validation (codec, block-multiple K, alignment, dtypes, workspace
// size) happens before any launch and reports a KQ_ERR_* code plus a
// thread-local message; nothing throws across the ABI.  Mirrors the loud
// failures of the reference's module swap (unknown codec -> error,
// gmlx/modules.py:1561-1574; geometry rules gmlx/modules.py:502-509).
#include <cuda_runtime.h>
#include <algorithm>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "../../include/kq_cuda.h"
#include "kq_internal.cuh"

namespace kq {

int num_sms() {
    static int cache[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!cache[dev]) {
        int v = 0;
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        cache[dev] = v > 0 ? v : 148;
    }
    return cache[dev];
}

}  // namespace kq

using namespace kq;

namespace {

thread_local char g_msg[512];

int fail(int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
    va_end(ap);
    return code;
}

int cuda_status(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return KQ_OK;
    return fail(KQ_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool codec_ok(int c) {
    return c == KQ_Q4_K || c == KQ_Q5_K || c == KQ_Q6_K || c == KQ_IQ2_XXS || c == KQ_Q8_0 || c == KQ_IQ3_XXS ||
           c == KQ_IQ4_XS || c == KQ_Q4_0 || c == KQ_IQ4_NL || c == KQ_Q2_K || c == KQ_Q3_K || c == KQ_Q4_1 ||
           c == KQ_Q5_0 || c == KQ_Q5_1 || c == KQ_TQ2_0 || c == KQ_MXFP4 || c == KQ_IQ2_XS || c == KQ_IQ2_S ||
           c == KQ_IQ3_S || c == KQ_IQ1_S || c == KQ_IQ1_M || c == KQ_TQ1_0 || c == KQ_NVFP4;
}
// codecs whose only GEMV is the one-row (lane-per-row) path
bool onerow_only(int c) {
    return c == KQ_Q5_K || c == KQ_Q8_0 || c == KQ_IQ3_XXS || c == KQ_IQ4_XS || c == KQ_Q4_0 || c == KQ_IQ4_NL ||
           c == KQ_Q2_K || c == KQ_Q3_K || c == KQ_Q4_1 || c == KQ_Q5_0 || c == KQ_Q5_1 || c == KQ_TQ2_0 || c == KQ_MXFP4 ||
           c == KQ_IQ2_XS || c == KQ_IQ2_S || c == KQ_IQ3_S || c == KQ_IQ1_S || c == KQ_IQ1_M ||
           c == KQ_TQ1_0 || c == KQ_NVFP4;
}
bool act_dtype_ok(int d) { return d == KQ_F16 || d == KQ_BF16; }
bool out_dtype_ok(int d) { return d == KQ_F32 || d == KQ_F16 || d == KQ_BF16; }
size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

// ragged: K may end in a partial 256-weight group (a whole number of the
// codec's 32- or 64-weight blocks); only the entry points that handle it pass true
int check_weights(int codec, const void *w, int64_t k, int64_t row_stride, const char *what, bool ragged = false) {
    if (!codec_ok(codec)) return fail(KQ_ERR_CODEC, "%s: unsupported codec %d (have q8_0=8, q4_k=12, q5_k=13, q6_k=14, iq2_xxs=16, iq3_xxs=18, iq4_xs=23, q4_0=2, iq4_nl=20, q2_k=10, q3_k=11, q4_1=3, q5_0=6, q5_1=7, tq2_0=35, mxfp4=39, iq2_xs=17, iq2_s=22, iq3_s=21, iq1_s=19, iq1_m=29, tq1_0=34, nvfp4=40)", what, codec);
    const int gran = ragged ? sub_block_weights(codec) : QK;
    if (k <= 0 || k % gran) return fail(KQ_ERR_SHAPE, "%s: K=%lld is not a positive multiple of %d", what, (long long)k, gran);
    const int64_t rb = wire_row_bytes(codec, k);
    if (row_stride < rb) return fail(KQ_ERR_SHAPE, "%s: row stride %lld < row bytes %lld", what, (long long)row_stride, (long long)rb);
    const int64_t need = (codec == KQ_Q4_K || codec == KQ_Q5_K) ? 16 : codec == KQ_IQ4_XS ? 8 : codec == KQ_Q2_K ? 4 : 2;
    if (((uintptr_t)w | (uintptr_t)row_stride) % need)
        return fail(KQ_ERR_ALIGN, "%s: weight base/row stride must be %lld-byte aligned for codec %d", what, (long long)need, codec);
    return KQ_OK;
}

int check_x(const void *x, int dtype, int64_t row_stride, const char *what) {
    if (!act_dtype_ok(dtype)) return fail(KQ_ERR_DTYPE, "%s: activations must be f16 or bf16 (got dtype %d)", what, dtype);
    if ((uintptr_t)x % 16 || row_stride % 8)
        return fail(KQ_ERR_ALIGN, "%s: activation base must be 16-byte aligned and row stride a multiple of 8", what);
    return KQ_OK;
}

// Workspace layout: [0,256) header (err int, n_groups int); [256, 256+CNT)
// the stream-K tile counters -- a fixed region that only the GEMV touches and
// always leaves zero, so every call can rely on it whatever ran before; then
// the group tables, the per-slot f32 outputs / GEMM scratch, the partials.
constexpr size_t CNT_RESERVE = 1024 * 1024;  // 262144 (group, tile) counters
struct WsPlan {
    size_t cnt_off = 256, groups_off = 256 + CNT_RESERVE, ys_off = 0, part_off = 0, total = 256;
    int max_groups = 0;
};

int moe_max_groups(int64_t slots, int64_t e, int gsize) {
    return (int)(slots / gsize + (slots < e ? slots : e) + 1);
}

WsPlan plan(size_t group_ints, size_t ys_bytes, size_t cnt_bytes, size_t part_bytes) {
    WsPlan p;
    (void)cnt_bytes;  // checked against CNT_RESERVE by the callers
    p.ys_off = align256(p.groups_off + group_ints * sizeof(int));
    p.part_off = align256(p.ys_off + ys_bytes);
    p.total = align256(p.part_off + part_bytes);
    return p;
}

GemvArgs dense_args(int codec, const void *x, int x_dtype, int64_t m, int64_t k, int64_t xs, const void *w,
                    const void *w2, int64_t n, int64_t ws_, void *y, int y_dtype, int64_t ys, int act) {
    GemvArgs a{};
    a.codec = codec;
    a.w = (const uint8_t *)w;
    a.w_row_stride = ws_;
    a.w2 = (const uint8_t *)w2;
    a.w2_row_stride = ws_;
    a.N = (int)n;
    a.K = (int)k;
    a.x = x;
    a.x_dtype = x_dtype;
    a.x_row_stride = xs;
    a.dense_m = (int)m;
    a.max_groups = (int)((m + 31) / 32);
    a.y = y;
    a.y_dtype = y_dtype;
    a.y_row_stride = ys;
    a.act = act;
    a.max_tokens = (int)(m < 32 ? m : 32);
#ifdef KQ_DEVELOPMENT
    // development builds only: skip parts of the GEMV / write per-CTA timestamps
    // into a second output row (the caller must provide it)
    const char *dbg = getenv("KQ_GEMV_DEBUG");
    a.debug = dbg ? atoi(dbg) : 0;
#endif
    return a;
}

int gemm_min_m() {
    static int v = -1;
    if (v < 0) {
        const char *e = dev_env("KQ_GEMM_MIN_M");  // development override of the GEMV/GEMM crossover
        v = e ? atoi(e) : GEMM_MIN_M;
    }
    return v;
}

// Q5_K, Q8_0, IQ3_XXS, IQ4_XS, Q2_K, Q3_K and the legacy 32-weight codecs have a one-row GEMV only: every other batch
// goes to the tcgen05 GEMM
bool use_gemm(int64_t m, int codec = 0) {
    return m >= gemm_min_m() || (onerow_only(codec) && m >= 2);
}

// workspace bytes of the path run_dense takes for these activations (the
// GEMM when the batch is prefill-sized and the GEMM takes this layout)
size_t dense_ws_x(int codec, int64_t m, int64_t n, int64_t k, int act, int x_dtype, int64_t xs) {
    if ((use_gemm(m, codec) || k % QK) && gemm_supported(codec, m, n, k, x_dtype, xs))
        return plan(0, gemm_scratch_bytes(codec, m, n, k, act != ACT_NONE), 0, 0).total;
    GemvArgs a = dense_args(codec, nullptr, x_dtype, m, k, xs, nullptr, nullptr, n, 0, nullptr, KQ_BF16, n, act);
    size_t pb, cb;
    gemv_scratch_need(a, &pb, &cb);
    return plan(0, 0, cb, pb).total;
}

size_t dense_ws(int codec, int64_t m, int64_t n, int64_t k, int act) {
    return dense_ws_x(codec, m, n, k, act, KQ_BF16, k);
}

int run_dense(int codec, const void *x, int x_dtype, int64_t m, int64_t k, int64_t xs, const void *w, const void *w2,
              int64_t n, int64_t wstride, int act, void *y, int y_dtype, int64_t ys, void *ws, size_t ws_bytes,
              void *stream, const char *what, const void *bias = nullptr, int bias_dtype = 0) {
    if (bias && (w2 || !out_dtype_ok(bias_dtype))) return fail(KQ_ERR_DTYPE, "%s: bad bias", what);
    int rc;
    if ((rc = check_weights(codec, w, k, wstride, what, true))) return rc;
    if (w2 && (rc = check_weights(codec, w2, k, wstride, what, true))) return rc;
    if ((rc = check_x(x, x_dtype, xs, what))) return rc;
    // K ending in a partial 256-weight group (32/64-weight codecs): every batch
    // size runs on the GEMM over a dequantized copy, which takes K % 64 == 0
    const bool ragged = k % QK != 0;
    if (ragged && !gemm_supported(codec, m > 0 ? m : 1, n, k, x_dtype, xs))
        return fail(KQ_ERR_SHAPE, "%s: K=%lld is not a multiple of 256; a partial last group needs K %% 64 == 0", what,
                    (long long)k);
    if (!out_dtype_ok(y_dtype)) return fail(KQ_ERR_DTYPE, "%s: bad output dtype %d", what, y_dtype);
    if (m < 0 || n <= 0 || xs < k || ys < n) return fail(KQ_ERR_SHAPE, "%s: bad sizes m=%lld n=%lld", what, (long long)m, (long long)n);
    if (m == 0) return KQ_OK;
    if (n > 0x7fffffff || k > 0x7fffffff) return fail(KQ_ERR_SHAPE, "%s: n/k too large", what);
    if ((use_gemm(m, codec) || ragged) && gemm_supported(codec, m, n, k, x_dtype, xs)) {
        const WsPlan p = plan(0, gemm_scratch_bytes(codec, m, n, k, act != ACT_NONE), 0, 0);
        if (!ws || ws_bytes < p.total || ((uintptr_t)ws & 255))
            return fail(KQ_ERR_WORKSPACE, "%s: workspace of %zu bytes (256-aligned) required, got %zu", what, p.total, ws_bytes);
        GemmArgs g{};
        g.codec = codec;
        g.M = (int)m;
        g.N = (int)n;
        g.K = (int)k;
        g.x = x;
        g.x_dtype = x_dtype;
        g.x_row_stride = xs;
        g.w = (const uint8_t *)w;
        g.w_row_stride = wstride;
        g.w2 = (const uint8_t *)w2;
        g.act = w2 ? act : ACT_NONE;
        g.y = y;
        g.y_dtype = y_dtype;
        g.y_row_stride = ys;
        g.err = (int *)ws;
#ifdef KQ_DEVELOPMENT
        if (const char *gd = getenv("KQ_GEMM_DEBUG")) g.debug = atoi(gd);
#endif
        cudaError_t ce = launch_gemm(g, (char *)ws + p.ys_off, (cudaStream_t)stream);
        if (ce == cudaSuccess && bias)
            ce = launch_add_bias(y, y_dtype, ys, m, n, bias, bias_dtype, (cudaStream_t)stream);
        return cuda_status(ce, what);
    }
    GemvArgs a = dense_args(codec, x, x_dtype, m, k, xs, w, w2, n, wstride, y, y_dtype, ys, act);
    size_t pb, cb;
    gemv_scratch_need(a, &pb, &cb);
    const WsPlan p = plan(0, 0, cb, pb);
    if (cb > CNT_RESERVE) return fail(KQ_ERR_SHAPE, "%s: too many output tiles (%zu counter bytes)", what, cb);
    if (!ws || ws_bytes < p.total || ((uintptr_t)ws & 255))
        return fail(KQ_ERR_WORKSPACE, "%s: workspace of %zu bytes (256-aligned) required, got %zu", what, p.total, ws_bytes);
    a.err = (int *)ws;
    a.counters = (int *)((char *)ws + p.cnt_off);
    a.partial = (float *)((char *)ws + p.part_off);
    a.bias = bias;
    a.bias_dtype = bias_dtype;
    return cuda_status(launch_gemv(a, (cudaStream_t)stream), what);
}

// Grouped tensor-core path for routed calls with many rows per expert (MoE
// prefill): sort the slots by local expert, gather their activation rows
// contiguously, run one tcgen05 GEMM over a device table of (expert, 128-row
// tile) -- every expert's weights stream once per 256 output columns instead of
// once per 8 rows -- and scatter the outputs back to slot order.
constexpr size_t GROUPED_B_CHUNK = (size_t)1 << 30;  // dequantized-expert scratch per launch (non-Q4_K codecs)

bool use_grouped(int codec, int64_t slots, int64_t etotal, int64_t n, int64_t kin, int act, bool glu, int x_dtype,
                 int64_t xs) {
    if (act != ACT_NONE && !glu) return false;
    if (n % 4 || n > 0x7fffffff || kin > 0x7fffffff) return false;
    if (slots < (int64_t)GEMM_MIN_M * etotal) return false;  // fewer than ~33 rows per expert: GEMV
    return gemm_supported(codec, slots, n, kin, x_dtype, xs);
}

struct GroupedPlan {
    size_t perm_off, scr_off, misc_off, tiles_off, mix_off, xs_off, g_off, b_off, total;
    int max_tiles, chunk_e, mt;
};

GroupedPlan grouped_plan(int codec, int64_t slots, int64_t e, int64_t etotal, int64_t n, int64_t kin, bool glu,
                         bool f32_out) {
    GroupedPlan g;
    // 256-row tiles (two accumulators per CTA) once experts average >= 192 rows
    g.mt = slots >= 192 * etotal ? 2 : 1;
    if (const char *e = dev_env("KQ_GROUPED_MT")) g.mt = atoi(e) == 2 ? 2 : 1;  // development override
    g.max_tiles = (int)(slots / (128 * g.mt) + (slots < e ? slots : e) + 1);
    const size_t per_e = (size_t)n * kin * 2 * (glu ? 2 : 1);
    g.chunk_e = codec == KQ_Q4_K ? (int)e : (int)std::max<int64_t>(1, std::min<int64_t>(e, GROUPED_B_CHUNK / per_e));
    size_t o = 256 + CNT_RESERVE;
    g.perm_off = o;
    o = align256(o + (size_t)slots * sizeof(int));
    g.scr_off = o;
    o = align256(o + (size_t)(slots + e) * sizeof(int));
    g.misc_off = o;
    o = align256(o + 2 * sizeof(int));
    g.tiles_off = o;
    o = align256(o + (size_t)g.max_tiles * 3 * sizeof(int));
    g.mix_off = o;  // fused score mix: token and score of each sorted row
    if (f32_out) o = align256(o + (size_t)slots * 2 * sizeof(int));
    g.xs_off = o;
    o = align256(o + (size_t)slots * kin * 2);
    g.g_off = o;
    if (f32_out) o = align256(o + (size_t)slots * n * sizeof(float));
    g.b_off = o;
    if (codec != KQ_Q4_K) o = align256(o + (size_t)g.chunk_e * per_e);
    g.total = o;
    return g;
}

int run_grouped(int codec, const void *x, int x_dtype, int64_t xs, int64_t kin, int64_t slots, int kslot,
                int64_t tokens, const int32_t *idx, const int32_t *xidx, int mode, const void *w, const void *w2,
                int64_t e, int64_t n, int64_t wrs, int64_t wes, int act, void *y, int y_dtype, int64_t yrs,
                const float *scores, void *ws, size_t ws_bytes, void *stream, const char *what, int64_t ebase,
                int64_t etotal) {
    const bool glu = w2 != nullptr;
    const GroupedPlan p = grouped_plan(codec, slots, e, etotal, n, kin, glu, scores != nullptr);
    if (!ws || ws_bytes < p.total || ((uintptr_t)ws & 255))
        return fail(KQ_ERR_WORKSPACE, "%s: workspace of %zu bytes (256-aligned) required, got %zu", what, p.total, ws_bytes);
    char *base = (char *)ws;
    int *err = (int *)base;
    int *cnt = (int *)(base + 256);  // zero on entry, left zero (counter region)
    int *perm = (int *)(base + p.perm_off), *scr = (int *)(base + p.scr_off);
    int *count = (int *)(base + p.misc_off), *ntiles = count + 1;
    int *te = (int *)(base + p.tiles_off), *tr0 = te + p.max_tiles, *tre = tr0 + p.max_tiles;
    void *xsorted = base + p.xs_off;
    cudaStream_t st = (cudaStream_t)stream;
    // score mix fused into the GEMM epilogue (atomic f32 adds into y) when y is
    // a contiguous f32 [tokens, n]; otherwise per-slot rows and the mix kernel
    const bool fused_mix = scores && y_dtype == KQ_F32 && yrs == n;
    int *tok_of = (int *)(base + p.mix_off);
    float *scale_of = (float *)(tok_of + slots);
    cudaError_t ce = launch_moe_sort(idx, (int)slots, kslot, (int)ebase, (int)e, (int)etotal, mode == 1, xidx, x, xs,
                                     (int)kin, xsorted, 128 * p.mt, cnt, scr, perm, count, ntiles, te, tr0, tre,
                                     p.max_tiles, err, fused_mix ? scores : nullptr, tok_of, scale_of, st);
    if (ce != cudaSuccess) return cuda_status(ce, what);
    GemmArgs g{};
    g.codec = codec;
    g.M = (int)slots;
    g.N = (int)n;
    g.K = (int)kin;
    g.x = xsorted;
    g.x_dtype = x_dtype;
    g.x_row_stride = kin;
    g.w_row_stride = wrs;
    g.w_expert_stride = wes;
    g.n_per_expert = (int)n;
    g.err = err;
    g.n_tiles = ntiles;
    g.tile_e = te;
    g.tile_row0 = tr0;
    g.tile_rowend = tre;
    g.out_row = perm;
    g.act = glu ? act : ACT_NONE;
    g.y = scores ? (void *)(base + p.g_off) : y;
    g.y_dtype = scores ? KQ_F32 : y_dtype;
    g.y_row_stride = scores ? n : yrs;
    if (fused_mix) {
        if ((ce = cudaMemsetAsync(y, 0, (size_t)tokens * n * sizeof(float), st)) != cudaSuccess)
            return cuda_status(ce, what);
        g.y = y;
        g.out_row = tok_of;
        g.row_scale = scale_of;
    }
    for (int64_t c0 = 0; c0 < e; c0 += p.chunk_e) {
        const int64_t c1 = std::min<int64_t>(e, c0 + p.chunk_e);
        g.ex_lo = (int)c0;
        g.ex_hi = (int)c1;
        void *bd = nullptr;
        if (codec == KQ_Q4_K) {
            g.w = (const uint8_t *)w;
            g.w2 = (const uint8_t *)w2;
        } else {
            bd = base + p.b_off;
            for (int half = 0; half < (glu ? 2 : 1); half++) {
                const uint8_t *wp = (const uint8_t *)(half ? w2 : w);
                char *dst = (char *)bd + (size_t)half * (c1 - c0) * n * kin * 2;
                if (wes == n * wrs) {  // contiguous expert stack: one launch for the chunk
                    ce = launch_dequantize(codec, wp + c0 * wes, (c1 - c0) * n, kin, wrs, dst, x_dtype, st);
                } else {
                    for (int64_t ex = c0; ex < c1 && ce == cudaSuccess; ex++)
                        ce = launch_dequantize(codec, wp + ex * wes, n, kin, wrs, dst + (ex - c0) * n * kin * 2, x_dtype,
                                               st);
                }
                if (ce != cudaSuccess) return cuda_status(ce, what);
            }
        }
        if ((ce = launch_gemm_grouped(g, p.mt, p.max_tiles, bd, st)) != cudaSuccess) return cuda_status(ce, what);
    }
    if (scores && !fused_mix)
        ce = launch_moe_mix((const float *)(base + p.g_off), scores, idx, (int)ebase, (int)e, (int)tokens, kslot, (int)n,
                            y, y_dtype, st);
    return cuda_status(ce, what);
}

// Whole expert layer on the grouped path: one sort of the routed slots, the
// gate/up GEMM writes h in expert-sorted row order, and the down GEMM reads it
// in place with the same tile table (no second sort, gather or h scatter);
// the score mix is fused into the down epilogue when y is a contiguous f32.
struct LayerPlan {
    size_t perm_off, scr_off, misc_off, tiles_off, mix_off, xs_off, hs_off, ys_off, b_off, total;
    int max_tiles, mt, chunk_gu, chunk_d;
};

LayerPlan layer_plan(int cgu, int cd, int64_t slots, int64_t e, int64_t etotal, int64_t d, int64_t f, bool need_ys) {
    LayerPlan g;
    g.mt = slots >= 192 * etotal ? 2 : 1;
    g.max_tiles = (int)(slots / (128 * g.mt) + (slots < e ? slots : e) + 1);
    const size_t per_gu = (size_t)f * d * 2 * 2, per_d = (size_t)d * f * 2;
    g.chunk_gu = cgu == KQ_Q4_K ? (int)e : (int)std::max<int64_t>(1, std::min<int64_t>(e, GROUPED_B_CHUNK / per_gu));
    g.chunk_d = cd == KQ_Q4_K ? (int)e : (int)std::max<int64_t>(1, std::min<int64_t>(e, GROUPED_B_CHUNK / per_d));
    size_t o = 256 + CNT_RESERVE;
    g.perm_off = o;
    o = align256(o + (size_t)slots * sizeof(int));
    g.scr_off = o;
    o = align256(o + (size_t)(slots + e) * sizeof(int));
    g.misc_off = o;
    o = align256(o + 2 * sizeof(int));
    g.tiles_off = o;
    o = align256(o + (size_t)g.max_tiles * 3 * sizeof(int));
    g.mix_off = o;
    o = align256(o + (size_t)slots * 2 * sizeof(int));
    g.xs_off = o;
    o = align256(o + (size_t)slots * d * 2);
    g.hs_off = o;
    o = align256(o + (size_t)slots * f * 2);
    g.ys_off = o;
    if (need_ys) o = align256(o + (size_t)slots * d * sizeof(float));
    g.b_off = o;
    const size_t bgu = cgu == KQ_Q4_K ? 0 : (size_t)g.chunk_gu * per_gu;
    const size_t bd = cd == KQ_Q4_K ? 0 : (size_t)g.chunk_d * per_d;
    g.total = align256(o + std::max(bgu, bd));
    return g;
}

// grouped GEMM over [c0, c1) expert chunks of one stack (dequantizing non-Q4_K chunks first)
int grouped_pass(GemmArgs g, int codec, const uint8_t *w, const uint8_t *w2, int64_t e, int chunk, int64_t n,
                 int64_t kin, int64_t wrs, int64_t wes, int x_dtype, char *bscratch, int mt, int max_tiles,
                 cudaStream_t st, const char *what) {
    const bool glu = w2 != nullptr;
    for (int64_t c0 = 0; c0 < e; c0 += chunk) {
        const int64_t c1 = std::min<int64_t>(e, c0 + chunk);
        g.ex_lo = (int)c0;
        g.ex_hi = (int)c1;
        void *bd = nullptr;
        cudaError_t ce = cudaSuccess;
        if (codec == KQ_Q4_K) {
            g.w = w;
            g.w2 = w2;
        } else {
            bd = bscratch;
            for (int half = 0; half < (glu ? 2 : 1) && ce == cudaSuccess; half++) {
                const uint8_t *wp = half ? w2 : w;
                char *dst = bscratch + (size_t)half * (c1 - c0) * n * kin * 2;
                if (wes == n * wrs) {
                    ce = launch_dequantize(codec, wp + c0 * wes, (c1 - c0) * n, kin, wrs, dst, x_dtype, st);
                } else {
                    for (int64_t ex = c0; ex < c1 && ce == cudaSuccess; ex++)
                        ce = launch_dequantize(codec, wp + ex * wes, n, kin, wrs, dst + (ex - c0) * n * kin * 2, x_dtype,
                                               st);
                }
            }
            if (ce != cudaSuccess) return cuda_status(ce, what);
        }
        if ((ce = launch_gemm_grouped(g, mt, max_tiles, bd, st)) != cudaSuccess) return cuda_status(ce, what);
    }
    return KQ_OK;
}

int run_grouped_layer(int cgu, int cd, const void *x, int x_dtype, int64_t t, int64_t d, const int32_t *idx, int k,
                      const float *scores, const void *gate_w, const void *up_w, int64_t gu_rs, int64_t gu_es,
                      const void *down_w, int64_t d_rs, int64_t d_es, int64_t e, int64_t f, int64_t ebase,
                      int64_t etotal, int act, void *y, int y_dtype, void *ws, size_t ws_bytes, void *stream) {
    const char *what = "moe_expert_layer_local";
    const int64_t slots = t * k;
    const bool fused_mix = y_dtype == KQ_F32;
    const LayerPlan p = layer_plan(cgu, cd, slots, e, etotal, d, f, !fused_mix);
    if (ws_bytes < p.total) return fail(KQ_ERR_WORKSPACE, "%s: workspace of %zu bytes required, got %zu", what, p.total, ws_bytes);
    char *base = (char *)ws;
    int *err = (int *)base, *cnt = (int *)(base + 256);
    int *perm = (int *)(base + p.perm_off), *scr = (int *)(base + p.scr_off);
    int *count = (int *)(base + p.misc_off), *ntiles = count + 1;
    int *te = (int *)(base + p.tiles_off), *tr0 = te + p.max_tiles, *tre = tr0 + p.max_tiles;
    int *tok_of = (int *)(base + p.mix_off);
    float *scale_of = (float *)(tok_of + slots);
    cudaStream_t st = (cudaStream_t)stream;
    cudaError_t ce = launch_moe_sort(idx, (int)slots, k, (int)ebase, (int)e, (int)etotal, 0, nullptr, x, d, (int)d,
                                     base + p.xs_off, 128 * p.mt, cnt, scr, perm, count, ntiles, te, tr0, tre,
                                     p.max_tiles, err, fused_mix ? scores : nullptr, tok_of, scale_of, st);
    if (ce != cudaSuccess) return cuda_status(ce, what);
    GemmArgs g{};
    g.M = (int)slots;
    g.x_dtype = x_dtype;
    g.err = err;
    g.n_tiles = ntiles;
    g.tile_e = te;
    g.tile_row0 = tr0;
    g.tile_rowend = tre;
    // gate/up: sorted x -> sorted h (row p of h is sorted row p)
    g.codec = cgu;
    g.N = (int)f;
    g.K = (int)d;
    g.x = base + p.xs_off;
    g.x_row_stride = d;
    g.w_row_stride = gu_rs;
    g.w_expert_stride = gu_es;
    g.n_per_expert = (int)f;
    g.act = act;
    g.y = base + p.hs_off;
    g.y_dtype = x_dtype;
    g.y_row_stride = f;
    int rc = grouped_pass(g, cgu, (const uint8_t *)gate_w, (const uint8_t *)up_w, e, p.chunk_gu, f, d, gu_rs, gu_es,
                          x_dtype, base + p.b_off, p.mt, p.max_tiles, st, what);
    if (rc) return rc;
    // down: sorted h -> token rows (fused score mix) or per-slot f32 rows + mix kernel
    g.codec = cd;
    g.N = (int)d;
    g.K = (int)f;
    g.x = base + p.hs_off;
    g.x_row_stride = f;
    g.w_row_stride = d_rs;
    g.w_expert_stride = d_es;
    g.n_per_expert = (int)d;
    g.act = ACT_NONE;
    g.w2 = nullptr;
    if (fused_mix) {
        if ((ce = cudaMemsetAsync(y, 0, (size_t)t * d * sizeof(float), st)) != cudaSuccess) return cuda_status(ce, what);
        g.y = y;
        g.y_dtype = KQ_F32;
        g.y_row_stride = d;
        g.out_row = tok_of;
        g.row_scale = scale_of;
    } else {
        g.y = base + p.ys_off;
        g.y_dtype = KQ_F32;
        g.y_row_stride = d;
        g.out_row = perm;
    }
    rc = grouped_pass(g, cd, (const uint8_t *)down_w, nullptr, e, p.chunk_d, d, f, d_rs, d_es, x_dtype, base + p.b_off,
                      p.mt, p.max_tiles, st, what);
    if (rc) return rc;
    if (!fused_mix)
        return cuda_status(launch_moe_mix((const float *)(base + p.ys_off), scores, idx, (int)ebase, (int)e, (int)t, k,
                                          (int)d, y, y_dtype, st),
                           what);
    return KQ_OK;
}

// Routed (MoE) GEMV over expert stacks.  mode: 0 glu (x row = slot/k),
// 1 per-slot rows (x row = slot), 2 explicit x_index.
// Slots per group of the routed GEMV.  per_expert bounds the slots one expert
// can receive (distinct experts per token).  IQ2_XXS decode is ALU-bound: with
// up to two routed slots per expert on average, groups of <= 4 slots take the
// lane-per-row path with every slot's row staged (each weight decoded once for
// the group; a one-slot group is the one-row dot).
int routed_gsize(int codec, int64_t slots, int64_t per_expert, int64_t etotal) {
    if (onerow_only(codec)) return 1;  // one-row-only codecs: the one-row path is their only GEMV
    if (codec == KQ_IQ2_XXS && slots <= 2 * etotal) return (int)(per_expert < 4 ? per_expert : 4);
    return (int)(per_expert < 8 ? per_expert : 8);
}

int run_routed(int codec, const void *x, int x_dtype, int64_t xs, int64_t kin, int64_t slots, int kslot,
               int64_t tokens, const int32_t *idx, const int32_t *xidx, int mode, const void *w, const void *w2,
               int64_t e, int64_t n, int64_t wrs, int64_t wes, int act, void *y, int y_dtype, int64_t yrs,
               const float *scores, void *ws, size_t ws_bytes, void *stream, const char *what, int64_t ebase = 0,
               int64_t etotal = -1, bool reuse_groups = false) {
    if (etotal < 0) etotal = e;
    int rc;
    if ((rc = check_weights(codec, w, kin, wrs, what))) return rc;
    if (w2 && (rc = check_weights(codec, w2, kin, wrs, what))) return rc;
    if ((rc = check_x(x, x_dtype, xs, what))) return rc;
    if (!out_dtype_ok(y_dtype)) return fail(KQ_ERR_DTYPE, "%s: bad output dtype %d", what, y_dtype);
    if (e <= 0 || e > 1024) return fail(KQ_ERR_SHAPE, "%s: expert count %lld outside 1..1024", what, (long long)e);
    if (wes < n * wrs) return fail(KQ_ERR_SHAPE, "%s: expert stride smaller than one expert", what);
    if (slots == 0) return KQ_OK;
    if (slots < 0 || slots > (1 << 20)) return fail(KQ_ERR_SHAPE, "%s: slot count %lld out of range", what, (long long)slots);
    if (use_grouped(codec, slots, etotal, n, kin, act, w2 != nullptr, x_dtype, xs))
        return run_grouped(codec, x, x_dtype, xs, kin, slots, kslot, tokens, idx, xidx, mode, w, w2, e, n, wrs, wes, act,
                           y, y_dtype, yrs, scores, ws, ws_bytes, stream, what, ebase, etotal);
    // groups of <= 8 slots: one MMA n-tile; an expert with more routed rows
    // streams its weights once per 8 rows (decode routes few rows per expert)
    const int gsize = routed_gsize(codec, slots, mode == 2 ? slots : tokens, etotal);
    const int maxg = moe_max_groups(slots, e, gsize);
    GemvArgs a{};
    a.codec = codec;
    a.w = (const uint8_t *)w;
    a.w_row_stride = wrs;
    a.w_expert_stride = wes;
    a.w2 = (const uint8_t *)w2;
    a.w2_row_stride = wrs;
    a.w2_expert_stride = wes;
    a.N = (int)n;
    a.K = (int)kin;
    a.x = x;
    a.x_dtype = x_dtype;
    a.x_row_stride = xs;
    a.dense_m = 0;
    a.max_groups = maxg;
    a.act = act;
    a.max_tokens = gsize;
    size_t pb, cb;
    gemv_scratch_need(a, &pb, &cb);
    const size_t ys_bytes = scores ? (size_t)slots * n * sizeof(float) : 0;
    const WsPlan p = plan((size_t)maxg * 66, ys_bytes, cb, pb);
    if (cb > CNT_RESERVE) return fail(KQ_ERR_SHAPE, "%s: too many output tiles (%zu counter bytes)", what, cb);
    if (!ws || ws_bytes < p.total || ((uintptr_t)ws & 255))
        return fail(KQ_ERR_WORKSPACE, "%s: workspace of %zu bytes (256-aligned) required, got %zu", what, p.total, ws_bytes);
    char *base = (char *)ws;
    int *err = (int *)base, *ng = (int *)(base + 4);
    int *gexp = (int *)(base + p.groups_off), *gcnt = gexp + maxg, *gx = gcnt + maxg, *go = gx + (size_t)maxg * 32;
    cudaStream_t st = (cudaStream_t)stream;
    cudaError_t ce = cudaSuccess;
    // reuse_groups (down projection of an expert layer, mode 1): the gate/up
    // call on this workspace grouped the same slots with the same group size,
    // and a slot's activation row here is the slot itself, its output row
    if (!reuse_groups)
        ce = launch_moe_groups(idx, (int)slots, kslot, (int)ebase, (int)e, (int)etotal, mode == 1, xidx, gsize, ng, gexp,
                               gcnt, gx, go, maxg, err, st);
    if (ce != cudaSuccess) return cuda_status(ce, what);
    a.n_groups = ng;
    a.grp_expert = gexp;
    a.grp_count = gcnt;
    a.grp_xrow = reuse_groups ? go : gx;
    a.grp_orow = go;
    a.err = err;
    a.counters = (int *)(base + p.cnt_off);
    a.partial = (float *)(base + p.part_off);
    if (scores) {
        a.y = base + p.ys_off;
        a.y_dtype = KQ_F32;
        a.y_row_stride = n;
    } else {
        a.y = y;
        a.y_dtype = y_dtype;
        a.y_row_stride = yrs;
    }
    if ((ce = launch_gemv(a, st)) != cudaSuccess) return cuda_status(ce, what);
    if (scores)
        if ((ce = launch_moe_mix((const float *)(base + p.ys_off), scores, idx, (int)ebase, (int)e, (int)tokens, kslot,
                                 (int)n, y, y_dtype, st)) !=
            cudaSuccess)
            return cuda_status(ce, what);
    return KQ_OK;
}

size_t routed_ws(int codec, int64_t slots, int64_t per_expert, int64_t e, int64_t n, int64_t kin, int act,
                 bool mix) {
    // IQ2_XXS may run with one-slot groups (see run_routed): size for those too
    const int gsize = (codec == KQ_IQ2_XXS || onerow_only(codec)) ? 1
                                                                 : (int)(per_expert < 8 ? (per_expert > 0 ? per_expert : 1) : 8);
    const int maxg = moe_max_groups(slots, e, gsize);
    GemvArgs a{};
    a.codec = codec;
    a.N = (int)n;
    a.K = (int)kin;
    a.max_groups = maxg;
    a.act = act;
    a.max_tokens = gsize;
    size_t pb, cb;
    gemv_scratch_need(a, &pb, &cb);
    size_t t = plan((size_t)maxg * 66, mix ? (size_t)slots * n * sizeof(float) : 0, cb, pb).total;
    // the grouped GEMM path may be taken once slots >= GEMM_MIN_M * total experts >= GEMM_MIN_M * e
    if (slots >= (int64_t)GEMM_MIN_M * e && n % 4 == 0 && kin % 64 == 0) {
        const size_t gt = std::max(grouped_plan(codec, slots, e, e, n, kin, act != ACT_NONE, mix).total,
                                   grouped_plan(codec, slots, e, slots, n, kin, act != ACT_NONE, mix).total);
        t = gt > t ? gt : t;
    }
    return t;
}

}  // namespace

namespace kq {
size_t dense_matmul_workspace_bytes(int codec, int64_t m, int64_t n, int64_t k, int x_dtype, int64_t x_row_stride) {
    return dense_ws_x(codec, m, n, k, ACT_NONE, x_dtype, x_row_stride);
}
}  // namespace kq

void kq::set_last_error(const char *msg) { snprintf(g_msg, sizeof(g_msg), "%s", msg); }

extern "C" {

int kq_version(void) { return 100; }

const char *kq_last_error(void) { return g_msg; }

int kq_codecs(int *out, int cap) {
    static const int ids[23] = {KQ_Q4_K, KQ_Q5_K, KQ_Q6_K, KQ_IQ2_XXS, KQ_Q8_0, KQ_IQ3_XXS, KQ_IQ4_XS, KQ_Q4_0,
                                KQ_IQ4_NL, KQ_Q2_K, KQ_Q3_K, KQ_Q4_1, KQ_Q5_0, KQ_Q5_1, KQ_TQ2_0, KQ_MXFP4,
                                KQ_IQ2_XS, KQ_IQ2_S, KQ_IQ3_S, KQ_IQ1_S, KQ_IQ1_M, KQ_TQ1_0, KQ_NVFP4};
    for (int i = 0; out && i < 23 && i < cap; i++) out[i] = ids[i];
    return 23;
}

int kq_codec_has_matmul(int codec) { return codec_ok(codec) ? 1 : 0; }

int kq_block_bytes(int codec) { return codec_ok(codec) ? block_bytes(codec) : -1; }

int kq_dequantize(int codec, const void *w, int64_t rows, int64_t k, int64_t w_row_stride, void *out, int out_dtype,
                  void *stream) {
    g_msg[0] = 0;
    if (!codec_ok(codec)) return fail(KQ_ERR_CODEC, "dequantize: unsupported codec %d", codec);
    if (k <= 0 || k % sub_block_weights(codec))
        return fail(KQ_ERR_SHAPE, "dequantize: K=%lld is not a positive multiple of %d", (long long)k,
                    sub_block_weights(codec));
    if (rows < 0) return fail(KQ_ERR_SHAPE, "dequantize: rows < 0");
    if (!out_dtype_ok(out_dtype)) return fail(KQ_ERR_DTYPE, "dequantize: bad output dtype %d", out_dtype);
    if ((uintptr_t)out % 16) return fail(KQ_ERR_ALIGN, "dequantize: output must be 16-byte aligned");
    if (w_row_stride < wire_row_bytes(codec, k)) return fail(KQ_ERR_SHAPE, "dequantize: row stride too small");

    return cuda_status(launch_dequantize(codec, (const uint8_t *)w, rows, k, w_row_stride, out, out_dtype,
                                         (cudaStream_t)stream),
                       "dequantize");
}

size_t kq_quantized_matmul_workspace_size(int codec, int64_t m, int64_t n, int64_t k) {
    if (!codec_ok(codec) || k <= 0 || k % sub_block_weights(codec) || n <= 0 || m <= 0) return 256;
    return dense_ws(codec, m, n, k, ACT_NONE);
}

int kq_quantized_matmul(int codec, const void *x, int x_dtype, int64_t m, int64_t k, int64_t x_row_stride,
                        const void *w, int64_t n, int64_t w_row_stride, void *y, int y_dtype, int64_t y_row_stride,
                        void *workspace, size_t workspace_bytes, void *stream) {
    g_msg[0] = 0;
    return run_dense(codec, x, x_dtype, m, k, x_row_stride, w, nullptr, n, w_row_stride, ACT_NONE, y, y_dtype,
                     y_row_stride, workspace, workspace_bytes, stream, "quantized_matmul");
}

int kq_quantized_matmul_bias(int codec, const void *x, int x_dtype, int64_t m, int64_t k, int64_t x_row_stride,
                             const void *w, int64_t n, int64_t w_row_stride, const void *bias, int bias_dtype, void *y,
                             int y_dtype, int64_t y_row_stride, void *workspace, size_t workspace_bytes, void *stream) {
    g_msg[0] = 0;
    if (!bias) return fail(KQ_ERR_SHAPE, "quantized_matmul_bias: bias required");
    return run_dense(codec, x, x_dtype, m, k, x_row_stride, w, nullptr, n, w_row_stride, ACT_NONE, y, y_dtype,
                     y_row_stride, workspace, workspace_bytes, stream, "quantized_matmul_bias", bias, bias_dtype);
}

size_t kq_allreduce_buffer_bytes(int world, int64_t n) {
    return (world < 1 || n < 1) ? 0 : ar_buffer_bytes(world, n);
}

int kq_quantized_matmul_allreduce(int codec, const void *x, int x_dtype, int64_t k, const void *w, int64_t n,
                                  int64_t w_row_stride, void *y, int y_dtype, int world, int rank,
                                  void *const *comm_bufs, void *workspace, size_t workspace_bytes, void *stream) {
    g_msg[0] = 0;
    const char *what = "quantized_matmul_allreduce";
    int rc;
    if ((rc = check_weights(codec, w, k, w_row_stride, what))) return rc;
    if ((rc = check_x(x, x_dtype, k, what))) return rc;
    if (!out_dtype_ok(y_dtype)) return fail(KQ_ERR_DTYPE, "%s: bad output dtype %d", what, y_dtype);
    if (n <= 0 || n > 0x7fffffff || k > 0x7fffffff) return fail(KQ_ERR_SHAPE, "%s: bad sizes n=%lld", what, (long long)n);
    if (world < 1 || world > 64 || rank < 0 || rank >= world || !comm_bufs)
        return fail(KQ_ERR_SHAPE, "%s: bad world %d / rank %d / buffers", what, world, rank);
    GemvArgs a = dense_args(codec, x, x_dtype, 1, k, k, w, nullptr, n, w_row_stride, y, y_dtype, n, ACT_NONE);
    a.ar_bufs = reinterpret_cast<unsigned char *const *>(comm_bufs);
    a.ar_world = world;
    a.ar_rank = rank;
    size_t pb, cb;
    gemv_scratch_need(a, &pb, &cb);
    const WsPlan p = plan(0, 0, cb, pb);
    if (cb > CNT_RESERVE) return fail(KQ_ERR_SHAPE, "%s: too many output tiles (%zu counter bytes)", what, cb);
    if (!workspace || workspace_bytes < p.total || ((uintptr_t)workspace & 255))
        return fail(KQ_ERR_WORKSPACE, "%s: workspace of %zu bytes (256-aligned) required, got %zu", what, p.total,
                    workspace_bytes);
    a.err = (int *)workspace;
    a.counters = (int *)((char *)workspace + p.cnt_off);
    a.partial = (float *)((char *)workspace + p.part_off);
    return cuda_status(launch_gemv(a, (cudaStream_t)stream), what);
}

int kq_allreduce(const void *x, int x_dtype, void *y, int y_dtype, int64_t n, int64_t buf_n, int world, int rank,
                 void *const *comm_bufs, void *stream) {
    g_msg[0] = 0;
    const char *what = "allreduce";
    if (!x || !y) return fail(KQ_ERR_SHAPE, "%s: null pointer", what);
    if (!out_dtype_ok(x_dtype) || !out_dtype_ok(y_dtype)) return fail(KQ_ERR_DTYPE, "%s: bad dtype", what);
    if (n < 0 || n > buf_n || buf_n > 0x7fffffff)
        return fail(KQ_ERR_SHAPE, "%s: bad size n=%lld (buffers for %lld)", what, (long long)n, (long long)buf_n);
    if (world < 1 || world > AR_MAX_WORLD || rank < 0 || rank >= world || !comm_bufs)
        return fail(KQ_ERR_SHAPE, "%s: bad world %d (1..%d) / rank %d / buffers", what, world, AR_MAX_WORLD, rank);
    if (n == 0) return KQ_OK;
    return cuda_status(launch_allreduce(x, x_dtype, y, y_dtype, n, buf_n, world, rank,
                                        reinterpret_cast<unsigned char *const *>(comm_bufs), (cudaStream_t)stream),
                       what);
}

int kq_comm_error(void *own_buf, int clear, void *stream) {
    g_msg[0] = 0;
    if (!own_buf) return fail(KQ_ERR_SHAPE, "comm_error: null buffer");
    int v = 0;
    cudaStream_t st = (cudaStream_t)stream;
    char *p = (char *)own_buf + AR_ERR;
    cudaError_t e = cudaMemcpyAsync(&v, p, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e == cudaSuccess && clear) e = cudaMemsetAsync(p, 0, sizeof(int), st);
    if (e != cudaSuccess) return -cuda_status(e, "comm_error");
    return v;
}

int kq_comm_alloc(size_t bytes, void **ptr) {
    g_msg[0] = 0;
    if (!ptr || !bytes) return fail(KQ_ERR_SHAPE, "comm_alloc: bad arguments");
    cudaError_t e = cudaMalloc(ptr, bytes);
    if (e == cudaSuccess) e = cudaMemset(*ptr, 0, bytes);
    return cuda_status(e, "comm_alloc");
}

int kq_comm_free(void *ptr) { return cuda_status(cudaFree(ptr), "comm_free"); }

int kq_ipc_handle(const void *ptr, void *handle64) {
    g_msg[0] = 0;
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void *>(ptr));
    if (e == cudaSuccess) memcpy(handle64, &h, sizeof(h));
    return cuda_status(e, "ipc_handle");
}

int kq_ipc_open(const void *handle64, void **ptr) {
    g_msg[0] = 0;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle64, sizeof(h));
    return cuda_status(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), "ipc_open");
}

int kq_ipc_close(void *ptr) { return cuda_status(cudaIpcCloseMemHandle(ptr), "ipc_close"); }

size_t kq_quantized_glu_workspace_size(int codec, int64_t m, int64_t n, int64_t k) {
    if (!codec_ok(codec) || k <= 0 || k % sub_block_weights(codec) || n <= 0 || m <= 0) return 256;
    return dense_ws(codec, m, n, k, ACT_SILU);
}

int kq_quantized_glu(int codec, const void *x, int x_dtype, int64_t m, int64_t k, int64_t x_row_stride,
                     const void *gate_w, const void *up_w, int64_t n, int64_t w_row_stride, int act, void *y,
                     int y_dtype, int64_t y_row_stride, void *workspace, size_t workspace_bytes, void *stream) {
    g_msg[0] = 0;
    if (act < KQ_ACT_SILU || act > KQ_ACT_GELU_TANH) return fail(KQ_ERR_SHAPE, "quantized_glu: bad activation %d", act);
    return run_dense(codec, x, x_dtype, m, k, x_row_stride, gate_w, up_w, n, w_row_stride, act, y, y_dtype,
                     y_row_stride, workspace, workspace_bytes, stream, "quantized_glu");
}

int kq_moe_router_topk(const float *logits, int64_t t, int64_t e, int k, int norm_topk_prob, int32_t *idx,
                       float *scores, void *stream) {
    g_msg[0] = 0;
    if (e <= 0 || e > 1024) return fail(KQ_ERR_SHAPE, "moe_router_topk: expert count %lld outside 1..1024", (long long)e);
    if (k <= 0 || k > 16 || k > e) return fail(KQ_ERR_SHAPE, "moe_router_topk: k=%d outside 1..min(16, E)", k);
    if (t < 0) return fail(KQ_ERR_SHAPE, "moe_router_topk: t < 0");
    return cuda_status(launch_router_topk(logits, (int)t, (int)e, k, norm_topk_prob, idx, scores, 0, nullptr,
                                          (cudaStream_t)stream),
                       "moe_router_topk");
}

int kq_moe_router_topk_ex(const float *logits, int64_t t, int64_t e, int k, int norm_topk_prob, int shared_gate,
                          const float *per_expert_scale, int32_t *idx, float *scores, void *stream) {
    g_msg[0] = 0;
    if (e <= 0 || e > 1024) return fail(KQ_ERR_SHAPE, "moe_router_topk: expert count %lld outside 1..1024", (long long)e);
    if (k <= 0 || k > 16 || k > e) return fail(KQ_ERR_SHAPE, "moe_router_topk: k=%d outside 1..min(16, E)", k);
    if (t < 0) return fail(KQ_ERR_SHAPE, "moe_router_topk: t < 0");
    return cuda_status(launch_router_topk(logits, (int)t, (int)e, k, norm_topk_prob, idx, scores, shared_gate ? 1 : 0,
                                          per_expert_scale, (cudaStream_t)stream),
                       "moe_router_topk");
}

size_t kq_moe_workspace_size(int codec, int64_t slots, int64_t e, int64_t n, int64_t k_in) {
    if (!codec_ok(codec) || k_in <= 0 || k_in % QK || n <= 0 || e <= 0) return 256;
    if (slots <= 0) slots = 1;
    // the largest plan over every group size the calls can pick
    size_t best = 256;
    const int64_t pe[8] = {1, 2, 3, 4, 5, 6, 7, 8};
    for (int i = 0; i < 8; i++)
        for (int act = 0; act < 2; act++) {
            const size_t s = routed_ws(codec, slots, pe[i], e, n, k_in, act ? ACT_SILU : ACT_NONE, true);
            best = s > best ? s : best;
        }
    return best;
}

int kq_moe_glu_gather(int codec, const void *x, int x_dtype, int64_t t, int64_t d, const int32_t *idx, int k,
                      const void *gate_w, const void *up_w, int64_t e, int64_t f, int64_t w_row_stride,
                      int64_t w_expert_stride, int act, void *h, int h_dtype, void *workspace,
                      size_t workspace_bytes, void *stream) {
    g_msg[0] = 0;
    if (act < KQ_ACT_SILU || act > KQ_ACT_GELU_TANH) return fail(KQ_ERR_SHAPE, "moe_glu_gather: bad activation %d", act);
    if (k <= 0) return fail(KQ_ERR_SHAPE, "moe_glu_gather: k <= 0");
    return run_routed(codec, x, x_dtype, d, d, t * k, k, t, idx, nullptr, 0, gate_w, up_w, e, f, w_row_stride,
                      w_expert_stride, act, h, h_dtype, f, nullptr, workspace, workspace_bytes, stream,
                      "moe_glu_gather");
}

int kq_gather_qmv(int codec, const void *h, int h_dtype, int64_t t, int k, int64_t f, const int32_t *idx,
                  const void *w, int64_t e, int64_t n, int64_t w_row_stride, int64_t w_expert_stride, void *y,
                  int y_dtype, void *workspace, size_t workspace_bytes, void *stream) {
    g_msg[0] = 0;
    if (k <= 0) return fail(KQ_ERR_SHAPE, "gather_qmv: k <= 0");
    return run_routed(codec, h, h_dtype, f, f, t * k, k, t, idx, nullptr, 1, w, nullptr, e, n, w_row_stride,
                      w_expert_stride, ACT_NONE, y, y_dtype, n, nullptr, workspace, workspace_bytes, stream,
                      "gather_qmv");
}

int kq_gather_qmv_mix(int codec, const void *h, int h_dtype, int64_t t, int k, int64_t f, const int32_t *idx,
                      const float *scores, const void *w, int64_t e, int64_t n, int64_t w_row_stride,
                      int64_t w_expert_stride, void *y, int y_dtype, void *workspace, size_t workspace_bytes,
                      void *stream) {
    g_msg[0] = 0;
    if (k <= 0) return fail(KQ_ERR_SHAPE, "gather_qmv_mix: k <= 0");
    if (!scores) return fail(KQ_ERR_SHAPE, "gather_qmv_mix: scores required");
    return run_routed(codec, h, h_dtype, f, f, t * k, k, t, idx, nullptr, 1, w, nullptr, e, n, w_row_stride,
                      w_expert_stride, ACT_NONE, y, y_dtype, n, scores, workspace, workspace_bytes, stream,
                      "gather_qmv_mix");
}

int kq_gather_qmm(int codec, const void *x, int x_dtype, int64_t k, int64_t x_row_stride, int64_t rows,
                  const int32_t *x_index, const int32_t *expert_index, const void *w, int64_t e, int64_t n,
                  int64_t w_row_stride, int64_t w_expert_stride, void *y, int y_dtype, void *workspace,
                  size_t workspace_bytes, void *stream) {
    g_msg[0] = 0;
    return run_routed(codec, x, x_dtype, x_row_stride, k, rows, 1, rows, expert_index, x_index, x_index ? 2 : 1, w,
                      nullptr, e, n, w_row_stride, w_expert_stride, ACT_NONE, y, y_dtype, n, nullptr, workspace,
                      workspace_bytes, stream, "gather_qmm");
}

size_t kq_moe_expert_layer_workspace_size(int codec_gu, int codec_d, int64_t t, int k, int64_t e_local, int64_t d,
                                          int64_t f, int h_dtype) {
    if (!codec_ok(codec_gu) || !codec_ok(codec_d) || t <= 0 || k <= 0 || e_local <= 0 || d % QK || f % QK) return 256;
    const int64_t slots = t * k;
    const size_t a = routed_ws(codec_gu, slots, t, e_local, f, d, ACT_SILU, false);
    const size_t b = routed_ws(codec_d, slots, t, e_local, d, f, ACT_NONE, true);
    const size_t esz = h_dtype == KQ_F32 ? 4 : 2;
    size_t need = align256(a > b ? a : b) + align256((size_t)slots * f * esz);
    if (slots >= (int64_t)GEMM_MIN_M * e_local)  // the grouped layer path may be taken (see the entry point)
        for (int mt_total = 0; mt_total < 2; mt_total++) {
            const LayerPlan lp = layer_plan(codec_gu, codec_d, slots, e_local, mt_total ? e_local : slots, d, f, true);
            need = std::max(need, lp.total);
        }
    return need;
}

int kq_moe_expert_layer_local(int codec_gu, int codec_d, const void *x, int x_dtype, int64_t t, int64_t d,
                              const int32_t *idx, int k, const float *scores, const void *gate_w, const void *up_w,
                              int64_t gu_row_stride, int64_t gu_expert_stride, const void *down_w,
                              int64_t d_row_stride, int64_t d_expert_stride, int64_t e_local, int64_t f,
                              int64_t expert_base, int64_t e_total, int act, void *y, int y_dtype, void *workspace,
                              size_t workspace_bytes, void *stream) {
    g_msg[0] = 0;
    if (act < KQ_ACT_SILU || act > KQ_ACT_GELU_TANH) return fail(KQ_ERR_SHAPE, "moe_expert_layer_local: bad activation %d", act);
    if (k <= 0 || t < 0) return fail(KQ_ERR_SHAPE, "moe_expert_layer_local: bad t/k");
    if (expert_base < 0 || e_local <= 0 || expert_base + e_local > e_total)
        return fail(KQ_ERR_SHAPE, "moe_expert_layer_local: local experts [%lld, %lld) outside %lld", (long long)expert_base,
                    (long long)(expert_base + e_local), (long long)e_total);
    if (t == 0) return KQ_OK;
    const int64_t slots = t * k;
    const size_t a = routed_ws(codec_gu, slots, t, e_local, f, d, ACT_SILU, false);
    const size_t b = routed_ws(codec_d, slots, t, e_local, d, f, ACT_NONE, true);
    const size_t routed = align256(a > b ? a : b);
    const size_t need = routed + align256((size_t)slots * f * 2);
    if (!workspace || workspace_bytes < need || ((uintptr_t)workspace & 255))
        return fail(KQ_ERR_WORKSPACE, "moe_expert_layer_local: workspace of %zu bytes required, got %zu", need,
                    workspace_bytes);
    if (use_grouped(codec_gu, slots, e_total, f, d, act, true, x_dtype, d) &&
        use_grouped(codec_d, slots, e_total, d, f, ACT_NONE, false, x_dtype, f) &&
        workspace_bytes >= layer_plan(codec_gu, codec_d, slots, e_local, e_total, d, f, y_dtype != KQ_F32).total) {
        const char *what = "moe_expert_layer_local";
        int rc;
        if ((rc = check_weights(codec_gu, gate_w, d, gu_row_stride, what)) ||
            (rc = check_weights(codec_gu, up_w, d, gu_row_stride, what)) ||
            (rc = check_weights(codec_d, down_w, f, d_row_stride, what)) || (rc = check_x(x, x_dtype, d, what)))
            return rc;
        if (!out_dtype_ok(y_dtype)) return fail(KQ_ERR_DTYPE, "%s: bad output dtype %d", what, y_dtype);
        return run_grouped_layer(codec_gu, codec_d, x, x_dtype, t, d, idx, k, scores, gate_w, up_w, gu_row_stride,
                                 gu_expert_stride, down_w, d_row_stride, d_expert_stride, e_local, f, expert_base,
                                 e_total, act, y, y_dtype, workspace, workspace_bytes, stream);
    }
    void *h = (char *)workspace + routed;
    int rc = run_routed(codec_gu, x, x_dtype, d, d, slots, k, t, idx, nullptr, 0, gate_w, up_w, e_local, f,
                        gu_row_stride, gu_expert_stride, act, h, x_dtype, f, nullptr, workspace, routed, stream,
                        "moe_expert_layer_local", expert_base, e_total);
    if (rc) return rc;
    // both projections on the routed GEMV with the same group size: the down
    // projection reads the gate/up call's group tables (one grouping launch per layer)
    const bool reuse = !use_grouped(codec_gu, slots, e_total, f, d, act, true, x_dtype, d) &&
                       !use_grouped(codec_d, slots, e_total, d, f, ACT_NONE, false, x_dtype, f) &&
                       routed_gsize(codec_gu, slots, t, e_total) == routed_gsize(codec_d, slots, t, e_total);
    return run_routed(codec_d, h, x_dtype, f, f, slots, k, t, idx, nullptr, 1, down_w, nullptr, e_local, d, d_row_stride,
                      d_expert_stride, ACT_NONE, y, y_dtype, d, scores, workspace, routed, stream,
                      "moe_expert_layer_local", expert_base, e_total, reuse);
}

// ---- chain of one-row projections (kq_chain.cu) ----

static int chain_descs(const kq_chain_problem *pr, int count, int x_dtype, kq::ChainProblemDesc *d, bool check) {
    const char *what = "quantized_matmul_chain";
    if (count < 1 || count > KQ_CHAIN_MAX || !pr)
        return fail(KQ_ERR_SHAPE, "%s: count %d outside 1..%d", what, count, KQ_CHAIN_MAX);
    if (check && !act_dtype_ok(x_dtype)) return fail(KQ_ERR_DTYPE, "%s: activations must be f16 or bf16", what);
    for (int q = 0; q < count; q++) {
        const kq_chain_problem &p = pr[q];
        if (check) {
            int rc;
            if ((rc = check_weights(p.codec, p.w, p.k, p.w_row_stride, what))) return rc;
            if (p.act != ACT_NONE && (rc = check_weights(p.codec, p.w2, p.k, p.w_row_stride, what))) return rc;
            if ((rc = check_x(p.x, x_dtype, p.k, what))) return rc;
            if (!out_dtype_ok(p.y_dtype)) return fail(KQ_ERR_DTYPE, "%s: problem %d: bad output dtype", what, q);
            if (p.bias && (p.act != ACT_NONE || !out_dtype_ok(p.bias_dtype)))
                return fail(KQ_ERR_DTYPE, "%s: problem %d: bias only on plain projections", what, q);
            if (p.act < ACT_NONE || p.act > ACT_GELU_TANH) return fail(KQ_ERR_SHAPE, "%s: problem %d: bad act", what, q);
            if (p.n <= 0 || p.n > 0x7fffffff || p.k > 0x7fffffff)
                return fail(KQ_ERR_SHAPE, "%s: problem %d: bad n / k", what, q);
            if (p.depends_on >= q || p.depends_on < -1)
                return fail(KQ_ERR_SHAPE, "%s: problem %d depends on %d (must be an earlier problem or -1)", what, q,
                            p.depends_on);
        } else if (p.k <= 0 || p.k % QK || p.n <= 0) {
            return 1;
        }
        kq::ChainProblemDesc &e = d[q];
        e.codec = p.codec;
        e.x = p.x;
        e.w = p.w;
        e.w2 = p.w2;
        e.n = p.n;
        e.k = p.k;
        e.w_row_stride = p.w_row_stride;
        e.act = p.act;
        e.y = p.y;
        e.y_dtype = p.y_dtype;
        e.bias = p.bias;
        e.bias_dtype = p.bias_dtype;
        e.dep = p.depends_on;
    }
    return KQ_OK;
}

// chain workspace: [0, 256) error word; the work / exit / completion counters
// and the K-split tile counters in the last 64 KB of the counter region that
// every kq call leaves zero (the chain leaves its counters zero too, so calls
// sharing one workspace never see each other's counts); the partial rows,
// scratch, after that region
constexpr size_t CHAIN_CTL = 256 + CNT_RESERVE - 65536;
constexpr long CHAIN_MAX_SPLIT_TILES = (65536 - 256) / 4;
struct ChainWs {
    size_t ctl_off = CHAIN_CTL, tcnt_off = CHAIN_CTL + 256, part_off = 256 + CNT_RESERVE, total = 0;
};
static ChainWs chain_ws(const kq::ChainPlan &pl) {
    ChainWs w;
    w.total = align256(w.part_off + (size_t)pl.partial_floats * sizeof(float));
    return w;
}

static bool chain_fits(const kq::ChainPlan &pl) { return pl.split_tiles <= CHAIN_MAX_SPLIT_TILES; }

size_t kq_quantized_matmul_chain_workspace_size(const kq_chain_problem *problems, int count) {
    kq::ChainProblemDesc d[KQ_CHAIN_MAX];
    if (chain_descs(problems, count, KQ_BF16, d, false)) return 0;
    size_t need = 256;
    kq::ChainPlan pl;
    if (kq::chain_plan(d, count, &pl) && chain_fits(pl)) need = chain_ws(pl).total;
    // the per-problem path's workspace, should the fused kernel not take the chain
    for (int q = 0; q < count; q++)
        need = std::max(need, dense_ws(d[q].codec, 1, d[q].n, d[q].k, d[q].act));
    return need;
}

int kq_quantized_matmul_chain(const kq_chain_problem *problems, int count, int x_dtype, void *workspace,
                              size_t workspace_bytes, void *stream) {
    g_msg[0] = 0;
    const char *what = "quantized_matmul_chain";
    kq::ChainProblemDesc d[KQ_CHAIN_MAX];
    int rc = chain_descs(problems, count, x_dtype, d, true);
    if (rc) return rc;
    if (!workspace || ((uintptr_t)workspace & 255))
        return fail(KQ_ERR_WORKSPACE, "%s: a 256-byte aligned workspace is required", what);
    kq::ChainPlan pl;
    if (!dev_env("KQ_CHAIN_UNFUSED") && kq::chain_plan(d, count, &pl) && chain_fits(pl)) {
        const ChainWs w = chain_ws(pl);
        if (workspace_bytes < w.total)
            return fail(KQ_ERR_WORKSPACE, "%s: workspace of %zu bytes required, got %zu", what, w.total, workspace_bytes);
        char *ws = (char *)workspace;
        return cuda_status(kq::launch_chain(d, count, pl, x_dtype, (int *)ws, (int *)(ws + w.ctl_off),
                                            (int *)(ws + w.tcnt_off), (float *)(ws + w.part_off), (cudaStream_t)stream),
                           what);
    }
    // no fused kernel for this chain: one launch per problem, in order
    for (int q = 0; q < count; q++) {
        const kq::ChainProblemDesc &e = d[q];
        rc = run_dense(e.codec, e.x, x_dtype, 1, e.k, e.k, e.w, e.act != ACT_NONE ? e.w2 : nullptr, e.n,
                       e.w_row_stride, e.act, e.y, e.y_dtype, e.n, workspace, workspace_bytes, stream, what, e.bias,
                       e.bias_dtype);
        if (rc) return rc;
    }
    return KQ_OK;
}

int kq_workspace_error(void *workspace, int clear, void *stream) {
    if (!workspace) return 0;
    int v = 0;
    cudaStream_t st = (cudaStream_t)stream;
    if (cudaMemcpyAsync(&v, workspace, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess) return -1;
    if (cudaStreamSynchronize(st) != cudaSuccess) return -1;
    if (clear && v) {
        int z = 0;
        cudaMemcpyAsync(workspace, &z, sizeof(int), cudaMemcpyHostToDevice, st);
        cudaStreamSynchronize(st);
    }
    return v;
}

}  // extern "C"
