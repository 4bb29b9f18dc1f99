// kq_internal.cuh -- launchers shared between the kernel files and the C ABI.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>

#include "kq_formats.cuh"

namespace kq {

// Activation functions of the fused gate/up epilogue (gmlx/modules.py:522-525
// lists silu and gelu for the kq fused MoE ops).
enum Act : int { ACT_NONE = 0, ACT_SILU = 1, ACT_GELU = 2, ACT_GELU_TANH = 3 };

__device__ __forceinline__ void store_out(void *y, int dtype, int64_t i, float v) {
    if (dtype == F32) reinterpret_cast<float *>(y)[i] = v;
    else if (dtype == BF16) reinterpret_cast<__nv_bfloat16 *>(y)[i] = __float2bfloat16_rn(v);
    else reinterpret_cast<__half *>(y)[i] = __float2half_rn(v);
}

__device__ __forceinline__ float apply_act(int act, float g) {
    if (act == ACT_SILU) return g / (1.0f + expf(-g));
    if (act == ACT_GELU) return 0.5f * g * (1.0f + erff(g * 0.70710678118654752f));
    const float c = 0.7978845608028654f;  // tanh approximation
    return 0.5f * g * (1.0f + tanhf(c * (g + 0.044715f * g * g * g)));
}

cudaError_t launch_dequantize(int codec, const uint8_t *w, int64_t rows, int64_t k, int64_t row_stride, void *out,
                              int dtype, cudaStream_t st);

// Decode-shaped GEMV over groups of <= 32 activation rows sharing one weight
// matrix (dense decode: one group per 32 rows; MoE decode: one group per
// routed expert).  See kq_gemv.cu.
struct GemvArgs {
    int codec;
    const uint8_t *w;  // weights [E][N] rows of nb blocks
    int64_t w_row_stride, w_expert_stride;
    const uint8_t *w2;  // up weights for the fused GLU (same codec / shape)
    int64_t w2_row_stride, w2_expert_stride;
    int N, K;
    const void *x;  // activations, row i at x + i*x_row_stride elements
    int x_dtype;    // F16 or BF16
    int64_t x_row_stride;
    // Groups.  dense_m > 0: implicit groups of rows [32g, 32g+32) of x/y.
    // Otherwise the routed tables (device): *n_groups, expert, count, xrow/orow[32 per group].
    int dense_m;
    int max_groups;
    const int *n_groups;
    const int *grp_expert, *grp_count, *grp_xrow, *grp_orow;
    void *y;
    int y_dtype;
    int64_t y_row_stride;
    int act;         // ACT_NONE: plain; otherwise fused GLU y = act(x.Wg) * (x.Wu)
    float *partial;  // stream-K partial tiles: 2 x grid x 1024 floats
    int *counters;   // one per (group, tile), zero on entry, left zero
    int *err;
    int max_tokens;  // upper bound of rows in any group (<= 32)
    // fused all-reduce (row-parallel decode, one activation row): every rank
    // stores its f32 partial rows into each peer's communication buffer, then
    // sums all ranks' partials into y.  ar_bufs: device array [ar_world] of the
    // buffers (this rank's own at [ar_rank]); ar_world == 0: plain output.
    const void *bias;  // optional [N] per-output bias (dense plain GEMV), bias_dtype F32/F16/BF16
    int bias_dtype;
    unsigned char *const *ar_bufs;
    int ar_world, ar_rank;
    int dyn;         // set by the launcher: lane-per-row tiles handed out dynamically
    int ksplit;      // set by the launcher: K chunks per dynamic unit (1 = whole tiles)
    int debug;       // development only: 1 = skip decode, 2 = skip weight copies
};
cudaError_t launch_gemv(const GemvArgs &a, cudaStream_t st);
// A chain of one-row GEMVs in one persistent launch (kq_chain.cu).
struct ChainProblemDesc {
    int codec;
    const void *x, *w, *w2;
    int64_t n, k, w_row_stride;
    int act;
    void *y;
    int y_dtype;
    const void *bias;
    int bias_dtype;
    int dep;  // index of an earlier problem whose output this one reads, or -1
};
struct ChainPlan {
    int pair, total_units;
    int tiles[8], nst[8], S[8], chunk[8], unit_base[8], split_base[8], xreg[8], xoff[8], nreg;
    long split_tiles, partial_floats;
};
// false when no fused chain kernel takes these problems (codec mix, sizes)
bool chain_plan(const ChainProblemDesc *pd, int count, ChainPlan *out);
cudaError_t launch_chain(const ChainProblemDesc *pd, int count, const ChainPlan &pl, int x_dtype, int *err, int *ctl,
                         int *tcnt, float *partial, cudaStream_t st);

// Communication buffer of the fused all-reduce: a 4 KB header (word 0: this
// rank's call epoch; flags at 64 + 4 * (parity * world + rank)) and f32 slots
// [parity][world][n] from byte 4096.
constexpr size_t AR_HDR = 4096;
// f32 slots of the fused GEMV, then the one-shot all-reduce's (kq_allreduce.cu)
// 8-byte {value, flag} slots [parity][world][n]; its done counter sits at
// header byte 16 and its error word at 32.
inline size_t ar_ll_offset(int world, int64_t n) { return AR_HDR + (size_t)2 * world * n * sizeof(float); }
inline size_t ar_buffer_bytes(int world, int64_t n) { return ar_ll_offset(world, n) + (size_t)2 * world * n * 8; }
constexpr int AR_CNT = 16, AR_ERR = 32, AR_CMAX = 256, AR_MAX_WORLD = 8;
int allreduce_ctas(int world, int64_t n);
cudaError_t launch_allreduce(const void *x, int x_dtype, void *y, int y_dtype, int64_t n, int64_t buf_n, int world,
                             int rank, unsigned char *const *bufs, cudaStream_t st);
// Scratch the GEMV needs for `a` (bytes of f32 partials, bytes of counters).
void gemv_scratch_need(const GemvArgs &a, size_t *partial_bytes, size_t *counter_bytes);

// Prefill-shaped GEMM on tcgen05 (see kq_gemm_sm100.cu).
struct GemmArgs {
    int codec;
    int M, N, K;
    const void *x;
    int x_dtype;
    int64_t x_row_stride;  // elements
    const uint8_t *w;
    int64_t w_row_stride;  // bytes
    void *y;
    int y_dtype;
    int64_t y_row_stride;  // elements
    int *err;
    // grouped (MoE) mode: blockIdx.x indexes a device table of row tiles
    // (expert, first row, end row) over expert-sorted activation rows; output
    // row r goes to y row out_row[r]
    const int *n_tiles;  // device count; null = dense mode
    const int *tile_e, *tile_row0, *tile_rowend;
    const int *out_row;
    int64_t w_expert_stride;  // bytes (Q4_K fused mode)
    int n_per_expert;         // rows of B per expert (dense B-by-TMA map is [E*N, K])
    int ex_lo, ex_hi;         // grouped: only tiles of experts [ex_lo, ex_hi) run; B row base (e-ex_lo)*N
    // fused GLU (act != ACT_NONE): y = act(x.Wg) * (x.Wu); w2 = up weights (Q4_K
    // fused), or for dense B the up rows follow the gate rows of the scratch
    const uint8_t *w2;
    int act;
    // mixed output (grouped MoE down projection): y is f32 and sorted row r
    // adds row_scale[r] * (its output row) into y row out_row[r] atomically
    const float *row_scale;
    // dense, non-GLU split-K (gridDim.z = ksplit = 2): each split writes its f32
    // partial tile to part[z][M][N]; the last of a tile's splits (counter in
    // tile_cnt, zero on entry and left zero) adds the other one and stores y
    int ksplit;
    float *part;
    int *tile_cnt;
    int debug;  // development builds only (KQ_GEMM_DEBUG); 0 otherwise
};
// split-K factor the dense GEMM uses for this shape (1 or 2)
int gemm_ksplit(int codec, int64_t m, int64_t n, int64_t k, bool glu);
bool gemm_supported(int codec, int64_t m, int64_t n, int64_t k, int x_dtype, int64_t x_row_stride);
size_t gemm_scratch_bytes(int codec, int64_t m, int64_t n, int64_t k, bool glu);
cudaError_t launch_gemm(const GemmArgs &a, void *scratch, cudaStream_t st);
constexpr int GEMM_MIN_M = 33;  // activation rows from which the tensor-core GEMM takes over
// Grouped GEMM over expert-sorted rows (see kq_gemm_sm100.cu); the caller
// prepared the table of (128*mt)-row tiles with launch_moe_sort.  b_dense:
// dequantized experts [ex_lo, ex_hi) as [(ex_hi-ex_lo)*N, K] in the activation
// type (GLU: gate rows, then up rows) when the codec has no fused path, else null.
cudaError_t launch_gemm_grouped(const GemmArgs &a, int mt, int max_tiles, const void *b_dense, cudaStream_t st);
// Counting sort of routed slots by local expert + (expert, tile_rows-row tile)
// table for the grouped GEMM + gathered activation rows.  perm[p] = slot at
// sorted row p.  cnt: ecount ints that are zero on entry and left zero;
// scratch: S + ecount ints.
cudaError_t launch_moe_sort(const int32_t *idx, int S, int k, int ebase, int ecount, int etotal, int xrow_is_slot,
                            const int32_t *xidx, const void *x, int64_t x_row_stride, int K, void *xs, int tile_rows,
                            int *cnt, int *scratch, int *perm, int *counts, int *n_tiles, int *tile_e, int *tile_row0,
                            int *tile_rowend, int max_tiles, int *err, const float *scores, int *tok_of,
                            float *scale_of, cudaStream_t st);

// MoE slot grouping: idx[S] (S = T*k slots) -> groups of <= gsize slots per
// local expert (experts [ebase, ebase+ecount); ascending slot order inside a
// group, groups ordered by expert).  Activation row of slot s: xidx[s] if
// given, else s (xrow_is_slot) or s/k.  Group expert ids are local.
cudaError_t launch_moe_groups(const int32_t *idx, int S, int k, int ebase, int ecount, int etotal, int xrow_is_slot,
                              const int32_t *xidx, int gsize, int *n_groups, int *grp_expert, int *grp_count,
                              int *grp_xrow, int *grp_orow, int max_groups, int *err, cudaStream_t st);
// y[t][n] = sum over local slots j of scores[t][j] * ys[t*k+j][n]  (fixed j order).
// y[r][n] += bias[n] for rows r < m (the prefill path of the bias op)
cudaError_t launch_add_bias(void *y, int y_dtype, int64_t y_row_stride, int64_t m, int64_t n, const void *bias,
                            int bias_dtype, cudaStream_t st);
cudaError_t launch_moe_mix(const float *ys, const float *scores, const int32_t *idx, int ebase, int ecount, int T,
                           int k, int N, void *y, int y_dtype, cudaStream_t st);
cudaError_t launch_router_topk(const float *logits, int T, int E, int k, int norm, int32_t *idx, float *scores,
                               int shared_gate, const float *per_expert_scale, cudaStream_t st);

int num_sms();
// Development-only environment switches (grid / schedule overrides used while
// tuning): read only in builds with KQ_DEVELOPMENT, nullptr otherwise.
inline const char *dev_env(const char *name) {
#ifdef KQ_DEVELOPMENT
    return getenv(name);
#else
    (void)name;
    return nullptr;
#endif
}
// Sets the calling thread's kq_last_error() message.
void set_last_error(const char *msg);
// workspace bytes kq_quantized_matmul needs for exactly these activations
// (the same GEMV / GEMM choice the call makes)
size_t dense_matmul_workspace_bytes(int codec, int64_t m, int64_t n, int64_t k, int x_dtype, int64_t x_row_stride);

}  // namespace kq
