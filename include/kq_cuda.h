/*
 * kq_cuda.h -- C ABI of libkq_cuda.so, the B200 (sm_100a) fused
 * dequantize-and-multiply library for GGUF K-quant / IQ-quant weights.
 *
 * It replaces the kernel library that gmlx reaches as ``import mlx_kquant as
 * kq`` (gmlx/modules.py:35-40; pinned mlx-kquant>=0.3.13,<0.4 at
 * pyproject.toml:33).  Each entry point below names the kq op and the gmlx
 * call site(s) it serves.  Conventions:
 *
 *  - All pointers are device pointers unless stated; sizes are element counts
 *    unless the name ends in _bytes / _stride (bytes for weights, elements for
 *    activations).  Weight rows are raw GGUF wire bytes, never repacked.
 *  - Every call is asynchronous on `stream` (a cudaStream_t; NULL = legacy
 *    default stream) and returns KQ_OK or a KQ_ERR_* code; a human-readable
 *    message for the calling thread is available from kq_last_error().
 *    Nothing crosses the ABI as an exception.
 *  - Calls that take a `workspace` need kq_*_workspace_size() bytes of device
 *    memory, 256-byte aligned and zero-filled before its first use.  The
 *    library leaves it zeroed after every successful call (self-resetting
 *    split-K counters), so one workspace can be reused by consecutive calls
 *    on one stream; calls that overlap in time must use different workspaces.
 *    The first int of a workspace is a sticky device error word set by a
 *    kernel whose bounded wait ran out (read it with kq_workspace_error).
 *  - Codec ids are ggml's: Q8_0 = 8, Q4_K = 12, Q5_K = 13, Q6_K = 14, IQ2_XXS = 16,
 *    IQ3_XXS = 18, IQ4_XS = 23, Q4_0 = 2, IQ4_NL = 20, Q2_K = 10, Q3_K = 11, Q4_1 = 3,
 *    Q5_0 = 6, Q5_1 = 7, TQ2_0 = 35, MXFP4 = 39, IQ2_XS = 17, IQ2_S = 22, IQ3_S = 21,
 *    IQ1_S = 19, IQ1_M = 29, TQ1_0 = 34, NVFP4 = 40.
 *    Activation / output dtypes: KQ_F32 = 0, KQ_F16 = 1, KQ_BF16 = 2.
 */
#ifndef KQ_CUDA_H
#define KQ_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KQ_Q4_0 2   /* groups of eight 18-byte blocks (144 bytes per 256 weights) */
#define KQ_IQ4_NL 20 /* groups of eight 18-byte blocks (144 bytes per 256 weights) */
#define KQ_Q4_1 3   /* groups of eight 20-byte blocks (160 bytes per 256 weights) */
#define KQ_Q5_0 6   /* groups of eight 22-byte blocks (176 bytes per 256 weights) */
#define KQ_Q5_1 7   /* groups of eight 24-byte blocks (192 bytes per 256 weights) */
#define KQ_IQ1_S 19  /* 50-byte blocks */
#define KQ_IQ1_M 29  /* 56-byte blocks */
#define KQ_IQ2_XS 17 /* 74-byte blocks */
#define KQ_IQ3_S 21  /* 110-byte blocks */
#define KQ_IQ2_S 22  /* 82-byte blocks */
#define KQ_NVFP4 40 /* groups of four 36-byte blocks of 64 weights (144 bytes per 256) */
#define KQ_TQ1_0 34 /* 54-byte blocks */
#define KQ_TQ2_0 35 /* 66-byte blocks */
#define KQ_MXFP4 39 /* groups of eight 17-byte blocks (136 bytes per 256 weights) */
#define KQ_Q2_K 10  /* 84-byte blocks; weights 4-byte aligned */
#define KQ_Q3_K 11  /* 110-byte blocks */
#define KQ_Q8_0 8   /* handled in groups of eight 34-byte blocks (272 bytes per 256 weights) */
#define KQ_Q4_K 12
#define KQ_Q5_K 13
#define KQ_Q6_K 14
#define KQ_IQ2_XXS 16
#define KQ_IQ3_XXS 18 /* 98-byte blocks */
#define KQ_IQ4_XS 23  /* 136-byte blocks; weights 8-byte aligned */

#define KQ_F32 0
#define KQ_F16 1
#define KQ_BF16 2

#define KQ_ACT_NONE 0
#define KQ_ACT_SILU 1
#define KQ_ACT_GELU 2
#define KQ_ACT_GELU_TANH 3

#define KQ_OK 0
#define KQ_ERR_CODEC 1     /* unknown / unsupported codec */
#define KQ_ERR_SHAPE 2     /* K not a whole number of blocks, bad sizes */
#define KQ_ERR_ALIGN 3     /* pointer or stride alignment */
#define KQ_ERR_DTYPE 4     /* unsupported activation / output dtype */
#define KQ_ERR_CUDA 5      /* CUDA runtime error (launch, attribute) */
#define KQ_ERR_WORKSPACE 6 /* workspace missing or too small */

/* Library version (major*10000 + minor*100 + patch). */
int kq_version(void);

/* Message describing the last failed call on this thread ("" if none). */
const char *kq_last_error(void);

/* Codec capability query; replaces kq.codecs() (checked against the loader's
 * whitelist at gmlx/preflight.py:625-632, tests/test_preflight.py:99).
 * Writes up to `cap` codec ids to `out`, returns how many codecs exist. */
int kq_codecs(int *out, int cap);

/* 1 when `codec` has matmul / gather kernels here (gmlx probes this through
 * _FusedMoeCaps, gmlx/modules.py:155-234), else 0. */
int kq_codec_has_matmul(int codec);

/* Bytes per 256-weight super-block of `codec` (gguf GGML_QUANT_SIZES, used by
 * gmlx/modules.py:250-255 _kq_wire_k), or -1. */
int kq_block_bytes(int codec);

/* kq.dequantize(w, scales, codec, dtype): rows x k weights, row r at
 * w + r*w_row_stride bytes -> out[rows][k] (dense, out_dtype).  f32 output is
 * bit-identical to ggml/gguf-py block dequantization.
 * Call sites: gmlx/modules.py:1461, gmlx/loader.py:3046-3048,
 * gmlx/dsv32_patches.py:229. */
int kq_dequantize(int codec, const void *w, int64_t rows, int64_t k, int64_t w_row_stride, void *out, int out_dtype,
                  void *stream);

/* kq.quantized_matmul(x, w, scales, codec, transpose=True):
 *   y[m][n] = sum_k x[m][k] * dequant(W)[n][k]   (f32 accumulate)
 * x: [m][k] f16/bf16, row stride x_row_stride elements (multiple of 8);
 * w: [n] rows of k/256 blocks, row stride w_row_stride bytes;
 * y: [m][n] f32/f16/bf16 with row stride y_row_stride elements.
 * Decode-sized m uses the streaming GEMV kernels; prefill-sized m the
 * tensor-core (tcgen05) GEMM.
 * Call sites: KQuantLinear (gmlx/modules.py:1535-1539), gmlx/occupancy_fuse.py:
 * 284-287, 412-418, 434-437, gmlx/mtp_load.py:298. */
int kq_quantized_matmul(int codec, const void *x, int x_dtype, int64_t m, int64_t k, int64_t x_row_stride,
                        const void *w, int64_t n, int64_t w_row_stride, void *y, int y_dtype, int64_t y_row_stride,
                        void *workspace, size_t workspace_bytes, void *stream);
size_t kq_quantized_matmul_workspace_size(int codec, int64_t m, int64_t n, int64_t k);

/* Fused gate/up projection with activation, one launch:
 *   y[m][n] = act(x[m] . Wg[n]) * (x[m] . Wu[n])
 * The dense analogue of moe_glu_gather_kq for a row-concatenated gate/up pair
 * (gmlx/occupancy_fuse.py:412-418 splits a fused gate+up matmul, then applies
 * the activation in Python). */
int kq_quantized_glu(int codec, const void *x, int x_dtype, int64_t m, int64_t k, int64_t x_row_stride,
                     const void *gate_w, const void *up_w, int64_t n, int64_t w_row_stride, int act, void *y,
                     int y_dtype, int64_t y_row_stride, void *workspace, size_t workspace_bytes, void *stream);
size_t kq_quantized_glu_workspace_size(int codec, int64_t m, int64_t n, int64_t k);

/* kq.moe_router_topk(logits, k, norm_topk_prob): softmax over E (f32),
 * top-k (descending; ties -> lower id), optional renormalisation.
 * logits [t][e] f32, e <= 1024, k <= 16 -> idx [t][k] int32, scores [t][k] f32.
 * Call sites: gmlx/modules.py:446-447, 751-752; semantics of the stock
 * forward gmlx/moe_experts.py:226-240. */
int kq_moe_router_topk(const float *logits, int64_t t, int64_t e, int k, int norm_topk_prob, int32_t *idx,
                       float *scores, void *stream);

/* The full router surface kq.moe_router_topk(logits, k, norm_topk_prob,
 * shared_gate=True, per_expert_scale=None) (gmlx/modules.py:751-752 with the
 * shared-gate row appended by _build_router_cat, :294-313; shared_gate=False
 * at :446-447; per_expert_scale at :1043-1046).  e = routed experts.
 * shared_gate != 0: logits rows have e + 1 columns, the last the shared
 * expert's gate; scores rows have k + 1 columns, the last sigmoid(gate).
 * per_expert_scale [e] f32 (nullable) multiplies each picked score. */
int kq_moe_router_topk_ex(const float *logits, int64_t t, int64_t e, int k, int norm_topk_prob, int shared_gate,
                          const float *per_expert_scale, int32_t *idx, float *scores, void *stream);

/* kq.moe_glu_gather_kq(x, gate_w, up_w, codec, idx, act):
 *   h[t][j][f] = act(x[t] . Wg[idx[t][j]][f]) * (x[t] . Wu[idx[t][j]][f])
 * x [t][d] f16/bf16; idx [t][k] int32 device; gate/up stacks [e][f] rows of
 * d/256 blocks (row / expert strides in bytes, shared by both stacks);
 * h [t][k][f] in h_dtype.  Each routed expert's weights stream once.
 * Call sites: gmlx/modules.py:585-588, 980-983. */
int kq_moe_glu_gather(int codec, const void *x, int x_dtype, int64_t t, int64_t d, const int32_t *idx, int k,
                      const void *gate_w, const void *up_w, int64_t e, int64_t f, int64_t w_row_stride,
                      int64_t w_expert_stride, int act, void *h, int h_dtype, void *workspace,
                      size_t workspace_bytes, void *stream);

/* kq.gather_qmv_kq(h, w, codec, idx):  y[t][j][n] = h[t][j] . W[idx[t][j]][n]
 * h [t][k][f] f16/bf16 -> y [t][k][n].  Call site: gmlx/modules.py:596-598. */
int kq_gather_qmv(int codec, const void *h, int h_dtype, int64_t t, int k, int64_t f, const int32_t *idx,
                  const void *w, int64_t e, int64_t n, int64_t w_row_stride, int64_t w_expert_stride, void *y,
                  int y_dtype, void *workspace, size_t workspace_bytes, void *stream);

/* kq.gather_qmv_mix_ns_kq(h, w, codec, idx, scores):
 *   y[t][n] = sum_j scores[t][j] * (h[t][j] . W[idx[t][j]][n])   (f32, fixed j order)
 * scores [t][k] f32.  Call sites: gmlx/modules.py:591-593, 989-991. */
int kq_gather_qmv_mix(int codec, const void *h, int h_dtype, int64_t t, int k, int64_t f, const int32_t *idx,
                      const float *scores, const void *w, int64_t e, int64_t n, int64_t w_row_stride,
                      int64_t w_expert_stride, void *y, int y_dtype, void *workspace, size_t workspace_bytes,
                      void *stream);

/* kq.gather_qmm(x, w, scales, rhs_indices=...) flattened to rows:
 *   y[r][n] = x[x_index[r]] . W[expert_index[r]][n]   for r < rows
 * (KQuantSwitchLinear, gmlx/modules.py:1548-1552; the sorted-indices prefill
 * variant at gmlx/modules.py:1308-1309).  x_index may be NULL (row r). */
int kq_gather_qmm(int codec, const void *x, int x_dtype, int64_t k, int64_t x_row_stride, int64_t rows,
                  const int32_t *x_index, const int32_t *expert_index, const void *w, int64_t e, int64_t n,
                  int64_t w_row_stride, int64_t w_expert_stride, void *y, int y_dtype, void *workspace,
                  size_t workspace_bytes, void *stream);

/* Workspace bytes for the MoE calls above with `slots` = t*k routed rows
 * (or `rows` for kq_gather_qmm), over stacks of e experts, n outputs, k_in
 * inputs. */
size_t kq_moe_workspace_size(int codec, int64_t slots, int64_t e, int64_t n, int64_t k_in);

/* One expert-parallel rank's share of a routed MoE expert layer (decode), in
 * one call: y[t] = sum over the slots j whose expert lies in this rank's
 * range [expert_base, expert_base + e_local) of
 *     scores[t][j] * down_e( act(gate_e(x[t])) * up_e(x[t]) ),
 * with e = idx[t][j] - expert_base indexing the local stacks.  Summing y over
 * the ranks (all-reduce) gives the full layer: the reference shards SwitchGLU
 * experts this way and all_sums the result (gmlx/moe_experts.py:250-266;
 * fused decode ops gmlx/modules.py:585-594).  idx holds global expert ids in
 * [0, e_total).  y is [t][d] in y_dtype. */
int kq_moe_expert_layer_local(int codec_gu, int codec_d, const void *x, int x_dtype, int64_t t, int64_t d,
                              const int32_t *idx, int k, const float *scores, const void *gate_w, const void *up_w,
                              int64_t gu_row_stride, int64_t gu_expert_stride, const void *down_w,
                              int64_t d_row_stride, int64_t d_expert_stride, int64_t e_local, int64_t f,
                              int64_t expert_base, int64_t e_total, int act, void *y, int y_dtype, void *workspace,
                              size_t workspace_bytes, void *stream);
size_t kq_moe_expert_layer_workspace_size(int codec_gu, int codec_d, int64_t t, int k, int64_t e_local, int64_t d,
                                          int64_t f, int h_dtype);

/* kq.quantized_matmul_qmv_bias(x, w, scales, bias, codec): y = x . dequant(w)^T
 * + bias in one dispatch (gmlx/qkv_fuse.py:80, the row-concatenated q|k|v
 * projection with its biases).  bias [n] in KQ_F32 / KQ_F16 / KQ_BF16; the
 * workspace is kq_quantized_matmul_workspace_size's.  Decode shapes add the
 * bias in the GEMV's store; prefill shapes add it after the GEMM. */
int kq_quantized_matmul_bias(int codec, const void *x, int x_dtype, int64_t m, int64_t k, int64_t x_row_stride,
                             const void *w, int64_t n, int64_t w_row_stride, const void *bias, int bias_dtype, void *y,
                             int y_dtype, int64_t y_row_stride, void *workspace, size_t workspace_bytes, void *stream);

/* ---- Row-parallel decode with the all-reduce fused in (tensor parallelism)
 *
 * Replaces the pair "quantized_matmul on this rank's K shard, then sum over
 * ranks" of a row-parallel (K-split) projection: the all_sum that follows the
 * sharded projections in gmlx's tensor-parallel layers
 * (gmlx/hy_v3_model.py:259 after shard_linear, gmlx/hy_v3_model.py:396-443).
 * One kernel computes this rank's partial y (one activation row), stores it
 * into every rank's communication buffer over NVLink (peer stores), raises
 * this rank's flag there, waits for all ranks' flags (bounded, ~2 s: on
 * expiry the workspace error word becomes 7) and writes the rank-order sum to
 * y, identical bits on every rank.
 *
 * comm_bufs: device array of `world` device pointers, the communication
 * buffers of all ranks mapped into this process (own buffer at [rank]), each
 * kq_allreduce_buffer_bytes(world, n) bytes, zero-filled before the first
 * call (kq_comm_alloc does both).  All ranks must make the same sequence of
 * calls on a buffer set.  Peer buffers come from kq_ipc_handle / kq_ipc_open
 * (CUDA IPC; handles are 64 bytes). */
size_t kq_allreduce_buffer_bytes(int world, int64_t n);
int kq_quantized_matmul_allreduce(int codec, const void *x, int x_dtype, int64_t k, const void *w, int64_t n,
                                  int64_t w_row_stride, void *y, int y_dtype, int world, int rank,
                                  void *const *comm_bufs, void *workspace, size_t workspace_bytes, void *stream);
/* One-shot all-reduce (sum) of n values over the ranks of a buffer set, for
 * the cross-rank sum after a row-parallel decode projection: the all_sum of
 * gmlx's tensor-parallel layers (gmlx/hy_v3_model.py:259 after shard_linear,
 * :396-443).  Every rank stores each value, as one 8-byte word {f32 bits,
 * call flag}, into every rank's communication buffer over NVLink, waits for
 * all ranks' words of this call (bounded, ~2 s: on expiry the buffer's error
 * word, read by kq_comm_error, becomes 7 and y is left incomplete) and writes
 * the rank-order f32 sum to y in y_dtype, identical bits on every rank.  y may
 * equal x.  x_dtype / y_dtype: KQ_F32 / KQ_F16 / KQ_BF16; buf_n: the n the
 * buffers were sized for (kq_allreduce_buffer_bytes(world, buf_n)), n <= buf_n;
 * world <= 8.  Shares the buffers, epoch and call-order rule of
 * kq_quantized_matmul_allreduce. */
int kq_allreduce(const void *x, int x_dtype, void *y, int y_dtype, int64_t n, int64_t buf_n, int world, int rank,
                 void *const *comm_bufs, void *stream);
/* Error word of this rank's communication buffer (0 = no expired wait), read
 * after synchronizing `stream`; clear != 0 resets it.  Negative: -KQ_ERR_CUDA. */
int kq_comm_error(void *own_buf, int clear, void *stream);
int kq_comm_alloc(size_t bytes, void **ptr);
int kq_comm_free(void *ptr);
int kq_ipc_handle(const void *ptr, void *handle64);
int kq_ipc_open(const void *handle64, void **ptr);
int kq_ipc_close(void *ptr);

/* Size of the fixed scratch array behind kq_quantized_matmul_noalloc. */
#define KQ_NOALLOC_SCRATCH_BYTES (4 << 20)

/* kq_quantized_matmul for callers that cannot allocate device memory (a host
 * framework whose allocator owns the GPU, a plugin that may not allocate after
 * start-up, a latency-critical path where an allocation could block or fail).
 * No counterpart in the reference: it is an addition of this library.  Same
 * arguments and result as kq_quantized_matmul minus the workspace: the split-K
 * scratch comes from one library-owned device array of KQ_NOALLOC_SCRATCH_BYTES
 * per GPU (held until exit).  It allocates nothing.  The first call on a
 * device looks up that array's device address (make it before any stream
 * capture); each call clears the scratch it uses on `stream`; calls whose GPU
 * work overlaps race on the shared array.  Shapes needing more scratch than
 * the array holds return KQ_ERR_WORKSPACE.  The cached address is not valid
 * across cudaDeviceReset: do not use this entry point after resetting a
 * device it has run on. */
int kq_quantized_matmul_noalloc(int codec, const void *x, int x_dtype, int64_t m, int64_t k, int64_t x_row_stride,
                                const void *w, int64_t n, int64_t w_row_stride, void *y, int y_dtype,
                                int64_t y_row_stride, void *stream);

/* The device error word of kq_quantized_matmul_noalloc's scratch on the
 * current device (no counterpart in the reference; the accessor of the
 * allocation-free entry point): 0, or the code that a kernel of the last call
 * recorded when a bounded wait ran out.  Read it before the next call, which
 * clears it.  Synchronises `stream`; clear != 0 resets the word; < 0 on a
 * CUDA failure. */
int kq_noalloc_error(int clear, void *stream);

/* ---- A chain of one-row decode projections in one launch
 *
 * The dense decode of one token is a short chain of quantized matmuls on one
 * activation row: q|k|v, o, gate+up, down (gmlx's occupancy fusions row-
 * concatenate the ones that share an input, gmlx/occupancy_fuse.py:141-200
 * and :272-330, to launch fewer kernels).  kq_quantized_matmul_chain runs up
 * to KQ_CHAIN_MAX such projections in ONE persistent launch: the GPU flows
 * from one projection's weights into the next with no per-launch ramp or
 * tail.  A problem whose input is an earlier problem's output names it in
 * depends_on; its weights stream in while it waits, and its activations are
 * read only once that problem's every output tile is stored (device-side
 * completion counters, bounded waits: on expiry the workspace error word
 * becomes 3 or 4).  Each problem computes what kq_quantized_matmul (act ==
 * KQ_ACT_NONE, optional bias) or kq_quantized_glu (act != KQ_ACT_NONE, w2 =
 * up weights) computes for one activation row.  The fused kernel takes
 * chains of Q4_K and Q6_K problems (the Q4_K_M mix) with k <= 16384; any
 * other chain runs as one launch per problem, in order, with the same
 * results. */
#define KQ_CHAIN_MAX 8
typedef struct kq_chain_problem {
    int codec;
    const void *x;        /* one activation row [k] of the chain's x_dtype, 16-byte aligned */
    const void *w;        /* [n] rows of k/256 blocks at w_row_stride bytes */
    const void *w2;       /* up weights of a fused gate/up (act != KQ_ACT_NONE), else NULL */
    int64_t n, k, w_row_stride;
    int act;              /* KQ_ACT_NONE, or the gate activation of a fused gate/up */
    void *y;              /* [n] outputs in y_dtype */
    int y_dtype;
    const void *bias;     /* optional [n] bias (act == KQ_ACT_NONE only), NULL if none */
    int bias_dtype;
    int depends_on;       /* index of an earlier problem whose output x reads, or -1 */
} kq_chain_problem;
size_t kq_quantized_matmul_chain_workspace_size(const kq_chain_problem *problems, int count);
int kq_quantized_matmul_chain(const kq_chain_problem *problems, int count, int x_dtype, void *workspace,
                              size_t workspace_bytes, void *stream);

/* Reads (and with clear != 0 resets) the workspace's device error word;
 * synchronises `stream`.  Returns the word (0 = no device-side error). */
int kq_workspace_error(void *workspace, int clear, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* KQ_CUDA_H */
