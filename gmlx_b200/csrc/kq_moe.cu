// kq_moe.cu -- MoE routing support kernels.
//
//  * router_topk: softmax -> top-k -> optional renormalisation in one launch,
//    the kq.moe_router_topk op (gmlx/modules.py:751-752) and the stock
//    Qwen3-MoE selection it replaces (gmlx/moe_experts.py:226-240:
//    softmax(precise) -> argpartition top-k -> take -> scores/sum).  Output
//    order is descending probability, ties to the lower expert id.
//  * moe_groups: bucket the T*k routed slots by expert into groups of <= 32
//    slots so the GEMV streams every touched expert's weights exactly once.
//  * moe_mix: y[t] = sum_j scores[t,j] * ys[t,j] in a fixed j order (the
//    gather_qmv_mix_ns_kq combine, gmlx/modules.py:589-594, in f32).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "kq_internal.cuh"

namespace kq {
namespace {

constexpr int RT_MAXE = 1024, RT_MAXK = 16;

// shared_gate: each logits row has E + 1 columns, the last one the shared
// expert's gate; its sigmoid becomes score column k (scores rows of k + 1).
// pes: optional per-expert scale applied to each picked score last.
__global__ void router_kernel(const float *__restrict__ logits, int T, int E, int k, int norm, int32_t *__restrict__ idx,
                              float *__restrict__ scores, int shared_gate, const float *__restrict__ pes) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= T) return;
    const int ld = E + (shared_gate ? 1 : 0), sk = k + (shared_gate ? 1 : 0);
    const float *l = logits + (int64_t)warp * ld;
    constexpr int PER = RT_MAXE / 32;
    float p[PER];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < PER; i++) {
        const int e = lane + 32 * i;
        p[i] = e < E ? l[e] : -INFINITY;
        mx = fmaxf(mx, p[i]);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < PER; i++) {
        const int e = lane + 32 * i;
        p[i] = e < E ? expf(p[i] - mx) : 0.f;
        s += p[i];
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float inv = 1.0f / s;
#pragma unroll
    for (int i = 0; i < PER; i++) p[i] = (lane + 32 * i) < E ? p[i] * inv : -1.0f;
    float sel[RT_MAXK];
    int seli[RT_MAXK];
    float tot = 0.f;
    for (int c = 0; c < k; c++) {
        float bv = -2.0f;
        int bi = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < PER; i++) {
            const int e = lane + 32 * i;
            if (p[i] > bv || (p[i] == bv && e < bi)) { bv = p[i]; bi = e; }
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        sel[c] = bv;
        seli[c] = bi;
        tot += bv;
#pragma unroll
        for (int i = 0; i < PER; i++)
            if (lane + 32 * i == bi) p[i] = -1.0f;
    }
    if (lane == 0) {
        for (int c = 0; c < k; c++) {
            idx[(int64_t)warp * k + c] = seli[c];
            const float v = norm ? sel[c] / tot : sel[c];
            scores[(int64_t)warp * sk + c] = pes ? v * pes[seli[c]] : v;
        }
        if (shared_gate) scores[(int64_t)warp * sk + k] = 1.0f / (1.0f + expf(-l[E]));
    }
}

// Groups over the local expert range [ebase, ebase + ecount): slots routed
// elsewhere are skipped (expert-parallel ranks); ids outside [0, etotal) are
// an error.  Slots of an expert keep their slot order (group g of expert e
// holds its slots gsize*g .. gsize*g + gsize - 1).  Three passes in one CTA:
// per-expert counts (shared-memory atomics), group offsets (one warp's scan),
// then one warp places the slots 32 at a time, ranking equal experts within
// the chunk with __match_any_sync, so the work is O(slots + experts).
__global__ void groups_kernel(const int32_t *__restrict__ idx, int S, int k, int ebase, int ecount, int etotal,
                              int xrow_is_slot, const int32_t *__restrict__ xidx, int gsize,
                              int *__restrict__ n_groups, int *__restrict__ grp_expert, int *__restrict__ grp_count,
                              int *__restrict__ grp_xrow, int *__restrict__ grp_orow, int max_groups,
                              int *__restrict__ err) {
    constexpr int SIDX = 4096;  // routing ids staged in shared memory for the placement pass
    __shared__ int s_cnt[RT_MAXE], s_first[RT_MAXE + 1], s_base[RT_MAXE], s_idx[SIDX];
    __shared__ int s_bad;
    // launched as a programmatic dependent: the routing ids may be the
    // previous kernel's output (no early trigger here: the GEMV that follows
    // reads the group tables before its own dependency wait)
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) s_bad = 0;
    for (int e = threadIdx.x; e < ecount; e += blockDim.x) s_cnt[e] = 0, s_base[e] = 0;
    __syncthreads();
    for (int s = threadIdx.x; s < S; s += blockDim.x) {
        const int v = idx[s];
        if (s < SIDX) s_idx[s] = v;
        if (v < 0 || v >= etotal) s_bad = 1;
        else if (v >= ebase && v < ebase + ecount) atomicAdd(&s_cnt[v - ebase], 1);
    }
    __syncthreads();
    if (warp == 0) {  // s_first[e] = groups of experts < e (lane-chunked exclusive scan)
        const int per = (ecount + 31) / 32, e0 = lane * per, e1 = min(ecount, e0 + per);
        int t = 0;
        for (int e = e0; e < e1; e++) t += (s_cnt[e] + gsize - 1) / gsize;
        int incl = t;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int u = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += u;
        }
        int run = incl - t;
        for (int e = e0; e < e1; e++) {
            s_first[e] = run;
            run += (s_cnt[e] + gsize - 1) / gsize;
        }
        if (lane == 31) {
            s_first[ecount] = incl;
            *n_groups = s_bad ? 0 : min(incl, max_groups);
            if (s_bad) atomicCAS(err, 0, 3);
            else if (incl > max_groups) atomicCAS(err, 0, 4);
        }
    }
    __syncthreads();
    if (s_bad || warp != 0) return;
    for (int c = 0; c < S; c += 32) {  // stable placement, 32 slots at a time
        const int s = c + lane;
        const int v = s < S ? (s < SIDX ? s_idx[s] : idx[s]) : -1;
        const bool local = v >= ebase && v < ebase + ecount;
        const int e = v - ebase;
        const unsigned peers = __match_any_sync(0xffffffffu, local ? e : -1 - lane);
        int p = 0;
        if (local) p = s_base[e] + __popc(peers & ((1u << lane) - 1u));
        __syncwarp();
        if (local && lane == 31 - __clz(peers)) s_base[e] += __popc(peers);
        __syncwarp();
        if (!local) continue;
        const int gi = s_first[e] + p / gsize, n = p % gsize;
        if (gi >= max_groups) continue;
        grp_xrow[gi * 32 + n] = xidx ? xidx[s] : xrow_is_slot ? s : s / k;
        grp_orow[gi * 32 + n] = s;
        if (n == 0) {
            grp_expert[gi] = e;
            grp_count[gi] = min(gsize, s_cnt[e] - p);
        }
    }
}

__global__ void mix_kernel(const float *__restrict__ ys, const float *__restrict__ scores,
                           const int32_t *__restrict__ idx, int ebase, int ecount, int T, int k, int N,
                           void *__restrict__ y, int y_dtype) {
    asm volatile("griddepcontrol.wait;" ::: "memory");  // ys is the previous kernel's output
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)T * N) return;
    const int t = (int)(i / N), n = (int)(i - (int64_t)t * N);
    float v = 0.f;
    for (int j = 0; j < k; j++) {
        const int e = idx[t * k + j] - ebase;
        if (e >= 0 && e < ecount) v = fmaf(scores[t * k + j], ys[((int64_t)t * k + j) * N + n], v);
    }
    if (y_dtype == F32) reinterpret_cast<float *>(y)[i] = v;
    else if (y_dtype == BF16) reinterpret_cast<__nv_bfloat16 *>(y)[i] = __float2bfloat16_rn(v);
    else reinterpret_cast<__half *>(y)[i] = __float2half_rn(v);
}

__global__ void add_bias_kernel(void *y, int y_dtype, int64_t ys, int64_t m, int64_t n, const void *bias, int bd) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= m * n) return;
    const int64_t r = i / n, c = i - r * n;
    const float b = bd == F32 ? reinterpret_cast<const float *>(bias)[c]
                  : bd == BF16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(bias)[c])
                               : __half2float(reinterpret_cast<const __half *>(bias)[c]);
    const int64_t o = r * ys + c;
    if (y_dtype == F32) reinterpret_cast<float *>(y)[o] += b;
    else if (y_dtype == BF16) {
        __nv_bfloat16 *p = reinterpret_cast<__nv_bfloat16 *>(y) + o;
        *p = __float2bfloat16_rn(__bfloat162float(*p) + b);
    } else {
        __half *p = reinterpret_cast<__half *>(y) + o;
        *p = __float2half_rn(__half2float(*p) + b);
    }
}

}  // namespace

cudaError_t launch_add_bias(void *y, int y_dtype, int64_t y_row_stride, int64_t m, int64_t n, const void *bias,
                            int bias_dtype, cudaStream_t st) {
    if (m * n == 0) return cudaSuccess;
    add_bias_kernel<<<(unsigned)((m * n + 255) / 256), 256, 0, st>>>(y, y_dtype, y_row_stride, m, n, bias, bias_dtype);
    return cudaGetLastError();
}

cudaError_t launch_router_topk(const float *logits, int T, int E, int k, int norm, int32_t *idx, float *scores,
                               int shared_gate, const float *per_expert_scale, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    const int threads = 256, per = threads / 32;
    router_kernel<<<(T + per - 1) / per, threads, 0, st>>>(logits, T, E, k, norm, idx, scores, shared_gate,
                                                           per_expert_scale);
    return cudaGetLastError();
}

cudaError_t launch_moe_groups(const int32_t *idx, int S, int k, int ebase, int ecount, int etotal, int xrow_is_slot,
                              const int32_t *xidx, int gsize, int *n_groups, int *grp_expert, int *grp_count,
                              int *grp_xrow, int *grp_orow, int max_groups, int *err, cudaStream_t st) {
    if (ecount > RT_MAXE) return cudaErrorInvalidValue;  // per-expert tables live in shared memory
    // programmatic dependent launch: the launch overlaps the previous kernel's
    // tail; the kernel waits for that kernel's completion before reading idx
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(1024);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, groups_kernel, idx, S, k, ebase, ecount, etotal, xrow_is_slot, xidx, gsize,
                              n_groups, grp_expert, grp_count, grp_xrow, grp_orow, max_groups, err);
}

cudaError_t launch_moe_mix(const float *ys, const float *scores, const int32_t *idx, int ebase, int ecount, int T,
                           int k, int N, void *y, int y_dtype, cudaStream_t st) {
    const int64_t n = (int64_t)T * N;
    if (n == 0) return cudaSuccess;
    cudaLaunchConfig_t cfg = {};  // programmatic dependent of the down-projection GEMV
    cfg.gridDim = dim3((unsigned)((n + 255) / 256));
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, mix_kernel, ys, scores, idx, ebase, ecount, T, k, N, y, y_dtype);
}

}  // namespace kq
