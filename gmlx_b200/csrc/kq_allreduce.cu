// kq_allreduce.cu -- one-shot all-reduce of a short vector over NVLink peer
// memory, for the row-parallel (K-split) decode projections of tensor-parallel
// layers: the all_sum after gmlx's sharded o / down projections
// (gmlx/hy_v3_model.py:259 after shard_linear, :396-443).  At decode sizes
// (one activation row: a few thousand outputs) an all-reduce is pure latency,
// so the vector is pushed once to every rank and summed there.
//
// Per call, on every rank, one kernel of C CTAs; CTA c owns the slice
// [c * per, (c + 1) * per) of the n outputs:
//   1. wait for the producer of x (programmatic dependent launch);
//   2. store each value of the slice, as one 8-byte word {f32 bits, epoch + 1},
//      into slot [parity][rank] of EVERY rank's communication buffer (peer
//      stores over NVLink, own buffer included);
//   3. read each rank's word of each value from the own buffer, waiting
//      (bounded, ~2 s) until its high half reads epoch + 1, and sum the values
//      in rank order (identical bits on every rank).
// A value and its flag arrive together in one single-copy-atomic 8-byte store,
// so no memory fence or separate flag round trip is needed.  The last CTA out
// bumps the own epoch.  Two parities: a rank can be at most one call ahead of
// a peer that is still reading, so slots of consecutive calls never collide.
// CTAs only wait on other GPUs' CTAs, never on CTAs of this GPU.  Buffer layout
// (kq_internal.cuh): epoch word 0, done counter at byte 16, error word at 32;
// the 8-byte slots [2][world][n] after the fused GEMV's f32 slots.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "kq_internal.cuh"

namespace kq {
namespace {

__device__ __forceinline__ uint64_t ar_timer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ float load_in(const void *x, int dtype, int64_t i) {
    if (dtype == F32) return reinterpret_cast<const float *>(x)[i];
    if (dtype == BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(x)[i]);
    return __half2float(reinterpret_cast<const __half *>(x)[i]);
}

__device__ __forceinline__ void st_u64_volatile(uint64_t *p, uint64_t v) {
    asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_u64_volatile(const uint64_t *p) {
    uint64_t v;
    asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __launch_bounds__(256) allreduce_kernel(const void *x, int x_dtype, void *y, int y_dtype, int64_t n,
                                                        int world, int rank, unsigned char *const *bufs,
                                                        int64_t ll_off) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    __shared__ unsigned s_epoch;
    __shared__ int s_abort_;
    volatile int &s_abort = s_abort_;
    unsigned char *own = bufs[rank];
    if (threadIdx.x == 0) {
        s_epoch = *reinterpret_cast<volatile unsigned *>(own);
        s_abort = 0;
    }
    __syncthreads();
    const unsigned next = s_epoch + 1u;
    const int par = (int)(s_epoch & 1u);
    const int64_t per = (n + gridDim.x - 1) / gridDim.x;
    const int64_t lo = (int64_t)blockIdx.x * per, hi = lo + per < n ? lo + per : n;
    // each value travels with its call's flag in one 8-byte store (low word:
    // the f32 bits, high word: epoch + 1), so no fence or separate flag
    const int64_t slot_me = ((int64_t)par * world + rank) * n;
    for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        const uint64_t w = (uint64_t)__float_as_uint(load_in(x, x_dtype, i)) | ((uint64_t)next << 32);
        for (int p = 0; p < world; p++) st_u64_volatile(reinterpret_cast<uint64_t *>(bufs[p] + ll_off) + slot_me + i, w);
    }
    // the next kernel on the stream may launch now (it waits for this one to
    // complete before reading its output)
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const uint64_t *slots = reinterpret_cast<const uint64_t *>(own + ll_off) + (int64_t)par * world * n;
    const uint64_t t0 = ar_timer();
    for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        float v = 0.f;
        for (int r = 0; r < world && !s_abort; r++) {
            uint64_t w;
            for (uint32_t it = 0;; it++) {  // bounded wait for rank r's value of this call
                w = ld_u64_volatile(slots + (int64_t)r * n + i);
                if ((unsigned)(w >> 32) == next) break;
                if ((it & 255) == 255 && (s_abort || ar_timer() - t0 > 2000000000ull)) {
                    atomicCAS(reinterpret_cast<int *>(own + AR_ERR), 0, 7);  // a peer never signalled
                    s_abort = 1;
                    break;
                }
            }
            v += __uint_as_float((unsigned)w);
        }
        if (!s_abort) store_out(y, y_dtype, i, v);
    }
    __syncthreads();
    if (threadIdx.x == 0) {  // the last CTA out advances the epoch (every CTA has read it)
        __threadfence();
        int *cnt = reinterpret_cast<int *>(own + AR_CNT);
        if (atomicAdd(cnt, 1) == (int)gridDim.x - 1) {
            *cnt = 0;
            __threadfence();
            *reinterpret_cast<volatile unsigned *>(own) = next;
        }
    }
}

}  // namespace

int allreduce_ctas(int world, int64_t n) {
    // about 512 outputs per CTA (two per thread), at most AR_CMAX CTAs
    (void)world;
    const int64_t c = (n + 511) / 512;
    return (int)(c < AR_CMAX ? (c > 0 ? c : 1) : AR_CMAX);
}

cudaError_t launch_allreduce(const void *x, int x_dtype, void *y, int y_dtype, int64_t n, int64_t buf_n, int world,
                             int rank, unsigned char *const *bufs, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)allreduce_ctas(world, n));
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, allreduce_kernel, x, x_dtype, y, y_dtype, n, world, rank, bufs,
                              (int64_t)ar_ll_offset(world, buf_n));
}

}  // namespace kq
