// kq_noalloc.cu -- kq_quantized_matmul_noalloc: the decode/prefill matmul for
// callers that cannot allocate device memory.
//
// Some callers cannot call cudaMalloc (or any allocating library routine):
// code running inside a host framework whose allocator owns all device
// memory, plugins loaded into a process that forbids new allocations after
// start-up, or real-time paths where an allocation could block or fail.  They
// still need the split-K scratch (f32 partial tiles, tile counters, an error
// word) that kq_quantized_matmul takes as a caller-provided workspace.  This
// entry point uses instead a fixed scratch array that lives in this library's
// own device memory: KQ_NOALLOC_SCRATCH_BYTES per GPU that loads the library,
// held until the process exits.
//
// Rules for callers:
//  * The first call on a device looks up the array's device address (once per
//    device, with that device current); make that first call before any
//    stream capture.
//  * Every call shares the one array, and each call clears the parts that
//    must start at zero.  Calls whose GPU work overlaps (different streams,
//    or different host threads on one device) race on the array; serialise
//    them on one stream.
//  * Shapes whose scratch would exceed the array are rejected with
//    KQ_ERR_WORKSPACE and a message; nothing is allocated in any case.
//  * A kernel whose bounded device wait ran out records a code in the
//    array's first word; kq_noalloc_error reads it.  The next call clears it,
//    so read it before that call.
//  * The cached device address is not valid across cudaDeviceReset (the
//    module may come back at another address): do not use this entry point
//    after resetting a device it has run on.
#include <cuda_runtime.h>
#include <stdio.h>

#include <atomic>

#include "../../include/kq_cuda.h"
#include "kq_internal.cuh"

// The scratch.  In host code `g_noalloc_scratch` names a host-side stand-in,
// not device memory: only the address obtained from cudaGetSymbolAddress may
// be handed to kernels.
static __device__ __align__(256) unsigned char g_noalloc_scratch[KQ_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;
// per-device address of the array; atomic so host threads making their first
// calls at the same time agree (both look up the same address)
std::atomic<void *> g_dev_ptr[kMaxDevices];
thread_local char g_noalloc_msg[256];

// failures are reported through kq_last_error() like every other entry point
int noalloc_fail(int code) {
    kq::set_last_error(g_noalloc_msg);
    return code;
}

// The array's device address on `dev` (the current device), looked up once.
int scratch_of(int dev, void **out, const char *what) {
    void *p = g_dev_ptr[dev].load(std::memory_order_acquire);
    if (!p) {
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            snprintf(g_noalloc_msg, sizeof(g_noalloc_msg), "%s: cudaGetSymbolAddress failed: %s", what,
                     cudaGetErrorString(e));
            return 1;
        }
        g_dev_ptr[dev].store(p, std::memory_order_release);
    }
    *out = p;
    return 0;
}

}  // namespace

extern "C" {

int kq_quantized_matmul_noalloc(int codec, const void *x, int x_dtype, int64_t m, int64_t k, int64_t x_row_stride,
                                const void *w, int64_t n, int64_t w_row_stride, void *y, int y_dtype,
                                int64_t y_row_stride, void *stream) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    {
        snprintf(g_noalloc_msg, sizeof(g_noalloc_msg), "quantized_matmul_noalloc: no usable current CUDA device");
        return noalloc_fail(KQ_ERR_CUDA);
    }
    void *scratch = nullptr;
    if (scratch_of(dev, &scratch, "quantized_matmul_noalloc")) return noalloc_fail(KQ_ERR_CUDA);
    // the scratch of the path this call will take (GEMV or GEMM, chosen from
    // the activations' dtype and row stride as kq_quantized_matmul does)
    const size_t need = kq::dense_matmul_workspace_bytes(codec, m, n, k, x_dtype, x_row_stride);
    if (need > (size_t)KQ_NOALLOC_SCRATCH_BYTES) {
        snprintf(g_noalloc_msg, sizeof(g_noalloc_msg),
                 "quantized_matmul_noalloc: this shape needs %zu bytes of scratch, above the fixed %d-byte "
                 "array; use kq_quantized_matmul with a workspace",
                 need, (int)KQ_NOALLOC_SCRATCH_BYTES);
        return noalloc_fail(KQ_ERR_WORKSPACE);
    }
    // the previous call's counters and error word are not trusted: start from zero
    const cudaError_t ce = cudaMemsetAsync(scratch, 0, need, (cudaStream_t)stream);
    if (ce != cudaSuccess) {
        snprintf(g_noalloc_msg, sizeof(g_noalloc_msg), "quantized_matmul_noalloc: clearing scratch: %s",
                 cudaGetErrorString(ce));
        return noalloc_fail(KQ_ERR_CUDA);
    }
    return kq_quantized_matmul(codec, x, x_dtype, m, k, x_row_stride, w, n, w_row_stride, y, y_dtype, y_row_stride,
                               scratch, (size_t)KQ_NOALLOC_SCRATCH_BYTES, stream);
}

// The device error word of the array on the current device: 0, or the code a
// kernel of the last kq_quantized_matmul_noalloc call recorded when one of
// its bounded waits ran out (that call's output is then incomplete).
// Synchronises `stream`; clear != 0 resets the word.  Negative on failure.
int kq_noalloc_error(int clear, void *stream) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -1;
    void *scratch = nullptr;
    if (scratch_of(dev, &scratch, "noalloc_error")) return -1;
    return kq_workspace_error(scratch, clear, stream);
}

}  // extern "C"
