// kq_torch.cpp -- native fast path of the decode-time kq ops for torch tensors.
//
// kq.quantized_matmul / kq.quantized_glu are called once per projection per
// token; going through Python argument handling and ctypes costs ~15-20 us a
// call on the host, more than a decode GEMV takes on the GPU, so an eager
// decode loop would be host-bound.  This extension does the same work -- shape
// and layout checks, output allocation, the per-(device, stream) workspace,
// the libkq_cuda C-ABI call on torch's current stream -- in one native call.
//
// It only takes the common well-formed case (2-D wire weights with whole
// 256-weight groups, bf16/f16 activations whose rows are 16-byte aligned);
// for anything else, or when the C call reports an error, it returns None and
// the Python op runs its full path, which raises the reference's exception
// types.  The C entry points come in as addresses of the already-loaded
// libkq_cuda.so (set_entry_points), so this module has no link-time
// dependency on it.  The workspace registry here is the one the Python layer
// uses too (workspace()), so kq.workspace_error() sees every call's error word.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/extension.h>

#include <cstdint>
#include <map>
#include <mutex>
#include <tuple>

namespace {

using MatmulFn = int (*)(int, const void *, int, int64_t, int64_t, int64_t, const void *, int64_t, int64_t, void *,
                         int, int64_t, void *, size_t, void *);
using GluFn = int (*)(int, const void *, int, int64_t, int64_t, int64_t, const void *, const void *, int64_t, int64_t,
                      int, void *, int, int64_t, void *, size_t, void *);
using WsFn = size_t (*)(int, int64_t, int64_t, int64_t);

MatmulFn g_matmul = nullptr;
GluFn g_glu = nullptr;
WsFn g_matmul_ws = nullptr, g_glu_ws = nullptr;

std::mutex g_mu;
std::map<std::pair<int, int64_t>, at::Tensor> g_ws;                    // (device, stream) -> workspace
std::map<std::tuple<int, int, int64_t, int64_t, int64_t>, size_t> g_ws_bytes;  // (op, codec, m, n, k) -> bytes

int dtype_code(at::ScalarType t) {
    return t == at::kFloat ? 0 : t == at::kHalf ? 1 : t == at::kBFloat16 ? 2 : -1;
}

void set_entry_points(int64_t matmul, int64_t glu, int64_t matmul_ws, int64_t glu_ws) {
    g_matmul = reinterpret_cast<MatmulFn>(matmul);
    g_glu = reinterpret_cast<GluFn>(glu);
    g_matmul_ws = reinterpret_cast<WsFn>(matmul_ws);
    g_glu_ws = reinterpret_cast<WsFn>(glu_ws);
}

// The zero-filled workspace of (device, stream), grown to at least nbytes
// (at least 1 MiB); the library leaves every workspace zero after each call.
at::Tensor workspace(int64_t device, int64_t stream, int64_t nbytes) {
    std::lock_guard<std::mutex> lk(g_mu);
    auto key = std::make_pair((int)device, stream);
    auto it = g_ws.find(key);
    if (it != g_ws.end() && it->second.numel() >= nbytes) return it->second;
    if (nbytes <= 0 && it != g_ws.end()) return it->second;
    const int64_t sz = nbytes > (1 << 20) ? nbytes : (1 << 20);
    at::Tensor t = at::zeros({sz}, at::TensorOptions().dtype(at::kByte).device(at::kCUDA, (int)device));
    g_ws[key] = t;
    return t;
}

// The existing workspace of (device, stream), or an undefined tensor.
at::Tensor workspace_peek(int64_t device, int64_t stream) {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_ws.find(std::make_pair((int)device, stream));
    return it == g_ws.end() ? at::Tensor() : it->second;
}

size_t ws_bytes(int op, int codec, int64_t m, int64_t n, int64_t k) {
    const auto key = std::make_tuple(op, codec, m, n, k);
    {
        std::lock_guard<std::mutex> lk(g_mu);
        auto it = g_ws_bytes.find(key);
        if (it != g_ws_bytes.end()) return it->second;
    }
    const size_t v = op == 0 ? g_matmul_ws(codec, m, n, k) : g_glu_ws(codec, m, n, k);
    std::lock_guard<std::mutex> lk(g_mu);
    g_ws_bytes[key] = v;
    return v;
}

// The checks both ops share; false sends the call down the Python path.
bool common(const at::Tensor &x, const at::Tensor &w, int64_t bpb, int64_t &k, int64_t &wstride) {
    if (!x.is_cuda() || !w.is_cuda() || w.scalar_type() != at::kByte || w.dim() != 2 || x.dim() < 1) return false;
    if (dtype_code(x.scalar_type()) < 1 || w.stride(1) != 1 || bpb <= 0) return false;
    const int64_t rb = w.size(1);
    if (rb % bpb) return false;
    k = rb / bpb * 256;
    if (x.size(-1) != k || w.size(0) < 1) return false;
    wstride = w.size(0) > 1 ? w.stride(0) : rb;
    return true;
}

bool act_rows(const at::Tensor &x, int64_t k, at::Tensor &x2) {
    x2 = x.reshape({-1, k});
    if (x2.stride(1) != 1 || x2.stride(0) % 8 || (reinterpret_cast<uintptr_t>(x2.data_ptr()) & 15)) x2 = x2.contiguous();
    return true;
}

at::Tensor shaped(const at::Tensor &y, const at::Tensor &x, int64_t n) {
    auto sizes = x.sizes().vec();
    sizes.back() = n;
    return y.view(sizes);
}

// kq.quantized_matmul(x, w, None, codec) for 2-D wire weights; out_code < 0:
// the activation dtype.  None: take the Python path.
py::object quantized_matmul(const at::Tensor &x, const at::Tensor &w, int64_t codec, int64_t bpb, int64_t out_code) {
    int64_t k, wstride;
    if (!g_matmul || !common(x, w, bpb, k, wstride)) return py::none();
    at::Tensor x2;
    act_rows(x, k, x2);
    const int64_t m = x2.size(0), n = w.size(0);
    const at::ScalarType od = out_code == 0 ? at::kFloat : out_code == 1 ? at::kHalf : out_code == 2 ? at::kBFloat16
                                                                                                  : x.scalar_type();
    at::Tensor y = at::empty({m, n}, x.options().dtype(od));
    if (m) {
        const int dev = x.get_device();
        cudaStream_t st = at::cuda::getCurrentCUDAStream(dev).stream();
        at::Tensor ws = workspace(dev, reinterpret_cast<int64_t>(st), (int64_t)ws_bytes(0, (int)codec, m, n, k));
        const int rc = g_matmul((int)codec, x2.data_ptr(), dtype_code(x2.scalar_type()), m, k, x2.stride(0),
                                w.data_ptr(), n, wstride, y.data_ptr(), dtype_code(od), n, ws.data_ptr(),
                                (size_t)ws.numel(), st);
        if (rc) return py::none();
    }
    return py::cast(shaped(y, x, n));
}

// kq.quantized_glu(x, gate_w, up_w, codec, act) for 2-D wire weights of one shape.
py::object quantized_glu(const at::Tensor &x, const at::Tensor &wg, const at::Tensor &wu, int64_t codec, int64_t bpb,
                         int64_t act, int64_t out_code) {
    int64_t k, wstride, k2, wstride2;
    if (!g_glu || !common(x, wg, bpb, k, wstride) || !common(x, wu, bpb, k2, wstride2)) return py::none();
    if (wg.sizes() != wu.sizes() || wstride != wstride2) return py::none();
    at::Tensor x2;
    act_rows(x, k, x2);
    const int64_t m = x2.size(0), n = wg.size(0);
    const at::ScalarType od = out_code == 0 ? at::kFloat : out_code == 1 ? at::kHalf : out_code == 2 ? at::kBFloat16
                                                                                                  : x.scalar_type();
    at::Tensor y = at::empty({m, n}, x.options().dtype(od));
    if (m) {
        const int dev = x.get_device();
        cudaStream_t st = at::cuda::getCurrentCUDAStream(dev).stream();
        at::Tensor ws = workspace(dev, reinterpret_cast<int64_t>(st), (int64_t)ws_bytes(1, (int)codec, m, n, k));
        const int rc = g_glu((int)codec, x2.data_ptr(), dtype_code(x2.scalar_type()), m, k, x2.stride(0), wg.data_ptr(),
                             wu.data_ptr(), n, wstride, (int)act, y.data_ptr(), dtype_code(od), n, ws.data_ptr(),
                             (size_t)ws.numel(), st);
        if (rc) return py::none();
    }
    return py::cast(shaped(y, x, n));
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    m.def("set_entry_points", &set_entry_points);
    m.def("workspace", &workspace);
    m.def("workspace_peek", &workspace_peek);
    m.def("quantized_matmul", &quantized_matmul);
    m.def("quantized_glu", &quantized_glu);
}
