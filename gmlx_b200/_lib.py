"""ctypes binding of ``libkq_cuda.so`` (declared in ``include/kq_cuda.h``).

The shared object is built in-tree by ``gmlx_b200/build.py`` (``__graft_entry__
.build()``).  There is no fallback: if the library is missing or fails to load,
every op raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libkq_cuda.so")

KQ_OK, KQ_ERR_CODEC, KQ_ERR_SHAPE, KQ_ERR_ALIGN, KQ_ERR_DTYPE, KQ_ERR_CUDA, KQ_ERR_WORKSPACE = range(7)
KQ_F32, KQ_F16, KQ_BF16 = 0, 1, 2
ACTS = {"none": 0, "silu": 1, "gelu": 2, "gelu_approx": 3, "gelu_tanh": 3}

class ChainProblem(ctypes.Structure):
    """struct kq_chain_problem (include/kq_cuda.h)."""
    _fields_ = [("codec", ctypes.c_int), ("x", ctypes.c_void_p), ("w", ctypes.c_void_p), ("w2", ctypes.c_void_p),
                ("n", ctypes.c_int64), ("k", ctypes.c_int64), ("w_row_stride", ctypes.c_int64), ("act", ctypes.c_int),
                ("y", ctypes.c_void_p), ("y_dtype", ctypes.c_int), ("bias", ctypes.c_void_p),
                ("bias_dtype", ctypes.c_int), ("depends_on", ctypes.c_int)]


KQ_CHAIN_MAX = 8

# Every symbol include/kq_cuda.h declares, with its ctypes signature.
_vp, _i32, _i64, _sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t
SIGNATURES = {
    "kq_version": (_i32, []),
    "kq_last_error": (ctypes.c_char_p, []),
    "kq_codecs": (_i32, [_vp, _i32]),
    "kq_codec_has_matmul": (_i32, [_i32]),
    "kq_block_bytes": (_i32, [_i32]),
    "kq_dequantize": (_i32, [_i32, _vp, _i64, _i64, _i64, _vp, _i32, _vp]),
    "kq_quantized_matmul": (_i32, [_i32, _vp, _i32, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i32, _i64, _vp, _sz, _vp]),
    "kq_quantized_matmul_workspace_size": (_sz, [_i32, _i64, _i64, _i64]),
    "kq_quantized_glu": (_i32, [_i32, _vp, _i32, _i64, _i64, _i64, _vp, _vp, _i64, _i64, _i32, _vp, _i32, _i64, _vp,
                                _sz, _vp]),
    "kq_quantized_glu_workspace_size": (_sz, [_i32, _i64, _i64, _i64]),
    "kq_moe_router_topk": (_i32, [_vp, _i64, _i64, _i32, _i32, _vp, _vp, _vp]),
    "kq_moe_router_topk_ex": (_i32, [_vp, _i64, _i64, _i32, _i32, _i32, _vp, _vp, _vp, _vp]),
    "kq_moe_glu_gather": (_i32, [_i32, _vp, _i32, _i64, _i64, _vp, _i32, _vp, _vp, _i64, _i64, _i64, _i64, _i32, _vp,
                                 _i32, _vp, _sz, _vp]),
    "kq_gather_qmv": (_i32, [_i32, _vp, _i32, _i64, _i32, _i64, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _i32, _vp, _sz,
                             _vp]),
    "kq_gather_qmv_mix": (_i32, [_i32, _vp, _i32, _i64, _i32, _i64, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _i32,
                                 _vp, _sz, _vp]),
    "kq_gather_qmm": (_i32, [_i32, _vp, _i32, _i64, _i64, _i64, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _i32, _vp,
                             _sz, _vp]),
    "kq_moe_workspace_size": (_sz, [_i32, _i64, _i64, _i64, _i64]),
    "kq_workspace_error": (_i32, [_vp, _i32, _vp]),
    "kq_moe_expert_layer_local": (_i32, [_i32, _i32, _vp, _i32, _i64, _i64, _vp, _i32, _vp, _vp, _vp, _i64, _i64, _vp,
                                         _i64, _i64, _i64, _i64, _i64, _i64, _i32, _vp, _i32, _vp, _sz, _vp]),
    "kq_moe_expert_layer_workspace_size": (_sz, [_i32, _i32, _i64, _i32, _i64, _i64, _i64, _i32]),
    "kq_quantized_matmul_noalloc": (_i32, [_i32, _vp, _i32, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i32, _i64, _vp]),
    "kq_noalloc_error": (_i32, [_i32, _vp]),
    "kq_quantized_matmul_chain_workspace_size": (_sz, [_vp, _i32]),
    "kq_quantized_matmul_chain": (_i32, [_vp, _i32, _i32, _vp, _sz, _vp]),
    "kq_quantized_matmul_bias": (_i32, [_i32, _vp, _i32, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i32, _vp, _i32, _i64,
                                        _vp, _sz, _vp]),
    "kq_allreduce_buffer_bytes": (_sz, [_i32, _i64]),
    "kq_quantized_matmul_allreduce": (_i32, [_i32, _vp, _i32, _i64, _vp, _i64, _i64, _vp, _i32, _i32, _i32, _vp, _vp,
                                             _sz, _vp]),
    "kq_allreduce": (_i32, [_vp, _i32, _vp, _i32, _i64, _i64, _i32, _i32, _vp, _vp]),
    "kq_comm_error": (_i32, [_vp, _i32, _vp]),
    "kq_comm_alloc": (_i32, [_sz, _vp]),
    "kq_comm_free": (_i32, [_vp]),
    "kq_ipc_handle": (_i32, [_vp, _vp]),
    "kq_ipc_open": (_i32, [_vp, _vp]),
    "kq_ipc_close": (_i32, [_vp]),
}

_lib = None
_lock = threading.Lock()


class KQError(RuntimeError):
    """A libkq_cuda call returned a non-zero status."""

    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


def load():
    """Load the library (once); raises if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"libkq_cuda.so not found at {LIB_PATH}; build it with `python -m gmlx_b200.build` "
                    "(there is no CPU fallback)")
            L = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def check(rc: int, what: str = "") -> None:
    if rc != KQ_OK:
        msg = load().kq_last_error().decode(errors="replace")
        if rc == KQ_ERR_CODEC:
            raise NotImplementedError(msg or what)
        if rc in (KQ_ERR_SHAPE, KQ_ERR_DTYPE, KQ_ERR_ALIGN):
            raise ValueError(msg or what)
        raise KQError(rc, msg or what)
