"""The ``mlx_kquant`` op surface that gmlx calls, on B200.

gmlx reaches its quantized kernels as ``import mlx_kquant as kq``
(gmlx/modules.py:35-40).  This module offers the same names, argument meaning
and error behaviour over torch CUDA tensors, each backed by one entry point of
``libkq_cuda.so`` (``include/kq_cuda.h``):

=========================  =============================================
kq op                      gmlx call sites
=========================  =============================================
``dequantize``             modules.py:1461, loader.py:3046-3048
``quantized_matmul``       KQuantLinear (modules.py:1535-1539),
                           occupancy_fuse.py:284-287, 412-418, 434-437
``gather_qmm``             KQuantSwitchLinear (modules.py:1548-1552),
                           sorted prefill path modules.py:1308-1309
``moe_glu_gather_kq``      modules.py:585-588, 980-983
``gather_qmv_kq``          modules.py:596-598
``gather_qmv_mix_ns_kq``   modules.py:591-593, 989-991
``moe_router_topk``        modules.py:446-447, 751-752
``codecs`` /               preflight.py:625-632, _FusedMoeCaps
``codec_has_matmul``       (modules.py:155-234)
=========================  =============================================

Weights are uint8 wire-byte tensors ``[N, K/256*bpb]`` (or ``[E, N, ...]``),
never repacked; ``scales`` is the reference's ``(1,)`` placeholder and is
ignored.  Outputs are fresh tensors in the activation dtype.  Unknown codecs
raise ``NotImplementedError``; bad shapes ``ValueError``.  All work is enqueued
on the current torch CUDA stream.
"""
from __future__ import annotations

import ctypes as _ct

import torch

from . import _lib
from .synth import BLOCK_BYTES, CODECS, QK, SUB_BLOCK, codec_id

__all__ = [
    "codecs", "all_codecs", "codec_has_matmul", "codec_has_moe_glu", "block_bytes", "dequantize", "quantized_matmul", "quantized_glu", "gather_qmm",
    "moe_glu_gather_kq", "gather_qmv_kq", "gather_qmv_mix_ns_kq", "moe_router_topk", "workspace_error",
    "moe_expert_layer_local", "quantized_matmul_chain", "quantized_matmul_allreduce", "quantized_matmul_qmv_bias", "moe_glu_gather_shexp_kq", "gather_qmv_mix_kq",
]

_DT = {torch.float32: _lib.KQ_F32, torch.float16: _lib.KQ_F16, torch.bfloat16: _lib.KQ_BF16}
_TORCH_DT = {v: k for k, v in _DT.items()}


# The codec names gmlx's loader whitelists (gmlx/preflight.py:23-30); the
# reference's own check compares kq.codecs() with this set for EQUALITY
# (tests/test_preflight.py:96-99), so the ternary TQ1_0 / TQ2_0 codecs, which
# have kernels here but are not on gmlx's list, are reported by all_codecs().
GMLX_CODECS = ("q2_k", "q3_k", "q4_k", "q5_k", "q6_k", "q4_0", "q4_1", "q5_0", "q5_1", "q8_0", "iq4_nl",
               "iq4_xs", "iq3_s", "iq3_xxs", "iq2_xxs", "iq2_xs", "iq2_s", "iq1_s", "iq1_m", "mxfp4", "nvfp4")


def all_codecs() -> list[str]:
    """Every codec name with kernels in libkq_cuda.so (the C ABI's
    kq_codecs list, sized from its own count)."""
    L = _lib.load()
    n = L.kq_codecs(None, 0)
    buf = (_ct.c_int * max(n, 1))()
    n = L.kq_codecs(buf, n)
    names = {v: k for k, v in CODECS.items()}
    return [names[buf[i]] for i in range(n)]


def codecs() -> list[str]:
    """Codec names the loader may serve (gmlx gates loading on
    ``set(kq.codecs())``, modules.py:1442, :1524, loader.py:2798-2801): the
    21 codecs of gmlx's list, every one backed by kernels here."""
    have = set(all_codecs())
    return [c for c in GMLX_CODECS if c in have]


def codec_has_matmul(codec) -> bool:
    try:
        c = codec_id(codec)
    except ValueError:
        return False
    return bool(_lib.load().kq_codec_has_matmul(c))


def codec_has_moe_glu(codec) -> bool:
    """Whether the fused MoE ops (``moe_glu_gather_kq`` and the down/mix
    gathers) take ``codec``: gmlx's fused-MoE capability probe asks this for
    the native-fp codecs (modules.py:177-181).  Every codec with kernels here
    qualifies (decode groups of one slot or the grouped tensor-core GEMM)."""
    return codec_has_matmul(codec)


def block_bytes(codec) -> int:
    return BLOCK_BYTES[codec_id(codec)]


def _cid(codec) -> int:
    try:
        c = codec_id(codec)
    except ValueError as e:
        raise NotImplementedError(f"[gmlx_b200.kq] unsupported codec {codec!r}") from e
    if c not in BLOCK_BYTES:
        raise NotImplementedError(f"[gmlx_b200.kq] unsupported codec {codec!r}")
    return c


def _stream(dev: torch.device) -> int:
    # plain ints: the ctypes signatures declare c_void_p and convert them
    return torch.cuda.current_stream(dev).cuda_stream


def _p(t: torch.Tensor | None) -> int:
    return t.data_ptr() if t is not None else 0


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("[gmlx_b200.kq] tensors must be CUDA tensors (there is no CPU implementation)")


def _wire_k(w: torch.Tensor, c: int) -> int:
    bpb = BLOCK_BYTES[c]
    if w.dtype != torch.uint8:
        raise ValueError(f"wire weights must be uint8, got {w.dtype}")
    if w.shape[-1] % bpb == 0:
        return w.shape[-1] // bpb * QK
    if c in SUB_BLOCK and w.shape[-1] % SUB_BLOCK[c][1] == 0:  # a partial last 256-weight group
        bw, bb = SUB_BLOCK[c]
        return w.shape[-1] // bb * bw
    raise ValueError(f"wire row of {w.shape[-1]} bytes is not a whole number of {bpb}-byte blocks")


def _rows2d(w: torch.Tensor) -> tuple[torch.Tensor, int]:
    """View w [..., R, bytes] with unit byte stride; return (w, row stride bytes)."""
    if w.stride(-1) != 1:
        w = w.contiguous()
    if w.dim() >= 2 and w.shape[-2] > 1:
        return w, w.stride(-2)
    return w, w.shape[-1]


# --------------------------------------------------------------------------
# per-(device, stream) workspaces, zero-filled once and kept zero by the library

_WS: dict[tuple[int, int], torch.Tensor] = {}


_WS_SIZE: dict[tuple, int] = {}


def _ws_size(fn_name: str, *args) -> int:
    """Workspace size query, memoized (a pure function of its arguments)."""
    key = (fn_name,) + args
    v = _WS_SIZE.get(key)
    if v is None:
        v = getattr(_lib.load(), fn_name)(*args)
        _WS_SIZE[key] = v
    return v


_EXT = None  # the native fast path (gmlx_b200/_ext/kq_torch.so) once loaded; False: not built


def _ext():
    """The torch C++ extension of the decode ops, bound to this process's
    libkq_cuda entry points; None if it was not built."""
    global _EXT
    if _EXT is None:
        from . import build as _build
        e = _build.load_torch_ext()
        if e is not None:
            L = _lib.load()
            addr = lambda f: _ct.cast(f, _ct.c_void_p).value  # noqa: E731
            e.set_entry_points(addr(L.kq_quantized_matmul), addr(L.kq_quantized_glu),
                               addr(L.kq_quantized_matmul_workspace_size), addr(L.kq_quantized_glu_workspace_size))
        _EXT = e if e is not None else False
    return _EXT or None


_FAST_CODEC: dict = {}  # codec argument -> (codec id, block bytes)


def _fast_codec(codec):
    v = _FAST_CODEC.get(codec)
    if v is None:
        c = _cid(codec)
        v = (c, BLOCK_BYTES[c])
        _FAST_CODEC[codec] = v
    return v


def _workspace(dev: torch.device, nbytes: int) -> torch.Tensor:
    key = (dev.index if dev.index is not None else torch.cuda.current_device(),
           torch.cuda.current_stream(dev).cuda_stream)
    e = _ext()
    if e is not None:  # one registry for both paths
        return e.workspace(key[0], key[1], nbytes)
    ws = _WS.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=dev)
        _WS[key] = ws
    return ws


def workspace_error(device=None, clear: bool = True) -> int:
    """Device-side error word of the current stream's workspace (syncs)."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    key = (dev.index, torch.cuda.current_stream(dev).cuda_stream)
    e = _ext()
    ws = e.workspace_peek(key[0], key[1]) if e is not None else _WS.get(key)
    if ws is None:  # (an undefined tensor from the extension arrives as None)
        return 0
    return _lib.load().kq_workspace_error(_p(ws), int(clear), _stream(dev))


# --------------------------------------------------------------------------
# ops


def dequantize(w: torch.Tensor, scales=None, codec=None, dtype: torch.dtype = torch.float32,
               biases=None) -> torch.Tensor:
    """``kq.dequantize``: wire ``[..., nb*bpb]`` -> ``[..., nb*256]`` in ``dtype``."""
    c = _cid(codec)
    _need_cuda(w)
    if dtype not in _DT:
        raise ValueError(f"unsupported dequantize dtype {dtype}")
    k = _wire_k(w, c)
    w = w.contiguous()
    rows = w.numel() // w.shape[-1] if w.numel() else 0
    out = torch.empty(*w.shape[:-1], k, dtype=dtype, device=w.device)
    if rows == 0:
        return out
    L = _lib.load()
    _lib.check(L.kq_dequantize(c, _p(w), rows, k, w.shape[-1], _p(out), _DT[dtype], _stream(w.device)), "dequantize")
    return out


def _act_2d(x: torch.Tensor, k: int) -> torch.Tensor:
    if x.shape[-1] != k:
        raise ValueError(f"activation K={x.shape[-1]} does not match weight K={k}")
    if x.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError(f"activations must be bf16 or fp16, got {x.dtype}")
    x2 = x.reshape(-1, k)
    if x2.stride(-1) != 1 or x2.stride(0) % 8 or x2.data_ptr() % 16:
        x2 = x2.contiguous()
    return x2


def quantized_matmul(x: torch.Tensor, w: torch.Tensor, scales=None, codec=None, transpose: bool = True,
                     out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """``kq.quantized_matmul(x, w, scales, codec, transpose=True)``: ``x @ dequant(w).T``."""
    if transpose and w.dim() == 2 and (out_dtype is None or out_dtype in _DT):
        e = _ext()
        if e is not None:  # native fast path; None: the full path below (and its errors)
            c, bpb = _fast_codec(codec)
            y = e.quantized_matmul(x, w, c, bpb, -1 if out_dtype is None else _DT[out_dtype])
            if y is not None:
                return y
    if not transpose:
        raise NotImplementedError("kq.quantized_matmul: only transpose=True (wire rows are outputs)")
    c = _cid(codec)
    _need_cuda(x, w)
    k = _wire_k(w, c)
    w, wstride = _rows2d(w)
    n = w.shape[-2] if w.dim() >= 2 else 1
    x2 = _act_2d(x, k)
    m = x2.shape[0]
    od = out_dtype or x.dtype
    y = torch.empty(m, n, dtype=od, device=x.device)
    if m:
        L = _lib.load()
        ws = _workspace(x.device, _ws_size("kq_quantized_matmul_workspace_size", c, m, n, k))
        _lib.check(L.kq_quantized_matmul(c, _p(x2), _DT[x2.dtype], m, k, x2.stride(0), _p(w), n, wstride, _p(y),
                                         _DT[od], n, _p(ws), ws.numel(), _stream(x.device)), "quantized_matmul")
    return y.reshape(*x.shape[:-1], n)


def quantized_matmul_qmv_bias(x: torch.Tensor, w: torch.Tensor, scales, bias: torch.Tensor, codec=None,
                              out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """``kq.quantized_matmul_qmv_bias(x, w, scales, bias, codec)``: ``x @ dequant(w).T + bias``
    in one dispatch (gmlx/qkv_fuse.py:80)."""
    c = _cid(codec)
    _need_cuda(x, w, bias)
    k = _wire_k(w, c)
    w, wstride = _rows2d(w)
    n = w.shape[-2] if w.dim() >= 2 else 1
    b = bias.reshape(-1).contiguous()
    if b.numel() != n or b.dtype not in _DT:
        raise ValueError(f"bias must have {n} f32/f16/bf16 entries")
    x2 = _act_2d(x, k)
    m = x2.shape[0]
    od = out_dtype or x.dtype
    y = torch.empty(m, n, dtype=od, device=x.device)
    if m:
        L = _lib.load()
        ws = _workspace(x.device, _ws_size("kq_quantized_matmul_workspace_size", c, m, n, k))
        _lib.check(L.kq_quantized_matmul_bias(c, _p(x2), _DT[x2.dtype], m, k, x2.stride(0), _p(w), n, wstride, _p(b),
                                              _DT[b.dtype], _p(y), _DT[od], n, _p(ws), ws.numel(), _stream(x.device)),
                   "quantized_matmul_qmv_bias")
    return y.reshape(*x.shape[:-1], n)


def quantized_matmul_allreduce(x: torch.Tensor, w: torch.Tensor, codec, comm,
                               out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """Row-parallel decode projection with the cross-rank sum fused in: this
    rank's ``x @ dequant(w_shard).T`` for one activation row, summed over the
    ranks of ``comm`` (a ``gmlx_b200.parallel.PeerComm``) inside the kernel.
    Every rank gets the same bits.  Stands for ``quantized_matmul`` on a K
    shard followed by ``all_sum`` (gmlx/hy_v3_model.py:259)."""
    c = _cid(codec)
    _need_cuda(x, w)
    k = _wire_k(w, c)
    w, wstride = _rows2d(w)
    n = w.shape[-2]
    x2 = _act_2d(x, k)
    if x2.shape[0] != 1:
        raise ValueError("quantized_matmul_allreduce: one activation row (decode)")
    if n > comm.n:
        raise ValueError(f"quantized_matmul_allreduce: {n} outputs exceed the communication buffer ({comm.n})")
    od = out_dtype or x.dtype
    y = torch.empty(1, n, dtype=od, device=x.device)
    L = _lib.load()
    ws = _workspace(x.device, _ws_size("kq_quantized_matmul_workspace_size", c, 1, n, k))
    _lib.check(L.kq_quantized_matmul_allreduce(c, _p(x2), _DT[x2.dtype], k, _p(w), n, wstride, _p(y), _DT[od],
                                               comm.world, comm.rank, _p(comm.table), _p(ws), ws.numel(),
                                               _stream(x.device)), "quantized_matmul_allreduce")
    return y.reshape(*x.shape[:-1], n)


def all_reduce(x: torch.Tensor, comm, out: torch.Tensor | None = None) -> torch.Tensor:
    """Sum of ``x`` over the ranks of ``comm`` (a ``gmlx_b200.parallel.PeerComm``)
    in one launch: one-shot push of {value, flag} words over NVLink peer
    memory, f32 rank-order sum,
    the same bits on every rank.  For the short vectors of decode (the all_sum
    after a row-parallel projection, gmlx/hy_v3_model.py:259).  ``out``
    defaults to ``x`` (in place)."""
    _need_cuda(x)
    if not x.is_contiguous():
        raise ValueError("all_reduce: contiguous tensor expected")
    if x.dtype not in _DT:
        raise TypeError(f"all_reduce: unsupported dtype {x.dtype}")
    n = x.numel()
    if n > comm.n:
        raise ValueError(f"all_reduce: {n} values exceed the communication buffer ({comm.n})")
    y = x if out is None else out
    if y.shape != x.shape or not y.is_contiguous() or y.dtype not in _DT:
        raise ValueError("all_reduce: out must be a contiguous tensor of x's shape")
    L = _lib.load()
    _lib.check(L.kq_allreduce(_p(x), _DT[x.dtype], _p(y), _DT[y.dtype], n, comm.n, comm.world, comm.rank, _p(comm.table),
                              _stream(x.device)), "all_reduce")
    return y


def quantized_glu(x: torch.Tensor, gate_w: torch.Tensor, up_w: torch.Tensor, codec=None, act: str = "silu",
                  out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """Fused ``act(x @ Wg.T) * (x @ Wu.T)`` for a dense gate/up pair (one launch)."""
    if gate_w.dim() == 2 and act in _lib.ACTS and (out_dtype is None or out_dtype in _DT):
        e = _ext()
        if e is not None:  # native fast path; None: the full path below (and its errors)
            c, bpb = _fast_codec(codec)
            y = e.quantized_glu(x, gate_w, up_w, c, bpb, _lib.ACTS[act], -1 if out_dtype is None else _DT[out_dtype])
            if y is not None:
                return y
    c = _cid(codec)
    _need_cuda(x, gate_w, up_w)
    k = _wire_k(gate_w, c)
    if gate_w.shape != up_w.shape:
        raise ValueError("gate and up wire tensors must have the same shape")
    gate_w, ws_ = _rows2d(gate_w)
    up_w, ws2 = _rows2d(up_w)
    if ws_ != ws2:
        up_w = up_w.contiguous()
        gate_w = gate_w.contiguous()
        ws_ = gate_w.shape[-1]
    n = gate_w.shape[-2]
    x2 = _act_2d(x, k)
    m = x2.shape[0]
    od = out_dtype or x.dtype
    y = torch.empty(m, n, dtype=od, device=x.device)
    if m:
        L = _lib.load()
        ws = _workspace(x.device, _ws_size("kq_quantized_glu_workspace_size", c, m, n, k))
        _lib.check(L.kq_quantized_glu(c, _p(x2), _DT[x2.dtype], m, k, x2.stride(0), _p(gate_w), _p(up_w), n, ws_,
                                      _lib.ACTS[act], _p(y), _DT[od], n, _p(ws), ws.numel(), _stream(x.device)),
                   "quantized_glu")
    return y.reshape(*x.shape[:-1], n)


def _stack(w: torch.Tensor) -> tuple[torch.Tensor, int, int]:
    """Expert stack [E, N, bytes] (unit byte stride) -> (w, row stride, expert stride)."""
    if w.dim() != 3:
        raise ValueError(f"expert stack must be [E, N, bytes], got shape {tuple(w.shape)}")
    if w.stride(-1) != 1:
        w = w.contiguous()
    return w, w.stride(1), w.stride(0)


def moe_router_topk(logits: torch.Tensor, k: int, norm_topk_prob: bool = True, shared_gate: bool = True,
                    per_expert_scale: torch.Tensor | None = None):
    """``kq.moe_router_topk(logits, k, norm_topk_prob, shared_gate=True, per_expert_scale=None)``:
    softmax over the routed experts -> top-k (descending, ties to the lower id)
    -> optional renormalisation, in f32, one launch.

    shared_gate (the reference default): the last logits column is the shared
    expert's gate (gmlx/modules.py:294-313 appends it); scores gain a last
    column sigmoid(gate), idx stays [..., k].  shared_gate=False: every column
    is a routed expert (gmlx/modules.py:446-447).  per_expert_scale [E]
    multiplies each picked score (gmlx/modules.py:1043-1046)."""
    _need_cuda(logits)
    lg = logits.reshape(-1, logits.shape[-1]).float().contiguous()
    t, cols = lg.shape
    e = cols - 1 if shared_gate else cols
    pes = None
    if per_expert_scale is not None:
        pes = per_expert_scale.reshape(-1).float().contiguous()
        if pes.numel() != e:
            raise ValueError(f"moe_router_topk: per_expert_scale has {pes.numel()} entries for {e} experts")
    idx = torch.empty(t, k, dtype=torch.int32, device=lg.device)
    sk = k + 1 if shared_gate else k
    sc = torch.empty(t, sk, dtype=torch.float32, device=lg.device)
    if t:
        _lib.check(_lib.load().kq_moe_router_topk_ex(_p(lg), t, e, k, int(bool(norm_topk_prob)), int(bool(shared_gate)),
                                                     _p(pes), _p(idx), _p(sc), _stream(lg.device)),
                   "moe_router_topk")
    return idx.reshape(*logits.shape[:-1], k), sc.reshape(*logits.shape[:-1], sk)


def _idx2d(idx: torch.Tensor, t: int) -> torch.Tensor:
    i = idx.reshape(t, -1)
    if i.dtype != torch.int32:
        i = i.to(torch.int32)
    return i.contiguous()


def moe_glu_gather_kq(x: torch.Tensor, gate_w: torch.Tensor, up_w: torch.Tensor, codec, idx: torch.Tensor,
                      act: str = "silu", out_dtype: torch.dtype | None = None, **kw) -> torch.Tensor:
    """``kq.moe_glu_gather_kq(x[T,D], Wg, Wu, codec, idx[T,k], act)`` -> ``h[T,k,F]`` (f32 epilogue)."""
    if kw:
        raise NotImplementedError(f"moe_glu_gather_kq: unsupported arguments {sorted(kw)}")
    c = _cid(codec)
    _need_cuda(x, gate_w, up_w, idx)
    d = _wire_k(gate_w, c)
    gate_w, wrs, wes = _stack(gate_w)
    up_w, wrs2, wes2 = _stack(up_w)
    if (wrs, wes) != (wrs2, wes2) or gate_w.shape != up_w.shape:
        raise ValueError("gate and up stacks must share shape and layout")
    e, f = gate_w.shape[0], gate_w.shape[1]
    x2 = _act_2d(x, d)
    t = x2.shape[0]
    i2 = _idx2d(idx, t)
    k = i2.shape[1]
    od = out_dtype or x.dtype
    h = torch.empty(t, k, f, dtype=od, device=x.device)
    if t:
        L = _lib.load()
        ws = _workspace(x.device, _ws_size("kq_moe_workspace_size", c, t * k, e, f, d))
        _lib.check(L.kq_moe_glu_gather(c, _p(x2), _DT[x2.dtype], t, d, _p(i2), k, _p(gate_w), _p(up_w), e, f, wrs,
                                       wes, _lib.ACTS[act], _p(h), _DT[od], _p(ws), ws.numel(), _stream(x.device)),
                   "moe_glu_gather_kq")
    return h


def moe_glu_gather_shexp_kq(x: torch.Tensor, gate_w: torch.Tensor, up_w: torch.Tensor, shexp_gate_w: torch.Tensor,
                            shexp_up_w: torch.Tensor, codec, idx: torch.Tensor, act: str = "silu",
                            shexp_kquant_type=None, out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """``kq.moe_glu_gather_shexp_kq`` (gmlx/modules.py:764-770): the routed GLU
    gather with the shared expert riding along as slot ``k``:
    ``h[t, :k] = moe_glu_gather_kq(...)``, ``h[t, k] = act(x Sg^T) * (x Su^T)``.
    The shared expert's codec may differ (``shexp_kquant_type``); its
    intermediate width must equal the routed experts'."""
    t = x.reshape(-1, x.shape[-1]).shape[0]
    k = idx.shape[-1]
    sc = shexp_kquant_type or codec
    f = gate_w.shape[-2]
    if shexp_gate_w.shape[-2] != f:
        raise ValueError(f"shared expert width {shexp_gate_w.shape[-2]} != routed width {f}")
    od = out_dtype or x.dtype
    h = torch.empty(t, k + 1, f, dtype=od, device=x.device)
    h[:, :k] = moe_glu_gather_kq(x, gate_w, up_w, codec, idx, act=act, out_dtype=od).reshape(t, k, f)
    h[:, k] = quantized_glu(x.reshape(t, -1), shexp_gate_w, shexp_up_w, sc, act=act, out_dtype=od)
    return h


def gather_qmv_mix_kq(h: torch.Tensor, w: torch.Tensor, shexp_w: torch.Tensor, codec, idx: torch.Tensor,
                      scores: torch.Tensor, shexp_kquant_type=None, out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """``kq.gather_qmv_mix_kq`` (gmlx/modules.py:775-779): the down projection of
    the routed slots and the shared-expert slot with the routing mix in f32:
    ``y[t] = sum_{j<k} scores[t,j] (h[t,j] W[idx[t,j]]^T) + scores[t,k] (h[t,k] S^T)``
    (``scores[:, k]`` is the sigmoid shared gate from ``moe_router_topk``)."""
    t, kp1 = h.shape[0], h.shape[1]
    k = kp1 - 1
    if idx.shape[-1] != k or scores.shape[-1] != kp1:
        raise ValueError("gather_qmv_mix_kq: h [T, k+1, F], idx [T, k], scores [T, k+1]")
    sc = shexp_kquant_type or codec
    y = gather_qmv_mix_ns_kq(h[:, :k].contiguous(), w, codec, idx, scores[:, :k].contiguous(),
                             out_dtype=torch.float32)
    ys = quantized_matmul(h[:, k].contiguous(), shexp_w, None, sc, out_dtype=torch.float32)
    y = y.reshape(t, -1) + scores[:, k:kp1].float() * ys
    return y.to(out_dtype or h.dtype)


def gather_qmv_kq(h: torch.Tensor, w: torch.Tensor, codec, idx: torch.Tensor, bias=None,
                  out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """``kq.gather_qmv_kq(h[T,k,F], W, codec, idx[T,k])`` -> ``y[T,k,N]``."""
    c = _cid(codec)
    _need_cuda(h, w, idx)
    f = _wire_k(w, c)
    w, wrs, wes = _stack(w)
    e, n = w.shape[0], w.shape[1]
    t = h.shape[0]
    i2 = _idx2d(idx, t)
    k = i2.shape[1]
    h2 = _act_2d(h.reshape(t * k, f), f)
    od = out_dtype or h.dtype
    y = torch.empty(t, k, n, dtype=od, device=h.device)
    if t:
        L = _lib.load()
        ws = _workspace(h.device, _ws_size("kq_moe_workspace_size", c, t * k, e, n, f))
        _lib.check(L.kq_gather_qmv(c, _p(h2), _DT[h2.dtype], t, k, f, _p(i2), _p(w), e, n, wrs, wes, _p(y), _DT[od],
                                   _p(ws), ws.numel(), _stream(h.device)), "gather_qmv_kq")
    if bias is not None:
        y = y + bias[idx.long()].to(y.dtype)
    return y


def gather_qmv_mix_ns_kq(h: torch.Tensor, w: torch.Tensor, codec, idx: torch.Tensor, scores: torch.Tensor,
                         out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """``kq.gather_qmv_mix_ns_kq``: ``y[t] = sum_j scores[t,j] * (h[t,j] @ W[idx[t,j]].T)`` (f32)."""
    c = _cid(codec)
    _need_cuda(h, w, idx, scores)
    f = _wire_k(w, c)
    w, wrs, wes = _stack(w)
    e, n = w.shape[0], w.shape[1]
    t = h.shape[0]
    i2 = _idx2d(idx, t)
    k = i2.shape[1]
    h2 = _act_2d(h.reshape(t * k, f), f)
    s2 = scores.reshape(t, k).float().contiguous()
    od = out_dtype or h.dtype
    y = torch.empty(t, n, dtype=od, device=h.device)
    if t:
        L = _lib.load()
        ws = _workspace(h.device, _ws_size("kq_moe_workspace_size", c, t * k, e, n, f))
        _lib.check(L.kq_gather_qmv_mix(c, _p(h2), _DT[h2.dtype], t, k, f, _p(i2), _p(s2), _p(w), e, n, wrs, wes,
                                       _p(y), _DT[od], _p(ws), ws.numel(), _stream(h.device)), "gather_qmv_mix_ns_kq")
    return y


def gather_qmm(x: torch.Tensor, w: torch.Tensor, scales=None, codec=None, lhs_indices=None, rhs_indices=None,
               transpose: bool = True, sorted_indices: bool = False,
               out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """``kq.gather_qmm`` (mlx ``gather_qmm`` semantics over wire stacks):
    ``out[b] = x[lhs[b]] @ dequant(w[rhs[b]]).T`` with ``b`` over the broadcast of
    the index shapes (``x``'s batch dims stand in for ``lhs`` when it is None)."""
    if not transpose:
        raise NotImplementedError("kq.gather_qmm: only transpose=True")
    c = _cid(codec)
    _need_cuda(x, w)
    kin = _wire_k(w, c)
    w, wrs, wes = _stack(w)
    e, n = w.shape[0], w.shape[1]
    if x.shape[-1] != kin:
        raise ValueError(f"activation K={x.shape[-1]} does not match weight K={kin}")
    m = x.shape[-2]
    xb_shape = x.shape[:-2]
    xb = torch.arange(int(torch.tensor(xb_shape).prod().item()) if len(xb_shape) else 1, device=x.device)
    xb = xb.reshape(xb_shape) if len(xb_shape) else xb.reshape(())
    if lhs_indices is not None:
        xb = xb.reshape(-1)[lhs_indices.long()]
    rhs = torch.zeros((), dtype=torch.long, device=x.device) if rhs_indices is None else rhs_indices.long()
    xb, rhs = torch.broadcast_tensors(xb, rhs)
    bshape = xb.shape
    xb, rhs = xb.reshape(-1), rhs.reshape(-1)
    ar = torch.arange(m, device=x.device)
    xrow = (xb[:, None] * m + ar[None, :]).reshape(-1).to(torch.int32).contiguous()
    expert = rhs[:, None].expand(-1, m).reshape(-1).to(torch.int32).contiguous()
    rows = xrow.numel()
    x2 = _act_2d(x.reshape(-1, kin), kin)
    od = out_dtype or x.dtype
    y = torch.empty(rows, n, dtype=od, device=x.device)
    if rows:
        L = _lib.load()
        ws = _workspace(x.device, _ws_size("kq_moe_workspace_size", c, rows, e, n, kin))
        _lib.check(L.kq_gather_qmm(c, _p(x2), _DT[x2.dtype], kin, x2.stride(0), rows, _p(xrow), _p(expert), _p(w),
                                   e, n, wrs, wes, _p(y), _DT[od], _p(ws), ws.numel(), _stream(x.device)),
                   "gather_qmm")
    return y.reshape(*bshape, m, n)


def moe_expert_layer_local(x: torch.Tensor, idx: torch.Tensor, scores: torch.Tensor, gate_w: torch.Tensor,
                           up_w: torch.Tensor, down_w: torch.Tensor, codec_gu, codec_d, expert_base: int = 0,
                           n_experts_total: int | None = None, act: str = "silu",
                           out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """One expert-parallel rank's share of the routed expert layer (decode):
    ``sum_j scores[t,j] * down(act(gate(x)) * up(x))`` over the slots routed to
    the local experts ``[expert_base, expert_base + gate_w.shape[0])``; summed
    over ranks it is the full layer (gmlx/moe_experts.py:250-266)."""
    cg, cd = _cid(codec_gu), _cid(codec_d)
    _need_cuda(x, idx, scores, gate_w, up_w, down_w)
    d = _wire_k(gate_w, cg)
    f = _wire_k(down_w, cd)
    gate_w, grs, ges = _stack(gate_w)
    up_w, urs, ues = _stack(up_w)
    down_w, drs, des = _stack(down_w)
    if (grs, ges) != (urs, ues) or gate_w.shape != up_w.shape:
        raise ValueError("gate and up stacks must share shape and layout")
    e_local = gate_w.shape[0]
    e_total = n_experts_total if n_experts_total is not None else expert_base + e_local
    x2 = _act_2d(x, d)
    t = x2.shape[0]
    i2 = _idx2d(idx, t)
    k = i2.shape[1]
    s2 = scores.reshape(t, k).float().contiguous()
    od = out_dtype or x.dtype
    y = torch.empty(t, down_w.shape[1], dtype=od, device=x.device)
    if t:
        L = _lib.load()
        ws = _workspace(x.device, _ws_size("kq_moe_expert_layer_workspace_size", cg, cd, t, k, e_local, d, f, _DT[x2.dtype]))
        _lib.check(L.kq_moe_expert_layer_local(cg, cd, _p(x2), _DT[x2.dtype], t, d, _p(i2), k, _p(s2), _p(gate_w),
                                               _p(up_w), grs, ges, _p(down_w), drs, des, e_local, f, expert_base,
                                               e_total, _lib.ACTS[act], _p(y), _DT[od], _p(ws), ws.numel(),
                                               _stream(x.device)), "moe_expert_layer_local")
    return y


def quantized_matmul_chain(problems, out_dtype: torch.dtype | None = None) -> list[torch.Tensor]:
    """A chain of one-row decode projections in one launch (the dense decode
    of one token: q|k|v, o, gate+up, down).  gmlx fuses projections that share
    an input by row-concatenation (occupancy_fuse.py:141-200, 272-330); this
    op streams every projection of the list in a single persistent kernel.

    ``problems``: up to 8 dicts with keys ``x`` (one activation row ``[k]`` or
    ``[1, k]``, or the int index of an earlier problem whose output it is),
    ``w`` (wire weights), ``codec``, optional ``w2`` + ``act`` (fused gate/up,
    as ``quantized_glu``) or ``bias`` (as ``quantized_matmul_qmv_bias``).
    Returns the outputs ``[1, n]`` in order (a problem read by a later one
    keeps the activation dtype); each equals the single-op result for that
    row within the kernels' tolerance."""
    L = _lib.load()
    n = len(problems)
    if not 1 <= n <= _lib.KQ_CHAIN_MAX:
        raise ValueError(f"quantized_matmul_chain takes 1..{_lib.KQ_CHAIN_MAX} problems, got {n}")
    arr = (_lib.ChainProblem * n)()
    outs, keep = [], []
    x_dtype, dev = None, None
    for i, pr in enumerate(problems):
        c = _cid(pr["codec"])
        w, rs = _rows2d(pr["w"])
        _need_cuda(w)
        k = _wire_k(w, c)
        x = pr["x"]
        dep = -1
        if isinstance(x, int):
            if not 0 <= x < i:
                raise ValueError(f"problem {i}: x index {x} is not an earlier problem")
            dep = x
            x = outs[x]
        _need_cuda(x)
        x = x.reshape(-1)
        if x.numel() != k:
            raise ValueError(f"problem {i}: activation row of {x.numel()} values for K={k}")
        x = x.contiguous()
        if x_dtype is None:
            x_dtype, dev = x.dtype, x.device
        if x.dtype != x_dtype or x.dtype not in (torch.float16, torch.bfloat16):
            raise ValueError("chain activations must all be f16 or all bf16")
        w2 = None
        act = "none"
        if pr.get("w2") is not None:
            w2, rs2 = _rows2d(pr["w2"])
            if rs2 != rs or w2.shape != w.shape:
                raise ValueError(f"problem {i}: gate and up weights must share shape and layout")
            act = pr.get("act", "silu")
        nout = w.shape[-2] if w.dim() >= 2 else 1
        od = out_dtype or x_dtype
        if any(isinstance(p.get("x"), int) and p["x"] == i for p in problems[i + 1:]):
            od = x_dtype  # read back as a later problem's activations
        y = torch.empty(1, nout, dtype=od, device=dev)
        b = pr.get("bias")
        if b is not None:
            _need_cuda(b)
            b = b.contiguous()
        arr[i].codec, arr[i].x, arr[i].w = c, _p(x), _p(w)
        arr[i].w2 = _p(w2)
        arr[i].n, arr[i].k, arr[i].w_row_stride = nout, k, rs
        arr[i].act = _lib.ACTS[act]
        arr[i].y, arr[i].y_dtype = _p(y), _DT[od]
        arr[i].bias, arr[i].bias_dtype = _p(b), (_DT[b.dtype] if b is not None else 0)
        arr[i].depends_on = dep
        outs.append(y)
        keep += [x, w, w2, b]
    ws = _workspace(dev, int(L.kq_quantized_matmul_chain_workspace_size(arr, n)))
    _lib.check(L.kq_quantized_matmul_chain(arr, n, _DT[x_dtype], _p(ws), ws.numel(), _stream(dev)),
               "quantized_matmul_chain")
    return outs
