"""Module counterparts of ``mlx_kquant.nn`` used by gmlx's module swap
(``install_kquant_modules``, gmlx/modules.py:1473-1576).

* ``KQuantLinear(in_dims, out_dims, bias, codec)`` (gmlx/modules.py:1539)
* ``KQuantSwitchLinear(num_experts, out_dims, in_dims, bias, codec)`` (:1552)
* ``KQuantEmbedding(num_embeddings, dims, codec, out_dtype)`` (:1545) and
  ``KQuantMultiLinear(in_dims, out_dims, num_heads, codec)`` (:1530, :1556)
* ``KQuantSwitchGLU`` -- SwitchGLU over three KQuantSwitchLinear stacks with
  the fused decode path of ``_FusedKQuantSwitchGLU`` (gmlx/modules.py:540-605):
  ``moe_glu_gather_kq`` + ``gather_qmv_mix_ns_kq`` when fewer than 64 routed
  slots and bf16/fp16 activations, the stock gather_qmm path otherwise.

``.weight`` is the uint8 wire tensor (``[out, nb*bpb]`` / ``[E, out, nb*bpb]``),
``.scales`` the ``(1,)`` placeholder, ``.kquant_type`` the codec string.
Modules are frozen and inference-only.
"""
from __future__ import annotations

import torch
from torch import nn

from . import kq
from .synth import BLOCK_BYTES, QK, codec_id


def _wire_bytes(codec: str, in_dims: int) -> int:
    c = codec_id(codec)
    if in_dims % QK:
        raise ValueError(f"{codec}: in_dims={in_dims} is not a whole number of {QK}-weight blocks")
    return in_dims // QK * BLOCK_BYTES[c]


class KQuantLinear(nn.Module):
    def __init__(self, in_dims: int, out_dims: int, bias: bool = False, codec: str = "q4_k", device=None):
        super().__init__()
        if not kq.codec_has_matmul(codec):
            raise NotImplementedError(f"no K-quant kernels for codec {codec!r}")
        self.in_dims, self.out_dims, self.kquant_type = in_dims, out_dims, codec
        self.register_buffer("weight", torch.zeros(out_dims, _wire_bytes(codec, in_dims), dtype=torch.uint8,
                                                   device=device))
        self.register_buffer("scales", torch.zeros(1, dtype=torch.uint8, device=device))
        self.bias = nn.Parameter(torch.zeros(out_dims, device=device), requires_grad=False) if bias else None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = kq.quantized_matmul(x, self.weight, self.scales, self.kquant_type)
        return y + self.bias.to(y.dtype) if self.bias is not None else y


class KQuantSwitchLinear(nn.Module):
    def __init__(self, num_experts: int, out_dims: int, in_dims: int, bias: bool = False, codec: str = "q4_k",
                 device=None):
        super().__init__()
        if not kq.codec_has_matmul(codec):
            raise NotImplementedError(f"no K-quant kernels for codec {codec!r}")
        self.num_experts, self.in_dims, self.out_dims, self.kquant_type = num_experts, in_dims, out_dims, codec
        self.register_buffer("weight", torch.zeros(num_experts, out_dims, _wire_bytes(codec, in_dims),
                                                   dtype=torch.uint8, device=device))
        self.register_buffer("scales", torch.zeros(1, dtype=torch.uint8, device=device))
        self.bias = (nn.Parameter(torch.zeros(num_experts, out_dims, device=device), requires_grad=False)
                     if bias else None)

    def forward(self, x: torch.Tensor, indices: torch.Tensor, sorted_indices: bool = False) -> torch.Tensor:
        """mlx-lm SwitchLinear semantics: x [..., M, K] broadcast against indices."""
        y = kq.gather_qmm(x, self.weight, self.scales, self.kquant_type, rhs_indices=indices,
                          sorted_indices=sorted_indices)
        if self.bias is not None:
            y = y + self.bias[indices.long()].unsqueeze(-2).to(y.dtype)
        return y


class KQuantEmbedding(nn.Module):
    """``KQuantEmbedding(num_embeddings, dims, codec, out_dtype=...)``
    (gmlx/modules.py:1545-1547): token rows are dequantized on lookup;
    ``as_linear`` is the tied output head, ``x @ dequant(W).T`` (used as
    ``embed_tokens.as_linear`` by gmlx/hy_v3_model.py:341)."""

    def __init__(self, num_embeddings: int, dims: int, codec: str = "q4_k", out_dtype=torch.bfloat16, device=None):
        super().__init__()
        if not kq.codec_has_matmul(codec):
            raise NotImplementedError(f"no K-quant kernels for codec {codec!r}")
        self.num_embeddings, self.dims, self.kquant_type, self.out_dtype = num_embeddings, dims, codec, out_dtype
        self.register_buffer("weight", torch.zeros(num_embeddings, _wire_bytes(codec, dims), dtype=torch.uint8,
                                                   device=device))
        self.register_buffer("scales", torch.zeros(1, dtype=torch.uint8, device=device))

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        rows = self.weight[ids.reshape(-1).long()]
        out = kq.dequantize(rows, self.scales, self.kquant_type, dtype=self.out_dtype)
        return out.reshape(*ids.shape, self.dims)

    def as_linear(self, x: torch.Tensor) -> torch.Tensor:
        return kq.quantized_matmul(x, self.weight, self.scales, self.kquant_type)


class KQuantMultiLinear(nn.Module):
    """``KQuantMultiLinear(in_dims, out_dims, num_heads, codec)`` (gmlx/modules.py:1530,
    1556): one wire matrix per head, ``weight [num_heads, out, nb*bpb]``, with
    mlx-lm MultiLinear semantics over ``x [..., num_heads, L, K]``:
    ``transpose=True`` -> ``x @ W[h].T`` through ``gather_qmm`` (the reference
    dispatches these tensors to ``kq.gather_qmm`` too); ``transpose=False`` ->
    ``x @ W[h]`` (the absorbed-MLA un-embedding) on the dequantized heads."""

    def __init__(self, in_dims: int, out_dims: int, num_heads: int, codec: str = "q4_k", device=None):
        super().__init__()
        if not kq.codec_has_matmul(codec):
            raise NotImplementedError(f"no K-quant kernels for codec {codec!r}")
        self.in_dims, self.out_dims, self.num_heads, self.kquant_type = in_dims, out_dims, num_heads, codec
        self.register_buffer("weight", torch.zeros(num_heads, out_dims, _wire_bytes(codec, in_dims),
                                                   dtype=torch.uint8, device=device))
        self.register_buffer("scales", torch.zeros(1, dtype=torch.uint8, device=device))

    def forward(self, x: torch.Tensor, transpose: bool = True) -> torch.Tensor:
        h = self.num_heads
        if transpose:
            if x.shape[-3] != h or x.shape[-1] != self.in_dims:
                raise ValueError(f"MultiLinear expects [..., {h}, L, {self.in_dims}], got {tuple(x.shape)}")
            # batch element (..., head) of x takes expert `head` of the stack
            heads = torch.arange(h, device=x.device, dtype=torch.int32).expand(*x.shape[:-2])
            return kq.gather_qmm(x, self.weight, self.scales, self.kquant_type, rhs_indices=heads)
        if x.shape[-3] != h or x.shape[-1] != self.out_dims:
            raise ValueError(f"MultiLinear expects [..., {h}, L, {self.out_dims}], got {tuple(x.shape)}")
        w = kq.dequantize(self.weight, self.scales, self.kquant_type, dtype=x.dtype)  # [H, out, in]
        return torch.matmul(x, w)


class KQuantSwitchGLU(nn.Module):
    """SwitchGLU (gate/up/down expert stacks, SiLU) with the fused decode path."""

    def __init__(self, input_dims: int, hidden_dims: int, num_experts: int, gate_codec="q4_k", down_codec=None,
                 act: str = "silu", device=None):
        super().__init__()
        down_codec = down_codec or gate_codec
        self.gate_proj = KQuantSwitchLinear(num_experts, hidden_dims, input_dims, False, gate_codec, device)
        self.up_proj = KQuantSwitchLinear(num_experts, hidden_dims, input_dims, False, gate_codec, device)
        self.down_proj = KQuantSwitchLinear(num_experts, input_dims, hidden_dims, False, down_codec, device)
        self.act = act

    def _act(self, g):
        if self.act == "silu":
            return torch.nn.functional.silu(g)
        if self.act == "gelu":
            return torch.nn.functional.gelu(g)
        return torch.nn.functional.gelu(g, approximate="tanh")

    def forward(self, x: torch.Tensor, indices: torch.Tensor, scores: torch.Tensor | None = None) -> torch.Tensor:
        d = x.shape[-1]
        t = x.numel() // d
        k = indices.shape[-1]
        if indices.numel() < 64 and x.dtype in (torch.bfloat16, torch.float16):
            # fused decode (gmlx/modules.py:542-604): f32 GLU epilogue, mix folded into the down gather
            idx = indices.reshape(t, k)
            h = kq.moe_glu_gather_kq(x.reshape(t, d), self.gate_proj.weight, self.up_proj.weight,
                                     self.gate_proj.kquant_type, idx, act=self.act)
            if scores is not None:
                y = kq.gather_qmv_mix_ns_kq(h, self.down_proj.weight, self.down_proj.kquant_type, idx,
                                            scores.reshape(t, k))
                return y.reshape(*indices.shape[:-1], y.shape[-1])
            y = kq.gather_qmv_kq(h, self.down_proj.weight, self.down_proj.kquant_type, idx)
            return y.reshape(*indices.shape, y.shape[-1])
        # stock SwitchGLU: x -> [..., 1, 1, D], gather per slot
        xe = x.reshape(*x.shape[:-1], 1, 1, d)
        g = self.gate_proj(xe, indices)
        u = self.up_proj(xe, indices)
        h = (self._act(g.float()) * u.float()).to(x.dtype)
        y = self.down_proj(h, indices).squeeze(-2)
        if scores is not None:
            y = (y.float() * scores[..., None].float()).sum(-2).to(x.dtype)
        return y


def qwen3_moe_forward(gate: nn.Module, switch_mlp: KQuantSwitchGLU, x: torch.Tensor, top_k: int,
                      norm_topk_prob: bool = True) -> torch.Tensor:
    """Qwen3-MoE block forward (gmlx/moe_experts.py:226-240) on the fused ops:
    router logits -> kq.moe_router_topk (softmax, top-k, renorm) -> experts."""
    logits = gate(x).float()
    idx, scores = kq.moe_router_topk(logits, top_k, norm_topk_prob, shared_gate=False)
    return switch_mlp(x, idx, scores)
