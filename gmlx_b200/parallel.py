"""Tensor- and expert-parallel layers over the kq ops (one process per GPU,
torch.distributed for the collectives: NCCL on B200s, gloo in CPU tests).

Dense decoder layer: column-parallel q/k/v and gate/up
(split the output rows -- wire rows are independent, so any row split is exact,
gmlx/occupancy_fuse.py:32-34), row-parallel o and down (split K at whole
256-weight-block granularity, i.e. a byte range of every wire row), one
all-reduce of the partial sums after each row-parallel projection.  This is the
shard_linear layout gmlx uses for hy_v3 (gmlx/hy_v3_model.py:396-443) with the
all_sum of gmlx/hy_v3_model.py:259.

MoE expert layer, two ways, experts split by contiguous expert-id range:
 * route-all + all-reduce (ep_moe_forward): every rank routes the same tokens,
   runs the routed slots whose expert it owns, and the per-rank partial
   outputs are summed -- the sharding_group all_sum of
   gmlx/moe_experts.py:250-266;
 * all-to-all dispatch / combine (ep_moe_alltoall, ep_dispatch_combine): each
   rank holds its own tokens, routes them, and sends every routed slot's
   token row, expert id and score to the expert's owner (NCCL all-to-all with
   the per-destination counts exchanged first); the owner runs its local
   experts on the rows it received and sends the score-weighted rows back
   (the inverse all-to-all), where they are added per token.  Only routed
   rows cross NVLink, instead of a [T, hidden] f32 all-reduce.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist

from .synth import BLOCK_BYTES, QK, codec_id


def block_split(n_blocks: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous whole-block range [b0, b1) of rank `rank`."""
    if n_blocks % world:
        raise ValueError(f"{n_blocks} blocks do not split evenly over {world} ranks")
    per = n_blocks // world
    return rank * per, (rank + 1) * per


def row_split(n_rows: int, world: int, rank: int) -> tuple[int, int]:
    if n_rows % world:
        raise ValueError(f"{n_rows} rows do not split evenly over {world} ranks")
    per = n_rows // world
    return rank * per, (rank + 1) * per


def shard_rows(w, world: int, rank: int):
    """Column-parallel shard: this rank's output rows of a wire tensor [N, bytes]."""
    r0, r1 = row_split(w.shape[0], world, rank)
    return w[r0:r1]


def shard_k(w, codec, world: int, rank: int):
    """Row-parallel shard: this rank's whole-block K range of every wire row."""
    bpb = BLOCK_BYTES[codec_id(codec)]
    nb = w.shape[-1] // bpb
    b0, b1 = block_split(nb, world, rank)
    return w[..., b0 * bpb:b1 * bpb]


def shard_llama_layer(full: dict, world: int, rank: int) -> dict:
    """Shard a Llama-style layer dict (numpy or torch wire tensors):
    q/k/v/gate/up by rows, o/down by K blocks.  Returns contiguous shards with a
    fused q|k|v tensor."""
    cat = np.concatenate if isinstance(full["q"], np.ndarray) else torch.cat

    def c(t):
        return np.ascontiguousarray(t) if isinstance(t, np.ndarray) else t.contiguous()
    return {
        "qkv": c(cat([shard_rows(full[n], world, rank) for n in ("q", "k", "v")], 0)),
        "o": c(shard_k(full["o"], "q4_k", world, rank)),
        "gate": c(shard_rows(full["gate"], world, rank)),
        "up": c(shard_rows(full["up"], world, rank)),
        "down": c(shard_k(full["down"], "q6_k", world, rank)),
    }


class TPDecoderMLP:
    """The seven projections of one decoder layer on this rank's shards.

    forward(x, attn_local) -> (qkv_local, o_full, y_full): qkv for this rank's
    heads; o-proj of this rank's slice of the attention output, summed over
    ranks; gate/up/SiLU on this rank's FFN slice and the down projection summed
    over ranks.  (Attention itself is outside the quantized-matmul path.)"""

    def __init__(self, shards: dict, group=None, codecs=("q4_k", "q6_k"), comm: "PeerComm | None" = None):
        self.s = shards
        self.group = group
        self.cg, self.cd = codecs
        self.comm = comm

    def forward(self, x, attn_local):
        from . import kq
        qkv = kq.quantized_matmul(x, self.s["qkv"], None, self.cg)
        h = kq.quantized_glu(x, self.s["gate"], self.s["up"], self.cg, act="silu")
        if self.comm is not None and x.reshape(-1, x.shape[-1]).shape[0] == 1:
            # decode: each row-parallel projection and its cross-rank sum in one kernel
            o = kq.quantized_matmul_allreduce(attn_local, self.s["o"], self.cg, self.comm, out_dtype=torch.float32)
            y = kq.quantized_matmul_allreduce(h, self.s["down"], self.cd, self.comm, out_dtype=torch.float32)
            return qkv, o, y
        o = kq.quantized_matmul(attn_local, self.s["o"], None, self.cg, out_dtype=torch.float32)
        y = kq.quantized_matmul(h, self.s["down"], None, self.cd, out_dtype=torch.float32)
        if dist.is_initialized() and dist.get_world_size(self.group) > 1:
            dist.all_reduce(o, group=self.group)
            dist.all_reduce(y, group=self.group)
        return qkv, o, y


class PeerComm:
    """Communication buffers of the fused row-parallel all-reduce
    (``kq.quantized_matmul_allreduce``): one zero-filled device buffer per rank,
    each mapped into every rank's process over CUDA IPC, and a device table of
    the `world` buffer pointers (own at [rank]).  One set serves every
    projection of up to `n` outputs, as long as all ranks make the same calls
    in the same order."""

    def __init__(self, n: int, device, group=None):
        import ctypes
        from . import _lib
        L = _lib.load()
        self.n = int(n)
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self._L = L
        own = ctypes.c_void_p()
        with torch.cuda.device(device):
            _lib.check(L.kq_comm_alloc(L.kq_allreduce_buffer_bytes(self.world, self.n), ctypes.byref(own)),
                       "comm_alloc")
            self._own = own.value
            ptrs, self._opened = [], []
            if self.world > 1:
                h = ctypes.create_string_buffer(64)
                _lib.check(L.kq_ipc_handle(ctypes.c_void_p(self._own), h), "ipc_handle")
                handles = [None] * self.world
                dist.all_gather_object(handles, h.raw, group=group)
                for r in range(self.world):
                    if r == self.rank:
                        ptrs.append(self._own)
                        continue
                    p = ctypes.c_void_p()
                    _lib.check(L.kq_ipc_open(ctypes.create_string_buffer(handles[r], 64), ctypes.byref(p)),
                               "ipc_open")
                    self._opened.append(p.value)
                    ptrs.append(p.value)
            else:
                ptrs = [self._own]
            self.table = torch.tensor(ptrs, dtype=torch.int64, device=device)

    def error(self, clear: bool = False) -> int:
        """Error word of this rank's buffer (7: a one-shot all-reduce gave up
        waiting for a peer); synchronizes the current stream."""
        import ctypes
        from . import _lib
        v = self._L.kq_comm_error(ctypes.c_void_p(self._own), int(clear),
                                  ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        if v < 0:
            _lib.check(-v, "comm_error")
        return v

    def close(self):
        import ctypes
        for p in self._opened:
            self._L.kq_ipc_close(ctypes.c_void_p(p))
        self._opened = []
        if self._own:
            self._L.kq_comm_free(ctypes.c_void_p(self._own))
            self._own = None


def expert_range(n_experts: int, world: int, rank: int) -> tuple[int, int]:
    return row_split(n_experts, world, rank)


def ep_moe_forward(x, logits, top_k, gate_w, up_w, down_w, codec_gu, codec_d, expert_base, group=None,
                   norm_topk_prob=True):
    """Expert-parallel MoE layer (decode): route all tokens, run the slots whose
    expert lies in [expert_base, expert_base + local experts), sum over ranks."""
    from . import kq
    idx, scores = kq.moe_router_topk(logits, top_k, norm_topk_prob, shared_gate=False)
    y = kq.moe_expert_layer_local(x, idx, scores, gate_w, up_w, down_w, codec_gu, codec_d, expert_base)
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(y, group=group)
    return y


def ep_dispatch_combine(x: torch.Tensor, idx: torch.Tensor, scores: torch.Tensor, n_experts: int, expert_fn,
                        group=None) -> torch.Tensor:
    """All-to-all expert-parallel dispatch and combine for this rank's tokens.

    x [t, D] (t may be 0), idx [t, k] global expert ids, scores [t, k] routing
    weights.  Experts are owned in contiguous ranges of n_experts / world.
    expert_fn(rows [R, D], local_expert [R] int32, score [R] f32) -> [R, D]
    f32, the score-weighted expert outputs of the rows this rank received.
    Returns y [t, D] f32 = sum_j scores[t, j] * expert_{idx[t, j]}(x[t]).
    Steps: counts per destination rank (all-to-all), rows + (expert, score)
    to the owners (all-to-all with those splits), local expert compute,
    weighted rows back (the inverse all-to-all), per-token add."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if n_experts % world:
        raise ValueError(f"{n_experts} experts do not split over {world} ranks")
    el = n_experts // world
    t, k = idx.shape
    d = x.shape[1]
    flat = idx.reshape(-1).long()
    dest = flat // el
    order = torch.argsort(dest, stable=True)                     # slots grouped by owner rank
    tok = order // k                                             # token of each sent slot
    send_counts = torch.bincount(dest, minlength=world).to(torch.int64)
    xs = x.index_select(0, tok)
    meta = torch.stack([(flat - dest * el)[order].to(torch.float32),  # local expert id (exact in f32)
                        scores.reshape(-1)[order].float()], 1)
    if world == 1:
        yb = expert_fn(xs, meta[:, 0].to(torch.int32), meta[:, 1].contiguous())
    else:
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=group)
        sc, rc = send_counts.tolist(), recv_counts.tolist()      # the split sizes the row exchange needs
        r = sum(rc)
        xr = x.new_empty(r, d)
        dist.all_to_all_single(xr, xs.contiguous(), rc, sc, group=group)
        mr = meta.new_empty(r, 2)
        dist.all_to_all_single(mr, meta, rc, sc, group=group)
        yr = expert_fn(xr, mr[:, 0].to(torch.int32), mr[:, 1].contiguous()).float().contiguous()
        yb = yr.new_empty(t * k, d)
        dist.all_to_all_single(yb, yr, sc, rc, group=group)
    y = torch.zeros(t, d, dtype=torch.float32, device=x.device)
    if t * k:
        y.index_add_(0, tok, yb.float())
    return y


def ep_moe_alltoall(x, logits, top_k, gate_w, up_w, down_w, codec_gu, codec_d, n_experts, group=None,
                    norm_topk_prob=True, act="silu"):
    """Expert-parallel MoE layer with all-to-all dispatch / combine on the kq
    ops: route this rank's tokens (kq.moe_router_topk), exchange the routed
    rows, run the local experts (kq.moe_expert_layer_local over one slot per
    received row, the score applied there), send the weighted rows back and
    add them per token.  x [t, D] this rank's tokens; the stacks hold this
    rank's n_experts / world experts."""
    from . import kq
    idx, scores = kq.moe_router_topk(logits, top_k, norm_topk_prob, shared_gate=False)

    def local(rows, e_local, score):
        if rows.shape[0] == 0:
            return torch.zeros(0, rows.shape[1], dtype=torch.float32, device=rows.device)
        return kq.moe_expert_layer_local(rows, e_local.reshape(-1, 1), score.reshape(-1, 1), gate_w, up_w, down_w,
                                         codec_gu, codec_d, 0, gate_w.shape[0], act=act, out_dtype=torch.float32)
    return ep_dispatch_combine(x, idx, scores, n_experts, local, group)


def ep_partial_reference(x_f32: np.ndarray, idx: np.ndarray, scores: np.ndarray, expert_out, expert_base: int,
                         n_local: int) -> np.ndarray:
    """Host statement of one rank's share of the expert layer (tests): sum over
    the routed slots whose expert is local of score * expert_out(e, x)."""
    t, k = idx.shape
    y = np.zeros((t, x_f32.shape[1]), np.float64)
    for ti in range(t):
        for j in range(k):
            e = int(idx[ti, j])
            if expert_base <= e < expert_base + n_local:
                y[ti] += float(scores[ti, j]) * expert_out(e, x_f32[ti])
    return y


__all__ = ["block_split", "row_split", "shard_rows", "shard_k", "shard_llama_layer", "TPDecoderMLP", "PeerComm",
           "expert_range", "ep_moe_forward", "ep_dispatch_combine", "ep_moe_alltoall", "ep_partial_reference", "QK"]
