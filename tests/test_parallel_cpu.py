"""Multi-process host logic of the tensor/expert-parallel layers, as gloo ranks
on CPU (world_size 2): shard math + all-reduce reproduce the unsharded oracle."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gmlx_b200 import parallel as par
from gmlx_b200 import synth
from oracle import oracle as O


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _tp_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        full = {
            "q": synth.random_weight("q4_k", 64, 1024, seed=1), "k": synth.random_weight("q4_k", 32, 1024, seed=2),
            "v": synth.random_weight("q4_k", 32, 1024, seed=3), "o": synth.random_weight("q4_k", 64, 1024, seed=4),
            "gate": synth.random_weight("q4_k", 128, 1024, seed=5), "up": synth.random_weight("q4_k", 128, 1024, seed=6),
            "down": synth.random_weight("q6_k", 64, 2048, seed=7)}
        sh = par.shard_llama_layer(full, world, rank)
        x = synth.random_activations(2, 1024, seed=8)
        a = synth.random_activations(2, 1024, seed=9)
        h = synth.random_activations(2, 2048, seed=10)
        ka, kh = 1024 // world, 2048 // world
        o = torch.from_numpy(O.matmul(a[:, rank * ka:(rank + 1) * ka], sh["o"], "q4_k"))
        y = torch.from_numpy(O.matmul(h[:, rank * kh:(rank + 1) * kh], sh["down"], "q6_k"))
        dist.all_reduce(o)
        dist.all_reduce(y)
        qkv = O.matmul(x, sh["qkv"], "q4_k")
        if rank == 0:
            q.put(("o", float(np.abs(o.numpy() - O.matmul(a, full["o"], "q4_k")).max())))
            q.put(("y", float(np.abs(y.numpy() - O.matmul(h, full["down"], "q6_k")).max())))
        rows = [par.row_split(full[n].shape[0], world, rank) for n in ("q", "k", "v")]
        ref = np.concatenate([O.matmul(x, full[n][r0:r1], "q4_k") for n, (r0, r1) in zip(("q", "k", "v"), rows)], 1)
        q.put((f"qkv{rank}", float(np.abs(qkv - ref).max())))
    finally:
        dist.destroy_process_group()


def _ep_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        e, d, k, t = 8, 256, 2, 3
        w = synth.random_weight("q4_k", d, d, seed=3, experts=e)
        x = synth.random_activations(t, d, seed=4)
        xf = O.bf16_bits_to_f32(x).astype(np.float64)
        idx, sc = O.router_topk(synth.random_logits(t, e, seed=5), k, True)
        deq = O.dequantize(w, "q4_k").astype(np.float64)
        b0, b1 = par.expert_range(e, world, rank)
        part = par.ep_partial_reference(xf, idx, sc, lambda ex, xr: deq[ex] @ xr, b0, b1 - b0)
        tp = torch.from_numpy(part)
        dist.all_reduce(tp)
        full = par.ep_partial_reference(xf, idx, sc, lambda ex, xr: deq[ex] @ xr, 0, e)
        if rank == 0:
            q.put(("ep", float(np.abs(tp.numpy() - full).max() / np.abs(full).max())))
    finally:
        dist.destroy_process_group()


def _a2a_worker(rank, world, port, q):
    """All-to-all dispatch / combine: each rank routes ITS tokens (an uneven
    split, one rank may have none), experts split by id range; the combined
    rows equal the full layer on those tokens computed in one process."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        e, d, k, t = 6 * world, 256, 3, 7
        w = synth.random_weight("q4_k", d, d, seed=13, experts=e)
        deq = torch.from_numpy(O.dequantize(w, "q4_k").astype(np.float64))
        x = torch.from_numpy(O.bf16_bits_to_f32(synth.random_activations(t, d, seed=14)).astype(np.float64))
        idx, sc = O.router_topk(synth.random_logits(t, e, seed=15), k, True)
        idx, sc = torch.from_numpy(idx), torch.from_numpy(sc)
        # tokens of this rank: an uneven split of the t tokens (the last rank gets none when t < world * 2)
        bounds = [0, 4, t, t, t][:world + 1] if world <= 4 else None
        bounds[-1] = t
        t0, t1 = bounds[rank], bounds[rank + 1]
        el = e // world
        seen = []

        def expert_fn(rows, e_local, score):
            seen.append(int(rows.shape[0]))
            assert bool(((e_local >= 0) & (e_local < el)).all())
            out = torch.zeros(rows.shape[0], d, dtype=torch.float64)
            for r in range(rows.shape[0]):
                out[r] = float(score[r]) * (deq[rank * el + int(e_local[r])] @ rows[r].double())
            return out.float()
        y = par.ep_dispatch_combine(x[t0:t1].float(), idx[t0:t1], sc[t0:t1], e, expert_fn)
        ref = torch.zeros(t1 - t0, d, dtype=torch.float64)
        for ti in range(t0, t1):
            for j in range(k):
                ref[ti - t0] += float(sc[ti, j]) * (deq[int(idx[ti, j])] @ x[ti].float().double())
        err = float((y.double() - ref).abs().max() / max(float(ref.abs().max()), 1e-30)) if t1 > t0 else 0.0
        q.put((f"a2a{rank}", err))
        q.put((f"rows{rank}", seen[0]))
        q.put((f"shape{rank}", tuple(y.shape) == (t1 - t0, d)))
    finally:
        dist.destroy_process_group()


def _run(worker, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    out = {}
    while not q.empty():
        kk, v = q.get()
        out[kk] = v
    return out


def test_tensor_parallel_layer_gloo():
    out = _run(_tp_worker)
    assert out["o"] < 1e-3 and out["y"] < 1e-3
    assert out["qkv0"] == 0.0 and out["qkv1"] == 0.0


def test_expert_parallel_gloo():
    out = _run(_ep_worker)
    assert out["ep"] < 1e-12


def test_split_helpers():
    assert par.block_split(56, 8, 3) == (21, 28)
    with pytest.raises(ValueError):
        par.block_split(3, 2, 0)
    w = synth.random_weight("q6_k", 4, 2048, seed=1)
    s = par.shard_k(w, "q6_k", 4, 1)
    assert s.shape == (4, 2 * 210) and np.array_equal(s, w[:, 420:840])


def test_k_shards_of_every_codec_sum_to_the_full_product():
    """Row-parallel K shards cut at whole 256-weight groups for every codec
    (the 32/64-weight codecs' groups of blocks included): the shards
    reassemble the wire rows and their oracle products sum to the full one."""
    from gmlx_b200 import parallel as par, synth
    from oracle import oracle as O
    for codec in sorted(synth.CODECS):
        w = synth.random_weight(codec, 16, 2048, seed=5)
        x = synth.random_activations(2, 2048, seed=6)
        full = O.matmul(x, w, codec).astype(np.float64)
        parts, acc, k0 = [], np.zeros_like(full), 0
        for r in range(4):
            ws = np.ascontiguousarray(par.shard_k(w, codec, 4, r))
            kk = ws.shape[1] // synth.BLOCK_BYTES[synth.codec_id(codec)] * 256
            acc += O.matmul(np.ascontiguousarray(x[:, k0:k0 + kk]), ws, codec)
            parts.append(ws)
            k0 += kk
        assert k0 == 2048 and np.array_equal(np.concatenate(parts, 1), w), codec
        assert np.abs(acc - full).max() <= 1e-4 * np.abs(full).max(), codec


@pytest.mark.parametrize("world", [2, 3])
def test_expert_parallel_all_to_all_gloo(world):
    """Dispatch / combine over gloo ranks: every rank's combined rows match
    the full layer on its own tokens, and all routed slots were computed
    exactly once (received rows over the ranks = t * k)."""
    out = _run(_a2a_worker, world)
    for r in range(world):
        assert out[f"a2a{r}"] < 1e-5, out
        assert out[f"shape{r}"]
    assert sum(out[f"rows{r}"] for r in range(world)) == 7 * 3
