"""Tensor-parallel decode on 2 GPUs (skipped with fewer): the fused
row-parallel all-reduce kernel against the unsharded projection, and the same
bits on every rank.  Ranks are processes (one per GPU, NCCL for the handle
exchange), rendezvous on 127.0.0.1."""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
WORLD = 2


def _rank_main(rank, port, out_q):
    import torch.distributed as dist
    from gmlx_b200 import kq, parallel as par, synth
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, device_id=dev)
    try:
        comm = par.PeerComm(4096, dev)
        res = {}
        for codec, n, k in (("q4_k", 4096, 4096), ("q6_k", 4096, 14336)):
            w = synth.random_weight(codec, n, k, seed=7)
            x = synth.random_activations(1, k, seed=8)
            xd = torch.from_numpy(x.view(np.int16).copy()).view(torch.bfloat16).to(dev)
            full = kq.quantized_matmul(xd, torch.from_numpy(w).to(dev), None, codec, out_dtype=torch.float32)
            kk = k // WORLD
            ws = par.shard_k(torch.from_numpy(w), codec, WORLD, rank).contiguous().to(dev)
            ys = [kq.quantized_matmul_allreduce(xd[:, rank * kk:(rank + 1) * kk].contiguous(), ws, codec, comm,
                                                out_dtype=torch.float32) for _ in range(3)]
            torch.cuda.synchronize()
            res[codec] = (full.cpu().numpy(), [y.cpu().numpy() for y in ys], kq.workspace_error())
        dist.barrier()
        comm.close()
        out_q.put((rank, res))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
def test_fused_allreduce_two_ranks():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 200
    procs = [ctx.Process(target=_rank_main, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in range(WORLD))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for codec in ("q4_k", "q6_k"):
        full = got[0][codec][0]
        for r in range(WORLD):
            _, ys, err = got[r][codec]
            assert err == 0
            for y in ys:
                assert np.abs(y - full).max() / np.abs(full).max() <= 1e-4
                assert np.array_equal(y.view(np.uint32), got[0][codec][1][0].view(np.uint32))  # same bits everywhere


def _ep_rank_main(rank, port, out_q):
    import torch.distributed as dist
    from gmlx_b200 import kq, parallel as par, synth
    from oracle import oracle as O
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, device_id=dev)
    try:
        e, d, f, k, t = 16, 1024, 512, 4, 9
        wg = synth.random_weight("q4_k", f, d, seed=31, experts=e)
        wu = synth.random_weight("q4_k", f, d, seed=32, experts=e)
        wd = synth.random_weight("q6_k", d, f, seed=33, experts=e)
        el = e // WORLD
        loc = [torch.from_numpy(a[rank * el:(rank + 1) * el]).to(dev) for a in (wg, wu, wd)]
        x = synth.random_activations(t, d, seed=34)
        lg = synth.random_logits(t, e, seed=35)
        t0, t1 = (0, 5) if rank == 0 else (5, t)  # uneven token split
        xd = torch.from_numpy(x[t0:t1].view(np.int16).copy()).view(torch.bfloat16).to(dev)
        y = par.ep_moe_alltoall(xd, torch.from_numpy(lg[t0:t1]).to(dev), k, *loc, "q4_k", "q6_k", e)
        idx, sc = O.router_topk(lg, k, True)
        ref = np.zeros((t1 - t0, d))
        for ti in range(t0, t1):
            for j in range(k):
                ex = idx[ti, j]
                g = O.matmul(x[ti:ti + 1], wg[ex], "q4_k")[0].astype(np.float64)
                u = O.matmul(x[ti:ti + 1], wu[ex], "q4_k")[0].astype(np.float64)
                hb = synth.f32_to_bf16_bits((g / (1 + np.exp(-g)) * u).astype(np.float32))
                ref[ti - t0] += float(sc[ti, j]) * O.matmul(hb[None], wd[ex], "q6_k")[0]
        torch.cuda.synchronize()
        out_q.put((rank, (float(np.abs(y.cpu().numpy() - ref).max() / np.abs(ref).max()), kq.workspace_error())))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
def test_expert_parallel_all_to_all_two_ranks():
    """All-to-all dispatch / combine over NCCL on 2 GPUs: each rank's combined
    rows for its own tokens against the CPU oracle's full expert layer."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29800 + os.getpid() % 200
    procs = [ctx.Process(target=_ep_rank_main, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in range(WORLD))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(WORLD):
        err, werr = got[r]
        assert werr == 0 and err <= 1e-2, got


def _ar_rank_main(rank, port, out_q):
    import torch.distributed as dist
    from gmlx_b200 import kq, parallel as par
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, device_id=dev)
    try:
        comm = par.PeerComm(8192, dev)
        res = []
        g = torch.Generator(device="cpu").manual_seed(100 + rank)
        # sizes off the 512-value CTA slices, both dtypes, in place and out of
        # place, and more calls than the two buffer parities
        for i, (n, dt, inplace) in enumerate([(4096, torch.bfloat16, True), (4095, torch.float32, False),
                                              (1, torch.float32, True), (8192, torch.float16, False),
                                              (1000, torch.bfloat16, False)]):
            x = torch.randn(n, generator=g).to(dt).to(dev)
            xin = x.clone()
            y = kq.all_reduce(x, comm) if inplace else kq.all_reduce(x, comm, out=torch.empty_like(x))
            parts = [torch.empty_like(xin) for _ in range(WORLD)]
            dist.all_gather(parts, xin)
            ref = torch.zeros(n, dtype=torch.float32, device=dev)
            for p in parts:  # the kernel's rank-order f32 sum
                ref = ref + p.float()
            torch.cuda.synchronize()
            res.append((y.float().cpu().numpy(), ref.to(dt).float().cpu().numpy()))
        err = comm.error()
        dist.barrier()
        comm.close()
        out_q.put((rank, (res, err)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
def test_peer_allreduce_two_ranks():
    """kq.all_reduce (one-shot over NVLink peer memory) equals the rank-order
    f32 sum of the gathered inputs bit for bit, on every rank."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29800 + os.getpid() % 150
    procs = [ctx.Process(target=_ar_rank_main, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in range(WORLD))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(WORLD):
        res, err = got[r]
        assert err == 0
        for (y, ref), (y0, _) in zip(res, got[0][0]):
            assert np.array_equal(y, ref)
            assert np.array_equal(y, y0)
