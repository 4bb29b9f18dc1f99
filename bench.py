"""Benchmark: K-quant decode over Llama-3-8B Q4_K_M decoder layers on B200.

Workload: the seven projections of a Llama-3-8B
layer -- q/k/v/o/gate/up in Q4_K, down in Q6_K (137,822,208 wire bytes) --
applied to M bf16 activation rows (M=1 headline; M in {4, 16, 32} reported
under ``sweep``).  One step = one token through all 32 layers of the model
(32 distinct layers, 4.41 GB of weights, far larger than the 126 MB L2); per
layer, through the kq ops:

    qkv = quantized_matmul(x, Wqkv)           row-concatenated q|k|v wire, as gmlx/occupancy_fuse.py does
    o   = quantized_matmul(a, Wo)             a = this rank's slice of the attention output stand-in
    h   = quantized_glu(x, Wgate, Wup, silu)  fused gate/up
    y   = quantized_matmul(h, Wdown)          Q6_K

(``--chain``, M = 1: the four as ONE persistent launch, quantized_matmul_chain,
down reading h through device-side completion counters; both launch
structures are reported under ``decode_launch_modes``.)
Weights and activations are seeded synthetic data with the configuration's
block statistics (no GGUF files on the box).  ``value`` is device-timed over
exactly ``--steps`` replays of the step's CUDA graph (CUDA events on the
launching stream, max over ranks); ``e2e`` runs the same steps through the
public Python op API with the step input copied from pinned host memory and
the output read back every step.  Every cell (decode, prefill, MoE) checks
one untimed step against f32 dequantization + an f32 torch matmul and
reports the max relative error.

``--impl reference`` times the CPU dequantize-then-matmul path (the C oracle
restating the ggml block formats; the reference's own kernels are Apple Metal
in the external mlx-kquant and cannot run here) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "K/IQ-quant qmatmul: decode GB/s as % HBM peak, prefill TFLOP/s, at 1/2/4/8 GPU"
UNIT = "GB/s"
N_LAYERS = 32  # Llama-3-8B: one decode step = one token through its 32 layers
LAYER_WEIGHT_BYTES = 137_822_208


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.out = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.out.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=2)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        mhz, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.out:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                mhz.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(mhz)}


def build_layers(dev, n_layers, world=1, rank=0, seed0=100):
    """n_layers distinct Llama-3-8B layers; with world > 1 this rank's tensor-
    parallel shards (q/k/v/gate/up by output rows, o/down by K blocks)."""
    import torch

    from gmlx_b200 import parallel as par
    from gmlx_b200 import synth
    layers = []
    for li in range(n_layers):
        s = seed0 + 10 * li
        full = {
            "q": synth.random_weight("q4_k", 4096, 4096, seed=s),
            "k": synth.random_weight("q4_k", 1024, 4096, seed=s + 1),
            "v": synth.random_weight("q4_k", 1024, 4096, seed=s + 2),
            "o": synth.random_weight("q4_k", 4096, 4096, seed=s + 3),
            "gate": synth.random_weight("q4_k", 14336, 4096, seed=s + 4),
            "up": synth.random_weight("q4_k", 14336, 4096, seed=s + 5),
            "down": synth.random_weight("q6_k", 4096, 14336, seed=s + 6),
        }
        sh = par.shard_llama_layer(full, world, rank)
        layers.append({k: torch.from_numpy(v).to(dev) for k, v in sh.items()})
    return layers


def layer_step(kq, L, x, a=None, dist=None, comm=None, mode="chain", ar="nccl"):
    """One decoder-layer pass of the seven quantized projections.

    mode "chain" (M = 1): q|k|v, o, gate+up and down in ONE persistent launch
    (kq.quantized_matmul_chain), down reading the gate/up output through the
    kernel's completion counters.  mode "chain_dep" (M = 1, one GPU): the same
    launch with every projection reading the previous one's output (q rows ->
    o -> gate/up -> down), the dependency shape of a real layer minus
    attention and norms.  mode "ops": one kq op per projection group (4
    launches).  Under tensor parallelism the row-parallel o and down outputs
    are summed over ranks: at M=1 optionally inside their GEMV kernels (peer
    stores over NVLink, `comm`, ar "fused"), after them with the one-shot
    peer-memory all-reduce kernel (kq.all_reduce, ar "peer"), or with NCCL
    all-reduces (ar "nccl").  `a` stands in for this rank's slice of the
    attention output."""
    xa = x if a is None else a
    if x.shape[0] == 1 and comm is None and mode == "chain":
        qkv, o, h, y = kq.quantized_matmul_chain([
            {"x": x, "w": L["qkv"], "codec": "q4_k"},
            {"x": xa, "w": L["o"], "codec": "q4_k"},
            {"x": x, "w": L["gate"], "w2": L["up"], "act": "silu", "codec": "q4_k"},
            {"x": 2, "w": L["down"], "codec": "q6_k"}])
        if dist is not None:
            dist.all_reduce(o)
            dist.all_reduce(y)
        return qkv, o, y
    if x.shape[0] == 1 and mode == "chain_dep":
        nq = L["o"].shape[1] // 144 * 256
        q, kv, o, h, y = kq.quantized_matmul_chain([
            {"x": x, "w": L["qkv"][:nq], "codec": "q4_k"},
            {"x": x, "w": L["qkv"][nq:], "codec": "q4_k"},
            {"x": 0, "w": L["o"], "codec": "q4_k"},
            {"x": 2, "w": L["gate"], "w2": L["up"], "act": "silu", "codec": "q4_k"},
            {"x": 3, "w": L["down"], "codec": "q6_k"}])
        return q, o, y
    qkv = kq.quantized_matmul(x, L["qkv"], None, "q4_k")
    h = kq.quantized_glu(x, L["gate"], L["up"], "q4_k", act="silu")
    if comm is not None and x.shape[0] == 1 and ar == "fused":
        o = kq.quantized_matmul_allreduce(xa, L["o"], "q4_k", comm)
        y = kq.quantized_matmul_allreduce(h, L["down"], "q6_k", comm)
        return qkv, o, y
    o = kq.quantized_matmul(xa, L["o"], None, "q4_k")
    y = kq.quantized_matmul(h, L["down"], None, "q6_k")
    if dist is not None and ar == "peer" and comm is not None:
        kq.all_reduce(o, comm)
        kq.all_reduce(y, comm)
    elif dist is not None:
        dist.all_reduce(o)
        dist.all_reduce(y)
    return qkv, o, y


def step_bytes(m):
    # algorithmic bytes: wire weights + activations in (x read by 3 launches
    # counted once per launch) + outputs
    return LAYER_WEIGHT_BYTES + m * 2 * (4096 * 3 + 14336) + m * 2 * (6144 + 4096 + 14336 + 4096)


def time_graph(torch, fn, steps, warmup, stream, min_warm_s=0.0):
    """Capture `fn` (one pass over all layers) in a CUDA graph; time replays."""
    with torch.cuda.stream(stream):
        for _ in range(2):
            fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        fn()
    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize()
    if min_warm_s > 0:  # keep the GPU busy (clock sampling sees a loaded GPU) before timing
        t0 = time.perf_counter()
        while time.perf_counter() - t0 < min_warm_s:
            for _ in range(16):
                g.replay()
            torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        a.record(stream)
        for _ in range(steps):
            g.replay()
        b.record(stream)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / 1e3  # seconds for `steps` replays


GLU_LAUNCH_DRAM_BYTES = 67_143_936  # ncu: fused gate/up GEMV, Q4_K 2 x 14336 x 4096, M = 1 (read + write)
CHAIN_LAUNCH_DRAM_BYTES = None      # ncu: one chain launch (a whole layer), from the capture in profiles/


def _rel(y, ref):
    return float((y.float() - ref).abs().max() / ref.abs().max().clamp_min(1e-30))


def _deq(kq, w, codec):
    return kq.dequantize(w, None, codec)  # f32, bit-exact with the ggml block formats


def verify_layer(torch, kq, L, m, dev, mode, ka):
    """Max relative error of one layer step's outputs at the bench's own shapes
    (this rank's shards), each against f32 dequantization then an f32 torch
    matmul (TF32 off).  Outside every timed region."""
    torch.backends.cuda.matmul.allow_tf32 = False
    g = torch.Generator(device="cpu").manual_seed(7)
    x = torch.randn(m, 4096, generator=g).to(torch.bfloat16).to(dev)
    a = x[:, :ka].contiguous()
    if mode == "chain":
        qkv, o, h, y = kq.quantized_matmul_chain([
            {"x": x, "w": L["qkv"], "codec": "q4_k"}, {"x": a, "w": L["o"], "codec": "q4_k"},
            {"x": x, "w": L["gate"], "w2": L["up"], "act": "silu", "codec": "q4_k"},
            {"x": 2, "w": L["down"], "codec": "q6_k"}], out_dtype=torch.float32)
    else:
        qkv = kq.quantized_matmul(x, L["qkv"], None, "q4_k", out_dtype=torch.float32)
        o = kq.quantized_matmul(a, L["o"], None, "q4_k", out_dtype=torch.float32)
        h = kq.quantized_glu(x, L["gate"], L["up"], "q4_k", act="silu")
        y = kq.quantized_matmul(h, L["down"], None, "q6_k", out_dtype=torch.float32)
    xf, af = x.float(), a.float()
    gt = xf @ _deq(kq, L["gate"], "q4_k").t()
    ut = xf @ _deq(kq, L["up"], "q4_k").t()
    errs = {"qkv": _rel(qkv, xf @ _deq(kq, L["qkv"], "q4_k").t()),
            "o": _rel(o, af @ _deq(kq, L["o"], "q4_k").t()),
            "gate_up": _rel(h, torch.nn.functional.silu(gt) * ut),
            "down": _rel(y, h.float() @ _deq(kq, L["down"], "q6_k").t())}
    torch.cuda.empty_cache()
    return {"max_rel_err": max(errs.values()), "per_projection": errs, "tolerance": 1e-2,
            "reference": "kq.dequantize (f32) then torch f32 matmul, TF32 off"}

MOE_CONFIGS = (
    # (name, experts, top_k, hidden, ffn, gate/up codec, down codec, token counts)
    ("qwen3-30b-a3b-like", 128, 8, 2048, 768, "q4_k", "q6_k", (1, 64, 4096)),
    ("deepseek-v3-like-iq2", 256, 8, 7168, 2048, "iq2_xxs", "iq2_xxs", (1, 8, 64)),
)


def moe_check(torch, kq, x, idx, sc, y, wg, wu, wd, cgu, cd, base, toks):
    """Max relative error of an expert layer's output rows `toks` (this rank's
    experts [base, base + len(wg))) against f32 dequantization + f32 torch
    matmuls, with the gate/up product rounded to the activation dtype as the
    layer keeps it."""
    torch.backends.cuda.matmul.allow_tf32 = False
    el = wg.shape[0]
    ref = torch.zeros(len(toks), wd.shape[1], device=x.device)
    ic, scc = idx.cpu(), sc.cpu()
    for r, t in enumerate(toks):
        xt = x[t].float()
        for j in range(ic.shape[1]):
            e = int(ic[t, j]) - base
            if not 0 <= e < el:
                continue
            g = _deq(kq, wg[e], cgu) @ xt
            u = _deq(kq, wu[e], cgu) @ xt
            h = (torch.nn.functional.silu(g) * u).to(x.dtype).float()
            ref[r] += float(scc[t, j]) * (_deq(kq, wd[e], cd) @ h)
    return _rel(y[toks], ref) if ref.abs().max() > 0 else 0.0


def expert_stack(torch, codec, n, k, seed, e0, e1, dev):
    """Experts [e0, e1) of a seeded synthetic stack, each expert from its own
    seed, so every rank builds only the experts it owns and the values do not
    depend on the world size."""
    from gmlx_b200 import synth
    return torch.stack([torch.from_numpy(synth.random_weight(codec, n, k, seed=seed * 100_000 + e)).to(dev)
                        for e in range(e0, e1)])


def run_moe(torch, kq, dist, dev, world, rank, stream, hbm_peak):
    """Expert-parallel routed expert layer (configs 4 and 5), experts split by
    id range over ranks.  Reported per token count: layer ms (max over ranks)
    and GB/s of the expert bytes the routing touched (unique experts x expert
    bytes).  Two ways to move tokens at N > 1:
      allreduce -- every rank routes all T tokens, runs its experts' slots,
                   partial outputs summed with one all-reduce (graph-timed):
                   the one-shot peer-memory kernel (kq.all_reduce) up to
                   64 x 7168 values, NCCL above;
      alltoall  -- each rank routes its own T / N tokens and sends the routed
                   rows to the experts' owners and back (NCCL all-to-all with
                   host-side split sizes, so timed eagerly with CUDA events)."""
    from gmlx_b200 import parallel as par
    out = {}
    comm = par.PeerComm(64 * 7168, dev) if world > 1 else None
    for name, E, K, D, F, cgu, cd, ts in MOE_CONFIGS:
        el = E // world
        base = rank * el
        wg = expert_stack(torch, cgu, F, D, 11, base, base + el, dev)
        wu = expert_stack(torch, cgu, F, D, 12, base, base + el, dev)
        wd = expert_stack(torch, cd, D, F, 13, base, base + el, dev)
        router_w = torch.randn(E, D, device=dev, generator=torch.Generator(device=dev).manual_seed(5)) / D ** 0.5
        ebytes = (wg[0].numel() + wu[0].numel() + wd[0].numel())
        cell = {}
        for t in ts:
            x = torch.randn(t, D, device=dev, generator=torch.Generator(device=dev).manual_seed(t)).to(torch.bfloat16)
            logits = x.float() @ router_w.t()

            def layer():
                idx, sc = kq.moe_router_topk(logits, K, True, shared_gate=False)
                y = kq.moe_expert_layer_local(x, idx, sc, wg, wu, wd, cgu, cd, base, E, out_dtype=torch.float32)
                if world > 1 and y.numel() <= comm.n:
                    kq.all_reduce(y, comm)
                elif world > 1:
                    dist.all_reduce(y)
                return idx
            idx = layer()
            uniq = int(torch.unique(idx).numel())
            reps = 20
            secs = time_graph(torch, layer, reps, 3, stream) / reps
            tt = torch.tensor([secs], device=dev, dtype=torch.float64)
            if world > 1:
                dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            secs = float(tt.item())
            gbs = uniq * ebytes / secs / 1e9
            # parity of this cell, outside the timed region: this rank's share of
            # the layer for up to 8 sampled tokens against f32 dequantization
            idx, sc = kq.moe_router_topk(logits, K, True, shared_gate=False)
            yl = kq.moe_expert_layer_local(x, idx, sc, wg, wu, wd, cgu, cd, base, E, out_dtype=torch.float32)
            toks = torch.randperm(t, generator=torch.Generator().manual_seed(t))[:8].tolist()
            err = moe_check(torch, kq, x, idx, sc, yl, wg, wu, wd, cgu, cd, base, toks)
            c = {"ms": secs * 1e3, "unique_experts": uniq, "GB/s": gbs, "frac_hbm_per_gpu": gbs / world / hbm_peak,
                 "TFLOP/s": 2.0 * t * K * 3 * D * F / secs / 1e12, "rel_err": err, "rel_err_tokens_checked": len(toks)}
            if world > 1:
                c = {"allreduce": c, "alltoall": moe_alltoall_cell(torch, kq, dist, par, x, logits, K, wg, wu, wd,
                                                                   cgu, cd, E, world, rank, dev, uniq, ebytes,
                                                                   hbm_peak)}
                c["alltoall"]["rel_err_vs_allreduce"] = moe_a2a_vs_allreduce(torch, kq, dist, par, x, logits, K, wg,
                                                                             wu, wd, cgu, cd, E, world, rank, base)
            cell[f"t{t}"] = c
        out[name] = cell
        del wg, wu, wd
        torch.cuda.empty_cache()
    if comm is not None:
        dist.barrier()
        comm.close()
    return out


def _local_tokens(t, world, rank):
    per, extra = divmod(t, world)
    t0 = rank * per + min(rank, extra)
    return t0, t0 + per + (1 if rank < extra else 0)


def moe_alltoall_cell(torch, kq, dist, par, x, logits, K, wg, wu, wd, cgu, cd, E, world, rank, dev, uniq, ebytes,
                      hbm_peak):
    """Time the all-to-all expert-parallel layer: this rank's share of the T
    tokens, routed, dispatched, computed by the experts' owners, combined."""
    t0, t1 = _local_tokens(x.shape[0], world, rank)
    xl, ll = x[t0:t1].contiguous(), logits[t0:t1].contiguous()

    def layer():
        return par.ep_moe_alltoall(xl, ll, K, wg, wu, wd, cgu, cd, E)
    for _ in range(3):
        layer()
    torch.cuda.synchronize()
    dist.barrier()
    reps = 20
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        layer()
    b.record()
    torch.cuda.synchronize()
    tt = torch.tensor([a.elapsed_time(b) / 1e3 / reps], device=dev, dtype=torch.float64)
    dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    secs = float(tt.item())
    gbs = uniq * ebytes / secs / 1e9
    return {"ms": secs * 1e3, "GB/s": gbs, "frac_hbm_per_gpu": gbs / world / hbm_peak,
            "tokens_per_rank": [_local_tokens(x.shape[0], world, r)[1] - _local_tokens(x.shape[0], world, r)[0]
                                for r in range(world)]}


def moe_a2a_vs_allreduce(torch, kq, dist, par, x, logits, K, wg, wu, wd, cgu, cd, E, world, rank, base):
    """Max relative difference (over ranks) between the all-to-all layer's
    rows and the all-reduce layer's rows for the same tokens (the latter is
    checked against f32 dequantization per rank)."""
    idx, sc = kq.moe_router_topk(logits, K, True, shared_gate=False)
    yf = kq.moe_expert_layer_local(x, idx, sc, wg, wu, wd, cgu, cd, base, E, out_dtype=torch.float32)
    dist.all_reduce(yf)
    t0, t1 = _local_tokens(x.shape[0], world, rank)
    ya = par.ep_moe_alltoall(x[t0:t1].contiguous(), logits[t0:t1].contiguous(), K, wg, wu, wd, cgu, cd, E)
    e = torch.tensor([float((ya - yf[t0:t1]).abs().max() / yf.abs().max().clamp_min(1e-30)) if t1 > t0 else 0.0],
                     device=x.device, dtype=torch.float64)
    dist.all_reduce(e, op=dist.ReduceOp.MAX)
    return float(e.item())


_CPU_LAYER = None


def _cpu_layer():
    """One Llama-3-8B Q4_K_M layer (the seven projections) and its inputs, host side."""
    global _CPU_LAYER
    if _CPU_LAYER is None:
        from gmlx_b200 import synth
        w = {name: (codec, synth.random_weight(codec, n, k, seed=500 + i))
             for i, (name, codec, n, k) in enumerate(synth.LLAMA3_8B_LAYER)}
        x = synth.random_activations(1, 4096, seed=3)
        h = synth.random_activations(1, 14336, seed=4)
        _CPU_LAYER = (w, x, h)
    return _CPU_LAYER


def cpu_baseline_run(seconds=12.0, threads=None):
    """C oracle dequantize-then-matmul (OpenMP, all host threads) on the GPU
    arm's per-layer workload: the seven projections of one layer at M = 1,
    repeated for `seconds`; the median layer time gives the rate."""
    from oracle import oracle as O
    O.build()
    thr = threads or os.cpu_count() or 1
    w, x, h = _cpu_layer()

    def layer():
        for name, (codec, wb) in w.items():
            O.matmul(h if name == "down_proj" else x, wb, codec, threads=thr)
    layer()
    times, t0 = [], time.perf_counter()
    while time.perf_counter() - t0 < seconds or len(times) < 3:
        t1 = time.perf_counter()
        layer()
        times.append(time.perf_counter() - t1)
    med = statistics.median(times)
    return {"value": LAYER_WEIGHT_BYTES / med / 1e9, "unit": UNIT, "cores": thr, "kind": "port",
            "os_cpu_count": os.cpu_count(),
            "sample": f"{len(times)} x one Llama-3-8B Q4_K_M layer (7 projections, 137.8 MB of weights) at M=1, "
                      f"median {med * 1e3:.1f} ms, C oracle dequantize-then-matmul (OpenMP, {thr} threads)"}


def cpu_gguf_arm(reps=3):
    """gguf-py arm: gguf.quants.dequantize (the ggml formats' Python reference,
    a declared gmlx dependency) to f32 W, then x @ W.T in torch on the CPU;
    dequantize and matmul timed separately over one full layer, median of
    `reps` warm repetitions."""
    import torch
    try:
        import gguf.quants as gq
        from gguf.constants import GGMLQuantizationType as T
    except ImportError as e:
        return {"unavailable": f"gguf-py not importable: {e}"}
    qt = {"q4_k": T.Q4_K, "q6_k": T.Q6_K}
    w, x, h = _cpu_layer()
    xt = torch.from_numpy(x.view(np.int16).copy()).view(torch.bfloat16).float()
    ht = torch.from_numpy(h.view(np.int16).copy()).view(torch.bfloat16).float()
    deq_t, mm_t = [], []
    for r in range(reps + 1):
        td = tm = 0.0
        for name, (codec, wb) in w.items():
            t0 = time.perf_counter()
            W = torch.from_numpy(gq.dequantize(wb, qt[codec]))
            t1 = time.perf_counter()
            _ = (ht if name == "down_proj" else xt) @ W.t()
            t2 = time.perf_counter()
            td += t1 - t0
            tm += t2 - t1
        if r:  # the first pass warms up
            deq_t.append(td)
            mm_t.append(tm)
    d, m = statistics.median(deq_t), statistics.median(mm_t)
    return {"value": LAYER_WEIGHT_BYTES / (d + m) / 1e9, "unit": UNIT, "dequant_s": d, "matmul_s": m,
            "total_s": d + m, "dequant_GB/s": LAYER_WEIGHT_BYTES / d / 1e9,
            "os_cpu_count": os.cpu_count(), "torch_threads": torch.get_num_threads(),
            "sample": f"median of {reps} x one Llama-3-8B Q4_K_M layer at M=1 (gguf-py dequantize, numpy; "
                      "torch CPU matmul)"}


def run_reference(args, rank, world):
    if rank != 0:
        return
    res = []
    for _ in range(args.warmup):
        cpu_baseline_run(seconds=1.0)
    for _ in range(args.steps):
        res.append(cpu_baseline_run(seconds=max(1.0, 30.0 / max(1, args.steps))))
    v = statistics.median(r["value"] for r in res)
    cb = dict(res[0])
    cb["value"] = v
    line = {"metric": METRIC, "value": v, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "llama3-8b Q4_K_M decode step (32 layers; CPU sample: whole layers)", "m": 1},
            "cpu_baseline": cb,
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--m", type=int, default=1)
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-moe", action="store_true")
    ap.add_argument("--fused-allreduce", action="store_true", help="same as --allreduce fused")
    ap.add_argument("--allreduce", default="peer", choices=["peer", "nccl", "fused"],
                    help="cross-rank sum of the row-parallel decode projections (N > 1)")
    ap.add_argument("--chain", action="store_true", help="one chain launch per layer instead of one launch per op")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch
    import torch.distributed as dist

    from gmlx_b200 import _lib, kq
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    _lib.load()
    hbm_peak, tc_peak, peak_kind = _peaks()

    layers = build_layers(dev, N_LAYERS, world, rank)
    stream = torch.cuda.Stream(dev)
    dd = dist if world > 1 else None
    ka = 4096 // world  # this rank's slice of the attention output (o_proj K)
    from gmlx_b200 import parallel as par
    # cross-rank sum of the row-parallel o/down outputs: "peer" (default) the
    # one-shot all-reduce kernel over NVLink peer memory after each GEMV;
    # "fused" inside their GEMV kernels (M = 1); "nccl" NCCL all-reduce
    ar = "fused" if args.fused_allreduce else args.allreduce
    comm = par.PeerComm(32 * 4096, dev) if (world > 1 and ar != "nccl") else None
    # headline launch structure: one kq op per projection group (measured the
    # faster of the two on B200); --chain times the single persistent chain launch
    head_mode = "chain" if (args.m == 1 and comm is None and args.chain) else "ops"

    def measure(m, steps, warmup, mode, min_warm_s=0.0):
        """Seconds per decode step (one token through all N_LAYERS layers),
        timed over exactly `steps` replays of the step's CUDA graph."""
        g = torch.Generator(device="cpu").manual_seed(0)
        xs = [torch.randn(m, 4096, generator=g).to(torch.bfloat16).to(dev) for _ in range(N_LAYERS)]
        att = [x[:, :ka].contiguous() for x in xs]

        def one_step():
            for li, L in enumerate(layers):
                layer_step(kq, L, xs[li], att[li], dd, comm, mode, ar)
        return time_graph(torch, one_step, steps, warmup, stream, min_warm_s) / steps

    # timed region (headline), with clock sampling and barrier + max over ranks
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        t_step = measure(args.m, args.steps, args.warmup, head_mode, min_warm_s=1.0)
    tt = torch.tensor([t_step], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    t_step = float(tt.item())
    nbytes = N_LAYERS * step_bytes(args.m)
    value = nbytes / t_step / 1e9  # all layers' bytes (strong scaling: each layer is split over ranks)

    # parity of one step's outputs at these full shapes, outside the timed region
    check = verify_layer(torch, kq, layers[0], args.m, dev, head_mode, ka)

    # dominant kernel: the chain launch (one layer) or, per op, the fused
    # gate/up GEMV; its average launch duration over many launches
    if head_mode == "chain":
        per_launch = t_step / N_LAYERS
        dom_bytes = nbytes // N_LAYERS // world
        kernel_name = "chain_kernel<Q4_K,Q6_K> (one layer: q|k|v, o, gate+up, down in one launch)"
        traffic = CHAIN_LAUNCH_DRAM_BYTES if world == 1 else None
    else:
        x = torch.randn(args.m, 4096, device=dev).to(torch.bfloat16)

        def glu_pass():
            for L in layers:
                kq.quantized_glu(x, L["gate"], L["up"], "q4_k", act="silu")
        reps = 4
        per_launch = time_graph(torch, glu_pass, reps, 2, stream) / (reps * N_LAYERS)
        dom_bytes = 2 * (14336 // world) * 2304 + args.m * 4096 * 2 + args.m * (14336 // world) * 2
        kernel_name = "gemv_kernel<Q4_K, GLU> (gate+up 14336x4096)"
        traffic = GLU_LAUNCH_DRAM_BYTES if (world == 1 and args.m == 1) else None
    achieved = dom_bytes / per_launch / 1e9

    # e2e through the public op API: pinned host input -> device, one token
    # through every layer, output -> host, all inside the timed region
    hx = torch.randn(args.m, 4096).to(torch.bfloat16).pin_memory()
    hy = torch.empty(args.m, 4096, dtype=torch.bfloat16).pin_memory()

    def e2e_step():
        dx = hx.to(dev, non_blocking=True)
        y = dx
        for L in layers:
            _, _, y = layer_step(kq, L, dx, dx[:, :ka].contiguous(), dd, comm, head_mode, ar)
        hy.copy_(y, non_blocking=True)
    for _ in range(args.warmup):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ea, eb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ea.record()
    for _ in range(args.steps):
        e2e_step()
    eb.record()
    torch.cuda.synchronize()
    e2e_t = ea.elapsed_time(eb) / 1e3 / args.steps
    te = torch.tensor([e2e_t], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_t = float(te.item())

    # the other decode launch structures at M = 1 (same work per step)
    modes = {}
    if not args.no_sweep and args.m == 1:
        for mode in ("ops", "chain", "chain_dep"):
            if (mode == "chain_dep" and world > 1) or (comm is not None and mode != "ops"):
                continue
            tm = measure(1, 10, 3, mode)
            if world > 1:
                tt = torch.tensor([tm], device=dev, dtype=torch.float64)
                dist.all_reduce(tt, op=dist.ReduceOp.MAX)
                tm = float(tt.item())
            modes[mode] = {"ms_per_step": tm * 1e3, "us_per_layer": tm / N_LAYERS * 1e6,
                           "GB/s": N_LAYERS * step_bytes(1) / tm / 1e9,
                           "frac_hbm": N_LAYERS * step_bytes(1) / tm / 1e9 / world / hbm_peak}

    sweep = {}
    if not args.no_sweep:
        for m in (1, 4, 16, 32):
            mode = head_mode if m == 1 else "ops"
            ts = measure(m, 10, 3, mode)
            if world > 1:
                tt = torch.tensor([ts], device=dev, dtype=torch.float64)
                dist.all_reduce(tt, op=dist.ReduceOp.MAX)
                ts = float(tt.item())
            gbs = N_LAYERS * step_bytes(m) / ts / 1e9
            sweep[f"m{m}"] = {"ms_per_step": ts * 1e3, "us_per_layer": ts / N_LAYERS * 1e6, "GB/s": gbs,
                              "frac_hbm": gbs / world / hbm_peak, "launch": mode}

    # prefill: the layer's matmuls (qkv | o | gate+up concatenated | down) at
    # M = 512 / 2048 / 8192 tokens on the tcgen05 GEMM, TFLOP/s over 2*M*N*K
    prefill = {}
    if not args.no_sweep:
        L0 = layers[0]
        # this rank's shards (tensor parallel: o and down split along K, the
        # others along N); K from the wire row length
        kof = {"q4_k": 144, "q6_k": 210}
        mats = [(L0[n], c, L0[n].shape[1] // kof[c] * 256) for n, c in
                (("qkv", "q4_k"), ("o", "q4_k"), ("gate", "q4_k"), ("up", "q4_k"), ("down", "q6_k"))]
        flops_per_tok = sum(2 * w.shape[0] * k for w, _, k in mats)  # this rank's share
        k_in, k_o, k_down = mats[0][2], mats[1][2], mats[4][2]
        for m in (512, 2048, 8192):
            xs = {k: torch.randn(m, k, device=dev).to(torch.bfloat16) for k in {k_in, k_o, k_down}}

            def pf():  # gate/up/SiLU*up fused in one tcgen05 GEMM (two accumulators per tile)
                kq.quantized_matmul(xs[k_in], L0["qkv"], None, "q4_k")
                o = kq.quantized_matmul(xs[k_o], L0["o"], None, "q4_k")
                kq.quantized_glu(xs[k_in], L0["gate"], L0["up"], "q4_k", act="silu")
                y = kq.quantized_matmul(xs[k_down], L0["down"], None, "q6_k")
                if dd is not None:  # row-parallel partial sums over ranks (bf16, NCCL)
                    dist.all_reduce(o)
                    dist.all_reduce(y)
            reps = 3 if m == 8192 else 6
            t = time_graph(torch, pf, reps, 1, stream) / reps
            if dd is not None:  # slowest rank; every rank computes its own shard
                tt = torch.tensor([t], device=dev)
                dist.all_reduce(tt, op=dist.ReduceOp.MAX)
                t = float(tt.item())
            tflops = flops_per_tok * world * m / t / 1e12  # whole job
            # parity of this cell (outside the timed region): 64 sampled rows of
            # every product against f32 dequantization + f32 torch matmul
            rows = torch.randperm(m, generator=torch.Generator().manual_seed(m))[:64].to(dev)
            errs = {}
            for name, w, c, xin in (("qkv", L0["qkv"], "q4_k", xs[k_in]), ("o", L0["o"], "q4_k", xs[k_o]),
                                    ("down", L0["down"], "q6_k", xs[k_down])):
                yv = kq.quantized_matmul(xin, w, None, c, out_dtype=torch.float32)[rows]
                errs[name] = _rel(yv, xin[rows].float() @ _deq(kq, w, c).t())
            hv = kq.quantized_glu(xs[k_in], L0["gate"], L0["up"], "q4_k", act="silu", out_dtype=torch.float32)[rows]
            xr = xs[k_in][rows].float()
            errs["gate_up"] = _rel(hv, torch.nn.functional.silu(xr @ _deq(kq, L0["gate"], "q4_k").t())
                                   * (xr @ _deq(kq, L0["up"], "q4_k").t()))
            torch.cuda.empty_cache()
            prefill[f"m{m}"] = {"ms": t * 1e3, "TFLOP/s": tflops, "frac_tensor": tflops / world / tc_peak,
                                "rel_err": max(errs.values()), "rel_err_rows_checked": 64}

    moe = {} if args.no_moe else run_moe(torch, kq, dist, dev, world, rank, stream, hbm_peak)

    if rank == 0:
        cpu = None if args.no_cpu or world > 1 else cpu_baseline_run()
        cpu_arms = None if args.no_cpu or world > 1 else {"c_oracle_openmp": cpu, "gguf_py_torch_cpu": cpu_gguf_arm()}
        launches_per_layer = 1 if head_mode == "chain" else 4
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t_step * 1e3, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "llama3-8b Q4_K_M decode step: one token through 32 decoder layers "
                                   "(q/k/v/o/gate/up Q4_K, down Q6_K)",
                       "m": args.m, "layers": N_LAYERS, "weight_bytes_per_layer": LAYER_WEIGHT_BYTES,
                       "weight_bytes_per_step": N_LAYERS * LAYER_WEIGHT_BYTES,
                       "launch": ("one chain launch per layer (q|k|v, o, gate+up, down)" if head_mode == "chain"
                                  else "one launch per projection group (q|k|v, o, gate+up, down)"),
                       "l2": "inputs larger than L2 (32 distinct layers, 4.41 GB per step)",
                       "parallelism": (f"tp{world} (column-parallel qkv/gate/up, row-parallel o/down, "
                                       + {"fused": "cross-rank sum fused into their GEMV kernels over NVLink peer stores)",
                                          "peer": "one-shot all-reduce kernel over NVLink peer memory)",
                                          "nccl": "NCCL all-reduce)"}[ar]) if world > 1 else "single"},
            "frac_hbm": value / world / hbm_peak,
            "us_per_layer": t_step / N_LAYERS * 1e6,
            "rel_err": check["max_rel_err"], "parity": check,
            "decode_launch_modes": modes,
            "moe": moe,
            "roofline": {"bound": "hbm", "kernel": kernel_name,
                         "achieved": achieved, "peak": hbm_peak, "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": achieved / hbm_peak,
                         "algorithmic_bytes_per_launch": dom_bytes,
                         # dram__bytes_read.sum + dram__bytes_write.sum of this launch at this
                         # shape from an ncu capture (profiles/)
                         "traffic": traffic, "traffic_unit": "bytes per launch"},
            "cpu_baseline": cpu,
            "cpu_baseline_arms": cpu_arms,
            "e2e": {"value": nbytes / e2e_t / 1e9, "unit": UNIT,
                    "h2d_bytes_per_step": int(hx.numel() * 2), "d2h_bytes_per_step": int(hy.numel() * 2)},
            "gpu_launches": launches_per_layer * N_LAYERS * args.steps,
            "clocks": clk.summary(),
            "sweep": sweep,
            "prefill": prefill,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
