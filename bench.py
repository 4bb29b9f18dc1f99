"""Benchmark: K-quant decode GEMV over a Llama-3-8B Q4_K_M decoder layer on B200.

Workload: the seven projections of one Llama-3-8B
layer -- q/k/v/o/gate/up in Q4_K, down in Q6_K (137,822,208 wire bytes) --
applied to M bf16 activation rows (M=1 headline; M in {4, 16, 32} reported
under ``sweep``).  One step = one layer forward through the kq ops:

    qkv   = quantized_matmul(x, Wqkv)            (row-concatenated q|k|v wire,
                                                  as gmlx/occupancy_fuse.py does)
    o     = quantized_matmul(x, Wo)
    h     = quantized_glu(x, Wgate, Wup, silu)    (gate+up+SiLU*up in one launch)
    y     = quantized_matmul(h, Wdown)            (Q6_K)

Eight distinct layers (1.10 GB) are cycled so every step streams weights that
are not resident in the 126 MB L2.  Weights and activations are seeded
synthetic data with the configuration's block statistics (no GGUF files on the
box).  ``value`` is device-timed (CUDA graph replay, CUDA events, max over
ranks); ``e2e`` goes through the public Python op API with the step input
copied from pinned host memory and the output read back every step.

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
N_LAYERS = 8
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


def layer_step(kq, L, x, a=None, dist=None, comm=None):
    """One decoder-layer pass of the seven quantized projections (4 launches).
    Under tensor parallelism the row-parallel o and down outputs are summed
    over ranks: at M=1 inside their GEMV kernels (peer stores over NVLink,
    `comm`), otherwise with NCCL all-reduces.  `a` stands in for this rank's
    slice of the attention output."""
    qkv = kq.quantized_matmul(x, L["qkv"], None, "q4_k")
    h = kq.quantized_glu(x, L["gate"], L["up"], "q4_k", act="silu")
    xa = x if a is None else a
    if comm is not None and x.shape[0] == 1:
        o = kq.quantized_matmul_allreduce(xa, L["o"], "q4_k", comm)
        y = kq.quantized_matmul_allreduce(h, L["down"], "q6_k", comm)
        return qkv, o, y
    o = kq.quantized_matmul(xa, L["o"], None, "q4_k")
    y = kq.quantized_matmul(h, L["down"], None, "q6_k")
    if dist is not None:
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


GLU_LAUNCH_DRAM_BYTES = 66_643_712  # ncu: fused gate/up GEMV, Q4_K 2 x 14336 x 4096, M = 1

MOE_CONFIGS = (
    # (name, experts, top_k, hidden, ffn, gate/up codec, down codec, token counts)
    ("qwen3-30b-a3b-like", 128, 8, 2048, 768, "q4_k", "q6_k", (1, 64, 4096)),
    ("deepseek-v3-like-iq2", 256, 8, 7168, 2048, "iq2_xxs", "iq2_xxs", (1, 8, 64)),
)


def run_moe(torch, kq, dist, dev, world, rank, stream, hbm_peak):
    """Expert-parallel routed expert layer (configs 4 and 5): experts split by
    id range over ranks, all ranks route the same tokens, partial outputs are
    all-reduced.  Reported per token count: layer ms (max over ranks) and GB/s
    of the expert bytes the routing touched (unique experts x expert bytes)."""
    from gmlx_b200 import synth
    out = {}
    for name, E, K, D, F, cgu, cd, ts in MOE_CONFIGS:
        el = E // world
        base = rank * el
        wg = torch.from_numpy(synth.random_weight(cgu, F, D, seed=11, experts=E)[base:base + el]).to(dev)
        wu = torch.from_numpy(synth.random_weight(cgu, F, D, seed=12, experts=E)[base:base + el]).to(dev)
        wd = torch.from_numpy(synth.random_weight(cd, D, F, seed=13, experts=E)[base:base + el]).to(dev)
        router_w = torch.randn(E, D, device=dev, generator=torch.Generator(device=dev).manual_seed(5)) / D ** 0.5
        ebytes = (wg[0].numel() + wu[0].numel() + wd[0].numel())
        cell = {}
        for t in ts:
            x = torch.randn(t, D, device=dev, generator=torch.Generator(device=dev).manual_seed(t)).to(torch.bfloat16)
            logits = x.float() @ router_w.t()

            def layer():
                idx, sc = kq.moe_router_topk(logits, K, True, shared_gate=False)
                y = kq.moe_expert_layer_local(x, idx, sc, wg, wu, wd, cgu, cd, base, E, out_dtype=torch.float32)
                if world > 1:
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
            cell[f"t{t}"] = {"ms": secs * 1e3, "unique_experts": uniq, "GB/s": gbs,
                             "frac_hbm_per_gpu": gbs / world / hbm_peak,
                             "TFLOP/s": 2.0 * t * K * 3 * D * F / secs / 1e12}
        out[name] = cell
        del wg, wu, wd
        torch.cuda.empty_cache()
    return out


def cpu_baseline_run(seconds=12.0, threads=None):
    """C oracle dequantize-then-matmul (all host threads) on a bounded sample:
    repeated q_proj-sized Q4_K layers (4096x4096) and the Q6_K down_proj at M=1."""
    from gmlx_b200 import synth
    from oracle import oracle as O
    O.build()
    thr = threads or os.cpu_count() or 1
    wq = synth.random_weight("q4_k", 4096, 4096, seed=1)
    wd = synth.random_weight("q6_k", 4096, 14336, seed=2)
    x1 = synth.random_activations(1, 4096, seed=3)
    x2 = synth.random_activations(1, 14336, seed=4)
    O.matmul(x1, wq, "q4_k", threads=thr)
    done, t0 = 0, time.perf_counter()
    nbytes = 0
    while time.perf_counter() - t0 < seconds:
        O.matmul(x1, wq, "q4_k", threads=thr)
        O.matmul(x2, wd, "q6_k", threads=thr)
        nbytes += wq.nbytes + wd.nbytes
        done += 1
    dt = time.perf_counter() - t0
    return {"value": nbytes / dt / 1e9, "unit": UNIT, "cores": thr, "kind": "port",
            "sample": f"{done} x (Q4_K 4096x4096 + Q6_K 4096x14336) GEMV at M=1, {dt:.1f} s, "
                      "C oracle dequantize-then-matmul (OpenMP)"}


def run_reference(args, rank, world):
    if rank != 0:
        return
    res = []
    for _ in range(args.warmup):
        cpu_baseline_run(seconds=1.0)
    for _ in range(args.steps):
        res.append(cpu_baseline_run(seconds=max(2.0, 30.0 / max(1, args.steps))))
    v = statistics.median(r["value"] for r in res)
    cb = dict(res[0])
    cb["value"] = v
    line = {"metric": METRIC, "value": v, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "llama3-8b Q4_K_M decoder layer decode GEMV (CPU sample)", "m": 1},
            "cpu_baseline": cb,
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--m", type=int, default=1)
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-moe", action="store_true")
    ap.add_argument("--fused-allreduce", action="store_true")
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
    # --fused-allreduce: row-parallel o/down with the cross-rank sum inside their
    # GEMV kernels (peer stores over NVLink); default: GEMV + NCCL all-reduce,
    # which measured faster at tp2 (2460 vs 1929 GB/s aggregate)
    comm = par.PeerComm(4096, dev) if (world > 1 and args.fused_allreduce) else None

    def measure(m, steps, warmup, min_warm_s=0.0):
        g = torch.Generator(device="cpu").manual_seed(0)
        xs = [torch.randn(m, 4096, generator=g).to(torch.bfloat16).to(dev) for _ in range(N_LAYERS)]
        att = [x[:, :ka].contiguous() for x in xs]

        def one_pass():
            for li, L in enumerate(layers):
                layer_step(kq, L, xs[li], att[li], dd, comm)
        reps = max(1, steps // N_LAYERS)
        secs = time_graph(torch, one_pass, reps, max(1, warmup // N_LAYERS), stream, min_warm_s)
        return secs / (reps * N_LAYERS)

    # timed region (headline), with clock sampling and barrier + max over ranks
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        t_step = measure(args.m, args.steps, args.warmup, min_warm_s=1.0)
    tt = torch.tensor([t_step], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    t_step = float(tt.item())
    nbytes = step_bytes(args.m)
    value = nbytes / t_step / 1e9  # the whole layer's bytes (strong scaling: the layer is split over ranks)

    # dominant kernel: the fused gate/up GLU GEMV (66 MB of the 138 MB step),
    # timed alone on its launch stream with CUDA events over many launches
    x = torch.randn(args.m, 4096, device=dev).to(torch.bfloat16)

    def glu_pass():
        for L in layers:
            kq.quantized_glu(x, L["gate"], L["up"], "q4_k", act="silu")
    reps = 6
    glu_t = time_graph(torch, glu_pass, reps, 2, stream) / (reps * N_LAYERS)
    glu_bytes = 2 * (14336 // world) * 2304 + args.m * 4096 * 2 + args.m * (14336 // world) * 2
    achieved = glu_bytes / glu_t / 1e9

    # e2e through the public op API: pinned host input -> device, layer, output -> host
    hx = torch.randn(args.m, 4096).to(torch.bfloat16).pin_memory()
    hy = torch.empty(args.m, 4096, dtype=torch.bfloat16).pin_memory()
    e2e_steps = max(args.steps, 16)
    torch.cuda.synchronize()
    for i in range(args.warmup):
        dx = hx.to(dev, non_blocking=True)
        _, _, y = layer_step(kq, layers[i % N_LAYERS], dx, dx[:, :ka], dd, comm)
        hy.copy_(y, non_blocking=True)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(e2e_steps):
        dx = hx.to(dev, non_blocking=True)
        _, _, y = layer_step(kq, layers[i % N_LAYERS], dx, dx[:, :ka].contiguous(), dd, comm)
        hy.copy_(y, non_blocking=True)
    b.record()
    torch.cuda.synchronize()
    e2e_t = a.elapsed_time(b) / 1e3 / e2e_steps
    te = torch.tensor([e2e_t], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_t = float(te.item())

    sweep = {}
    if not args.no_sweep:
        for m in (1, 4, 16, 32):
            ts = measure(m, 16, 8)
            sweep[f"m{m}"] = {"ms_per_step": ts * 1e3, "GB/s": step_bytes(m) / ts / 1e9,
                              "frac_hbm": step_bytes(m) / ts / 1e9 / hbm_peak}

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
                kq.quantized_matmul(xs[k_o], L0["o"], None, "q4_k")
                kq.quantized_glu(xs[k_in], L0["gate"], L0["up"], "q4_k", act="silu")
                kq.quantized_matmul(xs[k_down], L0["down"], None, "q6_k")
            reps = 3 if m == 8192 else 6
            t = time_graph(torch, pf, reps, 1, stream) / reps
            if dd is not None:  # slowest rank; every rank computes its own shard
                tt = torch.tensor([t], device=dev)
                dist.all_reduce(tt, op=dist.ReduceOp.MAX)
                t = float(tt.item())
            tflops = flops_per_tok * world * m / t / 1e12  # whole job
            prefill[f"m{m}"] = {"ms": t * 1e3, "TFLOP/s": tflops, "frac_tensor": tflops / world / tc_peak}

    moe = {} if args.no_moe else run_moe(torch, kq, dist, dev, world, rank, stream, hbm_peak)

    if rank == 0:
        cpu = None if args.no_cpu or world > 1 else cpu_baseline_run()
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t_step * 1e3, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "llama3-8b Q4_K_M decoder layer decode GEMV (q/k/v/o/gate/up Q4_K, down Q6_K)",
                       "m": args.m, "layers_cycled": N_LAYERS, "weight_bytes_per_step": LAYER_WEIGHT_BYTES,
                       "l2": "inputs larger than L2 (8 distinct layers, 1.10 GB, cycled)",
                       "parallelism": (f"tp{world} (column-parallel qkv/gate/up, row-parallel o/down, "
                                       + ("cross-rank sum fused into their GEMV kernels over NVLink peer stores)"
                                          if comm is not None else "NCCL all-reduce)")) if world > 1 else "single"},
            "frac_hbm": value / world / hbm_peak,
            "moe": moe,
            "roofline": {"bound": "hbm", "kernel": "gemv_kernel<Q4_K, GLU> (gate+up 14336x4096)",
                         "achieved": achieved, "peak": hbm_peak, "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": achieved / hbm_peak,
                         # dram__bytes_read.sum + dram__bytes_write.sum of this launch at this
                         # shape from an ncu capture (66.14 MB read + 0.51 MB written); the
                         # algorithmic bytes are 66.07 MB
                         "traffic": GLU_LAUNCH_DRAM_BYTES if (world == 1 and args.m == 1) else None,
                         "traffic_unit": "bytes per launch"},
            "cpu_baseline": cpu,
            "e2e": {"value": nbytes / e2e_t / 1e9, "unit": UNIT,
                    "h2d_bytes_per_step": int(hx.numel() * 2), "d2h_bytes_per_step": int(hy.numel() * 2)},
            "gpu_launches": 4 * args.steps,
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
