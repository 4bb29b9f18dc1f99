"""Profiler-capture harness (not collected by pytest): small, fixed invocations of single kq ops for profiler captures.

    python tests/profile_cases.py <case> [launches]

Each case builds seeded synthetic weights (the bench's shapes), runs the op
`launches` times (default 3) on cuda:0 and synchronizes.  Cases:
  glu_m1        fused gate/up GEMV, Q4_K 14336x4096 (x2), one activation row
  down_m1       Q6_K 4096x14336 GEMV, one row
  iq2_m1        IQ2_XXS 2048x7168 GEMV, one row (DeepSeek-like expert)
  prefill_glu   fused gate/up tcgen05 GEMM, Q4_K 14336x4096 (x2), M=2048
                (dequantized copy + B by TMA)
  prefill_glu_m512  the same at M=512 (Q4_K dequantized inside the GEMM
                from raw bytes brought in by TMA)
  prefill_down  Q6_K 4096x14336 GEMM, M=2048
  moe_prefill   Qwen3-like expert layer, T=512 (grouped GEMM path)
  moe_iq2_t64   DeepSeek-like IQ2_XXS expert layer (256 experts, top-8,
                hidden 7168, ffn 2048), T=64 decode (grouped MMA GEMV path)
  glu_m32       fused gate/up GEMV, Q4_K 14336x4096 (x2), 32 activation rows
  glu_m4        the same with 4 activation rows
  chain_layer   one Llama-3-8B Q4_K_M layer at M=1 in one chain launch
                (q|k|v, o, gate+up, down reading the gate/up output)
"""
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from gmlx_b200 import kq, synth  # noqa: E402


def _w(codec, n, k, seed, experts=None):
    return torch.from_numpy(synth.random_weight(codec, n, k, seed=seed, experts=experts)).cuda()


def _x(m, k):
    return torch.randn(m, k, device="cuda", generator=torch.Generator(device="cuda").manual_seed(0)).to(torch.bfloat16)


def build(case):
    if case == "glu_m1":
        g, u, x = _w("q4_k", 14336, 4096, 1), _w("q4_k", 14336, 4096, 2), _x(1, 4096)
        return lambda: kq.quantized_glu(x, g, u, "q4_k", act="silu")
    if case == "down_m1":
        w, x = _w("q6_k", 4096, 14336, 3), _x(1, 14336)
        return lambda: kq.quantized_matmul(x, w, None, "q6_k")
    if case == "iq2_m1":
        w, x = _w("iq2_xxs", 2048, 7168, 4), _x(1, 7168)
        return lambda: kq.quantized_matmul(x, w, None, "iq2_xxs")
    if case == "prefill_glu_m512":
        g, u, x = _w("q4_k", 14336, 4096, 1), _w("q4_k", 14336, 4096, 2), _x(512, 4096)
        return lambda: kq.quantized_glu(x, g, u, "q4_k", act="silu")
    if case == "prefill_glu":
        g, u, x = _w("q4_k", 14336, 4096, 1), _w("q4_k", 14336, 4096, 2), _x(2048, 4096)
        return lambda: kq.quantized_glu(x, g, u, "q4_k", act="silu")
    if case == "prefill_down":
        w, x = _w("q6_k", 4096, 14336, 3), _x(2048, 14336)
        return lambda: kq.quantized_matmul(x, w, None, "q6_k")
    if case == "moe_prefill":
        e, k, d, f, t = 128, 8, 2048, 768, 512
        wg, wu, wd = _w("q4_k", f, d, 11, e), _w("q4_k", f, d, 12, e), _w("q6_k", d, f, 13, e)
        x = _x(t, d)
        logits = torch.randn(t, e, device="cuda", generator=torch.Generator(device="cuda").manual_seed(1))
        idx, sc = kq.moe_router_topk(logits, k, True, shared_gate=False)
        return lambda: kq.moe_expert_layer_local(x, idx, sc, wg, wu, wd, "q4_k", "q6_k", 0, e)
    if case == "moe_iq2_t64":
        e, k, d, f, t = 256, 8, 7168, 2048, 64
        wg, wu, wd = _w("iq2_xxs", f, d, 11, e), _w("iq2_xxs", f, d, 12, e), _w("iq2_xxs", d, f, 13, e)
        x = _x(t, d)
        logits = torch.randn(t, e, device="cuda", generator=torch.Generator(device="cuda").manual_seed(1))
        idx, sc = kq.moe_router_topk(logits, k, True, shared_gate=False)
        return lambda: kq.moe_expert_layer_local(x, idx, sc, wg, wu, wd, "iq2_xxs", "iq2_xxs", 0, e)
    if case in ("glu_m32", "glu_m4"):
        g, u, x = _w("q4_k", 14336, 4096, 1), _w("q4_k", 14336, 4096, 2), _x(int(case[5:]), 4096)
        return lambda: kq.quantized_glu(x, g, u, "q4_k", act="silu")
    if case == "chain_layer":
        x = _x(1, 4096)
        qkv, o = _w("q4_k", 6144, 4096, 5), _w("q4_k", 4096, 4096, 6)
        g, u, d = _w("q4_k", 14336, 4096, 1), _w("q4_k", 14336, 4096, 2), _w("q6_k", 4096, 14336, 3)
        pr = [{"x": x, "w": qkv, "codec": "q4_k"}, {"x": x, "w": o, "codec": "q4_k"},
              {"x": x, "w": g, "w2": u, "act": "silu", "codec": "q4_k"}, {"x": 2, "w": d, "codec": "q6_k"}]
        return lambda: kq.quantized_matmul_chain(pr)
    raise SystemExit(f"unknown case {case!r}; see the module docstring")


def main(argv):
    if not argv:
        raise SystemExit(__doc__)
    fn = build(argv[0])
    for _ in range(int(argv[1]) if len(argv) > 1 else 3):
        fn()
    torch.cuda.synchronize()
    print("ok", argv[0])


if __name__ == "__main__":
    main(sys.argv[1:])
