"""GPU parity: the CUDA kernels (through the C ABI / kq ops) against the CPU
oracle on seeded synthetic blocks.

* dequantize: bit-exact (f32) with the oracle, which is pinned to gguf-py.
* matmul-shaped ops: max |y - ref| / max |ref| <= 1e-2 against the oracle's
  f32 dequantize-then-matmul; the decode kernels
  compute exact products and in practice land near 1e-3.
"""
import numpy as np
import pytest
import torch

from gmlx_b200 import kq, synth
from oracle import oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-2
CODECS = ["q4_k", "q5_k", "q6_k", "iq2_xxs", "q8_0", "iq3_xxs", "iq4_xs", "q4_0", "iq4_nl", "q2_k", "q3_k", "q4_1",
          "q5_0", "q5_1", "tq2_0", "mxfp4", "iq2_xs", "iq2_s", "iq3_s", "iq1_s", "iq1_m", "tq1_0", "nvfp4"]


def rel_err(y, ref):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30))


def to_dev_x(xbits, dev, dtype=torch.bfloat16):
    x = torch.from_numpy(xbits.view(np.int16).copy()).view(torch.bfloat16).to(dev)
    return x.to(dtype)


@pytest.mark.parametrize("codec", CODECS)
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_dequantize_bitexact(cuda, codec, dtype):
    w = synth.random_weight(codec, 96, 1024, seed=11)
    ref = O.dequantize(w, codec)
    out = kq.dequantize(torch.from_numpy(w).to(cuda), None, codec, dtype=dtype)
    got = out.float().cpu().numpy()
    if dtype == torch.float32:
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    else:
        assert np.array_equal(got, torch.from_numpy(ref).to(dtype).float().numpy())


@pytest.mark.parametrize("codec,rows,k", [("q4_k", 600, 4096), ("q6_k", 4000, 768), ("iq2_xxs", 1500, 1792)])
def test_dequantize_large_contiguous_bitexact(cuda, codec, rows, k):
    """Large contiguous weights take the chunked bulk-copy dequantizer
    (unaligned chunk starts for Q6_K 630-byte and IQ2_XXS 462-byte rows)."""
    w = synth.random_weight(codec, rows, k, seed=130)
    ref = O.dequantize(w, codec)
    wd = torch.from_numpy(w).to(cuda)
    out = kq.dequantize(wd, None, codec).cpu().numpy()
    assert np.array_equal(out.view(np.uint32), ref.view(np.uint32))
    bf = kq.dequantize(wd, None, codec, dtype=torch.bfloat16).float().cpu().numpy()
    assert np.array_equal(bf, torch.from_numpy(ref).to(torch.bfloat16).float().numpy())


@pytest.mark.parametrize("codec", CODECS)
@pytest.mark.parametrize("m", [1, 3, 8, 17, 32, 40])
@pytest.mark.parametrize("n,k", [(256, 1024), (200, 2048)])
def test_quantized_matmul(cuda, codec, m, n, k):
    w = synth.random_weight(codec, n, k, seed=5)
    x = synth.random_activations(m, k, seed=6)
    ref = O.matmul(x, w, codec)
    y = kq.quantized_matmul(to_dev_x(x, cuda), torch.from_numpy(w).to(cuda), None, codec)
    assert y.dtype == torch.bfloat16 and tuple(y.shape) == (m, n)
    assert rel_err(y.float().cpu().numpy(), ref) <= TOL


@pytest.mark.parametrize("codec,n,k", [
    ("q5_k", 19200, 512),
    ("q5_k", 256, 8192),
    ("q8_0", 19200, 512),
    ("q8_0", 512, 14336),
    ("iq3_xxs", 19200, 512),
    ("iq3_xxs", 512, 14336),
    ("iq4_xs", 4096, 4096),
    ("iq4_xs", 256, 8192),
    ("q4_0", 19200, 512),
    ("q4_0", 512, 14336),
    ("iq4_nl", 4096, 4096),
    ("q2_k", 19200, 512),
    ("q4_1", 19200, 512),
    ("tq2_0", 19200, 512),
    ("iq2_xs", 4096, 4096),
    ("iq2_s", 512, 14336),
    ("iq3_s", 19200, 512),
    ("iq1_s", 4096, 4096),
    ("iq1_m", 512, 14336),
    ("tq1_0", 19200, 512),
    ("nvfp4", 4096, 4096),
    ("mxfp4", 512, 14336),
    ("q5_0", 512, 14336),
    ("q5_1", 4096, 4096),
    ("q3_k", 512, 14336),
    ("q3_k", 4096, 4096),
    ("q4_k", 19200, 512),   # >= 2 tiles per CTA: whole tiles handed out dynamically
    ("q4_k", 4096, 4096),   # one whole tile per CTA (stages fit the ring)
    ("q4_k", 256, 8192),    # few tiles, long K: K split into dynamic chunks
    ("q6_k", 512, 14336),   # Q6_K K split (unaligned 210-byte blocks)
    ("q6_k", 6144, 1024),
])
@pytest.mark.parametrize("ksplit", [False, True])
def test_one_row_schedules(cuda, codec, n, k, ksplit, monkeypatch):
    """Decode (one activation row) schedules, each called three times in a row:
    the work counters the dynamic schedule uses must come back to zero.
    ksplit: dynamic K-chunk units instead of stream-K for few long tiles."""
    if ksplit:
        monkeypatch.setenv("KQ_GEMV_KSPLIT", "1")
    w = synth.random_weight(codec, n, k, seed=9)
    x = synth.random_activations(1, k, seed=10)
    ref = O.matmul(x, w, codec)
    wd, xd = torch.from_numpy(w).to(cuda), to_dev_x(x, cuda)
    for _ in range(3):
        y = kq.quantized_matmul(xd, wd, None, codec, out_dtype=torch.float32)
        assert rel_err(y.cpu().numpy(), ref) <= TOL
    wu = synth.random_weight(codec, n, k, seed=11)
    g, u = ref.astype(np.float64), O.matmul(x, wu, codec).astype(np.float64)
    h = kq.quantized_glu(xd, wd, torch.from_numpy(wu).to(cuda), codec, out_dtype=torch.float32)
    assert rel_err(h.cpu().numpy(), g / (1 + np.exp(-g)) * u) <= TOL
    assert kq.workspace_error() == 0


@pytest.mark.parametrize("codec", CODECS)
def test_quantized_matmul_f16_f32out(cuda, codec):
    w = synth.random_weight(codec, 128, 1024, seed=7)
    x = synth.random_activations(4, 1024, seed=8)
    ref = O.matmul(x, w, codec)
    y = kq.quantized_matmul(to_dev_x(x, cuda, torch.float16), torch.from_numpy(w).to(cuda), None, codec,
                            out_dtype=torch.float32)
    assert rel_err(y.cpu().numpy(), ref) <= TOL


@pytest.mark.parametrize("codec", CODECS)
def test_quantized_matmul_split_k(cuda, codec):
    # few rows, long K: the launcher splits K across CTAs (deterministic combine)
    w = synth.random_weight(codec, 64, 8192, seed=9)
    x = synth.random_activations(2, 8192, seed=10)
    ref = O.matmul(x, w, codec)
    wd, xd = torch.from_numpy(w).to(cuda), to_dev_x(x, cuda)
    y1 = kq.quantized_matmul(xd, wd, None, codec)
    y2 = kq.quantized_matmul(xd, wd, None, codec)
    assert torch.equal(y1, y2)
    assert rel_err(y1.float().cpu().numpy(), ref) <= TOL
    assert kq.workspace_error() == 0


@pytest.mark.parametrize("codec", CODECS)
def test_unaligned_row_pitch(cuda, codec):
    # K=768 (3 blocks): Q6_K rows of 630 B, IQ2_XXS rows of 198 B and IQ3_XXS rows of
    # 294 B are not 16-byte aligned
    if codec in ("q4_k", "q5_k"):
        pytest.skip("Q4_K / Q5_K rows are always 16-byte multiples")
    w = synth.random_weight(codec, 96, 768, seed=12)
    for m in (1, 5):  # the one-row path and the batched one
        x = synth.random_activations(m, 768, seed=13)
        ref = O.matmul(x, w, codec)
        y = kq.quantized_matmul(to_dev_x(x, cuda), torch.from_numpy(w).to(cuda), None, codec)
        assert rel_err(y.float().cpu().numpy(), ref) <= TOL


@pytest.mark.parametrize("codec", CODECS)
def test_quantized_glu(cuda, codec):
    n, k, m = 160, 1024, 3
    wg = synth.random_weight(codec, n, k, seed=21)
    wu = synth.random_weight(codec, n, k, seed=22)
    x = synth.random_activations(m, k, seed=23)
    g = O.matmul(x, wg, codec).astype(np.float64)
    u = O.matmul(x, wu, codec).astype(np.float64)
    ref = g / (1 + np.exp(-g)) * u
    y = kq.quantized_glu(to_dev_x(x, cuda), torch.from_numpy(wg).to(cuda), torch.from_numpy(wu).to(cuda), codec,
                         out_dtype=torch.float32)
    assert rel_err(y.cpu().numpy(), ref) <= TOL


def test_router_topk(cuda):
    lg = synth.random_logits(64, 128, seed=3)
    idx_ref, sc_ref = O.router_topk(lg, 8, True)
    idx, sc = kq.moe_router_topk(torch.from_numpy(lg).to(cuda), 8, True, shared_gate=False)
    assert np.array_equal(idx.cpu().numpy(), idx_ref)
    assert np.allclose(sc.cpu().numpy(), sc_ref, rtol=1e-5, atol=1e-7)


def test_router_topk_shared_gate_and_expert_scale(cuda):
    """The reference defaults: shared_gate=True reads the last logits column
    as the shared expert's gate (its sigmoid becomes score column k);
    per_expert_scale multiplies each picked score."""
    lg = synth.random_logits(64, 129, seed=4)
    idx_ref, sc_ref = O.router_topk(np.ascontiguousarray(lg[:, :128]), 8, True)
    idx, sc = kq.moe_router_topk(torch.from_numpy(lg).to(cuda), 8, True)
    assert tuple(idx.shape) == (64, 8) and tuple(sc.shape) == (64, 9)
    assert np.array_equal(idx.cpu().numpy(), idx_ref)
    sc = sc.cpu().numpy()
    assert np.allclose(sc[:, :8], sc_ref, rtol=1e-5, atol=1e-7)
    assert np.allclose(sc[:, 8], 1 / (1 + np.exp(-lg[:, 128].astype(np.float64))), rtol=1e-5, atol=1e-7)
    pes = np.random.default_rng(5).random(128).astype(np.float32) + 0.5
    idx2, sc2 = kq.moe_router_topk(torch.from_numpy(np.ascontiguousarray(lg[:, :128])).to(cuda), 8, True,
                                   shared_gate=False, per_expert_scale=torch.from_numpy(pes).to(cuda))
    assert np.array_equal(idx2.cpu().numpy(), idx_ref)
    assert np.allclose(sc2.cpu().numpy(), sc_ref * pes[idx_ref], rtol=1e-5, atol=1e-7)


def _moe_case(codec_gu, codec_d, e, d, f, t, k, seed):
    wg = synth.random_weight(codec_gu, f, d, seed=seed, experts=e)
    wu = synth.random_weight(codec_gu, f, d, seed=seed + 1, experts=e)
    wd = synth.random_weight(codec_d, d, f, seed=seed + 2, experts=e)
    x = synth.random_activations(t, d, seed=seed + 3)
    lg = synth.random_logits(t, e, seed=seed + 4)
    return wg, wu, wd, x, lg


@pytest.mark.parametrize("codec_gu,codec_d", [("q4_k", "q6_k"), ("iq2_xxs", "iq2_xxs"), ("q5_k", "q5_k"),
                                             ("q8_0", "q8_0"), ("iq3_xxs", "iq3_xxs"), ("iq4_xs", "iq4_xs"),
                                             ("q4_0", "iq4_nl"), ("q2_k", "q3_k"), ("q4_1", "q5_1"),
                                             ("q5_0", "q5_0"), ("mxfp4", "tq2_0"), ("iq2_xs", "iq2_s"),
                                             ("iq3_s", "iq3_s"), ("iq1_s", "iq1_m"),
                                             ("tq1_0", "tq1_0"), ("nvfp4", "nvfp4")])
@pytest.mark.parametrize("t", [1, 5])
def test_moe_decode_ops(cuda, codec_gu, codec_d, t):
    e, d, f, k = 16, 512, 256, 4
    wg, wu, wd, x, lg = _moe_case(codec_gu, codec_d, e, d, f, t, k, seed=40)
    idx, sc = O.router_topk(lg, k, True)
    # oracle: per-slot dense dequant-then-matmul
    h_ref = np.zeros((t, k, f))
    for ti in range(t):
        for j in range(k):
            ex = idx[ti, j]
            g = O.matmul(x[ti:ti + 1], wg[ex], codec_gu)[0].astype(np.float64)
            u = O.matmul(x[ti:ti + 1], wu[ex], codec_gu)[0].astype(np.float64)
            h_ref[ti, j] = g / (1 + np.exp(-g)) * u
    xd = to_dev_x(x, cuda)
    idd = torch.from_numpy(idx).to(cuda)
    h = kq.moe_glu_gather_kq(xd, torch.from_numpy(wg).to(cuda), torch.from_numpy(wu).to(cuda), codec_gu, idd)
    assert tuple(h.shape) == (t, k, f)
    assert rel_err(h.float().cpu().numpy(), h_ref) <= TOL
    # down projection per slot and mixed, from the kernel's own h (bf16)
    hb = synth.f32_to_bf16_bits(h.float().cpu().numpy())
    y_ref = np.zeros((t, k, d))
    for ti in range(t):
        for j in range(k):
            y_ref[ti, j] = O.matmul(hb[ti, j][None], wd[idx[ti, j]], codec_d)[0]
    wdd = torch.from_numpy(wd).to(cuda)
    ys = kq.gather_qmv_kq(h, wdd, codec_d, idd, out_dtype=torch.float32)
    assert rel_err(ys.cpu().numpy(), y_ref) <= TOL
    ym = kq.gather_qmv_mix_ns_kq(h, wdd, codec_d, idd, torch.from_numpy(sc).to(cuda), out_dtype=torch.float32)
    mix_ref = (y_ref * sc[..., None]).sum(1)
    assert rel_err(ym.cpu().numpy(), mix_ref) <= TOL
    assert kq.workspace_error() == 0


@pytest.mark.parametrize("codec", CODECS)
def test_gather_qmm(cuda, codec):
    e, n, kin, t, k = 8, 128, 512, 6, 2
    w = synth.random_weight(codec, n, kin, seed=60, experts=e)
    x = synth.random_activations(t, kin, seed=61)
    rng = np.random.default_rng(62)
    idx = rng.integers(0, e, size=(t, k)).astype(np.int32)
    ref = np.zeros((t, k, 1, n))
    for ti in range(t):
        for j in range(k):
            ref[ti, j, 0] = O.matmul(x[ti:ti + 1], w[idx[ti, j]], codec)[0]
    xd = to_dev_x(x, cuda).reshape(t, 1, 1, kin)
    y = kq.gather_qmm(xd, torch.from_numpy(w).to(cuda), None, codec, rhs_indices=torch.from_numpy(idx).to(cuda),
                      out_dtype=torch.float32)
    assert tuple(y.shape) == (t, k, 1, n)
    assert rel_err(y.cpu().numpy(), ref) <= TOL


@pytest.mark.parametrize("codec", CODECS)
def test_golden_vectors_on_gpu(cuda, codec):
    """Kernels against the committed gguf-py golden vectors (edge blocks included)."""
    import os
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden_blocks.npz"))
    w, deq, x, yref = g[f"{codec}_w"], g[f"{codec}_deq"], g[f"{codec}_x"], g[f"{codec}_y"]
    wd = torch.from_numpy(w).to(cuda)
    out = kq.dequantize(wd, None, codec).cpu().numpy()
    assert np.array_equal(out.view(np.uint32), deq.view(np.uint32))
    y = kq.quantized_matmul(to_dev_x(x, cuda), wd, None, codec, out_dtype=torch.float32).cpu().numpy()
    assert rel_err(y, yref) <= TOL


def test_nn_modules_fused_and_stock_paths_agree(cuda):
    """KQuantSwitchGLU's fused decode path and its stock gather path both match
    the oracle (each output is bf16, so each is checked against f64 separately)."""
    from gmlx_b200 import nn as knn
    e, d, f, k, t = 8, 512, 256, 2, 3
    wg = synth.random_weight("q4_k", f, d, seed=1, experts=e)
    wu = synth.random_weight("q4_k", f, d, seed=2, experts=e)
    wd = synth.random_weight("q6_k", d, f, seed=3, experts=e)
    m = knn.KQuantSwitchGLU(d, f, e, "q4_k", "q6_k", device=cuda)
    m.gate_proj.weight.copy_(torch.from_numpy(wg))
    m.up_proj.weight.copy_(torch.from_numpy(wu))
    m.down_proj.weight.copy_(torch.from_numpy(wd))
    xb = synth.random_activations(t, d, seed=4)
    x = to_dev_x(xb, cuda)
    idx, sc = kq.moe_router_topk(torch.from_numpy(synth.random_logits(t, e, seed=5)).to(cuda), k, True, shared_gate=False)
    y_fused = m(x, idx, sc).float().cpu().numpy()
    y_stock = m(x.repeat(32, 1), idx.repeat(32, 1), sc.repeat(32, 1))[:t].float().cpu().numpy()  # >= 64 slots
    ii, ss = idx.cpu().numpy(), sc.cpu().numpy()
    ref = np.zeros((t, d))
    for ti in range(t):
        for j in range(k):
            ex = ii[ti, j]
            g = O.matmul(xb[ti:ti + 1], wg[ex], "q4_k")[0].astype(np.float64)
            u = O.matmul(xb[ti:ti + 1], wu[ex], "q4_k")[0].astype(np.float64)
            hb = synth.f32_to_bf16_bits((g / (1 + np.exp(-g)) * u).astype(np.float32))[None]
            ref[ti] += ss[ti, j] * O.matmul(hb, wd[ex], "q6_k")[0]
    assert rel_err(y_fused, ref) <= TOL
    assert rel_err(y_stock, ref) <= TOL
    lin = knn.KQuantLinear(d, 128, True, "iq2_xxs", device=cuda)
    lin.weight.copy_(torch.from_numpy(synth.random_weight("iq2_xxs", 128, d, seed=4)))
    lin.bias.fill_(0.5)
    xl = synth.random_activations(2, d, seed=5)
    refl = O.matmul(xl, lin.weight.cpu().numpy(), "iq2_xxs") + 0.5
    assert rel_err(lin(to_dev_x(xl, cuda)).float().cpu().numpy(), refl) <= TOL



@pytest.mark.parametrize("codec", CODECS)
@pytest.mark.parametrize("m,n,k", [(64, 256, 512), (200, 320, 1024), (1000, 512, 2048), (4200, 128, 512)])
def test_prefill_gemm_tcgen05(cuda, codec, m, n, k):
    """Prefill-sized M runs the tcgen05 GEMM (weights rounded to bf16 before the MMA)."""
    w = synth.random_weight(codec, n, k, seed=31)
    x = synth.random_activations(m, k, seed=32)
    ref = O.matmul(x, w, codec)
    y = kq.quantized_matmul(to_dev_x(x, cuda), torch.from_numpy(w).to(cuda), None, codec, out_dtype=torch.float32)
    assert rel_err(y.cpu().numpy(), ref) <= TOL
    y16 = kq.quantized_matmul(to_dev_x(x, cuda, torch.float16), torch.from_numpy(w).to(cuda), None, codec)
    assert y16.dtype == torch.float16
    assert rel_err(y16.float().cpu().numpy(), ref) <= TOL


@pytest.mark.parametrize("codec", CODECS)
@pytest.mark.parametrize("act", ["silu", "gelu"])
@pytest.mark.parametrize("m", [200, 4200])
def test_prefill_glu_tcgen05(cuda, codec, act, m):
    """Prefill-sized fused GLU: one tcgen05 GEMM with gate and up accumulators
    side by side (128 output columns per tile; N=320 leaves a ragged tile).
    M=4200: Q4_K above 768 rows goes through the dequantized copy."""
    from math import erf
    n, k = 320, 1024
    wg = synth.random_weight(codec, n, k, seed=24)
    wu = synth.random_weight(codec, n, k, seed=25)
    x = synth.random_activations(m, k, seed=26)
    g = O.matmul(x, wg, codec).astype(np.float64)
    u = O.matmul(x, wu, codec).astype(np.float64)
    if act == "silu":
        ref = g / (1 + np.exp(-g)) * u
    else:
        ref = 0.5 * g * (1 + np.vectorize(erf)(g / np.sqrt(2))) * u
    y = kq.quantized_glu(to_dev_x(x, cuda), torch.from_numpy(wg).to(cuda), torch.from_numpy(wu).to(cuda), codec,
                         act=act, out_dtype=torch.float32)
    assert rel_err(y.cpu().numpy(), ref) <= TOL


@pytest.mark.parametrize("codec_gu,codec_d", [("q4_k", "q6_k"), ("iq2_xxs", "iq2_xxs")])
def test_expert_parallel_partials_sum_to_full_layer(cuda, codec_gu, codec_d):
    """Two expert-parallel 'ranks' (expert ranges) on one GPU: their partial
    layers sum to the full routed layer, which matches the oracle."""
    e, d, f, k, t = 16, 512, 256, 4, 3
    wg, wu, wd, x, lg = _moe_case(codec_gu, codec_d, e, d, f, t, k, seed=80)
    xd = to_dev_x(x, cuda)
    idx, sc = kq.moe_router_topk(torch.from_numpy(lg).to(cuda), k, True, shared_gate=False)
    tw = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    full = kq.moe_expert_layer_local(xd, idx, sc, tw(wg), tw(wu), tw(wd), codec_gu, codec_d, 0, e,
                                     out_dtype=torch.float32)
    parts = []
    for r in range(2):
        sl = slice(8 * r, 8 * r + 8)
        parts.append(kq.moe_expert_layer_local(xd, idx, sc, tw(wg[sl]), tw(wu[sl]), tw(wd[sl]), codec_gu, codec_d,
                                               8 * r, e, out_dtype=torch.float32))
    assert rel_err((parts[0] + parts[1]).cpu().numpy(), full.cpu().numpy()) <= 1e-5
    # oracle: f32 dequant-then-matmul per slot (h rounded to bf16 as the kernel does)
    ii, ss = idx.cpu().numpy(), sc.cpu().numpy()
    ref = np.zeros((t, d))
    for ti in range(t):
        for j in range(k):
            ex = ii[ti, j]
            g = O.matmul(x[ti:ti + 1], wg[ex], codec_gu)[0].astype(np.float64)
            u = O.matmul(x[ti:ti + 1], wu[ex], codec_gu)[0].astype(np.float64)
            hb = synth.f32_to_bf16_bits((g / (1 + np.exp(-g)) * u).astype(np.float32))[None]
            ref[ti] += ss[ti, j] * O.matmul(hb, wd[ex], codec_d)[0]
    assert rel_err(full.cpu().numpy(), ref) <= TOL


def test_tensor_parallel_shards_sum_to_full(cuda):
    """Row-parallel K shards (whole blocks, unaligned Q6_K byte offsets) of o and
    down summed over 4 'ranks' equal the unsharded projection."""
    from gmlx_b200 import parallel as par
    for codec, n, k in [("q4_k", 256, 2048), ("q6_k", 256, 4096)]:
        w = synth.random_weight(codec, n, k, seed=90)
        x = synth.random_activations(2, k, seed=91)
        full = kq.quantized_matmul(to_dev_x(x, cuda), torch.from_numpy(w).to(cuda), None, codec,
                                   out_dtype=torch.float32)
        acc = torch.zeros_like(full)
        for r in range(4):
            ws = par.shard_k(torch.from_numpy(w), codec, 4, r).contiguous().to(cuda)
            kk = k // 4
            acc += kq.quantized_matmul(to_dev_x(x[:, r * kk:(r + 1) * kk], cuda), ws, None, codec,
                                       out_dtype=torch.float32)
        assert rel_err(acc.cpu().numpy(), full.cpu().numpy()) <= 1e-4


def _skewed_ids(rng, shape, e):
    """Expert ids with a skewed load: expert 0 gets several 128-row tiles, the
    last expert none (the grouped path's empty and ragged groups)."""
    p = np.array([0.55, 0.25] + [0.2 / (e - 3)] * (e - 3) + [0.0])
    return rng.choice(e, size=shape, p=p).astype(np.int32)


@pytest.mark.parametrize("codec", CODECS)
def test_grouped_gather_qmm(cuda, codec):
    """Many routed rows per expert (>= 33 on average) take the grouped tcgen05
    GEMM: rows sorted by expert, one launch over (expert, 128-row tile), outputs
    scattered back.  N=320 leaves a ragged 256-column tile."""
    e, n, kin, rows = 4, 320, 512, 400
    w = synth.random_weight(codec, n, kin, seed=70, experts=e)
    x = synth.random_activations(rows, kin, seed=71)
    rng = np.random.default_rng(72)
    idx = _skewed_ids(rng, (rows,), e)
    ref = np.zeros((rows, n))
    for ex in range(e):
        sel = np.nonzero(idx == ex)[0]
        if len(sel):
            ref[sel] = O.matmul(np.ascontiguousarray(x[sel]), w[ex], codec)
    xd = to_dev_x(x, cuda).reshape(rows, 1, 1, kin)
    y = kq.gather_qmm(xd, torch.from_numpy(w).to(cuda), None, codec,
                      rhs_indices=torch.from_numpy(idx.reshape(rows, 1)).to(cuda), out_dtype=torch.float32)
    assert rel_err(y.reshape(rows, n).cpu().numpy(), ref) <= TOL
    assert kq.workspace_error() == 0


@pytest.mark.parametrize("codec_gu,codec_d", [("q4_k", "q6_k"), ("iq2_xxs", "iq2_xxs"), ("q5_k", "q6_k"),
                                              ("iq3_xxs", "iq4_xs")])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_grouped_moe_layer_prefill(cuda, codec_gu, codec_d, out_dtype):
    """MoE prefill (T*k >= 33 * experts) through the grouped GEMM: gate/up GEMMs,
    SiLU*up, down GEMM and the score mix; the full layer matches the oracle and
    two expert-parallel halves sum to it."""
    e, d, f, k, t = 8, 512, 256, 2, 200
    wg, wu, wd, x, _ = _moe_case(codec_gu, codec_d, e, d, f, t, k, seed=110)
    rng = np.random.default_rng(111)
    idx = np.stack([_skewed_ids(rng, (t,), e), rng.integers(0, e, size=t).astype(np.int32)], 1)
    sc = rng.random((t, k)).astype(np.float32)
    tw = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    xd = to_dev_x(x, cuda)
    # f32 output: the score mix runs in the down GEMM's epilogue (atomic adds);
    # bf16 output: per-slot rows and the mix kernel
    full = kq.moe_expert_layer_local(xd, tw(idx), tw(sc), tw(wg), tw(wu), tw(wd), codec_gu, codec_d, 0, e,
                                     out_dtype=out_dtype).float()
    parts = sum(kq.moe_expert_layer_local(xd, tw(idx), tw(sc), tw(wg[4 * r:4 * r + 4]), tw(wu[4 * r:4 * r + 4]),
                                          tw(wd[4 * r:4 * r + 4]), codec_gu, codec_d, 4 * r, e,
                                          out_dtype=torch.float32) for r in range(2))
    assert rel_err(parts.cpu().numpy(), full.cpu().numpy()) <= (1e-5 if out_dtype == torch.float32 else 1e-2)
    ref = np.zeros((t, d))
    for j in range(k):
        for ex in range(e):
            sel = np.nonzero(idx[:, j] == ex)[0]
            if not len(sel):
                continue
            xs = np.ascontiguousarray(x[sel])
            g = O.matmul(xs, wg[ex], codec_gu).astype(np.float64)
            u = O.matmul(xs, wu[ex], codec_gu).astype(np.float64)
            hb = synth.f32_to_bf16_bits((g / (1 + np.exp(-g)) * u).astype(np.float32))
            ref[sel] += sc[sel, j, None] * O.matmul(hb, wd[ex], codec_d)
    assert rel_err(full.cpu().numpy(), ref) <= TOL
    # the GLU op alone on the same routing
    h = kq.moe_glu_gather_kq(xd, tw(wg), tw(wu), codec_gu, tw(idx))
    assert tuple(h.shape) == (t, k, f)
    assert kq.workspace_error() == 0


@pytest.mark.parametrize("codec,n,k", [("q4_k", 4096, 512), ("q6_k", 4096, 1792), ("q6_k", 1000, 7168)])
def test_fused_allreduce_single_rank(cuda, codec, n, k):
    """The fused row-parallel all-reduce with one rank equals the plain GEMV
    (f32, same kernel arithmetic); repeated calls alternate the buffer parity."""
    from gmlx_b200 import parallel as par
    w = torch.from_numpy(synth.random_weight(codec, n, k, seed=120)).to(cuda)
    comm = par.PeerComm(4096, cuda)
    try:
        for i in range(5):
            x = to_dev_x(synth.random_activations(1, k, seed=121 + i), cuda)
            ref = kq.quantized_matmul(x, w, None, codec, out_dtype=torch.float32)
            y = kq.quantized_matmul_allreduce(x, w, codec, comm, out_dtype=torch.float32)
            assert torch.equal(y, ref)
        assert kq.workspace_error() == 0
    finally:
        torch.cuda.synchronize()
        comm.close()


def test_embedding_and_multilinear_modules(cuda):
    """KQuantEmbedding (row lookup, tied head) and KQuantMultiLinear (per-head
    stacks, both orientations) against the oracle's dequantized weights."""
    from gmlx_b200 import nn as knn
    vocab, dims = 300, 512
    we = synth.random_weight("q6_k", vocab, dims, seed=140)
    emb = knn.KQuantEmbedding(vocab, dims, "q6_k", out_dtype=torch.float32, device=cuda)
    emb.weight.copy_(torch.from_numpy(we))
    ids = torch.tensor([[3, 299, 0], [17, 3, 150]], device=cuda)
    deq = O.dequantize(we, "q6_k")
    assert np.array_equal(emb(ids).cpu().numpy(), deq[ids.cpu().numpy()])
    x = synth.random_activations(2, dims, seed=141)
    assert rel_err(emb.as_linear(to_dev_x(x, cuda)).float().cpu().numpy(), O.matmul(x, we, "q6_k")) <= TOL
    h, n, k, L = 4, 128, 512, 3
    wm = synth.random_weight("q4_k", n, k, seed=142, experts=h)
    ml = knn.KQuantMultiLinear(k, n, h, "q4_k", device=cuda)
    ml.weight.copy_(torch.from_numpy(wm))
    xm = synth.random_activations(2 * h * L, k, seed=143)
    xd = to_dev_x(xm, cuda).reshape(2, h, L, k)
    y = ml(xd).float().cpu().numpy()
    assert y.shape == (2, h, L, n)
    for b in range(2):
        for hh in range(h):
            rows = xm.reshape(2, h, L, k)[b, hh]
            assert rel_err(y[b, hh], O.matmul(np.ascontiguousarray(rows), wm[hh], "q4_k")) <= TOL
    # transpose=False: x [..., h, L, n] @ W[h] -> [..., h, L, k]
    xt = torch.randn(2, h, L, n, device=cuda).to(torch.bfloat16)
    yt = ml(xt, transpose=False).float().cpu().numpy()
    wd = np.stack([O.dequantize(wm[hh], "q4_k") for hh in range(h)])  # [h, n, k]
    ref = np.einsum("bhln,hnk->bhlk", xt.float().cpu().numpy(), wd.astype(np.float32))
    assert rel_err(yt, ref) <= TOL


def test_shared_expert_slot_ops(cuda):
    """moe_glu_gather_shexp_kq / gather_qmv_mix_kq (the shared expert as slot k,
    sigmoid-gated in the mix) against the oracle, shared expert in another codec."""
    e, d, f, k, t = 8, 512, 256, 2, 3
    wg, wu, wd, x, _ = _moe_case("q4_k", "q6_k", e, d, f, t, k, seed=150)
    sg = synth.random_weight("q6_k", f, d, seed=151)
    su = synth.random_weight("q6_k", f, d, seed=152)
    sd = synth.random_weight("q4_k", d, f, seed=153)
    lg = synth.random_logits(t, e + 1, seed=154)
    tw = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    idx, sc = kq.moe_router_topk(tw(lg), k, True)
    h = kq.moe_glu_gather_shexp_kq(to_dev_x(x, cuda), tw(wg), tw(wu), tw(sg), tw(su), "q4_k", idx,
                                   shexp_kquant_type="q6_k")
    assert tuple(h.shape) == (t, k + 1, f)
    ii, ss = idx.cpu().numpy(), sc.cpu().numpy()
    silu = lambda g: g / (1 + np.exp(-g))  # noqa: E731
    for ti in range(t):
        xr = x[ti:ti + 1]
        for j in range(k + 1):
            gw, uw, c = (wg[ii[ti, j]], wu[ii[ti, j]], "q4_k") if j < k else (sg, su, "q6_k")
            g = O.matmul(xr, gw, c)[0].astype(np.float64)
            u = O.matmul(xr, uw, c)[0].astype(np.float64)
            assert rel_err(h[ti, j].float().cpu().numpy(), silu(g) * u) <= TOL
    y = kq.gather_qmv_mix_kq(h, tw(wd), tw(sd), "q6_k", idx, sc, shexp_kquant_type="q4_k", out_dtype=torch.float32)
    hb = synth.f32_to_bf16_bits(h.float().cpu().numpy())
    ref = np.zeros((t, d))
    for ti in range(t):
        for j in range(k):
            ref[ti] += ss[ti, j] * O.matmul(hb[ti, j][None], wd[ii[ti, j]], "q6_k")[0]
        ref[ti] += ss[ti, k] * O.matmul(hb[ti, k][None], sd, "q4_k")[0]
    assert rel_err(y.cpu().numpy(), ref) <= TOL


def test_gguf_loaded_weights_drive_the_kernels(cuda, tmp_path):
    """A GGUF file written with gguf-py, loaded by gmlx_b200.gguf_io straight
    into HBM, feeds quantized_matmul (checked against the oracle)."""
    gguf = pytest.importorskip("gguf")
    from gmlx_b200 import gguf_io
    w = synth.random_weight("q6_k", 256, 768, seed=160)
    wr = gguf.GGUFWriter(str(tmp_path / "w.gguf"), "llama")
    wr.add_tensor("blk.0.ffn_down.weight", w, raw_dtype=gguf.GGMLQuantizationType.Q6_K)
    wr.write_header_to_file()
    wr.write_kv_data_to_file()
    wr.write_tensors_to_file()
    wr.close()
    arrays, codecs, _, shapes = gguf_io.load_gguf(str(tmp_path / "w.gguf"), device=cuda)
    wd = arrays["blk.0.ffn_down.weight"]
    assert wd.is_cuda and codecs["blk.0.ffn_down.weight"] == "q6_k" and shapes["blk.0.ffn_down.weight"] == (768, 256)
    x = synth.random_activations(2, 768, seed=161)
    y = kq.quantized_matmul(to_dev_x(x, cuda), wd, arrays["blk.0.ffn_down.scales"], "q6_k", out_dtype=torch.float32)
    assert rel_err(y.cpu().numpy(), O.matmul(x, w, "q6_k")) <= TOL


@pytest.mark.parametrize("codec,m", [("q4_k", 1), ("q6_k", 1), ("iq2_xxs", 3), ("q4_k", 64)])
def test_quantized_matmul_qmv_bias(cuda, codec, m):
    """x @ W^T + bias in one dispatch (decode: in the GEMV store; prefill: after the GEMM)."""
    n, k = 320, 1024
    w = synth.random_weight(codec, n, k, seed=170)
    x = synth.random_activations(m, k, seed=171)
    b = np.random.default_rng(172).standard_normal(n).astype(np.float32)
    ref = O.matmul(x, w, codec) + b
    y = kq.quantized_matmul_qmv_bias(to_dev_x(x, cuda), torch.from_numpy(w).to(cuda), None,
                                     torch.from_numpy(b).to(cuda).to(torch.bfloat16), codec, out_dtype=torch.float32)
    bb = torch.from_numpy(b).to(torch.bfloat16).float().numpy()
    assert rel_err(y.cpu().numpy(), O.matmul(x, w, codec) + bb) <= TOL
    assert rel_err(y.cpu().numpy(), ref) <= 2 * TOL


def test_iq2_sparse_routing_single_slot_groups(cuda):
    """IQ2_XXS with sparse routing (slots * 4 <= experts) runs one-slot groups on
    the one-row path; experts routed by two tokens are streamed twice."""
    e, d, f, k, t = 64, 512, 256, 8, 2
    wg, wu, wd, x, _ = _moe_case("iq2_xxs", "iq2_xxs", e, d, f, t, k, seed=180)
    idx = np.array([[3, 7, 9, 11, 20, 33, 40, 63], [7, 3, 1, 2, 9, 50, 60, 61]], np.int32)  # 3, 7, 9 twice
    sc = np.random.default_rng(181).random((t, k)).astype(np.float32)
    tw = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    y = kq.moe_expert_layer_local(to_dev_x(x, cuda), tw(idx), tw(sc), tw(wg), tw(wu), tw(wd), "iq2_xxs", "iq2_xxs",
                                  0, e, out_dtype=torch.float32).cpu().numpy()
    ref = np.zeros((t, d))
    for ti in range(t):
        for j in range(k):
            ex = idx[ti, j]
            g = O.matmul(x[ti:ti + 1], wg[ex], "iq2_xxs")[0].astype(np.float64)
            u = O.matmul(x[ti:ti + 1], wu[ex], "iq2_xxs")[0].astype(np.float64)
            hb = synth.f32_to_bf16_bits((g / (1 + np.exp(-g)) * u).astype(np.float32))[None]
            ref[ti] += sc[ti, j] * O.matmul(hb, wd[ex], "iq2_xxs")[0]
    assert rel_err(y, ref) <= TOL
    assert kq.workspace_error() == 0


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_grouped_moe_layer_two_row_tiles(cuda, out_dtype):
    """Experts averaging >= 192 routed rows take 256-row tiles (two accumulators
    per CTA); the layer sorts once and the down GEMM reads h in sorted order."""
    e, d, f, k, t = 4, 512, 256, 2, 600
    wg, wu, wd, x, _ = _moe_case("q4_k", "q6_k", e, d, f, t, k, seed=120)
    rng = np.random.default_rng(121)
    idx = np.stack([_skewed_ids(rng, (t,), e), rng.integers(0, e, size=t).astype(np.int32)], 1)
    sc = rng.random((t, k)).astype(np.float32)
    tw = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    y = kq.moe_expert_layer_local(to_dev_x(x, cuda), tw(idx), tw(sc), tw(wg), tw(wu), tw(wd), "q4_k", "q6_k", 0, e,
                                  out_dtype=out_dtype).float()
    ref = np.zeros((t, d))
    for j in range(k):
        for ex in range(e):
            sel = np.nonzero(idx[:, j] == ex)[0]
            if not len(sel):
                continue
            xs = np.ascontiguousarray(x[sel])
            g = O.matmul(xs, wg[ex], "q4_k").astype(np.float64)
            u = O.matmul(xs, wu[ex], "q4_k").astype(np.float64)
            hb = synth.f32_to_bf16_bits((g / (1 + np.exp(-g)) * u).astype(np.float32))
            ref[sel] += sc[sel, j, None] * O.matmul(hb, wd[ex], "q6_k")
    assert rel_err(y.cpu().numpy(), ref) <= TOL
    assert kq.workspace_error() == 0


@pytest.mark.parametrize("codec", CODECS)
@pytest.mark.parametrize("m", [300, 1000])
def test_gemm_split_k_deterministic(cuda, codec, m):
    """Plain GEMMs on the dequantized-copy path (every codec but Q4_K at this M)
    that fill at most half of the SMs split K in two: each half
    posts an f32 partial tile and the last one adds the other.  Ragged M and N,
    bit-identical across calls, and every tile counter is left zero (the
    workspace is reused)."""
    n, k = 320, 2048
    w = synth.random_weight(codec, n, k, seed=130)
    x = synth.random_activations(m, k, seed=131)
    ref = O.matmul(x, w, codec)
    wd, xd = torch.from_numpy(w).to(cuda), to_dev_x(x, cuda)
    ys = [kq.quantized_matmul(xd, wd, None, codec, out_dtype=torch.float32) for _ in range(3)]
    assert torch.equal(ys[0], ys[1]) and torch.equal(ys[0], ys[2])
    assert rel_err(ys[0].cpu().numpy(), ref) <= TOL
    assert kq.workspace_error() == 0
