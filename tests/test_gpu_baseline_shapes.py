"""GPU parity at the benchmark's own shapes.

The other parity tests sweep codecs and schedule branches at reduced sizes;
these run every benchmarked cell at full size, because large shapes take
their own schedule branches (dynamic tiles, stream-K, 2-row-tile grouped
GEMM, dequantization chunks, split-K on SM fill).  Each output is compared
with the CPU oracle's f32 dequantize-then-matmul (max |y - ref| / max |ref|
<= 1e-2).  Where the oracle over every row would
take minutes (prefill at M = 8192, 4096-token expert layers) a seeded sample
of rows is checked against it over all output columns.

Synthetic weights and activations carry BASELINE.json's statistics (fp16 d /
dmin U[1e-4, 2e-3], Q6_K scales U[-64, 63], uniform quants / IQ2_XXS words,
bf16 N(0, 1) activations, f32 N(0, 1) router logits).
"""
import numpy as np
import pytest
import torch

from gmlx_b200 import kq, synth
from oracle import oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-2
SAMPLE_ROWS = 64


def rel_err(y, ref):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30))


def dev_x(bits, cuda):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16).copy()).view(torch.bfloat16).to(cuda)


def sample_rows(m, seed, count=SAMPLE_ROWS):
    if m <= count:
        return np.arange(m)
    rng = np.random.default_rng(seed)
    # always the first and last rows (tile edges) plus a seeded spread
    r = np.concatenate([[0, m - 1], rng.choice(np.arange(1, m - 1), count - 2, replace=False)])
    return np.sort(r)


@pytest.fixture(scope="module")
def llama_layer():
    """One Llama-3-8B Q4_K_M decoder layer (config 2/3 weights), host and device."""
    w = {}
    for i, (name, codec, n, k) in enumerate(synth.LLAMA3_8B_LAYER):
        w[name] = (codec, synth.random_weight(codec, n, k, seed=300 + i))
    return w


def _dev(llama_layer, name, cuda, cache={}):
    key = (name, str(cuda))
    if key not in cache:
        cache[key] = torch.from_numpy(llama_layer[name][1]).to(cuda)
    return cache[key]


def test_config1_single_q4k_linear(cuda):
    """Config 1: Q4_K 4096 x 4096, one bf16 activation row, seed 0."""
    w = synth.random_weight("q4_k", 4096, 4096, seed=0)
    x = synth.random_activations(1, 4096, seed=0)
    ref = O.matmul(x, w, "q4_k")
    wd = torch.from_numpy(w).to(cuda)
    for od in (torch.float32, torch.bfloat16):
        y = kq.quantized_matmul(dev_x(x, cuda), wd, None, "q4_k", out_dtype=od)
        assert rel_err(y.float().cpu().numpy(), ref) <= TOL
    assert kq.workspace_error() == 0


@pytest.mark.parametrize("m", [1, 4, 16, 32])
def test_config2_decode_layer_projections(cuda, llama_layer, m):
    """Config 2: every projection of the layer at M in {1, 4, 16, 32}, plus the
    fused gate/up/SiLU and the row-concatenated q|k|v the bench runs."""
    for i, (name, codec, n, k) in enumerate(synth.LLAMA3_8B_LAYER):
        x = synth.random_activations(m, k, seed=400 + 10 * m + i)
        ref = O.matmul(x, llama_layer[name][1], codec)
        y = kq.quantized_matmul(dev_x(x, cuda), _dev(llama_layer, name, cuda), None, codec, out_dtype=torch.float32)
        assert rel_err(y.cpu().numpy(), ref) <= TOL, name
    x = synth.random_activations(m, 4096, seed=500 + m)
    g = O.matmul(x, llama_layer["gate_proj"][1], "q4_k").astype(np.float64)
    u = O.matmul(x, llama_layer["up_proj"][1], "q4_k").astype(np.float64)
    h_ref = g / (1 + np.exp(-g)) * u
    h = kq.quantized_glu(dev_x(x, cuda), _dev(llama_layer, "gate_proj", cuda), _dev(llama_layer, "up_proj", cuda),
                         "q4_k", act="silu", out_dtype=torch.float32)
    assert rel_err(h.cpu().numpy(), h_ref) <= TOL
    qkv = np.concatenate([llama_layer[p][1] for p in ("q_proj", "k_proj", "v_proj")])
    ref = O.matmul(x, qkv, "q4_k")
    y = kq.quantized_matmul(dev_x(x, cuda), torch.from_numpy(qkv).to(cuda), None, "q4_k", out_dtype=torch.float32)
    assert rel_err(y.cpu().numpy(), ref) <= TOL
    assert kq.workspace_error() == 0


@pytest.mark.parametrize("m", [512, 2048, 8192])
def test_config3_prefill(cuda, llama_layer, m):
    """Config 3: prefill GEMMs on the 14336 x 4096 Q4_K and 4096 x 14336 Q6_K
    weights, plain and fused gate/up, at M in {512, 2048, 8192}; a seeded
    sample of 64 rows (all 14336 / 4096 columns) against the oracle."""
    rows = sample_rows(m, seed=m)
    for name in ("gate_proj", "down_proj", "q_proj"):
        codec, wb = llama_layer[name]
        k = synth.LLAMA3_8B_LAYER[[p[0] for p in synth.LLAMA3_8B_LAYER].index(name)][3]
        x = synth.random_activations(m, k, seed=600 + m)
        y = kq.quantized_matmul(dev_x(x, cuda), _dev(llama_layer, name, cuda), None, codec, out_dtype=torch.float32)
        ys = y[torch.from_numpy(rows).to(cuda)].cpu().numpy()
        assert rel_err(ys, O.matmul(x[rows], wb, codec)) <= TOL, name
    x = synth.random_activations(m, 4096, seed=700 + m)
    h = kq.quantized_glu(dev_x(x, cuda), _dev(llama_layer, "gate_proj", cuda), _dev(llama_layer, "up_proj", cuda),
                         "q4_k", act="silu", out_dtype=torch.float32)
    g = O.matmul(x[rows], llama_layer["gate_proj"][1], "q4_k").astype(np.float64)
    u = O.matmul(x[rows], llama_layer["up_proj"][1], "q4_k").astype(np.float64)
    assert rel_err(h[torch.from_numpy(rows).to(cuda)].cpu().numpy(), g / (1 + np.exp(-g)) * u) <= TOL
    assert kq.workspace_error() == 0


def moe_layer_ref(x, idx, sc, wg, wu, wd, cgu, cd, tokens):
    """Oracle expert layer for the given token rows: per slot f32 gate/up,
    SiLU(g) * u rounded to bf16 (the layer's activation dtype), down, score mix."""
    d = wd.shape[1]
    out = np.zeros((len(tokens), d))
    for r, t in enumerate(tokens):
        for j in range(idx.shape[1]):
            e = idx[t, j]
            g = O.matmul(x[t:t + 1], wg[e], cgu)[0].astype(np.float64)
            u = O.matmul(x[t:t + 1], wu[e], cgu)[0].astype(np.float64)
            hb = synth.f32_to_bf16_bits((g / (1 + np.exp(-g)) * u).astype(np.float32))
            out[r] += float(sc[t, j]) * O.matmul(hb[None], wd[e], cd)[0]
    return out


MOE = {
    "qwen3": (synth.QWEN3_30B_A3B_MOE, (1, 64, 4096), 900),
    "deepseek": (synth.DEEPSEEK_V3_IQ2_MOE, (1, 8, 64), 950),
}


@pytest.fixture(scope="module")
def moe_weights(request):
    return {}


def _moe_case(cache, name, cuda):
    if name not in cache:
        cache.clear()  # one configuration's stacks on the device at a time
        cfg, _, seed = MOE[name]
        e, d, f = cfg["experts"], cfg["hidden"], cfg["ffn"]
        wg = synth.random_weight(cfg["gate_codec"], f, d, seed=seed, experts=e)
        wu = synth.random_weight(cfg["up_codec"], f, d, seed=seed + 1, experts=e)
        wd = synth.random_weight(cfg["down_codec"], d, f, seed=seed + 2, experts=e)
        cache[name] = (cfg, wg, wu, wd, [torch.from_numpy(a).to(cuda) for a in (wg, wu, wd)])
        torch.cuda.empty_cache()
    return cache[name]


@pytest.mark.parametrize("name,t", [("qwen3", t) for t in MOE["qwen3"][1]] +
                         [("deepseek", t) for t in MOE["deepseek"][1]])
def test_config45_moe_expert_layer(cuda, moe_weights, name, t):
    """Configs 4 and 5: the full routed expert layer (router softmax top-8 with
    renormalisation, fused gate/up/SiLU, down, score mix) at every token count
    the benchmark times, all experts of the configuration on one GPU."""
    cfg, wg, wu, wd, (dg, du, dd) = _moe_case(moe_weights, name, cuda)
    e, k, d = cfg["experts"], cfg["top_k"], cfg["hidden"]
    cgu, cd = cfg["gate_codec"], cfg["down_codec"]
    x = synth.random_activations(t, d, seed=1000 + t)
    lg = synth.random_logits(t, e, seed=1100 + t)
    idx_ref, sc_ref = O.router_topk(lg, k, True)
    idx, sc = kq.moe_router_topk(torch.from_numpy(lg).to(cuda), k, True, shared_gate=False)
    assert np.array_equal(idx.cpu().numpy(), idx_ref)
    assert np.allclose(sc.cpu().numpy(), sc_ref, rtol=1e-5, atol=1e-7)
    y = kq.moe_expert_layer_local(dev_x(x, cuda), idx, sc, dg, du, dd, cgu, cd, 0, e, out_dtype=torch.float32)
    tokens = sample_rows(t, seed=t, count=8 if name == "deepseek" else 16)
    ref = moe_layer_ref(x, idx_ref, sc_ref, wg, wu, wd, cgu, cd, tokens)
    assert rel_err(y[torch.from_numpy(tokens).to(cuda)].cpu().numpy(), ref) <= TOL
    assert kq.workspace_error() == 0
