"""GPU parity of kq_quantized_matmul_chain: a decoder layer's one-row
projections (q|k|v, o, fused gate/up, down reading the gate/up output) in one
persistent launch, against the CPU oracle and against the single-op entry
points it replaces (max |y - ref| / max |ref| <= 1e-2)."""
import ctypes

import numpy as np
import pytest
import torch

from gmlx_b200 import _lib, kq, synth
from oracle import oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-2


def rel_err(y, ref):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30))


def dev_x(bits, cuda):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16).copy()).view(torch.bfloat16).to(cuda)


def silu_glu(g, u):
    g = g.astype(np.float64)
    return g / (1 + np.exp(-g)) * u


def layer(cgu, cd, d, f, nqkv, seed):
    return {
        "qkv": synth.random_weight(cgu, nqkv, d, seed=seed),
        "o": synth.random_weight(cgu, d, d, seed=seed + 1),
        "gate": synth.random_weight(cgu, f, d, seed=seed + 2),
        "up": synth.random_weight(cgu, f, d, seed=seed + 3),
        "down": synth.random_weight(cd, d, f, seed=seed + 4),
    }


@pytest.mark.parametrize("cgu,cd,d,f,nqkv", [
    ("q4_k", "q6_k", 4096, 14336, 6144),   # Llama-3-8B Q4_K_M layer
    ("q4_k", "q6_k", 1024, 4096, 1000),    # ragged last tile (1000 rows), K chunks of 2 stages
    ("q6_k", "q6_k", 2048, 4096, 2560),    # Q6_K everywhere (Q6_K gate/up in the fused GLU)
    ("q4_k", "q6_k", 1024, 2816, 1536),    # Q6_K rows of 2310 bytes: no TMA tensor, one launch per problem
    ("q5_k", "q6_k", 2048, 5632, 2560),    # no fused kernel for this mix: one launch per problem
    ("iq4_xs", "q6_k", 2048, 2816, 2560),
])
def test_chain_decoder_layer(cuda, cgu, cd, d, f, nqkv):
    W = layer(cgu, cd, d, f, nqkv, seed=2000 + d)
    x = synth.random_activations(1, d, seed=2100)
    a = synth.random_activations(1, d, seed=2101)  # stands in for the attention output
    Wd = {k: torch.from_numpy(v).to(cuda) for k, v in W.items()}
    xd, ad = dev_x(x, cuda), dev_x(a, cuda)
    probs = [
        {"x": xd, "w": Wd["qkv"], "codec": cgu},
        {"x": ad, "w": Wd["o"], "codec": cgu},
        {"x": xd, "w": Wd["gate"], "w2": Wd["up"], "act": "silu", "codec": cgu},
        {"x": 2, "w": Wd["down"], "codec": cd},
    ]
    for call in range(2):  # twice: the workspace must come back zeroed
        qkv, o, h, y = kq.quantized_matmul_chain(probs, out_dtype=torch.float32)
        assert h.dtype == torch.bfloat16 and y.dtype == torch.float32
        assert rel_err(qkv.cpu().numpy(), O.matmul(x, W["qkv"], cgu)) <= TOL
        assert rel_err(o.cpu().numpy(), O.matmul(a, W["o"], cgu)) <= TOL
        h_ref = silu_glu(O.matmul(x, W["gate"], cgu), O.matmul(x, W["up"], cgu))
        assert rel_err(h.float().cpu().numpy(), h_ref) <= TOL
        hb = synth.f32_to_bf16_bits(h.float().cpu().numpy())
        assert rel_err(y.cpu().numpy(), O.matmul(hb, W["down"], cd)) <= TOL
        # the single-op entry point gives the same numbers
        y1 = kq.quantized_matmul(h, Wd["down"], None, cd, out_dtype=torch.float32)
        assert rel_err(y.cpu().numpy(), y1.cpu().numpy()) <= 1e-3
        if call == 0:
            first = [t.clone() for t in (qkv, o, h, y)]
        else:  # deterministic: bit-identical across calls
            for t0, t1 in zip(first, (qkv, o, h, y)):
                assert torch.equal(t0, t1)
    assert kq.workspace_error() == 0


def test_chain_dependency_chain_and_bias(cuda):
    """Every problem depends on the one before (the shape of a real layer,
    where o reads attention and gate/up read o); a bias on a plain problem."""
    d, f = 2048, 4096
    W = layer("q4_k", "q6_k", d, f, d, seed=2300)
    x = synth.random_activations(1, d, seed=2301)
    Wd = {k: torch.from_numpy(v).to(cuda) for k, v in W.items()}
    bias = torch.randn(d, device=cuda, dtype=torch.float32)
    probs = [
        {"x": dev_x(x, cuda), "w": Wd["qkv"], "codec": "q4_k"},
        {"x": 0, "w": Wd["o"], "codec": "q4_k", "bias": bias},
        {"x": 1, "w": Wd["gate"], "w2": Wd["up"], "act": "silu", "codec": "q4_k"},
        {"x": 2, "w": Wd["down"], "codec": "q6_k"},
    ]
    a, o, h, y = kq.quantized_matmul_chain(probs, out_dtype=torch.float32)
    assert rel_err(a.float().cpu().numpy(), O.matmul(x, W["qkv"], "q4_k")) <= TOL
    ab = synth.f32_to_bf16_bits(a.float().cpu().numpy())
    o_ref = O.matmul(ab, W["o"], "q4_k") + bias.cpu().numpy()
    assert rel_err(o.float().cpu().numpy(), o_ref) <= TOL
    ob = synth.f32_to_bf16_bits(o.float().cpu().numpy())
    h_ref = silu_glu(O.matmul(ob, W["gate"], "q4_k"), O.matmul(ob, W["up"], "q4_k"))
    assert rel_err(h.float().cpu().numpy(), h_ref) <= TOL
    hb = synth.f32_to_bf16_bits(h.float().cpu().numpy())
    assert rel_err(y.cpu().numpy(), O.matmul(hb, W["down"], "q6_k")) <= TOL
    assert kq.workspace_error() == 0


@pytest.mark.parametrize("codec", ["q4_k", "q6_k"])
@pytest.mark.parametrize("n,k", [(32, 256), (100, 2048), (4096, 16384), (33, 6144)])
def test_chain_single_problem_edges(cuda, codec, n, k):
    """One-problem chains at the smallest K, a ragged tile and the largest K
    the fused kernel holds; f16 activations too."""
    w = synth.random_weight(codec, n, k, seed=2400 + n)
    x = synth.random_activations(1, k, seed=2401)
    ref = O.matmul(x, w, codec)
    wd = torch.from_numpy(w).to(cuda)
    for dt in (torch.bfloat16, torch.float16):
        y, = kq.quantized_matmul_chain([{"x": dev_x(x, cuda).to(dt), "w": wd, "codec": codec}],
                                       out_dtype=torch.float32)
        assert rel_err(y.cpu().numpy(), ref) <= TOL
    assert kq.workspace_error() == 0


def test_chain_rejects_forward_dependency(cuda):
    L = _lib.load()
    arr = (_lib.ChainProblem * 2)()
    w = torch.from_numpy(synth.random_weight("q4_k", 32, 256, seed=1)).to(cuda)
    x = torch.zeros(256, dtype=torch.bfloat16, device=cuda)
    y = torch.empty(64, dtype=torch.bfloat16, device=cuda)
    for i in range(2):
        arr[i].codec, arr[i].x, arr[i].w = 12, x.data_ptr(), w.data_ptr()
        arr[i].n, arr[i].k, arr[i].w_row_stride = 32, 256, 144
        arr[i].y, arr[i].y_dtype, arr[i].depends_on = y.data_ptr() + 64 * i, _lib.KQ_BF16, -1
    arr[0].depends_on = 1
    ws = torch.zeros(1 << 20, dtype=torch.uint8, device=cuda)
    rc = L.kq_quantized_matmul_chain(arr, 2, _lib.KQ_BF16, ctypes.c_void_p(ws.data_ptr()), ws.numel(),
                                     ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == _lib.KQ_ERR_SHAPE and b"earlier" in L.kq_last_error()
