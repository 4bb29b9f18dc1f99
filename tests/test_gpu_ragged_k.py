"""GPU parity for rows that end in a partial 256-weight group: the 32- and
64-weight-block codecs (Q8_0, Q4_0/1, Q5_0/1, IQ4_NL, MXFP4, NVFP4) at any K
that is a whole number of their blocks, as gmlx serves them ("any K % block,
e.g. gemma's inter=704", gmlx/modules.py:502-507; gpt-oss's MXFP4 experts
have K = 2880 = 90 blocks).  The reference is gguf-py's block dequantization
(the format definition the CPU oracle is pinned to), then an f64 matmul.
Dequantize is bit-exact in f32; matmul-shaped outputs within 1e-2."""
import numpy as np
import pytest
import torch

from gmlx_b200 import kq, synth

gq = pytest.importorskip("gguf.quants")
from gguf.constants import GGMLQuantizationType as T  # noqa: E402

pytestmark = pytest.mark.gpu
TOL = 1e-2
RAGGED = {"q8_0": T.Q8_0, "q4_0": T.Q4_0, "q4_1": T.Q4_1, "q5_0": T.Q5_0, "q5_1": T.Q5_1, "iq4_nl": T.IQ4_NL,
          "mxfp4": T.MXFP4, "nvfp4": T.NVFP4}


def ref_deq(w, codec):
    return gq.dequantize(w, RAGGED[codec]).astype(np.float32)


def dev_x(m, k, seed, cuda):
    bits = synth.random_activations(m, k, seed=seed)
    x = torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).to(cuda)
    return x, x.float().cpu().numpy().astype(np.float64)


def rel_err(y, ref):
    return float(np.abs(np.asarray(y, np.float64) - ref).max() / max(np.abs(ref).max(), 1e-30))


@pytest.mark.parametrize("codec", sorted(RAGGED))
@pytest.mark.parametrize("k", [704, 2880])
def test_ragged_dequantize_bitexact(cuda, codec, k):
    w = synth.random_weight_ragged(codec, 48, k, seed=7)
    ref = ref_deq(w, codec)
    assert ref.shape == (48, k)
    out = kq.dequantize(torch.from_numpy(w).to(cuda), None, codec).cpu().numpy()
    assert np.array_equal(out.view(np.uint32), ref.view(np.uint32))
    bf = kq.dequantize(torch.from_numpy(w).to(cuda), None, codec, dtype=torch.bfloat16).float().cpu().numpy()
    assert np.array_equal(bf, torch.from_numpy(ref).to(torch.bfloat16).float().numpy())


@pytest.mark.parametrize("codec", sorted(RAGGED))
@pytest.mark.parametrize("k", [704, 2880])
@pytest.mark.parametrize("m", [1, 3, 70])
def test_ragged_quantized_matmul_and_glu(cuda, codec, k, m):
    n = 200
    w = synth.random_weight_ragged(codec, n, k, seed=8)
    w2 = synth.random_weight_ragged(codec, n, k, seed=9)
    x, xf = dev_x(m, k, 10 + m, cuda)
    deq, deq2 = ref_deq(w, codec).astype(np.float64), ref_deq(w2, codec).astype(np.float64)
    wd, wd2 = torch.from_numpy(w).to(cuda), torch.from_numpy(w2).to(cuda)
    y = kq.quantized_matmul(x, wd, None, codec, out_dtype=torch.float32)
    assert tuple(y.shape) == (m, n)
    assert rel_err(y.cpu().numpy(), xf @ deq.T) <= TOL
    g, u = xf @ deq.T, xf @ deq2.T
    h = kq.quantized_glu(x, wd, wd2, codec, act="silu", out_dtype=torch.float32)
    assert rel_err(h.cpu().numpy(), g / (1 + np.exp(-g)) * u) <= TOL
    assert kq.workspace_error() == 0


def test_ragged_k_needs_multiple_of_64_for_matmul(cuda):
    """K = 96 (three 32-weight blocks) dequantizes; the matmul (tcgen05 GEMM
    over 64-value K tiles) refuses it with a clear error."""
    w = synth.random_weight_ragged("q8_0", 16, 96, seed=3)
    wd = torch.from_numpy(w).to(cuda)
    out = kq.dequantize(wd, None, "q8_0").cpu().numpy()
    assert np.array_equal(out.view(np.uint32), ref_deq(w, "q8_0").view(np.uint32))
    x, _ = dev_x(1, 96, 4, cuda)
    with pytest.raises(Exception, match="partial last group"):
        kq.quantized_matmul(x, wd, None, "q8_0")
