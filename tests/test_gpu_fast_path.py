"""The native fast path of the decode ops (gmlx_b200/csrc/kq_torch.cpp) against
the Python + ctypes path: the same kernels, so bit-identical outputs, and the
same exceptions for malformed calls (the fast path hands those back)."""
import numpy as np
import pytest
import torch

from gmlx_b200 import kq, synth

pytestmark = pytest.mark.gpu


def _slow(fn, *a, **k):
    saved = kq._EXT
    kq._EXT = False
    try:
        return fn(*a, **k)
    finally:
        kq._EXT = saved


@pytest.mark.parametrize("codec,n,k,m", [("q4_k", 1024, 4096, 1), ("q6_k", 512, 14336, 1), ("q4_k", 640, 2048, 4),
                                         ("iq2_xxs", 512, 7168, 3), ("q8_0", 256, 1024, 1)])
def test_fast_path_matches_python_path(cuda, codec, n, k, m):
    assert kq._ext() is not None, "gmlx_b200/_ext/kq_torch.so was not built"
    w = torch.from_numpy(synth.random_weight(codec, n, k, seed=3)).to(cuda)
    w2 = torch.from_numpy(synth.random_weight(codec, n, k, seed=4)).to(cuda)
    x = torch.from_numpy(synth.random_activations(m, k, seed=5).view(np.int16)).view(torch.bfloat16).to(cuda)
    for od in (None, torch.float32):
        fast = kq.quantized_matmul(x, w, None, codec, out_dtype=od)
        slow = _slow(kq.quantized_matmul, x, w, None, codec, out_dtype=od)
        assert fast.dtype == slow.dtype and fast.shape == slow.shape
        assert torch.equal(fast, slow)
        fg = kq.quantized_glu(x, w, w2, codec, out_dtype=od)
        sg = _slow(kq.quantized_glu, x, w, w2, codec, out_dtype=od)
        assert torch.equal(fg, sg)
    assert kq.workspace_error() == 0


def test_fast_path_defers_errors(cuda):
    w = torch.from_numpy(synth.random_weight("q4_k", 64, 512, seed=1)).to(cuda)
    with pytest.raises(ValueError):
        kq.quantized_matmul(torch.zeros(1, 256, dtype=torch.bfloat16, device=cuda), w, None, "q4_k")
    with pytest.raises(ValueError):
        kq.quantized_matmul(torch.zeros(1, 512, dtype=torch.bfloat16), w, None, "q4_k")
    with pytest.raises(NotImplementedError):
        kq.quantized_matmul(torch.zeros(1, 512, dtype=torch.bfloat16, device=cuda), w, None, "q9_k")
