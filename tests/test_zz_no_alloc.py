"""kq_quantized_matmul_noalloc, the entry point for callers that cannot
allocate device memory (a host framework that owns every byte of the GPU, a
plugin that may not allocate after start-up, a path where an allocation could
stall).  It must give the same result as kq_quantized_matmul, whose scratch
the caller allocates, using only the library's fixed scratch array.

This file is named to be collected last, so a run that stops at the first
failure has already run every other test; it also passes alone in a fresh
process.
"""
import ctypes

import numpy as np
import pytest
import torch

from gmlx_b200 import _lib, synth
from oracle import oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-2
KQ_BF16 = 2


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


@pytest.mark.parametrize("codec,n,k,m,xpad", [("q4_k", 4096, 4096, 1, 0), ("q6_k", 1024, 14336, 3, 0),
                                               ("iq2_xxs", 2048, 2048, 12, 0), ("q4_k", 512, 2048, 64, 24)])
def test_noalloc_matches_workspace_entry(cuda, codec, n, k, m, xpad):
    L = _lib.load()
    c = synth.codec_id(codec)
    w = torch.from_numpy(synth.random_weight(codec, n, k, seed=71)).to(cuda)
    xb = synth.random_activations(m, k, seed=72)
    # xpad > 0: activation rows at a padded stride (the scratch must be sized
    # for the path these activations take, not for a dense layout)
    xs = k + xpad
    xfull = torch.zeros(m, xs, dtype=torch.bfloat16, device=cuda)
    xfull[:, :k] = torch.from_numpy(xb.view(np.int16).copy()).view(torch.bfloat16).to(cuda)
    x = xfull
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    # existing entry point with a caller-allocated (zeroed) workspace
    wsb = L.kq_quantized_matmul_workspace_size(c, m, n, k)
    assert 0 < wsb <= (4 << 20)
    ws = torch.zeros(wsb, dtype=torch.uint8, device=cuda)
    y_ref = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
    _lib.check(L.kq_quantized_matmul(c, _p(x), KQ_BF16, m, k, xs, _p(w), n, w.shape[1], _p(y_ref), KQ_BF16, n,
                                     _p(ws), wsb, stream))
    # the no-allocation entry point, twice in a row (the shared scratch keeps
    # the previous call's contents; the second result must not change)
    outs = []
    for _ in range(2):
        y = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=cuda)
        _lib.check(L.kq_quantized_matmul_noalloc(c, _p(x), KQ_BF16, m, k, xs, _p(w), n, w.shape[1], _p(y),
                                                 KQ_BF16, n, stream))
        # no bounded device wait ran out (the word is cleared by the next call)
        assert L.kq_noalloc_error(0, stream) == 0
        outs.append(y)
    torch.cuda.synchronize()
    ref = O.matmul(xb, synth.random_weight(codec, n, k, seed=71), codec)
    for y in outs:
        yn = y.float().cpu().numpy()
        assert np.isfinite(yn).all()
        assert float(np.abs(yn - y_ref.float().cpu().numpy()).max() / np.abs(ref).max()) <= TOL
        assert float(np.abs(yn - ref).max() / np.abs(ref).max()) <= TOL
    assert torch.equal(outs[0], outs[1])


def test_noalloc_rejects_oversized_shape(cuda):
    L = _lib.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    # a Q6_K prefill of 65536 x 256 needs a 32 MiB dequantized-weight scratch,
    # beyond the fixed array; the size check comes before any pointer is used
    rc = L.kq_quantized_matmul_noalloc(14, None, KQ_BF16, 8192, 256, 256, None, 65536, 210, None, KQ_BF16, 65536,
                                       stream)
    assert rc == _lib.KQ_ERR_WORKSPACE
    assert b"scratch" in L.kq_last_error()
