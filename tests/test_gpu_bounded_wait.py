"""The bounded device waits report failure instead of hanging.

Every device-side wait in the kernels (mbarrier phases, peer flags,
completion counters) gives up after about two seconds, records a code in the
workspace's error word and lets the kernel finish, so the CUDA context stays
usable.  This test makes one such wait run out without any fault: a fused
row-parallel all-reduce launched as rank 0 of a two-rank group whose second
"rank" is only a local buffer, so the flag it waits for is never raised.
The call must return, the error word must read 7 (peer-flag wait expired),
and the next ordinary call on the same device must compute correctly.
"""
import ctypes
import time

import numpy as np
import pytest
import torch

from gmlx_b200 import _lib, kq, synth
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def test_peer_flag_wait_runs_out_and_reports(cuda):
    L = _lib.load()
    n, k = 256, 1024
    wb = synth.random_weight("q4_k", n, k, seed=3)
    xb = synth.random_activations(1, k, seed=4)
    w = torch.from_numpy(wb).to(cuda)
    x = torch.from_numpy(xb.view(np.int16).copy()).view(torch.bfloat16).to(cuda)
    y = torch.empty(1, n, dtype=torch.float32, device=cuda)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    bufs = []
    nbytes = L.kq_allreduce_buffer_bytes(2, n)
    for _ in range(2):  # this rank's buffer and a stand-in for the peer's, both local
        p = ctypes.c_void_p()
        _lib.check(L.kq_comm_alloc(nbytes, ctypes.byref(p)), "comm_alloc")
        bufs.append(p.value)
    table = torch.tensor(bufs, dtype=torch.int64, device=cuda)
    wsb = L.kq_quantized_matmul_workspace_size(12, 1, n, k)
    ws = torch.zeros(max(wsb, 1 << 20), dtype=torch.uint8, device=cuda)
    try:
        t0 = time.perf_counter()
        rc = L.kq_quantized_matmul_allreduce(12, ctypes.c_void_p(x.data_ptr()), _lib.KQ_BF16, k,
                                             ctypes.c_void_p(w.data_ptr()), n, w.shape[1],
                                             ctypes.c_void_p(y.data_ptr()), _lib.KQ_F32, 2, 0,
                                             ctypes.c_void_p(table.data_ptr()), ctypes.c_void_p(ws.data_ptr()),
                                             ws.numel(), stream)
        assert rc == _lib.KQ_OK  # the launch itself is fine; the failure is on the device
        err = L.kq_workspace_error(ctypes.c_void_p(ws.data_ptr()), 1, stream)
        waited = time.perf_counter() - t0
        assert err == 7, err
        assert 0.5 < waited < 30.0  # it gave up after its limit, it did not hang
        # the context is intact: an ordinary call computes the right answer
        y2 = kq.quantized_matmul(x, w, None, "q4_k", out_dtype=torch.float32).cpu().numpy()
        ref = O.matmul(xb, wb, "q4_k")
        assert np.abs(y2 - ref).max() <= 1e-2 * np.abs(ref).max()
        assert L.kq_workspace_error(ctypes.c_void_p(ws.data_ptr()), 0, stream) == 0
    finally:
        torch.cuda.synchronize()
        for p in bufs:
            L.kq_comm_free(ctypes.c_void_p(p))
