"""CPU tests of the C ABI: the library loads and exports every symbol that
include/kq_cuda.h declares; host-side validation answers without a GPU."""
import ctypes
import os
import re

import pytest

from gmlx_b200 import _lib

HDR = os.path.join(os.path.dirname(os.path.dirname(__file__)), "include", "kq_cuda.h")


def declared():
    src = open(HDR).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(kq_\w+)\s*\(", src, re.M)))


def test_header_symbols_exported():
    L = _lib.load()
    names = declared()
    assert len(names) >= 15
    for n in names:
        assert hasattr(L, n), n
    assert set(names) == set(_lib.SIGNATURES), set(names) ^ set(_lib.SIGNATURES)


def test_codecs_and_block_bytes():
    L = _lib.load()
    buf = (ctypes.c_int * 24)()
    assert L.kq_codecs(None, 0) == 23
    assert L.kq_codecs(buf, 24) == 23
    ids = [12, 13, 14, 16, 8, 18, 23, 2, 20, 10, 11, 3, 6, 7, 35, 39, 17, 22, 21, 19, 29, 34, 40]
    assert list(buf[:23]) == ids
    assert [L.kq_block_bytes(c) for c in ids + [1]] == [
        144, 176, 210, 66, 272, 98, 136, 144, 144, 84, 110, 160, 176, 192, 66, 136, 74, 82, 110, 50, 56, 54, 144, -1]
    assert L.kq_codec_has_matmul(12) == 1 and L.kq_codec_has_matmul(8) == 1 and L.kq_codec_has_matmul(1) == 0
    assert L.kq_version() >= 100


def test_validation_without_gpu():
    L = _lib.load()
    # unknown codec -> KQ_ERR_CODEC, message names the op (validated before any launch)
    rc = L.kq_dequantize(1, None, 1, 256, 144, None, 0, None)
    assert rc == _lib.KQ_ERR_CODEC
    assert b"dequantize" in L.kq_last_error()
    rc = L.kq_dequantize(12, None, 1, 300, 144, None, 0, None)
    assert rc == _lib.KQ_ERR_SHAPE
    rc = L.kq_moe_router_topk(None, 1, 2048, 8, 1, None, None, None)
    assert rc == _lib.KQ_ERR_SHAPE


def test_python_ops_fail_loudly_without_cuda():
    import torch
    from gmlx_b200 import kq
    w = torch.zeros(4, 144, dtype=torch.uint8)
    with pytest.raises(ValueError, match="CUDA"):
        kq.dequantize(w, None, "q4_k")
    with pytest.raises(NotImplementedError):
        kq.dequantize(w, None, "iq4_ks")


def test_capability_queries_for_the_fused_moe_probe():
    """gmlx's fused-MoE probe asks codec_has_moe_glu for mxfp4 / nvfp4 and reads
    the kq ops' docstrings for the kwargs they take (modules.py:161-234)."""
    from gmlx_b200 import kq
    assert kq.codec_has_moe_glu("mxfp4") and kq.codec_has_moe_glu("nvfp4") and kq.codec_has_moe_glu("q4_k")
    assert not kq.codec_has_moe_glu("iq4_ks")
    assert "per_expert_scale" in kq.moe_router_topk.__doc__
    assert all(hasattr(kq, n) for n in ("moe_glu_gather_kq", "gather_qmv_kq", "gather_qmv_mix_kq",
                                        "gather_qmv_mix_ns_kq", "moe_router_topk", "codecs"))


# gmlx's loader whitelist (gmlx/preflight.py:23-30, SUPPORTED_QUANT_TYPES)
GMLX_SUPPORTED_QUANT_TYPES = {"Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K", "Q4_0", "Q4_1", "Q5_0", "Q5_1", "Q8_0",
                              "IQ4_NL", "IQ4_XS", "IQ3_S", "IQ3_XXS", "IQ2_XXS", "IQ2_XS", "IQ2_S", "IQ1_S",
                              "IQ1_M", "MXFP4", "NVFP4"}


def test_codecs_match_the_loader_whitelist():
    """gmlx gates loading on set(kq.codecs()) (modules.py:1442, :1524,
    loader.py:2798-2801), and its own preflight test asks for equality with
    SUPPORTED_QUANT_TYPES (tests/test_preflight.py:96-99)."""
    from gmlx_b200 import kq
    assert {c.lower() for c in GMLX_SUPPORTED_QUANT_TYPES} == set(kq.codecs())
    assert len(kq.codecs()) == 21
    assert set(kq.all_codecs()) == set(kq.codecs()) | {"tq1_0", "tq2_0"}
    assert all(kq.codec_has_matmul(c) for c in kq.all_codecs())


def test_torch_extension_exports():
    """The decode fast path extension (built by build()) loads and exports its ops."""
    from gmlx_b200 import build
    mod = build.load_torch_ext()
    if mod is None:
        pytest.skip("gmlx_b200/_ext/kq_torch.so not built")
    for name in ("set_entry_points", "workspace", "workspace_peek", "quantized_matmul", "quantized_glu"):
        assert hasattr(mod, name)
