"""CPU tests: the oracle (C and numpy restatements) pinned to gguf-py and to
the committed golden vectors, plus known-answer cases.  No GPU needed."""
import os

import numpy as np
import pytest

from gmlx_b200 import synth
from oracle import oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden", "golden_blocks.npz")
CODECS = ["q4_k", "q5_k", "q6_k", "iq2_xxs", "q8_0", "iq3_xxs", "iq4_xs", "q4_0", "iq4_nl", "q2_k", "q3_k", "q4_1",
          "q5_0", "q5_1", "tq2_0", "mxfp4", "iq2_xs", "iq2_s", "iq3_s", "iq1_s", "iq1_m", "tq1_0", "nvfp4"]


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD)


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("codec", CODECS)
def test_oracle_matches_golden_dequant(gold, codec):
    w, deq = gold[f"{codec}_w"], gold[f"{codec}_deq"]
    assert np.array_equal(bits(O.dequantize(w, codec)), bits(deq))
    assert np.array_equal(bits(O.np_dequantize(w, codec)), bits(deq))


@pytest.mark.parametrize("codec", CODECS)
def test_oracle_matmul_matches_golden(gold, codec):
    y = O.matmul(gold[f"{codec}_x"], gold[f"{codec}_w"], codec)
    ref = gold[f"{codec}_y"]
    assert np.abs(y - ref).max() <= 1e-5 * np.abs(ref).max()
    # one-hot rows reproduce dequantized columns exactly (x = 1.0 and -2.0)
    deq = gold[f"{codec}_deq"]
    assert np.array_equal(y[3], deq[:, 5])          # value-exact (+0 == -0)
    assert np.array_equal(y[4], -2.0 * deq[:, -1])


@pytest.mark.parametrize("codec", CODECS)
@pytest.mark.parametrize("seed", [0, 1, 2])
def test_oracle_matches_gguf_py_random(codec, seed):
    gq = pytest.importorskip("gguf.quants")
    from gguf.constants import GGMLQuantizationType as T
    qt = {"q4_k": T.Q4_K, "q5_k": T.Q5_K, "q6_k": T.Q6_K, "iq2_xxs": T.IQ2_XXS, "q8_0": T.Q8_0,
          "iq3_xxs": T.IQ3_XXS, "iq4_xs": T.IQ4_XS, "q4_0": T.Q4_0, "iq4_nl": T.IQ4_NL, "q2_k": T.Q2_K,
          "q3_k": T.Q3_K, "q4_1": T.Q4_1, "q5_0": T.Q5_0, "q5_1": T.Q5_1, "tq2_0": T.TQ2_0,
          "mxfp4": T.MXFP4, "iq2_xs": T.IQ2_XS, "iq2_s": T.IQ2_S, "iq3_s": T.IQ3_S,
          "iq1_s": T.IQ1_S, "iq1_m": T.IQ1_M, "tq1_0": T.TQ1_0, "nvfp4": T.NVFP4}[codec]
    w = synth.random_weight(codec, 256, 2048, seed=seed)  # 2048 blocks per seed
    assert np.array_equal(bits(O.dequantize(w, codec)), bits(gq.dequantize(w, qt)))


def test_raw_random_bytes_match_where_finite():
    # fully random bytes (fp16 scales may be NaN/Inf/subnormal): bit patterns of
    # every finite result agree with gguf-py
    gq = pytest.importorskip("gguf.quants")
    from gguf.constants import GGMLQuantizationType as T
    rng = np.random.default_rng(5)
    for codec, qt, bpb in [("q4_k", T.Q4_K, 144), ("q5_k", T.Q5_K, 176), ("q6_k", T.Q6_K, 210),
                           ("iq2_xxs", T.IQ2_XXS, 66), ("q8_0", T.Q8_0, 272), ("iq3_xxs", T.IQ3_XXS, 98),
                           ("iq4_xs", T.IQ4_XS, 136), ("q4_0", T.Q4_0, 144), ("iq4_nl", T.IQ4_NL, 144),
                           ("q2_k", T.Q2_K, 84), ("q3_k", T.Q3_K, 110), ("q4_1", T.Q4_1, 160),
                           ("q5_0", T.Q5_0, 176), ("q5_1", T.Q5_1, 192), ("tq2_0", T.TQ2_0, 66),
                           ("mxfp4", T.MXFP4, 136), ("iq2_xs", T.IQ2_XS, 74), ("iq2_s", T.IQ2_S, 82),
                           ("iq3_s", T.IQ3_S, 110), ("iq1_s", T.IQ1_S, 50), ("iq1_m", T.IQ1_M, 56),
                           ("tq1_0", T.TQ1_0, 54), ("nvfp4", T.NVFP4, 144)]:
        w = rng.integers(0, 256, size=(64, 4 * bpb), dtype=np.uint8)
        a, b = O.dequantize(w, codec), gq.dequantize(w, qt).astype(np.float32)
        fin = np.isfinite(b)
        assert np.array_equal(bits(a)[fin], bits(b)[fin])
        assert np.array_equal(np.isnan(a), np.isnan(b))


def test_known_answer_q4k_zero_quants():
    # all-zero quants: w = -dmin * m for every weight of sub-block j
    b = np.zeros((1, 144), np.uint8)
    b[0, 0:2] = np.array([1e-3], np.float16).view(np.uint8)
    b[0, 2:4] = np.array([2.5e-4], np.float16).view(np.uint8)
    b[0, 8:12] = [1, 2, 3, 4]   # m0..m3
    b[0, 12:16] = [5 << 4, 6 << 4, 7 << 4, 8 << 4]  # m4..m7 (low bits), sc4..7 = 0
    w = O.dequantize(b, "q4_k")[0]
    dmin = np.float32(np.float16(2.5e-4))
    for j, m in enumerate([1, 2, 3, 4, 5, 6, 7, 8]):
        assert np.all(w[32 * j:32 * j + 32] == -(dmin * np.float32(m)))


def test_ksigns_parity_rule():
    gq = pytest.importorskip("gguf.quants")
    assert np.array_equal(O.ksigns_table(), np.frombuffer(gq.IQ2_XXS.ksigns, np.uint8))


def test_iq2xxs_grid_matches_gguf():
    gq = pytest.importorskip("gguf.quants")
    gq.IQ2_XXS.init_grid()
    assert np.array_equal(O.iq2xxs_grid().astype(np.float32), np.asarray(gq.IQ2_XXS.grid).reshape(256, 8))


@pytest.mark.parametrize("name,macro,entries,width", [("IQ2_XS", "KQ_IQ2XS_GRID_INIT", 512, 8),
                                                     ("IQ2_S", "KQ_IQ2S_GRID_INIT", 1024, 8),
                                                     ("IQ3_S", "KQ_IQ3S_GRID_INIT", 512, 4),
                                                     ("IQ1_S", "KQ_IQ1S_GRID_INIT", 2048, 8)])
def test_generated_grids_match_gguf(name, macro, entries, width):
    gq = pytest.importorskip("gguf.quants")
    cls = getattr(gq, name)
    cls.init_grid()
    assert np.array_equal(O._grid(macro, width, entries).view(np.int8).astype(np.float32),
                          np.asarray(cls.grid).reshape(entries, width))


def test_iq3xxs_grid_and_iq4nl_values_match_gguf():
    gq = pytest.importorskip("gguf.quants")
    gq.IQ3_XXS.init_grid()
    assert np.array_equal(O.iq3xxs_grid().astype(np.float32), np.asarray(gq.IQ3_XXS.grid).reshape(256, 4))
    assert O._table_values("KQ_IQ4NL_VALUES_INIT") == list(gq.IQ4_NL.kvalues)


def test_router_topk_semantics():
    lg = synth.random_logits(16, 64, seed=3)
    idx, sc = O.router_topk(lg, 8, True)
    p = np.exp(lg - lg.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    ref_idx = np.argsort(-p, axis=1, kind="stable")[:, :8]
    assert np.array_equal(idx, ref_idx)
    top = np.take_along_axis(p, ref_idx, 1)
    assert np.allclose(sc, top / top.sum(1, keepdims=True), rtol=1e-5)
    idx2, sc2 = O.router_topk(lg, 8, False)
    assert np.allclose(sc2, top, rtol=1e-5)


def test_synthetic_block_statistics():
    for codec in CODECS:
        w = synth.random_blocks(codec, 4096, seed=1)
        if codec in ("q4_k", "q5_k"):
            d = w[:, 0:2].copy().view(np.float16).astype(np.float32)
            dm = w[:, 2:4].copy().view(np.float16).astype(np.float32)
            assert d.min() >= 9e-5 and d.max() <= 2.01e-3 and dm.min() >= 9e-5
        elif codec in ("q8_0", "q4_0", "iq4_nl", "q4_1", "q5_0", "q5_1"):
            d = w.reshape(-1, synth.BLOCK_BYTES[synth.codec_id(codec)] // 8)[:, 0:2].copy().view(np.float16)
            d = d.astype(np.float32)
            assert d.min() >= 9e-5 and d.max() <= 2.01e-3
        elif codec == "iq1_m":  # d's nibbles are the top nibbles of the last four u16
            sc = w[:, 48:56].copy().view(np.uint16).astype(np.int64)
            db = (sc[:, 0] >> 12) | ((sc[:, 1] >> 8) & 0xF0) | ((sc[:, 2] >> 4) & 0xF00) | (sc[:, 3] & 0xF000)
            d = db.astype(np.uint16).view(np.float16).astype(np.float32)
            assert d.min() >= 9e-5 and d.max() <= 2.01e-3
        elif codec == "nvfp4":
            e = (w.reshape(-1, 36)[:, 0:4] >> 3) & 15
            assert e.min() >= 1 and e.max() <= 6
        elif codec == "mxfp4":
            e = w.reshape(-1, 17)[:, 0]
            assert e.min() >= 115 and e.max() <= 125
        elif codec in ("q2_k", "q3_k", "tq2_0", "tq1_0"):
            off = {"q2_k": 80, "q3_k": 108, "tq2_0": 64, "tq1_0": 52}[codec]
            d = w[:, off:off + 2].copy().view(np.float16).astype(np.float32)
            assert d.min() >= 9e-5 and d.max() <= 2.01e-3
        elif codec == "q6_k":
            sc = w[:, 192:208].view(np.int8)
            assert sc.min() == -64 and sc.max() == 63
            d = w[:, 208:210].copy().view(np.float16).astype(np.float32)
            assert d.min() >= 9e-5 and d.max() <= 2.01e-3
        else:
            d = w[:, 0:2].copy().view(np.float16).astype(np.float32)
            assert d.min() >= 9e-5 and d.max() <= 2.01e-3


def test_q8_0_round_trip_through_gguf_quantizer():
    """Q8_0 is the one codec here gguf-py can quantize: real weights ->
    gguf-py quantize -> our dequantize equals gguf-py's dequantize bit for bit."""
    from gguf import quants as gq
    from gguf.constants import GGMLQuantizationType as T
    rng = np.random.default_rng(9)
    wf = (rng.standard_normal((64, 512)) * 0.02).astype(np.float32)
    w = gq.quantize(wf, T.Q8_0)
    assert w.shape == (64, 512 // 32 * 34)
    assert np.array_equal(bits(O.dequantize(w, "q8_0")), bits(gq.dequantize(w, T.Q8_0).astype(np.float32)))
    assert np.abs(O.dequantize(w, "q8_0") - wf).max() <= np.abs(wf).max() / 127


@pytest.mark.parametrize("codec,bb", [("q4_0", 18), ("q4_1", 20), ("q5_0", 22), ("q5_1", 24), ("tq2_0", 66),
                                     ("mxfp4", 17), ("tq1_0", 54)])
def test_legacy_round_trip_through_gguf_quantizer(codec, bb):
    """gguf-py quantizes the legacy 32-weight codecs too: its blocks
    dequantize bit-identically here."""
    from gguf import quants as gq
    from gguf.constants import GGMLQuantizationType as T
    qt = {"q4_0": T.Q4_0, "q4_1": T.Q4_1, "q5_0": T.Q5_0, "q5_1": T.Q5_1, "tq2_0": T.TQ2_0, "mxfp4": T.MXFP4,
          "tq1_0": T.TQ1_0, "nvfp4": T.NVFP4}[codec]
    rng = np.random.default_rng(10)
    wf = (rng.standard_normal((32, 1024)) * 0.02).astype(np.float32)
    w = gq.quantize(wf, qt)
    assert w.shape == (32, 1024 // {"tq2_0": 256, "tq1_0": 256, "nvfp4": 64}.get(codec, 32) * bb)
    assert np.array_equal(bits(O.dequantize(w, codec)), bits(gq.dequantize(w, qt).astype(np.float32)))


@pytest.mark.slow
@pytest.mark.parametrize("codec", ["q4_k", "q6_k", "iq2_xxs"])
def test_oracle_matches_gguf_py_million_blocks(codec):
    """The north-star codecs: 2^20 seeded random super-blocks each (16 chunks
    of 65536), the C oracle bit-identical to gguf-py's dequantize."""
    gq = pytest.importorskip("gguf.quants")
    from gguf.constants import GGMLQuantizationType as T
    qt = {"q4_k": T.Q4_K, "q6_k": T.Q6_K, "iq2_xxs": T.IQ2_XXS}[codec]
    n = 0
    for chunk in range(16):
        w = synth.random_weight(codec, 256, 65536, seed=10_000 + chunk)
        assert np.array_equal(bits(O.dequantize(w, codec)), bits(gq.dequantize(w, qt))), chunk
        n += w.shape[0] * (w.shape[1] // synth.BLOCK_BYTES[synth.codec_id(codec)])
    assert n == 1 << 20
