"""Seeded synthetic K-quant / IQ-quant weights and activations.

There are no GGUF files or datasets on the benchmark hosts, so every weight is
a stack of random super-blocks drawn the way the benchmark configurations
prescribe:

* Q4_K (144 B): uniform random bytes, then the two fp16 scales ``d`` and
  ``dmin`` overwritten with fp16(U[1e-4, 2e-3]).  (Raw random fp16 bytes would
  hold NaN/Inf.)
* Q6_K (210 B): random ``ql``/``qh``, the 16 int8 sub-block scales uniform in
  [-64, 63], ``d`` (the last two bytes) fp16(U[1e-4, 2e-3]).
* IQ2_XXS (66 B): random ``qs`` words (grid indices, sign indices and 4-bit
  sub-scales all uniform), ``d`` fp16(U[1e-4, 2e-3]).
* Q5_K (176 B): as Q4_K (``d``, ``dmin`` fp16(U[1e-4, 2e-3]), the rest random).
* Q8_0 (34 B per 32 weights, counted here as 272 B per 256): random int8
  quants, ``d`` fp16(U[1e-4, 2e-3]).
* IQ3_XXS (98 B), IQ4_XS (136 B): random bytes, ``d`` (the first two bytes)
  fp16(U[1e-4, 2e-3]).
* Q2_K (84 B): random scale and quant bytes, ``d``, ``dmin`` (the last four
  bytes) fp16(U[1e-4, 2e-3]).  Q3_K (110 B): random, ``d`` (the last two
  bytes) fp16(U[1e-4, 2e-3]).
* NVFP4 (36 B per 64 weights, 144 B per 256): random nibbles, the four UE4M3
  scale bytes of a block with exponent field 1..6 and any mantissa.
* TQ1_0 (54 B): random digit bytes, ``d`` (the last two bytes)
  fp16(U[1e-4, 2e-3]).
* MXFP4 (17 B per 32 weights, 136 B per 256): random nibbles, the e8m0
  exponent byte uniform in [115, 125] (scales 2^-13 .. 2^-3).  TQ2_0 (66 B):
  random 2-bit values, ``d`` fp16(U[1e-4, 2e-3]).
* IQ2_XS (74 B), IQ2_S (82 B), IQ3_S (110 B), IQ1_S (50 B): random, ``d``
  (the first two bytes) fp16(U[1e-4, 2e-3]).  IQ1_M (56 B): random, its fp16
  ``d`` (the top nibbles of the last four u16) fp16(U[1e-4, 2e-3]).
* Q4_0, IQ4_NL (18 B per 32 weights, counted as 144 B per 256), Q4_1 (20 B),
  Q5_0 (22 B), Q5_1 (24 B): random quant bytes, ``d`` fp16(U[1e-4, 2e-3]) per
  32-weight block, ``m`` (Q4_1 / Q5_1) fp16(-U[1e-3, 2e-2]).

Activations are bf16 N(0, 1); router logits are f32 N(0, 1).  All draws use
``numpy.random.default_rng(seed)``.
"""
from __future__ import annotations

import numpy as np

Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, Q2_K, Q3_K, TQ2_0, MXFP4 = 2, 3, 6, 7, 8, 10, 11, 35, 39
Q4_K, Q5_K, Q6_K, IQ2_XXS, IQ2_XS, IQ3_XXS, IQ4_NL, IQ3_S, IQ2_S, IQ4_XS = 12, 13, 14, 16, 17, 18, 20, 21, 22, 23
IQ1_S, IQ1_M, TQ1_0, NVFP4 = 19, 29, 34, 40
CODECS = {"q4_k": Q4_K, "q5_k": Q5_K, "q6_k": Q6_K, "iq2_xxs": IQ2_XXS, "q8_0": Q8_0, "iq3_xxs": IQ3_XXS,
          "iq4_xs": IQ4_XS, "q4_0": Q4_0, "iq4_nl": IQ4_NL, "q2_k": Q2_K, "q3_k": Q3_K, "q4_1": Q4_1,
          "q5_0": Q5_0, "q5_1": Q5_1, "tq2_0": TQ2_0, "mxfp4": MXFP4, "iq2_xs": IQ2_XS, "iq2_s": IQ2_S,
          "iq3_s": IQ3_S, "iq1_s": IQ1_S, "iq1_m": IQ1_M, "tq1_0": TQ1_0, "nvfp4": NVFP4}
CODEC_NAMES = {v: k for k, v in CODECS.items()}
# bytes per 256 weights (Q8_0: eight 34-byte ggml blocks of 32 weights)
BLOCK_BYTES = {Q4_K: 144, Q5_K: 176, Q6_K: 210, IQ2_XXS: 66, Q8_0: 272, IQ3_XXS: 98, IQ4_XS: 136,
               Q4_0: 144, IQ4_NL: 144, Q2_K: 84, Q3_K: 110, Q4_1: 160, Q5_0: 176, Q5_1: 192,
               TQ2_0: 66, MXFP4: 136, IQ2_XS: 74, IQ2_S: 82, IQ3_S: 110,
               IQ1_S: 50, IQ1_M: 56, TQ1_0: 54, NVFP4: 144}
QK = 256
D_LO, D_HI = 1e-4, 2e-3
# codecs handled in 256-weight groups of smaller ggml blocks: (weights, bytes)
# per block; a row may end in a partial group
SUB_BLOCK = {Q8_0: (32, 34), Q4_0: (32, 18), Q4_1: (32, 20), Q5_0: (32, 22), Q5_1: (32, 24), IQ4_NL: (32, 18),
             MXFP4: (32, 17), NVFP4: (64, 36)}


def codec_id(codec) -> int:
    if isinstance(codec, str):
        try:
            return CODECS[codec.lower()]
        except KeyError:
            raise ValueError(f"unknown K-quant codec {codec!r}") from None
    return int(codec)


def row_bytes(codec, k: int) -> int:
    c = codec_id(codec)
    if k % QK:
        raise ValueError(f"K={k} is not a whole number of {QK}-weight blocks")
    return k // QK * BLOCK_BYTES[c]


def _fp16_bytes(rng, n: int) -> np.ndarray:
    v = rng.uniform(D_LO, D_HI, size=n).astype(np.float16)
    return v.view(np.uint8).reshape(n, 2)


def random_blocks(codec, n_blocks: int, seed: int = 0) -> np.ndarray:
    """``[n_blocks, bpb]`` uint8 of seeded random super-blocks."""
    c = codec_id(codec)
    rng = np.random.default_rng(seed)
    bpb = BLOCK_BYTES[c]
    b = rng.integers(0, 256, size=(n_blocks, bpb), dtype=np.uint8)
    if c in (Q4_K, Q5_K):
        b[:, 0:2] = _fp16_bytes(rng, n_blocks)
        b[:, 2:4] = _fp16_bytes(rng, n_blocks)
    elif c == Q6_K:
        b[:, 192:208] = rng.integers(-64, 64, size=(n_blocks, 16), dtype=np.int8).view(np.uint8)
        b[:, 208:210] = _fp16_bytes(rng, n_blocks)
    elif c == IQ1_M:  # d's four nibbles sit in the top nibbles of the last four u16
        dbits = _fp16_bytes(rng, n_blocks).copy().view(np.uint16).reshape(n_blocks).astype(np.uint16)
        s = b[:, 48:56].copy().view(np.uint16).reshape(n_blocks, 4)
        for t in range(4):
            s[:, t] = (s[:, t] & np.uint16(0x0FFF)) | (((dbits >> np.uint16(4 * t)) & np.uint16(15)) << np.uint16(12))
        b[:, 48:56] = s.view(np.uint8).reshape(n_blocks, 8)
    elif c in (IQ2_XXS, IQ3_XXS, IQ4_XS, IQ2_XS, IQ2_S, IQ3_S, IQ1_S):
        b[:, 0:2] = _fp16_bytes(rng, n_blocks)
    elif c == Q8_0:  # eight (fp16 d, 32 x int8) blocks per 256 weights
        sub = b.reshape(n_blocks * 8, 34)
        sub[:, 0:2] = _fp16_bytes(rng, n_blocks * 8)
    elif c == Q2_K:
        b[:, 80:82] = _fp16_bytes(rng, n_blocks)
        b[:, 82:84] = _fp16_bytes(rng, n_blocks)
    elif c == Q3_K:
        b[:, 108:110] = _fp16_bytes(rng, n_blocks)
    elif c == TQ2_0:
        b[:, 64:66] = _fp16_bytes(rng, n_blocks)
    elif c == TQ1_0:
        b[:, 52:54] = _fp16_bytes(rng, n_blocks)
    elif c == NVFP4:  # four 36-byte blocks per 256 weights
        sub = b.reshape(n_blocks * 4, 36)
        sub[:, 0:4] = (rng.integers(1, 7, size=(n_blocks * 4, 4)) << 3 | rng.integers(0, 8, size=(n_blocks * 4, 4)))
    elif c == MXFP4:
        b.reshape(n_blocks * 8, 17)[:, 0] = rng.integers(115, 126, size=n_blocks * 8, dtype=np.uint8)
    elif c in (Q4_0, Q4_1, Q5_0, Q5_1, IQ4_NL):  # eight 32-weight blocks per 256 weights
        sub = b.reshape(n_blocks * 8, BLOCK_BYTES[c] // 8)
        sub[:, 0:2] = _fp16_bytes(rng, n_blocks * 8)
        if c in (Q4_1, Q5_1):
            sub[:, 2:4] = (-rng.uniform(1e-3, 2e-2, size=n_blocks * 8)).astype(np.float16).view(np.uint8).reshape(-1, 2)
    else:
        raise ValueError(codec)
    return b


def random_weight(codec, n: int, k: int, seed: int = 0, experts: int | None = None) -> np.ndarray:
    """Wire bytes ``[n, k/256*bpb]`` (or ``[experts, n, ...]``)."""
    c = codec_id(codec)
    nb = k // QK
    e = 1 if experts is None else experts
    b = random_blocks(c, e * n * nb, seed)
    shape = (n, nb * BLOCK_BYTES[c]) if experts is None else (e, n, nb * BLOCK_BYTES[c])
    return b.reshape(shape)


def random_weight_ragged(codec, n: int, k: int, seed: int = 0) -> np.ndarray:
    """Wire bytes [n, k / bw * bb] of a 32/64-weight-block codec for any K that
    is a whole number of its blocks (the last 256-weight group may be partial)."""
    c = codec_id(codec)
    bw, bb = SUB_BLOCK[c]
    if k % bw:
        raise ValueError(f"K={k} is not a whole number of {bw}-weight blocks")
    full = random_weight(c, n, -(-k // QK) * QK, seed=seed)
    return np.ascontiguousarray(full[:, : k // bw * bb])


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def random_activations(m: int, k: int, seed: int = 0) -> np.ndarray:
    """bf16 N(0,1) activations as uint16 bits ``[m, k]``."""
    rng = np.random.default_rng(seed)
    return f32_to_bf16_bits(rng.standard_normal((m, k), dtype=np.float32))


def random_logits(t: int, e: int, seed: int = 0) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return rng.standard_normal((t, e), dtype=np.float32)


# Llama-3-8B decoder layer, Q4_K_M-style (benchmark configuration 2/3):
# (name, codec, out N, in K) in projection order; weight seed = position.
LLAMA3_8B_LAYER = (
    ("q_proj", "q4_k", 4096, 4096),
    ("k_proj", "q4_k", 1024, 4096),
    ("v_proj", "q4_k", 1024, 4096),
    ("o_proj", "q4_k", 4096, 4096),
    ("gate_proj", "q4_k", 14336, 4096),
    ("up_proj", "q4_k", 14336, 4096),
    ("down_proj", "q6_k", 4096, 14336),
)

# MoE expert layers (benchmark configurations 4 and 5)
QWEN3_30B_A3B_MOE = dict(experts=128, top_k=8, hidden=2048, ffn=768,
                         gate_codec="q4_k", up_codec="q4_k", down_codec="q6_k")
DEEPSEEK_V3_IQ2_MOE = dict(experts=256, top_k=8, hidden=7168, ffn=2048,
                           gate_codec="iq2_xxs", up_codec="iq2_xxs", down_codec="iq2_xxs")


def layer_weight_bytes(layer=LLAMA3_8B_LAYER) -> int:
    return sum(n * row_bytes(c, k) for _, c, n, k in layer)
