"""CPU oracle for the K-quant / IQ-quant fused dequantize-and-multiply path.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline legs of ``bench.py`` import this module; the product package
(``gmlx_b200``) never does.

Two restatements of the reference's block arithmetic live here:

* ``libkq_oracle.so`` (``kq_oracle.c``, OpenMP) -- dequantize, dequantize-then-
  matmul and the MoE router; it is the fast checker and the timed CPU baseline.
* ``np_dequantize`` -- a pure-numpy statement of the same three decoders used
  to cross-check the C file on small inputs.

Both follow gguf-py 0.19.0 ``gguf/quants.py`` (Q4_K ``:475-522``, Q6_K
``:552-572``, IQ2_XXS ``:766-829``), the ggml-format restatement that gmlx
itself depends on (gmlx ``pyproject.toml:62``); the external mlx-kquant
kernels that gmlx calls (gmlx ``modules.py:35-40``) are not available.  The
tests pin both against gguf-py and against committed golden vectors.

MoE helpers restate gmlx's routing forward (``gmlx/moe_experts.py:226-240``)
and the fused decode ops' semantics (``gmlx/modules.py:514-605``).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libkq_oracle.so")

Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, Q2_K, Q3_K, TQ2_0, MXFP4 = 2, 3, 6, 7, 8, 10, 11, 35, 39
Q4_K, Q5_K, Q6_K, IQ2_XXS, IQ2_XS, IQ3_XXS, IQ4_NL, IQ3_S, IQ2_S, IQ4_XS = 12, 13, 14, 16, 17, 18, 20, 21, 22, 23
IQ1_S, IQ1_M, TQ1_0, NVFP4 = 19, 29, 34, 40
CODEC_IDS = {"q4_k": Q4_K, "q5_k": Q5_K, "q6_k": Q6_K, "iq2_xxs": IQ2_XXS, "q8_0": Q8_0, "iq3_xxs": IQ3_XXS,
             "iq4_xs": IQ4_XS, "q4_0": Q4_0, "iq4_nl": IQ4_NL, "q2_k": Q2_K, "q3_k": Q3_K, "q4_1": Q4_1,
             "q5_0": Q5_0, "q5_1": Q5_1, "tq2_0": TQ2_0, "mxfp4": MXFP4, "iq2_xs": IQ2_XS, "iq2_s": IQ2_S,
             "iq3_s": IQ3_S, "iq1_s": IQ1_S, "iq1_m": IQ1_M, "tq1_0": TQ1_0, "nvfp4": NVFP4}
BLOCK_BYTES = {Q4_K: 144, Q5_K: 176, Q6_K: 210, IQ2_XXS: 66, Q8_0: 272, IQ3_XXS: 98, IQ4_XS: 136,
               Q4_0: 144, IQ4_NL: 144, Q2_K: 84, Q3_K: 110, Q4_1: 160, Q5_0: 176, Q5_1: 192,
               TQ2_0: 66, MXFP4: 136, IQ2_XS: 74, IQ2_S: 82, IQ3_S: 110,
               IQ1_S: 50, IQ1_M: 56, TQ1_0: 54, NVFP4: 144}  # per 256 weights
QK = 256

_lib = None


def build(force: bool = False) -> str:
    """Compile ``libkq_oracle.so`` with the committed Makefile."""
    if force or not os.path.exists(LIB_PATH):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        i64, vp, i32 = ctypes.c_int64, ctypes.c_void_p, ctypes.c_int
        L.kqo_dequantize.argtypes = [i32, vp, i64, i64, i64, vp, i32]
        L.kqo_matmul.argtypes = [i32, vp, i32, i64, i64, vp, i64, i64, vp, i32]
        L.kqo_router_topk.argtypes = [vp, i64, i64, i32, i32, vp, vp]
        for f in (L.kqo_dequantize, L.kqo_matmul, L.kqo_router_topk):
            f.restype = i32
        _lib = L
    return _lib


def codec_id(codec) -> int:
    return CODEC_IDS[codec.lower()] if isinstance(codec, str) else int(codec)


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def dequantize(w: np.ndarray, codec, threads: int = 0) -> np.ndarray:
    """Wire bytes ``[rows, nb*bpb]`` (uint8, C-contiguous) -> f32 ``[rows, nb*256]``."""
    c = codec_id(codec)
    w = np.ascontiguousarray(w, dtype=np.uint8)
    rows, nbytes = w.reshape(-1, w.shape[-1]).shape
    assert nbytes % BLOCK_BYTES[c] == 0
    k = nbytes // BLOCK_BYTES[c] * QK
    out = np.empty((rows, k), np.float32)
    rc = lib().kqo_dequantize(c, _ptr(w), rows, k, nbytes, _ptr(out), threads)
    assert rc == 0, rc
    return out.reshape(*w.shape[:-1], k)


def matmul(x_bf16_bits: np.ndarray, w: np.ndarray, codec, threads: int = 0) -> np.ndarray:
    """``y = x @ dequant(w).T`` in f32; x given as uint16 bf16 bits ``[M, K]``."""
    c = codec_id(codec)
    x = np.ascontiguousarray(x_bf16_bits, dtype=np.uint16)
    w = np.ascontiguousarray(w, dtype=np.uint8)
    m, k = x.shape
    n, nbytes = w.shape
    assert nbytes // BLOCK_BYTES[c] * QK == k
    y = np.empty((m, n), np.float32)
    rc = lib().kqo_matmul(c, _ptr(x), 1, m, k, _ptr(w), n, nbytes, _ptr(y), threads)
    assert rc == 0, rc
    return y


def router_topk(logits: np.ndarray, k: int, norm_topk_prob: bool = True):
    """softmax -> top-k -> optional renorm; returns (idx int32 [T,k], scores f32 [T,k])."""
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    t, e = lg.shape
    idx = np.empty((t, k), np.int32)
    sc = np.empty((t, k), np.float32)
    rc = lib().kqo_router_topk(_ptr(lg), t, e, k, int(norm_topk_prob), _ptr(idx), _ptr(sc))
    assert rc == 0, rc
    return idx, sc


# --------------------------------------------------------------------------
# bf16 helpers (round-to-nearest-even, as torch and the kernels round)

def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return r.astype(np.uint16)


# --------------------------------------------------------------------------
# pure-numpy restatement (small inputs)

def _half(b2: np.ndarray) -> np.ndarray:
    return b2.copy().view(np.float16).astype(np.float32)


def np_dequantize(w: np.ndarray, codec) -> np.ndarray:
    """numpy statement of the decoders (follows gguf/quants.py)."""
    c = codec_id(codec)
    bpb = BLOCK_BYTES[c]
    blocks = np.ascontiguousarray(w, np.uint8).reshape(-1, bpb)
    n = blocks.shape[0]
    if c == Q4_K:  # quants.py:504-522
        d = _half(blocks[:, 0:2]).reshape(n, 1)
        dmin = _half(blocks[:, 2:4]).reshape(n, 1)
        s = blocks[:, 4:16].astype(np.uint8)
        sc = np.concatenate([s[:, 0:4] & 63, (s[:, 8:12] & 15) | ((s[:, 0:4] >> 2) & 48)], 1)
        mn = np.concatenate([s[:, 4:8] & 63, (s[:, 8:12] >> 4) | ((s[:, 4:8] >> 2) & 48)], 1)
        q = blocks[:, 16:].reshape(n, 4, 1, 32) >> np.array([0, 4], np.uint8).reshape(1, 1, 2, 1)
        q = (q & 15).reshape(n, 8, 32).astype(np.float32)
        dl = (d * sc.astype(np.float32)).reshape(n, 8, 1)
        ml = (dmin * mn.astype(np.float32)).reshape(n, 8, 1)
        out = dl * q - ml
    elif c == Q5_K:  # quants.py:525-549
        d = _half(blocks[:, 0:2]).reshape(n, 1)
        dmin = _half(blocks[:, 2:4]).reshape(n, 1)
        s = blocks[:, 4:16].astype(np.uint8)
        sc = np.concatenate([s[:, 0:4] & 63, (s[:, 8:12] & 15) | ((s[:, 0:4] >> 2) & 48)], 1)
        mn = np.concatenate([s[:, 4:8] & 63, (s[:, 8:12] >> 4) | ((s[:, 4:8] >> 2) & 48)], 1)
        qh = blocks[:, 16:48].reshape(n, 1, 32) >> np.arange(8, dtype=np.uint8).reshape(1, 8, 1)
        ql = blocks[:, 48:].reshape(n, 4, 1, 32) >> np.array([0, 4], np.uint8).reshape(1, 1, 2, 1)
        q = ((ql & 15).reshape(n, 8, 32) | ((qh & 1) << 4)).astype(np.float32)
        dl = (d * sc.astype(np.float32)).reshape(n, 8, 1)
        ml = (dmin * mn.astype(np.float32)).reshape(n, 8, 1)
        out = dl * q - ml
    elif c == Q6_K:  # quants.py:554-572
        ql, qh = blocks[:, :128], blocks[:, 128:192]
        sc = blocks[:, 192:208].view(np.int8).astype(np.float32)
        d = _half(blocks[:, 208:210]).reshape(n, 1)
        dl = (d * sc).reshape(n, 16, 1)
        lo = (ql.reshape(n, 2, 1, 64) >> np.array([0, 4], np.uint8).reshape(1, 1, 2, 1)) & 15
        hi = (qh.reshape(n, 2, 1, 32) >> np.array([0, 2, 4, 6], np.uint8).reshape(1, 1, 4, 1)) & 3
        q = (lo.reshape(n, 8, 32) | (hi.reshape(n, 8, 32) << 4)).astype(np.int8) - np.int8(32)
        out = dl * q.reshape(n, 16, 16).astype(np.float32)
    elif c == Q8_0:  # Q8_0.dequantize_blocks: eight (fp16 d, 32 x int8) blocks per 256 weights
        sub = blocks.reshape(n * 8, 34)
        d = _half(sub[:, 0:2]).reshape(n * 8, 1)
        out = sub[:, 2:].copy().view(np.int8).astype(np.float32) * d
    elif c == IQ2_XXS:  # quants.py:802-829
        from_grid = iq2xxs_grid()
        d = _half(blocks[:, 0:2]).reshape(n, 1)
        qs = blocks[:, 2:].copy().view(np.uint32).reshape(n, 8, 2)
        db = (d * (np.float32(0.5) + (qs[..., 1] >> 28).astype(np.float32)) * np.float32(0.25))
        db = db.reshape(n, 8, 1, 1)
        sidx = (qs[..., 1].reshape(n, 8, 1) >> np.array([0, 7, 14, 21], np.uint32)) & 127
        ks = ksigns_table()[sidx].reshape(n, 8, 4, 1)
        sgn = np.where((ks >> np.arange(8, dtype=np.uint8)) & 1, np.float32(-1), np.float32(1))
        gidx = qs[..., 0].copy().view(np.uint8).reshape(n, 8, 4)
        g = from_grid[gidx].astype(np.float32)
        out = db * g * sgn
    elif c == IQ3_XXS:  # quants.py:1027-1054
        d = _half(blocks[:, 0:2]).reshape(n, 1)
        gidx = blocks[:, 2:66].reshape(n, 8, 4, 2)
        aux = blocks[:, 66:98].copy().view(np.uint32).reshape(n, 8)
        db = (d * (np.float32(0.5) + (aux >> 28).astype(np.float32)) * np.float32(0.5)).reshape(n, 8, 1, 1)
        sidx = (aux.reshape(n, 8, 1) >> np.array([0, 7, 14, 21], np.uint32)) & 127
        ks = ksigns_table()[sidx].reshape(n, 8, 4, 1)
        sgn = np.where((ks >> np.arange(8, dtype=np.uint8)) & 1, np.float32(-1), np.float32(1))
        g = iq3xxs_grid()[gidx].reshape(n, 8, 4, 8).astype(np.float32)
        out = db * g * sgn
    elif c == IQ4_XS:  # quants.py:1351-1377
        d = _half(blocks[:, 0:2]).reshape(n, 1)
        sh = blocks[:, 2:4].copy().view(np.uint16).reshape(n, 1)
        sl = blocks[:, 4:8].reshape(n, 4, 1) >> np.array([0, 4], np.uint8).reshape(1, 1, 2)
        ls = (sl.reshape(n, 8) & 15).astype(np.int32) | (((sh >> (2 * np.arange(8, dtype=np.uint16))) & 3) << 4)
        dl = (d * (ls - 32).astype(np.float32)).reshape(n, 8, 1)
        q = blocks[:, 8:].reshape(n, 8, 1, 16) >> np.array([0, 4], np.uint8).reshape(1, 1, 2, 1)
        kv = np.array(_table_values("KQ_IQ4NL_VALUES_INIT"), np.float32)
        out = dl * kv[(q & 15).reshape(n, 8, 32)]
    elif c == Q2_K:  # quants.py:404-428
        sc = blocks[:, 0:16]
        d = _half(blocks[:, 80:82]).reshape(n, 1, 1)
        dmin = _half(blocks[:, 82:84]).reshape(n, 1, 1)
        q = (blocks[:, 16:80].reshape(n, 2, 1, 32) >> np.array([0, 2, 4, 6], np.uint8).reshape(1, 1, 4, 1)) & 3
        q = q.reshape(n, 16, 16).astype(np.float32)
        out = (d * (sc & 15).astype(np.float32).reshape(n, 16, 1)) * q - dmin * (sc >> 4).astype(np.float32).reshape(n, 16, 1)
    elif c == Q3_K:  # quants.py:431-472
        hm, qs, s = blocks[:, 0:32], blocks[:, 32:96], blocks[:, 96:108]
        d = _half(blocks[:, 108:110]).reshape(n, 1, 1)
        lo = np.concatenate([s[:, 0:8] & 15, s[:, 0:8] >> 4], 1)
        hi = (s[:, 8:12].reshape(n, 1, 4) >> np.array([0, 2, 4, 6], np.uint8).reshape(1, 4, 1)).reshape(n, 16) & 3
        sc = ((lo | (hi << 4)).astype(np.int16) - 32).astype(np.float32)
        q2 = (qs.reshape(n, 2, 1, 32) >> np.array([0, 2, 4, 6], np.uint8).reshape(1, 1, 4, 1)) & 3
        hb = (hm.reshape(n, 1, 32) >> np.arange(8, dtype=np.uint8).reshape(1, 8, 1)) & 1
        q = q2.reshape(n, 8, 32).astype(np.int16) - 4 * (1 - hb.astype(np.int16))
        out = (d * sc.reshape(n, 16, 1)) * q.reshape(n, 16, 16).astype(np.float32)
    elif c == MXFP4:  # MXFP4.dequantize_blocks: eight (e8m0 e, 16 nibble bytes) blocks
        sub = blocks.reshape(n * 8, 17)
        e = sub[:, 0].astype(np.uint32)
        bits_ = np.where(e < 2, np.uint32(0x00200000) << e, (e - 1) << np.uint32(23)).astype(np.uint32)
        d = bits_.view(np.float32).reshape(n * 8, 1)
        q = ((sub[:, 1:].reshape(n * 8, 1, 16) >> np.array([0, 4], np.uint8).reshape(1, 2, 1)) & 15).reshape(n * 8, 32)
        out = d * np.array(_table_values("KQ_MXFP4_VALUES_INIT"), np.float32)[q]
    elif c in (IQ2_XS, IQ2_S):  # IQ2_XS / IQ2_S.dequantize_blocks: 32 entries of 8 weights
        d = _half(blocks[:, 0:2]).reshape(n, 1, 1)
        if c == IQ2_XS:
            v = blocks[:, 2:66].copy().view(np.uint16).reshape(n, 32).astype(np.int64)
            idx, sg = v & 511, ksigns_table()[v >> 9]
            sc = blocks[:, 66:74]
            grid = _grid("KQ_IQ2XS_GRID_INIT", 8, 512)
        else:
            qh = (blocks[:, 66:74].reshape(n, 8, 1) >> np.array([0, 2, 4, 6], np.uint8).reshape(1, 1, 4)) & 3
            idx = blocks[:, 2:34].astype(np.int64) | (qh.reshape(n, 32).astype(np.int64) << 8)
            sg = blocks[:, 34:66]
            sc = blocks[:, 74:82]
            grid = _grid("KQ_IQ2S_GRID_INIT", 8, 1024)
        s = ((sc.reshape(n, 8, 1) >> np.array([0, 4], np.uint8).reshape(1, 1, 2)) & 15).reshape(n, 16)
        db = (d * (np.float32(0.5) + s.astype(np.float32).reshape(n, 16, 1)) * np.float32(0.25)).reshape(n, 16, 1, 1)
        sgn = np.where((sg.reshape(n, 32, 1) >> np.arange(8, dtype=np.uint8)) & 1, np.float32(-1), np.float32(1))
        out = db * grid[idx].astype(np.float32).reshape(n, 16, 2, 8) * sgn.reshape(n, 16, 2, 8)
    elif c == IQ3_S:  # IQ3_S.dequantize_blocks: 64 entries of 4 weights
        d = _half(blocks[:, 0:2]).reshape(n, 1)
        qh = (blocks[:, 66:74].reshape(n, 8, 1) >> np.arange(8, dtype=np.uint8).reshape(1, 1, 8)) & 1
        idx = blocks[:, 2:66].astype(np.int64) | (qh.reshape(n, 64).astype(np.int64) << 8)
        s = ((blocks[:, 106:110].reshape(n, 4, 1) >> np.array([0, 4], np.uint8).reshape(1, 1, 2)) & 15).reshape(n, 8)
        db = (d * (1 + 2 * s).astype(np.float32)).reshape(n, 8, 1, 1)
        sgn = np.where((blocks[:, 74:106].reshape(n, 32, 1) >> np.arange(8, dtype=np.uint8)) & 1, np.float32(-1),
                       np.float32(1))
        out = db * _grid("KQ_IQ3S_GRID_INIT", 4, 512)[idx].astype(np.float32).reshape(n, 8, 4, 8) * \
            sgn.reshape(n, 8, 4, 8)
    elif c in (IQ1_S, IQ1_M):  # IQ1_S / IQ1_M.dequantize_blocks: 32 entries of 8 weights
        grid = _grid("KQ_IQ1S_GRID_INIT", 8, 2048).view(np.int8).astype(np.float32)
        if c == IQ1_S:
            d = _half(blocks[:, 0:2]).reshape(n, 1)
            qh = blocks[:, 34:50].copy().view(np.uint16).reshape(n, 8).astype(np.int64)
            dl = np.repeat(d * (2 * ((qh >> 12) & 7) + 1).astype(np.float32), 4, axis=1)
            delta = np.repeat(np.where(qh & 0x8000, np.float32(-0.125), np.float32(0.125)), 4, axis=1)
            hi = ((qh.reshape(n, 8, 1) >> np.array([0, 3, 6, 9]).reshape(1, 1, 4)) & 7).reshape(n, 32)
            idx = blocks[:, 2:34].astype(np.int64) | (hi << 8)
        else:
            s = blocks[:, 48:56].copy().view(np.uint16).reshape(n, 4).astype(np.int64)
            dbits = (s[:, 0] >> 12) | ((s[:, 1] >> 8) & 0xF0) | ((s[:, 2] >> 4) & 0xF00) | (s[:, 3] & 0xF000)
            d = dbits.astype(np.uint16).view(np.float16).astype(np.float32).reshape(n, 1)
            sc = ((s.reshape(n, 4, 1) >> np.array([0, 3, 6, 9]).reshape(1, 1, 4)) & 7).reshape(n, 16)
            dl = np.repeat(d * (2 * sc + 1).astype(np.float32), 2, axis=1)
            nib = ((blocks[:, 32:48].reshape(n, 16, 1) >> np.array([0, 4], np.uint8).reshape(1, 1, 2)) & 15).reshape(n, 32)
            delta = np.where(nib & 8, np.float32(-0.125), np.float32(0.125))
            idx = blocks[:, 0:32].astype(np.int64) | ((nib & 7).astype(np.int64) << 8)
        out = dl.reshape(n, 32, 1) * (grid[idx] + delta.reshape(n, 32, 1))
    elif c == NVFP4:  # NVFP4.dequantize_blocks (quants.py:707-763): four 36-byte blocks of 64
        sub = blocks.reshape(n * 4, 36)
        x = sub[:, 0:4].astype(np.int32)
        e, m = (x >> 3) & 15, (x & 7).astype(np.float32)
        raw = np.where(e == 0, m * np.float32(2.0 ** -9),
                       (np.float32(1) + m / np.float32(8)) * np.exp2(e - 7).astype(np.float32))
        d = np.where((x == 0) | (x == 0x7F), np.float32(0), raw * np.float32(0.5)).astype(np.float32)
        q = sub[:, 4:].reshape(n * 4, 4, 1, 8) >> np.array([0, 4], np.uint8).reshape(1, 1, 2, 1)
        v = np.array(_table_values("KQ_MXFP4_VALUES_INIT"), np.float32)[(q & 15).reshape(n * 4, 4, 16)]
        out = d.reshape(n * 4, 4, 1) * v
    elif c == TQ1_0:  # TQ1_0.dequantize_blocks (quants.py:602-620)
        p5 = np.array([1, 3, 9, 27, 81], np.uint16)
        t0 = (blocks[:, 0:32].reshape(n, 1, 32).astype(np.uint16) * p5.reshape(1, 5, 1)) & 255
        t1 = (blocks[:, 32:48].reshape(n, 1, 16).astype(np.uint16) * p5.reshape(1, 5, 1)) & 255
        t2 = (blocks[:, 48:52].reshape(n, 1, 4).astype(np.uint16) * p5[:4].reshape(1, 4, 1)) & 255
        t = np.concatenate([t0.reshape(n, 160), t1.reshape(n, 80), t2.reshape(n, 16)], 1)
        out = _half(blocks[:, 52:54]).reshape(n, 1) * (((t * 3) >> 8).astype(np.float32) - np.float32(1))
    elif c == TQ2_0:  # TQ2_0.dequantize_blocks
        d = _half(blocks[:, 64:66]).reshape(n, 1)
        q = (blocks[:, 0:64].reshape(n, 2, 1, 32) >> np.array([0, 2, 4, 6], np.uint8).reshape(1, 1, 4, 1)) & 3
        out = d * (q.reshape(n, 256).astype(np.float32) - np.float32(1))
    elif c in (Q4_0, Q4_1, Q5_0, Q5_1, IQ4_NL):  # quants.py:241-336 / 1333-1348: eight 32-weight blocks
        has_m, has_h = c in (Q4_1, Q5_1), c in (Q5_0, Q5_1)
        bb = 18 + 2 * has_m + 4 * has_h
        sub = blocks.reshape(n * 8, bb)
        d = _half(sub[:, 0:2]).reshape(n * 8, 1)
        q = (sub[:, bb - 16:].reshape(n * 8, 1, 16) >> np.array([0, 4], np.uint8).reshape(1, 2, 1)) & 15
        q = q.reshape(n * 8, 32).astype(np.int32)
        if has_h:
            qh = sub[:, 2 + 2 * has_m:6 + 2 * has_m].copy().view(np.uint32).reshape(n * 8, 1)
            q |= (((qh >> np.arange(32, dtype=np.uint32)) & 1) << 4).astype(np.int32)
        if c == IQ4_NL:
            kv = np.array(_table_values("KQ_IQ4NL_VALUES_INIT"), np.float32)
            out = d * kv[q]
        elif has_m:
            out = d * q.astype(np.float32) + _half(sub[:, 2:4]).reshape(n * 8, 1)
        else:
            out = d * (q - (8 if c == Q4_0 else 16)).astype(np.float32)
    else:
        raise ValueError(codec)
    return out.reshape(*np.asarray(w).shape[:-1], -1).astype(np.float32)


def ksigns_table() -> np.ndarray:
    """ggml ksigns: 7-bit index with an even-parity bit 7."""
    i = np.arange(128, dtype=np.uint8)
    p = np.zeros(128, np.uint8)
    for b in range(7):
        p ^= (i >> b) & 1
    return (i | (p << 7)).astype(np.uint8)


_GRIDS = {}


def _table_values(macro: str) -> list:
    """Integer entries of one ``#define <macro> { ... }`` of the generated header."""
    hdr = os.path.join(HERE, "..", "gmlx_b200", "csrc", "_gen", "kq_tables.h")
    if not os.path.exists(hdr):
        build(force=True)
    body = open(hdr).read().split("#define " + macro, 1)[1].split("{", 1)[1].split("}")[0]
    return [int(t.rstrip("ul"), 0) for t in body.replace("\\", " ").replace(",", " ").split()]


def _grid(macro: str, width: int, entries: int = 256) -> np.ndarray:
    if macro not in _GRIDS:
        vals = _table_values(macro)
        assert len(vals) == entries
        _GRIDS[macro] = np.array([[(v >> (8 * i)) & 0xFF for i in range(width)] for v in vals], np.uint8)
    return _GRIDS[macro]


def iq2xxs_grid() -> np.ndarray:
    """``[256, 8]`` uint8 magnitudes, parsed from the generated kernel header."""
    return _grid("KQ_IQ2XXS_GRID_INIT", 8)


def iq3xxs_grid() -> np.ndarray:
    """``[256, 4]`` uint8 magnitudes, parsed from the generated kernel header."""
    return _grid("KQ_IQ3XXS_GRID_INIT", 4)
