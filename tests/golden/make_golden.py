"""Generate the committed golden vectors for the block formats.

Source of truth: gguf-py 0.19.0 (``gguf.quants.dequantize``), the restatement
of ggml's block formats that gmlx depends on (gmlx pyproject.toml:62).  The
reference's own kernels (external mlx-kquant) ship no numeric tests; these
vectors pin the oracle and the CUDA kernels instead.  Run from the repo root:

    python tests/golden/make_golden.py

Each codec gets (a) seeded random blocks per the benchmark statistics and
(b) known-answer / edge blocks:
  Q4_K   all-zero quants (w = -dmin*m), scale/min = 0 and 63 on every
         sub-block, one-hot sub-block scales;
  Q5_K   the same scale/min edges, fifth bits all 0 / all 1 / one sub-block
         at a time;
  Q8_0   quants -128, -127, 0, 127 and d = 0, negative d, the largest fp16;
  Q6_K   int8 scales at -128, -64, 0, 63, 127; quants all 0 / all 63;
  IQ2_XXS every grid index and every 7-bit sign index, ls = 0 and 15;
  IQ3_XXS the same sweep over its 256-entry grid;
  IQ4_XS  every nibble value, 6-bit scales 0 / 31 / 32 / 63, negative d;
  Q4_0    quants all 0 / all 15 / every value, d = 0, negative, 65504;
  Q4_1, Q5_0, Q5_1  the same with m = 0 / negative / positive and the fifth
          bits all clear / all set / alternating;
  MXFP4   every nibble value, exponents 0, 1 (subnormal scales), 2, 127, 140;
  IQ2_XS, IQ2_S, IQ3_S  every grid index, every sign pattern index / byte
          sweep, 4-bit scales 0 and 15;
  IQ1_S, IQ1_M  every grid index, both delta signs, 3-bit scales 0 and 7;
  TQ1_0   every byte value in every digit position, d < 0;
  NVFP4   every UE4M3 scale byte (0, subnormals, 0x7F, normals), every nibble;
  TQ2_0   values all 0 / 1 / 2 / 3 (3 is outside the ternary set but decodes), d < 0;
  IQ4_NL  every nibble value on every block, negative d;
  Q2_K    scale / min nibbles 0 and 15, quants all 0 / all 3, one-hot
          sub-block scales;
  Q3_K    6-bit scales 0 / 31 / 32 / 63 (-32 .. 31), high bits all set /
          all clear / one plane at a time.
Matmul references are x @ dequant(W).T in float64 for bf16 x (N(0,1)) plus
one-hot x rows, which must reproduce single dequantized columns exactly.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from gguf.constants import GGMLQuantizationType as T  # noqa: E402
from gguf.quants import dequantize  # noqa: E402

from gmlx_b200 import synth  # noqa: E402

QT = {"q4_k": T.Q4_K, "q5_k": T.Q5_K, "q6_k": T.Q6_K, "iq2_xxs": T.IQ2_XXS, "q8_0": T.Q8_0,
      "iq3_xxs": T.IQ3_XXS, "iq4_xs": T.IQ4_XS, "q4_0": T.Q4_0, "iq4_nl": T.IQ4_NL, "q2_k": T.Q2_K,
      "q3_k": T.Q3_K, "q4_1": T.Q4_1, "q5_0": T.Q5_0, "q5_1": T.Q5_1, "tq2_0": T.TQ2_0,
      "mxfp4": T.MXFP4, "iq2_xs": T.IQ2_XS, "iq2_s": T.IQ2_S, "iq3_s": T.IQ3_S,
      "iq1_s": T.IQ1_S, "iq1_m": T.IQ1_M, "tq1_0": T.TQ1_0, "nvfp4": T.NVFP4}


def fp16(v):
    return np.array([v], np.float16).view(np.uint8)


def edge_blocks(codec):
    rng = np.random.default_rng(123)
    blocks = []
    if codec == "q4_k":
        for sc_val, m_val in [(0, 0), (63, 63), (63, 0), (0, 63), (17, 42)]:
            b = np.zeros(144, np.uint8)
            b[0:2], b[2:4] = fp16(1e-3), fp16(5e-4)
            # pack sc/m = (sc_val, m_val) into all 8 sub-blocks (quants.py:479-501 layout)
            for j in range(4):
                b[4 + j] = (sc_val & 63) | ((sc_val >> 4) << 6)
                b[8 + j] = (m_val & 63) | ((m_val >> 4) << 6)
                b[12 + j] = (sc_val & 15) | ((m_val & 15) << 4)
            b[16:] = 0 if (sc_val, m_val) == (0, 0) else rng.integers(0, 256, 128, dtype=np.uint8)
            blocks.append(b)
        for one in range(8):  # one-hot sub-block scale, zero min
            b = np.zeros(144, np.uint8)
            b[0:2], b[2:4] = fp16(1e-3), fp16(1e-3)
            if one < 4:
                b[4 + one] = 1
            else:
                b[12 + one - 4] = 1
            b[16:] = rng.integers(0, 256, 128, dtype=np.uint8)
            blocks.append(b)
    elif codec == "q5_k":
        for sc_val, m_val, qh_fill in [(0, 0, 0), (63, 63, 255), (63, 0, 0), (0, 63, 255), (17, 42, None)]:
            b = np.zeros(176, np.uint8)
            b[0:2], b[2:4] = fp16(1e-3), fp16(5e-4)
            for j in range(4):
                b[4 + j] = (sc_val & 63) | ((sc_val >> 4) << 6)
                b[8 + j] = (m_val & 63) | ((m_val >> 4) << 6)
                b[12 + j] = (sc_val & 15) | ((m_val & 15) << 4)
            b[16:48] = rng.integers(0, 256, 32, dtype=np.uint8) if qh_fill is None else qh_fill
            b[48:] = 0 if (sc_val, m_val) == (0, 0) else rng.integers(0, 256, 128, dtype=np.uint8)
            blocks.append(b)
        for one in range(8):  # fifth bit set for one sub-block only, one-hot scale
            b = np.zeros(176, np.uint8)
            b[0:2], b[2:4] = fp16(1e-3), fp16(1e-3)
            b[4 + (one % 4)] = 1 if one < 4 else 0
            if one >= 4:
                b[12 + one - 4] = 1
            b[16:48] = 1 << one
            b[48:] = rng.integers(0, 256, 128, dtype=np.uint8)
            blocks.append(b)
    elif codec == "q8_0":  # 272-byte groups of eight 34-byte blocks
        for dv, qv in [(1e-3, -128), (1e-3, 127), (0.0, 55), (-2e-3, -127), (65504.0, 1), (5e-4, None)]:
            b = np.zeros((8, 34), np.uint8)
            b[:, 0:2] = fp16(dv)
            b[:, 2:] = (rng.integers(-128, 128, (8, 32)) if qv is None else np.full((8, 32), qv)).astype(np.int8).view(np.uint8)
            blocks.append(b.reshape(272))
    elif codec == "q6_k":
        for scv, qfill in [(-128, None), (-64, 0), (0, None), (63, 255), (127, None)]:
            b = rng.integers(0, 256, 210, dtype=np.uint8)
            if qfill is not None:
                b[:192] = qfill
            b[192:208] = np.array([scv] * 16, np.int8).view(np.uint8)
            b[208:210] = fp16(2e-3)
            blocks.append(b)
    elif codec == "iq3_xxs":
        # every grid index (64 per block -> 4 blocks), sign indices sweeping
        # 0..127, ls alternating 0 / 15 over the sub-blocks
        k = 0
        for blk in range(4):
            b = np.zeros(98, np.uint8)
            b[0:2] = fp16(1.5e-3 if blk % 2 else -7e-4)
            b[2:66] = np.arange(64 * blk, 64 * blk + 64, dtype=np.uint32).astype(np.uint8)
            for j in range(8):
                aux = 0
                for s in range(4):
                    aux |= ((k + s) % 128) << (7 * s)
                k += 4
                aux |= (15 if (j + blk) % 2 else 0) << 28
                b[66 + 4 * j:70 + 4 * j] = np.array([aux], np.uint32).view(np.uint8)
            blocks.append(b)
    elif codec == "q2_k":
        for scv, qv in [(0x00, 0x00), (0xff, 0xff), (0x0f, 0x55), (0xf0, None), (None, None)]:
            b = np.zeros(84, np.uint8)
            b[0:16] = rng.integers(0, 256, 16, dtype=np.uint8) if scv is None else scv
            b[16:80] = rng.integers(0, 256, 64, dtype=np.uint8) if qv is None else qv
            b[80:82], b[82:84] = fp16(1e-3), fp16(5e-4)
            blocks.append(b)
        for one in range(16):  # one-hot sub-block scale (min 0)
            b = np.zeros(84, np.uint8)
            b[one] = 1
            b[16:80] = rng.integers(0, 256, 64, dtype=np.uint8)
            b[80:82], b[82:84] = fp16(1e-3), fp16(1e-3)
            blocks.append(b)
    elif codec == "q3_k":
        for sv, hfill in [(0, 0x00), (63, 0xff), (32, None), (31, 0x55), (None, None)]:
            b = np.zeros(110, np.uint8)
            sc = rng.integers(0, 64, 16) if sv is None else np.full(16, sv)
            for j in range(16):
                b[96 + (j % 8)] |= (int(sc[j]) & 15) << (4 * (j // 8))
                b[104 + (j & 3)] |= ((int(sc[j]) >> 4) & 3) << (2 * (j >> 2))
            b[0:32] = rng.integers(0, 256, 32, dtype=np.uint8) if hfill is None else hfill
            b[32:96] = rng.integers(0, 256, 64, dtype=np.uint8)
            b[108:110] = fp16(1.5e-3)
            blocks.append(b)
        for plane in range(8):  # high bits set on one plane only
            b = rng.integers(0, 256, 110, dtype=np.uint8)
            b[0:32] = 1 << plane
            b[108:110] = fp16(-1e-3)
            blocks.append(b)
    elif codec in ("iq2_xs", "iq2_s", "iq3_s"):
        entries = {"iq2_xs": 512, "iq2_s": 1024, "iq3_s": 512}[codec]
        per = 64 if codec == "iq3_s" else 32  # index entries per block
        for blk in range(entries // per):
            b = rng.integers(0, 256, {"iq2_xs": 74, "iq2_s": 82, "iq3_s": 110}[codec], dtype=np.uint8)
            b[0:2] = fp16(1.5e-3 if blk % 2 else -7e-4)
            idx = np.arange(per * blk, per * blk + per)
            if codec == "iq2_xs":
                v = idx | ((idx % 128) << 9)
                b[2:66] = v.astype(np.uint16).view(np.uint8)
                b[66:74] = 0x00 if blk % 2 else 0xff
            elif codec == "iq2_s":
                b[2:34] = (idx & 255).astype(np.uint8)
                hi = (idx >> 8) & 3
                b[66:74] = (hi.reshape(8, 4) << np.array([0, 2, 4, 6])).sum(1).astype(np.uint8)
                b[34:66] = ((idx * 37) & 255).astype(np.uint8)
                b[74:82] = 0x00 if blk % 2 else 0xff
            else:
                b[2:66] = (idx & 255).astype(np.uint8)
                hi = (idx >> 8) & 1
                b[66:74] = (hi.reshape(8, 8) << np.arange(8)).sum(1).astype(np.uint8)
                b[74:106] = ((np.arange(32) * 53 + blk) & 255).astype(np.uint8)
                b[106:110] = 0x00 if blk % 2 else 0xff
            blocks.append(b)
    elif codec in ("iq1_s", "iq1_m"):
        for blk in range(64):
            idx = np.arange(32 * blk, 32 * blk + 32)
            if codec == "iq1_s":
                b = np.zeros(50, np.uint8)
                b[0:2] = fp16(1.5e-3 if blk % 2 else -7e-4)
                b[2:34] = (idx & 255).astype(np.uint8)
                hi = ((idx >> 8) & 7).reshape(8, 4)
                qh = (hi << np.array([0, 3, 6, 9])).sum(1) | ((7 if blk % 3 else 0) << 12) | ((blk % 2) << 15)
                b[34:50] = qh.astype(np.uint16).view(np.uint8)
            else:
                b = np.zeros(56, np.uint8)
                b[0:32] = (idx & 255).astype(np.uint8)
                nib = ((idx >> 8) & 7) | ((np.arange(32) + blk) % 2 << 3)
                b[32:48] = (nib[0::2] | (nib[1::2] << 4)).astype(np.uint8)
                dbits = int(np.array([1.5e-3 if blk % 2 else -7e-4], np.float16).view(np.uint16)[0])
                sv = 7 if blk % 3 else 0
                s = [(sv | sv << 3 | sv << 6 | sv << 9) | (((dbits >> (4 * t)) & 15) << 12) for t in range(4)]
                b[48:56] = np.array(s, np.uint16).view(np.uint8)
            blocks.append(b)
    elif codec == "mxfp4":
        for ev in (0, 1, 2, 127, 140, None):
            b = np.zeros((8, 17), np.uint8)
            b[:, 0] = rng.integers(110, 130, 8) if ev is None else ev
            b[:, 1:] = (np.arange(16) | (((np.arange(16) + 3) % 16) << 4)).astype(np.uint8)
            blocks.append(b.reshape(136))
    elif codec == "nvfp4":  # 144-byte groups of four 36-byte blocks
        for grp in range(16):
            b = np.zeros((4, 36), np.uint8)
            b[:, 0:4] = (np.arange(16) + 16 * grp).reshape(4, 4).astype(np.uint8)
            b[:, 4:] = ((np.arange(32) * 7 + grp) % 256).astype(np.uint8)
            blocks.append(b.reshape(144))
    elif codec == "tq1_0":
        for blk in range(6):
            b = np.zeros(54, np.uint8)
            b[0:52] = ((np.arange(52) + 52 * blk) % 256).astype(np.uint8)
            b[52:54] = fp16(-1e-3 if blk % 2 else 1.5e-3)
            blocks.append(b)
    elif codec == "tq2_0":
        for qv, dv in [(0x00, 1e-3), (0x55, 1e-3), (0xaa, -2e-3), (0xff, 5e-4), (None, 1.5e-3)]:
            b = np.zeros(66, np.uint8)
            b[0:64] = rng.integers(0, 256, 64, dtype=np.uint8) if qv is None else qv
            b[64:66] = fp16(dv)
            blocks.append(b)
    elif codec in ("q4_0", "iq4_nl", "q4_1", "q5_0", "q5_1"):  # groups of eight 32-weight blocks
        has_m, has_h = codec in ("q4_1", "q5_1"), codec in ("q5_0", "q5_1")
        bb = 18 + 2 * has_m + 4 * has_h
        cases = [(1e-3, 0x00, 0.0, 0x00), (1e-3, 0xff, -0.02, 0xff), (0.0, None, 0.01, 0x55),
                 (-2e-3, None, -1e-3, None), (65504.0, 0x88, 0.0, 0xaa), (5e-4, None, -0.5, None)]
        for dv, qv, mv, hv in cases:
            b = np.zeros((8, bb), np.uint8)
            b[:, 0:2] = fp16(dv)
            if has_m:
                b[:, 2:4] = fp16(mv)
            if has_h:
                o = 2 + 2 * has_m
                b[:, o:o + 4] = rng.integers(0, 256, (8, 4), dtype=np.uint8) if hv is None else hv
            if qv is None:  # every nibble value in both halves
                b[:, bb - 16:] = (np.arange(16) | (((np.arange(16) + 5) % 16) << 4)).astype(np.uint8)
            else:
                b[:, bb - 16:] = qv
            blocks.append(b.reshape(8 * bb))
    elif codec == "iq4_xs":
        # every nibble value on every sub-block; 6-bit scales 0, 31, 32, 63
        for blk, (dv, ls) in enumerate([(1e-3, 0), (1e-3, 63), (-2e-3, 32), (5e-4, 31), (1e-3, None)]):
            b = np.zeros(136, np.uint8)
            b[0:2] = fp16(dv)
            lsv = rng.integers(0, 64, 8) if ls is None else np.full(8, ls)
            sh = 0
            for j in range(8):
                sh |= int(lsv[j] >> 4) << (2 * j)
                b[4 + j // 2] |= int(lsv[j] & 15) << (4 * (j % 2))
            b[2:4] = np.array([sh], np.uint16).view(np.uint8)
            q = (np.arange(128) + blk) % 16
            b[8:] = (q | (((q + 7) % 16) << 4)).astype(np.uint8)
            blocks.append(b)
    else:
        # every grid index (4 per 8-byte group, 8 groups per block -> 8 blocks)
        # with sign indices sweeping 0..127 and ls alternating 0 / 15
        gi = np.arange(256, dtype=np.uint32)
        si = np.arange(128, dtype=np.uint32)
        k = 0
        for blk in range(8):
            b = np.zeros(66, np.uint8)
            b[0:2] = fp16(1.5e-3)
            for g in range(8):
                a0 = 0
                a1 = 0
                for s in range(4):
                    a0 |= int(gi[(k + s) % 256]) << (8 * s)
                    a1 |= int(si[(k + s) % 128]) << (7 * s)
                a1 |= (15 if (g + blk) % 2 else 0) << 28
                k += 4
                b[2 + 8 * g:6 + 8 * g] = np.array([a0], np.uint32).view(np.uint8)
                b[6 + 8 * g:10 + 8 * g] = np.array([a1], np.uint32).view(np.uint8)
            blocks.append(b)
    return np.stack(blocks)


def main():
    out = {}
    for codec in QT:
        k = 1024
        rand = synth.random_weight(codec, 12, k, seed=2024)
        edge = edge_blocks(codec)
        nb = k // 256
        pad = (-len(edge)) % nb
        if pad:
            edge = np.concatenate([edge, synth.random_blocks(codec, pad, seed=7)])
        edge = edge.reshape(-1, nb * edge.shape[1])
        w = np.concatenate([rand, edge], 0)
        deq = dequantize(w, QT[codec]).astype(np.float32)
        x = synth.random_activations(3, k, seed=99)
        xf = (x.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
        onehot = np.zeros((2, k), np.float32)
        onehot[0, 5] = 1.0
        onehot[1, k - 1] = -2.0
        xo = synth.f32_to_bf16_bits(onehot)
        xall = np.concatenate([x, xo], 0)
        xallf = (xall.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
        y = xallf @ deq.astype(np.float64).T
        out[f"{codec}_w"] = w
        out[f"{codec}_deq"] = deq
        out[f"{codec}_x"] = xall
        out[f"{codec}_y"] = y
        del xf
    np.savez_compressed(os.path.join(HERE, "golden_blocks.npz"), **out)
    print("wrote", os.path.join(HERE, "golden_blocks.npz"))


if __name__ == "__main__":
    main()
