"""GGUF wire-byte loader: the ``kq.load_gguf`` / ``load_gguf_wire_bytes`` step
of gmlx (gmlx/loader.py:92-145) that feeds the kernels.

A small reader of the GGUF v2/v3 container written from the format: a header
(magic ``GGUF``, version, tensor and key/value counts), the key/value
metadata, the tensor table (name, dims in GGUF order ``ne0, ne1, ...``, ggml
type, offset) and the tensor data after the table, aligned to
``general.alignment`` (default 32).  Tensors come back as memory-mapped views
(``zero_copy``) or copies, optionally moved to a device:

* quantized types: uint8 wire bytes ``[rows, row_bytes]`` plus the vestigial
  ``<prefix>.scales`` placeholder and the codec name (``"q4_k"``, ...);
* F32 / F16 / BF16 / I8 / I16 / I32 / I64 / F64: their native dtype, ``ne`` reversed.

Codecs without kernels here still load; the ops reject them by name.
"""
from __future__ import annotations

import os
import re
import struct

import numpy as np
import torch

# ggml type id -> (name, weights per block, bytes per block): the ggml format's
# type table (the same numbers as gguf-py's GGML_QUANT_SIZES)
GGML_TYPES = {
    0: ("f32", 1, 4), 1: ("f16", 1, 2), 2: ("q4_0", 32, 18), 3: ("q4_1", 32, 20), 6: ("q5_0", 32, 22),
    7: ("q5_1", 32, 24), 8: ("q8_0", 32, 34), 9: ("q8_1", 32, 40), 10: ("q2_k", 256, 84), 11: ("q3_k", 256, 110),
    12: ("q4_k", 256, 144), 13: ("q5_k", 256, 176), 14: ("q6_k", 256, 210), 15: ("q8_k", 256, 292),
    16: ("iq2_xxs", 256, 66), 17: ("iq2_xs", 256, 74), 18: ("iq3_xxs", 256, 98), 19: ("iq1_s", 256, 50),
    20: ("iq4_nl", 32, 18), 21: ("iq3_s", 256, 110), 22: ("iq2_s", 256, 82), 23: ("iq4_xs", 256, 136),
    24: ("i8", 1, 1), 25: ("i16", 1, 2), 26: ("i32", 1, 4), 27: ("i64", 1, 8), 28: ("f64", 1, 8),
    29: ("iq1_m", 256, 56), 30: ("bf16", 1, 2), 34: ("tq1_0", 256, 54), 35: ("tq2_0", 256, 66),
    39: ("mxfp4", 32, 17), 40: ("nvfp4", 64, 36),
}
_NATIVE = {0: np.float32, 1: np.float16, 24: np.int8, 25: np.int16, 26: np.int32, 27: np.int64, 28: np.float64,
           30: np.uint16}  # bf16 is read as uint16 bits, viewed as torch.bfloat16

# metadata value types: id -> struct format (scalars)
_SCALAR = {0: "B", 1: "b", 2: "H", 3: "h", 4: "I", 5: "i", 6: "f", 7: "?", 10: "Q", 11: "q", 12: "d"}
_STRING, _ARRAY = 8, 9


class _Cursor:
    def __init__(self, buf, off: int = 0):
        self.buf, self.off = buf, off

    def take(self, fmt: str):
        v = struct.unpack_from("<" + fmt, self.buf, self.off)
        self.off += struct.calcsize("<" + fmt)
        return v[0] if len(v) == 1 else v

    def string(self) -> str:
        n = self.take("Q")
        s = bytes(self.buf[self.off:self.off + n]).decode("utf-8", errors="replace")
        self.off += n
        return s

    def value(self, vtype: int):
        if vtype in _SCALAR:
            return self.take(_SCALAR[vtype])
        if vtype == _STRING:
            return self.string()
        if vtype == _ARRAY:
            etype, n = self.take("I"), self.take("Q")
            if etype in _SCALAR and etype != 7:
                arr = np.frombuffer(self.buf, dtype="<" + _SCALAR[etype], count=n, offset=self.off)
                self.off += arr.nbytes
                return arr.tolist()
            return [self.value(etype) for _ in range(n)]
        raise ValueError(f"GGUF: unknown metadata value type {vtype}")


def read_gguf(path: str):
    """Parse one GGUF file.  Returns ``(meta, infos, data_offset, mm)``: the
    key/value dict, a list of ``(name, ne, type_id, offset)``, the absolute
    offset of the data section and the read-only memory map."""
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    c = _Cursor(mm)
    if bytes(mm[:4]) != b"GGUF":
        raise ValueError(f"{path}: not a GGUF file")
    c.off = 4
    version = c.take("I")
    if version not in (2, 3):
        raise ValueError(f"{path}: GGUF version {version} not supported")
    n_tensors, n_kv = c.take("Q"), c.take("Q")
    meta = {}
    for _ in range(n_kv):
        key = c.string()
        meta[key] = c.value(c.take("I"))
    infos = []
    for _ in range(n_tensors):
        name = c.string()
        nd = c.take("I")
        ne = tuple(c.take("Q") for _ in range(nd))
        infos.append((name, ne, c.take("I"), c.take("Q")))
    align = int(meta.get("general.alignment", 32))
    data = (c.off + align - 1) // align * align
    return meta, infos, data, mm


def _tensor(mm, data: int, ne, tid: int, off: int, zero_copy: bool):
    if tid not in GGML_TYPES:
        raise ValueError(f"GGUF: unknown ggml type {tid}")
    name, bw, bb = GGML_TYPES[tid]
    rows = int(np.prod(ne[1:])) if len(ne) > 1 else 1
    if ne[0] % bw:
        raise ValueError(f"GGUF: row of {ne[0]} weights is not a whole number of {name} blocks")
    row_bytes = ne[0] // bw * bb
    start = data + off
    raw = mm[start:start + rows * row_bytes]
    if tid in _NATIVE:
        arr = raw.view(_NATIVE[tid]).reshape(tuple(reversed(ne)))
        t = _view(arr) if zero_copy else torch.from_numpy(np.array(arr))
        if tid == 30:
            t = t.view(torch.bfloat16)
        return t, None
    arr = raw.reshape(rows, row_bytes)
    return (_view(arr) if zero_copy else torch.from_numpy(np.array(arr))), name


def _view(arr):
    # a zero-copy tensor over the read-only mapping (never written through)
    import warnings
    with warnings.catch_warnings():
        warnings.simplefilter("ignore", UserWarning)
        return torch.from_numpy(arr)


def load_gguf(path: str, zero_copy: bool = True, device=None):
    """``kq.load_gguf(path, zero_copy)`` -> ``(arrays, codecs, meta, shapes)``:
    tensors by name, ``name -> codec`` for the quantized ones, the metadata
    dict and ``name -> GGUF-order shape``.  ``device``: copy every tensor there
    (weights stay in wire form)."""
    meta, infos, data, mm = read_gguf(path)
    arrays, codecs, shapes = {}, {}, {}
    for name, ne, tid, off in infos:
        t, codec = _tensor(mm, data, ne, tid, off, zero_copy)
        if device is not None:
            t = t.to(device)
        arrays[name] = t
        shapes[name] = tuple(int(v) for v in ne)
        if codec is not None:
            codecs[name] = codec
            prefix = name[:-len(".weight")] if name.endswith(".weight") else name
            arrays[prefix + ".scales"] = torch.zeros(1, dtype=torch.uint8, device=device)
    return arrays, codecs, meta, shapes


_SPLIT = re.compile(r"^(?P<base>.*)-(?P<i>\d{5})-of-(?P<n>\d{5})\.gguf$")


def find_split_shards(path: str) -> list[str]:
    """All shards of a split GGUF (``name-00001-of-00003.gguf``), else ``[path]``."""
    m = _SPLIT.match(path)
    if not m:
        return [path]
    n = int(m.group("n"))
    shards = [f"{m.group('base')}-{i:05d}-of-{n:05d}.gguf" for i in range(1, n + 1)]
    missing = [s for s in shards if not os.path.exists(s)]
    if missing:
        raise FileNotFoundError(f"missing GGUF shards: {missing}")
    return shards


def load_gguf_wire_bytes(gguf_path: str, zero_copy: bool = True, shards=None, device=None):
    """gmlx's ``load_gguf_wire_bytes`` (gmlx/loader.py:92-145): every shard
    merged; returns ``(arrays, kquant_meta, arch, meta, tensor_shapes)`` with
    metadata and shapes of the first shard as the reference does."""
    shards = shards or find_split_shards(gguf_path)
    arrays, codecs, meta, shapes = {}, {}, {}, {}
    for i, s in enumerate(shards):
        a, c, m, sh = load_gguf(s, zero_copy, device)
        arrays.update(a)
        codecs.update(c)
        shapes.update(sh)
        if i == 0:
            meta = m
    return arrays, codecs, meta.get("general.architecture"), meta, shapes


__all__ = ["GGML_TYPES", "read_gguf", "load_gguf", "find_split_shards", "load_gguf_wire_bytes"]
