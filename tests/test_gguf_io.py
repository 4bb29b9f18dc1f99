"""GGUF wire-byte loader (gmlx_b200.gguf_io) against gguf-py: files written
with gguf-py's GGUFWriter, read back with our reader and with GGUFReader."""
import numpy as np
import pytest
import torch

gguf = pytest.importorskip("gguf")
from gguf import GGMLQuantizationType as Q  # noqa: E402

from gmlx_b200 import gguf_io, synth  # noqa: E402


def _write(path, tensors, kv=()):
    w = gguf.GGUFWriter(str(path), "llama")
    for k, v in kv:
        if isinstance(v, str):
            w.add_string(k, v)
        elif isinstance(v, list):
            w.add_array(k, v)
        else:
            w.add_uint32(k, v)
    for name, arr, qt in tensors:
        if qt is None:
            w.add_tensor(name, arr)
        else:
            w.add_tensor(name, arr, raw_dtype=qt)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


def _case():
    q4 = synth.random_weight("q4_k", 24, 512, seed=1)
    q6 = synth.random_weight("q6_k", 5, 768, seed=2)     # 630-byte rows: unaligned tensor data
    iq2 = synth.random_weight("iq2_xxs", 7, 1792, seed=3)
    f32 = np.random.default_rng(4).standard_normal((3, 64)).astype(np.float32)
    f16 = np.random.default_rng(5).standard_normal(40).astype(np.float16)
    i32 = np.arange(12, dtype=np.int32).reshape(3, 4)
    return [("blk.0.ffn_up.weight", q4, Q.Q4_K), ("blk.0.ffn_down.weight", q6, Q.Q6_K),
            ("blk.0.exp.weight", iq2, Q.IQ2_XXS), ("token_embd_norm.weight", f32, None),
            ("rope.freqs", f16, None), ("blk.0.ids", i32, None)]


def test_type_table_matches_ggml():
    for tid, (name, bw, bb) in gguf_io.GGML_TYPES.items():
        qt = Q(tid)
        assert qt.name.lower() == name
        assert gguf.GGML_QUANT_SIZES[qt] == (bw, bb)


@pytest.mark.parametrize("zero_copy", [True, False])
def test_load_gguf_matches_writer_and_reader(tmp_path, zero_copy):
    path = tmp_path / "m.gguf"
    tensors = _case()
    _write(path, tensors, kv=[("llama.block_count", 1), ("general.name", "tiny"), ("tok.list", [3, 1, 4])])
    arrays, codecs, meta, shapes = gguf_io.load_gguf(str(path), zero_copy=zero_copy)
    ref = {t.name: t for t in gguf.GGUFReader(str(path)).tensors}
    for name, arr, qt in tensors:
        got = arrays[name].numpy()
        assert np.array_equal(got.reshape(arr.shape), arr)
        assert np.array_equal(got.reshape(-1).view(np.uint8), np.asarray(ref[name].data).reshape(-1).view(np.uint8))
        assert shapes[name] == tuple(int(v) for v in ref[name].shape)
        if qt is not None:
            assert codecs[name] == qt.name.lower()
            assert arrays[name].dtype == torch.uint8 and arrays[name].shape == arr.shape
            assert arrays[name[:-len(".weight")] + ".scales"].shape == (1,)
        else:
            assert name not in codecs
    assert meta["general.architecture"] == "llama" and meta["llama.block_count"] == 1
    assert meta["general.name"] == "tiny" and meta["tok.list"] == [3, 1, 4]


def test_split_shards(tmp_path):
    tensors = _case()
    a = tmp_path / "m-00001-of-00002.gguf"
    b = tmp_path / "m-00002-of-00002.gguf"
    _write(a, tensors[:3], kv=[("general.name", "first")])
    _write(b, tensors[3:], kv=[("general.name", "second")])
    assert gguf_io.find_split_shards(str(a)) == [str(a), str(b)]
    arrays, codecs, arch, meta, shapes = gguf_io.load_gguf_wire_bytes(str(a))
    assert arch == "llama" and meta["general.name"] == "first"
    assert set(codecs) == {n for n, _, q in tensors if q is not None}
    assert all(n in arrays for n, _, _ in tensors)


def test_not_gguf(tmp_path):
    p = tmp_path / "x.gguf"
    p.write_bytes(b"NOTGGUF" + b"\0" * 64)
    with pytest.raises(ValueError):
        gguf_io.load_gguf(str(p))


def test_every_kernel_codec_survives_a_gguf_file(tmp_path):
    """Each codec with kernels here, written by gguf-py into one GGUF file, comes
    back from our loader under the codec name the ops take, with the wire row
    length the ops expect (the 32-weight ggml codecs: whole 256-weight groups)
    and bytes that dequantize (oracle) exactly as gguf-py's own dequantizer."""
    from gguf import quants as gq
    from oracle import oracle as O
    tensors = []
    for i, name in enumerate(sorted(synth.CODECS)):
        w = synth.random_weight(name, 3, 512, seed=40 + i)
        tensors.append((f"t.{name}.weight", w, Q[name.upper()]))
    path = tmp_path / "codecs.gguf"
    _write(path, tensors)
    arrays, codecs, _, _ = gguf_io.load_gguf(str(path), zero_copy=False)
    for name, w, qt in tensors:
        codec = codecs[name]
        assert synth.codec_id(codec) == synth.CODECS[codec]
        got = arrays[name].numpy()
        assert got.shape == (3, synth.row_bytes(codec, 512)) and np.array_equal(got, w)
        ref = gq.dequantize(got, qt).astype(np.float32)
        assert np.array_equal(O.dequantize(got, codec).view(np.uint32), ref.view(np.uint32))
