"""GGUF files (pkg/gguf/reader.go, format.go) through the library's host
parser, against files built by an independent writer (tests/gguf_writer.py).

The reference ships no GGUF fixtures and its tests do not cover the reader,
so the cases follow reader.go's behaviour: header checks (magic, version 2
or 3, minimum size), all thirteen metadata value types with arrays, Go's
type-asserting getters, tensor infos in GGUF dimension order with Shape()
reversed, SizeBytes over whole blocks, the data section aligned to
`general.alignment` only when that key is a uint32, later duplicates winning
lookups, and GetTensorData refusing data past the end of the file.  Beyond
the reference, every truncation of a file and random corruption of its
header must end in an error, never a crash."""
import struct

import numpy as np
import pytest

from gollama_b200 import gguf
from gollama_b200.device import GlcError
from tests import gguf_writer as W

GLC_ERR_IO = -7


def sample(alignment=32, version=3, align_key_type=None):
    rng = np.random.default_rng(0)
    meta = [
        ("general.architecture", W.STRING, "llama"),
        ("general.name", W.STRING, "tiny test model"),
        ("llama.context_length", W.U32, 2048),
        ("llama.embedding_length", W.U32, 64),
        ("llama.attention.head_count_kv", W.I32, -3),
        ("llama.rope.freq_base", W.F32, 10000.0),
        ("llama.attention.layer_norm_rms_epsilon", W.F32, 1e-5),
        ("u8", W.U8, 200), ("i8", W.I8, -100), ("u16", W.U16, 65000), ("i16", W.I16, -30000),
        ("u64", W.U64, 2**63 + 5), ("i64", W.I64, -(2**62)), ("f64", W.F64, 3.141592653589793), ("flag", W.BOOL, True),
        ("tokenizer.ggml.tokens", W.ARRAY, ["<s>", "</s>", "héllo", ""], W.STRING),
        ("tokenizer.ggml.scores", W.ARRAY, [0.0, -1.5, 2.25], W.F32),
        ("tokenizer.ggml.token_type", W.ARRAY, [1, 2, 3, -4], W.I32),
        ("nested", W.ARRAY, [(W.U8, [1, 2]), (W.STRING, ["a"])], W.ARRAY),
        ("empty", W.ARRAY, [], W.U64),
    ]
    if align_key_type is not None:
        meta.append(("general.alignment", align_key_type, alignment))
    tensors = [
        ("token_embd.weight", [64, 10], 0, rng.standard_normal(640).astype(np.float32).tobytes()),
        ("blk.0.attn_q.weight", [64, 64], 1, rng.standard_normal(4096).astype(np.float16).tobytes()),
        ("blk.0.ffn_down.weight", [64, 3], 8, rng.integers(0, 256, 3 * 2 * 34, dtype=np.uint8).tobytes()),
        ("blk.0.ffn_gate.weight", [256, 2], 12, rng.integers(0, 256, 2 * 144, dtype=np.uint8).tobytes()),
        ("blk.0.ffn_up.weight", [256, 1], 14, rng.integers(0, 256, 210, dtype=np.uint8).tobytes()),
        ("output_norm.weight", [64], 0, np.ones(64, np.float32).tobytes()),
        ("odd.weight", [33], 2, rng.integers(0, 256, 2 * 18, dtype=np.uint8).tobytes()),  # 2 blocks: 33 rounds up
    ]
    data_align = alignment if align_key_type == W.U32 else 32
    blob, data_off, offsets = W.gguf_bytes(meta, tensors, version=version, alignment=data_align)
    return blob, data_off, meta, tensors


def write(tmp_path, blob, name="m.gguf"):
    p = tmp_path / name
    p.write_bytes(blob)
    return p


def test_header_metadata_and_tensors(tmp_path):
    blob, data_off, meta, tensors = sample()
    with gguf.Open(write(tmp_path, blob)) as r:
        h = r.Header()
        assert (h.Magic, h.Version, h.TensorCount, h.MetadataKVCount) == (0x46554747, 3, len(tensors), len(meta))
        assert r.data_offset == data_off and data_off % 32 == 0
        assert r.Architecture() == "llama"
        md = r.Metadata()
        assert md["llama.context_length"] == 2048 and isinstance(md["llama.context_length"], np.uint32)
        assert md["u8"] == 200 and md["i8"] == -100 and md["u16"] == 65000 and md["i16"] == -30000
        assert md["u64"] == 2**63 + 5 and md["i64"] == -(2**62) and md["f64"] == 3.141592653589793
        assert md["flag"] is True
        assert md["llama.rope.freq_base"] == np.float32(10000.0)
        assert md["llama.attention.layer_norm_rms_epsilon"] == np.float32(1e-5)
        assert md["nested"] == [None, None] and md["empty"] == []
        # Go's type assertions: the getter of another type reports ok = false
        assert r.GetUint32("llama.context_length") == (2048, True)
        assert r.GetUint32("llama.attention.head_count_kv") == (0, False)
        assert r.GetInt32("llama.attention.head_count_kv") == (-3, True)
        assert r.GetUint64("llama.context_length") == (0, False)
        assert r.GetFloat32("llama.rope.freq_base") == (np.float32(10000.0), True)
        assert r.GetString("general.name") == ("tiny test model", True)
        assert r.GetString("missing") == ("", False)
        assert r.GetStringArray("tokenizer.ggml.tokens") == (["<s>", "</s>", "héllo", ""], True)
        assert r.GetFloat32Array("tokenizer.ggml.scores") == ([0.0, -1.5, 2.25], True)
        assert r.GetInt32Array("tokenizer.ggml.token_type") == ([1, 2, 3, -4], True)
        assert r.GetInt32Array("tokenizer.ggml.scores") == (None, False)
        assert r.GetMetadata("u8") == (200, True) and r.GetMetadata("nope") == (None, False)
        got = r.Tensors()
        assert [t.Name for t in got] == [t[0] for t in tensors]
        for t, (name, dims, gt, data) in zip(got, tensors):
            assert (t.NDims, t.Dimensions, t.Type) == (len(dims), dims, gt)
            assert t.Shape() == list(reversed(dims))
            assert t.SizeBytes() == len(data)
            assert r.GetTensorData(name) == data
        info, ok = r.GetTensorInfo("blk.0.ffn_gate.weight")
        assert ok and info.TypeName() == "Q4_K" and info.NumElements() == 512 and info.Shape() == [2, 256]
        assert r.GetTensorInfo("nope") == (None, False)
        with pytest.raises(KeyError):
            r.GetTensorData("nope")


@pytest.mark.parametrize("align,key_type,expect", [(64, W.U32, 64), (256, W.U32, 256), (64, W.U64, 32)])
def test_data_alignment(tmp_path, align, key_type, expect):
    """general.alignment counts only as a uint32 (reader.go:112-117)."""
    blob, data_off, _, tensors = sample(alignment=align, align_key_type=key_type)
    with gguf.Open(write(tmp_path, blob)) as r:
        assert r.data_offset == data_off and data_off % expect == 0
        for name, _, _, data in tensors:
            assert r.GetTensorData(name) == data


def test_version_2_and_refusals(tmp_path):
    blob, *_ = sample(version=2)
    with gguf.Open(write(tmp_path, blob)) as r:
        assert r.Header().Version == 2
    for v in (1, 4):
        b, *_ = sample(version=v)
        with pytest.raises(GlcError) as e:
            gguf.Open(write(tmp_path, b))
        assert e.value.code == GLC_ERR_IO and "version" in str(e.value)
    bad = b"GGUG" + blob[4:]
    with pytest.raises(GlcError) as e:
        gguf.Open(write(tmp_path, bad))
    assert "magic" in str(e.value)
    with pytest.raises(GlcError) as e:
        gguf.Open(write(tmp_path, blob[:23]))
    assert "too small" in str(e.value)
    with pytest.raises(GlcError) as e:
        gguf.Open(tmp_path / "missing.gguf")
    assert e.value.code == GLC_ERR_IO


def test_unknown_value_type_and_huge_counts(tmp_path):
    base = struct.pack("<IIQQ", 0x46554747, 3, 0, 1) + W.enc_string("k")
    with pytest.raises(GlcError) as e:
        gguf.Open(write(tmp_path, base + struct.pack("<I", 13) + b"\0" * 16))
    assert "unknown metadata value type" in str(e.value)
    # an array claiming 2^60 elements, a string claiming 2^62 bytes, 2^40 keys
    for tail in (struct.pack("<IIQ", W.ARRAY, W.U32, 2**60), struct.pack("<IQ", W.STRING, 2**62)):
        with pytest.raises(GlcError) as e:
            gguf.Open(write(tmp_path, base + tail + b"\0" * 8))
        assert e.value.code == GLC_ERR_IO
    with pytest.raises(GlcError):
        gguf.Open(write(tmp_path, struct.pack("<IIQQ", 0x46554747, 3, 0, 2**40) + b"\0" * 64))


def test_overflowing_dimensions_are_refused(tmp_path):
    blob, *_ = W.gguf_bytes([], [], extra_tensor_infos=[("huge", [2**40, 2**40], 0, 0)])
    with pytest.raises(GlcError) as e:
        gguf.Open(write(tmp_path, blob))
    assert e.value.code == GLC_ERR_IO and "overflow" in str(e.value)


def test_duplicates_and_data_past_the_end(tmp_path):
    meta = [("x", W.U32, 1), ("x", W.U32, 2)]
    t1 = ("w", [4], 0, np.arange(4, dtype=np.float32).tobytes())
    t2 = ("w", [8], 0, np.arange(8, dtype=np.float32).tobytes())
    blob, *_ = W.gguf_bytes(meta, [t1, t2], extra_tensor_infos=[("far", [1024], 0, 4096)])
    with gguf.Open(write(tmp_path, blob)) as r:
        assert r.GetUint32("x") == (2, True)  # a later key replaces the earlier (Go map)
        assert r.GetTensorInfo("w")[0].Dimensions == [8]
        assert r.GetTensorData("w") == t2[3]
        with pytest.raises(GlcError) as e:
            r.GetTensorData("far")
        assert e.value.code == GLC_ERR_IO and "beyond" in str(e.value)


def test_every_truncation_fails_cleanly(tmp_path):
    blob, data_off, meta, tensors = sample()
    path = tmp_path / "t.gguf"
    for cut in range(0, data_off + 1):
        path.write_bytes(blob[:cut])
        try:
            r = gguf.Open(path)
        except GlcError as e:
            assert e.code == GLC_ERR_IO
            continue
        # parsed (the cut fell in the padding before the data): every tensor's data is past the end
        with r:
            for name, _, _, data in tensors:
                with pytest.raises(GlcError):
                    r.GetTensorData(name)


def test_random_header_corruption_never_crashes(tmp_path):
    blob, data_off, *_ = sample()
    rng = np.random.default_rng(7)
    path = tmp_path / "c.gguf"
    for _ in range(400):
        b = bytearray(blob)
        for _ in range(int(rng.integers(1, 6))):
            b[int(rng.integers(0, data_off))] = int(rng.integers(0, 256))
        path.write_bytes(bytes(b))
        try:
            with gguf.Open(path) as r:
                for t in r.Tensors():
                    try:
                        r.GetTensorData(t.Name)
                    except GlcError:
                        pass
        except GlcError as e:
            assert e.code in (GLC_ERR_IO, -1)
