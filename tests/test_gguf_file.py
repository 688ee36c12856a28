"""The GGUF reader (mote_b200/gguf_file.py) against files the gguf package
(llama.cpp project, 0.19.0) writes: metadata of every value type, tensors of
the encodings the data plane runs (F32, F16, Q4_0, Q8_0, Q4_K, Q6_K) and one
it does not (Q5_K), a custom alignment, and malformed files."""
from __future__ import annotations

import struct

import numpy as np
import pytest

gguf = pytest.importorskip("gguf")
from gguf import GGMLQuantizationType as T  # noqa: E402

from mote_b200.gguf_file import GGUFError, GGUFFile  # noqa: E402
from mote_b200.types import DType, QuantFormat  # noqa: E402

BLOCK = {T.Q4_0: (32, 18), T.Q8_0: (32, 34), T.Q4_K: (256, 144), T.Q6_K: (256, 210),
         T.Q5_K: (256, 176)}


def raw_blocks(rng, qtype, n, k):
    be, bb = BLOCK[qtype]
    return rng.integers(0, 256, (n, k // be * bb), dtype=np.uint8)


@pytest.fixture
def written(tmp_path):
    rng = np.random.default_rng(1)
    path = tmp_path / "model.gguf"
    w = gguf.GGUFWriter(str(path), "llama")
    w.add_uint32("llama.block_count", 16)
    w.add_float32("llama.attention.layer_norm_rms_epsilon", 1e-5)
    w.add_string("general.name", "tiny")
    w.add_bool("general.flag", True)
    w.add_array("tokenizer.ggml.scores", [0.5, -1.25, 3.0])
    w.add_array("tokenizer.ggml.tokens", ["<s>", "a", "bc"])
    w.add_uint64("general.size", 1 << 40)
    w.add_int32("general.neg", -7)
    tensors = {
        "norm.weight": (rng.normal(0, 1, 2048).astype(np.float32), None),
        "emb.weight": (rng.normal(0, 1, (8, 64)).astype(np.float16), None),
        "q40.weight": (raw_blocks(rng, T.Q4_0, 48, 512), T.Q4_0),
        "q80.weight": (raw_blocks(rng, T.Q8_0, 16, 256), T.Q8_0),
        "q4k.weight": (raw_blocks(rng, T.Q4_K, 40, 1024), T.Q4_K),
        "q6k.weight": (raw_blocks(rng, T.Q6_K, 24, 512), T.Q6_K),
        "q5k.weight": (raw_blocks(rng, T.Q5_K, 4, 256), T.Q5_K),
    }
    for name, (arr, qt) in tensors.items():
        w.add_tensor(name, arr, raw_dtype=qt)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return path, tensors


def test_metadata_round_trip(written):
    path, _ = written
    with GGUFFile(path) as f:
        md = f.metadata
        assert f.version == 3
        assert md["general.architecture"] == "llama"
        assert md["llama.block_count"] == 16
        assert md["llama.attention.layer_norm_rms_epsilon"] == pytest.approx(1e-5)
        assert md["general.name"] == "tiny"
        assert md["general.flag"] is True
        assert md["tokenizer.ggml.scores"] == [0.5, -1.25, 3.0]
        assert md["tokenizer.ggml.tokens"] == ["<s>", "a", "bc"]
        assert md["general.size"] == 1 << 40
        assert md["general.neg"] == -7


def test_tensors_shapes_types_and_bytes(written):
    path, tensors = written
    k_of = {"q40.weight": 512, "q80.weight": 256, "q4k.weight": 1024, "q6k.weight": 512,
            "q5k.weight": 256}
    with GGUFFile(path) as f:
        assert list(f.tensors) == list(tensors)
        for name, (arr, qt) in tensors.items():
            info = f.tensors[name]
            assert info.offset % f.alignment == 0
            want_shape = arr.shape if qt is None else (arr.shape[0], k_of[name])
            assert info.shape == want_shape, name
            got = f.tensor_bytes(name)
            assert got.tobytes() == np.ascontiguousarray(arr).tobytes(), name
        assert f.descriptor("norm.weight").shape == (2048,)
        assert f.descriptor("emb.weight").encoding.plain is DType.F16
        assert f.descriptor("q4k.weight").encoding.quantized is QuantFormat.Q4_K
        assert f.descriptor("q4k.weight").required_span_bytes == 40 * 4 * 144
        assert f.descriptor("q6k.weight").encoding.quantized is QuantFormat.Q6_K
        assert f.descriptor("q40.weight").encoding.quantized is QuantFormat.Q4_0
        assert f.descriptor("q80.weight").encoding.quantized is QuantFormat.Q8_0
        with pytest.raises(GGUFError, match="no encoding"):
            f.descriptor("q5k.weight")
        with pytest.raises(GGUFError, match="no tensor"):
            f.descriptor("missing")


def test_custom_alignment(tmp_path):
    path = tmp_path / "aligned.gguf"
    w = gguf.GGUFWriter(str(path), "llama")
    w.add_custom_alignment(64)
    a = np.arange(33, dtype=np.float32)
    b = np.arange(7, dtype=np.float16)
    w.add_tensor("a", a)
    w.add_tensor("b", b)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    with GGUFFile(path) as f:
        assert f.alignment == 64
        assert f.data_offset % 64 == 0
        assert all(t.offset % 64 == 0 for t in f.tensors.values())
        assert np.array_equal(f.tensor_bytes("a").view(np.float32), a)
        assert np.array_equal(f.tensor_bytes("b").view(np.float16), b)


def test_malformed_files(tmp_path, written):
    path, _ = written
    data = path.read_bytes()
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGML" + data[4:])
    with pytest.raises(GGUFError, match="magic"):
        GGUFFile(bad)
    bad.write_bytes(data[:4] + struct.pack("<I", 9) + data[8:])
    with pytest.raises(GGUFError, match="version"):
        GGUFFile(bad)
    bad.write_bytes(data[:200])
    with pytest.raises(GGUFError):
        GGUFFile(bad)
    bad.write_bytes(data[:-64])  # the last tensor's data cut short
    with pytest.raises(GGUFError, match="past the end"):
        GGUFFile(bad)
    bad.write_bytes(b"GGUF")
    with pytest.raises(GGUFError, match="too short"):
        GGUFFile(bad)
