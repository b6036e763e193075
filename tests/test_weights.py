"""The TMLLWGHT weight codec and config.json (src/model/weights.rs, weight_codec.rs,
config.rs) on the host: the reference's own round-trip tests, the byte layout, and every
rejection the reference's loader makes."""
from __future__ import annotations

import json
import struct

import numpy as np
import pytest

import rustllm_b200 as rb
from rustllm_b200 import _lib
from rustllm_b200.decoder import ModelConfig
from rustllm_b200.weights import ModelWeights, load_config_json, save_config_json


def test_saves_and_loads_a_weight_collection(tmp_path):
    """weights.rs:189-207."""
    w = ModelWeights()
    w.insert_f32("layer.weight", [2, 2], [1.0, 2.0, 3.0, 4.0])
    path = tmp_path / "w.bin"
    w.save(path)
    loaded = ModelWeights.load(path)
    assert loaded["layer.weight"].shape == (2, 2)
    assert loaded["layer.weight"].data.ravel().tolist() == [1.0, 2.0, 3.0, 4.0]


def test_file_bytes_follow_the_format(tmp_path):
    """The exact bytes weight_codec.rs:18-42 and :236-274 write for that collection."""
    w = ModelWeights()
    w.insert_f32("layer.weight", [2, 2], [1.0, 2.0, 3.0, 4.0])
    path = tmp_path / "w.bin"
    w.save(path)
    want = (b"TMLLWGHT" + struct.pack("<II", 1, 1) + struct.pack("<I", 12) + b"layer.weight"
            + bytes([1]) + struct.pack("<I", 2) + struct.pack("<QQ", 2, 2)
            + struct.pack("<Q", 4) + struct.pack("<4f", 1.0, 2.0, 3.0, 4.0))
    assert path.read_bytes() == want


def test_saves_and_loads_f16_weight_collection(tmp_path):
    """weights.rs:209-232: save_as(F16) converts F32 sources."""
    w = ModelWeights()
    w.insert_f32("layer.weight", [2, 2], [1.0, -2.0, 0.5, 3.25])
    path = tmp_path / "w16.bin"
    w.save(path, dtype="f16")
    loaded = ModelWeights.load(path)
    t = loaded["layer.weight"]
    assert t.data.dtype == np.float16 and t.shape == (2, 2)
    assert t.data.astype(np.float32).ravel().tolist() == [1.0, -2.0, 0.5, 3.25]


def test_saves_and_loads_mixed_dtype_weights(tmp_path):
    """weights.rs:235-290."""
    w = ModelWeights()
    w.insert_f16("embedding.weight", [2], [1.0, 2.0])
    w.insert_i8("linear.weight", [2, 2], [127, -127, 64, -64])
    w.insert_f32("linear.scale", [2], [0.01, 0.02])
    path = tmp_path / "mixed.bin"
    w.save(path)
    loaded = ModelWeights.load(path)
    assert loaded["embedding.weight"].data.dtype == np.float16
    assert loaded["linear.weight"].data.dtype == np.int8
    assert loaded["linear.weight"].data.ravel().tolist() == [127, -127, 64, -64]
    assert loaded["linear.scale"].data.dtype == np.float32


def test_insert_checks():
    """weights.rs:82-181: empty names or shapes, zero dims, count mismatches, duplicates."""
    w = ModelWeights()
    with pytest.raises(rb.ModelFormat):
        w.insert_f32("", [1], [0.0])
    with pytest.raises(rb.ModelFormat):
        w.insert_f32("a", [2, 0], [])
    with pytest.raises(rb.ModelFormat, match="has 3 values"):
        w.insert_f32("a", [2, 2], [1.0, 2.0, 3.0])
    w.insert_f32("a", [1], [1.0])
    with pytest.raises(rb.ModelFormat, match="duplicate weight: a"):
        w.insert_f16("a", [1], [1.0])
    with pytest.raises(_lib.MissingWeight, match="missing model weight: b"):
        w.take("b")


def _header(count=1):
    return b"TMLLWGHT" + struct.pack("<II", 1, count)


def _tensor(name=b"w", tag=1, dims=(2,), count=None, data=None):
    count = int(np.prod(dims)) if count is None else count
    data = b"\0" * (count * {1: 4, 2: 2, 3: 1}.get(tag, 4)) if data is None else data
    return (struct.pack("<I", len(name)) + name + bytes([tag]) + struct.pack("<I", len(dims))
            + struct.pack(f"<{len(dims)}Q", *dims) + struct.pack("<Q", count) + data)


@pytest.mark.parametrize("blob,kind,msg", [
    (b"NOTMAGIC" + struct.pack("<II", 1, 0), rb.ModelFormat, "invalid model weight magic"),
    (b"TMLLWGHT" + struct.pack("<II", 2, 0), rb.ModelFormat, "unsupported weight format version"),
    (_header() + struct.pack("<I", 0), rb.ModelFormat, "invalid weight name length 0"),
    (_header() + struct.pack("<I", 1025), rb.ModelFormat, "invalid weight name length 1025"),
    (_header() + _tensor(name=b"\xff"), rb.ModelFormat, "invalid UTF-8 weight name"),
    (_header() + _tensor(tag=4), rb.ModelFormat, "unsupported dtype 4 for weight w"),
    (_header() + _tensor(dims=()), rb.ModelFormat, "invalid rank 0 for weight w"),
    (_header() + _tensor(dims=(1,) * 17), rb.ModelFormat, "invalid rank 17 for weight w"),
    (_header() + _tensor(dims=(2, 0), count=0), rb.ModelFormat, "zero-sized dimension"),
    (_header() + _tensor(dims=(2, 3), count=5, data=b"\0" * 20), rb.ModelFormat,
     "declares an invalid element count"),
    (_header() + _tensor(dims=(4,), data=b"\0" * 10), _lib.IoError, "I/O error"),
    (_header(2) + _tensor(), _lib.IoError, "I/O error"),
])
def test_load_rejects_malformed_files(tmp_path, blob, kind, msg):
    """weight_codec.rs:100-230: each check, with its error kind and message."""
    path = tmp_path / "bad.bin"
    path.write_bytes(blob)
    with pytest.raises(kind, match=msg):
        ModelWeights.load(path)


def test_repeated_name_replaces_earlier_tensor(tmp_path):
    """weight_codec.rs:225-227 inserts into a map: the last tensor of a name wins."""
    path = tmp_path / "dup.bin"
    path.write_bytes(_header(2) + _tensor(data=struct.pack("<2f", 1, 2))
                     + _tensor(data=struct.pack("<2f", 3, 4)))
    assert ModelWeights.load(path)["w"].data.tolist() == [3.0, 4.0]


def test_config_json_round_trip_and_checks(tmp_path):
    """config.rs: load_json / save_json and the GQA validation tests (:160-189)."""
    cfg = ModelConfig(100, 576, 1536, 4, 9, 3, 1024, 1e-5, 10000.0)
    path = tmp_path / "config.json"
    save_config_json(cfg, path)
    assert load_config_json(path) == cfg
    assert cfg.head_dim == 64
    bad = json.loads(path.read_text())
    bad.update(num_heads=10, hidden_size=640)
    path.write_text(json.dumps(bad))
    with pytest.raises(rb.ModelFormat, match="num_heads 10 must be divisible by num_kv_heads 3"):
        load_config_json(path)
    del bad["rope_theta"]
    path.write_text(json.dumps(bad))
    with pytest.raises(rb.ModelFormat, match="invalid config.json"):
        load_config_json(path)
    with pytest.raises(_lib.IoError):
        load_config_json(tmp_path / "missing.json")
