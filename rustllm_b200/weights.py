"""The reference's model files: `model.bin` in the TMLLWGHT format and `config.json`.

Restates src/model/weights.rs and src/model/weight_codec.rs (the little-endian binary
codec, its validation and its error kinds) and src/model/config.rs (the JSON config), and
maps a loaded weight collection onto this package's decoder (src/model/transformer.rs:
203-318 names and shapes).  Host-side file IO; nothing here touches the GPU except the
final copy of the decoder's weights to the device.

File layout (all integers little-endian):

    b"TMLLWGHT"  u32 version (1)  u32 tensor count
    per tensor, in name order:
        u32 name length (1..1024)  name (UTF-8)  u8 dtype (1 F32, 2 F16, 3 I8)
        u32 rank (1..16)  rank x u64 dims (non-zero)  u64 element count (= product)
        element count x element size bytes
"""
from __future__ import annotations

import json
import os
import struct
from dataclasses import dataclass

import numpy as np

from . import _lib

MAGIC = b"TMLLWGHT"          # weights.rs:7
VERSION = 1                  # weights.rs:8
DTYPE_F32, DTYPE_F16, DTYPE_I8 = 1, 2, 3  # weights.rs:9-11
MAX_RANK = 16                # weights.rs:12
MAX_NAME_LEN = 1024          # weights.rs:13
_NP = {DTYPE_F32: np.dtype("<f4"), DTYPE_F16: np.dtype("<f2"), DTYPE_I8: np.dtype("i1")}


@dataclass
class WeightTensor:
    """One named tensor of a weight file: shape and host data (float32, float16 or int8)."""

    shape: tuple
    data: np.ndarray

    @property
    def dtype_tag(self) -> int:
        return {np.dtype("float32"): DTYPE_F32, np.dtype("float16"): DTYPE_F16,
                np.dtype("int8"): DTYPE_I8}[self.data.dtype]


def _numel(shape) -> int:
    n = 1
    for d in shape:
        n *= int(d)
    return n


class ModelWeights(dict):
    """src/model/weights.rs:52-182: name -> WeightTensor, with the reference's insert
    checks (non-empty name, non-empty shape without zeros, matching element count, no
    duplicates)."""

    def _insert(self, name: str, shape, data: np.ndarray, what: str) -> None:
        shape = tuple(int(d) for d in shape)
        if not name or not shape or 0 in shape:
            raise _lib.ModelFormat(f"invalid shape or name for {what}weight {name}")
        if data.size != _numel(shape):
            raise _lib.ModelFormat(f"weight {name} has {data.size} values, but shape "
                                   f"{list(shape)} requires {_numel(shape)}")
        if name in self:
            raise _lib.ModelFormat(f"duplicate weight: {name}")
        self[name] = WeightTensor(shape, np.ascontiguousarray(data).reshape(shape))

    def insert_f32(self, name: str, shape, data) -> None:
        self._insert(name, shape, np.asarray(data, np.float32).ravel(), "")

    def insert_f16(self, name: str, shape, data) -> None:
        self._insert(name, shape, np.asarray(data, np.float16).ravel(), "F16 ")

    def insert_i8(self, name: str, shape, data) -> None:
        self._insert(name, shape, np.asarray(data, np.int8).ravel(), "INT8 ")

    def take(self, name: str) -> WeightTensor:
        if name not in self:
            raise _lib.MissingWeight(f"missing model weight: {name}")
        return self.pop(name)

    def save(self, path, dtype: str | None = None) -> None:
        """weight_codec.rs:18-99: `save` keeps each tensor's dtype; `save_as` (dtype "f32"
        or "f16") converts F32 sources and keeps INT8 as it is."""
        with open(path, "wb") as f:
            f.write(MAGIC)
            f.write(struct.pack("<II", VERSION, len(self)))
            for name in sorted(self):
                t = self[name]
                data = t.data
                if dtype is not None and data.dtype != np.int8:
                    if data.dtype != np.float32:
                        raise _lib.ModelFormat(f"cannot save non-F32 source weight {name}")
                    data = data.astype(np.float16 if dtype == "f16" else np.float32)
                tag = WeightTensor(t.shape, data).dtype_tag
                b = name.encode()
                f.write(struct.pack("<I", len(b)))
                f.write(b)
                f.write(struct.pack("<BI", tag, len(t.shape)))
                f.write(struct.pack(f"<{len(t.shape)}Q", *t.shape))
                f.write(struct.pack("<Q", _numel(t.shape)))
                f.write(np.ascontiguousarray(data, _NP[tag]).tobytes())

    @classmethod
    def load(cls, path) -> "ModelWeights":
        """weight_codec.rs:100-230, with its checks and messages.  A file that ends early
        raises IoError (the reference's read_exact failure)."""
        try:
            with open(path, "rb") as f:
                buf = f.read()
        except OSError as e:
            raise _lib.IoError(f"I/O error: {e}") from e
        pos = 0

        def take(n: int) -> bytes:
            nonlocal pos
            if pos + n > len(buf):
                raise _lib.IoError("I/O error: failed to fill whole buffer")
            out = buf[pos:pos + n]
            pos += n
            return out

        def u32() -> int:
            return struct.unpack("<I", take(4))[0]

        def u64() -> int:
            return struct.unpack("<Q", take(8))[0]

        if take(8) != MAGIC:
            raise _lib.ModelFormat("invalid model weight magic")
        if u32() != VERSION:
            raise _lib.ModelFormat("unsupported weight format version")
        weights = cls()
        for _ in range(u32()):
            n = u32()
            if n == 0 or n > MAX_NAME_LEN:
                raise _lib.ModelFormat(f"invalid weight name length {n}")
            try:
                name = take(n).decode("utf-8")
            except UnicodeDecodeError as e:
                raise _lib.ModelFormat(f"invalid UTF-8 weight name: {e}") from e
            tag = take(1)[0]
            if tag not in _NP:
                raise _lib.ModelFormat(f"unsupported dtype {tag} for weight {name}")
            rank = u32()
            if rank == 0 or rank > MAX_RANK:
                raise _lib.ModelFormat(f"invalid rank {rank} for weight {name}")
            shape = []
            for _ in range(rank):
                d = u64()
                if d == 0:
                    raise _lib.ModelFormat(f"weight {name} has a zero-sized dimension")
                shape.append(d)
            count = u64()
            if count != _numel(shape):
                raise _lib.ModelFormat(f"weight {name} declares an invalid element count")
            raw = take(count * _NP[tag].itemsize)
            data = np.frombuffer(raw, dtype=_NP[tag]).astype(_NP[tag].newbyteorder("="))
            # a repeated name replaces the earlier tensor (weight_codec.rs:225-227)
            weights[name] = WeightTensor(tuple(shape), data.reshape(shape))
        return weights


def load_config_json(path):
    """ModelConfig::load_json (src/model/config.rs:123-131): the nine fields, validated."""
    from .decoder import ModelConfig
    try:
        with open(path) as f:
            text = f.read()
    except OSError as e:
        raise _lib.IoError(f"I/O error: {e}") from e
    keys = ("vocab_size", "hidden_size", "intermediate_size", "num_layers", "num_heads",
            "num_kv_heads", "max_seq_len", "rms_norm_eps", "rope_theta")
    try:
        raw = json.loads(text)
        ints = {k: raw[k] for k in keys[:7]}
        if any(not isinstance(v, int) or isinstance(v, bool) or v < 0 for v in ints.values()):
            raise ValueError("integer fields must be non-negative integers")
        cfg = ModelConfig(**ints, rms_norm_eps=float(raw["rms_norm_eps"]),
                          rope_theta=float(raw["rope_theta"]))
    except (ValueError, KeyError, TypeError) as e:
        raise _lib.ModelFormat(f"invalid config.json: {e}") from e
    cfg.validate()
    return cfg


def save_config_json(cfg, path) -> None:
    """ModelConfig::save_json (src/model/config.rs:133-143)."""
    cfg.validate()
    with open(path, "w") as f:
        json.dump({k: getattr(cfg, k) for k in (
            "vocab_size", "hidden_size", "intermediate_size", "num_layers", "num_heads",
            "num_kv_heads", "max_seq_len", "rms_norm_eps", "rope_theta")}, f, indent=2)


def load_model_dir(model_dir, *, device=None, dtype=None):
    """Transformer::load (src/model/transformer.rs:193-201): config.json + model.bin ->
    (ModelConfig, DecoderWeights) on `device`."""
    from .decoder import DecoderWeights
    cfg = load_config_json(os.path.join(model_dir, "config.json"))
    weights = ModelWeights.load(os.path.join(model_dir, "model.bin"))
    return cfg, DecoderWeights.from_weights(cfg, weights, device=device, dtype=dtype)
