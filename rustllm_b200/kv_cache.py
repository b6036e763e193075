"""KV caches with the reference's call surface (src/model/kv_cache.rs), backed by the
block-paged cache runtime of ``libtmllm_b200.so``.

``LayerKvCache`` and ``KvCache`` keep the reference's API and semantics: one sequence,
a per-layer length, append validates before it mutates (kv_cache.rs:18-53) and advances
the length, ``key()``/``value()`` return the [1, Hkv, len, D] prefix.  ``PagedKvCache`` is
the batched store the B200 path adds: many sequences, one block table per sequence shared
by all layers, blocks handed out from a pool (optionally in a seeded random order).
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from ._lib import CacheConfig, DecodeOpts, PagedKV, call
from .tensor_ops import dtype_code, on_device, stream_ptr

_TORCH = {_lib.F32: torch.float32, _lib.F16: torch.float16}


def _device_index(device) -> int:
    device = torch.device(device if device is not None else "cuda")
    if device.type != "cuda":
        raise _lib.InvalidArgument("the KV cache lives on a CUDA device")
    return device.index if device.index is not None else torch.cuda.current_device()


class _DeviceArray:
    """Exposes a raw device pointer through ``__cuda_array_interface__``."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": tuple(shape),
                                         "typestr": typestr, "version": 3, "strides": None}


class PagedKvCache:
    """Batched, block-paged K/V store for ``num_layers`` layers and ``num_seqs`` sequences.

    Arena layout per layer: [num_blocks, num_kv_heads, block_size, head_dim].  Lengths are
    per sequence and shared by all layers; ``append`` writes without advancing, ``advance``
    moves the length once per step (the ``self.len = new_len`` of kv_cache.rs:140)."""

    def __init__(self, num_layers: int, num_seqs: int, max_seq_len: int, num_kv_heads: int,
                 head_dim: int, dtype: torch.dtype = torch.float16, block_size: int = 16,
                 num_blocks: int = 0, shuffle_seed: int = 0, device=None):
        self._h = None
        self.device = torch.device("cuda", _device_index(device))
        cfg = CacheConfig(device=self.device.index, num_layers=num_layers, num_seqs=num_seqs,
                          max_seq_len=max_seq_len, block_size=block_size,
                          num_kv_heads=num_kv_heads, head_dim=head_dim,
                          dtype=dtype_code(dtype), num_blocks=num_blocks,
                          shuffle_seed=shuffle_seed)
        h = C.c_void_p()
        call("tmllm_cache_create", C.byref(cfg), C.byref(h))
        self._h = h
        self.num_layers, self.num_seqs = num_layers, num_seqs
        self.max_seq_len, self.num_kv_heads, self.head_dim = max_seq_len, num_kv_heads, head_dim
        self.block_size = block_size
        self.dtype = dtype

    def __del__(self):
        if getattr(self, "_h", None) is not None:
            try:
                _lib.load().tmllm_cache_destroy(self._h)
            except Exception:
                pass
            self._h = None

    @property
    def handle(self):
        return self._h

    def _stream(self) -> int:
        return stream_ptr(self.device)

    def len(self, seq: int = 0) -> int:
        out = C.c_int64()
        call("tmllm_cache_len", self._h, seq, C.byref(out))
        return out.value

    def lens(self) -> list[int]:
        return [self.len(s) for s in range(self.num_seqs)]

    def capacity(self) -> int:
        out = C.c_int64()
        call("tmllm_cache_capacity", self._h, C.byref(out))
        return out.value

    def storage_bytes(self) -> int:
        out = C.c_int64()
        call("tmllm_cache_storage_bytes", self._h, C.byref(out))
        return out.value

    def reset(self, seq: int = -1) -> None:
        call("tmllm_cache_reset", self._h, seq, self._stream())

    def reserve(self, seq: int, n: int) -> None:
        call("tmllm_cache_reserve", self._h, seq, n, self._stream())

    def append(self, layer: int, seq: int, key: torch.Tensor, value: torch.Tensor) -> None:
        """Writes key/value [Hkv, n, D] (or [1, Hkv, n, D]) at the sequence's length."""
        on_device(self.device, key, value)
        if key.dtype != value.dtype or key.dtype != self.dtype:
            raise _lib.UnsupportedDType(
                f"KV cache dtype mismatch: cache={self.dtype}, input={key.dtype}/{value.dtype}")
        k = key.reshape(key.shape[-3:]) if key.dim() == 4 else key
        v = value.reshape(value.shape[-3:]) if value.dim() == 4 else value
        if (k.dim() != 3 or k.shape != v.shape or k.shape[0] != self.num_kv_heads
                or k.shape[2] != self.head_dim):
            raise _lib.ModelFormat(
                f"KV cache write shape does not match this layer: cache has "
                f"{self.num_kv_heads} KV heads, input has shape {list(key.shape)}")
        k, v = k.contiguous(), v.contiguous()
        call("tmllm_cache_append", self._h, layer, seq, k.data_ptr(), v.data_ptr(), k.shape[1],
             dtype_code(k.dtype), self._stream())

    def advance(self, n: int = 1, seq: int = -1) -> None:
        call("tmllm_cache_advance", self._h, seq, n, self._stream())

    def view(self, layer: int) -> PagedKV:
        kv = PagedKV()
        call("tmllm_cache_view", self._h, layer, C.byref(kv))
        return kv

    def block_table(self, seq: int) -> list[int]:
        n = C.c_int64()
        call("tmllm_cache_block_table", self._h, seq, None, 0, C.byref(n))
        buf = (C.c_int32 * max(n.value, 1))()
        call("tmllm_cache_block_table", self._h, seq, buf, n.value, C.byref(n))
        return list(buf[: n.value])

    def gather(self, layer: int, seq: int = 0):
        """Dense copies [Hkv, len, D] of the sequence's keys and values."""
        n = self.len(seq)
        shape = (self.num_kv_heads, n, self.head_dim)
        k = torch.empty(shape, dtype=self.dtype, device=self.device)
        v = torch.empty(shape, dtype=self.dtype, device=self.device)
        call("tmllm_cache_gather", self._h, layer, seq, k.data_ptr(), v.data_ptr(),
             self._stream())
        return k, v

    def arena(self, layer: int):
        """The layer's K and V arenas as torch views [num_blocks, Hkv, block_size, D]
        (no copy; valid while this cache lives)."""
        kv = self.view(layer)
        shape = (kv.num_blocks, self.num_kv_heads, self.block_size, self.head_dim)
        typestr = "<f2" if self.dtype == torch.float16 else "<f4"
        return tuple(torch.as_tensor(_DeviceArray(ptr, shape, typestr), device=self.device)
                     for ptr in (kv.k_cache, kv.v_cache))

    def decode(self, layer: int, q: torch.Tensor, k_new: torch.Tensor | None,
               v_new: torch.Tensor | None, *, out: torch.Tensor | None = None,
               out_dtype: torch.dtype | None = None, lse: torch.Tensor | None = None,
               want_lse: bool = False, scale: float = 0.0, num_splits: int = 0, rope=None,
               rope_pos_offset: int = 0, variant: int = 0, overlap: bool = False):
        """Fused append + GQA decode attention for every sequence (one query token each).

        q [num_seqs, Hq, D]; k_new, v_new [num_seqs, Hkv, D] or None (attend only).
        Returns out [num_seqs, Hq, D] (and lse [num_seqs, Hq] F32 when ``want_lse`` or
        ``lse`` is given).  Lengths are not advanced; call ``advance()`` once per step
        after the last layer.  ``overlap`` (TMLLM_DECODE_OVERLAP) lets the tensor-core
        kernel start while the kernel ahead of it drains: the caller promises that kernel
        writes neither the lengths, the block table nor the cached K/V."""
        on_device(self.device, q, k_new, v_new, out, lse, rope)
        if q.dtype != self.dtype:
            raise _lib.UnsupportedDType(
                f"SelfAttention/cache dtype mismatch: attention={q.dtype}, cache={self.dtype}")
        if q.dim() != 3 or q.shape[0] != self.num_seqs or q.shape[2] != self.head_dim:
            raise _lib.ModelFormat(f"decode expects q [{self.num_seqs}, Hq, {self.head_dim}], "
                                   f"got {list(q.shape)}")
        hq = q.shape[1]
        if k_new is not None:
            for t in (k_new, v_new):
                if (t is None or t.dtype != self.dtype or tuple(t.shape) !=
                        (self.num_seqs, self.num_kv_heads, self.head_dim)):
                    raise _lib.ModelFormat("k_new/v_new must be [num_seqs, Hkv, D] in the "
                                           "cache dtype")
        if out is None:
            out = torch.empty((self.num_seqs, hq, self.head_dim), dtype=out_dtype or self.dtype,
                              device=self.device)
        if out.dtype not in (self.dtype, torch.float32) or tuple(out.shape) != (
                self.num_seqs, hq, self.head_dim) or not out.is_contiguous():
            raise _lib.InvalidArgument("out must be a contiguous [num_seqs, Hq, D] tensor in the "
                                       "cache dtype or F32")
        if lse is None and want_lse:
            lse = torch.empty((self.num_seqs, hq), dtype=torch.float32, device=self.device)
        opts = DecodeOpts(scale=scale, num_splits=num_splits, out_f32=int(out.dtype == torch.float32),
                          rope_pos_offset=rope_pos_offset, variant=variant,
                          flags=_lib.DECODE_OVERLAP if overlap else 0)
        if rope is not None:
            cos, sin = rope
            opts.rope_cos, opts.rope_sin, opts.rope_len = cos.data_ptr(), sin.data_ptr(), cos.shape[0]
        q = q.contiguous()
        kp = k_new.contiguous().data_ptr() if k_new is not None else None
        vp = v_new.contiguous().data_ptr() if v_new is not None else None
        call("tmllm_cache_decode", self._h, layer, q.data_ptr(), kp, vp, out.data_ptr(),
             lse.data_ptr() if lse is not None else None, hq, C.byref(opts), self._stream())
        return (out, lse) if (want_lse or lse is not None) else out


    def prefill(self, layer: int, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor, *,
                out: torch.Tensor | None = None, out_dtype: torch.dtype | None = None,
                scale: float = 0.0, rope=None, rope_pos_offset: int = 0, variant: int = 0):
        """Fused append + causal attention of ``n`` new tokens for every sequence.

        q [num_seqs, n, Hq, D]; k_new, v_new [num_seqs, n, Hkv, D] (or the same as
        [num_seqs * n, heads, D] row-strided views).  Token i of sequence s is appended at
        its length + i and attends positions [0, length + i].  Returns out
        [num_seqs * n, Hq, D].  Lengths are not advanced; call ``advance(n)`` after the last
        layer."""
        on_device(self.device, q, k_new, v_new, out, rope)
        if q.dtype != self.dtype:
            raise _lib.UnsupportedDType(
                f"SelfAttention/cache dtype mismatch: attention={q.dtype}, cache={self.dtype}")
        if q.dim() == 4:
            q, k_new, v_new = (t.reshape(-1, t.shape[2], t.shape[3]) for t in (q, k_new, v_new))
        rows, hq, d = q.shape
        if rows % self.num_seqs or d != self.head_dim:
            raise _lib.ModelFormat(f"prefill expects [num_seqs * n, Hq, {self.head_dim}] rows, "
                                   f"got {list(q.shape)}")
        n = rows // self.num_seqs
        from .attention import _row_stride
        qs = _row_stride(q, hq, d, "q")
        ks = _row_stride(k_new, self.num_kv_heads, d, "k_new")
        if (_row_stride(v_new, self.num_kv_heads, d, "v_new") != ks or k_new.dtype != self.dtype
                or v_new.dtype != self.dtype or k_new.shape[0] != rows or v_new.shape[0] != rows):
            raise _lib.ModelFormat("k_new/v_new must be [rows, Hkv, D] in the cache dtype with "
                                   "one row stride")
        if out is None:
            out = torch.empty((rows, hq, d), dtype=out_dtype or self.dtype, device=self.device)
        if out.dtype not in (self.dtype, torch.float32) or tuple(out.shape) != (
                rows, hq, d) or not out.is_contiguous():
            raise _lib.InvalidArgument("out must be a contiguous [rows, Hq, D] tensor in the "
                                       "cache dtype or F32")
        opts = DecodeOpts(scale=scale, out_f32=int(out.dtype == torch.float32),
                          rope_pos_offset=rope_pos_offset, variant=variant, q_seq_stride=qs,
                          kv_seq_stride=ks)
        if rope is not None:
            cos, sin = rope
            opts.rope_cos, opts.rope_sin, opts.rope_len = cos.data_ptr(), sin.data_ptr(), cos.shape[0]
        call("tmllm_cache_prefill", self._h, layer, q.data_ptr(), k_new.data_ptr(),
             v_new.data_ptr(), n, out.data_ptr(), hq, C.byref(opts), self._stream())
        return out


class LayerKvCache:
    """src/model/kv_cache.rs:9-143 — one layer, one sequence.

    ``block_size`` defaults to the capacity, which stores exactly the reference's
    [1, Hkv, max, D] buffer; a smaller block size pages it."""

    def __init__(self, num_kv_heads: int, max: int, dim: int,
                 dtype: torch.dtype = torch.float16, device=None, block_size: int | None = None):
        if num_kv_heads == 0 or max == 0 or dim == 0:  # kv_cache.rs:61-65
            raise _lib.InvalidShape("KV cache dimensions must be positive")
        self._store = PagedKvCache(1, 1, max, num_kv_heads, dim, dtype=dtype,
                                   block_size=block_size or max, device=device)
        self.num_kv_heads, self.max_seq_len, self.head_dim = num_kv_heads, max, dim

    @property
    def store(self) -> PagedKvCache:
        return self._store

    def len(self) -> int:
        return self._store.len(0)

    def __len__(self) -> int:
        return self.len()

    def is_empty(self) -> bool:
        return self.len() == 0

    def capacity(self) -> int:
        return self._store.capacity()

    def storage_bytes(self) -> int:
        """Bytes reserved for both key and value storage (kv_cache.rs:87-89)."""
        return 2 * self.num_kv_heads * self.max_seq_len * self.head_dim * \
            torch.finfo(self.dtype).bits // 8

    def reset(self) -> None:
        self._store.reset(0)

    @property
    def dtype(self) -> torch.dtype:
        return self._store.dtype

    def key(self) -> torch.Tensor:
        """[1, Hkv, len, D] (a dense copy; the reference returns a strided view)."""
        return self._store.gather(0, 0)[0].unsqueeze(0)

    def value(self) -> torch.Tensor:
        return self._store.gather(0, 0)[1].unsqueeze(0)

    def append(self, key: torch.Tensor, value: torch.Tensor) -> None:
        """kv_cache.rs:104-142: validate (dtype, [1, Hkv, S, D], capacity), write, then
        advance the length.  A rejected append changes nothing."""
        if key.dtype != self.dtype or value.dtype != self.dtype:
            raise _lib.UnsupportedDType(
                f"KV cache dtype mismatch: cache={self.dtype}/{self.dtype}, "
                f"input={key.dtype}/{value.dtype}")
        if (key.shape != value.shape or key.dim() != 4 or key.shape[0] != 1
                or key.shape[1] != self.num_kv_heads or key.shape[3] != self.head_dim):
            raise _lib.ModelFormat(
                f"KV cache write shape does not match this layer: cache has "
                f"{self.num_kv_heads} KV heads, input has {key.shape[1] if key.dim() > 1 else '?'} heads")
        seq = key.shape[2]
        if self.len() + seq > self.max_seq_len:
            raise _lib.PositionOutOfRange(start_pos=self.len(), seq_len=seq,
                                          max_seq_len=self.max_seq_len)
        self._store.append(0, 0, key, value)
        self._store.advance(seq, 0)


class KvCache:
    """src/model/kv_cache.rs:145-184 — a list of per-layer caches."""

    def __init__(self, layers: int, max: int, num_kv_heads: int, dim: int,
                 dtype: torch.dtype = torch.float16, device=None, block_size: int | None = None):
        self.layers = [LayerKvCache(num_kv_heads, max, dim, dtype, device, block_size)
                       for _ in range(layers)]
        self._max = max

    def layer_mut(self, index: int) -> LayerKvCache:
        if not 0 <= index < len(self.layers):
            raise _lib.ModelFormat(f"KV cache layer {index} does not exist")
        return self.layers[index]

    def num_layers(self) -> int:
        return len(self.layers)

    def max_seq_len(self) -> int:
        return self._max

    def storage_bytes(self) -> int:
        return sum(layer.storage_bytes() for layer in self.layers)

    def reset(self) -> None:
        for layer in self.layers:
            layer.reset()
