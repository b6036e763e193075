"""Multi-GPU forms of the decode path: one process per GPU over torch.distributed.

* ``SequenceSplitAttention`` — one long sequence split along its positions (BASELINE
  config 4).  Rank r holds positions [r*L/N, (r+1)*L/N) in its own paged cache; the last
  rank holds the tail and appends.  Every rank attends its range for all query heads and
  the partial (O_r, lse_r) are merged by log-sum-exp on every rank (see below for the two
  exchanges).
* ``shard_sequences`` — batch sharding (config 3): sequence s goes to rank s mod N; the
  ranks never exchange data.

The default exchange (``exchange="p2p"``) happens inside the decode kernel: each rank's
final CTAs write their rows into every rank's buffer over NVLink (CUDA IPC mappings from
``PeerExchange``) and merge what arrives, so a step is one launch per rank.  ``"nccl"``
keeps the all-gather + merge-kernel form for comparison.
"""
from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as dist

from . import _lib
from ._lib import DecodeOpts, call
from .attention import DecodeWorkspace, merge_packed
from .kv_cache import PagedKvCache
from .tensor_ops import stream_ptr

HANDLE_BYTES = 64


class PeerExchange:
    """This rank's ``tmllm_exchange``: a receive buffer shared with every rank by CUDA IPC.
    ``rows`` = num_seqs * q_heads, ``groups`` = num_seqs * kv_heads."""

    def __init__(self, rows: int, groups: int, head_dim: int, *, device=None, group=None,
                 timeout_s: float = 2.0):
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.device = torch.device(device or "cuda")
        self._h = None
        handle = (C.c_uint8 * HANDLE_BYTES)()
        h = C.c_void_p()
        with torch.cuda.device(self.device):
            call("tmllm_exchange_create", self.world, self.rank, rows, groups, head_dim,
                 C.byref(h), handle)
        self._h = h
        mine = bytes(handle)
        handles = [None] * self.world
        if self.world > 1:
            dist.all_gather_object(handles, mine, group=group)
        else:
            handles = [mine]
        buf = (C.c_uint8 * (HANDLE_BYTES * self.world)).from_buffer_copy(b"".join(handles))
        with torch.cuda.device(self.device):
            call("tmllm_exchange_connect", self._h, buf)
            call("tmllm_exchange_set_timeout", self._h, int(timeout_s * 1e9))

    @property
    def handle(self):
        return self._h

    def status(self) -> int:
        st = C.c_int32()
        with torch.cuda.device(self.device):
            call("tmllm_exchange_status", self._h, C.byref(st))
        return st.value

    def close(self) -> None:
        if self._h is not None:
            with torch.cuda.device(self.device):
                _lib.load().tmllm_exchange_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def shard_sequences(num_seqs: int, rank: int, world: int) -> list[int]:
    """Sequences owned by ``rank`` when ``num_seqs`` are sharded round-robin."""
    return list(range(rank, num_seqs, world))


def split_range(total: int, rank: int, world: int) -> tuple[int, int]:
    """Positions [lo, hi) of a ``total``-long sequence held by ``rank``."""
    return total * rank // world, total * (rank + 1) // world


def packed_width(q_heads: int, head_dim: int) -> int:
    """Floats one rank publishes: its normalised output [Hq, D], then lse [Hq]."""
    return q_heads * head_dim + q_heads


def pack_partial(out: torch.Tensor, lse: torch.Tensor, buf: torch.Tensor | None = None):
    """Packs (O [Hq, D] F32, lse [Hq] F32) into one [1, Hq*D + Hq] F32 row."""
    hq, d = out.shape[-2], out.shape[-1]
    if buf is None:
        buf = torch.empty((1, packed_width(hq, d)), dtype=torch.float32, device=out.device)
    buf[0, : hq * d] = out.reshape(-1)
    buf[0, hq * d:] = lse.reshape(-1)
    return buf


def unpack_parts(parts: torch.Tensor, q_heads: int, head_dim: int):
    """Views of gathered rows [n, Hq*D + Hq]: (O [n, Hq, D], lse [n, Hq])."""
    n = parts.shape[0]
    return (parts[:, : q_heads * head_dim].reshape(n, q_heads, head_dim),
            parts[:, q_heads * head_dim:])


class SequenceSplitAttention:
    def __init__(self, total_cached: int, q_heads: int, kv_heads: int, head_dim: int, *,
                 dtype=torch.float16, block_size: int = 16, max_new: int = 256,
                 shuffle_seed: int = 0, device=None, group=None, variant: int = 0,
                 num_splits: int = 0, exchange: str = "p2p", overlap: bool = False):
        self.group = group
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.lo, self.hi = split_range(total_cached, self.rank, self.world)
        self.owner = self.rank == self.world - 1
        self.hq, self.hkv, self.d = q_heads, kv_heads, head_dim
        self.device = torch.device(device or "cuda")
        cap = (self.hi - self.lo) + (max_new if self.owner else 0)
        self.cache = PagedKvCache(1, 1, max(cap, 1), kv_heads, head_dim, dtype=dtype,
                                  block_size=block_size, shuffle_seed=shuffle_seed,
                                  device=self.device)
        width = q_heads * head_dim + q_heads
        self.send = torch.zeros((1, width), dtype=torch.float32, device=self.device)
        self.recv = torch.zeros((self.world, width), dtype=torch.float32, device=self.device)
        self.global_len = total_cached
        self.kw = {"variant": variant, "num_splits": num_splits}
        # consecutive steps may overlap (TMLLM_DECODE_OVERLAP): one GPU, or the in-kernel
        # exchange; the caller promises that nothing between two steps writes this rank's
        # cache
        self.overlap = overlap
        if exchange not in ("p2p", "nccl"):
            raise ValueError(f"unknown exchange {exchange!r}")
        self.exchange = exchange if self.world > 1 else "none"
        self.peer = None
        self._kv = None  # p2p step state, made on first use
        if self.exchange == "p2p":
            self.peer = PeerExchange(q_heads, kv_heads, head_dim, device=self.device, group=group)
            self.ws = DecodeWorkspace(1, q_heads, kv_heads, head_dim, device=self.device)

    def fill(self, k: torch.Tensor, v: torch.Tensor) -> None:
        """Writes this rank's share: k, v [Hkv, hi-lo, D]."""
        n = self.hi - self.lo
        if k.shape[1] != n:
            raise ValueError(f"rank {self.rank} holds {n} positions, got {k.shape[1]}")
        if n:
            self.cache.append(0, 0, k, v)
            self.cache.advance(n, 0)
        self._kv = None  # lengths changed: refresh the p2p step state

    def attend_local(self, q: torch.Tensor, k_new: torch.Tensor | None,
                     v_new: torch.Tensor | None, rope=None) -> None:
        """This rank's partial (O_r, lse_r) into the send buffer."""
        o = self.send[0, : self.hq * self.d].view(1, self.hq, self.d)
        lse = self.send[0, self.hq * self.d:].view(1, self.hq)
        off = self.global_len - self.cache.len(0)
        if self.owner:
            self.cache.decode(0, q, k_new, v_new, out=o, lse=lse, rope=rope, rope_pos_offset=off,
                              **self.kw)
        else:
            self.cache.decode(0, q, None, None, out=o, lse=lse, rope=rope, rope_pos_offset=off,
                              **self.kw)

    def exchange_and_merge(self, out: torch.Tensor) -> torch.Tensor:
        if self.world > 1:
            dist.all_gather_into_tensor(self.recv, self.send, group=self.group)
            parts = self.recv
        else:
            parts = self.send
        return merge_packed(parts, self.hq, self.d, out=out.view(self.hq, self.d))

    def step_p2p(self, q: torch.Tensor, k_new: torch.Tensor | None,
                 v_new: torch.Tensor | None, out: torch.Tensor, rope=None) -> torch.Tensor:
        """One decode token with the exchange inside the kernel: one launch per rank.

        At 8 GPUs a rank's kernel takes ~20 µs, so the host side is kept to one library
        call: the cache view (its device pointers never move), the options and the
        lengths are kept between steps and refreshed by ``fill`` / ``advance``."""
        if self._kv is None:
            self._kv = self.cache.view(0)
            self._opts = DecodeOpts(num_splits=self.kw["num_splits"], variant=self.kw["variant"],
                                    flags=_lib.DECODE_OVERLAP if self.overlap else 0)
            self._fn = _lib.load().tmllm_gqa_decode_exchange
            self._local_len = self.cache.len(0)
            self._reserved = self._local_len
            self._argc = {}
        if self.owner and self._reserved < self._local_len + 1:
            self.cache.reserve(0, 1)
            self._reserved = self._local_len + 1
            self._argc.clear()  # the reservation is a kernel ahead of this launch
        own = self.owner
        key = (q.data_ptr(), k_new.data_ptr() if own else None,
               v_new.data_ptr() if own else None, out.data_ptr(), out.dtype,
               None if rope is None else (rope[0].data_ptr(), rope[1].data_ptr()),
               self._local_len, self.global_len, stream_ptr(self.device))
        args = self._argc.get(key)
        if args is None:  # arguments rebuilt only when something changed
            if len(self._argc) >= 8:  # a few alternating buffer sets stay cached
                self._argc.clear()
            o = DecodeOpts(num_splits=self._opts.num_splits, variant=self._opts.variant,
                           flags=self._opts.flags)
            o.out_f32 = int(out.dtype == torch.float32)
            o.rope_pos_offset = self.global_len - self._local_len
            o.max_len_hint = self._local_len + 1
            if rope is not None:
                cos, sin = rope
                o.rope_cos, o.rope_sin, o.rope_len = cos.data_ptr(), sin.data_ptr(), cos.shape[0]
            args = (C.byref(self._kv), key[0], key[1], key[2], key[3], None, self.hq,
                    C.byref(o), self.ws.ptr, self.ws.nbytes, self.peer.handle, key[-1])
            self._argc[key] = args
        rc = self._fn(*args)
        if rc:
            _lib.check(rc)
        return out

    def step(self, q: torch.Tensor, k_new: torch.Tensor | None, v_new: torch.Tensor | None,
             out: torch.Tensor, rope=None) -> torch.Tensor:
        """One decode token: q [1, Hq, D]; k_new, v_new [1, Hkv, D] (used by the owner);
        out [1, Hq, D].  Lengths are not advanced (see ``advance``).  On one GPU the fused
        kernel writes ``out`` directly; there is nothing to merge."""
        if self.exchange == "p2p":
            return self.step_p2p(q, k_new, v_new, out, rope)
        if self.world == 1:
            off = self.global_len - self.cache.len(0)
            self.cache.decode(0, q, k_new, v_new, out=out, rope=rope, rope_pos_offset=off,
                              overlap=self.overlap, **self.kw)
            return out
        self.attend_local(q, k_new, v_new, rope)
        return self.exchange_and_merge(out)

    def advance(self) -> None:
        if self.owner:
            self.cache.advance(1, 0)
            if self._kv is not None:
                self._local_len += 1
        self.global_len += 1
