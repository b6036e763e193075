"""Multi-GPU forms of the decode path: one process per GPU over torch.distributed.

* ``SequenceSplitAttention`` — one long sequence split along its positions (BASELINE
  config 4).  Rank r holds positions [r*L/N, (r+1)*L/N) in its own paged cache; the last
  rank holds the tail and appends.  Every rank attends its range for all query heads and
  publishes (O_r F32, lse_r) packed in one buffer; one all-gather exchanges them and each
  rank merges by log-sum-exp (``tmllm_merge_lse``).
* ``shard_sequences`` — batch sharding (config 3): sequence s goes to rank s mod N; the
  ranks never exchange data.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .attention import merge_packed
from .kv_cache import PagedKvCache


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
                 num_splits: int = 0):
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

    def fill(self, k: torch.Tensor, v: torch.Tensor) -> None:
        """Writes this rank's share: k, v [Hkv, hi-lo, D]."""
        n = self.hi - self.lo
        if k.shape[1] != n:
            raise ValueError(f"rank {self.rank} holds {n} positions, got {k.shape[1]}")
        if n:
            self.cache.append(0, 0, k, v)
            self.cache.advance(n, 0)

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

    def step(self, q: torch.Tensor, k_new: torch.Tensor | None, v_new: torch.Tensor | None,
             out: torch.Tensor, rope=None) -> torch.Tensor:
        """One decode token: q [1, Hq, D]; k_new, v_new [1, Hkv, D] (used by the owner);
        out [1, Hq, D].  Lengths are not advanced (see ``advance``).  On one GPU the fused
        kernel writes ``out`` directly; there is nothing to merge."""
        if self.world == 1:
            off = self.global_len - self.cache.len(0)
            self.cache.decode(0, q, k_new, v_new, out=out, rope=rope, rope_pos_offset=off,
                              **self.kw)
            return out
        self.attend_local(q, k_new, v_new, rope)
        return self.exchange_and_merge(out)

    def advance(self) -> None:
        if self.owner:
            self.cache.advance(1, 0)
        self.global_len += 1
