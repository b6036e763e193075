"""Host-side logic of the multi-GPU forms on CPU ranks (gloo, world sizes 2 and 4): the
position split, the packed partial layout, one all-gather and the log-sum-exp merge, with
each rank's partial computed by the oracle.  The merged result equals attending the whole
sequence.  Also: batch sharding covers every sequence exactly once."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from rustllm_b200.distributed import (pack_partial, packed_width, shard_sequences, split_range,
                                      unpack_parts)

HQ, HKV, D, TOTAL = 8, 2, 32, 1001


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _data():
    rng = np.random.default_rng(21)
    q = rng.standard_normal((1, HQ, 1, D)).astype(np.float32)
    k = rng.standard_normal((1, HKV, TOTAL, D)).astype(np.float32)
    v = rng.standard_normal((1, HKV, TOTAL, D)).astype(np.float32)
    return q, k, v


def _worker(rank, world, port, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import oracle as orc
        q, k, v = _data()
        lo, hi = split_range(TOTAL, rank, world)
        o, lse = orc.attention_core_wide(q, np.ascontiguousarray(k[:, :, lo:hi]),
                                         np.ascontiguousarray(v[:, :, lo:hi]), hi - lo,
                                         hi - lo - 1)
        buf = pack_partial(torch.from_numpy(o[0, :, 0].astype(np.float32)),
                           torch.from_numpy(lse[0, :, 0].astype(np.float32)))
        parts = torch.empty((world, packed_width(HQ, D)), dtype=torch.float32)
        dist.all_gather_into_tensor(parts, buf)
        po, pl = unpack_parts(parts, HQ, D)
        out, out_lse = orc.merge_lse(po.numpy(), pl.numpy())
        result_q.put((rank, out, out_lse, (lo, hi)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_sequence_split_merge_equals_whole(orc, world):
    ctx = mp.get_context("spawn")
    q_ = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q_)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q_.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    q, k, v = _data()
    whole, whole_lse = orc.attention_core_wide(q, k, v, TOTAL, TOTAL - 1)
    ranges = sorted(r[3] for r in results)
    assert ranges[0][0] == 0 and ranges[-1][1] == TOTAL
    assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
    for _, out, out_lse, _ in results:
        assert np.max(np.abs(out - whole[0, :, 0])) < 1e-5
        assert np.max(np.abs(out_lse - whole_lse[0, :, 0])) < 1e-4


@pytest.mark.parametrize("n,world", [(64, 1), (64, 2), (64, 8), (7, 4)])
def test_batch_sharding_covers_each_sequence_once(n, world):
    seen = sorted(s for r in range(world) for s in shard_sequences(n, r, world))
    assert seen == list(range(n))


def test_split_range_partitions():
    for total in (1, 7, 131072):
        for world in (1, 2, 3, 8):
            spans = [split_range(total, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
