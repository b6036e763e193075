"""Sequence split across GPUs (config 4's multi-GPU form), one rank per GPU: every rank
attends its share of positions with the fused kernel and the (O, lse) partials are
exchanged either inside the kernel over NVLink (p2p) or by an NCCL all-gather plus a merge
kernel (nccl); the result equals the float64 oracle over the whole sequence within the
F16 tolerance, on every rank.  Needs two GPUs; skipped otherwise.  The bounded wait of the
in-kernel exchange is tested on one GPU."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

HQ, HKV, D, TOTAL = 32, 8, 128, 20000


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _full_data():
    g = torch.Generator().manual_seed(5)
    k = torch.randn((HKV, TOTAL, D), generator=g).half()
    v = torch.randn((HKV, TOTAL, D), generator=g).half()
    q = torch.randn((1, HQ, D), generator=g).half()
    kn = torch.randn((1, HKV, D), generator=g).half()
    vn = torch.randn((1, HKV, D), generator=g).half()
    return k, v, q, kn, vn


def _rank(rank, world, port, out_q, exchange):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=timedelta(seconds=60))
    try:
        from rustllm_b200.distributed import SequenceSplitAttention
        k, v, q, kn, vn = _full_data()
        sp = SequenceSplitAttention(TOTAL, HQ, HKV, D, dtype=torch.float16, block_size=16,
                                    shuffle_seed=3 + rank, device=dev, exchange=exchange)
        sp.fill(k[:, sp.lo:sp.hi].to(dev), v[:, sp.lo:sp.hi].to(dev))
        out = torch.empty((1, HQ, D), dtype=torch.float16, device=dev)
        for _ in range(3):  # repeated steps exercise the alternating exchange slots
            sp.step(q.to(dev), kn.to(dev), vn.to(dev), out)
        torch.cuda.synchronize()
        if sp.peer is not None:
            assert sp.peer.status() == 0
        row = None
        if sp.owner:  # the appended row landed at the end of the owner's share
            sp.advance()
            kk, _ = sp.cache.gather(0, 0)
            row = kk[:, -1].cpu().numpy()
        out_q.put((rank, out.float().cpu().numpy(), row))
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("exchange", ["p2p", "nccl"])
def test_sequence_split_all_ranks_match_oracle(orc, exchange):
    """Every GPU of the box as one rank (2 to 8)."""
    import torch.multiprocessing as mp
    world = min(torch.cuda.device_count(), 8)
    ctx = mp.get_context("spawn")
    q_ = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q_, exchange)) for r in range(world)]
    for p in procs:
        p.start()
    results = sorted(q_.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    k, v, q, kn, vn = _full_data()
    kc = torch.cat([k, kn[0][:, None]], 1)[None].numpy()
    vc = torch.cat([v, vn[0][:, None]], 1)[None].numpy()
    wide, _ = orc.attention_core_wide(q[:, :, None].numpy(), kc, vc, TOTAL + 1, TOTAL,
                                      threads=os.cpu_count() or 4)
    want = wide[0, :, 0]
    for _, out, _ in results:
        got = out[0]
        assert np.max(np.abs(got - want)) / np.max(np.abs(want)) < 2e-3
    owner_row = results[-1][2]
    assert np.array_equal(owner_row.view(np.uint16), kn[0].numpy().view(np.uint16))


def test_exchange_wait_expires_with_status(cuda):
    """The in-kernel wait for other ranks is bounded: rank 0 of a 2-rank exchange runs
    alone (rank 1's buffer exists on the same GPU but rank 1 never launches), so the
    arrival it waits for never comes.  The launch must end after the timeout and report
    TMLLM_TIMEOUT, with the GPU still usable."""
    import ctypes as C
    import time

    import rustllm_b200 as rb
    from rustllm_b200 import _lib

    hq, hkv, d, n = 8, 2, 128, 300
    h = [C.c_void_p(), C.c_void_p()]
    for r in range(2):
        _lib.call("tmllm_exchange_create", 2, r, hq, hkv, d, C.byref(h[r]), None)
    arr = (C.c_void_p * 2)(h[0], h[1])
    _lib.call("tmllm_exchange_connect_local", h[0], arr)
    _lib.call("tmllm_exchange_set_timeout", h[0], 5_000_000)  # 5 ms
    try:
        cache = rb.PagedKvCache(1, 1, n + 1, hkv, d, dtype=torch.float16, device=cuda)
        x = torch.randn((hkv, n, d), device=cuda).half()
        cache.append(0, 0, x, x)
        cache.advance(n, 0)
        kv = cache.view(0)
        ws = rb.DecodeWorkspace(1, hq, hkv, d, device=cuda)
        q = torch.randn((1, hq, d), device=cuda).half()
        out = torch.full((1, hq, d), 7.0, dtype=torch.float16, device=cuda)
        opts = _lib.DecodeOpts()
        t0 = time.time()
        _lib.call("tmllm_gqa_decode_exchange", C.byref(kv), q.data_ptr(), None, None,
                  out.data_ptr(), None, hq, C.byref(opts), ws.ptr, ws.nbytes, h[0],
                  torch.cuda.current_stream(cuda).cuda_stream)
        torch.cuda.synchronize()
        assert time.time() - t0 < 10.0
        st = C.c_int32()
        _lib.call("tmllm_exchange_status", h[0], C.byref(st))
        assert st.value == _lib.DeviceTimeout.status
        assert torch.count_nonzero(out) == 0  # an expired exchange writes zeros
        _lib.call("tmllm_exchange_status", h[0], C.byref(st))
        assert st.value == 0  # reading clears it
        # the context is still usable
        assert float(torch.ones(4, device=cuda).sum()) == 4.0
    finally:
        for r in range(2):
            _lib.load().tmllm_exchange_destroy(h[r])


def test_exchange_shape_mismatch_carries_both_shapes(cuda):
    """A call whose shape differs from the exchange's is refused on the host with
    ShapeMismatch {left = the exchange's [rows, groups, head_dim], right = the call's}."""
    import ctypes as C

    import rustllm_b200 as rb
    from rustllm_b200 import _lib

    hq, hkv, d = 8, 2, 128
    h = C.c_void_p()
    _lib.call("tmllm_exchange_create", 1, 0, hq, hkv, d, C.byref(h), None)
    arr = (C.c_void_p * 1)(h)
    _lib.call("tmllm_exchange_connect_local", h, arr)
    try:
        cache = rb.PagedKvCache(1, 2, 64, hkv, d, dtype=torch.float16, device=cuda)
        kv = cache.view(0)  # two sequences: 16 rows, 4 groups
        opts = _lib.DecodeOpts()
        p = torch.zeros((2, hq, d), dtype=torch.float16, device=cuda)
        with pytest.raises(_lib.ShapeMismatch) as e:
            _lib.call("tmllm_gqa_decode_exchange", C.byref(kv), p.data_ptr(), None, None,
                      p.data_ptr(), None, hq, C.byref(opts), None, 0, h, None)
        assert (e.value.left, e.value.right) == ([hq, hkv, d], [2 * hq, 2 * hkv, d])
    finally:
        _lib.load().tmllm_exchange_destroy(h)
