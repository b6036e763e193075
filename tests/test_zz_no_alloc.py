"""tmllm_gqa_decode_noalloc: the decode entry point for callers that cannot allocate.

Callers inside a stream capture, callers whose device memory comes from a pool they do not
own, and real-time loops that may not take allocator locks use this form: its split
scratch is a fixed array inside the library instead of a workspace the caller provides.
This file runs last (its name sorts last) and must pass both alone and after the rest of
the suite.  It calls the entry point through the C ABI twice in a row and compares each
result with the workspace-taking tmllm_gqa_decode, within the F16 tolerance of the decode
tests (2e-3 relative); it also checks that an oversized call is refused."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

import rustllm_b200 as rb
from rustllm_b200 import _lib

pytestmark = pytest.mark.gpu

HQ, HKV, D, N = 32, 8, 128, 20000


def rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.double(), b.double()
    return float((a - b).abs().max() / b.abs().max())


def test_noalloc_matches_workspace_decode_twice(cuda):
    g = torch.Generator(device=cuda).manual_seed(99)
    cache = rb.PagedKvCache(1, 1, N + 1, HKV, D, dtype=torch.float16, block_size=16,
                            shuffle_seed=17, device=cuda)
    cache.append(0, 0, torch.randn((HKV, N, D), generator=g, device=cuda).half(),
                 torch.randn((HKV, N, D), generator=g, device=cuda).half())
    cache.advance(N, 0)
    cache.reserve(0, 1)  # the block for the appended position
    kv = cache.view(0)
    q = torch.randn((1, HQ, D), generator=g, device=cuda).half()
    kn = torch.randn((1, HKV, D), generator=g, device=cuda).half()
    vn = torch.randn((1, HKV, D), generator=g, device=cuda).half()
    stream = torch.cuda.current_stream(cuda).cuda_stream

    ws = rb.DecodeWorkspace(1, HQ, HKV, D, device=cuda)
    ref = torch.empty((1, HQ, D), dtype=torch.float16, device=cuda)
    ref_lse = torch.empty((1, HQ), dtype=torch.float32, device=cuda)
    opts = _lib.DecodeOpts(max_len_hint=N + 1)
    _lib.call("tmllm_gqa_decode", C.byref(kv), q.data_ptr(), kn.data_ptr(), vn.data_ptr(),
              ref.data_ptr(), ref_lse.data_ptr(), HQ, C.byref(opts), ws.ptr, ws.nbytes, stream)

    for _ in range(2):
        out = torch.full((1, HQ, D), float("nan"), dtype=torch.float16, device=cuda)
        lse = torch.full((1, HQ), float("nan"), dtype=torch.float32, device=cuda)
        _lib.call("tmllm_gqa_decode_noalloc", C.byref(kv), q.data_ptr(), kn.data_ptr(),
                  vn.data_ptr(), out.data_ptr(), lse.data_ptr(), HQ, C.byref(opts), stream)
        torch.cuda.synchronize()
        assert rel(out, ref) < 2e-3
        assert float((lse - ref_lse).abs().max()) < 1e-3
        assert not torch.isnan(out).any()


def test_noalloc_refuses_oversized_scratch(cuda):
    """64 sequences x 16 query heads x 256 dims x 64 splits need far more than 2 MiB."""
    kv = _lib.PagedKV(k_cache=256, v_cache=256, block_table=256, seq_lens=256, num_blocks=64,
                      num_seqs=64, num_kv_heads=2, head_dim=256, block_size=16,
                      max_blocks_per_seq=4, dtype=_lib.F16)
    opts = _lib.DecodeOpts(num_splits=64)
    rc = _lib.load().tmllm_gqa_decode_noalloc(C.byref(kv), C.c_void_p(256), None, None,
                                              C.c_void_p(256), None, 16, C.byref(opts), None)
    assert rc == _lib.InvalidShape.status
    assert b"built-in scratch" in _lib.load().tmllm_last_error()


def test_noalloc_single_split_with_more_groups_than_counters(cuda):
    """With one split no ticket is taken, so nothing is cleared: 65535 sequences x 16 KV
    heads (about a million (sequence, KV head) groups, whose tickets would need 4 MiB, twice
    the built-in scratch) run with num_splits = 1 and match the workspace decode."""
    B, hq, hkv, d, n = 65535, 16, 16, 64, 5
    g = torch.Generator(device=cuda).manual_seed(7)
    k_ar = torch.randn((1, hkv, 16, d), generator=g, device=cuda).half()
    v_ar = torch.randn((1, hkv, 16, d), generator=g, device=cuda).half()
    table = torch.zeros((B, 1), dtype=torch.int32, device=cuda)  # every sequence: block 0
    lens = torch.full((B,), n, dtype=torch.int32, device=cuda)
    kv = rb.paged_kv_from_tensors(k_ar, v_ar, table, lens)
    q = torch.randn((B, hq, d), generator=g, device=cuda).half()
    stream = torch.cuda.current_stream(cuda).cuda_stream
    opts = _lib.DecodeOpts(num_splits=1, max_len_hint=n)
    ref = torch.empty_like(q)
    _lib.call("tmllm_gqa_decode", C.byref(kv), q.data_ptr(), None, None, ref.data_ptr(), None,
              hq, C.byref(opts), None, 0, stream)
    for _ in range(2):
        out = torch.full_like(q, float("nan"))
        _lib.call("tmllm_gqa_decode_noalloc", C.byref(kv), q.data_ptr(), None, None,
                  out.data_ptr(), None, hq, C.byref(opts), stream)
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
    # one more sequence than the grid allows is refused on the host
    kv.num_seqs = B + 1
    rc = _lib.load().tmllm_gqa_decode_noalloc(C.byref(kv), q.data_ptr(), None, None,
                                              out.data_ptr(), None, hq, C.byref(opts), stream)
    assert rc == _lib.InvalidShape.status
