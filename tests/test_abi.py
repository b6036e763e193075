"""The C-ABI library loads, exports every function include/tmllm.h declares, and rejects
bad arguments on the host with the reference's error kinds -- all without a GPU (no call
here reaches a kernel)."""
from __future__ import annotations

import ctypes as C
import os
import re

import numpy as np
import pytest

from rustllm_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions() -> list[str]:
    src = open(os.path.join(ROOT, "include", "tmllm.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(tmllm_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_functions()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # and the Python binding covers all of them
    assert set(names) <= set(_lib._PROTOS), set(names) - set(_lib._PROTOS)


def test_status_names_and_version():
    lib = _lib.load()
    assert lib.tmllm_version() >= 100
    for code, cls in _lib._BY_STATUS.items():
        assert lib.tmllm_status_name(code).decode().startswith("TMLLM_")
        assert cls.status == code
    assert lib.tmllm_status_name(0) == b"TMLLM_OK"


def rc(name, *args):
    return getattr(_lib.load(), name)(*args)


def test_host_validation_codes():
    """Argument errors are reported before any device work (kv_cache_write.rs:577-586,
    repeat_kv.rs:20-25, attention_scale_mask.rs validate, softmax.rs validate, ...)."""
    dummy = C.c_void_p(16)
    # start + source_seq > max_seq
    assert rc("tmllm_kv_cache_write", 1, dummy, dummy, 2, 8, 4, 7, 2, None) == 7
    assert rc("tmllm_kv_cache_write", 7, dummy, dummy, 2, 8, 4, 0, 1, None) == 5
    assert rc("tmllm_repeat_kv", 0, dummy, dummy, 1, 2, 2, 2, 0, None) == 8
    assert rc("tmllm_gqa_qk", 0, dummy, dummy, dummy, 1, 5, 2, 1, 4, 4, 4, None) == 8
    assert rc("tmllm_gqa_qk", 0, dummy, dummy, dummy, 1, 4, 2, 1, 5, 4, 4, None) == 2
    assert rc("tmllm_attention_scale_mask", 0, dummy, dummy, 9, 3, 3, 0, 0.0, None) == 2
    assert rc("tmllm_attention_scale_mask", 0, dummy, dummy, 9, 3, 3, 1, 0.5, None) == 2
    assert rc("tmllm_attention_scale_mask", 0, dummy, dummy, 8, 3, 3, 0, 0.5, None) == 2
    assert rc("tmllm_softmax_last_dim", 0, dummy, dummy, 0, 4, None) == 2
    assert rc("tmllm_rope", 0, dummy, dummy, dummy, dummy, 8, 1, 2, 3, 0, None) == 2
    assert rc("tmllm_rope", 0, dummy, dummy, dummy, dummy, 8, 1, 4, 4, 5, None) == 2
    assert b"position range is invalid" in _lib.load().tmllm_last_error()
    cfg = _lib.CacheConfig(device=0, num_layers=1, num_seqs=1, max_seq_len=0, block_size=16,
                           num_kv_heads=2, head_dim=4, dtype=1)
    h = C.c_void_p()
    assert rc("tmllm_cache_create", C.byref(cfg), C.byref(h)) == 2  # kv_cache.rs:61-65
    assert h.value is None
    opts = _lib.DecodeOpts()
    kv = _lib.PagedKV(k_cache=16, v_cache=16, block_table=16, seq_lens=16, num_blocks=4,
                      num_seqs=1, num_kv_heads=3, head_dim=64, block_size=16,
                      max_blocks_per_seq=4, dtype=1)
    assert rc("tmllm_gqa_decode", C.byref(kv), dummy, None, None, dummy, None, 8,
              C.byref(opts), None, 0, None) == 8  # 8 q heads over 3 kv heads
    assert rc("tmllm_gqa_decode", C.byref(kv), dummy, dummy, None, dummy, None, 9,
              C.byref(opts), None, 0, None) == 1  # k_new without v_new


def test_error_mapping_raises_reference_kinds():
    with pytest.raises(_lib.PositionOutOfRange):
        _lib.call("tmllm_kv_cache_write", 1, C.c_void_p(16), C.c_void_p(16), 2, 8, 4, 7, 2, None)
    with pytest.raises(_lib.ModelFormat):
        _lib.call("tmllm_repeat_kv", 0, C.c_void_p(16), C.c_void_p(16), 1, 2, 2, 2, 0, None)


def test_structured_error_fields():
    """PositionOutOfRange {start_pos, seq_len, max_seq_len} and ShapeMismatch {left, right}
    cross the ABI with their fields (src/error.rs:6-9,19-23; raised as in
    src/ops/kv_cache_write.rs:100-110 and src/tensor/gqa_matmul.rs:111-116)."""
    lib = _lib.load()
    dummy = C.c_void_p(16)
    # a cache write of positions [7, 9) into an 8-position cache
    assert rc("tmllm_kv_cache_write", 1, dummy, dummy, 2, 8, 4, 7, 2, None) == 7
    f = _lib.last_error_fields()
    assert (f.status, f.start_pos, f.seq_len, f.max_seq_len) == (7, 7, 2, 8)
    assert (f.left_rank, f.right_rank) == (0, 0)
    assert lib.tmllm_last_error() == b"position range [7, 9) exceeds max sequence length 8"
    with pytest.raises(_lib.PositionOutOfRange) as e:
        _lib.call("tmllm_kv_cache_write", 0, dummy, dummy, 3, 100, 4, 99, 5, None)
    assert (e.value.start_pos, e.value.seq_len, e.value.max_seq_len) == (99, 5, 100)
    # any other failure, and any success, replaces the record
    assert rc("tmllm_repeat_kv", 0, dummy, dummy, 1, 2, 2, 2, 0, None) == 8
    f = _lib.last_error_fields()
    assert (f.status, f.start_pos, f.seq_len, f.max_seq_len) == (8, 0, 0, 0)
    cos = np.empty((4, 2), np.float32)
    sin = np.empty((4, 2), np.float32)
    assert rc("tmllm_rope_tables", cos.ctypes.data, sin.ctypes.data, 4, 4, 10000.0) == 0
    assert _lib.last_error_fields().status == 0
    assert lib.tmllm_last_error_fields(None) == _lib.InvalidArgument.status
    # the Python mirror of the reference's Tensor API validates shapes on the host first
    import torch
    from rustllm_b200 import tensor_ops
    q = torch.zeros((1, 4, 1, 64), dtype=torch.float16)
    k = torch.zeros((2, 2, 8, 64), dtype=torch.float16)
    with pytest.raises(_lib.ShapeMismatch) as e:
        tensor_ops.gqa_qk_matmul(q, k)
    assert (e.value.left, e.value.right) == ([1, 4, 1, 64], [2, 2, 8, 64])
    a = torch.zeros((3, 2, 5), dtype=torch.float32)
    b = torch.zeros((3, 4, 6), dtype=torch.float32)
    with pytest.raises(_lib.ShapeMismatch) as e:
        tensor_ops.batched_matmul(a, b)
    assert (e.value.left, e.value.right) == ([3, 2, 5], [3, 4, 6])
    assert str(_lib.PositionOutOfRange(start_pos=3, seq_len=2, max_seq_len=4)) == \
        "position range [3, 5) exceeds max sequence length 4"


def test_rope_tables_bit_exact_with_oracle(orc):
    """tmllm_rope_tables (host-side, as the reference builds them) equals the oracle."""
    for d, n, theta in [(64, 300, 100000.0), (4, 8, 10000.0), (128, 64, 500000.0)]:
        cos = np.empty((n, d // 2), np.float32)
        sin = np.empty((n, d // 2), np.float32)
        _lib.call("tmllm_rope_tables", cos.ctypes.data, sin.ctypes.data, d, n, theta)
        oc, os_ = orc.rope_tables(d, n, theta)
        assert np.array_equal(cos, oc) and np.array_equal(sin, os_)


def test_workspace_size_arithmetic():
    lib = _lib.load()
    b, hq, hkv, d, s = 2, 32, 8, 128, 37
    got = lib.tmllm_decode_workspace_bytes(b, hq, hkv, d, s)

    def up(x):
        return (x + 255) // 256 * 256
    assert got == up(b * hkv * 4) + up(b * hq * s * 2 * 4) + up(b * hq * s * d * 4)
    assert lib.tmllm_decode_workspace_bytes(0, hq, hkv, d, s) == 0


def test_linear_host_validation():
    """tmllm_linear rejects bad shapes, strides, alignment and option mixes on the host,
    before any device work; its statistics buffer size is [ceil(n/64)][64] floats."""
    lib = _lib.load()
    p = C.c_void_p(256)  # 16-byte aligned, never dereferenced

    def lin(x=p, ldx=64, norm=None, stats_in=None, eps=1e-5, w=p, ldw=64, out=p, ldo=64,
            res=None, ldr=0, stats_out=None, rows=4, k=64, n=64, swiglu=0, flags=0):
        return lib.tmllm_linear(x, ldx, norm, stats_in, eps, w, ldw, out, ldo, res, ldr,
                                stats_out, rows, k, n, swiglu, flags, None)
    assert lin(rows=0) == 2 and lin(rows=65) == 2      # 1..64 rows
    assert lin(k=60, ldx=64) == 2 and lin(n=60) == 2   # whole 16-byte chunks
    assert lin(swiglu=2) == 1
    assert lin(flags=2) == 1                           # only TMLLM_LINEAR_OVERLAP
    assert lin(swiglu=1, ldw=128, res=p, ldr=64) == 1  # SwiGLU and a residual together
    assert lin(stats_in=p) == 1                        # statistics without a norm
    assert lin(x=None) == 1 and lin(out=None) == 1
    assert lin(ldx=32) == 2                            # stride shorter than a row
    assert lin(swiglu=1, ldw=64) == 2                  # [gate | up] needs 2n columns
    assert lin(x=C.c_void_p(258)) == 1                 # 16-byte alignment
    assert lin(ldx=68) == 1                            # row stride in whole chunks
    assert lin(norm=p, eps=0.0) == 2 and lin(norm=p, eps=float("nan")) == 2
    assert b"epsilon" in lib.tmllm_last_error()
    assert lib.tmllm_linear_stats_bytes(960) == 60 * 64 * 4   # one partial per 16 columns
    assert lib.tmllm_linear_stats_bytes(1000) == 63 * 64 * 4
    assert lib.tmllm_linear_stats_bytes(0) == 0


def test_lm_head_host_validation():
    """tmllm_lm_head rejects bad shapes, strides, alignment and a missing workspace on the
    host, before any device work; its workspace is 1 KB."""
    lib = _lib.load()
    p = C.c_void_p(256)  # 16-byte aligned, never dereferenced

    def head(x=p, ldx=64, res=None, ldr=0, norm=None, eps=1e-5, w=p, ldw=64, out=p, ldo=64,
             ids=None, ws=None, rows=4, k=64, n=64, flags=0):
        return lib.tmllm_lm_head(x, ldx, res, ldr, norm, eps, w, ldw, out, ldo, ids, ws, rows,
                                 k, n, flags, None)
    assert lib.tmllm_lm_head_workspace_bytes() == 1024
    assert head(rows=0) == 2 and head(rows=65) == 2      # 1..64 rows
    assert head(k=60, ldx=64) == 2 and head(n=60) == 2   # whole 16-byte chunks
    assert head(flags=2) == 1                            # only TMLLM_LINEAR_OVERLAP
    assert head(x=None) == 1 and head(out=None) == 1 and head(w=None) == 1
    assert head(ids=p) == 1                              # the argmax needs the workspace
    assert head(ids=p, ws=C.c_void_p(260)) == 1          # 8-byte aligned workspace
    assert head(ldx=32) == 2 and head(ldo=32) == 2       # stride shorter than a row
    assert head(res=p, ldr=32) == 2
    assert head(x=C.c_void_p(258)) == 1 and head(res=C.c_void_p(264), ldr=64) == 1
    assert head(ldw=68) == 1                             # row stride in whole chunks
    assert head(norm=p, eps=0.0) == 2
    assert head(rows=64, k=1408, ldx=1408) == 2          # rows too large for shared memory
    assert b"shared memory" in lib.tmllm_last_error()


def test_argmax_and_decode_flag_validation():
    lib = _lib.load()
    p = C.c_void_p(256)
    assert lib.tmllm_argmax(1, p, p, 2, 0, None) == 2          # empty vocabulary
    assert lib.tmllm_argmax(1, None, p, 2, 8, None) == 1
    assert lib.tmllm_argmax(9, p, p, 2, 8, None) == 5          # unknown dtype
    assert lib.tmllm_argmax(1, p, p, 0, 8, None) == 0          # no rows: nothing to do
    kv = _lib.PagedKV(k_cache=256, v_cache=256, block_table=256, seq_lens=256, num_blocks=4,
                      num_seqs=1, num_kv_heads=2, head_dim=64, block_size=16,
                      max_blocks_per_seq=4, dtype=1)
    opts = _lib.DecodeOpts(flags=4)  # only TMLLM_DECODE_OVERLAP is defined
    assert lib.tmllm_gqa_decode(C.byref(kv), p, None, None, p, None, 4, C.byref(opts), None,
                                0, None) == 1
    assert b"flags" in lib.tmllm_last_error()


def test_linear_wrapper_refuses_host_tensors():
    """The Python wrapper checks placement before any pointer reaches the library."""
    import torch
    from rustllm_b200.decoder import linear
    x = torch.zeros((2, 64), dtype=torch.float16)
    w = torch.zeros((64, 64), dtype=torch.float16)
    with pytest.raises(_lib.InvalidArgument):
        linear(x, w)


def test_attention_wrappers_refuse_host_tensors():
    """gqa_decode / gqa_prefill / merge_lse check tensor placement before any pointer
    reaches the library (a host pointer in a kernel would fault the device)."""
    import torch
    import rustllm_b200 as rb
    q = torch.zeros((1, 4, 64), dtype=torch.float16)
    kv = _lib.PagedKV(num_seqs=1, num_kv_heads=2, head_dim=64, block_size=16, dtype=1)
    with pytest.raises(_lib.InvalidArgument):
        rb.gqa_decode(kv, q, None, None, None)
    with pytest.raises(_lib.InvalidArgument):
        rb.gqa_prefill(kv, q, None, None, rows_per_seq=1)
    with pytest.raises(_lib.InvalidArgument):
        rb.merge_lse(torch.zeros((2, 4, 64)), torch.zeros((2, 4)))
