"""ctypes binding of ``libtmllm_b200.so`` (the C ABI declared in ``include/tmllm.h``).

There is no fallback: if the library is missing or a call fails, an exception is raised.
Status codes map onto the reference's ``TinyError`` variants (src/error.rs:3-43).
"""
from __future__ import annotations

import ctypes as C
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libtmllm_b200.so")

F32 = 0
F16 = 1
DECODE_OVERLAP = 1  # TMLLM_DECODE_OVERLAP
LINEAR_OVERLAP = 1  # TMLLM_LINEAR_OVERLAP

vp = C.c_void_p
i32 = C.c_int32
i64 = C.c_int64
sz = C.c_size_t


class TinyError(Exception):
    """Mirror of the reference's ``TinyError`` (src/error.rs:3-43)."""

    status = -1

    def __init__(self, message: str, status: int | None = None):
        super().__init__(message)
        if status is not None:
            self.status = status


class InvalidArgument(TinyError):
    status = 1


class InvalidShape(TinyError):
    status = 2


class ShapeMismatch(TinyError):
    """TinyError::ShapeMismatch { left, right } (src/error.rs:6-9): the two shapes."""

    status = 3

    def __init__(self, message: str, status: int | None = None, *, left=None, right=None):
        super().__init__(message, status)
        self.left = [int(d) for d in left] if left is not None else []
        self.right = [int(d) for d in right] if right is not None else []


class InvalidDimension(TinyError):
    status = 4


class UnsupportedDType(TinyError):
    status = 5


class NonContiguousTensor(TinyError):
    status = 6


class PositionOutOfRange(TinyError):
    """TinyError::PositionOutOfRange { start_pos, seq_len, max_seq_len } (src/error.rs:19-23)."""

    status = 7

    def __init__(self, message: str | None = None, status: int | None = None, *,
                 start_pos: int = 0, seq_len: int = 0, max_seq_len: int = 0):
        if message is None:  # the reference's Display text (src/error.rs:86-95)
            message = (f"position range [{start_pos}, {start_pos + seq_len}) exceeds max "
                       f"sequence length {max_seq_len}")
        super().__init__(message, status)
        self.start_pos, self.seq_len, self.max_seq_len = int(start_pos), int(seq_len), \
            int(max_seq_len)


class ModelFormat(TinyError):
    status = 8


class DeviceError(TinyError):
    """CUDA runtime failure (the reference's ``TinyError::Metal``)."""

    status = 9


class OutOfBlocks(TinyError):
    status = 10


class DeviceTimeout(TinyError):
    status = 11


class NotReserved(TinyError):
    status = 12


class IoError(TinyError):
    """TinyError::Io (src/error.rs:30): a file could not be read or written (host only)."""


class MissingWeight(TinyError):
    """TinyError::MissingWeight (src/error.rs:36): a weight the model needs is absent."""


_BY_STATUS = {cls.status: cls for cls in (
    InvalidArgument, InvalidShape, ShapeMismatch, InvalidDimension, UnsupportedDType,
    NonContiguousTensor, PositionOutOfRange, ModelFormat, DeviceError, OutOfBlocks,
    DeviceTimeout, NotReserved)}


class PagedKV(C.Structure):
    """``tmllm_paged_kv``: device pointers of one layer's block-paged store."""

    _fields_ = [("k_cache", vp), ("v_cache", vp), ("block_table", vp), ("seq_lens", vp),
                ("num_blocks", i64), ("num_seqs", i32), ("num_kv_heads", i32),
                ("head_dim", i32), ("block_size", i32), ("max_blocks_per_seq", i32),
                ("dtype", i32)]


class DecodeOpts(C.Structure):
    """``tmllm_decode_opts``."""

    _fields_ = [("scale", C.c_float), ("num_splits", i32), ("out_f32", i32),
                ("rope_cos", vp), ("rope_sin", vp), ("rope_len", i32),
                ("rope_pos_offset", i32), ("max_len_hint", i64), ("variant", i32),
                ("flags", i32), ("q_seq_stride", i64), ("kv_seq_stride", i64)]


class CacheConfig(C.Structure):
    """``tmllm_cache_config``."""

    _fields_ = [("device", i32), ("num_layers", i32), ("num_seqs", i32),
                ("max_seq_len", i32), ("block_size", i32), ("num_kv_heads", i32),
                ("head_dim", i32), ("dtype", i32), ("num_blocks", i64),
                ("shuffle_seed", C.c_uint64)]


MAX_RANK = 8


class ErrorFields(C.Structure):
    """``tmllm_error_fields``: the fields of the last failure's structured variant."""

    _fields_ = [("status", i32), ("left_rank", i32), ("right_rank", i32), ("reserved", i32),
                ("start_pos", i64), ("seq_len", i64), ("max_seq_len", i64),
                ("left", i64 * MAX_RANK), ("right", i64 * MAX_RANK)]


_PROTOS = {
    "tmllm_version": (C.c_int, []),
    "tmllm_status_name": (C.c_char_p, [C.c_int]),
    "tmllm_last_error": (C.c_char_p, []),
    "tmllm_last_error_fields": (C.c_int, [C.POINTER(ErrorFields)]),
    "tmllm_sync": (C.c_int, [vp]),
    "tmllm_kv_cache_write": (C.c_int, [C.c_int, vp, vp, sz, sz, sz, sz, sz, vp]),
    "tmllm_concat_sequence": (C.c_int, [C.c_int, vp, vp, vp, sz, sz, sz, sz, sz, vp]),
    "tmllm_repeat_kv": (C.c_int, [C.c_int, vp, vp, sz, sz, sz, sz, sz, vp]),
    "tmllm_gqa_qk": (C.c_int, [C.c_int, vp, vp, vp, sz, sz, sz, sz, sz, sz, sz, vp]),
    "tmllm_gqa_pv": (C.c_int, [C.c_int, vp, vp, vp, sz, sz, sz, sz, sz, sz, sz, vp]),
    "tmllm_attention_scale_mask": (C.c_int, [C.c_int, vp, vp, sz, sz, sz, sz, C.c_float, vp]),
    "tmllm_softmax_last_dim": (C.c_int, [C.c_int, vp, vp, sz, sz, vp]),
    "tmllm_batched_matmul": (C.c_int, [C.c_int, vp, vp, vp, sz, sz, sz, sz, vp]),
    "tmllm_rope_tables": (C.c_int, [vp, vp, sz, sz, C.c_float]),
    "tmllm_rope": (C.c_int, [C.c_int, vp, vp, vp, vp, sz, sz, sz, sz, sz, vp]),
    "tmllm_embedding": (C.c_int, [C.c_int, vp, vp, vp, sz, sz, sz, vp, vp]),
    "tmllm_add_rmsnorm": (C.c_int, [C.c_int, vp, vp, vp, vp, vp, sz, sz, C.c_float, vp]),
    "tmllm_swiglu": (C.c_int, [C.c_int, vp, vp, sz, sz, vp]),
    "tmllm_argmax": (C.c_int, [C.c_int, vp, vp, sz, sz, vp]),
    "tmllm_linear_stats_bytes": (sz, [i32]),
    "tmllm_linear_status": (C.c_int, [vp]),
    "tmllm_linear": (C.c_int, [vp, i64, vp, vp, C.c_float, vp, i64, vp, i64, vp, i64, vp, i32,
                               i32, i32, i32, C.c_uint32, vp]),
    "tmllm_lm_head_workspace_bytes": (sz, []),
    "tmllm_lm_head": (C.c_int, [vp, i64, vp, i64, vp, C.c_float, vp, i64, vp, i64, vp, vp, i32,
                                i32, i32, C.c_uint32, vp]),
    "tmllm_decode_workspace_bytes": (sz, [i32, i32, i32, i32, i32]),
    "tmllm_decode_workspace_init": (C.c_int, [vp, sz, vp]),
    "tmllm_decode_auto_splits": (i32, [i32, i32, i64]),
    "tmllm_gqa_decode": (C.c_int, [C.POINTER(PagedKV), vp, vp, vp, vp, vp, i32,
                                   C.POINTER(DecodeOpts), vp, sz, vp]),
    "tmllm_gqa_decode_noalloc": (C.c_int, [C.POINTER(PagedKV), vp, vp, vp, vp, vp, i32,
                                           C.POINTER(DecodeOpts), vp]),
    "tmllm_gqa_prefill": (C.c_int, [C.POINTER(PagedKV), vp, vp, vp, vp, i32, i32, i32, vp, i32,
                                    C.POINTER(DecodeOpts), vp]),
    "tmllm_prefill_status": (C.c_int, [C.POINTER(i32)]),
    "tmllm_merge_lse": (C.c_int, [vp, vp, i32, i32, i32, i64, i64, vp, i32, vp, vp]),
    "tmllm_exchange_create": (C.c_int, [i32, i32, i32, i32, i32, C.POINTER(vp), vp]),
    "tmllm_exchange_connect": (C.c_int, [vp, vp]),
    "tmllm_exchange_connect_local": (C.c_int, [vp, C.POINTER(vp)]),
    "tmllm_exchange_set_timeout": (C.c_int, [vp, C.c_uint64]),
    "tmllm_exchange_status": (C.c_int, [vp, C.POINTER(i32)]),
    "tmllm_exchange_destroy": (C.c_int, [vp]),
    "tmllm_gqa_decode_exchange": (C.c_int, [C.POINTER(PagedKV), vp, vp, vp, vp, vp, i32,
                                            C.POINTER(DecodeOpts), vp, sz, vp, vp]),
    "tmllm_cache_create": (C.c_int, [C.POINTER(CacheConfig), C.POINTER(vp)]),
    "tmllm_cache_destroy": (C.c_int, [vp]),
    "tmllm_cache_len": (C.c_int, [vp, i32, C.POINTER(i64)]),
    "tmllm_cache_capacity": (C.c_int, [vp, C.POINTER(i64)]),
    "tmllm_cache_storage_bytes": (C.c_int, [vp, C.POINTER(i64)]),
    "tmllm_cache_reset": (C.c_int, [vp, i32, vp]),
    "tmllm_cache_reserve": (C.c_int, [vp, i32, i64, vp]),
    "tmllm_cache_append": (C.c_int, [vp, i32, i32, vp, vp, i64, i32, vp]),
    "tmllm_cache_advance": (C.c_int, [vp, i32, i64, vp]),
    "tmllm_cache_view": (C.c_int, [vp, i32, C.POINTER(PagedKV)]),
    "tmllm_cache_block_table": (C.c_int, [vp, i32, vp, i64, C.POINTER(i64)]),
    "tmllm_cache_gather": (C.c_int, [vp, i32, i32, vp, vp, vp]),
    "tmllm_cache_decode": (C.c_int, [vp, i32, vp, vp, vp, vp, vp, i32, C.POINTER(DecodeOpts),
                                     vp]),
    "tmllm_cache_prefill": (C.c_int, [vp, i32, vp, vp, vp, i64, vp, i32, C.POINTER(DecodeOpts),
                                      vp]),
}

_lib = None
_lock = threading.Lock()


def load():
    """Loads the C-ABI library (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m rustllm_b200.build` "
                "(there is no CPU fallback)")
        lib = C.CDLL(LIB_PATH)
        for name, (res, args) in _PROTOS.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def last_error_fields() -> ErrorFields:
    """The calling thread's ``tmllm_error_fields`` record."""
    f = ErrorFields()
    load().tmllm_last_error_fields(C.byref(f))
    return f


def check(rc: int) -> None:
    """Raises the TinyError subclass for a non-zero status, with the fields of the
    structured variants (PositionOutOfRange, ShapeMismatch) taken from the library."""
    if rc == 0:
        return
    lib = load()
    msg = lib.tmllm_last_error().decode(errors="replace")
    name = lib.tmllm_status_name(rc).decode()
    cls = _BY_STATUS.get(rc, TinyError)
    text = f"{name}: {msg}"
    f = last_error_fields()
    if cls is PositionOutOfRange and f.status == rc:
        raise PositionOutOfRange(text, rc, start_pos=f.start_pos, seq_len=f.seq_len,
                                 max_seq_len=f.max_seq_len)
    if cls is ShapeMismatch and f.status == rc:
        raise ShapeMismatch(text, rc, left=list(f.left[: f.left_rank]),
                            right=list(f.right[: f.right_rank]))
    raise cls(text, rc)


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args))
