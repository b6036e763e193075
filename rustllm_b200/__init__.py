"""rustllm_b200 — B200 (sm_100a) implementation of RustLLM's per-layer KV-cache decode path.

The compute lives in ``libtmllm_b200.so`` (C ABI: ``include/tmllm.h``); this package is the
host-side mirror of the reference's Rust call surface on torch CUDA tensors.
"""
from ._lib import (DeviceError, DeviceTimeout, InvalidArgument, InvalidDimension, InvalidShape,
                   IoError, MissingWeight, ModelFormat, NonContiguousTensor, NotReserved,
                   OutOfBlocks, PositionOutOfRange, ShapeMismatch, TinyError, UnsupportedDType,
                   load)
from .attention import (DecodeWorkspace, auto_splits, gqa_decode, gqa_prefill, merge_lse,
                        paged_kv_from_tensors, prefill_status)
from .kv_cache import KvCache, LayerKvCache, PagedKvCache
from .tensor_ops import (attention_core, attention_scale_mask, batched_matmul, concat_sequence,
                         gqa_pv_matmul, gqa_qk_matmul, kv_cache_write, repeat_kv, rope,
                         rope_tables, softmax_last_dim)

__all__ = [
    "TinyError", "InvalidArgument", "InvalidShape", "ShapeMismatch", "InvalidDimension",
    "UnsupportedDType", "NonContiguousTensor", "PositionOutOfRange", "ModelFormat",
    "DeviceError", "OutOfBlocks", "DeviceTimeout", "NotReserved", "IoError", "MissingWeight",
    "load",
    "DecodeWorkspace", "auto_splits", "gqa_decode", "gqa_prefill", "merge_lse",
    "paged_kv_from_tensors", "prefill_status",
    "KvCache", "LayerKvCache", "PagedKvCache",
    "attention_core", "attention_scale_mask", "batched_matmul", "concat_sequence",
    "gqa_pv_matmul", "gqa_qk_matmul", "kv_cache_write", "repeat_kv", "rope", "rope_tables",
    "softmax_last_dim",
]
