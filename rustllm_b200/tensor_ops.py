"""Op-level front end: the reference's ``Tensor`` operators on torch CUDA tensors.

Each function validates like its reference counterpart, then calls one C-ABI entry point
of ``libtmllm_b200.so`` on the current CUDA stream.  torch supplies device memory and the
stream only; the arithmetic runs in this package's CUDA kernels.
"""
from __future__ import annotations

import math

import torch

from . import _lib
from ._lib import F16, F32, call

_DTYPES = {torch.float32: F32, torch.float16: F16}


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPES[dtype]
    except KeyError:
        raise _lib.UnsupportedDType(f"unsupported dtype {dtype} (F32 and F16 only)") from None


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _on_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if not t.is_cuda:
            raise _lib.InvalidArgument("tensors must live on a CUDA device")


def on_device(device: torch.device, *ts) -> None:
    """Every given tensor (None entries and (cos, sin) pairs allowed) lives on ``device``:
    a host or foreign-device pointer must never reach a kernel."""
    for t in ts:
        if t is None:
            continue
        if isinstance(t, (tuple, list)):
            on_device(device, *t)
            continue
        if not t.is_cuda or t.device != device:
            raise _lib.InvalidArgument(f"tensors must live on {device}, got one on {t.device}")


def _same_dtype(op: str, a: torch.Tensor, b: torch.Tensor) -> None:
    if a.dtype != b.dtype:
        raise _lib.UnsupportedDType(f"{op} dtype mismatch: {a.dtype} vs {b.dtype}")


def kv_cache_write(cache: torch.Tensor, source: torch.Tensor, start: int) -> None:
    """kv_cache_write_{f32,f16} (src/ops/kv_cache_write.rs:9-141): cache [1,H,max,D],
    source [1,H,S,D]; writes positions [start, start+S) in place."""
    _on_cuda(cache, source)
    _same_dtype("kv_cache_write", cache, source)
    if (cache.dim() != 4 or source.dim() != 4 or cache.shape[0] != 1 or source.shape[0] != 1
            or cache.shape[1] != source.shape[1] or cache.shape[3] != source.shape[3]):
        raise _lib.InvalidShape("invalid KV cache write shape")
    if not cache.is_contiguous():
        raise _lib.NonContiguousTensor("KV cache must be contiguous")
    source = source.contiguous()
    _, h, max_seq, d = cache.shape
    call("tmllm_kv_cache_write", dtype_code(cache.dtype), cache.data_ptr(), source.data_ptr(),
         h, max_seq, d, start, source.shape[2], stream_ptr(cache.device))


def concat_sequence(left: torch.Tensor, right: torch.Tensor) -> torch.Tensor:
    """concat_sequence_f32 (src/ops/concat_sequence.rs:13-115), F16 too: [B,H,Sl,D] ++
    [B,H,Sr,D] along the sequence axis."""
    _on_cuda(left, right)
    _same_dtype("concat_sequence", left, right)
    if left.dim() != 4 or right.dim() != 4:
        raise _lib.ModelFormat("concat_sequence expects rank-4 tensors")
    b, h, sl, d = left.shape
    if right.shape[0] != b or right.shape[1] != h or right.shape[3] != d:
        raise _lib.ModelFormat(
            f"concat_sequence incompatible shapes: {list(left.shape)} and {list(right.shape)}")
    left, right = left.contiguous(), right.contiguous()
    out = torch.empty((b, h, sl + right.shape[2], d), dtype=left.dtype, device=left.device)
    call("tmllm_concat_sequence", dtype_code(left.dtype), left.data_ptr(), right.data_ptr(),
         out.data_ptr(), b, h, sl, right.shape[2], d, stream_ptr(left.device))
    return out


def repeat_kv(x: torch.Tensor, repeats: int) -> torch.Tensor:
    """Tensor::repeat_kv (src/tensor/repeat_kv.rs:13-81): [B,Hkv,S,D] -> [B,Hkv*r,S,D]."""
    _on_cuda(x)
    if x.dim() != 4:
        raise _lib.ModelFormat(f"repeat_kv expects [B, KVH, S, D], got {list(x.shape)}")
    if repeats == 0:
        raise _lib.ModelFormat("repeat_kv repeats must be greater than zero")
    if repeats == 1:  # repeat_kv.rs:27-29 returns the input itself
        return x
    x = x.contiguous()
    b, h, s, d = x.shape
    out = torch.empty((b, h * repeats, s, d), dtype=x.dtype, device=x.device)
    call("tmllm_repeat_kv", dtype_code(x.dtype), x.data_ptr(), out.data_ptr(), b, h, s, d,
         repeats, stream_ptr(x.device))
    return out


def _kv_view(k: torch.Tensor, kv_len: int | None):
    """(capacity, length) of a [B,Hkv,cap,D] cache buffer read for kv_len rows."""
    cap = k.shape[2]
    return cap, cap if kv_len is None else kv_len


def gqa_qk_matmul(q: torch.Tensor, k: torch.Tensor, kv_len: int | None = None) -> torch.Tensor:
    """Tensor::gqa_qk_matmul (src/tensor/gqa_matmul.rs:16-62): Q [B,Hq,S,D] x K^T, K read
    as [B,Hkv,cap,D] for its first kv_len rows (a cache's narrow view)."""
    _same_dtype("GQA QK", q, k)
    if q.dim() != 4 or k.dim() != 4:
        raise _lib.ModelFormat(f"GQA QK expects Q [B,QH,Q,D] and K [B,KVH,K,D], got "
                               f"{list(q.shape)} and {list(k.shape)}")
    b, hq, s, d = q.shape
    if k.shape[0] != b or k.shape[3] != d:  # gqa_matmul.rs:111-116
        raise _lib.ShapeMismatch(f"shape mismatch: left={list(q.shape)}, right={list(k.shape)}",
                                 left=q.shape, right=k.shape)
    _on_cuda(q, k)
    cap, kv_len = _kv_view(k, kv_len)
    q, k = q.contiguous(), k.contiguous()
    out = torch.empty((b, hq, s, kv_len), dtype=q.dtype, device=q.device)
    call("tmllm_gqa_qk", dtype_code(q.dtype), q.data_ptr(), k.data_ptr(), out.data_ptr(), b,
         hq, k.shape[1], s, kv_len, d, cap, stream_ptr(q.device))
    return out


def gqa_pv_matmul(probs: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """Tensor::gqa_pv_matmul (src/tensor/gqa_matmul.rs:65-105): P [B,Hq,S,L] x V, V read
    as [B,Hkv,cap,D] for its first L rows."""
    _same_dtype("GQA PV", probs, v)
    if probs.dim() != 4 or v.dim() != 4:
        raise _lib.ModelFormat(f"GQA PV expects P [B,QH,Q,K] and V [B,KVH,K,D], got "
                               f"{list(probs.shape)} and {list(v.shape)}")
    b, hq, s, kv_len = probs.shape
    if v.shape[0] != b or v.shape[2] < kv_len:  # gqa_matmul.rs:130-135
        raise _lib.ShapeMismatch(
            f"shape mismatch: left={list(probs.shape)}, right={list(v.shape)}",
            left=probs.shape, right=v.shape)
    _on_cuda(probs, v)
    probs, v = probs.contiguous(), v.contiguous()
    d = v.shape[3]
    out = torch.empty((b, hq, s, d), dtype=probs.dtype, device=probs.device)
    call("tmllm_gqa_pv", dtype_code(probs.dtype), probs.data_ptr(), v.data_ptr(),
         out.data_ptr(), b, hq, v.shape[1], s, kv_len, d, v.shape[2], stream_ptr(v.device))
    return out


def attention_scale_mask(scores: torch.Tensor, scale: float, start: int) -> torch.Tensor:
    """Tensor::attention_scale_mask (src/tensor/tensor.rs:604-668)."""
    _on_cuda(scores)
    if scores.dim() < 2:
        raise _lib.InvalidDimension(f"attention scores require rank >= 2, got rank {scores.dim()}")
    scores = scores.contiguous()
    out = torch.empty_like(scores)
    call("tmllm_attention_scale_mask", dtype_code(scores.dtype), scores.data_ptr(),
         out.data_ptr(), scores.numel(), scores.shape[-2], scores.shape[-1], start, scale,
         stream_ptr(scores.device))
    return out


def softmax_last_dim(x: torch.Tensor) -> torch.Tensor:
    """Tensor::softmax_last_dim (src/tensor/tensor.rs:458-495)."""
    _on_cuda(x)
    if x.dim() == 0:
        raise _lib.InvalidDimension("Softmax requires at least one dimension")
    x = x.contiguous()
    out = torch.empty_like(x)
    width = x.shape[-1]
    call("tmllm_softmax_last_dim", dtype_code(x.dtype), x.data_ptr(), out.data_ptr(),
         x.numel() // max(width, 1), width, stream_ptr(x.device))
    return out


def batched_matmul(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Tensor::batched_matmul (src/tensor/tensor.rs:497-602)."""
    _same_dtype("batched matmul", a, b)
    if a.dim() < 3:
        raise _lib.InvalidDimension(f"batched matmul requires rank >= 3, left rank is {a.dim()}")
    if b.dim() != a.dim():
        raise _lib.InvalidDimension(
            f"batched matmul requires tensors with equal rank, got {a.dim()} and {b.dim()}")
    if a.shape[:-2] != b.shape[:-2] or a.shape[-1] != b.shape[-2]:  # tensor.rs:541-563
        raise _lib.ShapeMismatch(f"shape mismatch: left={list(a.shape)}, right={list(b.shape)}",
                                 left=a.shape, right=b.shape)
    _on_cuda(a, b)
    a, b = a.contiguous(), b.contiguous()
    m, k, n = a.shape[-2], a.shape[-1], b.shape[-1]
    batch = math.prod(a.shape[:-2])
    out = torch.empty(a.shape[:-2] + (m, n), dtype=a.dtype, device=a.device)
    call("tmllm_batched_matmul", dtype_code(a.dtype), a.data_ptr(), b.data_ptr(), out.data_ptr(),
         batch, m, k, n, stream_ptr(a.device))
    return out


def rope_tables(head_dim: int, max_seq_len: int, theta: float, device=None):
    """RotaryEmbedding::new's F32 tables (src/nn/rope.rs:44-62), built on the host as the
    reference does and copied to ``device``."""
    half = head_dim // 2
    cos = torch.empty((max_seq_len, half), dtype=torch.float32)
    sin = torch.empty((max_seq_len, half), dtype=torch.float32)
    call("tmllm_rope_tables", cos.data_ptr(), sin.data_ptr(), head_dim, max_seq_len, theta)
    if device is not None:
        cos, sin = cos.to(device), sin.to(device)
    return cos, sin


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, start: int) -> torch.Tensor:
    """rope_encode (src/ops/rope.rs:303-370) on x [..., seq, head_dim]."""
    _on_cuda(x, cos, sin)
    if x.dim() < 2:
        raise _lib.InvalidDimension(f"RoPE expects [..., sequence, head_dim], got rank {x.dim()}")
    if cos.dtype != torch.float32 or sin.dtype != torch.float32:
        raise _lib.UnsupportedDType("RoPE requires F32 cos/sin tables")
    x = x.contiguous()
    seq, d = x.shape[-2], x.shape[-1]
    if cos.dim() != 2 or cos.shape != sin.shape or cos.shape[1] != d // 2:
        raise _lib.InvalidShape("RoPE cos/sin table shape or position range is invalid")
    out = torch.empty_like(x)
    rows = x.numel() // max(seq * d, 1)
    call("tmllm_rope", dtype_code(x.dtype), x.data_ptr(), out.data_ptr(), cos.data_ptr(),
         sin.data_ptr(), cos.shape[0], rows, seq, d, start, stream_ptr(x.device))
    return out


def attention_core(q: torch.Tensor, key: torch.Tensor, value: torch.Tensor, start_pos: int,
                   kv_len: int | None = None) -> torch.Tensor:
    """SelfAttention::attention_core_encode (src/nn/attention.rs:216-247), op by op:
    QK -> scale/mask(1/sqrt(D), start_pos) -> softmax -> PV.  key/value [B,Hkv,cap,D] are
    read for kv_len rows.  The reference's MHA branch (Hq == Hkv) uses batched_matmul with
    a materialised K^T; its sums run over the same index in the same order as the GQA
    kernels with a group of one, so both branches go through the GQA kernels here."""
    d = q.shape[-1]
    _, kv_len = _kv_view(key, kv_len)
    scores = gqa_qk_matmul(q, key, kv_len)
    scores = attention_scale_mask(scores, 1.0 / math.sqrt(d), start_pos)
    probs = softmax_last_dim(scores)
    return gqa_pv_matmul(probs, value)
