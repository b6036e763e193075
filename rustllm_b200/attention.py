"""The fused decode-attention entry points on torch tensors.

``gqa_decode`` is the stateless form of the hot path (``tmllm_gqa_decode``): one query
token per sequence against a block-paged cache described by a ``PagedKV`` view, with the
new token's K/V appended inside the same kernel.  ``merge_lse`` combines partial results
of a sequence split across GPUs.  ``DecodeWorkspace`` owns the split-K scratch.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from ._lib import DecodeOpts, PagedKV, call
from .tensor_ops import dtype_code, on_device, stream_ptr


class DecodeWorkspace:
    """Zeroed split-K scratch for ``gqa_decode`` (partials plus the per-(seq, kv head)
    tickets of the last-CTA merge).  Every successful call leaves it ready for the next."""

    def __init__(self, num_seqs: int, q_heads: int, kv_heads: int, head_dim: int,
                 num_splits: int = 0, device=None):
        nbytes = _lib.load().tmllm_decode_workspace_bytes(num_seqs, q_heads, kv_heads,
                                                          head_dim, num_splits)
        if nbytes == 0:
            raise _lib.InvalidShape("decode workspace dimensions must be positive")
        self.buf = torch.zeros(nbytes, dtype=torch.uint8, device=device or "cuda")
        self.nbytes = nbytes

    @property
    def ptr(self) -> int:
        return self.buf.data_ptr()


def auto_splits(num_seqs: int, kv_heads: int, max_len: int) -> int:
    return _lib.load().tmllm_decode_auto_splits(num_seqs, kv_heads, max_len)


def gqa_decode(kv: PagedKV, q: torch.Tensor, k_new: torch.Tensor | None,
               v_new: torch.Tensor | None, workspace: DecodeWorkspace, *,
               out: torch.Tensor | None = None, out_dtype: torch.dtype | None = None,
               lse: torch.Tensor | None = None, scale: float = 0.0, num_splits: int = 0,
               max_len_hint: int = 0, rope=None, rope_pos_offset: int = 0,
               variant: int = 0) -> torch.Tensor:
    """Fused KV-append + GQA decode attention (``tmllm_gqa_decode``).

    q [num_seqs, Hq, D]; k_new, v_new [num_seqs, Hkv, D] or both None; out
    [num_seqs, Hq, D] in ``out_dtype`` (default: q's dtype); lse [num_seqs, Hq] F32."""
    on_device(q.device, q, k_new, v_new, out, lse, rope)
    if out is None:
        out = torch.empty(q.shape, dtype=out_dtype or q.dtype, device=q.device)
    if out.dtype not in (q.dtype, torch.float32) or out.shape != q.shape:
        raise _lib.InvalidArgument("out must be [num_seqs, Hq, D] in the cache dtype or F32")
    opts = DecodeOpts(scale=scale, num_splits=num_splits, out_f32=int(out.dtype == torch.float32),
                      rope_pos_offset=rope_pos_offset, max_len_hint=max_len_hint,
                      variant=variant)
    if rope is not None:
        cos, sin = rope
        opts.rope_cos, opts.rope_sin, opts.rope_len = cos.data_ptr(), sin.data_ptr(), cos.shape[0]
    call("tmllm_gqa_decode", C.byref(kv), q.data_ptr(),
         k_new.data_ptr() if k_new is not None else None,
         v_new.data_ptr() if v_new is not None else None, out.data_ptr(),
         lse.data_ptr() if lse is not None else None, q.shape[1], C.byref(opts),
         workspace.ptr, workspace.nbytes, stream_ptr(q.device))
    return out


def merge_lse(parts_o: torch.Tensor, parts_lse: torch.Tensor, *, out: torch.Tensor | None = None,
              out_dtype: torch.dtype = torch.float32, out_lse: torch.Tensor | None = None):
    """Log-sum-exp merge: parts_o [n, rows, D] F32 (normalised), parts_lse [n, rows] F32."""
    on_device(parts_o.device, parts_o, parts_lse, out, out_lse)
    n, rows, d = parts_o.shape
    if out is None:
        out = torch.empty((rows, d), dtype=out_dtype, device=parts_o.device)
    call("tmllm_merge_lse", parts_o.data_ptr(), parts_lse.data_ptr(), n, rows, d,
         parts_o.stride(0), parts_lse.stride(0), out.data_ptr(), dtype_code(out.dtype),
         out_lse.data_ptr() if out_lse is not None else None, stream_ptr(parts_o.device))
    return out


def merge_packed(parts: torch.Tensor, rows: int, head_dim: int, *, out: torch.Tensor,
                 out_lse: torch.Tensor | None = None) -> torch.Tensor:
    """Merge parts packed as [n, rows*head_dim + rows] F32 (output rows, then lse)."""
    n, width = parts.shape
    if width != rows * head_dim + rows or parts.dtype != torch.float32:
        raise _lib.InvalidShape("packed parts must be [n, rows*head_dim + rows] F32")
    base = parts.data_ptr()
    call("tmllm_merge_lse", base, base + rows * head_dim * 4, n, rows, head_dim, width, width,
         out.data_ptr(), dtype_code(out.dtype),
         out_lse.data_ptr() if out_lse is not None else None, stream_ptr(parts.device))
    return out


def _row_stride(t: torch.Tensor, heads: int, d: int, what: str) -> int:
    """Elements between consecutive rows of a [rows, heads, D] tensor whose last two
    dimensions are packed (a view into a wider fused projection is fine)."""
    if t.dim() != 3 or t.shape[1] != heads or t.shape[2] != d:
        raise _lib.ModelFormat(f"{what} must be [rows, {heads}, {d}], got {list(t.shape)}")
    if t.stride(2) != 1 or t.stride(1) != d:
        raise _lib.NonContiguousTensor(f"{what} heads must be packed rows of {d} elements")
    return t.stride(0)


def gqa_prefill(kv: PagedKV, q: torch.Tensor, k_new: torch.Tensor | None,
                v_new: torch.Tensor | None, *,
                q_start: torch.Tensor | None = None, rows_per_seq: int = 0, max_rows: int = 0,
                out: torch.Tensor | None = None, out_dtype: torch.dtype | None = None,
                scale: float = 0.0, rope=None, rope_pos_offset: int = 0,
                variant: int = 0) -> torch.Tensor:
    """Fused KV-append + causal prefill attention (``tmllm_gqa_prefill``).

    q [rows, Hq, D], k_new / v_new [rows, Hkv, D] (row-strided views allowed), rows grouped
    by sequence: ``q_start`` int32 [num_seqs + 1] row offsets on the device, or None with
    ``rows_per_seq`` rows per sequence.  Row i of sequence s is appended at seq_lens[s] + i
    and attends keys [0, seq_lens[s] + i]; with k_new = v_new = None nothing is appended
    (those positions already hold the rows).  Returns out [rows, Hq, D]."""
    on_device(q.device, q, k_new, v_new, out, q_start, rope)
    rows, hq, d = q.shape
    hkv = kv.num_kv_heads
    qs = _row_stride(q, hq, d, "q")
    ks = 0
    if (k_new is None) != (v_new is None):
        raise _lib.InvalidArgument("k_new and v_new must both be given or both be None")
    if k_new is not None:
        ks = _row_stride(k_new, hkv, d, "k_new")
        if (_row_stride(v_new, hkv, d, "v_new") != ks or k_new.shape[0] != rows
                or v_new.shape[0] != rows):
            raise _lib.ShapeMismatch("k_new and v_new must have q's rows and the same row stride",
                                     left=k_new.shape, right=v_new.shape)
    if out is None:
        out = torch.empty((rows, hq, d), dtype=out_dtype or q.dtype, device=q.device)
    if (out.dtype not in (q.dtype, torch.float32) or tuple(out.shape) != (rows, hq, d)
            or not out.is_contiguous()):
        raise _lib.InvalidArgument("out must be a contiguous [rows, Hq, D] tensor in the cache "
                                   "dtype or F32")
    opts = DecodeOpts(scale=scale, out_f32=int(out.dtype == torch.float32),
                      rope_pos_offset=rope_pos_offset, variant=variant, q_seq_stride=qs,
                      kv_seq_stride=ks)
    if rope is not None:
        cos, sin = rope
        opts.rope_cos, opts.rope_sin, opts.rope_len = cos.data_ptr(), sin.data_ptr(), cos.shape[0]
    if q_start is not None:
        if q_start.dtype != torch.int32 or q_start.numel() != kv.num_seqs + 1:
            raise _lib.InvalidArgument("q_start must be int32 [num_seqs + 1]")
        if max_rows <= 0:
            max_rows = int((q_start[1:] - q_start[:-1]).max())
        qp = q_start.data_ptr()
    else:
        if rows_per_seq * kv.num_seqs != rows:
            raise _lib.ShapeMismatch(f"{rows} rows are not {kv.num_seqs} x {rows_per_seq}",
                                     left=[rows], right=[kv.num_seqs * rows_per_seq])
        qp = None
    call("tmllm_gqa_prefill", C.byref(kv), q.data_ptr(),
         k_new.data_ptr() if k_new is not None else None,
         v_new.data_ptr() if v_new is not None else None, qp,
         rows_per_seq, max_rows, rows, out.data_ptr(), hq, C.byref(opts), stream_ptr(q.device))
    return out


def prefill_status() -> int:
    """Reads and clears the prefill kernel's wait status (0, or the TMLLM_TIMEOUT code)."""
    st = C.c_int32()
    call("tmllm_prefill_status", C.byref(st))
    return st.value


def paged_kv_from_tensors(k_arena: torch.Tensor, v_arena: torch.Tensor,
                          block_table: torch.Tensor, seq_lens: torch.Tensor) -> PagedKV:
    """A ``PagedKV`` over caller-owned tensors: arenas [num_blocks, Hkv, block_size, D],
    block_table int32 [num_seqs, max_blocks], seq_lens int32 [num_seqs]."""
    if block_table.dtype != torch.int32 or seq_lens.dtype != torch.int32:
        raise _lib.UnsupportedDType("block table and lengths must be int32")
    nb, hkv, bs, d = k_arena.shape
    return PagedKV(k_cache=k_arena.data_ptr(), v_cache=v_arena.data_ptr(),
                   block_table=block_table.data_ptr(), seq_lens=seq_lens.data_ptr(),
                   num_blocks=nb, num_seqs=block_table.shape[0], num_kv_heads=hkv, head_dim=d,
                   block_size=bs, max_blocks_per_seq=block_table.shape[1],
                   dtype=dtype_code(k_arena.dtype))
