"""Llama-family decoder around the fused decode path: the callers either side of it.

Mirrors the reference's cached forward (src/model/transformer/cache.rs:25-82,
src/nn/transformer_block.rs:128-159, src/nn/attention.rs:269-333, src/nn/mlp.rs) for a
batch of sequences, one decode token per sequence per step:

    embedding -> for each layer: [residual add +] RMSNorm -> fused QKV GEMM ->
    fused RoPE + KV append + GQA attention -> O GEMM -> residual add + RMSNorm ->
    fused gate/up GEMM -> SwiGLU -> down GEMM -> ... -> final norm -> lm_head -> argmax

Every piece is one of this package's CUDA kernels.  With at most 64 sequences (F16) a
decode step's layer projections run in ``linear`` (tmllm_linear), which folds the RMSNorm
into the projection that reads it, SwiGLU into the gate/up projection and each residual add
into the projection that produces it, so a layer is five launches:

    x -> [norm + QKV] -> attention -> [O + residual -> x] -> [norm + gate/up + SwiGLU]
      -> [down + residual -> x]

Prompts and larger batches use plain cuBLAS GEMMs (torch.matmul) between the norm, SwiGLU
and attention kernels.  With up to 16 sequences (F16) the step ends in one launch: the final
RMSNorm, the vocabulary head and the greedy pick (``lm_head``, tmllm_lm_head); larger
batches use a cuBLAS head between the norm and argmax kernels.  Weights keep the
reference's [in, out] layout (src/nn/linear.rs:26-27); Q, K, V and gate/up are concatenated
along `out` so each
pair/triple is one projection, and the attention reads q, k, v in place from the fused
output through per-sequence strides.  A whole step is captured into one CUDA graph
(``GraphedDecoder``).
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import DecodeOpts, call
from .kv_cache import PagedKvCache
from .tensor_ops import dtype_code, rope_tables, stream_ptr


@dataclass(frozen=True)
class ModelConfig:
    """src/model/config.rs:8-22."""

    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_layers: int
    num_heads: int
    num_kv_heads: int
    max_seq_len: int
    rms_norm_eps: float
    rope_theta: float

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_heads

    def validate(self) -> None:
        """src/model/config.rs:24-105, same checks, order, error kinds and messages."""
        for value, what in ((self.vocab_size, "vocab size"), (self.hidden_size, "hidden size"),
                            (self.intermediate_size, "intermediate size"),
                            (self.num_layers, "number of layers"),
                            (self.num_heads, "number of attention heads"),
                            (self.num_kv_heads, "number of key/value attention heads")):
            if value <= 0:
                raise _lib.InvalidShape(f"{what} cannot be zero")
        if self.hidden_size % self.num_heads:
            raise _lib.InvalidShape(f"hidden size {self.hidden_size} must be divisible by "
                                    f"num_heads {self.num_heads}")
        if self.head_dim % 2:
            raise _lib.InvalidShape(f"RoPE requires an even head dimension, got {self.head_dim}")
        if self.max_seq_len <= 0:
            raise _lib.InvalidShape("max sequence length cannot be zero")
        if not math.isfinite(self.rms_norm_eps) or self.rms_norm_eps <= 0:
            raise _lib.InvalidShape("RMSNorm epsilon must be positive and finite, got "
                                    f"{self.rms_norm_eps}")
        if not math.isfinite(self.rope_theta) or self.rope_theta <= 0:
            raise _lib.InvalidShape(f"RoPE theta must be positive and finite, got {self.rope_theta}")
        if self.num_heads % self.num_kv_heads:
            raise _lib.ModelFormat(f"num_heads {self.num_heads} must be divisible by "
                                   f"num_kv_heads {self.num_kv_heads}")

    def weight_params(self) -> int:
        h, i, d = self.hidden_size, self.intermediate_size, self.head_dim
        per_layer = (h * (self.num_heads + 2 * self.num_kv_heads) * d + self.num_heads * d * h
                     + 3 * h * i + 2 * h)
        return self.num_layers * per_layer + 2 * self.vocab_size * h + h


# BASELINE.json configs 2, 3 and 5.
PRESETS = {
    "smollm2-135m": ModelConfig(49152, 576, 1536, 30, 9, 3, 2048, 1e-5, 100000.0),
    "smollm2-360m": ModelConfig(49152, 960, 2560, 32, 15, 5, 2304, 1e-5, 100000.0),
    "tinystories-110m": ModelConfig(32000, 768, 2048, 12, 12, 12, 1024, 1e-5, 10000.0),
}


LINEAR_MAX_ROWS = 64
# Batches up to this many sequences run the fused projections in a decode step (every batch
# the kernel takes: at 64 rows the fused step measured the same as cuBLAS GEMMs with the
# separate norm and SwiGLU kernels, 1.828 vs 1.827 ms for config 3, with fewer launches).
FUSED_STEP_MAX_ROWS = LINEAR_MAX_ROWS
LINEAR_OVERLAP = 1  # TMLLM_LINEAR_OVERLAP
DECODE_OVERLAP = 1  # TMLLM_DECODE_OVERLAP


def linear_status() -> int:
    """Reads and clears the status word of the projection kernels (0, or TMLLM_TIMEOUT
    after an expired device-side wait)."""
    v = C.c_int32(0)
    call("tmllm_linear_status", C.byref(v))
    return int(v.value)


def linear_stats(n: int, *, device=None) -> torch.Tensor:
    """Device buffer for the row statistics of an [rows, n] projection output."""
    nbytes = _lib.load().tmllm_linear_stats_bytes(n)
    return torch.empty(int(nbytes) // 4, dtype=torch.float32, device=device)


def linear(x: torch.Tensor, w: torch.Tensor, *, norm_weight: torch.Tensor | None = None,
           eps: float = 1e-5, residual: torch.Tensor | None = None, swiglu: bool = False,
           out: torch.Tensor | None = None, stats_in: torch.Tensor | None = None,
           stats_out: torch.Tensor | None = None, overlap: bool = False) -> torch.Tensor:
    """out = x · w for x [rows <= 64, k], w [k, n] (F16, src/nn/linear.rs:105-170), with
    optional RMSNorm of x (norm_weight, kernels/rmsnorm.metal), SwiGLU over w = [gate | up]
    [k, 2n] (kernels/silu.metal) or a residual add (kernels/vector_add.metal) fused in.
    ``stats_out`` (``linear_stats(n)``) receives the row statistics of ``out``; a later call
    that normalises ``out`` takes them as ``stats_in`` instead of re-reading the rows.
    ``overlap`` lets the launch start while the previous work on the stream drains (the
    caller promises that work does not write ``w``)."""
    if x.dim() != 2 or w.dim() != 2:
        raise _lib.ModelFormat(f"Linear expects rank-2 input, got {tuple(x.shape)}")
    given = [t for t in (x, w, norm_weight, residual, out, stats_in, stats_out) if t is not None]
    if any(not t.is_cuda or t.device != x.device for t in given):
        raise _lib.InvalidArgument("linear tensors must live on one CUDA device")
    rows, k = x.shape
    if w.shape[0] != k:
        raise _lib.ModelFormat(f"Linear input feature mismatch: expected {w.shape[0]}, got {k}")
    if x.dtype != torch.float16 or w.dtype != torch.float16:
        raise _lib.UnsupportedDType(f"linear takes F16 input and weight, got {x.dtype}, {w.dtype}")
    n = w.shape[1] // 2 if swiglu else w.shape[1]
    if x.stride(1) != 1 or w.stride(1) != 1:
        raise _lib.NonContiguousTensor("linear needs unit column stride")
    if out is None:
        out = torch.empty((rows, n), dtype=x.dtype, device=x.device)
    for st, cols in ((stats_in, k), (stats_out, n)):
        if st is not None and (st.dtype != torch.float32 or
                               st.numel() * 4 < _lib.load().tmllm_linear_stats_bytes(cols)):
            raise _lib.InvalidArgument("row statistics need a linear_stats buffer")
    call("tmllm_linear", x.data_ptr(), x.stride(0),
         norm_weight.data_ptr() if norm_weight is not None else None,
         stats_in.data_ptr() if stats_in is not None else None, eps, w.data_ptr(),
         w.stride(0), out.data_ptr(), out.stride(0),
         residual.data_ptr() if residual is not None else None,
         residual.stride(0) if residual is not None else 0,
         stats_out.data_ptr() if stats_out is not None else None, rows, k, n, int(swiglu),
         LINEAR_OVERLAP if overlap else 0, stream_ptr(x.device))
    return out


HEAD_MAX_ROWS = 64
HEAD_STEP_MAX_ROWS = 16  # decode steps of up to this many sequences use lm_head
_HEAD_SMEM_MAX = 227 * 1024


def head_fits(rows: int, k: int, n: int) -> bool:
    """Whether ``lm_head`` takes these sizes: at most 64 rows whose staged copy (in 16-row
    tiles; K rounded up to a whole stage of 128 weight rows with up to 32 rows, 64 above,
    plus a 16-byte pad per row) and the norm weight fit beside the shallowest weight ring
    (three 16 KB stages on a 1024-byte boundary) in shared memory, K and N in whole 16-byte
    chunks."""
    mt = (rows + 15) // 16
    kr = 128 if mt <= 2 else 64  # weight rows a stage
    kp = (k + kr - 1) // kr * kr
    smem = 4 * 64 * 8 + 2 * 12 * 8 + 64 + mt * 16 * (2 * kp + 16) + 2 * kp + 1024 + 3 * 16384
    return 0 < rows <= HEAD_MAX_ROWS and k % 8 == 0 and n % 8 == 0 and smem <= _HEAD_SMEM_MAX


def head_workspace(*, device=None) -> torch.Tensor:
    """Zeroed device workspace for the argmax of ``lm_head`` (each call leaves it zeroed)."""
    nbytes = int(_lib.load().tmllm_lm_head_workspace_bytes())
    return torch.zeros(nbytes // 8, dtype=torch.int64, device=device)


def lm_head(x: torch.Tensor, w: torch.Tensor, *, norm_weight: torch.Tensor | None = None,
            eps: float = 1e-5, residual: torch.Tensor | None = None,
            logits: torch.Tensor | None = None, ids: torch.Tensor | None = None,
            workspace: torch.Tensor | None = None, overlap: bool = False) -> torch.Tensor:
    """The end of a decode step in one launch (transformer/cache.rs:72-77 and
    generation/sampler.rs:79-88): logits [rows <= 64, n] = half(rmsnorm(x [+ residual]) · w)
    for F16 x [rows, k] and w [k, n]; with ``ids`` (int32 [rows]) also the greedy token of
    every row, as ``tmllm_argmax`` picks it from the stored logits (``workspace`` from
    ``head_workspace``).  ``overlap`` as for ``linear``."""
    if x.dim() != 2 or w.dim() != 2:
        raise _lib.ModelFormat(f"Linear expects rank-2 input, got {tuple(x.shape)}")
    given = [t for t in (x, w, norm_weight, residual, logits, ids, workspace) if t is not None]
    if any(not t.is_cuda or t.device != x.device for t in given):
        raise _lib.InvalidArgument("lm_head tensors must live on one CUDA device")
    rows, k = x.shape
    if w.shape[0] != k:
        raise _lib.ModelFormat(f"Linear input feature mismatch: expected {w.shape[0]}, got {k}")
    if x.dtype != torch.float16 or w.dtype != torch.float16:
        raise _lib.UnsupportedDType(f"lm_head takes F16 input and weight, got {x.dtype}, {w.dtype}")
    if residual is not None and (residual.shape != x.shape or residual.dtype != x.dtype):
        raise _lib.ShapeMismatch("lm_head residual must match x", left=list(x.shape),
                                 right=list(residual.shape))
    if x.stride(1) != 1 or w.stride(1) != 1 or (residual is not None and residual.stride(1) != 1):
        raise _lib.NonContiguousTensor("lm_head needs unit column stride")
    n = w.shape[1]
    if logits is None:
        logits = torch.empty((rows, n), dtype=x.dtype, device=x.device)
    if ids is not None:
        if ids.dtype != torch.int32 or ids.numel() < rows or not ids.is_contiguous():
            raise _lib.InvalidArgument("lm_head ids must be a contiguous int32 buffer of rows")
        if workspace is None:
            raise _lib.InvalidArgument("lm_head argmax needs a head_workspace buffer")
    call("tmllm_lm_head", x.data_ptr(), x.stride(0),
         residual.data_ptr() if residual is not None else None,
         residual.stride(0) if residual is not None else 0,
         norm_weight.data_ptr() if norm_weight is not None else None, eps, w.data_ptr(),
         w.stride(0), logits.data_ptr(), logits.stride(0),
         ids.data_ptr() if ids is not None else None,
         workspace.data_ptr() if workspace is not None else None, rows, k, n,
         LINEAR_OVERLAP if overlap else 0, stream_ptr(x.device))
    return logits


class DecoderWeights:
    """Random-init weights, N(0, std) for every projection and the embedding (the
    BASELINE configs' synthetic models), unit RMSNorm scales, in the model dtype."""

    def __init__(self, cfg: ModelConfig, *, dtype=torch.float16, device=None, seed: int = 0,
                 std: float = 0.02):
        cfg.validate()
        dev = torch.device(device or "cuda")
        g = torch.Generator(device=dev).manual_seed(seed)
        h, i, d = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim
        qkv = (cfg.num_heads + 2 * cfg.num_kv_heads) * d

        def rnd(*shape):
            return (torch.randn(shape, generator=g, device=dev) * std).to(dtype)

        self.embedding = rnd(cfg.vocab_size, h)
        self.layers = []
        for _ in range(cfg.num_layers):
            self.layers.append({
                "attn_norm": torch.ones(h, dtype=dtype, device=dev),
                "wqkv": rnd(h, qkv),
                "wo": rnd(cfg.num_heads * d, h),
                "mlp_norm": torch.ones(h, dtype=dtype, device=dev),
                "wgu": rnd(h, 2 * i),
                "wd": rnd(i, h),
            })
        self.final_norm = torch.ones(h, dtype=dtype, device=dev)
        self.lm_head = rnd(h, cfg.vocab_size)
        self.dtype = dtype

    @classmethod
    def from_weights(cls, cfg: ModelConfig, weights, *, device=None,
                     dtype=None) -> "DecoderWeights":
        """Transformer::from_weights (src/model/transformer.rs:203-318): the reference's
        tensor names and [in, out] shapes, each checked as take_tensor / take_linear do
        (:333-398); q/k/v and gate/up are concatenated along `out` into the fused matrices.
        ``weights`` is a ``rustllm_b200.weights.ModelWeights`` (consumed).  INT8 linears
        (the reference's QuantizedLinear path) are not supported by this decoder."""
        import numpy as np
        cfg.validate()
        dev = torch.device(device or "cuda")
        dtype = dtype or torch.float16
        h, i = cfg.hidden_size, cfg.intermediate_size
        qp, kvp = cfg.num_heads * cfg.head_dim, cfg.num_kv_heads * cfg.head_dim

        def take(name, shape):
            t = weights.take(name)
            if tuple(t.shape) != tuple(shape):
                raise _lib.InvalidShape(f"weight {name} has shape {list(t.shape)}, expected "
                                        f"{list(shape)}")
            if t.data.dtype == np.int8:
                raise _lib.ModelFormat(f"INT8 weight {name}: quantized linear layers are not "
                                       "supported by this decoder")
            return torch.from_numpy(np.ascontiguousarray(t.data)).to(dev, dtype)

        self = cls.__new__(cls)
        self.embedding = take("token_embedding.weight", (cfg.vocab_size, h))
        self.layers = []
        for li in range(cfg.num_layers):
            p = f"layers.{li}"
            wq = take(f"{p}.attention.q_proj.weight", (h, qp))
            wk = take(f"{p}.attention.k_proj.weight", (h, kvp))
            wv = take(f"{p}.attention.v_proj.weight", (h, kvp))
            wo = take(f"{p}.attention.out_proj.weight", (qp, h))
            an = take(f"{p}.attention_norm.weight", (h,))
            mn = take(f"{p}.mlp_norm.weight", (h,))
            wg = take(f"{p}.mlp.gate_proj.weight", (h, i))
            wu = take(f"{p}.mlp.up_proj.weight", (h, i))
            wd = take(f"{p}.mlp.down_proj.weight", (i, h))
            self.layers.append({"attn_norm": an, "wqkv": torch.cat([wq, wk, wv], 1).contiguous(),
                                "wo": wo, "mlp_norm": mn,
                                "wgu": torch.cat([wg, wu], 1).contiguous(), "wd": wd})
        self.final_norm = take("final_norm.weight", (h,))
        self.lm_head = take("lm_head.weight", (h, cfg.vocab_size))
        self.dtype = dtype
        return self

    def to_weights(self, cfg: ModelConfig):
        """The inverse of ``from_weights``: a ModelWeights with the reference's names
        (F16 tensors when the decoder is F16, F32 otherwise), e.g. to write a model.bin."""
        from .weights import ModelWeights
        qp, kvp = cfg.num_heads * cfg.head_dim, cfg.num_kv_heads * cfg.head_dim
        i = cfg.intermediate_size
        out = ModelWeights()
        put = out.insert_f16 if self.dtype == torch.float16 else out.insert_f32

        def add(name, t):
            a = t.detach().cpu()
            put(name, tuple(a.shape), a.numpy())

        add("token_embedding.weight", self.embedding)
        for li, L in enumerate(self.layers):
            p = f"layers.{li}"
            add(f"{p}.attention.q_proj.weight", L["wqkv"][:, :qp])
            add(f"{p}.attention.k_proj.weight", L["wqkv"][:, qp:qp + kvp])
            add(f"{p}.attention.v_proj.weight", L["wqkv"][:, qp + kvp:])
            add(f"{p}.attention.out_proj.weight", L["wo"])
            add(f"{p}.attention_norm.weight", L["attn_norm"])
            add(f"{p}.mlp_norm.weight", L["mlp_norm"])
            add(f"{p}.mlp.gate_proj.weight", L["wgu"][:, :i])
            add(f"{p}.mlp.up_proj.weight", L["wgu"][:, i:])
            add(f"{p}.mlp.down_proj.weight", L["wd"])
        add("final_norm.weight", self.final_norm)
        add("lm_head.weight", self.lm_head)
        return out


class Decoder:
    """Batched greedy decoding for ``num_seqs`` sequences on one GPU."""

    def __init__(self, cfg: ModelConfig, weights: DecoderWeights, num_seqs: int, *,
                 block_size: int = 16, shuffle_seed: int = 0, device=None,
                 max_seq_len: int | None = None):
        self.cfg, self.w, self.B = cfg, weights, num_seqs
        self.device = torch.device(device or "cuda")
        self.dtype = weights.dtype
        self.max_seq_len = max_seq_len or cfg.max_seq_len
        self.cache = PagedKvCache(cfg.num_layers, num_seqs, self.max_seq_len, cfg.num_kv_heads,
                                  cfg.head_dim, dtype=self.dtype, block_size=block_size,
                                  shuffle_seed=shuffle_seed, device=self.device)
        self.rope = rope_tables(cfg.head_dim, self.max_seq_len + 1, cfg.rope_theta,
                                device=self.device)
        B, h, d = num_seqs, cfg.hidden_size, cfg.head_dim
        hq, hkv = cfg.num_heads, cfg.num_kv_heads
        e = dict(dtype=self.dtype, device=self.device)
        self.ids = torch.zeros(B, dtype=torch.int32, device=self.device)
        self.next_ids = torch.zeros(B, dtype=torch.int32, device=self.device)
        self.x = torch.empty((B, h), **e)
        self.hn = torch.empty((B, h), **e)
        self.qkv = torch.empty((B, (hq + 2 * hkv) * d), **e)
        self.attn = torch.empty((B, hq, d), **e)
        self.o = torch.empty((B, h), **e)
        self.gu = torch.empty((B, 2 * cfg.intermediate_size), **e)
        self.act = torch.empty((B, cfg.intermediate_size), **e)
        self.down = torch.empty((B, h), **e)
        self.logits = torch.empty((B, cfg.vocab_size), **e)
        self.bad = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.dt = dtype_code(self.dtype)
        self.max_len_hint = 0
        i = cfg.intermediate_size
        shapes = [(h, (hq + 2 * hkv) * d), (hq * d, h), (h, i), (i, h)]
        # the fused projections: F16, at most 64 rows, dimensions in whole 16-byte chunks
        self.fused = (self.dtype == torch.float16 and B <= FUSED_STEP_MAX_ROWS and
                      all(k % 8 == 0 and n % 8 == 0 for k, n in shapes))
        if self.fused:
            self.stats = linear_stats(h, device=self.device)  # row statistics of x
        # final norm + vocabulary head + greedy pick in one kernel (F16); measured faster
        # than the library GEMM with the separate norm and argmax up to 16 rows
        self.head = (self.dtype == torch.float16 and B <= HEAD_STEP_MAX_ROWS and
                     head_fits(B, h, cfg.vocab_size))
        if self.head:
            self.head_ws = head_workspace(device=self.device)

    def _head(self, residual) -> None:
        """logits and next_ids from the residual stream x (+ residual): final RMSNorm,
        lm_head and greedy argmax (transformer/cache.rs:72-77, sampler.rs:79-88)."""
        cfg, w = self.cfg, self.w
        if self.head:
            lm_head(self.x, w.lm_head, norm_weight=w.final_norm, eps=cfg.rms_norm_eps,
                    residual=residual, logits=self.logits, ids=self.next_ids,
                    workspace=self.head_ws, overlap=True)
            return
        self._norm(self.x, residual, w.final_norm, self.hn, None)
        torch.matmul(self.hn, w.lm_head, out=self.logits)
        call("tmllm_argmax", self.dt, self.logits.data_ptr(), self.next_ids.data_ptr(), self.B,
             cfg.vocab_size, stream_ptr(self.device))

    # -- pieces ------------------------------------------------------------------------
    def _norm(self, x, residual, weight, out, sum_out):
        call("tmllm_add_rmsnorm", self.dt, x.data_ptr(),
             residual.data_ptr() if residual is not None else None, weight.data_ptr(),
             out.data_ptr(), sum_out.data_ptr() if sum_out is not None else None, x.shape[0],
             x.shape[1], self.cfg.rms_norm_eps, stream_ptr(self.device))

    def _attention(self, layer: int) -> None:
        cfg, B = self.cfg, self.B
        hq, hkv, d = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
        w = self.qkv.shape[1]
        base = self.qkv.data_ptr()
        es = self.qkv.element_size()
        # the QKV projection ahead does not touch the cache: the attention may start its
        # K/V prefetch while that projection drains
        opts = DecodeOpts(q_seq_stride=w, kv_seq_stride=w, max_len_hint=self.max_len_hint,
                          flags=DECODE_OVERLAP)
        cos, sin = self.rope
        opts.rope_cos, opts.rope_sin, opts.rope_len = cos.data_ptr(), sin.data_ptr(), cos.shape[0]
        call("tmllm_cache_decode", self.cache.handle, layer, base, base + hq * d * es,
             base + (hq + hkv) * d * es, self.attn.data_ptr(), None, hq, C.byref(opts),
             stream_ptr(self.device))

    def _linear(self, x, w, out, *, norm=None, stats_in=False, residual=None,
                swiglu=False) -> None:
        """A projection of the residual stream; norm-fused ones read the row statistics
        the previous residual add wrote (stats_in), residual adds write them.  Weights are
        never written during a step, so every projection may start its weight prefetch
        while the kernel before it drains."""
        st = self.stats.data_ptr()
        call("tmllm_linear", x.data_ptr(), x.stride(0), norm.data_ptr() if norm is not None
             else None, st if stats_in else None, self.cfg.rms_norm_eps, w.data_ptr(),
             w.stride(0), out.data_ptr(), out.stride(0),
             residual.data_ptr() if residual is not None else None,
             residual.stride(0) if residual is not None else 0,
             st if residual is not None else None, x.shape[0], x.shape[1], out.shape[1],
             int(swiglu), LINEAR_OVERLAP, stream_ptr(self.device))

    def forward_step(self) -> None:
        """One decode step for every sequence: reads ``self.ids``, appends K/V at each
        sequence's length, writes ``self.next_ids``.  Lengths are not advanced."""
        cfg, w = self.cfg, self.w
        call("tmllm_embedding", self.dt, w.embedding.data_ptr(), self.ids.data_ptr(),
             self.x.data_ptr(), self.B, cfg.hidden_size, cfg.vocab_size, self.bad.data_ptr(),
             stream_ptr(self.device))
        if self.fused:
            # x carries the residual stream; each producing projection adds into it
            # (transformer_block.rs:137-158 with the adds and norms folded into projections)
            for li, L in enumerate(w.layers):
                # layer 0 reads the embedded rows once more for their statistics
                self._linear(self.x, L["wqkv"], self.qkv, norm=L["attn_norm"], stats_in=li > 0)
                self._attention(li)
                self._linear(self.attn.view(self.B, -1), L["wo"], self.x, residual=self.x)
                self._linear(self.x, L["wgu"], self.act, norm=L["mlp_norm"], stats_in=True,
                             swiglu=True)
                self._linear(self.act, L["wd"], self.x, residual=self.x)
            self._head(None)
            return
        residual = None
        for li, L in enumerate(w.layers):
            # x <- x + residual; hn <- rmsnorm(x)  (transformer_block.rs:137-139,148)
            self._norm(self.x, residual, L["attn_norm"], self.hn, self.x)
            torch.matmul(self.hn, L["wqkv"], out=self.qkv)
            self._attention(li)
            torch.matmul(self.attn.view(self.B, -1), L["wo"], out=self.o)
            self._norm(self.x, self.o, L["mlp_norm"], self.hn, self.x)
            torch.matmul(self.hn, L["wgu"], out=self.gu)
            call("tmllm_swiglu", self.dt, self.gu.data_ptr(), self.act.data_ptr(), self.B,
                 cfg.intermediate_size, stream_ptr(self.device))
            torch.matmul(self.act, L["wd"], out=self.down)
            residual = self.down
        self._head(residual)

    # -- driving -----------------------------------------------------------------------
    def check_ids(self, ids: torch.Tensor) -> None:
        bad = (ids < 0) | (ids >= self.cfg.vocab_size)
        if bool(bad.any()):  # TinyError::InvalidTokenId
            raise _lib.InvalidArgument(f"token id outside the vocabulary of {self.cfg.vocab_size}")

    def prefill(self, prompts: torch.Tensor) -> torch.Tensor:
        """Runs prompts [B, S] through the model in one pass per layer (the reference's
        forward_with_cache with S new tokens, transformer/cache.rs:59-70): every GEMM takes
        all B*S rows, and attention is the fused append + causal prefill kernel
        (tmllm_cache_prefill).  Fills the cache, advances every length by S and returns the
        greedy token after each prompt (logits of the last row, ``self.logits``)."""
        self.check_ids(prompts)
        B, S = prompts.shape
        if B != self.B:
            raise _lib.ShapeMismatch(f"prefill expects {self.B} prompts, got {B}",
                                     left=[self.B, S], right=list(prompts.shape))
        cfg, w = self.cfg, self.w
        T = B * S
        h, d = cfg.hidden_size, cfg.head_dim
        hq, hkv = cfg.num_heads, cfg.num_kv_heads
        e = dict(dtype=self.dtype, device=self.device)
        ids = prompts.reshape(-1).to(device=self.device, dtype=torch.int32).contiguous()
        x, hn = torch.empty((T, h), **e), torch.empty((T, h), **e)
        qkv = torch.empty((T, (hq + 2 * hkv) * d), **e)
        attn, o = torch.empty((T, hq, d), **e), torch.empty((T, h), **e)
        gu = torch.empty((T, 2 * cfg.intermediate_size), **e)
        act = torch.empty((T, cfg.intermediate_size), **e)
        down = torch.empty((T, h), **e)
        sp = stream_ptr(self.device)
        call("tmllm_embedding", self.dt, w.embedding.data_ptr(), ids.data_ptr(), x.data_ptr(),
             T, h, cfg.vocab_size, self.bad.data_ptr(), sp)
        residual = None
        for li, L in enumerate(w.layers):
            self._norm(x, residual, L["attn_norm"], hn, x)
            torch.matmul(hn, L["wqkv"], out=qkv)
            self.cache.prefill(li, qkv[:, :hq * d].view(T, hq, d),
                               qkv[:, hq * d:(hq + hkv) * d].view(T, hkv, d),
                               qkv[:, (hq + hkv) * d:].view(T, hkv, d), out=attn, rope=self.rope)
            torch.matmul(attn.view(T, -1), L["wo"], out=o)
            self._norm(x, o, L["mlp_norm"], hn, x)
            torch.matmul(hn, L["wgu"], out=gu)
            call("tmllm_swiglu", self.dt, gu.data_ptr(), act.data_ptr(), T,
                 cfg.intermediate_size, sp)
            torch.matmul(act, L["wd"], out=down)
            residual = down
        # only each prompt's last row reaches the head
        last = torch.arange(S - 1, T, S, device=self.device)
        self.x.copy_(x.index_select(0, last))
        self._head(down.index_select(0, last))
        self.cache.advance(S)
        return self.next_ids.clone()

    def prefill_stepwise(self, prompts: torch.Tensor) -> torch.Tensor:
        """Feeds prompts [B, S] token by token through the decode step (each position is
        one fused decode call); the same result as ``prefill`` up to F16 rounding."""
        self.check_ids(prompts)
        B, S = prompts.shape
        self.max_len_hint = max(self.cache.lens()) + S
        for t in range(S):
            self.ids.copy_(prompts[:, t].to(torch.int32))
            self.forward_step()
            self.cache.advance(1)
        return self.next_ids.clone()

    def decode(self, steps: int, first: torch.Tensor | None = None) -> torch.Tensor:
        """Greedy-decodes ``steps`` tokens per sequence without graphs; returns [steps, B]."""
        out = torch.empty((steps, self.B), dtype=torch.int32, device=self.device)
        self.ids.copy_(first if first is not None else self.next_ids)
        self.max_len_hint = max(self.cache.lens()) + steps
        for i in range(steps):
            self.forward_step()
            self.cache.advance(1)
            out[i].copy_(self.next_ids)
            self.ids.copy_(self.next_ids)
        return out


class GraphedDecoder:
    """Captures one decode step of a ``Decoder`` (embedding .. argmax, plus feeding the
    chosen token back as the next input) into a CUDA graph.  Blocks for ``steps`` more
    tokens per sequence are reserved before capture, since a replay cannot run the cache's
    host-side block allocation."""

    def __init__(self, dec: Decoder, steps: int):
        self.dec = dec
        for s in range(dec.B):
            dec.cache.reserve(s, steps + 1)
        dec.max_len_hint = max(dec.cache.lens()) + steps + 1
        stream = torch.cuda.Stream(dec.device)
        stream.wait_stream(torch.cuda.current_stream(dec.device))
        with torch.cuda.stream(stream):
            dec.forward_step()  # first call sizes the cache's workspace outside the capture
        torch.cuda.current_stream(dec.device).wait_stream(stream)
        torch.cuda.synchronize(dec.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=stream):
            dec.forward_step()
            dec.ids.copy_(dec.next_ids)
        self.steps_left = steps

    def step(self) -> None:
        if self.steps_left <= 0:
            pos = self.dec.cache.lens()[0]
            raise _lib.PositionOutOfRange(
                f"graph was captured for fewer steps: position range [{pos}, {pos + 1}) "
                f"is past the captured steps", start_pos=pos, seq_len=1, max_seq_len=pos)
        self.graph.replay()
        self.dec.cache.advance(1)
        self.steps_left -= 1

