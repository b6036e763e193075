"""TEST INFRASTRUCTURE ONLY — numpy front end of the C oracle (``liboracle.so``).

The oracle restates the reference's Metal kernels (Lee-Dongwook/RustLLM ``kernels/``)
on the CPU.  Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import this module; the product package ``rustllm_b200`` never does.

F16 arrays are passed as ``np.float16`` (IEEE binary16, the reference's ``half``).
"""
from __future__ import annotations

import ctypes as C
import math
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

u32 = C.c_uint32
vp = C.c_void_p


def build(force: bool = False) -> str:
    """Compile ``liboracle.so`` with the committed Makefile (gcc only)."""
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < max(
        os.path.getmtime(os.path.join(_HERE, f)) for f in ("tmllm_oracle.c", "tmllm_oracle.h")
    ):
        subprocess.run(["make", "-s", "-B" if force else "-s", "-C", _HERE, "liboracle.so"],
                       check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = C.CDLL(_LIB_PATH)
        L.orc_f32_to_f16.restype = C.c_uint16
        L.orc_f32_to_f16.argtypes = [C.c_float]
        L.orc_f16_to_f32.restype = C.c_float
        L.orc_f16_to_f32.argtypes = [C.c_uint16]
        L.orc_attention_core.restype = C.c_int
        L.orc_attention_core.argtypes = [C.c_int, vp, vp, vp, vp] + [u32] * 8 + [C.c_float, C.c_int]
        L.orc_attention_core_wide.restype = C.c_int
        L.orc_attention_core_wide.argtypes = [vp] * 5 + [u32] * 8 + [C.c_double, C.c_int]
        L.orc_scale_mask_f32.argtypes = [vp, vp, C.c_float, u32, u32, u32, u32]
        L.orc_scale_mask_f16.argtypes = [vp, vp, C.c_float, u32, u32, u32, u32]
        L.orc_rope_tables.argtypes = [vp, vp, u32, u32, C.c_float]
        L.orc_merge_lse.argtypes = [vp, vp, u32, u32, u32, vp, vp]
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(C.c_void_p)


def _dt(a: np.ndarray) -> int:
    if a.dtype == np.float32:
        return 0
    if a.dtype == np.float16:
        return 1
    raise TypeError(f"oracle supports float32/float16, got {a.dtype}")


# ---- conversions ------------------------------------------------------------------------

def f32_to_f16_bits(x: float) -> int:
    return lib().orc_f32_to_f16(float(x))


def f16_bits_to_f32(h: int) -> float:
    return lib().orc_f16_to_f32(int(h))


# ---- copies -----------------------------------------------------------------------------

def kv_cache_write(cache: np.ndarray, source: np.ndarray, start: int) -> None:
    """kernels/kv_cache_write.metal:13-18 on cache [1,H,max,D] and source [1,H,S,D]."""
    _, h, max_seq, d = cache.shape
    s = source.shape[2]
    lib().orc_kv_cache_write(C.c_int(cache.itemsize), _p(cache), _p(source), u32(start),
                             u32(s), u32(max_seq), u32(d), u32(source.size))


def concat_sequence(left: np.ndarray, right: np.ndarray) -> np.ndarray:
    """kernels/concat_sequence.metal:30-88."""
    b, h, sl, d = left.shape
    sr = right.shape[2]
    out = np.empty((b, h, sl + sr, d), dtype=left.dtype)
    lib().orc_concat_sequence(C.c_int(left.itemsize), _p(left), _p(right), _p(out), u32(b),
                              u32(h), u32(sl), u32(sr), u32(d))
    return out


def repeat_kv(x: np.ndarray, repeats: int) -> np.ndarray:
    """kernels/repeat_kv.metal:16-30."""
    b, h, s, d = x.shape
    out = np.empty((b, h * repeats, s, d), dtype=x.dtype)
    lib().orc_repeat_kv(C.c_int(x.itemsize), _p(x), _p(out), u32(b), u32(h), u32(s), u32(d),
                        u32(repeats))
    return out


# ---- attention ops ----------------------------------------------------------------------

def gqa_qk(q: np.ndarray, k: np.ndarray, kv_len: int | None = None) -> np.ndarray:
    """kernels/gqa_matmul.metal:7-321.  q [B,Hq,S,D]; k [B,Hkv,cap,D] read for kv_len keys."""
    b, hq, s, d = q.shape
    _, hkv, cap, _ = k.shape
    kv_len = cap if kv_len is None else kv_len
    out = np.empty((b, hq, s, kv_len), dtype=q.dtype)
    fn = lib().orc_gqa_qk_f32 if _dt(q) == 0 else lib().orc_gqa_qk_f16
    fn(_p(q), _p(k), _p(out), u32(b), u32(hq), u32(hkv), u32(s), u32(kv_len), u32(d), u32(cap))
    return out


def gqa_pv(p: np.ndarray, v: np.ndarray) -> np.ndarray:
    """kernels/gqa_matmul.metal:323-629.  p [B,Hq,S,L]; v [B,Hkv,cap,D]."""
    b, hq, s, kv_len = p.shape
    _, hkv, cap, d = v.shape
    out = np.empty((b, hq, s, d), dtype=p.dtype)
    fn = lib().orc_gqa_pv_f32 if _dt(p) == 0 else lib().orc_gqa_pv_f16
    fn(_p(p), _p(v), _p(out), u32(b), u32(hq), u32(hkv), u32(s), u32(kv_len), u32(d), u32(cap))
    return out


def attention_scale_mask(scores: np.ndarray, scale: float, start: int) -> np.ndarray:
    """kernels/attention_scale_mask.metal; scores [..., q_len, key_len]."""
    q_len, key_len = scores.shape[-2], scores.shape[-1]
    out = np.empty_like(scores)
    fn = lib().orc_scale_mask_f32 if _dt(scores) == 0 else lib().orc_scale_mask_f16
    fn(_p(scores), _p(out), C.c_float(scale), u32(q_len), u32(key_len), u32(start),
       u32(scores.size))
    return out


def softmax_last_dim(x: np.ndarray) -> np.ndarray:
    """kernels/softmax.metal (256-wide reduction order, F16 zero-row guard)."""
    width = x.shape[-1]
    out = np.empty_like(x)
    fn = lib().orc_softmax_f32 if _dt(x) == 0 else lib().orc_softmax_f16
    fn(_p(x), _p(out), u32(x.size // width), u32(width))
    return out


def batched_matmul(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """kernels/batched_matmul.metal; a [...,m,k] x b [...,k,n]."""
    m, k = a.shape[-2:]
    n = b.shape[-1]
    batch = a.size // (m * k)
    out = np.empty(a.shape[:-2] + (m, n), dtype=a.dtype)
    fn = lib().orc_batched_matmul_f32 if _dt(a) == 0 else lib().orc_batched_matmul_f16
    fn(_p(a), _p(np.ascontiguousarray(b)), _p(out), u32(batch), u32(m), u32(k), u32(n))
    return out


def rope_tables(head_dim: int, max_seq_len: int, theta: float):
    """src/nn/rope.rs:44-62."""
    half = head_dim // 2
    cos = np.empty((max_seq_len, half), dtype=np.float32)
    sin = np.empty((max_seq_len, half), dtype=np.float32)
    lib().orc_rope_tables(_p(cos), _p(sin), u32(head_dim), u32(max_seq_len), C.c_float(theta))
    return cos, sin


def rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray, start: int) -> np.ndarray:
    """kernels/rope.metal on x [..., seq, head_dim]."""
    seq, d = x.shape[-2], x.shape[-1]
    out = np.empty_like(x)
    fn = lib().orc_rope_f32 if _dt(x) == 0 else lib().orc_rope_f16
    fn(_p(x), _p(cos), _p(sin), _p(out), u32(seq), u32(d), u32(start), u32(x.size // 2))
    return out


def attention_core(q: np.ndarray, k: np.ndarray, v: np.ndarray, kv_len: int, start_pos: int,
                   scale: float | None = None, threads: int = 1) -> np.ndarray:
    """src/nn/attention.rs:216-247, faithful storage rounding.

    q [B,Hq,S,D]; k, v [B,Hkv,cap,D] (the cache with its capacity stride)."""
    b, hq, s, d = q.shape
    _, hkv, cap, _ = k.shape
    scale = 1.0 / math.sqrt(d) if scale is None else scale
    out = np.empty_like(q)
    rc = lib().orc_attention_core(_dt(q), _p(q), _p(k), _p(v), _p(out), b, hq, hkv, s, kv_len,
                                  d, cap, start_pos, scale, threads)
    if rc != 0:
        raise ValueError("oracle attention_core: invalid arguments")
    return out


def attention_core_wide(q: np.ndarray, k: np.ndarray, v: np.ndarray, kv_len: int,
                        start_pos: int, scale: float | None = None, threads: int = 1):
    """The same chain in float64 (no storage rounding); returns (out, lse)."""
    b, hq, s, d = q.shape
    _, hkv, cap, _ = k.shape
    scale = 1.0 / math.sqrt(d) if scale is None else scale
    qf = np.ascontiguousarray(q, dtype=np.float32)
    kf = np.ascontiguousarray(k, dtype=np.float32)
    vf = np.ascontiguousarray(v, dtype=np.float32)
    out = np.empty((b, hq, s, d), dtype=np.float64)
    lse = np.empty((b, hq, s), dtype=np.float64)
    rc = lib().orc_attention_core_wide(_p(qf), _p(kf), _p(vf), _p(out), _p(lse), b, hq, hkv, s,
                                       kv_len, d, cap, start_pos, scale, threads)
    if rc != 0:
        raise ValueError("oracle attention_core_wide: invalid arguments")
    return out, lse


def paged_gather(arena: np.ndarray, table: np.ndarray, seq: int, length: int, block_size: int,
                 num_kv_heads: int, head_dim: int) -> np.ndarray:
    """Dense [Hkv, len, D] copy of sequence ``seq`` from a block-paged arena."""
    table = np.ascontiguousarray(table, dtype=np.int32)
    out = np.empty((num_kv_heads, length, head_dim), dtype=arena.dtype)
    lib().orc_paged_gather(C.c_int(arena.itemsize), _p(arena), _p(table), u32(table.shape[1]),
                           u32(seq), u32(length), u32(block_size), u32(num_kv_heads),
                           u32(head_dim), _p(out))
    return out


def paged_scatter(arena: np.ndarray, table: np.ndarray, seq: int, start: int, x: np.ndarray,
                  block_size: int) -> None:
    """Write x [Hkv, n, D] at positions [start, start+n) of sequence ``seq``."""
    table = np.ascontiguousarray(table, dtype=np.int32)
    hkv, n, d = x.shape
    lib().orc_paged_scatter(C.c_int(arena.itemsize), _p(arena), _p(table), u32(table.shape[1]),
                            u32(seq), u32(start), u32(n), u32(block_size), u32(hkv), u32(d),
                            _p(np.ascontiguousarray(x)))


def merge_lse(parts_o: np.ndarray, parts_lse: np.ndarray):
    """Log-sum-exp merge of n partial results: parts_o [n, rows, D], parts_lse [n, rows]."""
    n, rows, d = parts_o.shape
    po = np.ascontiguousarray(parts_o, dtype=np.float32)
    pl = np.ascontiguousarray(parts_lse, dtype=np.float32)
    out = np.empty((rows, d), dtype=np.float32)
    lse = np.empty((rows,), dtype=np.float32)
    lib().orc_merge_lse(_p(po), _p(pl), n, rows, d, _p(out), _p(lse))
    return out, lse


def decode_step(q: np.ndarray, k_new: np.ndarray, v_new: np.ndarray, k_cache: np.ndarray,
                v_cache: np.ndarray, start_pos: int, cos: np.ndarray | None = None,
                sin: np.ndarray | None = None, threads: int = 1) -> np.ndarray:
    """One per-layer decode step in the reference's order (src/nn/attention.rs:303-313):
    RoPE q and k at start_pos (when tables are given), append k, v into the cache at
    start_pos (kv_cache.rs:112-142), then the attention core over start_pos+1 keys.

    q [B,Hq,1,D]; k_new, v_new [B,Hkv,1,D]; caches [B,Hkv,cap,D] are modified in place."""
    if cos is not None:
        q = rope(q, cos, sin, start_pos)
        k_new = rope(k_new, cos, sin, start_pos)
    b = q.shape[0]
    for i in range(b):
        kv_cache_write(k_cache[i:i + 1], np.ascontiguousarray(k_new[i:i + 1]), start_pos)
        kv_cache_write(v_cache[i:i + 1], np.ascontiguousarray(v_new[i:i + 1]), start_pos)
    return attention_core(q, k_cache, v_cache, start_pos + 1, start_pos, threads=threads)
