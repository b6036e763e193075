"""Op-level CUDA kernels against the CPU oracle and the reference's known answers.

Copies, QK, PV, scale/mask, batched matmul and RoPE sum in the reference's order without
contraction, so they must be bit-exact with the oracle.  Softmax calls exp(), whose last
bits may differ between CUDA and the C library: it is held to 16 ulp of F32 (and one
ulp step of F16)."""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import rustllm_b200 as rb

pytestmark = pytest.mark.gpu


def t(x: np.ndarray, dev) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def n(x: torch.Tensor) -> np.ndarray:
    return x.detach().cpu().numpy()


def bits(x: np.ndarray) -> np.ndarray:
    return x.view(np.uint16 if x.dtype == np.float16 else np.uint32)


def rnd(rng, shape, dtype):
    return rng.standard_normal(shape).astype(dtype)


DT = [np.float32, np.float16]


@pytest.mark.parametrize("dtype", DT)
def test_kv_cache_write_bit_exact(cuda, orc, dtype):
    rng = np.random.default_rng(1)
    for h, mx, d, start, s in [(2, 8, 4, 0, 3), (3, 129, 64, 128, 1), (8, 40, 128, 7, 33),
                               (1, 5, 3, 2, 3)]:
        cache = rnd(rng, (1, h, mx, d), dtype)
        src = rnd(rng, (1, h, s, d), dtype)
        want = cache.copy()
        orc.kv_cache_write(want, src, start)
        gc = t(cache, cuda)
        rb.kv_cache_write(gc, t(src, cuda), start)
        assert np.array_equal(bits(n(gc)), bits(want))


def test_kv_cache_write_rejects_overflow(cuda):
    cache = torch.zeros((1, 2, 8, 4), dtype=torch.float16, device=cuda)
    with pytest.raises(rb.PositionOutOfRange):
        rb.kv_cache_write(cache, torch.ones((1, 2, 2, 4), dtype=torch.float16, device=cuda), 7)
    assert torch.count_nonzero(cache) == 0


@pytest.mark.parametrize("dtype", DT)
def test_concat_sequence_bit_exact(cuda, orc, dtype):
    rng = np.random.default_rng(2)
    for b, h, sl, sr, d in [(1, 2, 3, 1, 4), (2, 8, 131, 1, 128), (1, 3, 0, 5, 64),
                            (2, 2, 4, 3, 5)]:
        left, right = rnd(rng, (b, h, sl, d), dtype), rnd(rng, (b, h, sr, d), dtype)
        want = orc.concat_sequence(left, right) if sl else right
        got = n(rb.concat_sequence(t(left, cuda), t(right, cuda)))
        assert np.array_equal(bits(got), bits(want))


@pytest.mark.parametrize("dtype", DT)
def test_repeat_kv_reference_kats(cuda, kats, dtype):
    """src/tensor/tensor.rs:791-831 on the GPU."""
    for name in ("repeat_kv_r3", "repeat_kv_r1"):
        k = kats[name]
        x = np.array(k["input"], np.float32).reshape(k["shape"]).astype(dtype)
        out = rb.repeat_kv(t(x, cuda), k["repeats"])
        assert list(out.shape) == k["expect_shape"]
        assert n(out).astype(np.float32).ravel().tolist() == k["expect"]


@pytest.mark.parametrize("dtype", DT)
def test_repeat_kv_bit_exact(cuda, orc, dtype):
    rng = np.random.default_rng(3)
    x = rnd(rng, (2, 3, 17, 64), dtype)
    assert np.array_equal(bits(n(rb.repeat_kv(t(x, cuda), 5))), bits(orc.repeat_kv(x, 5)))


@pytest.mark.parametrize("dtype", DT)
def test_gqa_qk_pv_bit_exact(cuda, orc, dtype):
    rng = np.random.default_rng(4)
    for b, hq, hkv, s, cap, kv_len, d in [(1, 9, 3, 1, 200, 129, 64), (2, 6, 2, 3, 8, 5, 4),
                                          (1, 4, 4, 2, 50, 50, 128)]:
        q = rnd(rng, (b, hq, s, d), dtype)
        k = rnd(rng, (b, hkv, cap, d), dtype)
        v = rnd(rng, (b, hkv, cap, d), dtype)
        scores = rb.gqa_qk_matmul(t(q, cuda), t(k, cuda), kv_len)
        assert np.array_equal(bits(n(scores)), bits(orc.gqa_qk(q, k, kv_len)))
        p = rng.random((b, hq, s, kv_len)).astype(dtype)
        out = rb.gqa_pv_matmul(t(p, cuda), t(v, cuda))
        assert np.array_equal(bits(n(out)), bits(orc.gqa_pv(p, v)))


@pytest.mark.parametrize("dtype", DT)
def test_scale_mask_and_bmm_bit_exact(cuda, orc, dtype):
    rng = np.random.default_rng(5)
    # key lengths that are not (9) and are (16, 40) whole 16-byte chunks: both kernels
    for shape in ((2, 3, 4, 9), (2, 3, 4, 16), (1, 2, 5, 40)):
        s = rnd(rng, shape, dtype) * 5
        for start in (0, 3, shape[-1] - shape[-2]):
            got = n(rb.attention_scale_mask(t(s, cuda), 0.125, start))
            assert np.array_equal(bits(got), bits(orc.attention_scale_mask(s, 0.125, start)))
    a, bm = rnd(rng, (3, 5, 7), dtype), rnd(rng, (3, 7, 11), dtype)
    assert np.array_equal(bits(n(rb.batched_matmul(t(a, cuda), t(bm, cuda)))),
                          bits(orc.batched_matmul(a, bm)))


def test_scale_mask_reference_kats(cuda, kats):
    """src/tensor/tensor.rs:1007-1035: exact F16 values on the GPU."""
    for name in ("scale_mask_decode_keeps_all", "scale_mask_intermediate_masks_future"):
        k = kats[name]
        s = np.array(k["scores"], np.float32).reshape(k["shape"]).astype(np.float16)
        out = n(rb.attention_scale_mask(t(s, cuda), k["scale"], k["start"])).astype(np.float32)
        assert out.ravel().tolist() == [-np.inf if v == "-inf" else v for v in k["expect"]]


@pytest.mark.parametrize("dtype", DT)
def test_softmax_close_to_oracle(cuda, orc, dtype):
    rng = np.random.default_rng(6)
    for rows, width in [(2, 3), (32, 131), (3, 1000), (1, 70000)]:
        x = (rnd(rng, (rows, width), dtype) * 4).astype(dtype)
        got = n(rb.softmax_last_dim(t(x, cuda)))
        want = orc.softmax_last_dim(x)
        if dtype == np.float32:
            assert np.max(np.abs(got - want) / np.maximum(np.abs(want), 1e-30)) < 16 * 2 ** -23
        else:
            diff = np.abs(bits(got).astype(np.int32) - bits(want).astype(np.int32))
            assert diff.max() <= 1


def test_softmax_f16_all_masked_row_is_zero(cuda):
    """softmax.metal:166-173: an all -inf F16 row becomes zeros."""
    x = torch.full((2, 5), float("-inf"), dtype=torch.float16, device=cuda)
    x[1] = 1.0
    out = rb.softmax_last_dim(x)
    assert torch.all(out[0] == 0)
    assert abs(float(out[1].float().sum()) - 1.0) < 1e-2


def test_mask_softmax_zeros_reference_kat(cuda, kats):
    """src/tensor/tensor.rs:1060-1089 on the GPU."""
    k = kats["mask_softmax_zeros"]
    s = torch.tensor(k["scores"], dtype=torch.float32).reshape(k["shape"]).to(cuda)
    e = rb.softmax_last_dim(rb.attention_scale_mask(s, k["scale"], k["start"]))
    a = rb.softmax_last_dim(rb.attention_scale_mask(s.half(), k["scale"], k["start"])).float()
    assert float((e - a).abs().max()) < k["tol"]
    for i in k["expect_zero_indices"]:
        assert float(a.flatten()[i]) == 0.0


@pytest.mark.parametrize("dtype", DT)
def test_rope_bit_exact(cuda, orc, dtype):
    rng = np.random.default_rng(7)
    cos, sin = orc.rope_tables(64, 300, 100000.0)
    gc, gs = rb.rope_tables(64, 300, 100000.0, device=cuda)
    assert np.array_equal(n(gc), cos) and np.array_equal(n(gs), sin)
    x = rnd(rng, (1, 9, 5, 64), dtype)
    got = n(rb.rope(t(x, cuda), gc, gs, 128))
    assert np.array_equal(bits(got), bits(orc.rope(x, cos, sin, 128)))


def test_attention_core_chain_reference_kat(cuda, orc, kats):
    """src/nn/attention.rs:591-668: the op chain on the GPU equals the oracle's (1e-5)."""
    k = kats["attention_core_matches_op_chain"]
    d, s, start = k["head_dim"], k["seq_len"], k["start_pos"]
    for hq, hkv in k["cases"]:
        q = np.array([(i % 5) - 2.0 for i in range(hq * s * d)], np.float32).reshape(1, hq, s, d)
        key = np.array([(i % 3) - 1.0 for i in range(hkv * (start + s) * d)],
                       np.float32).reshape(1, hkv, start + s, d)
        got = n(rb.attention_core(t(q, cuda), t(key, cuda), t(key, cuda), start))
        want = orc.attention_core(q, key, key, start + s, start)
        assert np.max(np.abs(got - want)) < k["tol"]
