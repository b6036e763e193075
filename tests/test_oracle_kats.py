"""The CPU oracle against the reference's own known-answer tests (transcribed in
tests/golden/reference_kats.json with their file:line).  This is what pins the oracle."""
from __future__ import annotations

import math

import numpy as np
import pytest

F = {"f32": np.float32, "f16": np.float16}


def arr(values, shape, dtype):
    vals = [-np.inf if v == "-inf" else v for v in values]
    return np.ascontiguousarray(np.array(vals, dtype=np.float32).reshape(shape).astype(dtype))


def test_kv_cache_two_decode_appends(orc, kats):
    """src/model/kv_cache.rs:214-258: exact layout of the key prefix after two appends."""
    k = kats["kv_cache_two_decode_appends"]
    cache_k = np.zeros((1, k["num_kv_heads"], k["max"], k["dim"]), np.float16)
    cache_v = np.zeros_like(cache_k)
    length = 0
    for ap in k["appends"]:
        key = arr(ap["key"], ap["shape"], np.float16)
        val = arr(ap["value"], ap["shape"], np.float16)
        orc.kv_cache_write(cache_k, key, length)
        orc.kv_cache_write(cache_v, val, length)
        length += ap["shape"][2]
    assert length == k["expect_len"]
    prefix = np.ascontiguousarray(cache_k[:, :, :length])
    assert list(prefix.shape) == k["expect_key_shape"]
    assert prefix.astype(np.float32).ravel().tolist() == k["expect_key"]


@pytest.mark.parametrize("name", ["kv_cache_prefill_append", "kv_cache_append_updates_prefix"])
def test_kv_cache_prefix_shapes(orc, kats, name):
    """src/model/kv_cache.rs:261-273 and 276-293."""
    k = kats[name]
    cache = np.zeros((1, k["num_kv_heads"], k["max"], k["dim"]), np.float16)
    length = 0
    for ap in k["appends"]:
        orc.kv_cache_write(cache, arr(ap["key"], ap["shape"], np.float16), length)
        length += ap["shape"][2]
    assert length == k["expect_len"]
    assert list(cache[:, :, :length].shape) == k["expect_key_shape"]
    assert np.all(cache[:, :, :length] == np.float16(k["appends"][0]["key"][0]))


@pytest.mark.parametrize("dtype", ["f32", "f16"])
def test_repeat_kv_exact(orc, kats, dtype):
    """src/tensor/tensor.rs:791-831: repeat_kv(3) and repeat_kv(1) values, both dtypes."""
    for name in ("repeat_kv_r3", "repeat_kv_r1"):
        k = kats[name]
        x = arr(k["input"], k["shape"], F[dtype])
        out = orc.repeat_kv(x, k["repeats"])
        assert list(out.shape) == k["expect_shape"]
        assert out.astype(np.float32).ravel().tolist() == k["expect"]


@pytest.mark.parametrize("dtype", ["f32", "f16"])
def test_gqa_qk_equals_repeat_then_bmm(orc, kats, dtype):
    """src/tensor/tensor.rs:850-876."""
    k = kats["gqa_qk_equals_repeat_bmm"]
    q = arr(k["q"], k["q_shape"], F[dtype])
    kk = arr(k["k"], k["k_shape"], F[dtype])
    expected = orc.batched_matmul(q, np.ascontiguousarray(orc.repeat_kv(kk, 3).transpose(0, 1, 3, 2)))
    actual = orc.gqa_qk(q, kk)
    assert actual.dtype == q.dtype
    tol = k["tol_f32"] if dtype == "f32" else k["tol_f16"]
    assert np.max(np.abs(expected.astype(np.float32) - actual.astype(np.float32))) < tol


@pytest.mark.parametrize("dtype", ["f32", "f16"])
def test_gqa_pv_equals_repeat_then_bmm(orc, kats, dtype):
    """src/tensor/tensor.rs:879-902."""
    k = kats["gqa_pv_equals_repeat_bmm"]
    p = arr(k["p"], k["p_shape"], F[dtype])
    v = arr(k["v"], k["v_shape"], F[dtype])
    expected = orc.batched_matmul(p, orc.repeat_kv(v, 3))
    actual = orc.gqa_pv(p, v)
    tol = k["tol_f32"] if dtype == "f32" else k["tol_f16"]
    assert np.max(np.abs(expected.astype(np.float32) - actual.astype(np.float32))) < tol


def test_bmm_f16_close_to_f32(orc, kats):
    """src/tensor/tensor.rs:905-926."""
    k = kats["bmm_f16_close_to_f32"]
    a32, b32 = arr(k["a"], k["a_shape"], np.float32), arr(k["b"], k["b_shape"], np.float32)
    e = orc.batched_matmul(a32, b32)
    a = orc.batched_matmul(a32.astype(np.float16), b32.astype(np.float16))
    assert a.dtype == np.float16
    assert np.max(np.abs(e - a.astype(np.float32))) < k["tol"]


def test_bmm_transposed_keys(orc, kats):
    """src/tensor/tensor.rs:952-982."""
    k = kats["bmm_transposed_keys"]
    q, kk = arr(k["q"], k["q_shape"], np.float32), arr(k["k"], k["k_shape"], np.float32)
    kt = np.ascontiguousarray(kk.transpose(0, 1, 3, 2))
    e = orc.batched_matmul(q, kt)
    a = orc.batched_matmul(q.astype(np.float16), kt.astype(np.float16))
    assert np.max(np.abs(e - a.astype(np.float32))) < k["tol"]


def test_scale_mask_prefill_f16_vs_f32(orc, kats):
    """src/tensor/tensor.rs:985-1004."""
    k = kats["scale_mask_prefill"]
    s = arr(k["scores"], k["shape"], np.float32)
    e = orc.attention_scale_mask(s, k["scale"], k["start"])
    a = orc.attention_scale_mask(s.astype(np.float16), k["scale"], k["start"]).astype(np.float32)
    for x, y in zip(e.ravel(), a.ravel()):
        if np.isinf(x):
            assert np.isinf(y) and np.signbit(x) == np.signbit(y)
        else:
            assert abs(x - y) < k["tol"]


@pytest.mark.parametrize("name", ["scale_mask_decode_keeps_all",
                                  "scale_mask_intermediate_masks_future"])
def test_scale_mask_exact(orc, kats, name):
    """src/tensor/tensor.rs:1007-1035: exact F16 values and the masked -inf."""
    k = kats[name]
    s = arr(k["scores"], k["shape"], np.float16)
    out = orc.attention_scale_mask(s, k["scale"], k["start"]).astype(np.float32).ravel()
    exp = [-np.inf if v == "-inf" else v for v in k["expect"]]
    assert out.tolist() == exp


def test_softmax_rows(orc, kats):
    """src/tensor/tensor.rs:1038-1057."""
    k = kats["softmax_rows"]
    x = arr(k["input"], k["shape"], np.float32)
    e = orc.softmax_last_dim(x)
    a = orc.softmax_last_dim(x.astype(np.float16)).astype(np.float32)
    assert np.max(np.abs(e - a)) < k["tol"]
    assert np.all(np.abs(a.sum(-1) - 1.0) < k["row_sum_tol"])


def test_mask_softmax_zeros(orc, kats):
    """src/tensor/tensor.rs:1060-1089: masked probabilities are exactly zero."""
    k = kats["mask_softmax_zeros"]
    s = arr(k["scores"], k["shape"], np.float32)
    e = orc.softmax_last_dim(orc.attention_scale_mask(s, k["scale"], k["start"]))
    a = orc.softmax_last_dim(orc.attention_scale_mask(s.astype(np.float16), k["scale"],
                                                      k["start"])).astype(np.float32)
    assert np.max(np.abs(e - a)) < k["tol"]
    for i in k["expect_zero_indices"]:
        assert a.ravel()[i] == 0.0 and e.ravel()[i] == 0.0


def attention_case(hq, hkv, d, s, start, dtype=np.float32):
    """The deterministic inputs of src/nn/attention.rs:620-634."""
    query = np.array([(i % 5) - 2.0 for i in range(hq * s * d)], np.float32)
    cached = np.array([(i % 3) - 1.0 for i in range(hkv * (start + s) * d)], np.float32)
    q = query.reshape(1, hq, s, d).astype(dtype)
    key = cached.reshape(1, hkv, start + s, d).astype(dtype)
    return q, key


def test_attention_core_matches_op_chain(orc, kats):
    """src/nn/attention.rs:591-668: the chained core equals QK -> scale/mask -> softmax -> PV
    run op by op, within 1e-5."""
    k = kats["attention_core_matches_op_chain"]
    d, s, start = k["head_dim"], k["seq_len"], k["start_pos"]
    for hq, hkv in k["cases"]:
        q, key = attention_case(hq, hkv, d, s, start)
        scores = orc.gqa_qk(q, key)
        scores = orc.attention_scale_mask(scores, 1.0 / math.sqrt(d), start)
        probs = orc.softmax_last_dim(scores)
        expected = orc.gqa_pv(probs, key)
        actual = orc.attention_core(q, key, key, start + s, start)
        assert np.max(np.abs(expected - actual)) < k["tol"]
        # and the float64 restatement agrees to F32 rounding
        wide, _ = orc.attention_core_wide(q, key, key, start + s, start)
        assert np.max(np.abs(wide - actual)) < 1e-5


def test_rope_f16_close_to_f32(orc, kats):
    """src/nn/rope.rs:186-208."""
    k = kats["rope_f16_close_to_f32"]
    cos, sin = orc.rope_tables(k["head_dim"], k["max_seq_len"], k["theta"])
    x = arr(k["input"], k["shape"], np.float32)
    e = orc.rope(x, cos, sin, k["start"])
    a = orc.rope(x.astype(np.float16), cos, sin, k["start"]).astype(np.float32)
    assert np.max(np.abs(e - a)) <= k["tol"]
