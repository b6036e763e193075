"""Self-consistency of the CPU oracle: binary16 rounding, faithful vs float64 chains,
paged layout round trips, the log-sum-exp merge, and the committed fixtures."""
from __future__ import annotations

import math

import numpy as np
import pytest


def test_f16_round_trip_matches_numpy(orc):
    rng = np.random.default_rng(0)
    x = np.concatenate([
        rng.standard_normal(20000).astype(np.float32) * 10.0 ** rng.integers(-9, 6, 20000),
        np.array([0.0, -0.0, 65504.0, 65520.0, 1e-8, 5.96e-8, 2.98e-8, np.inf, -np.inf],
                 np.float32)])
    got = np.array([orc.f32_to_f16_bits(v) for v in x], np.uint16)
    want = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(got, want)
    all_bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    finite = ~np.isnan(all_bits.view(np.float16))
    back = np.array([orc.f16_bits_to_f32(int(b)) for b in all_bits[finite][::7]], np.float32)
    assert np.array_equal(back, all_bits[finite][::7].view(np.float16).astype(np.float32))


@pytest.mark.parametrize("hq,hkv,d,cached", [(9, 3, 64, 128), (32, 8, 128, 257), (4, 4, 8, 5)])
def test_faithful_f16_chain_close_to_float64(orc, hq, hkv, d, cached):
    """The reference's F16 chain (four half roundings) stays within 2e-3 of the exact result
    (the north-star F16 tolerance, measured as max|a-b| / max|b|)."""
    rng = np.random.default_rng(hq * 1000 + d)
    q = rng.standard_normal((1, hq, 1, d)).astype(np.float16)
    k = rng.standard_normal((1, hkv, cached + 1, d)).astype(np.float16)
    v = rng.standard_normal((1, hkv, cached + 1, d)).astype(np.float16)
    faithful = orc.attention_core(q, k, v, cached + 1, cached).astype(np.float64)
    wide, _ = orc.attention_core_wide(q, k, v, cached + 1, cached)
    assert np.max(np.abs(faithful - wide)) / np.max(np.abs(wide)) < 2e-3


def test_faithful_f32_chain_close_to_float64(orc):
    rng = np.random.default_rng(7)
    q = rng.standard_normal((1, 9, 3, 64)).astype(np.float32)
    k = rng.standard_normal((1, 3, 200, 64)).astype(np.float32)
    v = rng.standard_normal((1, 3, 200, 64)).astype(np.float32)
    faithful = orc.attention_core(q, k, v, 150, 147)
    wide, _ = orc.attention_core_wide(q, k, v, 150, 147)
    assert np.max(np.abs(faithful - wide)) / np.max(np.abs(wide)) < 1e-5


def test_threaded_chain_equals_single_thread(orc):
    rng = np.random.default_rng(3)
    q = rng.standard_normal((2, 8, 1, 64)).astype(np.float16)
    k = rng.standard_normal((2, 2, 300, 64)).astype(np.float16)
    v = rng.standard_normal((2, 2, 300, 64)).astype(np.float16)
    a = orc.attention_core(q, k, v, 300, 299, threads=1)
    b = orc.attention_core(q, k, v, 300, 299, threads=5)
    assert np.array_equal(a.view(np.uint16), b.view(np.uint16))


def test_paged_scatter_gather_round_trip(orc):
    rng = np.random.default_rng(11)
    nb, hkv, bs, d, seqs, mb = 40, 3, 16, 8, 3, 10
    arena = np.zeros((nb, hkv, bs, d), np.float16)
    table = rng.permutation(nb)[: seqs * mb].reshape(seqs, mb).astype(np.int32)
    data = {}
    for s in range(seqs):
        n = int(rng.integers(1, mb * bs))
        x = rng.standard_normal((hkv, n, d)).astype(np.float16)
        orc.paged_scatter(arena, table, s, 0, x[:, : n // 2], bs)
        orc.paged_scatter(arena, table, s, n // 2, x[:, n // 2:], bs)
        data[s] = x
    for s, x in data.items():
        got = orc.paged_gather(arena, table, s, x.shape[1], bs, hkv, d)
        assert np.array_equal(got.view(np.uint16), x.view(np.uint16))


def test_merge_of_splits_equals_whole(orc):
    """Splitting the keys, attending each part and merging by log-sum-exp equals attending
    all keys (the identity the split-K kernel and the cross-GPU split rely on)."""
    rng = np.random.default_rng(5)
    hq, hkv, d, n = 8, 2, 32, 1000
    q = rng.standard_normal((1, hq, 1, d)).astype(np.float32)
    k = rng.standard_normal((1, hkv, n, d)).astype(np.float32)
    v = rng.standard_normal((1, hkv, n, d)).astype(np.float32)
    whole, whole_lse = orc.attention_core_wide(q, k, v, n, n - 1)
    cuts = [0, 100, 517, 518, 1000]
    parts_o, parts_l = [], []
    for a, b in zip(cuts[:-1], cuts[1:]):
        o, l = orc.attention_core_wide(q, np.ascontiguousarray(k[:, :, a:b]),
                                       np.ascontiguousarray(v[:, :, a:b]), b - a, b - a - 1)
        parts_o.append(o.reshape(hq, d))
        parts_l.append(l.reshape(hq))
    out, lse = orc.merge_lse(np.stack(parts_o), np.stack(parts_l))
    assert np.max(np.abs(out - whole.reshape(hq, d))) < 1e-5
    assert np.max(np.abs(lse - whole_lse.reshape(hq))) < 1e-4


def test_concat_sequence_is_a_split_inverse(orc):
    rng = np.random.default_rng(9)
    for dtype in (np.float32, np.float16):
        x = rng.standard_normal((2, 3, 17, 8)).astype(dtype)
        out = orc.concat_sequence(np.ascontiguousarray(x[:, :, :5]), np.ascontiguousarray(x[:, :, 5:]))
        assert np.array_equal(out, x)


def test_fixtures_reproduce(orc, fixtures):
    """The committed fixtures are what the oracle computes today."""
    f = fixtures
    kc, vc = f["cfg1_k_cache"].copy(), f["cfg1_v_cache"].copy()
    o = orc.decode_step(f["cfg1_q"], f["cfg1_k"], f["cfg1_v"], kc, vc, 128, f["cfg1_cos"],
                        f["cfg1_sin"])
    assert np.array_equal(o, f["cfg1_out"])
    assert np.array_equal(kc[:, :, 128], f["cfg1_k_row_after"])
    assert np.max(np.abs(o - f["cfg1_out_wide"])) / np.max(np.abs(f["cfg1_out_wide"])) < 1e-5
    kc, vc = f["f16_k_cache"].copy(), f["f16_v_cache"].copy()
    o = orc.decode_step(f["f16_q"], f["f16_k"], f["f16_v"], kc, vc, 150)
    assert np.array_equal(o.view(np.uint16), f["f16_out"].view(np.uint16))


def test_rope_tables_match_reference_formula(orc):
    """src/nn/rope.rs:50-61 in float32 arithmetic."""
    cos, sin = orc.rope_tables(64, 50, 100000.0)
    pos, i = 37, 5
    exponent = np.float32(2 * i) / np.float32(64)
    inv = np.float32(1.0) / np.power(np.float32(100000.0), exponent, dtype=np.float32)
    angle = np.float32(pos) * inv
    assert abs(cos[pos, i] - math.cos(angle)) < 1e-6
    assert abs(sin[pos, i] - math.sin(angle)) < 1e-6
