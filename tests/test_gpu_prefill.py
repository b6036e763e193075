"""Fused KV-append + causal prefill attention (tmllm_gqa_prefill / tmllm_cache_prefill)
against the CPU oracle.

Each sequence holds `cached` positions of seeded N(0,1) K/V, then `n` new tokens are
appended and attend causally: new row i sees positions [0, cached + i]
(attention_scale_mask.metal:21-41 with start = cached).  The oracle runs the reference's
chain on the RoPE'd, F16-rounded q and the full key range.  Tolerances: 2e-3 relative
(max|gpu - ref| / max|ref|) for F16 against the float64 chain, 1e-5 for F32; the appended
rows are bit-exact with the oracle's RoPE + storage rounding."""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

import rustllm_b200 as rb

pytestmark = pytest.mark.gpu

THREADS = os.cpu_count() or 4


def rel(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def elem_excess(a, b, tol) -> float:
    """max over elements of |a - b| / (tol * (|b| + rms(b))): <= 1 passes the element-wise
    bound (a per-element relative bound with a floor of tol * rms for outputs near zero)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    rms = float(np.sqrt(np.mean(b * b)))
    return float(np.max(np.abs(a - b) / (tol * (np.abs(b) + rms) + 1e-300)))


def run_case(dev, orc, *, npd=np.float16, hq=4, hkv=4, d=64, cached=(0,), n=128,
             block_size=16, theta=10000.0, variant=0, seed=0, ragged=None, out_f32=False,
             faithful=False):
    """Fills a paged cache, prefills n (or ragged[s]) rows per sequence, returns
    (max relative error vs the float64 oracle, appended rows bit-exact).  The outputs are
    also held to the element-wise bound against the float64 chain, and with `faithful`
    checked norm-relative against the reference's own chain (its F16 store points), inside
    this function."""
    rng = np.random.default_rng(seed)
    B = len(cached)
    rows = list(ragged) if ragged is not None else [n] * B
    tdt = torch.float16 if npd == np.float16 else torch.float32
    max_len = max(c + r for c, r in zip(cached, rows)) + 1
    cache = rb.PagedKvCache(1, B, max_len, hkv, d, dtype=tdt, block_size=block_size,
                            shuffle_seed=seed + 5, device=dev)
    kc = [rng.standard_normal((hkv, c, d)).astype(npd) for c in cached]
    vc = [rng.standard_normal((hkv, c, d)).astype(npd) for c in cached]
    for s in range(B):
        if cached[s]:
            cache.append(0, s, torch.from_numpy(kc[s]).to(dev), torch.from_numpy(vc[s]).to(dev))
            cache.advance(cached[s], s)
    for s in range(B):
        if rows[s]:
            cache.reserve(s, rows[s])
    total = sum(rows)
    q = rng.standard_normal((total, hq, d)).astype(npd)
    # k and v share one fused [rows, 2, Hkv, D] buffer: exercises row-strided inputs
    kv_new = rng.standard_normal((total, 2, hkv, d)).astype(npd)
    gq = torch.from_numpy(q).to(dev)
    gkv = torch.from_numpy(kv_new).to(dev)
    rope = rb.rope_tables(d, max_len + 1, theta, device=dev) if theta else None
    starts = np.concatenate([[0], np.cumsum(rows)]).astype(np.int32)
    kw = dict(rope=rope, variant=variant, out_dtype=torch.float32 if out_f32 else None)
    if ragged is not None:
        out = rb.gqa_prefill(cache.view(0), gq, gkv[:, 0], gkv[:, 1],
                             q_start=torch.from_numpy(starts).to(dev), **kw)
    else:
        out = rb.gqa_prefill(cache.view(0), gq, gkv[:, 0], gkv[:, 1], rows_per_seq=n, **kw)
    torch.cuda.synchronize()
    assert rb.prefill_status() == 0
    for s in range(B):
        if rows[s]:
            cache.advance(rows[s], s)
    out = out.float().cpu().numpy()
    cos, sin = (rope[0].cpu().numpy(), rope[1].cpu().numpy()) if rope else (None, None)
    worst, exact = 0.0, True
    for s in range(B):
        r0, r1 = starts[s], starts[s + 1]
        if r1 == r0:
            continue
        qs = np.ascontiguousarray(q[r0:r1].transpose(1, 0, 2))[None]    # [1, Hq, n, D]
        ks = np.ascontiguousarray(kv_new[r0:r1, 0].transpose(1, 0, 2))[None]
        vs = np.ascontiguousarray(kv_new[r0:r1, 1].transpose(1, 0, 2))[None]
        if rope:
            qs = orc.rope(qs, cos, sin, cached[s])
            ks = orc.rope(ks, cos, sin, cached[s])
        k_all = np.concatenate([kc[s][None], ks], 2)
        v_all = np.concatenate([vc[s][None], vs], 2)
        L = cached[s] + (r1 - r0)
        wide, _ = orc.attention_core_wide(qs, k_all, v_all, L, cached[s], threads=THREADS)
        want = wide[0].transpose(1, 0, 2)                                # [n, Hq, D]
        worst = max(worst, rel(out[r0:r1], want))
        tol = 2e-3 if npd == np.float16 else 1e-5
        assert elem_excess(out[r0:r1], want, tol) <= 1.0, ("float64 chain", s)
        if faithful:
            ref = orc.attention_core(qs, k_all, v_all, L, cached[s], threads=THREADS)
            ref = ref[0].transpose(1, 0, 2)
            # the faithful chain's own rounding error adds to the bound (triangle inequality)
            bound = tol + rel(ref, want)
            assert rel(out[r0:r1], ref) < bound, ("faithful chain", s, rel(out[r0:r1], ref))
        gk, gv = cache.gather(0, s)
        gk, gv = gk.cpu().numpy(), gv.cpu().numpy()
        exact &= bool(np.array_equal(gk[:, :L].view(np.uint8), k_all[0].view(np.uint8)) and
                      np.array_equal(gv[:, :L].view(np.uint8), v_all[0].view(np.uint8)))
    return worst, exact


@pytest.mark.parametrize("variant", [2, 1])
@pytest.mark.parametrize("d", [64, 128])
def test_prefill_f16_matches_oracle(cuda, orc, variant, d):
    """Tensor-core (2) and CUDA-core (1) prefill: fresh and partly cached sequences,
    GQA 4:1, a ragged last tile (200 rows = 128 + 72)."""
    err, exact = run_case(cuda, orc, hq=8, hkv=2, d=d, cached=(0, 37, 300), n=200,
                          variant=variant, seed=d + variant)
    assert exact
    assert err < 2e-3


@pytest.mark.parametrize("block_size", [16, 32, 128, 512])
def test_prefill_tc_page_sizes(cuda, orc, block_size):
    """Pages smaller than, equal to and larger than the 128-key tile."""
    err, exact = run_case(cuda, orc, hq=4, hkv=4, d=64, cached=(0, 129), n=260,
                          block_size=block_size, variant=2, seed=block_size)
    assert exact
    assert err < 2e-3


def test_prefill_tc_single_row_and_no_rope(cuda, orc):
    err, exact = run_case(cuda, orc, hq=2, hkv=1, d=128, cached=(5, 0), n=1, theta=None,
                          variant=2, seed=9)
    assert exact and err < 2e-3


def test_prefill_tc_ragged_rows(cuda, orc):
    """q_start row offsets: 5, 130, 0 and 257 new rows over 0..400 cached positions."""
    err, exact = run_case(cuda, orc, hq=6, hkv=3, d=64, cached=(400, 0, 17, 3),
                          ragged=(5, 130, 0, 257), variant=2, seed=4)
    assert exact and err < 2e-3


def test_prefill_tc_f32_output(cuda, orc):
    err, exact = run_case(cuda, orc, hq=4, hkv=2, d=64, cached=(64,), n=140, variant=2,
                          out_f32=True, seed=12)
    assert exact and err < 2e-3


def test_prefill_f32_generic(cuda, orc):
    """F32 caches run the CUDA-core kernel: 1e-5 relative."""
    err, exact = run_case(cuda, orc, npd=np.float32, hq=9, hkv=3, d=64, cached=(128, 3),
                          n=33, theta=100000.0, seed=2)
    assert exact and err < 1e-5


def test_prefill_cfg5_all_prompts(cuda, orc):
    """BASELINE config 5's whole prompt batch: 16 prompts x 512 tokens (MHA, 12 heads,
    D 64, RoPE theta 1e4, 16-token pages in a random permutation) on the tensor cores,
    every sequence against the float64 chain and the reference's faithful F16 chain."""
    err, exact = run_case(cuda, orc, hq=12, hkv=12, d=64, cached=(0,) * 16, n=512,
                          variant=2, seed=5, faithful=True)
    assert exact and err < 2e-3


def test_cache_prefill_then_decode_continues(cuda, orc):
    """tmllm_cache_prefill reserves blocks, the lengths advance by n, and a decode step on
    top of the prefilled cache equals the oracle over all positions."""
    rng = np.random.default_rng(21)
    B, hq, hkv, d, n = 3, 8, 2, 64, 150
    cache = rb.PagedKvCache(1, B, n + 4, hkv, d, dtype=torch.float16, block_size=16,
                            shuffle_seed=3, device=cuda)
    rope = rb.rope_tables(d, n + 8, 10000.0, device=cuda)
    q = rng.standard_normal((B, n, hq, d)).astype(np.float16)
    k = rng.standard_normal((B, n, hkv, d)).astype(np.float16)
    v = rng.standard_normal((B, n, hkv, d)).astype(np.float16)
    out = cache.prefill(0, torch.from_numpy(q).to(cuda), torch.from_numpy(k).to(cuda),
                        torch.from_numpy(v).to(cuda), rope=rope)
    cache.advance(n)
    assert cache.lens() == [n] * B
    qd = rng.standard_normal((B, hq, d)).astype(np.float16)
    kd = rng.standard_normal((B, hkv, d)).astype(np.float16)
    vd = rng.standard_normal((B, hkv, d)).astype(np.float16)
    dec = cache.decode(0, torch.from_numpy(qd).to(cuda), torch.from_numpy(kd).to(cuda),
                       torch.from_numpy(vd).to(cuda), rope=rope)
    torch.cuda.synchronize()
    cos, sin = rope[0].cpu().numpy(), rope[1].cpu().numpy()
    out = out.float().cpu().numpy().reshape(B, n, hq, d)
    dec = dec.float().cpu().numpy()
    for s in range(B):
        qs = orc.rope(np.ascontiguousarray(q[s].transpose(1, 0, 2))[None], cos, sin, 0)
        ks = orc.rope(np.ascontiguousarray(k[s].transpose(1, 0, 2))[None], cos, sin, 0)
        vs = np.ascontiguousarray(v[s].transpose(1, 0, 2))[None]
        wide, _ = orc.attention_core_wide(qs, ks, vs, n, 0, threads=THREADS)
        assert rel(out[s], wide[0].transpose(1, 0, 2)) < 2e-3
        qn = orc.rope(qd[s][None, :, None, :], cos, sin, n)
        kn = orc.rope(kd[s][None, :, None, :], cos, sin, n)
        kall = np.concatenate([ks, kn], 2)
        vall = np.concatenate([vs, vd[s][None, :, None, :]], 2)
        wide, _ = orc.attention_core_wide(qn, kall, vall, n + 1, n, threads=THREADS)
        assert rel(dec[s], wide[0, :, 0]) < 2e-3


def test_prefill_rejects_bad_arguments(cuda):
    cache = rb.PagedKvCache(1, 2, 40, 2, 64, dtype=torch.float16, device=cuda)
    q = torch.zeros((2, 30, 4, 64), dtype=torch.float16, device=cuda)
    kv = torch.zeros((2, 30, 2, 64), dtype=torch.float16, device=cuda)
    cache.append(0, 0, torch.zeros((2, 20, 64), dtype=torch.float16, device=cuda),
                 torch.zeros((2, 20, 64), dtype=torch.float16, device=cuda))
    cache.advance(20, 0)
    with pytest.raises(rb.PositionOutOfRange):  # 20 + 30 > 40: nothing reserved or written
        cache.prefill(0, q, kv, kv)
    assert cache.lens() == [20, 0]
    with pytest.raises(rb.ModelFormat):
        cache.prefill(0, q[:, :, :3], kv, kv)  # 3 query heads over 2 KV heads
    with pytest.raises(rb.InvalidArgument):  # the tensor-core path needs F16
        c32 = rb.PagedKvCache(1, 1, 8, 2, 64, dtype=torch.float32, device=cuda)
        z = torch.zeros((1, 4, 2, 64), device=cuda)
        c32.prefill(0, z, z, z, variant=2)
