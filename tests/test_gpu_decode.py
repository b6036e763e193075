"""Fused KV-append + GQA decode attention (the hot path) against the CPU oracle.

Tolerances (from the north star): attention outputs within 1e-5 relative for F32 and 2e-3
for F16.  Against the oracle's float64 chain (the exact result of the same inputs) this is
checked two ways: norm-relative, max|gpu - ref| / max|ref| over a sequence's output, and
element by element, |gpu - ref| <= tol * (|ref| + rms(ref)) (a per-element relative bound
whose floor, tol * rms, keeps outputs near zero from demanding more than the storage
precision).  The faithful chain (the reference's own F16 store points for scores,
probabilities and outputs) itself sits up to ~1.7e-3 from the exact result at config 3's
lengths, so against it the bound is the triangle inequality's: norm-relative within
tol + rel(faithful, float64).  The appended K/V rows and block tables are bit-exact."""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import rustllm_b200 as rb

pytestmark = pytest.mark.gpu

TOL = {np.float32: 1e-5, np.float16: 2e-3}


def rel(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def elem_excess(a, b, tol) -> float:
    """max over elements of |a - b| / (tol * (|b| + rms(b))): <= 1 passes the element-wise
    bound."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    rms = float(np.sqrt(np.mean(b * b)))
    return float(np.max(np.abs(a - b) / (tol * (np.abs(b) + rms) + 1e-300)))


def assert_close(got, want, tol, what="", elementwise=True):
    r = rel(got, want)
    e = elem_excess(got, want, tol) if elementwise else 0.0
    assert r < tol and e <= 1.0, (what, r, e)


def bits(x: np.ndarray) -> np.ndarray:
    return x.view(np.uint16 if x.dtype == np.float16 else np.uint32)


def torch_dtype(npd):
    return torch.float16 if npd == np.float16 else torch.float32


class Case:
    """A paged cache filled with seeded N(0,1) K/V for `lens`, plus one decode token."""

    def __init__(self, dev, npd, hq, hkv, d, lens, block_size=16, seed=0, layers=1,
                 max_len=None, shuffle=True, theta=None, std=1.0):
        rng = np.random.default_rng(seed)
        self.npd, self.hq, self.hkv, self.d, self.lens = npd, hq, hkv, d, list(lens)
        self.B = len(lens)
        self.max_len = max_len or (max(lens) + 2)
        bs = block_size or self.max_len
        self.cache = rb.PagedKvCache(layers, self.B, self.max_len, hkv, d, dtype=torch_dtype(npd),
                                     block_size=bs, shuffle_seed=(seed + 1) if shuffle else 0,
                                     device=dev)
        self.k = [(rng.standard_normal((hkv, n, d)) * std).astype(npd) for n in lens]
        self.v = [rng.standard_normal((hkv, n, d)).astype(npd) for n in lens]
        for s in range(self.B):
            if lens[s]:
                for layer in range(layers):
                    self.cache.append(layer, s, torch.from_numpy(self.k[s]).to(dev),
                                      torch.from_numpy(self.v[s]).to(dev))
                self.cache.advance(lens[s], s)
        self.q = (rng.standard_normal((self.B, hq, d)) * std).astype(npd)
        self.kn = (rng.standard_normal((self.B, hkv, d)) * std).astype(npd)
        self.vn = rng.standard_normal((self.B, hkv, d)).astype(npd)
        self.rope = None
        self.tables = None
        if theta is not None:
            cos, sin = rb.rope_tables(d, self.max_len + 1, theta, device=dev)
            self.rope = (cos, sin)
            self.tables = (cos.cpu().numpy(), sin.cpu().numpy())
        self.dev = dev

    def gpu(self, append=True, **kw):
        q = torch.from_numpy(self.q).to(self.dev)
        kn = torch.from_numpy(self.kn).to(self.dev) if append else None
        vn = torch.from_numpy(self.vn).to(self.dev) if append else None
        out, lse = self.cache.decode(0, q, kn, vn, want_lse=True, rope=self.rope, **kw)
        return out.float().cpu().numpy(), lse.cpu().numpy()

    def oracle(self, orc, s, append=True):
        """(faithful, wide, lse, appended_k_row) for sequence s."""
        n = self.lens[s]
        q = self.q[s][None, :, None, :]
        kn = self.kn[s][None, :, None, :]
        vn = self.vn[s][None, :, None, :]
        if self.tables is not None:
            q = orc.rope(np.ascontiguousarray(q), *self.tables, n)
            kn = orc.rope(np.ascontiguousarray(kn), *self.tables, n)
        L = n + (1 if append else 0)
        kc = np.zeros((1, self.hkv, max(L, 1), self.d), self.npd)
        vc = np.zeros_like(kc)
        kc[0, :, :n] = self.k[s]
        vc[0, :, :n] = self.v[s]
        if append:
            kc[0, :, n] = kn[0, :, 0]
            vc[0, :, n] = vn[0, :, 0]
        faithful = orc.attention_core(np.ascontiguousarray(q), kc, vc, L, L - 1)
        wide, lse = orc.attention_core_wide(np.ascontiguousarray(q), kc, vc, L, L - 1)
        return faithful[0, :, 0], wide[0, :, 0], lse[0, :, 0], kn[0, :, 0]


def check(case: Case, orc, got, lse, append=True, tol=None):
    tol = tol or TOL[case.npd]
    for s in range(case.B):
        faithful, wide, wlse, _ = case.oracle(orc, s, append)
        assert_close(got[s], wide, tol, ("float64 chain", s))
        assert_close(got[s], faithful, tol + rel(faithful, wide), ("faithful chain", s),
                     elementwise=False)
        assert np.max(np.abs(lse[s] - wlse)) < 1e-3 * max(1.0, float(np.max(np.abs(wlse))))


def test_config1_fixture(cuda, orc, fixtures):
    """BASELINE config 1 (F32, Hq 9 / Hkv 3, D 64, 128 cached, RoPE theta 1e5) through the
    reference's contiguous layout (block = capacity), RoPE fused into the kernel."""
    f = fixtures
    cache = rb.PagedKvCache(1, 1, 129, 3, 64, dtype=torch.float32, block_size=129, device=cuda)
    cache.append(0, 0, torch.from_numpy(f["cfg1_k_cache"][0, :, :128].copy()).to(cuda),
                 torch.from_numpy(f["cfg1_v_cache"][0, :, :128].copy()).to(cuda))
    cache.advance(128, 0)
    rope = (torch.from_numpy(f["cfg1_cos"]).to(cuda), torch.from_numpy(f["cfg1_sin"]).to(cuda))
    out = cache.decode(0, torch.from_numpy(f["cfg1_q"][:, :, 0].copy()).to(cuda),
                       torch.from_numpy(f["cfg1_k"][:, :, 0].copy()).to(cuda),
                       torch.from_numpy(f["cfg1_v"][:, :, 0].copy()).to(cuda), rope=rope)
    got = out.cpu().numpy()[0]
    assert_close(got, f["cfg1_out"][0, :, 0], 1e-5, "faithful chain", elementwise=False)
    assert_close(got, f["cfg1_out_wide"][0, :, 0], 1e-5, "float64 chain")
    cache.advance(1, 0)
    k, v = cache.gather(0, 0)
    assert np.array_equal(bits(k.cpu().numpy()[:, 128]), bits(f["cfg1_k_row_after"][0]))
    assert np.array_equal(bits(v.cpu().numpy()[:, 128]), bits(f["cfg1_v_row_after"][0]))


def test_f16_fixture(cuda, orc, fixtures):
    f = fixtures
    cache = rb.PagedKvCache(1, 1, 160, 2, 128, dtype=torch.float16, block_size=16,
                            shuffle_seed=5, device=cuda)
    cache.append(0, 0, torch.from_numpy(f["f16_k_cache"][0, :, :150].copy()).to(cuda),
                 torch.from_numpy(f["f16_v_cache"][0, :, :150].copy()).to(cuda))
    cache.advance(150, 0)
    out = cache.decode(0, torch.from_numpy(f["f16_q"][:, :, 0].copy()).to(cuda),
                       torch.from_numpy(f["f16_k"][:, :, 0].copy()).to(cuda),
                       torch.from_numpy(f["f16_v"][:, :, 0].copy()).to(cuda))
    got = out.float().cpu().numpy()[0]
    assert_close(got, f["f16_out"][0, :, 0], 2e-3, "faithful chain", elementwise=False)
    assert_close(got, f["f16_out_wide"][0, :, 0], 2e-3, "float64 chain")


CASES = [
    # npd, hq, hkv, d, lens, block_size, theta
    (np.float16, 32, 8, 128, [5000], 16, None),
    (np.float16, 9, 3, 64, [1, 17, 300], 16, 100000.0),
    (np.float16, 12, 12, 64, [512, 100], 16, None),
    (np.float16, 4, 2, 256, [700, 33], 16, None),
    (np.float32, 10, 2, 128, [129, 640], 16, 10000.0),
    (np.float32, 9, 3, 64, [128], 0, 100000.0),
    (np.float16, 16, 2, 128, [1000], 24, None),
    (np.float16, 15, 5, 64, [256, 2048, 1111, 300], 16, None),
    (np.float16, 2, 1, 4, [3, 7], 16, 10000.0),
    (np.float32, 3, 1, 4, [4], 0, 10000.0),
    (np.float16, 6, 2, 96, [200], 16, None),
    (np.float32, 4, 4, 2, [9], 4, None),
    (np.float16, 32, 8, 128, [0, 15, 16, 31], 16, None),
    (np.float16, 24, 3, 64, [777, 5, 64, 0], 24, 10000.0),  # D = 64, G = 8, ragged pages
    (np.float16, 7, 7, 64, [4099, 31], 48, None),
]


def variants(npd, d, hq, hkv):
    """Kernel variants a case can run: automatic, plus both explicit kernels where the
    tensor-core one applies (F16, D 64/128) and the CUDA-core one exists (G <= 8)."""
    out = [0]
    if npd == np.float16 and d in (64, 128):
        out.append(2)
        if hq // hkv <= 8:
            out.append(1)
    return out


@pytest.mark.parametrize("npd,hq,hkv,d,lens,bs,theta,variant",
                         [c + (v,) for c in CASES for v in variants(c[0], c[3], c[1], c[2])])
def test_decode_matches_oracle(cuda, orc, npd, hq, hkv, d, lens, bs, theta, variant):
    case = Case(cuda, npd, hq, hkv, d, lens, block_size=bs, seed=sum(lens) + d, theta=theta)
    got, lse = case.gpu(variant=variant)
    check(case, orc, got, lse)
    # the appended rows landed in their paged slots, bit-exact
    case.cache.advance(1)
    for s in range(case.B):
        k, v = case.cache.gather(0, s)
        _, _, _, kn = case.oracle(orc, s)
        assert np.array_equal(bits(k.cpu().numpy()[:, lens[s]]), bits(kn))
        assert np.array_equal(bits(v.cpu().numpy()[:, lens[s]]), bits(case.vn[s]))


@pytest.mark.parametrize("splits", [1, 2, 7, 64])
@pytest.mark.parametrize("variant", [1, 2])
def test_split_count_does_not_change_results(cuda, orc, splits, variant):
    case = Case(cuda, np.float16, 32, 8, 128, [3000, 17], seed=3)
    got, lse = case.gpu(num_splits=splits, variant=variant)
    check(case, orc, got, lse)
    # repeated calls reuse the workspace tickets: identical results
    for _ in range(3):
        again, _ = case.gpu(num_splits=splits, variant=variant)
        assert np.array_equal(again, got)


def test_group_of_sixteen_on_tensor_cores(cuda, orc):
    case = Case(cuda, np.float16, 32, 2, 64, [500, 77], seed=16)
    got, lse = case.gpu()
    check(case, orc, got, lse)


def test_attend_without_append(cuda, orc):
    """k_new = v_new = None attends the cached prefix only (the non-owning ranks of a
    sequence split)."""
    case = Case(cuda, np.float16, 8, 2, 128, [777, 64], seed=8)
    got, lse = case.gpu(append=False)
    check(case, orc, got, lse, append=False)


def test_f32_output_for_partials(cuda, orc):
    case = Case(cuda, np.float16, 8, 2, 128, [900], seed=9)
    q = torch.from_numpy(case.q).to(cuda)
    kn, vn = torch.from_numpy(case.kn).to(cuda), torch.from_numpy(case.vn).to(cuda)
    out = case.cache.decode(0, q, kn, vn, out_dtype=torch.float32)
    assert out.dtype == torch.float32
    _, wide, _, _ = case.oracle(orc, 0)
    assert rel(out.cpu().numpy()[0], wide) < 1e-3


def test_raw_entry_point_over_caller_tensors(cuda, orc):
    """tmllm_gqa_decode over torch-owned arenas, block table and lengths."""
    rng = np.random.default_rng(12)
    hq, hkv, d, bs, n = 16, 4, 128, 16, 1234
    nb = (n + 1 + bs - 1) // bs + 3
    k_ar = torch.zeros((nb, hkv, bs, d), dtype=torch.float16, device=cuda)
    v_ar = torch.zeros_like(k_ar)
    perm = rng.permutation(nb)[: (n + bs) // bs + 1].astype(np.int32)
    table = torch.from_numpy(perm[None, :].copy()).to(cuda)
    lens = torch.tensor([n], dtype=torch.int32, device=cuda)
    kd = rng.standard_normal((hkv, n, d)).astype(np.float16)
    vd = rng.standard_normal((hkv, n, d)).astype(np.float16)
    ka, va = np.zeros((nb, hkv, bs, d), np.float16), np.zeros((nb, hkv, bs, d), np.float16)
    orc.paged_scatter(ka, perm[None, :], 0, 0, kd, bs)
    orc.paged_scatter(va, perm[None, :], 0, 0, vd, bs)
    k_ar.copy_(torch.from_numpy(ka))
    v_ar.copy_(torch.from_numpy(va))
    kv = rb.paged_kv_from_tensors(k_ar, v_ar, table, lens)
    ws = rb.DecodeWorkspace(1, hq, hkv, d, device=cuda)
    q = rng.standard_normal((1, hq, d)).astype(np.float16)
    kn = rng.standard_normal((1, hkv, d)).astype(np.float16)
    vn = rng.standard_normal((1, hkv, d)).astype(np.float16)
    out = rb.gqa_decode(kv, torch.from_numpy(q).to(cuda), torch.from_numpy(kn).to(cuda),
                        torch.from_numpy(vn).to(cuda), ws, max_len_hint=n + 1)
    kc = np.concatenate([kd, kn[0][:, None]], 1)[None]
    vc = np.concatenate([vd, vn[0][:, None]], 1)[None]
    wide, _ = orc.attention_core_wide(q[:, :, None], kc, vc, n + 1, n)
    assert rel(out.float().cpu().numpy(), wide[:, :, 0]) < 2e-3
    blk, off = perm[n // bs], n % bs
    assert np.array_equal(bits(k_ar[blk, :, off].cpu().numpy()), bits(kn[0]))


@pytest.mark.parametrize("n,rows,d,out_dtype", [
    (5, 32, 128, torch.float32),   # warp per row, 16-byte loads
    (8, 37, 64, torch.float16),    # rows not a multiple of the 4 rows of a block, F16 out
    (33, 9, 128, torch.float32),   # more parts than a warp's lanes: one block per row
    (3, 10, 66, torch.float32),    # D not a multiple of 4 floats: one block per row
])
def test_merge_lse_kernel(cuda, orc, n, rows, d, out_dtype):
    rng = np.random.default_rng(13 + n + d)
    po = rng.standard_normal((n, rows, d)).astype(np.float32)
    pl = (rng.standard_normal((n, rows)) * 3).astype(np.float32)
    pl[0, 1] = -np.inf  # a part that saw no key
    pl[:, 2] = -np.inf  # a row no part saw: zeros and -inf
    want, wlse = orc.merge_lse(po, pl)
    lse = torch.empty(rows, dtype=torch.float32, device=cuda)
    got = rb.merge_lse(torch.from_numpy(po).to(cuda), torch.from_numpy(pl).to(cuda),
                       out_dtype=out_dtype, out_lse=lse)
    tol = 1e-5 if out_dtype == torch.float32 else 2e-3
    finite = np.isfinite(wlse)
    assert rel(got.float().cpu().numpy()[finite], want[finite]) < tol
    assert np.max(np.abs(lse.cpu().numpy()[finite] - wlse[finite])) < 1e-4
    assert not got.float()[2].any() and lse[2].item() == -np.inf


def test_decode_rejects_full_cache_without_mutation(cuda):
    case = Case(cuda, np.float16, 4, 2, 64, [10], seed=1, max_len=10, shuffle=False)
    before = case.cache.block_table(0)
    with pytest.raises(rb.PositionOutOfRange):
        case.gpu()
    assert case.cache.len(0) == 10 and case.cache.block_table(0) == before


def test_config4_full_size_against_oracle(cuda, orc):
    """BASELINE config 4 at full size (F16, Hq 32, Hkv 8, D 128, 131072 cached + 1): the
    fused kernel against the float64 oracle and the faithful F16 chain (both threaded),
    plus the constant-V identity."""
    hq, hkv, d, n = 32, 8, 128, 131072
    g = torch.Generator(device=cuda).manual_seed(4)
    kd = torch.randn((hkv, n, d), generator=g, device=cuda).half()
    vd = torch.randn((hkv, n, d), generator=g, device=cuda).half()
    cache = rb.PagedKvCache(1, 1, n + 1, hkv, d, dtype=torch.float16, block_size=16,
                            shuffle_seed=44, device=cuda)
    cache.append(0, 0, kd, vd)
    cache.advance(n, 0)
    q = torch.randn((1, hq, d), generator=g, device=cuda).half()
    kn = torch.randn((1, hkv, d), generator=g, device=cuda).half()
    vn = torch.randn((1, hkv, d), generator=g, device=cuda).half()
    out, lse = cache.decode(0, q, kn, vn, want_lse=True)
    kc = torch.cat([kd, kn[0][:, None]], 1)[None].cpu().numpy()
    vc = torch.cat([vd, vn[0][:, None]], 1)[None].cpu().numpy()
    import os
    threads = os.cpu_count() or 8
    qn = q[:, :, None].cpu().numpy()
    wide, wlse = orc.attention_core_wide(qn, kc, vc, n + 1, n, threads=threads)
    got = out.float().cpu().numpy()
    assert_close(got, wide[:, :, 0], 2e-3, "float64 chain")
    assert np.max(np.abs(lse.cpu().numpy() - wlse[:, :, 0])) < 1e-2
    # and the reference's own chain with its F16 store points (scores, probabilities)
    faithful = orc.attention_core(qn, kc, vc, n + 1, n, threads=threads)
    assert_close(got, faithful[:, :, 0], 2e-3 + rel(faithful[:, :, 0], wide[:, :, 0]),
                 "faithful chain", elementwise=False)
    # softmax weights sum to one: a constant V row gives back that constant
    cache2 = rb.PagedKvCache(1, 1, n + 1, hkv, d, dtype=torch.float16, block_size=16,
                             device=cuda)
    const = torch.linspace(-2, 2, d, device=cuda).half()
    vconst = const.expand(hkv, n, d).contiguous()
    cache2.append(0, 0, kd, vconst)
    cache2.advance(n, 0)
    out2 = cache2.decode(0, q, kn, const.expand(1, hkv, d).contiguous())
    assert float((out2.float() - const.float()).abs().max()) < 2e-3


def test_config3_attention_full_batch(cuda, orc):
    """BASELINE config 3's attention op at its real batch: 64 sequences with context lengths
    U[256, 2048] (seeded as the bench draws them), Hq 15 / Hkv 5 / D 64, 16-token pages in a
    random permutation, the split count the cache chooses from the actual lengths.  Every
    sequence against the faithful and the float64 chain; every appended row bit-exact."""
    gen = torch.Generator().manual_seed(1234)
    lens = torch.randint(256, 2049, (64,), generator=gen).tolist()
    case = Case(cuda, np.float16, 15, 5, 64, lens, block_size=16, seed=1234)
    got, lse = case.gpu()
    check(case, orc, got, lse)
    case.cache.advance(1)
    for s in range(case.B):
        k, v = case.cache.gather(0, s)
        _, _, _, kn = case.oracle(orc, s)
        assert np.array_equal(bits(k.cpu().numpy()[:, lens[s]]), bits(kn))
        assert np.array_equal(bits(v.cpu().numpy()[:, lens[s]]), bits(case.vn[s]))
