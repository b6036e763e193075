"""tmllm_linear (the decode step's projections with RMSNorm, SwiGLU and residual add fused)
against a float32 PyTorch restatement of the reference's unfused chain: the same F16 storage
roundings (normed rows, gate and up, the projection before the residual add) with float32
products in between.  Tolerance: 2e-3 relative to the largest output (a few F16 ulps where
the F32 sums differ in order), and bit-identical results across repeated calls."""
from __future__ import annotations

import pytest
import torch

import rustllm_b200 as rb
from rustllm_b200.decoder import linear, linear_stats, linear_status

pytestmark = pytest.mark.gpu

H = torch.float16


def rel(a, b) -> float:
    a, b = a.double(), b.double()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def reference(x, w, *, norm=None, eps=1e-5, residual=None, swiglu=False):
    f = torch.float32
    a = x.to(f)
    if norm is not None:  # kernels/rmsnorm.metal: half(x * rsqrt(mean(x^2) + eps) * w)
        a = (a * torch.rsqrt((a * a).mean(-1, keepdim=True) + eps) * norm.to(f)).to(H).to(f)
    y = a @ w.to(f)
    if swiglu:  # kernels/silu.metal on the stored gate and up
        n = w.shape[1] // 2
        g, u = y[:, :n].to(H).to(f), y[:, n:].to(H).to(f)
        return (g / (1 + torch.exp(-g)) * u).to(H)
    if residual is not None:  # kernels/vector_add.metal on the stored projection
        return (residual.to(f) + y.to(H).to(f)).to(H)
    return y.to(H)


def inputs(dev, rows, k, n, seed, *, swiglu=False):
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn((rows, k), generator=g, device=dev).to(H)
    w = (torch.randn((k, 2 * n if swiglu else n), generator=g, device=dev) / k ** 0.5).to(H)
    return g, x, w


@pytest.mark.parametrize("rows", [1, 7, 16, 33, 64])
@pytest.mark.parametrize("k,n", [(576, 960), (4096, 512), (200, 136), (1536, 576),
                                 (768, 32000), (7200, 64)])
def test_plain_projection(cuda, rows, k, n):
    """Unsplit (many column tiles) and split-K (few tiles, long K) plans; K and N that are
    not multiples of the tiles."""
    _, x, w = inputs(cuda, rows, k, n, rows * 7 + k)
    got = linear(x, w)
    assert rel(got, reference(x, w)) < 2e-3
    assert linear_status() == 0


@pytest.mark.parametrize("rows", [1, 5, 12, 64])
@pytest.mark.parametrize("k,n", [(576, 960), (2048, 256)])
def test_norm_fused_into_projection(cuda, rows, k, n):
    g, x, w = inputs(cuda, rows, k, n, 3 + rows)
    nw = (1 + 0.1 * torch.randn(k, generator=g, device=cuda)).to(H)
    got = linear(x, w, norm_weight=nw, eps=1e-5)
    assert rel(got, reference(x, w, norm=nw, eps=1e-5)) < 2e-3


@pytest.mark.parametrize("rows", [1, 9, 24, 64])
@pytest.mark.parametrize("k,n", [(576, 1536), (960, 2560), (4096, 256)])
def test_norm_and_swiglu(cuda, rows, k, n):
    g, x, w = inputs(cuda, rows, k, n, 11 + rows, swiglu=True)
    nw = (1 + 0.1 * torch.randn(k, generator=g, device=cuda)).to(H)
    got = linear(x, w, norm_weight=nw, swiglu=True)
    assert got.shape == (rows, n)
    assert rel(got, reference(x, w, norm=nw, swiglu=True)) < 2e-3


@pytest.mark.parametrize("rows", [1, 13, 64])
@pytest.mark.parametrize("k,n", [(1536, 576), (4096, 1024)])
def test_residual_in_place(cuda, rows, k, n):
    """out aliases the residual (the decoder's residual stream x += x_in · W)."""
    g, x, w = inputs(cuda, rows, k, n, 5 + rows)
    r = torch.randn((rows, n), generator=g, device=cuda).to(H)
    want = reference(x, w, residual=r)
    linear(x, w, residual=r, out=r)
    assert rel(r, want) < 2e-3


@pytest.mark.parametrize("rows", [16, 40])
@pytest.mark.parametrize("overlap", [False, True])
def test_strided_rows_and_repeat_calls_are_identical(cuda, overlap, rows):
    """Row strides wider than a row (x a column slice, out a column slice); repeated calls
    (split K over a cluster) give bit-identical results, with and without the overlapped
    launch."""
    g = torch.Generator(device=cuda).manual_seed(9)
    big = torch.randn((rows, 1024), generator=g, device=cuda).to(H)
    x = big[:, 256:256 + 512]
    w = (torch.randn((512, 256), generator=g, device=cuda) / 23).to(H)
    out = torch.zeros((rows, 384), dtype=H, device=cuda)
    linear(x, w, out=out[:, 64:320], overlap=overlap)
    first = out.clone()
    assert rel(out[:, 64:320], reference(x.contiguous(), w)) < 2e-3
    assert int(out[:, :64].abs().sum()) == 0 and int(out[:, 320:].abs().sum()) == 0
    for _ in range(3):
        linear(x, w, out=out[:, 64:320], overlap=overlap)
        assert torch.equal(out, first)


@pytest.mark.parametrize("rows", [8, 24])
def test_overlapped_chain_reads_the_previous_result(cuda, rows):
    """A chain of overlapped projections where each reads (and adds into) the rows the
    previous one wrote: the same as the chain launched without overlap."""
    g = torch.Generator(device=cuda).manual_seed(31)
    x0 = torch.randn((rows, 512), generator=g, device=cuda).to(H)
    ws = [(torch.randn((512, 512), generator=g, device=cuda) / 23).to(H) for _ in range(6)]
    nw = (1 + 0.1 * torch.randn(512, generator=g, device=cuda)).to(H)
    res = []
    for overlap in (False, True):
        x = x0.clone()
        st = linear_stats(512, device=cuda)
        h = torch.empty_like(x)
        for i, w in enumerate(ws):
            if i % 2 == 0:
                linear(x, w, norm_weight=nw, stats_in=st if i else None, out=h, overlap=overlap)
            else:
                linear(h, w, residual=x, out=x, stats_out=st, overlap=overlap)
        res.append(x.clone())
    assert torch.equal(res[0], res[1])


@pytest.mark.parametrize("rows", [1, 11, 19, 64])
def test_row_statistics_chain(cuda, rows):
    """A residual projection writes the row statistics of its output; the norm-fused
    projection that reads them equals one that recomputes them from the rows, and the
    float32 chain (O + residual, then norm + gate/up + SwiGLU)."""
    k, n, inter = 960, 1000, 512
    g, x, w = inputs(cuda, rows, k, n, 40 + rows)
    r = torch.randn((rows, n), generator=g, device=cuda).to(H)
    wgu = (torch.randn((n, 2 * inter), generator=g, device=cuda) / n ** 0.5).to(H)
    nw = (1 + 0.1 * torch.randn(n, generator=g, device=cuda)).to(H)
    st = linear_stats(n, device=cuda)
    h = r.clone()
    linear(x, w, residual=h, out=h, stats_out=st)
    sq = (h.float() ** 2).sum(-1)
    got_sq = st.view(-1, 64)[:, :rows].sum(0)
    assert float(((got_sq - sq).abs() / sq).max()) < 1e-5
    a = linear(h, wgu, norm_weight=nw, swiglu=True, stats_in=st)
    b = linear(h, wgu, norm_weight=nw, swiglu=True)
    assert rel(a, b) < 2e-3
    want = reference(reference(x, w, residual=r), wgu, norm=nw, swiglu=True)
    assert rel(a, want) < 2e-3


def test_rows_do_not_interact(cuda):
    """Row r of a 64-row call equals the same row computed alone and in 8-, 9- and 16-row
    calls, bit for bit (the summation order depends on K and N only)."""
    g, x, w = inputs(cuda, 64, 960, 2560, 4, swiglu=True)
    nw = (1 + 0.1 * torch.randn(960, generator=g, device=cuda)).to(H)
    full = linear(x, w, norm_weight=nw, swiglu=True)
    for r in (0, 7, 40, 63):
        one = linear(x[r:r + 1].contiguous(), w, norm_weight=nw, swiglu=True)
        assert torch.equal(one[0], full[r])
    for r, lo in ((7, 0), (9, 1), (40, 32), (63, 48)):
        part = linear(x[lo:r + 1].contiguous(), w, norm_weight=nw, swiglu=True)
        assert torch.equal(part[r - lo], full[r])


def test_rejects_bad_arguments(cuda):
    x = torch.zeros((65, 64), dtype=H, device=cuda)
    w = torch.zeros((64, 64), dtype=H, device=cuda)
    with pytest.raises(rb.InvalidShape):  # more than 64 rows
        linear(x, w)
    with pytest.raises(rb.InvalidShape):  # K not a multiple of 8
        linear(torch.zeros((2, 60), dtype=H, device=cuda), torch.zeros((60, 64), dtype=H,
                                                                           device=cuda))
    with pytest.raises(rb.ModelFormat):
        linear(x[:4], torch.zeros((32, 64), dtype=H, device=cuda))
    with pytest.raises(rb.UnsupportedDType):
        linear(x[:4].float(), w.float())
    with pytest.raises(rb.InvalidArgument):  # statistics without a norm
        linear(x[:4], w, stats_in=linear_stats(64, device=cuda))
    with pytest.raises(rb.InvalidArgument):  # SwiGLU and a residual together
        linear(x[:4], torch.zeros((64, 128), dtype=H, device=cuda), swiglu=True,
               residual=torch.zeros((4, 64), dtype=H, device=cuda))
