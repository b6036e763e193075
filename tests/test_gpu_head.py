"""tmllm_lm_head (the end of a decode step: final RMSNorm, the vocabulary head and the greedy
pick in one launch) against a float32 PyTorch restatement of the reference's chain
(kernels/rmsnorm.metal's stored half rows, the lm_head product with F32 sums, F16 logits)
and against this library's separate kernels: the normed rows are those of
tmllm_add_rmsnorm bit for bit (so the logits equal the head over those rows exactly), and
the token ids equal tmllm_argmax over the stored logits exactly.  Logit tolerance: 2e-3
relative to the largest logit (a few F16 ulps where the F32 sums differ in order)."""
from __future__ import annotations

import pytest
import torch

import rustllm_b200 as rb
from rustllm_b200 import _lib
from rustllm_b200.decoder import head_fits, head_workspace, linear, lm_head

pytestmark = pytest.mark.gpu

H = torch.float16


def rel(a, b) -> float:
    a, b = a.double(), b.double()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def stream(dev):
    return torch.cuda.current_stream(dev).cuda_stream


def reference(x, w, *, norm=None, eps=1e-5, residual=None):
    f = torch.float32
    a = x.to(f)
    if residual is not None:  # kernels/vector_add.metal: the sum stored as half
        a = (a + residual.to(f)).to(H).to(f)
    if norm is not None:  # kernels/rmsnorm.metal: half(x * rsqrt(mean(x^2) + eps) * w)
        a = (a * torch.rsqrt((a * a).mean(-1, keepdim=True) + eps) * norm.to(f)).to(H).to(f)
    return (a @ w.to(f)).to(H)


def add_rmsnorm(x, residual, weight, eps=1e-5):
    out = torch.empty_like(x)
    _lib.call("tmllm_add_rmsnorm", 1, x.data_ptr(),
              residual.data_ptr() if residual is not None else None, weight.data_ptr(),
              out.data_ptr(), None, x.shape[0], x.shape[1], eps, stream(x.device))
    return out


def argmax(logits):
    ids = torch.empty(logits.shape[0], dtype=torch.int32, device=logits.device)
    _lib.call("tmllm_argmax", 1, logits.data_ptr(), ids.data_ptr(), logits.shape[0],
              logits.shape[1], stream(logits.device))
    return ids


def inputs(dev, rows, k, n, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn((rows, k), generator=g, device=dev).to(H)
    w = (torch.randn((k, n), generator=g, device=dev) * 0.02).to(H)
    nw = (1 + 0.1 * torch.randn(k, generator=g, device=dev)).to(H)
    return g, x, w, nw


@pytest.mark.parametrize("rows", [1, 5, 16, 17, 33, 64])
@pytest.mark.parametrize("k,n", [(576, 49152), (768, 32000), (960, 49152), (200, 136),
                                 (64, 8)])
def test_head_matches_float32_and_the_separate_kernels(cuda, rows, k, n):
    """The BASELINE models' heads (SmolLM2 576 x 49152 and 960 x 49152, TinyStories 768 x
    32000) and ragged sizes (a partial column tile, K not a multiple of the 64-row stage,
    fewer columns than one warp's share)."""
    _, x, w, nw = inputs(cuda, rows, k, n, rows * 31 + k)
    ws = head_workspace(device=cuda)
    ids = torch.full((rows,), -7, dtype=torch.int32, device=cuda)
    got = lm_head(x, w, norm_weight=nw, ids=ids, workspace=ws)
    assert rel(got, reference(x, w, norm=nw)) < 2e-3
    # the fused norm gives tmllm_add_rmsnorm's rows bit for bit
    assert torch.equal(got, lm_head(add_rmsnorm(x, None, nw), w))
    assert torch.equal(ids, argmax(got))
    assert int(ws.count_nonzero()) == 0  # the workspace is left zeroed


@pytest.mark.parametrize("rows", [1, 16, 64])
def test_residual_add_before_the_norm(cuda, rows):
    """x + residual rounded to F16 first (the last layer's output joining the residual
    stream), as tmllm_add_rmsnorm does it."""
    g, x, w, nw = inputs(cuda, rows, 960, 49152, 5 + rows)
    r = torch.randn((rows, 960), generator=g, device=cuda).to(H)
    ws = head_workspace(device=cuda)
    ids = torch.empty(rows, dtype=torch.int32, device=cuda)
    got = lm_head(x, w, norm_weight=nw, residual=r, ids=ids, workspace=ws)
    assert rel(got, reference(x, w, norm=nw, residual=r)) < 2e-3
    assert torch.equal(got, lm_head(add_rmsnorm(x, r, nw), w))
    assert torch.equal(ids, argmax(got))
    plain = lm_head(x, w, residual=r)  # the add without a norm
    assert rel(plain, reference(x, w, residual=r)) < 2e-3


def test_greedy_pick_semantics(cuda):
    """sampler.rs:79-88: the last of equal maxima wins, and a row whose logits are all
    infinite (F16 overflow) has no token (-1)."""
    rows, k, n = 3, 64, 49152
    x = torch.zeros((rows, k), dtype=H, device=cuda)
    x[:, 0] = 1.0
    w = (torch.randn((k, n), device=cuda) * 0.01).to(H)
    w[0, 100] = 8.0   # row 0 and 1: columns 100 and 40000 tie at the maximum
    w[0, 40000] = 8.0
    w[0, 3] = 7.0
    x[2, :] = 30000.0  # row 2: with an all-ones weight every logit overflows to +inf
    w2 = w.clone()
    w2[:, :] = 1.0
    ws = head_workspace(device=cuda)
    ids = torch.empty(rows, dtype=torch.int32, device=cuda)
    lm_head(x[:2].contiguous(), w, ids=ids[:2], workspace=ws)
    assert ids[:2].tolist() == [40000, 40000]
    logits = lm_head(x, w2, ids=ids, workspace=ws)
    assert torch.isinf(logits[2].float()).all()
    assert int(ids[2]) == -1 and ids[:2].tolist() == [n - 1, n - 1]  # all equal: the last
    assert torch.equal(ids, argmax(logits))


def test_repeated_calls_share_one_workspace(cuda):
    """Each call leaves the workspace zeroed, so consecutive calls of different row counts
    on one workspace give the same ids as fresh workspaces."""
    ws = head_workspace(device=cuda)
    for rows, seed in ((64, 1), (3, 2), (64, 3), (16, 4), (1, 5)):
        _, x, w, nw = inputs(cuda, rows, 576, 49152, seed)
        ids = torch.empty(rows, dtype=torch.int32, device=cuda)
        fresh = torch.empty(rows, dtype=torch.int32, device=cuda)
        a = lm_head(x, w, norm_weight=nw, ids=ids, workspace=ws)
        b = lm_head(x, w, norm_weight=nw, ids=fresh, workspace=head_workspace(device=cuda))
        assert torch.equal(a, b) and torch.equal(ids, fresh)
        assert torch.equal(ids, argmax(a))


def test_overlapped_head_reads_the_previous_result(cuda):
    """With the overlapped launch the weight stream starts under the kernel ahead, but the
    rows are read only after it: a projection that writes x right before gives the head
    of the new x."""
    g, x, w, nw = inputs(cuda, 16, 960, 49152, 9)
    wd = (torch.randn((2560, 960), generator=g, device=cuda) * 0.02).to(H)
    act = torch.randn((16, 2560), generator=g, device=cuda).to(H)
    ws = head_workspace(device=cuda)
    ids = torch.empty(16, dtype=torch.int32, device=cuda)
    for _ in range(3):
        xr = x.clone()
        linear(act, wd, residual=xr, out=xr, overlap=True)
        got = lm_head(xr, w, norm_weight=nw, ids=ids, workspace=ws, overlap=True)
        torch.cuda.synchronize(cuda)
        assert torch.equal(got, lm_head(xr, w, norm_weight=nw))
        assert torch.equal(ids, argmax(got))


def test_head_fits_and_rejects(cuda):
    assert head_fits(64, 960, 49152) and head_fits(1, 4096, 32000)
    assert not head_fits(65, 960, 49152) and not head_fits(64, 1408, 49152)
    x = torch.zeros((65, 64), dtype=H, device=cuda)
    w = torch.zeros((64, 64), dtype=H, device=cuda)
    with pytest.raises(rb.InvalidShape):  # more than 64 rows
        lm_head(x, w)
    with pytest.raises(rb.ModelFormat):
        lm_head(x[:4], torch.zeros((32, 64), dtype=H, device=cuda))
    with pytest.raises(rb.UnsupportedDType):
        lm_head(x[:4].float(), w.float())
    with pytest.raises(rb.InvalidArgument):  # ids without a workspace
        lm_head(x[:4], w, ids=torch.empty(4, dtype=torch.int32, device=cuda))
