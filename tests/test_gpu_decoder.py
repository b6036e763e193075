"""The decoder around the decode path (embedding, add+RMSNorm, SwiGLU, argmax, GEMMs, the
fused attention) against a float32 PyTorch restatement of the same model, plus graph
replay against eager decoding.  Tolerances: kernels 1e-2 relative (F16 storage), model
logits 3e-2 relative to the largest logit after a few F16 layers."""
from __future__ import annotations

import ctypes as C

import pytest
import torch

import rustllm_b200 as rb
from rustllm_b200 import _lib
from rustllm_b200.decoder import Decoder, DecoderWeights, GraphedDecoder, ModelConfig

from model_reference import reference_forward

pytestmark = pytest.mark.gpu

TINY = ModelConfig(vocab_size=1000, hidden_size=256, intermediate_size=512, num_layers=2,
                   num_heads=4, num_kv_heads=2, max_seq_len=96, rms_norm_eps=1e-5,
                   rope_theta=10000.0)


def rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).abs().max() / b.abs().max())


def stream(dev):
    return torch.cuda.current_stream(dev).cuda_stream


def test_embedding_gathers_rows(cuda):
    table = torch.randn((50, 24), device=cuda).half()
    ids = torch.tensor([3, 0, 49, 7, 3], dtype=torch.int32, device=cuda)
    out = torch.empty((5, 24), dtype=torch.float16, device=cuda)
    bad = torch.zeros(1, dtype=torch.int32, device=cuda)
    _lib.call("tmllm_embedding", 1, table.data_ptr(), ids.data_ptr(), out.data_ptr(), 5, 24, 50,
              bad.data_ptr(), stream(cuda))
    assert torch.equal(out, table[ids.long()]) and int(bad) == 0
    ids[2] = 50  # outside the table: zero row, flag set
    _lib.call("tmllm_embedding", 1, table.data_ptr(), ids.data_ptr(), out.data_ptr(), 5, 24, 50,
              bad.data_ptr(), stream(cuda))
    assert int(bad) == 1 and torch.count_nonzero(out[2]) == 0


@pytest.mark.parametrize("hidden", [576, 960, 100, 2048, 2056])
def test_add_rmsnorm_matches_float32(cuda, hidden):
    """Warp-per-row kernel (hidden % 8 == 0, <= 2048) and the block-per-row kernel."""
    rows = 17
    x = torch.randn((rows, hidden), device=cuda).half()
    r = torch.randn((rows, hidden), device=cuda).half()
    w = (torch.rand(hidden, device=cuda) + 0.5).half()
    out = torch.empty_like(x)
    s = (x.float() + r.float()).half()
    want = s.float() * torch.rsqrt((s.float() ** 2).mean(-1, keepdim=True) + 1e-5) * w.float()
    xs = x.clone()
    _lib.call("tmllm_add_rmsnorm", 1, xs.data_ptr(), r.data_ptr(), w.data_ptr(), out.data_ptr(),
              xs.data_ptr(), rows, hidden, 1e-5, stream(cuda))  # in-place residual update
    assert torch.equal(xs, s)
    assert rel(out, want) < 1e-2
    with pytest.raises(rb.InvalidShape):
        _lib.call("tmllm_add_rmsnorm", 1, x.data_ptr(), None, w.data_ptr(), out.data_ptr(), None,
                  3, hidden, 0.0, stream(cuda))


@pytest.mark.parametrize("inter", [300, 320])
def test_swiglu_matches_float32(cuda, inter):
    """Scalar (300) and 16-byte vector (320) kernels."""
    gu = torch.randn((4, 2 * inter), device=cuda).half()
    out = torch.empty((4, inter), dtype=torch.float16, device=cuda)
    _lib.call("tmllm_swiglu", 1, gu.data_ptr(), out.data_ptr(), 4, inter, stream(cuda))
    g, u = gu[:, :inter].float(), gu[:, inter:].float()
    assert rel(out, g * torch.sigmoid(g) * u) < 1e-2


def test_argmax_takes_last_of_equal_maxima(cuda):
    """src/generation/sampler.rs:79-88 keeps the last maximum (Iterator::max_by)."""
    logits = torch.randn((3, 49152), device=cuda).half()
    logits[1, 100] = 30.0
    logits[1, 40000] = 30.0
    logits[2, 7] = 20.0
    ids = torch.empty(3, dtype=torch.int32, device=cuda)
    _lib.call("tmllm_argmax", 1, logits.data_ptr(), ids.data_ptr(), 3, 49152, stream(cuda))
    assert int(ids[0]) == int(logits[0].float().argmax())
    assert int(ids[1]) == 40000 and int(ids[2]) == 7


def greedy_from_slice(row):
    """sampler.rs:79-88 restated: finite logits only, f32::total_cmp, last maximum wins;
    None when no logit is finite."""
    import struct
    best, best_i = None, None
    for i, v in enumerate(row):
        if v != v or v in (float("inf"), float("-inf")):
            continue
        u = struct.unpack("<I", struct.pack("<f", v))[0]
        key = (~u & 0xFFFFFFFF) if u & 0x80000000 else (u | 0x80000000)
        if best is None or key >= best:
            best, best_i = key, i
    return best_i


@pytest.mark.parametrize("dtype,code", [(torch.float16, 1), (torch.float32, 0)])
@pytest.mark.parametrize("vocab", [49152, 1003])
def test_argmax_follows_greedy_from_slice(cuda, dtype, code, vocab):
    """Non-finite logits are skipped (even +inf), -0 < +0 under total_cmp, ties go to the
    last index, a row without a finite logit gives -1; 16-byte rows (vectorised loads) and
    odd rows (scalar loads), F16 and F32."""
    g = torch.Generator(device=cuda).manual_seed(vocab + code)
    x = torch.randn((6, vocab), generator=g, device=cuda).to(dtype)
    x[0, 5] = float("inf")              # skipped: the finite maximum wins
    x[0, 9] = float("nan")
    x[1].fill_(-1.0)
    x[1, 3] = -0.0
    x[1, 4] = 0.0                       # +0 above -0
    x[1, 2] = -0.0
    x[2].fill_(float("nan"))
    x[2, 0] = float("-inf")             # nothing finite: -1
    x[3].fill_(2.5)                     # all equal: the last index
    x[4, vocab - 1] = 50.0              # the tail of an odd row
    x[5, 0] = 50.0
    x[5, vocab // 2] = 50.0
    ids = torch.empty(6, dtype=torch.int32, device=cuda)
    _lib.call("tmllm_argmax", code, x.data_ptr(), ids.data_ptr(), 6, vocab, stream(cuda))
    host = x.float().cpu().tolist()
    for r in range(6):
        want = greedy_from_slice(host[r])
        assert int(ids[r]) == (-1 if want is None else want), r
    assert int(ids[1]) == 4 and int(ids[2]) == -1 and int(ids[3]) == vocab - 1
    assert int(ids[5]) == vocab // 2


def test_decoder_logits_match_float32_model(cuda):
    w = DecoderWeights(TINY, device=cuda, seed=1, std=0.08)
    dec = Decoder(TINY, w, 1, device=cuda)
    prompt = torch.randint(0, TINY.vocab_size, (12,), generator=torch.Generator().manual_seed(2))
    want = reference_forward(TINY, w, prompt.to(cuda))
    for t in range(12):
        dec.ids.copy_(prompt[t:t + 1].to(torch.int32))
        dec.forward_step()
        dec.cache.advance(1)
        assert rel(dec.logits[0], want[t]) < 3e-2, t
    assert dec.cache.len(0) == 12


def test_batched_decode_matches_single_sequences(cuda):
    w = DecoderWeights(TINY, device=cuda, seed=3, std=0.08)
    g = torch.Generator().manual_seed(4)
    prompts = torch.randint(0, TINY.vocab_size, (3, 9), generator=g)
    batch = Decoder(TINY, w, 3, device=cuda, shuffle_seed=9)
    nb = batch.prefill(prompts.to(cuda))
    toks = batch.decode(6, nb)
    for s in range(3):
        single = Decoder(TINY, w, 1, device=cuda)
        n1 = single.prefill(prompts[s:s + 1].to(cuda))
        assert int(n1[0]) == int(nb[s])
        t1 = single.decode(6, n1)
        assert torch.equal(t1[:, 0], toks[:, s])


def test_graph_replay_equals_eager_decoding(cuda):
    cfg = TINY
    w = DecoderWeights(cfg, device=cuda, seed=5, std=0.08)
    prompts = torch.randint(0, cfg.vocab_size, (2, 5), generator=torch.Generator().manual_seed(6))
    eager = Decoder(cfg, w, 2, device=cuda)
    first = eager.prefill(prompts.to(cuda))
    want = eager.decode(10, first)
    graphed = Decoder(cfg, w, 2, device=cuda)
    first2 = graphed.prefill(prompts.to(cuda))
    assert torch.equal(first, first2)
    graphed.ids.copy_(first2)
    runner = GraphedDecoder(graphed, 10)
    got = []
    for _ in range(10):
        runner.step()
        got.append(graphed.ids.clone())  # the graph fed the chosen token back
    assert torch.equal(torch.stack(got), want)
    assert graphed.cache.lens() == [15, 15]


def test_invalid_prompt_token_rejected(cuda):
    w = DecoderWeights(TINY, device=cuda, seed=0)
    dec = Decoder(TINY, w, 1, device=cuda)
    with pytest.raises(rb.InvalidArgument):
        dec.prefill(torch.tensor([[1, TINY.vocab_size]], device=cuda))


def test_prefill_logits_match_float32_model(cuda):
    """Whole-prompt prefill (one pass per layer through the fused prefill attention) of two
    prompts of 150 tokens: the last row's logits equal the float32 model's."""
    w = DecoderWeights(TINY, device=cuda, seed=7, std=0.08)
    g = torch.Generator().manual_seed(8)
    prompts = torch.randint(0, TINY.vocab_size, (2, 150), generator=g)
    dec = Decoder(TINY, w, 2, device=cuda, max_seq_len=160, shuffle_seed=4)
    nxt = dec.prefill(prompts.to(cuda))
    assert dec.cache.lens() == [150, 150]
    for s in range(2):
        want = reference_forward(TINY, w, prompts[s].to(cuda))[-1]
        assert rel(dec.logits[s], want) < 3e-2
        assert int(nxt[s]) == int(dec.logits[s].float().argmax())


def test_prefill_then_decode_matches_stepwise(cuda):
    """Decoding after a whole-prompt prefill gives the logits of decoding after a
    token-by-token prefill."""
    w = DecoderWeights(TINY, device=cuda, seed=11, std=0.08)
    prompts = torch.randint(0, TINY.vocab_size, (2, 40), generator=torch.Generator().manual_seed(12))
    a = Decoder(TINY, w, 2, device=cuda)
    b = Decoder(TINY, w, 2, device=cuda)
    a.prefill(prompts.to(cuda))
    b.prefill_stepwise(prompts.to(cuda))
    assert rel(a.logits, b.logits) < 2e-2
    nxt = torch.tensor([3, 5], dtype=torch.int32, device=cuda)
    for dec in (a, b):
        dec.ids.copy_(nxt)
        dec.forward_step()
    assert rel(a.logits, b.logits) < 2e-2


def test_model_dir_round_trip_gives_identical_logits(cuda, tmp_path):
    """A model written as the reference's model.bin + config.json and loaded back
    (Transformer::load, transformer.rs:193-201) decodes exactly like the original."""
    from rustllm_b200.weights import load_model_dir, save_config_json
    w = DecoderWeights(TINY, device=cuda, seed=13, std=0.08)
    w.to_weights(TINY).save(tmp_path / "model.bin")
    save_config_json(TINY, tmp_path / "config.json")
    cfg, w2 = load_model_dir(tmp_path, device=cuda)
    assert cfg == TINY
    prompts = torch.randint(0, TINY.vocab_size, (2, 20), generator=torch.Generator().manual_seed(14))
    a, b = Decoder(TINY, w, 2, device=cuda), Decoder(cfg, w2, 2, device=cuda)
    assert torch.equal(a.prefill(prompts.to(cuda)), b.prefill(prompts.to(cuda)))
    assert torch.equal(a.logits, b.logits)
    with pytest.raises(rb.InvalidShape, match="has shape"):
        bad = w.to_weights(TINY)
        bad["lm_head.weight"].data = bad["lm_head.weight"].data[:, :10].copy()
        bad["lm_head.weight"].shape = (TINY.hidden_size, 10)
        DecoderWeights.from_weights(TINY, bad, device=cuda)


@pytest.mark.parametrize("batch", [4, 40])
def test_fused_step_matches_library_step(cuda, batch):
    """The decode step with fused projections (tmllm_linear: norm, SwiGLU and residual adds
    folded in) gives the logits of the step built from cuBLAS GEMMs and the separate norm
    and SwiGLU kernels, for a few sequences (fused head too) and for a batch above 16 (the
    cuBLAS head after fused projections)."""
    w = DecoderWeights(TINY, device=cuda, seed=13, std=0.08)
    prompts = torch.randint(0, TINY.vocab_size, (batch, 20),
                            generator=torch.Generator().manual_seed(14))
    a = Decoder(TINY, w, batch, device=cuda)
    b = Decoder(TINY, w, batch, device=cuda)
    assert a.fused
    b.fused = False
    for dec in (a, b):
        dec.prefill(prompts.to(cuda))
    for _ in range(4):
        ids = a.next_ids.clone()
        for dec in (a, b):
            dec.ids.copy_(ids)
            dec.forward_step()
            dec.cache.advance(1)
        assert rel(a.logits, b.logits) < 2e-2


@pytest.mark.parametrize("variant,d", [(0, 64), (2, 128), (1, 64), (1, 128)])
def test_overlapped_decode_after_projection(cuda, variant, d):
    """TMLLM_DECODE_OVERLAP right behind a projection that writes q, k_new and v_new
    (tmllm_linear lets its dependents start as soon as it runs, so the decode really can
    start early): the tensor-core kernel reads them only after its grid-dependency wait, and
    the CUDA-core kernel (variant 1), which has no such wait, is launched plainly whatever
    the flag says.  Either way the result is bit-identical to the plain launch."""
    from rustllm_b200.decoder import linear
    B, hq, hkv, n, hidden = 3, 8, 2, 300, 256
    W = (hq + 2 * hkv) * d
    g = torch.Generator(device=cuda).manual_seed(17)
    wq = (torch.randn((hidden, W), generator=g, device=cuda) / 16).half()
    x = torch.randn((B, hidden), generator=g, device=cuda).half()
    kv_rows = [torch.randn((hkv, n - 40 * s, d), generator=g, device=cuda).half()
               for s in range(B)]
    outs = []
    for flags in (0, 1):
        cache = rb.PagedKvCache(1, B, n + 2, hkv, d, dtype=torch.float16, block_size=16,
                                shuffle_seed=2, device=cuda)
        for s in range(B):
            cache.append(0, s, kv_rows[s], kv_rows[s])
            cache.advance(n - 40 * s, s)
            cache.reserve(s, 1)
        qkv = torch.full((B, W), 3.0, dtype=torch.float16, device=cuda)  # stale values
        out = torch.empty((B, hq, d), dtype=torch.float16, device=cuda)
        torch.cuda.synchronize()
        opts = _lib.DecodeOpts(q_seq_stride=W, kv_seq_stride=W, flags=flags, variant=variant)
        base, es = qkv.data_ptr(), qkv.element_size()
        linear(x, wq, out=qkv, overlap=True)  # the kernel right ahead writes q, k_new, v_new
        _lib.call("tmllm_cache_decode", cache.handle, 0, base, base + hq * d * es,
                  base + (hq + hkv) * d * es, out.data_ptr(), None, hq, C.byref(opts),
                  stream(cuda))
        torch.cuda.synchronize()
        cache.advance(1)  # the appended rows are compared too
        k, v = cache.gather(0, 0)
        outs.append((out.clone(), k.clone(), v.clone()))
    assert all(torch.equal(a, b) for a, b in zip(outs[0], outs[1]))
    assert not torch.equal(outs[0][1][:, -1], torch.full_like(outs[0][1][:, -1], 3.0))


def test_overlapped_decode_launch_matches_plain(cuda):
    """TMLLM_DECODE_OVERLAP (the attention's K/V prefetch overlapping the kernel ahead) gives
    bit-identical outputs and appended rows to the plain launch, also right after a kernel
    that writes q and k_new."""
    B, hq, hkv, d, n = 3, 8, 2, 64, 300
    outs = []
    for flags in (0, 1):
        cache = rb.PagedKvCache(1, B, n + 2, hkv, d, dtype=torch.float16, block_size=16,
                                shuffle_seed=2, device=cuda)
        g = torch.Generator(device=cuda).manual_seed(3)
        for s in range(B):
            x = torch.randn((hkv, n - 40 * s, d), generator=g, device=cuda).half()
            cache.append(0, s, x, x)
            cache.advance(n - 40 * s, s)
            cache.reserve(s, 1)
        qkv = torch.empty((B, (hq + 2 * hkv) * d), dtype=torch.float16, device=cuda)
        src = torch.randn((B, (hq + 2 * hkv) * d), generator=g, device=cuda).half()
        out = torch.empty((B, hq, d), dtype=torch.float16, device=cuda)
        w = qkv.shape[1]
        opts = _lib.DecodeOpts(q_seq_stride=w, kv_seq_stride=w, flags=flags)
        base, es = qkv.data_ptr(), qkv.element_size()
        qkv.copy_(src * 1.5)  # the kernel right ahead writes q, k_new and v_new
        _lib.call("tmllm_cache_decode", cache.handle, 0, base, base + hq * d * es,
                  base + (hq + hkv) * d * es, out.data_ptr(), None, hq, C.byref(opts),
                  stream(cuda))
        torch.cuda.synchronize()
        k, v = cache.gather(0, 0)
        outs.append((out.clone(), k.clone(), v.clone()))
    assert all(torch.equal(a, b) for a, b in zip(outs[0], outs[1]))
    with pytest.raises(rb.InvalidArgument):
        opts = _lib.DecodeOpts(flags=2)
        _lib.call("tmllm_cache_decode", cache.handle, 0, base, base + hq * d * es,
                  base + (hq + hkv) * d * es, out.data_ptr(), None, hq, C.byref(opts),
                  stream(cuda))


def _greedy_against_float32(cuda, preset, B, prompt_len, steps, seed, check_seqs):
    """Whole-prompt prefill then `steps` greedy decode steps of a BASELINE model shape
    (random-init weights N(0, 0.02)); every emitted token's logits against the float32
    restatement run over the prompt plus the tokens emitted before it."""
    from rustllm_b200.decoder import PRESETS
    cfg = PRESETS[preset]
    w = DecoderWeights(cfg, device=cuda, seed=seed)
    prompts = torch.randint(0, cfg.vocab_size, (B, prompt_len),
                            generator=torch.Generator().manual_seed(seed + 1))
    dec = Decoder(cfg, w, B, device=cuda, max_seq_len=prompt_len + steps + 2,
                  shuffle_seed=seed)
    nxt = dec.prefill(prompts.to(cuda))
    logits, toks = [dec.logits.float().clone()], [nxt.clone()]
    for _ in range(steps):
        dec.ids.copy_(nxt)
        dec.forward_step()
        dec.cache.advance(1)
        logits.append(dec.logits.float().clone())
        nxt = dec.next_ids.clone()
        toks.append(nxt)
    assert dec.cache.lens() == [prompt_len + steps] * B
    toks = torch.stack(toks)  # [steps + 1, B]
    clear = 0
    for s in check_seqs:
        seq = torch.cat([prompts[s].to(cuda), toks[:-1, s].long()])
        want = reference_forward(cfg, w, seq)[prompt_len - 1:]  # row t: token t's logits
        for t in range(steps + 1):
            got, ref = logits[t][s], want[t]
            err = float((got - ref).abs().max())
            # the reference's own model-level bound (F16 model vs F32 model, absolute per
            # logit: src/model/transformer.rs:576-597) and a norm-relative one
            assert err < 0.2, (s, t, err)
            assert rel(got, ref) < 3e-2, (s, t, rel(got, ref))
            top = ref.topk(2).values
            if float(top[0] - top[1]) > 2 * err:  # the float32 model's choice is clear
                assert int(toks[t, s]) == int(ref.argmax()), (s, t)
                clear += 1
            if t < 2:  # the first greedy tokens are identical in any case
                assert int(toks[t, s]) == int(ref.argmax()), (s, t)
    return clear


def test_decoder_config2_shape_greedy_tokens(cuda):
    """BASELINE config 2's model (SmolLM2-135M shape: 30 layers, hidden 576, 9 / 3 heads,
    vocab 49152), batch 1, a 32-token prompt, then 8 greedy tokens."""
    assert _greedy_against_float32(cuda, "smollm2-135m", 1, 32, 8, 21, [0]) >= 5


def test_decoder_config5_shape_greedy_tokens(cuda):
    """BASELINE config 5's model (TinyStories-110M shape: 12 layers, dim 768, 12 heads MHA,
    vocab 32000), 16 prompts x 512 tokens through the tensor-core prefill, then 4 greedy
    tokens for every sequence, all 16 checked."""
    assert _greedy_against_float32(cuda, "tinystories-110m", 16, 512, 4, 31,
                                   list(range(16))) >= 40
