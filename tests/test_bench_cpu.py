"""The host-side legs of bench.py that need no GPU: the whole-model CPU baseline of the
decoder lines runs the reference's chain (numpy products, the C oracle's RoPE and faithful
attention) and reports a positive token rate within its time box."""
from __future__ import annotations

import torch

import bench
from rustllm_b200.decoder import DecoderWeights, ModelConfig

TINY = ModelConfig(vocab_size=500, hidden_size=128, intermediate_size=256, num_layers=2,
                   num_heads=4, num_kv_heads=2, max_seq_len=256, rms_norm_eps=1e-5,
                   rope_theta=10000.0)


def test_decoder_cpu_baseline_runs_the_chain():
    w = DecoderWeights(TINY, device=torch.device("cpu"), seed=3)
    n, secs, sample = bench.decoder_cpu_time(TINY, w, [17, 100, 33], 0.3, 2)
    assert n >= 3 and secs > 0
    assert "3 sequence(s)" in sample and "2 layers" in sample
