"""TEST INFRASTRUCTURE ONLY: a float32 PyTorch restatement of the whole decoder (the
checker the GPU decoder tests compare logits and greedy tokens against).  It follows the
reference's model code path (src/model/transformer.rs, src/nn/transformer_block.rs,
src/nn/attention.rs, src/nn/rope.rs:44-62, kernels/rope.metal:57-63, kernels/rmsnorm.metal,
kernels/silu.metal) in float32 arithmetic with full causal attention over the whole
sequence: no cache, no F16 rounding of intermediates."""
from __future__ import annotations

import math

import torch

from rustllm_b200.decoder import DecoderWeights, ModelConfig


def reference_forward(cfg: ModelConfig, w: DecoderWeights, tokens: torch.Tensor) -> torch.Tensor:
    """Float32 restatement of the whole model on one sequence (tokens [S]) with full causal
    attention, used as the test reference: logits [S, vocab]."""
    f = torch.float32
    x = w.embedding[tokens.long()].to(f)
    S = x.shape[0]
    hq, hkv, d = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
    pos = torch.arange(S, device=x.device, dtype=f)
    inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, d, 2, device=x.device, dtype=f) / d))
    ang = pos[:, None] * inv[None, :]
    cos, sin = torch.cos(ang), torch.sin(ang)

    def rope(t):  # t [S, H, d], half-split pairs (kernels/rope.metal:57-63)
        a, b = t[..., : d // 2], t[..., d // 2:]
        return torch.cat([a * cos[:, None] - b * sin[:, None], b * cos[:, None] + a * sin[:, None]], -1)

    def norm(t, wt):
        return t * torch.rsqrt((t * t).mean(-1, keepdim=True) + cfg.rms_norm_eps) * wt.to(f)

    mask = torch.full((S, S), float("-inf"), device=x.device).triu(1)
    for L in w.layers:
        hn = norm(x, L["attn_norm"])
        qkv = hn @ L["wqkv"].to(f)
        q = rope(qkv[:, : hq * d].view(S, hq, d))
        k = rope(qkv[:, hq * d:(hq + hkv) * d].view(S, hkv, d))
        v = qkv[:, (hq + hkv) * d:].view(S, hkv, d)
        k = k.repeat_interleave(hq // hkv, dim=1)
        v = v.repeat_interleave(hq // hkv, dim=1)
        att = torch.einsum("shd,thd->hst", q, k) / math.sqrt(d) + mask
        o = torch.einsum("hst,thd->shd", att.softmax(-1), v).reshape(S, hq * d)
        x = x + o @ L["wo"].to(f)
        hn = norm(x, L["mlp_norm"])
        gu = hn @ L["wgu"].to(f)
        g_, u_ = gu[:, : cfg.intermediate_size], gu[:, cfg.intermediate_size:]
        x = x + (g_ * torch.sigmoid(g_) * u_) @ L["wd"].to(f)
    return norm(x, w.final_norm) @ w.lm_head.to(f)
