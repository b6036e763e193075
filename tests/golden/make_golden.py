"""Writes the committed golden fixtures of the parity tests.

1. ``reference_kats.json`` — the known-answer tests of the reference's own test suite for
   this path (Lee-Dongwook/RustLLM, Rust ``#[test]`` functions), transcribed as data with
   their file:line.  The reference is Rust + Apple Metal and cannot run on Linux, so these
   transcribed inputs and asserted outputs are what pins the oracle.
2. ``oracle_fixtures.npz`` — seeded inputs and the CPU oracle's outputs (faithful and
   float64) for small cases of the decode path, including BASELINE config 1.

Run from the repository root:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
import math
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import oracle as orc  # noqa: E402


def reference_kats() -> list[dict]:
    kats = []
    # src/model/kv_cache.rs:214-258 — two decode appends into a [1,2,8,4] F16 cache.
    kats.append({
        "name": "kv_cache_two_decode_appends",
        "ref": "src/model/kv_cache.rs:214-258",
        "dtype": "f16", "num_kv_heads": 2, "max": 8, "dim": 4,
        "appends": [
            {"key": [1, 2, 3, 4, 5, 6, 7, 8], "value": [10, 20, 30, 40, 50, 60, 70, 80],
             "shape": [1, 2, 1, 4]},
            {"key": [9, 10, 11, 12, 13, 14, 15, 16],
             "value": [90, 100, 110, 120, 130, 140, 150, 160], "shape": [1, 2, 1, 4]},
        ],
        "expect_len": 2, "expect_key_shape": [1, 2, 2, 4],
        "expect_key": [1, 2, 3, 4, 9, 10, 11, 12, 5, 6, 7, 8, 13, 14, 15, 16],
    })
    # src/model/kv_cache.rs:261-273 — prefill append of three positions.
    kats.append({
        "name": "kv_cache_prefill_append",
        "ref": "src/model/kv_cache.rs:261-273",
        "dtype": "f16", "num_kv_heads": 2, "max": 8, "dim": 4,
        "appends": [{"key": [1.0] * 24, "value": [2.0] * 24, "shape": [1, 2, 3, 4]}],
        "expect_len": 3, "expect_key_shape": [1, 2, 3, 4],
    })
    # src/model/kv_cache.rs:276-293 — one append of [1,2,1,2].
    kats.append({
        "name": "kv_cache_append_updates_prefix",
        "ref": "src/model/kv_cache.rs:276-293",
        "dtype": "f16", "num_kv_heads": 2, "max": 8, "dim": 2,
        "appends": [{"key": [1.0] * 4, "value": [2.0] * 4, "shape": [1, 2, 1, 2]}],
        "expect_len": 1, "expect_key_shape": [1, 2, 1, 2],
    })
    # src/model/kv_cache.rs:296-306 — an F16 cache rejects F32 input; len stays 0.
    kats.append({
        "name": "kv_cache_rejects_dtype_mismatch",
        "ref": "src/model/kv_cache.rs:296-306",
        "dtype": "f16", "num_kv_heads": 2, "max": 8, "dim": 4,
        "input_dtype": "f32", "shape": [1, 2, 1, 4], "expect_error": True, "expect_len": 0,
    })
    # src/tensor/tensor.rs:791-818 — repeat_kv(3) of [1,2,2,2].
    kats.append({
        "name": "repeat_kv_r3",
        "ref": "src/tensor/tensor.rs:791-818",
        "input": [1, 2, 3, 4, 10, 20, 30, 40], "shape": [1, 2, 2, 2], "repeats": 3,
        "expect_shape": [1, 6, 2, 2],
        "expect": [1, 2, 3, 4, 1, 2, 3, 4, 1, 2, 3, 4, 10, 20, 30, 40, 10, 20, 30, 40,
                   10, 20, 30, 40],
    })
    # src/tensor/tensor.rs:821-831 — repeat_kv(1) is the identity.
    kats.append({
        "name": "repeat_kv_r1",
        "ref": "src/tensor/tensor.rs:821-831",
        "input": [1, 2, 3, 4], "shape": [1, 1, 2, 2], "repeats": 1,
        "expect_shape": [1, 1, 2, 2], "expect": [1, 2, 3, 4],
    })
    # src/tensor/tensor.rs:850-876 — gqa_qk == batched_matmul(q, repeat_kv(k,3)^T).
    kats.append({
        "name": "gqa_qk_equals_repeat_bmm",
        "ref": "src/tensor/tensor.rs:850-876",
        "q": [(i - 20.0) / 13.0 for i in range(48)], "q_shape": [1, 6, 2, 4],
        "k": [(i - 11.0) / 7.0 for i in range(24)], "k_shape": [1, 2, 3, 4],
        "tol_f32": 1e-4, "tol_f16": 0.05,
    })
    # src/tensor/tensor.rs:879-902 — gqa_pv == batched_matmul(p, repeat_kv(v,3)).
    kats.append({
        "name": "gqa_pv_equals_repeat_bmm",
        "ref": "src/tensor/tensor.rs:879-902",
        "p": [(i + 1.0) / 100.0 for i in range(36)], "p_shape": [1, 6, 2, 3],
        "v": [(i - 9.0) / 8.0 for i in range(24)], "v_shape": [1, 2, 3, 4],
        "tol_f32": 1e-4, "tol_f16": 0.05,
    })
    # src/tensor/tensor.rs:905-926 — F16 batched matmul within 0.05 of F32.
    kats.append({
        "name": "bmm_f16_close_to_f32",
        "ref": "src/tensor/tensor.rs:905-926",
        "a": [1, 2, 3, 4, 1, 2, 3, 4], "a_shape": [2, 2, 2],
        "b": [1, 0, 0, 1, 2, 2, 2, 2], "b_shape": [2, 2, 2], "tol": 0.05,
    })
    # src/tensor/tensor.rs:952-982 — q . k^T with a materialised transposed key, F16 vs F32.
    kats.append({
        "name": "bmm_transposed_keys",
        "ref": "src/tensor/tensor.rs:952-982",
        "q": [1, 2, 3, 4, 5, 6, 7, 8], "q_shape": [1, 2, 2, 2],
        "k": [1, 0, 0, 1, 2, 1, 1, 2], "k_shape": [1, 2, 2, 2], "tol": 0.05,
    })
    # src/tensor/tensor.rs:985-1004 — F16 scale/mask within 0.01 of F32, infinities kept.
    kats.append({
        "name": "scale_mask_prefill",
        "ref": "src/tensor/tensor.rs:985-1004",
        "scores": [1, 2, 3, 4, 5, 6, 7, 8, 9], "shape": [1, 1, 3, 3], "scale": 0.5, "start": 0,
        "tol": 0.01,
    })
    # src/tensor/tensor.rs:1007-1019 — decode position keeps every key, exact values.
    kats.append({
        "name": "scale_mask_decode_keeps_all",
        "ref": "src/tensor/tensor.rs:1007-1019",
        "scores": [1, 2, 3, 4], "shape": [1, 1, 1, 4], "scale": 0.5, "start": 3,
        "expect": [0.5, 1.0, 1.5, 2.0],
    })
    # src/tensor/tensor.rs:1022-1035 — position 2 masks key 3.
    kats.append({
        "name": "scale_mask_intermediate_masks_future",
        "ref": "src/tensor/tensor.rs:1022-1035",
        "scores": [1, 2, 3, 4], "shape": [1, 1, 1, 4], "scale": 0.5, "start": 2,
        "expect": [0.5, 1.0, 1.5, "-inf"],
    })
    # src/tensor/tensor.rs:1038-1057 — F16 softmax within 0.01 of F32; rows sum to 1 +- 0.01.
    kats.append({
        "name": "softmax_rows",
        "ref": "src/tensor/tensor.rs:1038-1057",
        "input": [1, 2, 3, 4, 5, 6], "shape": [2, 3], "tol": 0.01, "row_sum_tol": 0.01,
    })
    # src/tensor/tensor.rs:1060-1089 — masked probabilities are exactly zero.
    kats.append({
        "name": "mask_softmax_zeros",
        "ref": "src/tensor/tensor.rs:1060-1089",
        "scores": [1, 2, 3, 4, 5, 6, 7, 8, 9], "shape": [1, 1, 3, 3], "scale": 0.5, "start": 0,
        "tol": 0.01, "expect_zero_indices": [1, 2, 5],
    })
    # src/nn/attention.rs:591-668 — fused attention core == op-by-op chain (1e-5),
    # (Hq, Hkv) in {(2,2), (3,1)}, D=4, q_len=3, start_pos=2, key == value.
    kats.append({
        "name": "attention_core_matches_op_chain",
        "ref": "src/nn/attention.rs:591-668",
        "cases": [[2, 2], [3, 1]], "head_dim": 4, "seq_len": 3, "start_pos": 2,
        "query_rule": "(i % 5) - 2", "cached_rule": "(i % 3) - 1", "tol": 1e-5,
    })
    # src/nn/rope.rs:186-208 — F16 RoPE within 0.01 of F32 (D=4, max 8, theta 1e4, start 1).
    kats.append({
        "name": "rope_f16_close_to_f32",
        "ref": "src/nn/rope.rs:186-208",
        "input": [0.125, -1.25, 2.5, 3.75, -0.5, 1.5, -2.25, 4.0], "shape": [1, 1, 2, 4],
        "head_dim": 4, "max_seq_len": 8, "theta": 10000.0, "start": 1, "tol": 0.01,
    })
    # src/nn/attention.rs:534-560 — GQA prefill of 2 positions keeps the cache compact.
    kats.append({
        "name": "gqa_cache_stays_compact",
        "ref": "src/nn/attention.rs:534-560",
        "num_kv_heads": 1, "max": 8, "dim": 4, "q_heads": 3, "prefill": 2,
        "expect_key_shape": [1, 1, 2, 4],
    })
    # src/nn/attention.rs:736-766 — prefill of 3 then a decode step: len 3 then 4.
    kats.append({
        "name": "prefill_then_decode_lengths",
        "ref": "src/nn/attention.rs:736-766",
        "num_kv_heads": 2, "max": 8, "dim": 2, "prefill": 3, "expect_lens": [3, 4],
    })
    return kats


def oracle_fixtures() -> dict[str, np.ndarray]:
    out: dict[str, np.ndarray] = {}
    # SmolLM2-135M attention shape, F32, Hq 9, Hkv 3, D 64, cache
    # pre-filled to 128 with K,V ~ N(0,1), q,k,v ~ N(0,1) appended at 128, RoPE theta 1e5,
    # scale 1/8.  Seed 1234.
    rng = np.random.default_rng(1234)
    hq, hkv, d, cached, cap = 9, 3, 64, 128, 129
    k_cache = np.zeros((1, hkv, cap, d), np.float32)
    v_cache = np.zeros((1, hkv, cap, d), np.float32)
    k_cache[:, :, :cached] = rng.standard_normal((1, hkv, cached, d), dtype=np.float32)
    v_cache[:, :, :cached] = rng.standard_normal((1, hkv, cached, d), dtype=np.float32)
    q = rng.standard_normal((1, hq, 1, d), dtype=np.float32)
    k = rng.standard_normal((1, hkv, 1, d), dtype=np.float32)
    v = rng.standard_normal((1, hkv, 1, d), dtype=np.float32)
    cos, sin = orc.rope_tables(d, cap, 100000.0)
    out.update({"cfg1_k_cache": k_cache.copy(), "cfg1_v_cache": v_cache.copy(), "cfg1_q": q,
                "cfg1_k": k, "cfg1_v": v, "cfg1_cos": cos, "cfg1_sin": sin})
    kc, vc = k_cache.copy(), v_cache.copy()
    o = orc.decode_step(q, k, v, kc, vc, cached, cos, sin)
    qr = orc.rope(q, cos, sin, cached)
    wide, lse = orc.attention_core_wide(qr, kc, vc, cached + 1, cached)
    out.update({"cfg1_out": o, "cfg1_out_wide": wide, "cfg1_lse_wide": lse,
                "cfg1_k_row_after": kc[:, :, cached], "cfg1_v_row_after": vc[:, :, cached]})

    # F16 decode with the Llama-3 head size (D 128, G 4) at a short length.
    rng = np.random.default_rng(4321)
    hq, hkv, d, cached = 8, 2, 128, 150
    kd = rng.standard_normal((1, hkv, cached + 1, d), dtype=np.float32).astype(np.float16)
    vd = rng.standard_normal((1, hkv, cached + 1, d), dtype=np.float32).astype(np.float16)
    q = rng.standard_normal((1, hq, 1, d), dtype=np.float32).astype(np.float16)
    kd[:, :, cached:] = 0
    vd[:, :, cached:] = 0
    kn = rng.standard_normal((1, hkv, 1, d), dtype=np.float32).astype(np.float16)
    vn = rng.standard_normal((1, hkv, 1, d), dtype=np.float32).astype(np.float16)
    out.update({"f16_k_cache": kd.copy(), "f16_v_cache": vd.copy(), "f16_q": q, "f16_k": kn,
                "f16_v": vn})
    kc, vc = kd.copy(), vd.copy()
    o = orc.decode_step(q, kn, vn, kc, vc, cached)
    wide, lse = orc.attention_core_wide(q, kc, vc, cached + 1, cached)
    out.update({"f16_out": o, "f16_out_wide": wide, "f16_lse_wide": lse})
    return out


def main() -> None:
    with open(os.path.join(HERE, "reference_kats.json"), "w") as f:
        json.dump({"source": "Lee-Dongwook/RustLLM unit tests, transcribed",
                   "kats": reference_kats()}, f, indent=1)
    np.savez_compressed(os.path.join(HERE, "oracle_fixtures.npz"), **oracle_fixtures())
    print("wrote", os.listdir(HERE))


if __name__ == "__main__":
    main()
