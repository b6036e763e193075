"""The paged KV cache runtime on the GPU: the reference's LayerKvCache known answers,
bit-exact paged layout against the oracle, block tables, and reject-without-mutation."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import rustllm_b200 as rb

pytestmark = pytest.mark.gpu


def f16(values, shape, dev):
    return torch.tensor(values, dtype=torch.float32).reshape(shape).half().to(dev)


@pytest.mark.parametrize("block_size", [None, 1, 3])
def test_layer_cache_two_decode_appends(cuda, kats, block_size):
    """src/model/kv_cache.rs:214-258 (contiguous and paged layouts)."""
    k = kats["kv_cache_two_decode_appends"]
    cache = rb.LayerKvCache(k["num_kv_heads"], k["max"], k["dim"], torch.float16, cuda,
                            block_size=block_size)
    assert cache.dtype == torch.float16 and cache.len() == 0 and cache.is_empty()
    for ap in k["appends"]:
        cache.append(f16(ap["key"], ap["shape"], cuda), f16(ap["value"], ap["shape"], cuda))
    assert cache.len() == k["expect_len"]
    key = cache.key()
    assert list(key.shape) == k["expect_key_shape"] and key.dtype == torch.float16
    assert key.float().flatten().tolist() == k["expect_key"]
    assert cache.value().float().flatten().tolist() == [
        10, 20, 30, 40, 90, 100, 110, 120, 50, 60, 70, 80, 130, 140, 150, 160]


@pytest.mark.parametrize("name", ["kv_cache_prefill_append", "kv_cache_append_updates_prefix"])
def test_layer_cache_prefix_shapes(cuda, kats, name):
    """src/model/kv_cache.rs:261-273 and 276-293."""
    k = kats[name]
    cache = rb.LayerKvCache(k["num_kv_heads"], k["max"], k["dim"], torch.float16, cuda)
    for ap in k["appends"]:
        cache.append(f16(ap["key"], ap["shape"], cuda), f16(ap["value"], ap["shape"], cuda))
    assert cache.len() == k["expect_len"]
    assert list(cache.key().shape) == k["expect_key_shape"]
    assert list(cache.value().shape) == k["expect_key_shape"]


def test_layer_cache_rejects_dtype_mismatch_without_mutation(cuda, kats):
    """src/model/kv_cache.rs:296-306."""
    k = kats["kv_cache_rejects_dtype_mismatch"]
    cache = rb.LayerKvCache(k["num_kv_heads"], k["max"], k["dim"], torch.float16, cuda)
    key = torch.ones(k["shape"], dtype=torch.float32, device=cuda)
    with pytest.raises(rb.UnsupportedDType):
        cache.append(key, key * 2)
    assert cache.len() == k["expect_len"]
    # and at the C ABI, below the Python check
    with pytest.raises(rb.UnsupportedDType):
        rb._lib.call("tmllm_cache_append", cache.store.handle, 0, 0, key.data_ptr(),
                     key.data_ptr(), 1, 0, None)
    assert cache.len() == 0


def test_layer_cache_rejects_overflow_and_bad_shape(cuda):
    cache = rb.LayerKvCache(2, 4, 4, torch.float16, cuda)
    x = torch.ones((1, 2, 3, 4), dtype=torch.float16, device=cuda)
    cache.append(x, x)
    with pytest.raises(rb.PositionOutOfRange) as e:  # kv_cache.rs:40-51
        cache.append(x, x)
    assert (e.value.start_pos, e.value.seq_len, e.value.max_seq_len) == (3, 3, 4)
    assert cache.len() == 3
    with pytest.raises(rb.ModelFormat):
        cache.append(torch.ones((1, 3, 1, 4), dtype=torch.float16, device=cuda),
                     torch.ones((1, 3, 1, 4), dtype=torch.float16, device=cuda))
    assert cache.len() == 3
    cache.reset()
    assert cache.len() == 0 and cache.is_empty()
    with pytest.raises(rb.InvalidShape):
        rb.LayerKvCache(0, 4, 4, torch.float16, cuda)


def test_kv_cache_layers(cuda):
    """src/model/kv_cache.rs:145-184."""
    kv = rb.KvCache(3, 16, 2, 8, torch.float16, cuda)
    assert kv.num_layers() == 3 and kv.max_seq_len() == 16
    assert kv.storage_bytes() == 3 * 2 * 2 * 16 * 8 * 2
    kv.layer_mut(1).append(torch.ones((1, 2, 2, 8), dtype=torch.float16, device=cuda),
                           torch.ones((1, 2, 2, 8), dtype=torch.float16, device=cuda))
    assert [layer.len() for layer in kv.layers] == [0, 2, 0]
    with pytest.raises(rb.ModelFormat):
        kv.layer_mut(3)
    kv.reset()
    assert kv.layer_mut(1).len() == 0


@pytest.mark.parametrize("dtype,block_size", [(torch.float16, 16), (torch.float32, 16),
                                              (torch.float16, 5), (torch.float16, 64)])
def test_paged_layout_bit_exact_with_oracle(cuda, orc, dtype, block_size):
    """Appends in ragged pieces into a shuffled block pool; the arena equals the oracle's
    paged scatter through the same block tables, and gathers return the dense data."""
    rng = np.random.default_rng(block_size)
    layers, seqs, max_len, hkv, d = 2, 4, 100, 3, 64
    npd = np.float16 if dtype == torch.float16 else np.float32
    cache = rb.PagedKvCache(layers, seqs, max_len, hkv, d, dtype=dtype, block_size=block_size,
                            shuffle_seed=99, device=cuda)
    lens = rng.integers(1, max_len, seqs)
    dense = {}
    for s in range(seqs):
        for layer in range(layers):
            dense[(layer, s)] = (rng.standard_normal((2, hkv, int(lens[s]), d)).astype(npd))
    for s in range(seqs):
        cut = int(lens[s]) // 3
        for lo, hi in [(0, cut), (cut, int(lens[s]))]:
            for layer in range(layers):
                x = dense[(layer, s)]
                cache.append(layer, s, torch.from_numpy(x[0][:, lo:hi].copy()).to(cuda),
                             torch.from_numpy(x[1][:, lo:hi].copy()).to(cuda))
            cache.advance(hi - lo, s)
    assert cache.lens() == [int(x) for x in lens]
    nb = seqs * ((max_len + block_size - 1) // block_size)
    tables = np.full((seqs, (max_len + block_size - 1) // block_size), -1, np.int32)
    used = []
    for s in range(seqs):
        tbl = cache.block_table(s)
        assert len(tbl) == (int(lens[s]) + block_size - 1) // block_size
        tables[s, : len(tbl)] = tbl
        used += tbl
    assert len(set(used)) == len(used) and all(0 <= b < nb for b in used)
    assert used != sorted(used)  # the seeded shuffle took effect
    for layer in range(layers):
        ka, va = cache.arena(layer)
        want_k = np.zeros((nb, hkv, block_size, d), npd)
        want_v = np.zeros_like(want_k)
        got_k, got_v = ka.cpu().numpy(), va.cpu().numpy()
        for s in range(seqs):
            orc.paged_scatter(want_k, tables, s, 0, dense[(layer, s)][0], block_size)
            orc.paged_scatter(want_v, tables, s, 0, dense[(layer, s)][1], block_size)
            gk, gv = cache.gather(layer, s)
            assert np.array_equal(gk.cpu().numpy(), dense[(layer, s)][0])
            assert np.array_equal(gv.cpu().numpy(), dense[(layer, s)][1])
        for b in used:
            assert np.array_equal(got_k[b], want_k[b]) and np.array_equal(got_v[b], want_v[b])


def test_paged_pool_exhaustion_and_reset(cuda):
    cache = rb.PagedKvCache(1, 2, 64, 1, 8, block_size=16, num_blocks=5, device=cuda)
    x = torch.ones((1, 48, 8), dtype=torch.float16, device=cuda)
    cache.append(0, 0, x, x)
    cache.advance(48, 0)
    with pytest.raises(rb.OutOfBlocks):
        cache.append(0, 1, x, x)  # needs 3 blocks, 2 left
    assert cache.len(1) == 0 and cache.block_table(1) == []
    with pytest.raises(rb.NotReserved):
        cache.advance(1, 1)
    cache.reset(0)
    assert cache.len(0) == 0 and cache.block_table(0) == []
    cache.append(0, 1, x, x)
    cache.advance(48, 1)
    assert len(cache.block_table(1)) == 3
    with pytest.raises(rb.PositionOutOfRange) as e:  # through the C ABI's error fields
        cache.reserve(1, 17)
    assert (e.value.start_pos, e.value.seq_len, e.value.max_seq_len) == (48, 17, 64)
    assert "position range [48, 65) exceeds max sequence length 64" in str(e.value)
