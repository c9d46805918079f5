"""PagedRazorKVCache on the GPU: the reference's cache tests (razorkv tests/test_cache.py:41-260)
with CUDA tensors, and the paths around the decode step checked bit for bit against the
oracle -- prompts fed in chunks (razorkv/cache.py:395-407 on every chunk) and the batch
operations used by beam search (razorkv/cache.py:177-229)."""

import numpy as np
import pytest
import torch

from oracle import razorkv_oracle as O
from razorkv_b200 import PagedRazorKVCache, RazorConfig, RazorKVCache

pytestmark = pytest.mark.gpu


def _randn(*shape, dtype=torch.float32, seed=0):
    return torch.randn(*shape, generator=torch.Generator().manual_seed(seed)).to(dtype).cuda()


# --------------------------------------------------------------------------- reference tests
def test_razor_cache_prefill_and_eviction():
    config = RazorConfig(compression_ratio=0.30, sink_tokens=8, local_window=32, page_size=16,
                         pyramid_mode="linear", pyramid_min_ratio=0.20, pyramid_max_ratio=0.50)
    cache = RazorKVCache(config=config, num_layers=4)
    for layer in range(4):
        cache.update(_randn(1, 4, 500, 32, seed=layer), _randn(1, 4, 500, 32, seed=10 + layer), layer)
    l0, l3 = cache.get_cached_seq_length(0), cache.get_cached_seq_length(3)
    assert l0 < 500 and l0 <= l3 and l0 >= 8 + 32
    assert cache.get_seq_length(0) == 500 and cache.seen_tokens == 500


def test_razor_cache_autoregressive_decode():
    config = RazorConfig(compression_ratio=0.40, sink_tokens=8, local_window=16, page_size=8,
                         pyramid_mode="uniform")
    cache = RazorKVCache(config=config, num_layers=2)
    k, v = _randn(1, 2, 100, 16, seed=1), _randn(1, 2, 100, 16, seed=2)
    cache.update(k, v, 0)
    cache.update(k, v, 1)
    for step in range(20):
        ks, vs = _randn(1, 2, 1, 16, seed=100 + step), _randn(1, 2, 1, 16, seed=200 + step)
        cache.update(ks, vs, 0)
        cache.update(ks, vs, 1)
    assert cache.get_cached_seq_length(0) <= int(120 * 0.40) + 8 + (8 + 16)
    assert cache.seen_tokens == 120 and cache.get_seq_length(0) == 120


def test_razor_cache_sink_preservation():
    cache = RazorKVCache(config=RazorConfig(compression_ratio=0.25, sink_tokens=10,
                                            local_window=20, page_size=5), num_layers=1)
    k, v = _randn(1, 2, 200, 16, seed=3), _randn(1, 2, 200, 16, seed=4)
    k[:, :, :10, :] = 999.0
    v[:, :, :10, :] = 888.0
    cache.update(k, v, 0)
    assert torch.all(cache.key_cache[0][:, :, :10, :] == 999.0)
    assert torch.all(cache.value_cache[0][:, :, :10, :] == 888.0)


def test_memory_stats():
    cache = RazorKVCache(config=RazorConfig(compression_ratio=0.5), num_layers=2)
    k, v = _randn(1, 2, 50, 16, seed=5), _randn(1, 2, 50, 16, seed=6)
    cache.update(k, v, 0)
    cache.update(k, v, 1)
    stats = cache.get_memory_stats()
    assert stats["total_bytes"] == 2 * 2 * 50 * 16 * 4 * 2
    assert stats["total_mb"] > 0 and len(stats["per_layer_tokens"]) == 2
    assert stats["pool_slots"] >= stats["free_slots"] >= 0


def test_edge_case_sequence_shorter_than_window():
    cache = RazorKVCache(config=RazorConfig(sink_tokens=16, local_window=32,
                                            compression_ratio=0.10), num_layers=1)
    cache.update(_randn(1, 2, 20, 16, seed=7), _randn(1, 2, 20, 16, seed=8), 0)
    assert cache.get_cached_seq_length(0) == 20 and cache.get_seq_length(0) == 20


def test_multi_batch_handling():
    cache = RazorKVCache(config=RazorConfig(sink_tokens=4, local_window=8, compression_ratio=0.30,
                                            page_size=4), num_layers=2)
    cache.update(_randn(4, 2, 80, 16, seed=9), _randn(4, 2, 80, 16, seed=10), 0)
    assert cache.key_cache[0].shape[0] == 4 and cache.value_cache[0].shape[0] == 4
    assert cache.get_cached_seq_length(0) < 80 and cache.get_seq_length(0) == 80


def test_reorder_cache_for_beam_search():
    cache = RazorKVCache(config=RazorConfig(), num_layers=1)
    k = torch.tensor([[[[1.0]], [[2.0]]], [[[3.0]], [[4.0]]]]).cuda()   # batch 2, D 1
    v = torch.tensor([[[[10.0]], [[20.0]]], [[[30.0]], [[40.0]]]]).cuda()
    cache.update(k, v, 0)
    cache.reorder_cache(torch.tensor([1, 0], dtype=torch.long))
    assert torch.equal(cache.key_cache[0][0], k[1])
    assert torch.equal(cache.value_cache[0][0], v[1])


def test_cache_crop_and_reset():
    cache = RazorKVCache(config=RazorConfig(sink_tokens=4, local_window=8, compression_ratio=0.5),
                         num_layers=1)
    cache.update(_randn(1, 2, 20, 16, seed=11), _randn(1, 2, 20, 16, seed=12), 0)
    n = cache.get_cached_seq_length(0)
    cache.crop(5)
    assert cache.get_cached_seq_length(0) == n - 5 and cache.seen_tokens == 15
    cache.reset()
    assert cache.seen_tokens == 0 and cache.get_cached_seq_length(0) == 0
    assert len(cache.key_cache) == 0


def test_cache_batch_repeat_and_select():
    cache = RazorKVCache(config=RazorConfig(), num_layers=1)
    cache.update(_randn(2, 2, 10, 16, seed=13), _randn(2, 2, 10, 16, seed=14), 0)
    cache.batch_repeat_interleave(2)
    assert cache.batch_size == 4
    cache.batch_select_indices(torch.tensor([0, 2]))
    assert cache.batch_size == 2


def test_cache_get_mask_sizes_and_query_offset():
    cache = RazorKVCache(config=RazorConfig(), num_layers=1)
    assert cache.get_mask_sizes(10, 0) == (10, 0) and cache.get_query_offset(0) == 0
    cache.update(_randn(1, 2, 50, 16, seed=15), _randn(1, 2, 50, 16, seed=16), 0)
    kv_len, kv_off = cache.get_mask_sizes(1, 0)
    assert kv_len == cache.get_cached_seq_length(0) + 1 and kv_off == 0


# ------------------------------------------------------------------ against the oracle, bit for bit
def _oracle_cfg(c: RazorConfig) -> O.OracleConfig:
    return O.OracleConfig(compression_ratio=c.compression_ratio, sink_tokens=c.sink_tokens,
                          local_window=c.local_window, page_size=c.page_size,
                          pyramid_mode=c.pyramid_mode, pyramid_min_ratio=c.pyramid_min_ratio,
                          pyramid_max_ratio=c.pyramid_max_ratio)


def _check(cache, oc, layers, where):
    for l in range(layers):
        K = cache.key_cache[l].float().cpu().numpy()
        V = cache.value_cache[l].float().cpu().numpy()
        S = cache.salience_scores[l].cpu().numpy()
        assert np.array_equal(K, oc.K[l]), f"{where}: layer {l} K"
        assert np.array_equal(V, oc.V[l]), f"{where}: layer {l} V"
        assert np.array_equal(S.view(np.uint32), oc.S[l].view(np.uint32)), f"{where}: layer {l} S"


@pytest.mark.parametrize("dtype,D,Hq,Hkv", [(torch.bfloat16, 128, 8, 2), (torch.float32, 64, 4, 4)])
def test_chunked_prefill_matches_oracle(dtype, D, Hq, Hkv):
    """A 3000-token prompt fed as 1024 + 1024 + 952-token chunks, layer by layer as a model's
    chunked prefill does; every chunk appends and, past the budget, compacts at once."""
    layers, B = 2, 2
    rc = RazorConfig(compression_ratio=0.30, sink_tokens=32, local_window=128, page_size=16,
                     pyramid_mode="linear", pyramid_min_ratio=0.2, pyramid_max_ratio=0.5)
    cache = PagedRazorKVCache(rc, layers)
    oc = O.OracleCache(_oracle_cfg(rc), layers, 2 if dtype != torch.float32 else 4)
    pos, seed = 0, 0
    for chunk in (1024, 1024, 952):
        for l in range(layers):
            seed += 3
            k, v = _randn(B, Hkv, chunk, D, dtype=dtype, seed=seed), _randn(B, Hkv, chunk, D, dtype=dtype, seed=seed + 1)
            q = _randn(B, Hq, 4, D, dtype=dtype, seed=seed + 2)
            cache.update(k, v, l, {"query_states": q})
            oc.update(k.float().cpu().numpy(), v.float().cpu().numpy(), l, q.float().cpu().numpy())
        pos += chunk
        _check(cache, oc, layers, f"after prefill chunk ending at {pos}")
    assert cache.seen_tokens == 3000 and oc.seen == 3000
    for step in range(24):
        for l in range(layers):
            seed += 3
            q = _randn(B, Hq, 1, D, dtype=dtype, seed=seed)
            k, v = _randn(B, Hkv, 1, D, dtype=dtype, seed=seed + 1), _randn(B, Hkv, 1, D, dtype=dtype, seed=seed + 2)
            out = cache.decode_step(q, k, v, l)
            Kc, Vc = oc.update(k.float().cpu().numpy(), v.float().cpu().numpy(), l, q.float().cpu().numpy())
            atol, rtol = (2e-2, 1e-2) if dtype != torch.float32 else (1e-5, 1e-5)
            np.testing.assert_allclose(out.float().cpu().numpy(), O.attention(q.float().cpu().numpy(), Kc, Vc),
                                       atol=atol, rtol=rtol)
    _check(cache, oc, layers, "after decode")
    assert sum(1 for d in oc.decisions if d.kind == "pages") >= 2 * layers


def test_batch_ops_keep_oracle_parity():
    """reorder_cache / batch_repeat_interleave / batch_select_indices reindex every layer's
    sequences; decoding afterwards must equal the oracle with its arrays reindexed alike."""
    layers, B, Hq, Hkv, D = 2, 3, 8, 2, 128
    dt = torch.bfloat16
    rc = RazorConfig(compression_ratio=0.30, sink_tokens=32, local_window=64, page_size=16,
                     pyramid_mode="uniform")
    cache = PagedRazorKVCache(rc, layers)
    oc = O.OracleCache(_oracle_cfg(rc), layers, 2)

    def reindex(idx):
        for l in range(layers):
            for arr in (oc.K, oc.V, oc.S):
                arr[l] = np.ascontiguousarray(arr[l][idx])

    seed = 1000

    def steps(n, b):
        nonlocal seed
        for _ in range(n):
            for l in range(layers):
                seed += 3
                q = _randn(b, Hq, 1, D, dtype=dt, seed=seed)
                k, v = _randn(b, Hkv, 1, D, dtype=dt, seed=seed + 1), _randn(b, Hkv, 1, D, dtype=dt, seed=seed + 2)
                cache.decode_step(q, k, v, l)
                oc.update(k.float().cpu().numpy(), v.float().cpu().numpy(), l, q.float().cpu().numpy())

    for l in range(layers):
        k, v = _randn(B, Hkv, 700, D, dtype=dt, seed=l), _randn(B, Hkv, 700, D, dtype=dt, seed=50 + l)
        q = _randn(B, Hq, 1, D, dtype=dt, seed=90 + l)
        cache.update(k, v, l, {"query_states": q})
        oc.update(k.float().cpu().numpy(), v.float().cpu().numpy(), l, q.float().cpu().numpy())
    steps(10, 3)
    beam = [2, 0, 0]
    cache.reorder_cache(torch.tensor(beam))
    reindex(beam)
    _check(cache, oc, layers, "after reorder_cache")
    steps(10, 3)
    cache.batch_repeat_interleave(2)
    reindex(np.repeat(np.arange(3), 2))
    steps(5, 6)
    cache.batch_select_indices(torch.tensor([1, 4]))
    reindex([1, 4])
    steps(25, 2)
    _check(cache, oc, layers, "after batch ops and decoding")
    assert cache.batch_size == 2
