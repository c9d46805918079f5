"""Unit tests of the oracle's building blocks and of the host-side budget logic (CPU)."""

import math

import numpy as np
import pytest
import torch

from oracle import razorkv_oracle as O
from razorkv_b200.config import RazorConfig


def test_canonical_dot_order_definition():
    rng = np.random.default_rng(0)
    for D, elt in [(128, 2), (64, 4), (64, 2), (32, 2), (20, 4), (256, 2), (256, 4), (16, 4)]:
        a = rng.standard_normal(D).astype(np.float32)
        b = rng.standard_normal(D).astype(np.float32)
        ch = 16 // elt
        # restate the order in numpy float32 with an exact fma (via float64 product + one rounding)
        p = []
        for j in range(8):
            chains = [np.float32(0.0), np.float32(0.0)]   # even / odd positions
            pos = 0
            c = j
            while c * ch < D:
                for e in range(c * ch, min(D, c * ch + ch)):
                    acc = chains[pos & 1]
                    chains[pos & 1] = np.float32(np.float64(a[e]) * np.float64(b[e]) + np.float64(acc))
                    pos += 1
                c += 8
            p.append(np.float32(chains[0] + chains[1]))
        f = np.float32
        expect = f(f(f(p[0] + p[4]) + f(p[2] + p[6])) + f(f(p[1] + p[5]) + f(p[3] + p[7])))
        assert O.canon_dot(a, b, elt) == expect
        assert abs(float(expect) - float(np.dot(a.astype(np.float64), b))) < 1e-4


def test_page_pool_known_answer():
    # razorkv tests/test_kernels.py:35-46
    s = np.array([[1.0, 5.0, 2.0, 3.0, 8.0, 2.0, 1.0, 4.0]], np.float32)
    mx, n = O.page_pool(s, 4, "max")
    assert n == 2 and np.array_equal(mx, [[5.0, 8.0]])
    mn, n = O.page_pool(s, 4, "mean")
    assert np.allclose(mn, [[2.75, 3.75]])
    short, n = O.page_pool(s[:, :3], 4, "max")
    assert n == 1 and short.tolist() == [[5.0]]


def test_canonical_topk_ties_and_order():
    v = np.array([1, 2, 2, 2, 0, 2], np.float32)
    kept, margin = O.canonical_topk(v, 2)
    assert kept.tolist() == [1, 2] and margin == 0.0
    kept, margin = O.canonical_topk(v, 5)
    assert kept.tolist() == [0, 1, 2, 3, 5] and margin == 1.0
    kept, margin = O.canonical_topk(np.array([-1, -3, np.nan, 2], np.float32), 2)
    assert kept.tolist() == [2, 3]
    kept, margin = O.canonical_topk(np.array([3.0], np.float32), 1)
    assert kept.tolist() == [0] and margin == math.inf


def test_ewma_matches_torch_fp32():
    rng = np.random.default_rng(1)
    S = (rng.standard_normal(4096) * 5 + 10).astype(np.float32)
    R = rng.standard_normal(4096).astype(np.float32)
    d = 0.98
    t = (d * torch.from_numpy(S) + (1.0 - d) * torch.from_numpy(R)).numpy()
    assert np.array_equal(O.ewma(S, R, d).view(np.uint32), t.view(np.uint32))


def test_batch_mean_is_sequential():
    rng = np.random.default_rng(2)
    x = (rng.standard_normal((8, 300)) * 3 + 10).astype(np.float32)
    acc = x[0].copy()
    for b in range(1, 8):
        acc = (acc + x[b]).astype(np.float32)
    assert np.array_equal(O.batch_mean(x), (acc / np.float32(8)).astype(np.float32))
    assert np.array_equal(O.batch_mean(x[:1]), x[0])


def test_attention_matches_torch_sdpa():
    g = torch.Generator().manual_seed(3)
    q = torch.randn(2, 8, 1, 64, generator=g)
    k = torch.randn(2, 2, 300, 64, generator=g)
    v = torch.randn(2, 2, 300, 64, generator=g)
    ref = torch.nn.functional.scaled_dot_product_attention(
        q, k.repeat_interleave(4, 1), v.repeat_interleave(4, 1)).numpy()
    np.testing.assert_allclose(O.attention(q.numpy(), k.numpy(), v.numpy()), ref, atol=1e-5, rtol=1e-5)
    qc = torch.randn(1, 4, 5, 32, generator=g)
    kc = torch.randn(1, 2, 5, 32, generator=g)
    vc = torch.randn(1, 2, 5, 32, generator=g)
    ref = torch.nn.functional.scaled_dot_product_attention(
        qc, kc.repeat_interleave(2, 1), vc.repeat_interleave(2, 1), is_causal=True).numpy()
    np.testing.assert_allclose(O.attention(qc.numpy(), kc.numpy(), vc.numpy(), causal=True), ref,
                               atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("mode", ["uniform", "linear", "adaptive", "custom"])
def test_config_budget_matches_oracle_restatement(mode):
    kw = dict(pyramid_mode=mode, compression_ratio=0.3, sink_tokens=32, local_window=512)
    if mode == "custom":
        kw["custom_layer_ratios"] = [0.1, 0.5, 0.9]
    a = RazorConfig(**kw)
    b = O.OracleConfig(**kw)
    for L in [1, 2, 3, 24, 28, 32, 80]:
        for layer in range(L):
            for T in [1, 100, 544, 545, 2048, 4097, 32768, 33024, 131072]:
                assert a.get_layer_budget(layer, L, T) == b.budget(layer, L, T)


def test_config_budget_reference_properties():
    # razorkv tests/test_cache.py:19-38
    c = RazorConfig(compression_ratio=0.30, sink_tokens=16, local_window=64,
                    pyramid_mode="adaptive", pyramid_min_ratio=0.15, pyramid_max_ratio=0.70)
    b0, b16, b31 = (c.get_layer_budget(i, 32, 1000) for i in (0, 16, 31))
    assert b0 <= b16 <= b31 and b0 >= 80
    # the Llama-8B-shaped workload's pyramid (linear 15 % -> 70 %) at 32k: layer 0 keeps 4915 tokens, 31 keeps 22937
    lin = RazorConfig(pyramid_mode="linear")
    assert lin.get_layer_budget(0, 32, 32768) == 4915
    assert lin.get_layer_budget(31, 32, 32768) == 22937
    with pytest.raises(ValueError):
        RazorConfig(compression_ratio=0.0)
    with pytest.raises(ValueError):
        RazorConfig(page_size=0)
