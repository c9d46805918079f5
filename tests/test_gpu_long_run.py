"""A long decode run against the oracle: 600 steps with a small sink and window (a compaction
every ~20 steps per layer), starting from an 8-slot pool that has to grow several times.
Every step's output is checked; K, V and salience bit for bit every 150 steps; at the end
every pool slot is either in exactly one layer's page table or on the free stack."""

import numpy as np
import pytest
import torch

from oracle import razorkv_oracle as O
from razorkv_b200 import PagedRazorKVCache, RazorConfig

pytestmark = pytest.mark.gpu


def _randn(*shape, dtype, seed):
    return torch.randn(*shape, generator=torch.Generator().manual_seed(seed)).to(dtype).cuda()


@pytest.mark.parametrize("dtype,D,Hq,Hkv", [(torch.bfloat16, 128, 8, 2), (torch.float32, 64, 4, 2)])
def test_long_decode_run(dtype, D, Hq, Hkv):
    layers, B, T, steps = 2, 2, 400, 600
    rc = RazorConfig(compression_ratio=0.30, sink_tokens=16, local_window=32, page_size=16,
                     pyramid_mode="linear", pyramid_min_ratio=0.2, pyramid_max_ratio=0.5)
    cache = PagedRazorKVCache(rc, layers, max_slots=8)
    oc = O.OracleCache(O.OracleConfig(compression_ratio=0.30, sink_tokens=16, local_window=32,
                                      page_size=16, pyramid_mode="linear", pyramid_min_ratio=0.2,
                                      pyramid_max_ratio=0.5), layers,
                       4 if dtype == torch.float32 else 2)
    atol, rtol = (1e-5, 1e-5) if dtype == torch.float32 else (2e-2, 1e-2)
    for l in range(layers):
        k, v = _randn(B, Hkv, T, D, dtype=dtype, seed=l), _randn(B, Hkv, T, D, dtype=dtype, seed=10 + l)
        q = _randn(B, Hq, 1, D, dtype=dtype, seed=20 + l)
        cache.update(k, v, l, {"query_states": q})
        oc.update(k.float().cpu().numpy(), v.float().cpu().numpy(), l, q.float().cpu().numpy())
    slots0 = cache._slots
    seed = 1000
    for step in range(steps):
        for l in range(layers):
            seed += 3
            q = _randn(B, Hq, 1, D, dtype=dtype, seed=seed)
            kn = _randn(B, Hkv, 1, D, dtype=dtype, seed=seed + 1)
            vn = _randn(B, Hkv, 1, D, dtype=dtype, seed=seed + 2)
            out = cache.decode_step(q, kn, vn, l)
            Kc, Vc = oc.update(kn.float().cpu().numpy(), vn.float().cpu().numpy(), l,
                               q.float().cpu().numpy())
            np.testing.assert_allclose(out.float().cpu().numpy(),
                                       O.attention(q.float().cpu().numpy(), Kc, Vc),
                                       atol=atol, rtol=rtol, err_msg=f"step {step} layer {l}")
        if step % 150 == 149 or step == steps - 1:
            for l in range(layers):
                assert np.array_equal(cache.key_cache[l].float().cpu().numpy(), oc.K[l]), step
                assert np.array_equal(cache.value_cache[l].float().cpu().numpy(), oc.V[l]), step
                S = cache.salience_scores[l].cpu().numpy()
                assert np.array_equal(S.view(np.uint32), oc.S[l].view(np.uint32)), step
    per_layer = [sum(1 for d in oc.decisions if d.layer == l) for l in range(layers)]
    assert min(per_layer) >= 15, per_layer
    assert cache._slots > slots0 or slots0 > 8   # the 8-slot pool grew
    used = torch.cat([cache.page_table(l) for l in range(layers)]).cpu().numpy()
    free = cache._free[: cache._free_top].cpu().numpy()
    every = np.concatenate([used, free])
    assert len(np.unique(every)) == len(every) == cache._slots, "a slot leaked or is double-booked"
