"""Shapes outside the sm_100a decode kernel's coverage (more than 8 query heads per kv head,
kv-head counts other than 1/2/4/8) take the shape-general kernels; the cache must still match
the oracle bit for bit through prefill, decode steps and compactions."""

import numpy as np
import pytest
import torch

from oracle import razorkv_oracle as O
from razorkv_b200 import PagedRazorKVCache, RazorConfig

pytestmark = pytest.mark.gpu


def _randn(*shape, dtype, seed):
    return torch.randn(*shape, generator=torch.Generator().manual_seed(seed)).to(dtype).cuda()


@pytest.mark.parametrize("B,Hq,Hkv,D,dtype", [
    (2, 32, 2, 128, torch.bfloat16),    # GQA 16
    (1, 16, 16, 64, torch.float16),     # 16 kv heads
    (2, 12, 3, 128, torch.bfloat16),    # 3 kv heads
    (1, 24, 12, 64, torch.float32),     # fp32, 12 kv heads
])
def test_generic_shapes_match_oracle(B, Hq, Hkv, D, dtype):
    rc = RazorConfig(compression_ratio=0.30, sink_tokens=32, local_window=64, page_size=16,
                     pyramid_mode="uniform")
    cache = PagedRazorKVCache(rc, 1)
    oc = O.OracleCache(O.OracleConfig(compression_ratio=0.30, sink_tokens=32, local_window=64,
                                      page_size=16, pyramid_mode="uniform"), 1,
                       4 if dtype == torch.float32 else 2)
    k, v = _randn(B, Hkv, 600, D, dtype=dtype, seed=1), _randn(B, Hkv, 600, D, dtype=dtype, seed=2)
    q = _randn(B, Hq, 1, D, dtype=dtype, seed=3)
    cache.update(k, v, 0, {"query_states": q})
    oc.update(k.float().cpu().numpy(), v.float().cpu().numpy(), 0, q.float().cpu().numpy())
    atol, rtol = (1e-5, 1e-5) if dtype == torch.float32 else (2e-2, 1e-2)
    for step in range(40):
        q = _randn(B, Hq, 1, D, dtype=dtype, seed=10 + 3 * step)
        kn = _randn(B, Hkv, 1, D, dtype=dtype, seed=11 + 3 * step)
        vn = _randn(B, Hkv, 1, D, dtype=dtype, seed=12 + 3 * step)
        out = cache.decode_step(q, kn, vn, 0)
        Kc, Vc = oc.update(kn.float().cpu().numpy(), vn.float().cpu().numpy(), 0,
                           q.float().cpu().numpy())
        np.testing.assert_allclose(out.float().cpu().numpy(),
                                   O.attention(q.float().cpu().numpy(), Kc, Vc),
                                   atol=atol, rtol=rtol)
    assert len(oc.decisions) >= 2   # the prefill compaction and at least one while decoding
    assert np.array_equal(cache.key_cache[0].float().cpu().numpy(), oc.K[0])
    S = cache.salience_scores[0].cpu().numpy()
    assert np.array_equal(S.view(np.uint32), oc.S[0].view(np.uint32))
