"""The CUDA cache against the oracle (bit for bit) and the reference fixtures (GPU).

Each golden case is driven through ``PagedRazorKVCache`` in two ways:

* ``update``: the reference protocol -- ``update(k, v, l, {"query_states": q})`` then an
  attention call over the retained cache (score pass, compaction and attention separately);
* ``decode_step``: the fused step (score and attention in one pass on non-compacting steps).

After every step the retained K, V and salience of the layer are materialised and compared
with the oracle's arrays: K/V bit-identical (compaction moves data or pointers, never
values), salience bit-identical (canonical summation order), attention output within the
dtype tolerance.  The reference's kept token ids (fixture) are recovered from the GPU rows
and compared directly as well.
"""

import numpy as np
import pytest
import torch

from oracle import razorkv_oracle as O
from razorkv_b200.cache import PagedRazorKVCache
from razorkv_b200.config import RazorConfig
from tests.golden.cases import CASES, iter_inputs
from tests.protocol import elt_size, load_golden

pytestmark = pytest.mark.gpu

TOL = {torch.float32: (1e-5, 1e-5), torch.bfloat16: (2e-2, 1e-2)}


def _row_ids(rows, K):
    return np.array([rows[K[0, 0, t].tobytes()] for t in range(K.shape[2])], np.int64)


def _run(name, mode):
    case = CASES[name]
    w = case["workload"]
    cfg = RazorConfig(**case["razor"])
    cache = PagedRazorKVCache(cfg, w.num_layers)
    ocache = O.OracleCache(O.OracleConfig(**case["razor"]), w.num_layers, elt_size(w.dtype))
    g = load_golden(name)
    rows = [dict() for _ in range(w.num_layers)]
    nid = [0] * w.num_layers
    step_idx = [0] * w.num_layers
    atol, rtol = TOL[w.dtype]
    out_i = 0
    for kind, step, layer, tensors in iter_inputs(case):
        a, b, c = tensors
        newk = a if kind == "prefill" else b
        for t in range(newk.shape[2]):
            rows[layer][newk[0, 0, t].float().numpy().tobytes()] = nid[layer]
            nid[layer] += 1
        if kind == "prefill":
            K, V, q0 = a.cuda(), b.cuda(), c.cuda()
            kw = {"query_states": q0} if case["query"] else None
            cache.update(K, V, layer, kw)
            ocache.update(a.float().numpy(), b.float().numpy(), layer,
                          c.float().numpy() if case["query"] else None)
        else:
            q, k, v = a.cuda(), b.cuda(), c.cuda()
            if mode == "update":
                kw = {"query_states": q} if case["query"] else None
                cache.update(k, v, layer, kw)
                out = cache.attention(q, layer)
            else:
                out = cache.decode_step(q, k, v, layer)
            Kc, Vc = ocache.update(b.float().numpy(), c.float().numpy(), layer,
                                   a.float().numpy() if case["query"] else None)
            ref = O.attention(a.float().numpy(), Kc, Vc)
            got = out.float().cpu().numpy()
            np.testing.assert_allclose(got, ref, atol=atol, rtol=rtol)
            if name != "uniform_ties_fp32":   # the reference breaks that case's ties differently
                np.testing.assert_allclose(got[:, :, 0, :], g["out"][out_i], atol=atol, rtol=rtol)
            out_i += 1
        Kg = cache.key_cache[layer].float().cpu().numpy()
        Vg = cache.value_cache[layer].float().cpu().numpy()
        Sg = cache.salience_scores[layer].cpu().numpy()
        where = f"{name}/{mode} layer {layer} step {step}"
        assert Kg.shape == ocache.K[layer].shape, where
        assert np.array_equal(Kg, ocache.K[layer]), where
        assert np.array_equal(Vg, ocache.V[layer]), where
        assert np.array_equal(Sg.view(np.uint32), ocache.S[layer].view(np.uint32)), where
        gid = _row_ids(rows[layer], Kg)
        if name != "uniform_ties_fp32":
            assert np.array_equal(gid, g["ids"][layer][step_idx[layer]]), where
        step_idx[layer] += 1
    return cache


@pytest.mark.parametrize("name", list(CASES))
def test_golden_update_protocol(name):
    _run(name, "update")


@pytest.mark.parametrize("name", [n for n in CASES if CASES[n]["query"]])
def test_golden_decode_step_protocol(name):
    _run(name, "decode_step")
