"""The CUDA decode path against the reference at the measured workloads' scale (GPU).

Each scale case (a layer pair of the Llama-8B-shaped workload at batch 8 and 32k context, and
of the Qwen-7B-shaped workload at batch 1 and 128k context) is drawn on the CPU from its seeds,
copied to the GPU and driven through ``PagedRazorKVCache`` with the decode-step protocol the
benchmark uses (prefill with ``update``, then ``decode_step`` per layer and step).  Every
compaction decision is recorded and compared with the reference's (fixture): same layer,
cached length, budget, page count and k, and the same kept pages (a mismatch is reported with
whether it was a provable near-tie, the gap at the cut within 4e-6 of the largest salience).

The oracle runs beside the GPU on the layers it can afford here (both Qwen-shaped layers,
Llama-shaped layer 0): salience and retained K must equal it bit for bit after the last
step, attention outputs agree within the bf16 tolerance (2e-2 abs, 1e-2 rel) every 8th step.
The deep Llama-shaped layer (23k retained tokens at batch 8) is compared with the
reference's own salience sample (2e-6 relative) and last output.
"""

import numpy as np
import pytest
import torch

from razorkv_b200.cache import PagedRazorKVCache
from razorkv_b200.config import RazorConfig
from tests.golden.cases import SCALE_CASES, SCALE_SAL_STRIDE, iter_scale_inputs
from tests.protocol import elt_size, load_scale, near_tie, oracle_config

pytestmark = [pytest.mark.gpu, pytest.mark.timeout(900)]

ATOL, RTOL = 2e-2, 1e-2
# layers the oracle follows in this test (cost on the host: seconds to a minute)
ORACLE_LAYERS = {"llama8b_b8_32k_l0_l31": (0,), "qwen7b_b1_128k_l0_l27": (0, 27)}


@pytest.mark.parametrize("name", list(SCALE_CASES))
def test_cuda_keeps_the_reference_pages_at_scale(name):
    from oracle import razorkv_oracle as O

    case = SCALE_CASES[name]
    w = case["workload"]
    g = load_scale(name)
    ref = g["decisions"]
    cfg = RazorConfig(compression_ratio=w.compression_ratio, sink_tokens=w.sink_tokens,
                      local_window=w.local_window, page_size=w.page_size,
                      pyramid_mode=w.pyramid_mode, pyramid_min_ratio=w.pyramid_min_ratio,
                      pyramid_max_ratio=w.pyramid_max_ratio)
    cache = PagedRazorKVCache(cfg, w.num_layers)
    # the production path (fused score + pool pass, fused select + compact); decisions are
    # recorded and compared after the run
    cache.record_decisions = True

    olayers = ORACLE_LAYERS[name]
    ocache = O.OracleCache(oracle_config(w), w.num_layers, elt_size(w.dtype))
    oref = [d for d in ref if d["layer"] in olayers]

    def ofollow(layer, i, kept, margin):
        d = oref[i]
        return None if np.array_equal(kept, d["kept"]) else d["kept"]

    ocache.kept_override = ofollow
    last = case["decode_steps"] - 1
    for kind, step, layer, tensors in iter_scale_inputs(case):
        a, b, c = tensors
        if kind == "prefill":
            cache.update(a.cuda(), b.cuda(), layer, {"query_states": c.cuda()})
            if layer in olayers:
                ocache.update(a.float().numpy(), b.float().numpy(), layer, c.float().numpy())
            continue
        out = cache.decode_step(a.cuda(), b.cuda(), c.cuda(), layer)
        if layer in olayers:
            Kc, Vc = ocache.update(b.float().numpy(), c.float().numpy(), layer,
                                   a.float().numpy())
            if step % 8 == 0 or step == last:
                expect = O.attention(a.float().numpy(), Kc, Vc)
                np.testing.assert_allclose(out.float().cpu().numpy(), expect, atol=ATOL,
                                           rtol=RTOL, err_msg=f"layer {layer} step {step}")
        if step == last:
            np.testing.assert_allclose(out.float().cpu().numpy()[:, :, 0, :], g["out"][layer],
                                       atol=ATOL, rtol=RTOL, err_msg=f"layer {layer} last step")
    torch.cuda.synchronize()
    cache.check_errors()

    assert len(cache.decisions) == len(ref)
    for i, (d, r) in enumerate(zip(cache.decisions, ref)):
        assert (d.layer, d.seq_len, d.budget, d.num_pages, d.k) == (
            r["layer"], r["seq_len"], r["budget"], r["num_pages"], r["k"]), f"decision {i}"
        if not np.array_equal(d.kept.cpu().numpy(), r["kept"]):
            scale = float(cache.salience_scores[d.layer].abs().max())
            tie = near_tie(r["margin"], scale) or near_tie(float(d.margin.item()), scale)
            raise AssertionError(f"decision {i} (layer {d.layer}): kept pages differ from the "
                                 f"reference at margin {float(d.margin.item()):.3e} (reference "
                                 f"{r['margin']:.3e}; {'a' if tie else 'not a'} provable near-tie)")
    for layer in case["layers"]:
        assert cache.get_cached_seq_length(layer) == g["len"][layer]
        S = cache.salience_scores[layer].cpu().numpy()
        np.testing.assert_allclose(S[:, ::SCALE_SAL_STRIDE], g["sal"][layer], rtol=2e-6, atol=0)
        if layer in olayers:
            assert np.array_equal(S.view(np.uint32), ocache.S[layer].view(np.uint32)), layer
            Kg = cache.key_cache[layer].float().cpu().numpy()
            assert np.array_equal(Kg, ocache.K[layer]), layer
    print(f"{name}: {len(ref)} decisions equal to the reference")
