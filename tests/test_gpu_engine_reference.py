"""The HF drop-in against the reference engine itself (GPU).

tests/golden/make_engine_golden.py ran the reference's ``RazorEngine.patch_model``
(razorkv/engine.py:39-133) on a seeded 4-layer Llama (4 query / 1 kv head, head_dim 128,
fp32, batch 2, 768-token prompt, 64 greedy tokens) and recorded the logits of every forward
and every compaction of every layer (the forward, the layer, the retained token positions,
the gap at the top-k cut).  Here ``razorkv_b200.RazorEngine`` patches the same model (same
seeded weights, on the GPU) and is fed the same tokens (teacher forcing), forward by forward
as ``generate`` would call it.  Every compaction must happen in the same forward and layer
and keep the same token positions, and the logits must agree.  The model runs in fp32 on both
sides; the logit tolerance covers the CPU and GPU matmuls' different summation orders.
"""

import os

import numpy as np
import pytest
import torch

from tests.golden.make_engine_golden import ENGINE_CASE, RowIds, build_model

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "engine_llama4l_fp32.npz")


def _load():
    z = np.load(GOLDEN)
    off = z["ev_off"]
    events = [(int(z["ev_forward"][i]), int(z["ev_layer"][i]), z["ev_ids"][off[i]:off[i + 1]],
               float(z["ev_margin"][i])) for i in range(len(off) - 1)]
    return z["tokens"], z["logits"], events, z["final_len"]


def test_engine_matches_the_reference_engine():
    from razorkv_b200 import PagedRazorKVCache, RazorConfig, RazorEngine
    case = ENGINE_CASE
    tokens, ref_logits, ref_events, ref_len = _load()
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    model = build_model(case, device="cuda")
    RazorEngine.patch_model(model, config=RazorConfig(**case["razor"]))
    cache = PagedRazorKVCache(config=RazorConfig(**case["razor"]), num_layers=case["layers"])

    rows = RowIds()
    events = []
    state = {"fwd": 0}
    orig_update = cache.update

    def rec_update(k, v, layer_idx, cache_kwargs=None):
        before = cache.get_cached_seq_length(layer_idx)
        rows.add(layer_idx, k, len(rows.rows.get(layer_idx, {})))
        out = orig_update(k, v, layer_idx, cache_kwargs)
        after = cache.get_cached_seq_length(layer_idx)
        if after != before + k.shape[2]:   # compacted
            events.append((state["fwd"], layer_idx, rows.ids(layer_idx, cache.key_cache[layer_idx])))
        return out

    cache.update = rec_update
    P = case["prompt"]
    ids = torch.from_numpy(tokens).cuda()
    logits = []
    with torch.no_grad():
        out = model(input_ids=ids[:, :P], past_key_values=cache, use_cache=True)
        for step in range(case["new_tokens"]):
            logits.append(out.logits[:, -1, :].float().cpu().numpy())
            state["fwd"] += 1
            if step == case["new_tokens"] - 1:
                break
            out = model(input_ids=ids[:, P + step:P + step + 1], past_key_values=cache,
                        use_cache=True)
    torch.cuda.synchronize()
    cache.check_errors()

    assert [(f, l) for f, l, _ in events] == [(f, l) for f, l, _, _ in ref_events]
    for (f, l, got), (_, _, want, margin) in zip(events, ref_events):
        assert np.array_equal(got, want), f"forward {f} layer {l} (reference cut {margin:.2e})"
    assert [cache.get_cached_seq_length(l) for l in range(case["layers"])] == ref_len.tolist()
    np.testing.assert_allclose(np.stack(logits), ref_logits, atol=2e-3, rtol=1e-3)
    # the greedy choice the reference made is the GPU's choice too, wherever the reference's
    # top two logits are not within the tolerance of each other
    top2 = np.sort(ref_logits, axis=-1)[..., -2:]
    clear = (top2[..., 1] - top2[..., 0]) > 4e-3
    assert np.array_equal(np.stack(logits).argmax(-1)[clear], ref_logits.argmax(-1)[clear])
    RazorEngine.unpatch_model(model)
