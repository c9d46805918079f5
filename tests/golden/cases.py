"""Golden cases: workloads, cache settings and the decode-step protocol they run.

The protocol (shared by the fixture generator, the oracle tests and the GPU tests):
prefill every layer once with ``update(K, V, l, {"query_states": q0})``, then for each
decode step and each layer ``update(k, v, l, {"query_states": q})`` followed by attention
over the retained cache.  Cases with ``query=False`` never pass a query (norm-only
salience, as the reference's own benchmark does).
"""

import torch

from razorkv_b200.workload import DecodeWorkload, WORKLOADS, decode_inputs, layer_prefill


def _razor(w: DecodeWorkload, **over):
    d = dict(compression_ratio=w.compression_ratio, sink_tokens=w.sink_tokens,
             local_window=w.local_window, page_size=w.page_size, pyramid_mode=w.pyramid_mode,
             pyramid_min_ratio=w.pyramid_min_ratio, pyramid_max_ratio=w.pyramid_max_ratio)
    d.update(over)
    return d


_W1 = WORKLOADS["single-layer-fp32-4k"]
_W2 = DecodeWorkload("pyramid-bf16-small", num_layers=3, num_q_heads=8, num_kv_heads=2,
                     head_dim=128, batch=2, context=2048, decode_steps=40,
                     dtype=torch.bfloat16, local_window=128, seed=77)
# sink 10 is not a multiple of the page size and the window makes the prefill budget equal
# sink + window (the "zones" branch of the reference, razorkv/cache.py:310-320)
_W3 = DecodeWorkload("ragged-sink-fp32", num_layers=2, num_q_heads=6, num_kv_heads=3,
                     head_dim=32, batch=3, context=700, decode_steps=30, dtype=torch.float32,
                     sink_tokens=10, local_window=200, pyramid_mode="uniform",
                     compression_ratio=0.30, planted_pages=2, seed=5)
_W4 = DecodeWorkload("uniform-ties-fp32", num_layers=1, num_q_heads=4, num_kv_heads=2,
                     head_dim=16, batch=2, context=300, decode_steps=20, dtype=torch.float32,
                     sink_tokens=8, local_window=32, page_size=8, pyramid_mode="uniform",
                     compression_ratio=0.40, planted_pages=1, seed=9)
_W5 = DecodeWorkload("gqa7-bf16-page5", num_layers=2, num_q_heads=14, num_kv_heads=2,
                     head_dim=64, batch=1, context=900, decode_steps=24, dtype=torch.bfloat16,
                     sink_tokens=10, local_window=40, page_size=5, pyramid_mode="adaptive",
                     compression_ratio=0.30, planted_pages=3, seed=11)

CASES = {
    "single_layer_fp32_4k": dict(workload=_W1, razor=_razor(_W1), query=True),
    "pyramid_bf16_small": dict(workload=_W2, razor=_razor(_W2), query=True),
    "ragged_sink_fp32": dict(workload=_W3, razor=_razor(_W3), query=True),
    "uniform_ties_fp32": dict(workload=_W4, razor=_razor(_W4, salience_init="uniform"), query=False),
    "gqa7_bf16_page5": dict(workload=_W5, razor=_razor(_W5), query=True),
}


def iter_inputs(case, device="cpu"):
    """Yield ("prefill", -1, layer, (K, V, q0)) then ("decode", step, layer, (q, k, v))."""
    w = case["workload"]
    for layer in range(w.num_layers):
        yield "prefill", -1, layer, layer_prefill(w, layer, device)
    for step in range(w.decode_steps):
        for layer in range(w.num_layers):
            yield "decode", step, layer, decode_inputs(w, step, layer, device)


# Cases at the measured workloads' own scale.  Only a pair of layers of each model is run
# (the shallowest and the deepest, with the budgets of the full model), for enough decode
# steps that every layer compacts at least once after its prefill eviction.  Their fixtures
# record the reference's top-k decisions (kept pages and the gap at the cut), a strided
# sample of the final salience and the attention output of the last step, not every tensor.
SCALE_CASES = {
    # Llama-3.1-8B shape: batch 8, 32/8 heads, d128, bf16, 32768-token prefill, linear
    # pyramid 15 % -> 70 %; layer 31 first compacts at decode step 85
    "llama8b_b8_32k_l0_l31": dict(workload=WORKLOADS["llama8b-b8-32k-bf16"], layers=(0, 31),
                                  decode_steps=86, query=True),
    # Qwen-2.5-7B shape: batch 1, 28/4 heads (GQA 7), d128, bf16, 131072-token prefill
    # (8192 pages); layer 27 first compacts at decode step 74
    "qwen7b_b1_128k_l0_l27": dict(workload=WORKLOADS["qwen7b-b1-128k-bf16"], layers=(0, 27),
                                  decode_steps=75, query=True),
}

# salience sample stride of the scale fixtures (tokens)
SCALE_SAL_STRIDE = 7


def iter_scale_inputs(case, device="cpu", steps=None):
    """As ``iter_inputs`` for the selected layers of a scale case (real layer indices)."""
    w = case["workload"]
    for layer in case["layers"]:
        yield "prefill", -1, layer, layer_prefill(w, layer, device)
    n = case["decode_steps"] if steps is None else steps
    for step in range(n):
        for layer in case["layers"]:
            yield "decode", step, layer, decode_inputs(w, step, layer, device)


def scale_input_digest(sha, kind, tensors):
    """Adds a cheap digest of one step's inputs: prefill K/V every 61st token, all else."""
    for i, t in enumerate(tensors):
        if kind == "prefill" and i < 2:
            t = t[:, :, ::61]
        sha.update(t.float().contiguous().numpy().tobytes())
