"""Drivers that run a golden case through the oracle or through the CUDA cache.

Both return the same record layout as the golden fixtures: per-layer retained token ids
after every step, the attention output of every decode step, and the final salience.
"""

import hashlib
import os
import sys

import numpy as np
import torch

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from tests.golden.cases import CASES, iter_inputs  # noqa: E402

GOLDEN_DIR = os.path.join(ROOT, "tests", "golden")


def load_golden(name):
    z = np.load(os.path.join(GOLDEN_DIR, f"{name}.npz"))
    w = CASES[name]["workload"]
    g = {"input_sha": bytes(z["input_sha"]), "out": z["out"], "ids": [], "sal": []}
    for l in range(w.num_layers):
        ids, off = z[f"ids_{l}"], z[f"ids_off_{l}"]
        g["ids"].append([ids[off[i]:off[i + 1]] for i in range(len(off) - 1)])
        g["sal"].append(z[f"sal_{l}"])
    return g


def elt_size(dtype):
    return torch.tensor([], dtype=dtype).element_size()


def run_oracle(name):
    from oracle import razorkv_oracle as O
    case = CASES[name]
    w = case["workload"]
    cfg = O.OracleConfig(**case["razor"])
    cache = O.OracleCache(cfg, w.num_layers, elt_size(w.dtype))
    ids = [[] for _ in range(w.num_layers)]
    outs = []
    sha = hashlib.sha256()
    for kind, step, layer, tensors in iter_inputs(case):
        for t in tensors:
            sha.update(t.float().contiguous().numpy().tobytes())
        a, b, c = (t.float().numpy() for t in tensors)
        if kind == "prefill":
            K, V, q0 = a, b, c
            cache.update(K, V, layer, q0 if case["query"] else None)
        else:
            q, k, v = a, b, c
            Kc, Vc = cache.update(k, v, layer, q if case["query"] else None)
            outs.append(O.attention(q, Kc, Vc)[:, :, 0, :])
        ids[layer].append(cache.ids[layer].copy())
    return {"input_sha": sha.digest(), "out": np.stack(outs), "ids": ids,
            "sal": [s.copy() for s in cache.S], "decisions": cache.decisions, "cache": cache}


# ---- scale cases ------------------------------------------------------------------------------
def load_scale(name):
    """Reads a scale fixture: the reference's decisions, final lengths, salience sample and
    last-step outputs (see tests/golden/make_golden.py, run_reference_scale_case)."""
    from tests.golden.cases import SCALE_CASES
    z = np.load(os.path.join(GOLDEN_DIR, f"{name}.npz"))
    off = z["kept_off"]
    decisions = []
    for i in range(len(off) - 1):
        decisions.append(dict(layer=int(z["dec_layer"][i]), step=int(z["dec_step"][i]),
                              seq_len=int(z["dec_seq_len"][i]), budget=int(z["dec_budget"][i]),
                              num_pages=int(z["dec_num_pages"][i]), k=int(z["dec_k"][i]),
                              margin=float(z["dec_margin"][i]),
                              kept=z["kept"][off[i]:off[i + 1]].astype(np.int64)))
    layers = SCALE_CASES[name]["layers"]
    return {"input_sha": bytes(z["input_sha"]), "decisions": decisions,
            "len": {l: int(z[f"len_{l}"]) for l in layers},
            "sal": {l: z[f"sal_{l}"] for l in layers},
            "out": {l: z[f"out_{l}"] for l in layers}}


def near_tie(margin, score_scale):
    """True when a top-k cut is close enough to a tie that two fp32 summation orders may
    legitimately disagree on it: the gap at the cut is within 4e-6 of the largest salience
    (~34 ulps; the canonical order and torch's differ by <= 5e-7 relative on salience)."""
    return abs(margin) <= 4e-6 * max(abs(score_scale), 1.0)


def oracle_config(w):
    from oracle import razorkv_oracle as O
    return O.OracleConfig(compression_ratio=w.compression_ratio, sink_tokens=w.sink_tokens,
                          local_window=w.local_window, page_size=w.page_size,
                          pyramid_mode=w.pyramid_mode, pyramid_min_ratio=w.pyramid_min_ratio,
                          pyramid_max_ratio=w.pyramid_max_ratio)
