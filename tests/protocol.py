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
