"""Time the reference's own CPU decode path beside the oracle port, on the same sample.

Usage (in a checkout where the reference project is available):

    python tests/golden/time_reference.py /path/to/razorkv-reference

The reference is Python and cannot travel to the GPU box, so the benchmark's CPU baseline
times the oracle port there; this script calibrates that port against the reference itself
on one host.  Sample, for each workload: the shallowest and deepest layers after a full
prefill (untimed), then decode steps timed per layer -- the reference's
``RazorKVCache.update(k, v, l, {"query_states": q})`` followed by ``compacted_paged_sdpa``
(razorkv/cache.py:361-414, razorkv/kernels/torch_sparse.py:15-61) against the oracle's
``update`` + ``attention`` on identical inputs.  A full step is extrapolated from the sampled
layers' seconds per retained token, as the benchmark does.  The result is written to
tests/golden/reference_timing.json with the host's core count.
"""

import json
import os
import sys
import time

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.abspath(os.path.join(HERE, "..", "..")))

STEPS = 2


def _sample(w, ref_root):
    sys.path.insert(0, ref_root)
    from razorkv.cache import RazorKVCache
    from razorkv.config import RazorConfig
    from razorkv.kernels.torch_sparse import compacted_paged_sdpa

    from oracle import razorkv_oracle as O
    from razorkv_b200.workload import decode_inputs, layer_prefill

    L = w.num_layers
    layers = sorted({0, L - 1})
    kw = dict(compression_ratio=w.compression_ratio, sink_tokens=w.sink_tokens,
              local_window=w.local_window, page_size=w.page_size, pyramid_mode=w.pyramid_mode,
              pyramid_min_ratio=w.pyramid_min_ratio, pyramid_max_ratio=w.pyramid_max_ratio)
    ref = RazorKVCache(config=RazorConfig(**kw), num_layers=L)
    orc = O.OracleCache(O.OracleConfig(**kw), L, torch.tensor([], dtype=w.dtype).element_size())
    for l in layers:
        K, V, q0 = layer_prefill(w, l, "cpu")
        ref.update(K, V, l, {"query_states": q0})
        orc.update(K.float().numpy(), V.float().numpy(), l, q0.float().numpy())
        del K, V
    t_ref = t_orc = 0.0
    n_ref = n_orc = 0
    for step in range(STEPS):
        for l in layers:
            q, k, v = decode_inputs(w, step, l, "cpu")
            t0 = time.perf_counter()
            Kc, Vc = ref.update(k, v, l, {"query_states": q})
            compacted_paged_sdpa(q, Kc, Vc)
            t_ref += time.perf_counter() - t0
            n_ref += Kc.shape[2]
            qn, kn, vn = q.float().numpy(), k.float().numpy(), v.float().numpy()
            t0 = time.perf_counter()
            Ko, Vo = orc.update(kn, vn, l, qn)
            O.attention(qn, Ko, Vo)
            t_orc += time.perf_counter() - t0
            n_orc += Ko.shape[2]
    T = orc.seen
    retained = sum(orc.K[l].shape[2] if l in layers else orc.cfg.budget(l, L, T) for l in range(L))
    out = {}
    for name, t, n in (("reference_torch", t_ref, n_ref), ("oracle_port", t_orc, n_orc)):
        step_s = t / n * retained
        out[name] = {"tokens_per_s": w.batch / step_s, "ms_per_step_extrapolated": step_s * 1e3,
                     "sampled_seconds": t}
    out["port_over_reference"] = out["oracle_port"]["tokens_per_s"] / out["reference_torch"]["tokens_per_s"]
    out["sample"] = (f"layers {layers} of {L}, batch {w.batch}, {w.context}-token prefill "
                     f"(untimed), {STEPS} decode steps; full step extrapolated to {retained} "
                     f"retained tokens over {L} layers")
    return out


def main():
    ref_root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("RAZORKV_REFERENCE", "")
    if not ref_root or not os.path.isdir(os.path.join(ref_root, "razorkv")):
        raise SystemExit("pass the path of the reference project (the directory holding razorkv/)")
    from razorkv_b200.workload import WORKLOADS
    torch.set_num_threads(os.cpu_count() or 1)
    os.environ.setdefault("ORACLE_THREADS", str(os.cpu_count() or 1))
    res = {"cores": os.cpu_count(), "torch_threads": torch.get_num_threads(),
           "torch": torch.__version__, "workloads": {}}
    for name in sys.argv[2:] or ["llama8b-b8-32k-bf16", "qwen7b-b1-128k-bf16"]:
        res["workloads"][name] = _sample(WORKLOADS[name], ref_root)
        print(name, json.dumps(res["workloads"][name]), flush=True)
    with open(os.path.join(HERE, "reference_timing.json"), "w") as f:
        json.dump(res, f, indent=1)


if __name__ == "__main__":
    main()
