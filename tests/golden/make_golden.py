"""Regenerate the golden fixtures by running the REFERENCE implementation.

Usage (in a checkout where the reference project is available):

    python tests/golden/make_golden.py /path/to/razorkv-reference

For every case below the script draws the seeded synthetic workload with
``razorkv_b200.workload`` (CPU generators, deterministic for a given torch build), drives
the reference's own ``RazorKVCache.update(..., {"query_states": q})`` followed by
``compacted_paged_sdpa`` -- the decode-step protocol of the reference's benchmark loop
(razorkv/evaluation/benchmark_runner.py:259-281) with the query passed in ``cache_kwargs``
(razorkv/cache.py:392-393) -- and records what the reference produced:

* ``ids_<l>``/``ids_off_<l>``: the retained token ids of layer l after every step
  (prefill = step -1), recovered by matching retained key rows to the rows that were fed in;
* ``out``: the attention output of every decode step (fp32);
* ``sal_<l>``: the final salience of layer l (fp32);
* ``input_sha``: a digest of every input tensor, so tests can check that regeneration
  reproduces the exact inputs.

The fixtures are read by tests/test_oracle_golden.py (oracle vs reference, CPU) and by
tests/test_gpu_golden.py (CUDA path vs reference, GPU).

The scale cases (``SCALE_CASES``: a layer pair of the Llama-8B-shaped and Qwen-7B-shaped
workloads at their full batch and context) are too large to store tensor by tensor; for
them the script records the reference's top-k decisions instead (see
``run_reference_scale_case``).  They are read by tests/test_oracle_scale.py (CPU) and
tests/test_gpu_scale.py (GPU).
"""

import hashlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.abspath(os.path.join(HERE, "..", "..")))

from tests.golden.cases import CASES, iter_inputs  # noqa: E402


def row_key(x: torch.Tensor) -> bytes:
    return x.float().contiguous().numpy().tobytes()


def run_reference_case(name, case, ref_root):
    sys.path.insert(0, ref_root)
    from razorkv.cache import RazorKVCache
    from razorkv.config import RazorConfig
    from razorkv.kernels.torch_sparse import compacted_paged_sdpa

    w = case["workload"]
    cfg = RazorConfig(**case["razor"])
    cache = RazorKVCache(config=cfg, num_layers=w.num_layers)
    L = w.num_layers
    rows = [dict() for _ in range(L)]
    next_id = [0] * L
    ids_hist = [[] for _ in range(L)]
    outs = []
    sha = hashlib.sha256()

    def register(layer, k):
        # k [B, Hkv, T, D]: identify tokens by their (b=0, h=0) key row
        for t in range(k.shape[2]):
            key = row_key(k[0, 0, t])
            assert key not in rows[layer], "duplicate key row in workload"
            rows[layer][key] = next_id[layer]
            next_id[layer] += 1

    def retained(layer):
        K = cache.key_cache[layer]
        return np.array([rows[layer][row_key(K[0, 0, t])] for t in range(K.shape[2])], np.int64)

    for kind, step, layer, tensors in iter_inputs(case):
        for t in tensors:
            sha.update(t.float().contiguous().numpy().tobytes())
        if kind == "prefill":
            K, V, q0 = tensors
            register(layer, K)
            kw = {"query_states": q0} if case["query"] else None
            cache.update(K, V, layer, kw)
            ids_hist[layer].append(retained(layer))
        else:
            q, k, v = tensors
            register(layer, k)
            kw = {"query_states": q} if case["query"] else None
            Kc, Vc = cache.update(k, v, layer, kw)
            out = compacted_paged_sdpa(q, Kc, Vc)
            outs.append(out.float()[:, :, 0, :].numpy())
            ids_hist[layer].append(retained(layer))

    arrays = {"input_sha": np.frombuffer(sha.digest(), np.uint8), "out": np.stack(outs)}
    for l in range(L):
        arrays[f"ids_{l}"] = np.concatenate(ids_hist[l])
        arrays[f"ids_off_{l}"] = np.cumsum([0] + [len(a) for a in ids_hist[l]]).astype(np.int64)
        arrays[f"sal_{l}"] = cache.salience_scores[l].float().numpy()
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **arrays)
    print(f"{name}: {len(outs)} steps, final lengths",
          [cache.key_cache[l].shape[2] for l in range(L)])


def run_reference_scale_case(name, case, ref_root):
    """A scale case: records every top-k decision of the reference instead of every tensor.

    ``torch.topk`` is wrapped while the reference runs, so each call of its page selection
    (razorkv/cache.py:340) is seen with its own input -- the batch-mean page scores -- and its
    own result.  Per decision the fixture holds the layer, the decode step (-1 = prefill), the
    cached length and budget, the number of haystack pages, the kept page indices (sorted, as
    razorkv/cache.py:341 sorts them) and the gap between the k-th and (k+1)-th largest page
    score (the margin a few-ulp score difference would have to cross to change the set)."""
    import time

    sys.path.insert(0, ref_root)
    from razorkv.cache import RazorKVCache
    from razorkv.config import RazorConfig
    from razorkv.kernels.torch_sparse import compacted_paged_sdpa

    from tests.golden.cases import SCALE_SAL_STRIDE, iter_scale_inputs, scale_input_digest

    w = case["workload"]
    cfg = RazorConfig(compression_ratio=w.compression_ratio, sink_tokens=w.sink_tokens,
                      local_window=w.local_window, page_size=w.page_size,
                      pyramid_mode=w.pyramid_mode, pyramid_min_ratio=w.pyramid_min_ratio,
                      pyramid_max_ratio=w.pyramid_max_ratio)
    cache = RazorKVCache(config=cfg, num_layers=w.num_layers)
    seen_topk = []
    orig_topk = torch.topk

    def topk_spy(x, k, *a, **kw):
        res = orig_topk(x, k, *a, **kw)
        vals = torch.sort(x.detach().float(), descending=True).values
        margin = float(vals[k - 1] - vals[k]) if k < x.numel() else float("inf")
        seen_topk.append((x.numel(), k, torch.sort(res.indices).values.numpy().astype(np.int32),
                          margin))
        return res

    sha = hashlib.sha256()
    dec = {"layer": [], "step": [], "seq_len": [], "budget": [], "num_pages": [], "k": [],
           "margin": []}
    kept_all = []
    last_out = {}
    t_start = time.time()
    torch.topk = topk_spy
    try:
        for kind, step, layer, tensors in iter_scale_inputs(case):
            scale_input_digest(sha, kind, tensors)
            seen_topk.clear()
            before = cache.key_cache[layer].shape[2] if (
                layer < len(cache.key_cache) and cache.key_cache[layer] is not None) else 0
            if kind == "prefill":
                K, V, q0 = tensors
                cache.update(K, V, layer, {"query_states": q0} if case["query"] else None)
                before = K.shape[2]
            else:
                q, k, v = tensors
                before += 1
                Kc, Vc = cache.update(k, v, layer, {"query_states": q} if case["query"] else None)
                last_out[layer] = compacted_paged_sdpa(q, Kc, Vc).float()[:, :, 0, :].numpy()
            assert len(seen_topk) <= 1
            for n, k, kept, margin in seen_topk:
                seen = max(cache._seen_tokens, before)
                dec["layer"].append(layer)
                dec["step"].append(step)
                dec["seq_len"].append(before)
                dec["budget"].append(cfg.get_layer_budget(layer, w.num_layers, seen))
                dec["num_pages"].append(n)
                dec["k"].append(k)
                dec["margin"].append(margin)
                kept_all.append(kept)
                print(f"  {name}: layer {layer} step {step} N={before} pages={n} k={k} "
                      f"margin={margin:.3e} ({time.time() - t_start:.0f}s)", flush=True)
    finally:
        torch.topk = orig_topk

    arrays = {"input_sha": np.frombuffer(sha.digest(), np.uint8),
              "kept": np.concatenate(kept_all),
              "kept_off": np.cumsum([0] + [len(a) for a in kept_all]).astype(np.int64)}
    for key, vals in dec.items():
        arrays[f"dec_{key}"] = np.array(vals, np.float64 if key == "margin" else np.int64)
    for layer in case["layers"]:
        arrays[f"len_{layer}"] = np.array(cache.key_cache[layer].shape[2], np.int64)
        arrays[f"sal_{layer}"] = cache.salience_scores[layer].float().numpy()[:, ::SCALE_SAL_STRIDE].copy()
        arrays[f"out_{layer}"] = last_out[layer]
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **arrays)
    print(f"{name}: {len(kept_all)} decisions, final lengths",
          [cache.key_cache[l].shape[2] for l in case["layers"]],
          f"min margin {min(dec['margin']):.3e}, {time.time() - t_start:.0f}s")


def main():
    ref_root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("RAZORKV_REFERENCE", "")
    if not ref_root or not os.path.isdir(os.path.join(ref_root, "razorkv")):
        raise SystemExit("pass the path of the reference project (the directory holding razorkv/)")
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    from tests.golden.cases import SCALE_CASES
    only = sys.argv[2:] or list(CASES) + list(SCALE_CASES)
    for name in only:
        if name in SCALE_CASES:
            run_reference_scale_case(name, SCALE_CASES[name], ref_root)
        else:
            run_reference_case(name, CASES[name], ref_root)


if __name__ == "__main__":
    main()
