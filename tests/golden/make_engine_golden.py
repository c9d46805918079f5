"""Record the reference engine on a small Llama: logits and kept tokens under teacher forcing.

Usage (in a checkout where the reference project is available):

    python tests/golden/make_engine_golden.py /path/to/razorkv-reference

A random-init Llama-architecture model (``ENGINE_CASE``: 4 layers, 4 query / 1 kv head,
head_dim 128, seeded weights, fp32) is patched with the reference's own
``RazorEngine.patch_model`` (razorkv/engine.py:39-133): the q_proj hooks score the cached
tokens with the pre-RoPE query, then each layer's ``update`` appends and compacts
(razorkv/cache.py:249-414).  The script runs the model on the CPU like ``generate`` does --
one prompt forward, then one forward per token, greedy -- and records:

* ``tokens``: the prompt and the greedy continuation (the sequence every replay feeds);
* ``logits``: the last-position logits of every forward (fp32);
* every compaction of every layer: the forward it happened in, the layer, and the retained
  token positions afterwards (recovered by matching the layer's retained key rows to the rows
  it appended), plus the gap at the top-k cut of that compaction (from the reference's own
  ``torch.topk`` call; +inf for the no-haystack branch).

fp32 keeps the CPU and GPU model arithmetic within ~1e-6 relative of each other, far below
the recorded cuts; in bf16 the two sides' matmuls round differently by up to an ulp of
bf16, which is above them.  The fixture is read by tests/test_gpu_engine_reference.py.
"""

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.abspath(os.path.join(HERE, "..", "..")))

ENGINE_CASE = dict(layers=4, hidden=512, heads=4, kv_heads=1, head_dim=128,
                   intermediate=1024, vocab=512, batch=2, prompt=768, new_tokens=64,
                   weight_seed=0, prompt_seed=1,
                   razor=dict(compression_ratio=0.30, sink_tokens=32, local_window=128,
                              page_size=16))


def build_model(case, device="cpu", dtype=torch.float32):
    """The seeded model (same weights on any device: drawn on the CPU, then moved)."""
    from transformers import LlamaConfig, LlamaForCausalLM
    torch.manual_seed(case["weight_seed"])
    cfg = LlamaConfig(vocab_size=case["vocab"], hidden_size=case["hidden"],
                      num_hidden_layers=case["layers"], num_attention_heads=case["heads"],
                      num_key_value_heads=case["kv_heads"], head_dim=case["head_dim"],
                      intermediate_size=case["intermediate"], max_position_embeddings=4096,
                      attn_implementation="sdpa")
    return LlamaForCausalLM(cfg).to(device=device, dtype=dtype).eval()


def prompt_ids(case):
    g = torch.Generator().manual_seed(case["prompt_seed"])
    return torch.randint(0, case["vocab"], (case["batch"], case["prompt"]), generator=g)


class RowIds:
    """Maps each layer's appended key rows (sequence 0, kv head 0) to token positions."""

    def __init__(self):
        self.rows = {}

    def add(self, layer, k, first_pos):
        d = self.rows.setdefault(layer, {})
        k0 = k[0, 0].detach().float().cpu().contiguous().numpy()
        for i in range(k0.shape[0]):
            d[k0[i].tobytes()] = first_pos + i

    def ids(self, layer, K):
        d = self.rows[layer]
        k0 = K[0, 0].detach().float().cpu().contiguous().numpy()
        return np.array([d[k0[i].tobytes()] for i in range(k0.shape[0])], np.int64)


def main():
    ref_root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("RAZORKV_REFERENCE", "")
    if not ref_root or not os.path.isdir(os.path.join(ref_root, "razorkv")):
        raise SystemExit("pass the path of the reference project (the directory holding razorkv/)")
    sys.path.insert(0, ref_root)
    from razorkv.cache import RazorKVCache
    from razorkv.config import RazorConfig
    from razorkv.engine import RazorEngine

    case = ENGINE_CASE
    torch.set_num_threads(os.cpu_count() or 1)
    model = build_model(case)
    RazorEngine.patch_model(model, config=RazorConfig(**case["razor"]))
    cache = RazorKVCache(config=RazorConfig(**case["razor"]), num_layers=case["layers"])

    rows = RowIds()
    margins = []
    orig_topk = torch.topk

    def topk_spy(x, k, *a, **kw):
        vals = torch.sort(x.detach().float(), descending=True).values
        margins.append(float(vals[k - 1] - vals[k]) if k < x.numel() else float("inf"))
        return orig_topk(x, k, *a, **kw)

    orig_update = cache.update
    events = []            # (forward index, layer, retained positions, margin)
    state = {"fwd": 0}

    def rec_update(k, v, layer_idx, cache_kwargs=None):
        before = 0 if (layer_idx >= len(cache.key_cache) or cache.key_cache[layer_idx] is None) \
            else cache.key_cache[layer_idx].shape[2]
        # positions of the appended tokens: the layer's count of tokens appended so far
        seen = rows.rows.get(layer_idx, {})
        rows.add(layer_idx, k, len(seen))
        n_marg = len(margins)
        out = orig_update(k, v, layer_idx, cache_kwargs)
        after = cache.key_cache[layer_idx].shape[2]
        if after != before + k.shape[2]:   # compacted
            m = margins[n_marg] if len(margins) > n_marg else float("inf")
            events.append((state["fwd"], layer_idx, rows.ids(layer_idx, cache.key_cache[layer_idx]), m))
        return out

    cache.update = rec_update
    ids = prompt_ids(case)
    tokens = [ids]
    logits = []
    torch.topk = topk_spy
    try:
        with torch.no_grad():
            out = model(input_ids=ids, past_key_values=cache, use_cache=True)
            for step in range(case["new_tokens"]):
                last = out.logits[:, -1, :].float()
                logits.append(last.numpy())
                nxt = last.argmax(dim=-1, keepdim=True)
                tokens.append(nxt)
                state["fwd"] += 1
                if step == case["new_tokens"] - 1:
                    break
                out = model(input_ids=nxt, past_key_values=cache, use_cache=True)
    finally:
        torch.topk = orig_topk
    arrays = {
        "tokens": torch.cat(tokens, dim=1).numpy().astype(np.int64),
        "logits": np.stack(logits).astype(np.float32),
        "ev_forward": np.array([e[0] for e in events], np.int64),
        "ev_layer": np.array([e[1] for e in events], np.int64),
        "ev_margin": np.array([e[3] for e in events], np.float64),
        "ev_ids": np.concatenate([e[2] for e in events]) if events else np.zeros(0, np.int64),
        "ev_off": np.cumsum([0] + [len(e[2]) for e in events]).astype(np.int64),
        "final_len": np.array([cache.key_cache[l].shape[2] for l in range(case["layers"])], np.int64),
    }
    path = os.path.join(HERE, "engine_llama4l_fp32.npz")
    np.savez_compressed(path, **arrays)
    print(f"{len(events)} compactions over {case['layers']} layers "
          f"({sum(1 for e in events if e[0] > 0)} during decode), final lengths "
          f"{arrays['final_len'].tolist()}, min margin "
          f"{min((e[3] for e in events), default=float('inf')):.3e}")


if __name__ == "__main__":
    main()
