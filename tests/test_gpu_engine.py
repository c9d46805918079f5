"""RazorEngine with a real HF Llama on the GPU (razorkv tests/test_engine.py:68-103), and an
oracle replay of a patched model's generate: every hook score, cache update and decode
attention the model performs is recorded and replayed, in the same order, through the CPU
oracle; the retained K/V and salience must match bit for bit and every decode attention
output within the dtype's tolerance."""

import math

import numpy as np
import pytest
import torch

from oracle import razorkv_oracle as O
from razorkv_b200 import PagedKV, PagedRazorKVCache, RazorConfig, RazorEngine, RazorKVCache
from razorkv_b200 import engine as E

pytestmark = pytest.mark.gpu

TOL = {torch.float32: (1e-5, 1e-5), torch.bfloat16: (2e-2, 1e-2)}


def _llama(hidden, heads, kv_heads, layers, vocab=128, dtype=torch.float32, seed=0):
    from transformers import LlamaConfig, LlamaForCausalLM
    torch.manual_seed(seed)
    cfg = LlamaConfig(vocab_size=vocab, hidden_size=hidden, num_hidden_layers=layers,
                      num_attention_heads=heads, num_key_value_heads=kv_heads,
                      intermediate_size=2 * hidden, max_position_embeddings=4096)
    return LlamaForCausalLM(cfg).to(device="cuda", dtype=dtype).eval()


def test_engine_real_hf_model_patch_and_generate():
    model = _llama(64, 4, 2, 2)
    razor_cfg = RazorConfig(compression_ratio=0.30, sink_tokens=8, local_window=16, page_size=4)
    RazorEngine.patch_model(model, config=razor_cfg)
    prompt = torch.randint(0, 128, (1, 80), device="cuda")
    with torch.no_grad():
        out = model.generate(prompt, max_new_tokens=10, eos_token_id=None,
                             return_dict_in_generate=True)
    assert out.sequences.shape[1] == 90
    assert isinstance(out.past_key_values, RazorKVCache)
    assert out.past_key_values.get_cached_seq_length(0) < 80
    assert out.past_key_values.seen_tokens >= 89
    RazorEngine.unpatch_model(model)
    with torch.no_grad():
        stock = model.generate(prompt, max_new_tokens=2, return_dict_in_generate=True)
    assert not isinstance(stock.past_key_values, RazorKVCache)


def _oracle_config(c: RazorConfig) -> O.OracleConfig:
    return O.OracleConfig(compression_ratio=c.compression_ratio, sink_tokens=c.sink_tokens,
                          local_window=c.local_window, page_size=c.page_size,
                          pyramid_mode=c.pyramid_mode, pyramid_min_ratio=c.pyramid_min_ratio,
                          pyramid_max_ratio=c.pyramid_max_ratio,
                          salience_decay=c.salience_decay, salience_init=c.salience_init)


def _record(cache: PagedRazorKVCache, log):
    score, update = cache.update_salience_with_query, cache.update

    def rec_score(q, layer_idx):
        log.append(("score", layer_idx, q.detach().float().cpu()))
        return score(q, layer_idx)

    def rec_update(k, v, layer_idx, cache_kwargs=None):
        log.append(("update", layer_idx, k.detach().float().cpu(), v.detach().float().cpu()))
        return update(k, v, layer_idx, cache_kwargs)

    cache.update_salience_with_query = rec_score
    cache.update = rec_update


@pytest.mark.parametrize("dtype,hidden,heads,kv_heads", [
    (torch.float32, 256, 4, 2),       # head_dim 64, GQA 2: shape-general kernels
    (torch.bfloat16, 512, 4, 1),      # head_dim 128, GQA 4: the sm_100a decode kernel
])
def test_generate_replays_through_oracle(dtype, hidden, heads, kv_heads):
    from transformers.modeling_utils import AttentionInterface
    layers, T, new = 2, 300, 40
    D = hidden // heads
    model = _llama(hidden, heads, kv_heads, layers, vocab=256, dtype=dtype, seed=1)
    rcfg = RazorConfig(compression_ratio=0.30, sink_tokens=16, local_window=32, page_size=16)
    RazorEngine.patch_model(model, config=rcfg)
    log = []

    def rec_attention(module, query, key, value, mask, **kw):
        out, w = E.razorkv_paged_attention(module, query, key, value, mask, **kw)
        if query.shape[2] == 1:
            log.append(("attn", module.layer_idx, query.detach().float().cpu(),
                        out.detach().float().cpu(), isinstance(key, PagedKV)))
        return out, w

    AttentionInterface.register(E.ATTN_IMPLEMENTATION, rec_attention)
    try:
        cache = PagedRazorKVCache(config=rcfg, num_layers=layers)
        _record(cache, log)
        g = torch.Generator().manual_seed(2)
        prompt = torch.randint(1, 256, (2, T), generator=g).cuda()
        with torch.no_grad():
            model.generate(prompt, attention_mask=torch.ones_like(prompt), past_key_values=cache,
                           max_new_tokens=new, do_sample=False, eos_token_id=None,
                           pad_token_id=0)
        torch.cuda.synchronize()
    finally:
        E.register_attention()
        RazorEngine.unpatch_model(model)

    oc = O.OracleCache(_oracle_config(rcfg), layers, 4 if dtype == torch.float32 else 2)
    atol, rtol = TOL[dtype]
    n_attn = 0
    for ev in log:
        if ev[0] == "score":
            oc.update_salience_with_query(ev[2].numpy(), ev[1])
        elif ev[0] == "update":
            oc.update(ev[2].numpy(), ev[3].numpy(), ev[1])
        else:
            _, l, q, out, paged = ev
            assert paged, "decode attention did not run from the page pool"
            ref = O.attention(q.numpy(), oc.K[l], oc.V[l], scale=1.0 / math.sqrt(D))
            np.testing.assert_allclose(out.transpose(1, 2).numpy(), ref, atol=atol, rtol=rtol)
            n_attn += 1
    assert n_attn == layers * (new - 1)
    assert any(d.kind == "pages" for d in oc.decisions), "no compaction was exercised"
    for l in range(layers):   # one compaction at prefill and at least one while decoding
        assert sum(1 for d in oc.decisions if d.layer == l) >= 2, f"layer {l}: no decode compaction"
    for l in range(layers):
        K = cache._materialize(l, 0).float().cpu().numpy()
        S = cache._materialize(l, 2).cpu().numpy()
        assert np.array_equal(K, oc.K[l]), f"layer {l}: retained K differs"
        assert np.array_equal(S.view(np.uint32), oc.S[l].view(np.uint32)), f"layer {l}: salience"


def test_paged_attention_generates_the_same_tokens():
    model = _llama(256, 4, 2, 2, vocab=256, seed=3)
    rcfg = RazorConfig(compression_ratio=0.30, sink_tokens=16, local_window=32, page_size=16)
    prompt = torch.randint(1, 256, (2, 200), generator=torch.Generator().manual_seed(4)).cuda()
    outs = []
    for paged in (True, False):
        RazorEngine.patch_model(model, config=rcfg, paged_attention=paged)
        with torch.no_grad():
            outs.append(model.generate(prompt, attention_mask=torch.ones_like(prompt),
                                       max_new_tokens=24, do_sample=False, eos_token_id=None,
                                       pad_token_id=0))
        RazorEngine.unpatch_model(model)
    assert torch.equal(outs[0], outs[1])


@pytest.mark.parametrize("dtype,hidden,heads,kv_heads", [
    (torch.float32, 256, 4, 2),       # head_dim 64: shape-general kernels
    (torch.bfloat16, 512, 4, 1),      # head_dim 128: the sm_100a decode kernel
])
def test_beam_search_on_shared_pages(dtype, hidden, heads, kv_heads, monkeypatch):
    """HF beam search calls reorder_cache every step.  Sharing pages through the row map must
    generate exactly what moving the rows generates (same tokens, same beam scores), with
    compactions during the search."""
    model = _llama(hidden, heads, kv_heads, 2, vocab=256, dtype=dtype, seed=5)
    rcfg = RazorConfig(compression_ratio=0.30, sink_tokens=16, local_window=32, page_size=16)
    prompt = torch.randint(1, 256, (2, 300), generator=torch.Generator().manual_seed(6)).cuda()
    runs = []
    for share in (True, False):
        monkeypatch.setattr(PagedRazorKVCache, "share_pages_on_reorder", share)
        RazorEngine.patch_model(model, config=rcfg)
        with torch.no_grad():
            out = model.generate(prompt, attention_mask=torch.ones_like(prompt), num_beams=3,
                                 max_new_tokens=40, do_sample=False, eos_token_id=None,
                                 pad_token_id=0, return_dict_in_generate=True,
                                 output_scores=True)
        RazorEngine.unpatch_model(model)
        cache = out.past_key_values
        assert isinstance(cache, PagedRazorKVCache)
        assert (cache._rowmap is not None) == share
        assert cache.compactions > 2 * 2   # prefill compactions plus decode-time ones
        cache.check_errors()
        runs.append(out)
    assert torch.equal(runs[0].sequences, runs[1].sequences)
    assert torch.equal(runs[0].sequences_scores, runs[1].sequences_scores)
