"""RazorEngine (razorkv/engine.py) on the CPU: the reference's engine tests
(razorkv tests/test_engine.py:26-65) plus the wiring of the q-projection hooks, which the
model must call with the pre-RoPE query before the layer's cache update."""

import inspect

import torch

from razorkv_b200 import PagedRazorKVCache, RazorConfig, RazorEngine, RazorKVCache
from razorkv_b200.engine import ATTN_IMPLEMENTATION


class DummyModelConfig:
    def __init__(self, num_hidden_layers=12):
        self.num_hidden_layers = num_hidden_layers


class DummyHFModel:
    def __init__(self, num_layers=12):
        self.config = DummyModelConfig(num_hidden_layers=num_layers)

    def prepare_inputs_for_generation(self, input_ids, past_key_values=None, **kwargs):
        return {"input_ids": input_ids, "past_key_values": past_key_values}


def test_engine_create_cache():
    cache = RazorEngine.create_cache(DummyHFModel(num_layers=16))
    assert isinstance(cache, RazorKVCache) and isinstance(cache, PagedRazorKVCache)
    assert cache.num_layers == 16
    assert RazorEngine.create_cache(5).num_layers == 5


def test_engine_patch_and_unpatch():
    model = DummyHFModel(num_layers=8)
    ids = torch.tensor([[1, 2, 3]])
    assert model.prepare_inputs_for_generation(ids)["past_key_values"] is None
    RazorEngine.patch_model(model, config=RazorConfig(compression_ratio=0.35))
    pkv = model.prepare_inputs_for_generation(ids)["past_key_values"]
    assert isinstance(pkv, RazorKVCache)
    assert pkv.config.compression_ratio == 0.35 and pkv.num_layers == 8
    RazorEngine.unpatch_model(model)
    assert model.prepare_inputs_for_generation(ids)["past_key_values"] is None


def test_engine_vram_savings_calculator():
    s = RazorEngine.estimate_vram_savings(context_len=65536, num_layers=32, num_kv_heads=8,
                                          head_dim=128, dtype_bytes=2, compression_ratio=0.30)
    assert s["savings_percentage"] == 70.0
    assert s["dense_mb"] == 2 * 32 * 8 * 128 * 2 * 65536 / 2 ** 20
    assert s["razorkv_mb"] < s["dense_mb"]
    assert s["saved_mb"] == s["dense_mb"] - s["razorkv_mb"]


class RecordingCache(PagedRazorKVCache):
    """Dense CPU stand-in that records the calls the patched model makes."""

    def __init__(self, *a, **kw):
        super().__init__(*a, **kw)
        self.events = []
        self.dense = {}

    def update_salience_with_query(self, query_states, layer_idx):
        self.events.append(("score", layer_idx, query_states.detach().clone()))

    def update(self, key_states, value_states, layer_idx, cache_kwargs=None):
        self.events.append(("update", layer_idx, tuple(key_states.shape)))
        K, V = self.dense.get(layer_idx, (None, None))
        K = key_states if K is None else torch.cat([K, key_states], dim=2)
        V = value_states if V is None else torch.cat([V, value_states], dim=2)
        self.dense[layer_idx] = (K, V)
        if layer_idx == 0:
            self._seen_tokens += key_states.shape[2]
        return K, V

    def get_seq_length(self, layer_idx=0):
        return self._seen_tokens

    def get_mask_sizes(self, query_length, layer_idx=0):
        q_len = query_length.shape[0] if isinstance(query_length, torch.Tensor) else int(query_length)
        n = self.dense[layer_idx][0].shape[2] if layer_idx in self.dense else 0
        return n + q_len, 0


def _tiny_llama(layers=2):
    from transformers import LlamaConfig, LlamaForCausalLM
    torch.manual_seed(0)
    cfg = LlamaConfig(vocab_size=128, hidden_size=64, num_hidden_layers=layers,
                      num_attention_heads=4, num_key_value_heads=2, intermediate_size=128,
                      max_position_embeddings=512)
    return LlamaForCausalLM(cfg).eval()


def test_patched_model_scores_pre_rope_query_before_update():
    model = _tiny_llama()
    orig_impl = model.config._attn_implementation
    RazorEngine.patch_model(model, config=RazorConfig())
    assert model.config._attn_implementation == ATTN_IMPLEMENTATION
    assert len(model._razorkv_hook_handles) == 2
    # generate validates its kwargs against forward's signature: the wrapper must keep it
    assert "attention_mask" in inspect.signature(model.forward).parameters
    cache = RecordingCache(num_layers=2)
    ids = torch.randint(0, 128, (2, 7))
    with torch.no_grad():
        model(input_ids=ids, past_key_values=cache, use_cache=True)
        model(input_ids=ids[:, :1], past_key_values=cache, use_cache=True)
    assert RazorEngine._active_cache.get() is None
    kinds = [(e[0], e[1]) for e in cache.events]
    assert kinds == [("score", 0), ("update", 0), ("score", 1), ("update", 1)] * 2
    # the hook sees q_proj's output (pre-RoPE), [B, Hq, q_len, D]
    attn0 = model.model.layers[0].self_attn
    with torch.no_grad():
        h = model.model.layers[0].input_layernorm(model.model.embed_tokens(ids))
        q = attn0.q_proj(h).view(2, 7, 4, 16).transpose(1, 2)
    assert torch.equal(cache.events[0][2], q)
    assert cache.events[4][2].shape == (2, 4, 1, 16)
    # the paged-attention flag reached the cache through the patched forward
    assert cache.return_handles is True
    RazorEngine.unpatch_model(model)
    assert model.config._attn_implementation == orig_impl
    assert not hasattr(model, "_razorkv_hook_handles")
    assert all(not m._forward_hooks for m in model.modules())


def test_patch_without_paged_attention_keeps_implementation():
    model = _tiny_llama(layers=1)
    impl = model.config._attn_implementation
    RazorEngine.patch_model(model, paged_attention=False)
    assert model.config._attn_implementation == impl
    cache = RecordingCache(num_layers=1)
    with torch.no_grad():
        model(input_ids=torch.randint(0, 128, (1, 5)), past_key_values=cache, use_cache=True)
    assert cache.return_handles is False
    RazorEngine.unpatch_model(model)
