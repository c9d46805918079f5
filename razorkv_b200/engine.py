"""RazorEngine: the reference's HuggingFace model patcher (razorkv/engine.py:15-178) over the
paged cache.

``patch_model(model, config)`` keeps the reference's four patches:

1. ``generate`` injects a fresh cache when the caller passes none (razorkv/engine.py:69-76);
2. ``prepare_inputs_for_generation`` does the same for direct callers (:78-85);
3. ``forward`` makes the cache it is given the active one for the hooks (:87-99);
4. a forward hook on every attention block's ``q_proj`` scores the cached tokens with the
   pre-RoPE query, before the layer appends its new token (:101-130);

and adds one: the model's attention implementation becomes ``"razorkv_paged"``, registered
with transformers' ``AttentionInterface``.  On decode steps the cache's ``update`` then
returns ``PagedKV`` handles and the attention runs straight from the page pool (no gather of
the retained K/V).  Prefill, and any call that carries a mask or dropout, goes to
transformers' SDPA attention over materialised K/V -- what the reference model computes.
``patch_model(..., paged_attention=False)`` leaves the model's attention implementation
alone; ``update`` then returns gathered K/V like the reference cache.
"""

import contextvars
import functools
from typing import Any, Dict, Optional, Union

import torch

from .cache import PagedKV, PagedRazorKVCache
from .config import RazorConfig

ATTN_IMPLEMENTATION = "razorkv_paged"


def razorkv_paged_attention(module, query: torch.Tensor, key, value, attention_mask,
                            dropout: float = 0.0, scaling: Optional[float] = None,
                            is_causal: Optional[bool] = None, **kwargs):
    """transformers attention function: query [B, H, q_len, D] (post-RoPE) -> ([B, q_len, H, D],
    None).  Decode steps over a paged layer read the pool; everything else is SDPA."""
    if isinstance(key, PagedKV):
        if query.shape[2] == 1 and attention_mask is None and not dropout:
            out = key.cache.attention(query, key.layer, scaling)
            return out.transpose(1, 2), None
        key, value = key.materialize(), value.materialize()
    from transformers.integrations.sdpa_attention import sdpa_attention_forward
    return sdpa_attention_forward(module, query, key, value, attention_mask, dropout=dropout,
                                  scaling=scaling, is_causal=is_causal, **kwargs)


def register_attention() -> str:
    """Registers ``razorkv_paged`` (attention function and SDPA-style mask) with
    transformers; returns the name."""
    from transformers.masking_utils import AttentionMaskInterface, sdpa_mask
    from transformers.modeling_utils import AttentionInterface
    AttentionInterface.register(ATTN_IMPLEMENTATION, razorkv_paged_attention)
    AttentionMaskInterface.register(ATTN_IMPLEMENTATION, sdpa_mask)
    return ATTN_IMPLEMENTATION


def _num_layers(model: Any) -> int:
    cfg = getattr(model, "config", None)
    return getattr(cfg, "num_hidden_layers", getattr(cfg, "n_layer", 32))


def _decoder_layers(model: Any):
    # razorkv/engine.py:102-106
    layers = getattr(model, "layers", None)
    if layers is None and hasattr(model, "model") and hasattr(model.model, "layers"):
        layers = model.model.layers
    elif layers is None and hasattr(model, "transformer") and hasattr(model.transformer, "h"):
        layers = model.transformer.h
    return layers


class RazorEngine:
    """High-level engine: creates caches and patches HF models to use the paged cache."""

    _active_cache: contextvars.ContextVar = contextvars.ContextVar("active_razorkv_cache",
                                                                   default=None)

    @staticmethod
    def create_cache(model_or_num_layers: Union[int, Any],
                     config: Optional[RazorConfig] = None) -> PagedRazorKVCache:
        """razorkv/engine.py:20-37: a cache sized for the model (or the layer count)."""
        if isinstance(model_or_num_layers, int):
            num_layers = model_or_num_layers
        elif hasattr(model_or_num_layers, "config"):
            num_layers = _num_layers(model_or_num_layers)
        else:
            num_layers = 32
        return PagedRazorKVCache(config=config, num_layers=num_layers)

    @classmethod
    def patch_model(cls, model: Any, config: Optional[RazorConfig] = None,
                    paged_attention: bool = True) -> Any:
        """razorkv/engine.py:39-133: patch a PreTrainedModel so that ``generate`` uses the
        paged cache.  Non-destructive: ``unpatch_model`` restores the model."""
        razor_cfg = config or RazorConfig()
        num_layers = _num_layers(model)

        if not hasattr(model, "_orig_generate"):
            model._orig_generate = getattr(model, "generate", None)
            model._orig_prepare_inputs_for_generation = getattr(
                model, "prepare_inputs_for_generation", None)
            model._orig_forward = getattr(model, "forward", None)
            model._razorkv_hook_handles = []
            model._is_razorkv_patched = True
        else:   # re-patching: drop the previous hooks first
            for h in model._razorkv_hook_handles:
                h.remove()
            model._razorkv_hook_handles.clear()

        orig_gen = model._orig_generate
        orig_prepare = model._orig_prepare_inputs_for_generation
        orig_forward = model._orig_forward

        def new_cache():
            return PagedRazorKVCache(config=razor_cfg, num_layers=num_layers)

        if orig_gen is not None:
            @functools.wraps(orig_gen)
            def razor_generate(*args, **kwargs):
                if kwargs.get("past_key_values") is None:
                    kwargs["past_key_values"] = new_cache()
                return orig_gen(*args, **kwargs)

            model.generate = razor_generate

        if orig_prepare is not None:
            @functools.wraps(orig_prepare)
            def razor_prepare_inputs_for_generation(input_ids, past_key_values=None, **kwargs):
                if past_key_values is None:
                    past_key_values = new_cache()
                return orig_prepare(input_ids, past_key_values=past_key_values, **kwargs)

            model.prepare_inputs_for_generation = razor_prepare_inputs_for_generation

        if orig_forward is not None:
            # functools.wraps keeps the original signatures visible to inspect.signature, which
            # generate uses to validate its keyword arguments (attention_mask, ...)
            @functools.wraps(orig_forward)
            def razor_forward(*args, **kwargs):
                pkv = kwargs.get("past_key_values", None)
                if isinstance(pkv, PagedRazorKVCache):
                    pkv.return_handles = model._razorkv_paged_attention
                    token = cls._active_cache.set(pkv)
                    try:
                        return orig_forward(*args, **kwargs)
                    finally:
                        cls._active_cache.reset(token)
                return orig_forward(*args, **kwargs)

            model.forward = razor_forward

        layers = _decoder_layers(model)
        if layers is not None and hasattr(model, "config"):
            num_q_heads = getattr(model.config, "num_attention_heads", 32)
            head_dim = getattr(model.config, "head_dim", None) or (
                getattr(model.config, "hidden_size", 4096) // max(1, num_q_heads))
            for layer_idx, layer in enumerate(layers):
                attn = getattr(layer, "self_attn", getattr(layer, "attn", None))
                if attn is None or not hasattr(attn, "q_proj"):
                    continue

                def make_q_hook(l_idx, n_heads, h_dim):
                    def q_hook(module, inp, out):
                        cache = cls._active_cache.get()
                        if isinstance(cache, PagedRazorKVCache):
                            b, q_len = out.shape[0], out.shape[1]
                            q = out.view(b, q_len, n_heads, h_dim).transpose(1, 2)
                            cache.update_salience_with_query(q, l_idx)
                    return q_hook

                handle = attn.q_proj.register_forward_hook(make_q_hook(layer_idx, num_q_heads,
                                                                       head_dim))
                model._razorkv_hook_handles.append(handle)

        model._razorkv_paged_attention = bool(paged_attention)
        cfg = getattr(model, "config", None)
        if paged_attention and hasattr(cfg, "_attn_implementation"):   # a transformers config
            if not hasattr(model, "_razorkv_orig_attn_implementation"):
                model._razorkv_orig_attn_implementation = cfg._attn_implementation
            cfg._attn_implementation = register_attention()
        model._razorkv_config = razor_cfg
        return model

    @classmethod
    def unpatch_model(cls, model: Any) -> Any:
        """razorkv/engine.py:135-156, plus the attention implementation put back."""
        if getattr(model, "_orig_generate", None) is not None:
            model.generate = model._orig_generate
        if hasattr(model, "_orig_generate"):
            del model._orig_generate
        if getattr(model, "_orig_prepare_inputs_for_generation", None) is not None:
            model.prepare_inputs_for_generation = model._orig_prepare_inputs_for_generation
        if hasattr(model, "_orig_prepare_inputs_for_generation"):
            del model._orig_prepare_inputs_for_generation
        if getattr(model, "_orig_forward", None) is not None:
            model.forward = model._orig_forward
        if hasattr(model, "_orig_forward"):
            del model._orig_forward
        if hasattr(model, "_razorkv_hook_handles"):
            for h in model._razorkv_hook_handles:
                h.remove()
            model._razorkv_hook_handles.clear()
            del model._razorkv_hook_handles
        if hasattr(model, "_razorkv_orig_attn_implementation"):
            model.config._attn_implementation = model._razorkv_orig_attn_implementation
            del model._razorkv_orig_attn_implementation
        for name in ("_is_razorkv_patched", "_razorkv_config", "_razorkv_paged_attention"):
            if hasattr(model, name):
                delattr(model, name)
        return model

    @staticmethod
    def estimate_vram_savings(context_len: int, num_layers: int = 32, num_kv_heads: int = 8,
                              head_dim: int = 128, dtype_bytes: int = 2,
                              compression_ratio: float = 0.30) -> Dict[str, float]:
        """razorkv/engine.py:158-178: dense vs retained K/V megabytes (same formula)."""
        bytes_per_token = 2 * num_layers * num_kv_heads * head_dim * dtype_bytes
        dense_bytes = bytes_per_token * context_len
        razor_bytes = dense_bytes * compression_ratio
        saved_bytes = dense_bytes - razor_bytes
        return {
            "dense_mb": dense_bytes / (1024 * 1024),
            "razorkv_mb": razor_bytes / (1024 * 1024),
            "saved_mb": saved_bytes / (1024 * 1024),
            "savings_percentage": (1.0 - compression_ratio) * 100.0,
        }
