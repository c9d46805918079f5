"""Seeded synthetic decode workloads (the shapes the decode path is measured on).

The reference publishes no dataset for this path; its own benchmark draws K/V from
N(0, 1) (razorkv/evaluation/benchmark_runner.py:225-248).  Workloads here follow the same
distribution and add *planted* pages whose keys point along the query direction so that
the salience ranking is not trivially norm-driven:

    planted key = 0.5 * N(0, 1) + 3 * q_hat,
    q_hat       = unit(mean over the G query heads of the step-0 query of that (b, kv-head))

Planted pages are whole 16-token groups of the prefill inside the haystack zone
``[sink, T - window)``, chosen independently per (layer, sequence, kv-head).

Every draw comes from a generator seeded by (seed, layer) for the prefill and by
(seed, step, layer) for a decode step, so any single layer or step can be regenerated on
its own.  A CPU generator and a CUDA generator give different numbers for the same seed:
parity runs draw on the CPU and copy the tensors to the GPU; throughput runs draw on the
GPU.  Values are drawn in fp32 and cast to the workload dtype after planting.
"""

from dataclasses import dataclass, replace
from typing import Dict, Tuple

import torch

from .config import RazorConfig


@dataclass(frozen=True)
class DecodeWorkload:
    name: str
    num_layers: int
    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    batch: int
    context: int
    decode_steps: int
    dtype: torch.dtype
    sink_tokens: int = 32
    local_window: int = 512
    page_size: int = 16
    pyramid_mode: str = "linear"
    compression_ratio: float = 0.30
    pyramid_min_ratio: float = 0.15
    pyramid_max_ratio: float = 0.70
    planted_pages: int = 0          # fixed count per (layer, b, kv-head); 0 -> use planted_frac
    planted_frac: float = 0.01      # fraction of haystack pages per (layer, b, kv-head)
    seed: int = 1234

    @property
    def group(self) -> int:
        return self.num_q_heads // self.num_kv_heads

    def razor_config(self) -> RazorConfig:
        return RazorConfig(
            compression_ratio=self.compression_ratio,
            sink_tokens=self.sink_tokens,
            local_window=self.local_window,
            page_size=self.page_size,
            pyramid_mode=self.pyramid_mode,
            pyramid_min_ratio=self.pyramid_min_ratio,
            pyramid_max_ratio=self.pyramid_max_ratio,
        )

    def num_planted(self) -> int:
        hay_pages = max(0, (self.context - self.local_window - self.sink_tokens) // self.page_size)
        if self.planted_pages:
            return min(self.planted_pages, hay_pages)
        return min(hay_pages, max(1, round(self.planted_frac * hay_pages))) if hay_pages else 0

    def scaled(self, **kw) -> "DecodeWorkload":
        return replace(self, **kw)


# The measured shapes.  Names say what the workload is.
WORKLOADS: Dict[str, DecodeWorkload] = {
    # single layer, fp32, GQA 4, head_dim 64, 4096-token context, uniform 30 % retention
    "single-layer-fp32-4k": DecodeWorkload(
        "single-layer-fp32-4k", num_layers=1, num_q_heads=8, num_kv_heads=2, head_dim=64,
        batch=1, context=4096, decode_steps=64, dtype=torch.float32, pyramid_mode="uniform",
        compression_ratio=0.30, planted_pages=8),
    # Llama-3.1-8B-shaped cache: 32 layers, 32/8 heads, d128, batch 8, 32k, pyramid 15 -> 70 %
    "llama8b-b8-32k-bf16": DecodeWorkload(
        "llama8b-b8-32k-bf16", num_layers=32, num_q_heads=32, num_kv_heads=8, head_dim=128,
        batch=8, context=32768, decode_steps=256, dtype=torch.bfloat16),
    # Qwen-2.5-7B-shaped long context: 28 layers, 28/4 heads, d128, batch 1, 128k
    "qwen7b-b1-128k-bf16": DecodeWorkload(
        "qwen7b-b1-128k-bf16", num_layers=28, num_q_heads=28, num_kv_heads=4, head_dim=128,
        batch=1, context=131072, decode_steps=128, dtype=torch.bfloat16),
    # Llama-3-70B-shaped batched decode: 80 layers, 64/8 heads, d128, batch 64, 32k
    "llama70b-b64-32k-bf16": DecodeWorkload(
        "llama70b-b64-32k-bf16", num_layers=80, num_q_heads=64, num_kv_heads=8, head_dim=128,
        batch=64, context=32768, decode_steps=64, dtype=torch.bfloat16),
}


def _generator(device, *keys: int) -> torch.Generator:
    seed = 0x9E3779B1
    for k in keys:
        seed = (seed * 1000003 + int(k) + 1) % (1 << 62)
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def layer_prefill(w: DecodeWorkload, layer: int, device="cpu", batch_slice=None
                  ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Prefill K, V ``[B, Hkv, T, D]`` and the step-0 query ``[B, Hq, 1, D]`` of one layer."""
    g = _generator(device, w.seed, 1, layer)
    B, Hq, Hkv, T, D = w.batch, w.num_q_heads, w.num_kv_heads, w.context, w.head_dim
    K = torch.randn(B, Hkv, T, D, generator=g, device=device, dtype=torch.float32)
    V = torch.randn(B, Hkv, T, D, generator=g, device=device, dtype=torch.float32)
    q0 = torch.randn(B, Hq, 1, D, generator=g, device=device, dtype=torch.float32)
    n_plant = w.num_planted()
    if n_plant:
        P = w.page_size
        hay_pages = (T - w.local_window - w.sink_tokens) // P
        qhat = q0[:, :, 0, :].reshape(B, Hkv, w.group, D).mean(dim=2)
        qhat = qhat / qhat.norm(dim=-1, keepdim=True)
        noise = torch.randn(B, Hkv, n_plant, P, D, generator=g, device=device, dtype=torch.float32)
        for b in range(B):
            for h in range(Hkv):
                pages = torch.randperm(hay_pages, generator=g, device=device)[:n_plant]
                tok = (w.sink_tokens + pages[:, None] * P
                       + torch.arange(P, device=device)[None, :]).reshape(-1)
                K[b, h, tok, :] = (0.5 * noise[b, h] + 3.0 * qhat[b, h]).reshape(-1, D)
    if batch_slice is not None:
        K, V, q0 = K[batch_slice], V[batch_slice], q0[batch_slice]
    return K.to(w.dtype).contiguous(), V.to(w.dtype).contiguous(), q0.to(w.dtype).contiguous()


def decode_inputs(w: DecodeWorkload, step: int, layer: int, device="cpu", batch_slice=None
                  ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Fresh query ``[B, Hq, 1, D]`` and new key/value ``[B, Hkv, 1, D]`` of one step."""
    g = _generator(device, w.seed, 2, step, layer)
    B, D = w.batch, w.head_dim
    q = torch.randn(B, w.num_q_heads, 1, D, generator=g, device=device, dtype=torch.float32)
    k = torch.randn(B, w.num_kv_heads, 1, D, generator=g, device=device, dtype=torch.float32)
    v = torch.randn(B, w.num_kv_heads, 1, D, generator=g, device=device, dtype=torch.float32)
    if batch_slice is not None:
        q, k, v = q[batch_slice], k[batch_slice], v[batch_slice]
    return q.to(w.dtype), k.to(w.dtype), v.to(w.dtype)
