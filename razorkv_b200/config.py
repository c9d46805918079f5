"""Cache configuration and the per-layer retention budget.

Mirrors the reference's ``RazorConfig`` (razorkv/config.py:13-112) field for field, so a
config built for the reference cache drives this one unchanged.  The budget arithmetic is
host-side integer/float64 math and must match the reference exactly, because it decides
*when* a layer is compacted and *how many* pages survive:

* ``get_layer_ratio``  follows razorkv/config.py:65-95 (uniform / custom / linear /
  adaptive pyramid with exponent 1.8, rescaled to the mean ``compression_ratio`` and
  clamped to [0.05, 1.0]);
* ``get_layer_budget`` follows razorkv/config.py:98-112:
  ``min(T, max(sink + window, int(T * ratio)))`` with ``T`` returned as-is when
  ``T <= sink + window``.

``use_triton``, ``device`` and ``dtype`` are accepted for signature compatibility; as in the
reference they do not influence the cache (razorkv/config.py:49-51).
"""

from dataclasses import dataclass
from typing import List, Optional, Union

import torch


@dataclass
class RazorConfig:
    compression_ratio: float = 0.30
    sink_tokens: int = 32
    local_window: int = 512
    page_size: int = 16
    pyramid_mode: str = "adaptive"
    pyramid_min_ratio: float = 0.15
    pyramid_max_ratio: float = 0.70
    salience_decay: float = 0.98
    salience_init: str = "norm"
    custom_layer_ratios: Optional[List[float]] = None
    use_triton: bool = False
    device: Optional[Union[str, torch.device]] = None
    dtype: torch.dtype = torch.float16

    def __post_init__(self):
        # Same admissible ranges and messages as razorkv/config.py:53-63.
        if not (0.0 < self.compression_ratio <= 1.0):
            raise ValueError(f"compression_ratio must be in (0, 1], got {self.compression_ratio}")
        if self.sink_tokens < 0:
            raise ValueError(f"sink_tokens must be >= 0, got {self.sink_tokens}")
        if self.local_window < 0:
            raise ValueError(f"local_window must be >= 0, got {self.local_window}")
        if self.page_size < 1:
            raise ValueError(f"page_size must be >= 1, got {self.page_size}")
        if not (0.0 < self.salience_decay <= 1.0):
            raise ValueError(f"salience_decay must be in (0, 1], got {self.salience_decay}")

    # -- budgets -----------------------------------------------------------------------------
    def get_layer_ratio(self, layer_idx: int, num_layers: int) -> float:
        """Retention ratio of one layer (razorkv/config.py:65-95)."""
        mode = self.pyramid_mode
        if num_layers <= 1 or mode == "uniform":
            return self.compression_ratio
        if mode == "custom" and self.custom_layer_ratios is not None:
            if layer_idx < len(self.custom_layer_ratios):
                return self.custom_layer_ratios[layer_idx]
            return self.compression_ratio
        lo, hi = self.pyramid_min_ratio, self.pyramid_max_ratio
        depth = layer_idx / (num_layers - 1)
        if mode == "linear":
            return lo + depth * (hi - lo)
        if mode == "adaptive":
            # The curve is renormalised so its mean over the layers equals compression_ratio.
            shaped = [lo + (i / (num_layers - 1)) ** 1.8 * (hi - lo) for i in range(num_layers)]
            mean_shaped = sum(shaped) / len(shaped)
            gain = self.compression_ratio / max(mean_shaped, 1e-6)
            value = (lo + depth ** 1.8 * (hi - lo)) * gain
            return max(0.05, min(1.0, value))
        return self.compression_ratio

    def get_layer_budget(self, layer_idx: int, num_layers: int, total_seq_len: int) -> int:
        """Token budget of one layer (razorkv/config.py:98-112)."""
        floor_tokens = self.sink_tokens + self.local_window
        if total_seq_len <= floor_tokens:
            return total_seq_len
        wanted = int(total_seq_len * self.get_layer_ratio(layer_idx, num_layers))
        return min(total_seq_len, max(floor_tokens, wanted))
