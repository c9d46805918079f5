"""razorkv_b200: RazorKV's decode-time sparse attention path on B200 (sm_100a).

Public surface (names as in the reference package ``razorkv``):

* ``RazorConfig``                              razorkv/config.py
* ``PagedRazorKVCache`` (alias ``RazorKVCache``) razorkv/cache.py
* ``RazorEngine`` (HF model patcher; paged attention interface) razorkv/engine.py
* ``kernels``: ``triton_paged_sparse_attention``, ``compacted_paged_sdpa``,
  ``compute_page_salience_pool``, ``is_triton_available``   razorkv/kernels/

The CUDA library (librazorkv_b200.so, C ABI in include/razorkv_b200.h) is loaded on first
use; build it with ``python -m razorkv_b200.build``.
"""

from .config import RazorConfig
from .cache import PagedKV, PagedRazorKVCache, RazorKVCache, RazorLayerState
from .engine import RazorEngine
from . import kernels
from .kernels import (
    compacted_paged_sdpa,
    compute_page_salience_pool,
    is_triton_available,
    paged_sparse_attention,
    triton_paged_sparse_attention,
)

__version__ = "0.1.0"

__all__ = [
    "RazorConfig",
    "PagedRazorKVCache",
    "RazorKVCache",
    "RazorLayerState",
    "PagedKV",
    "RazorEngine",
    "kernels",
    "compacted_paged_sdpa",
    "compute_page_salience_pool",
    "is_triton_available",
    "paged_sparse_attention",
    "triton_paged_sparse_attention",
    "__version__",
]
