"""PagedRazorKVCache: the reference cache's decode path on a paged HBM pool.

Drop-in for ``razorkv.cache.RazorKVCache`` (razorkv/cache.py:72-436): same constructor,
same ``update`` / ``update_salience_with_query`` / ``_evict_layer`` semantics and the same
HF cache surface, but K/V never live as per-layer contiguous tensors:

* Storage.  One pool for all layers: K and V ``[slots, B, Hkv, P, D]`` and the token
  salience ``[slots, B, P]`` fp32, where a *slot* is one physical page of P tokens
  (P = ``config.page_size``) holding every (sequence, kv-head) plane.  A device free stack
  lists unused slots; its top is tracked on the host (every push and pop count is
  host-known, so no call ever waits on the device).
* Per layer: a device page table (logical page -> slot, shared by all sequences, because
  the reference selects the same pages for every sequence and head -- razorkv/cache.py:335-341)
  and the host-side token count.
* Append (razorkv/cache.py:369-390) writes the new rows into the last page, taking a slot
  from the free stack when a page starts; O(new tokens) instead of the reference's
  O(layer) ``torch.cat``.
* Scoring (razorkv/cache.py:249-287) is a fixed-order fp32 kernel whose results the CPU
  oracle reproduces bit for bit.
* Compaction (razorkv/cache.py:289-359).  When the sink is a whole number of pages every
  surviving 16-token group of the reference's new order is an existing page, so compaction
  is a page-table rewrite plus a free-stack push with no data movement; otherwise (unaligned
  sink, or the ``haystack_budget <= 0`` branch) tokens are copied into fresh pages.
* ``decode_step(q, k, v, layer)`` runs a whole decode step of one layer -- append, score,
  compact when the hysteresis threshold is crossed, attend -- with score and attention
  fused into one pass over K on steps that do not compact.

``key_cache`` / ``value_cache`` / ``salience_scores`` and the tensors ``update`` returns
are materialised from the pool on demand (a gather), so code written against the reference
cache keeps working; the paged fast path never materialises them.
"""

import math
from typing import Any, Callable, Dict, List, Optional, Tuple, Union

import torch

from . import _lib
from ._lib import (Exchange, KVLayout, Output, Query, Salience, check, dtype_code, require_cuda,
                   stream_ptr)
from .config import RazorConfig
from .kernels import Workspace

try:  # same base-class choice as the reference (razorkv/cache.py:19-29)
    from transformers.cache_utils import DynamicCache, Cache  # noqa: F401
    BaseCacheClass = DynamicCache
except ImportError:  # pragma: no cover - transformers is present in this environment
    try:
        from transformers.cache_utils import Cache
        BaseCacheClass = Cache
    except ImportError:
        class BaseCacheClass:
            pass


class RazorLayerState:
    """HF 5.x per-layer view (razorkv/cache.py:34-69); keys/values materialise on access."""

    is_compileable: bool = False
    is_sliding: bool = False
    is_croppable: bool = True

    def __init__(self, cache: "PagedRazorKVCache", layer_idx: int):
        self._cache = cache
        self._layer = layer_idx
        self.cumulative_length = 0

    @property
    def keys(self):
        return self._cache._materialize(self._layer, 0)

    @property
    def values(self):
        return self._cache._materialize(self._layer, 1)

    def get_seq_length(self) -> int:
        return self.cumulative_length

    def get_mask_sizes(self, query_length, *args) -> Tuple[int, int]:
        if isinstance(query_length, torch.Tensor):
            q_len = query_length.shape[0] if query_length.ndim > 0 else int(query_length.item())
        else:
            q_len = int(query_length)
        return self._cache.get_cached_seq_length(self._layer) + q_len, 0

    def crop(self, tokens_to_remove: int = 0) -> None:
        self._cache._crop_layer(self._layer, tokens_to_remove)
        self.cumulative_length = max(0, self.cumulative_length - tokens_to_remove)


class SelectionRecord:
    """One compaction decision of a layer (``PagedRazorKVCache.record_decisions``).

    ``kept`` (ascending haystack page indices, int64) and ``margin`` (one fp32: the k-th minus
    the (k+1)-th largest batch-mean page score, +inf when every page is kept) stay on the
    device until read."""

    __slots__ = ("layer", "seq_len", "budget", "kind", "num_pages", "k", "kept", "margin")

    def __init__(self, layer, seq_len, budget, kind, num_pages=0, k=0, kept=None, margin=None):
        self.layer, self.seq_len, self.budget, self.kind = layer, seq_len, budget, kind
        self.num_pages, self.k, self.kept, self.margin = num_pages, k, kept, margin


class PagedKV:
    """The K (which=0) or V (1) of one layer as ``update`` returns it on decode steps when
    ``return_handles`` is set: nothing is gathered; ``materialize()`` gives the contiguous
    ``[B, Hkv, N, D]`` tensor the reference would have returned."""

    __slots__ = ("cache", "layer", "which")

    def __init__(self, cache: "PagedRazorKVCache", layer: int, which: int):
        self.cache, self.layer, self.which = cache, layer, which

    @property
    def shape(self) -> torch.Size:
        c = self.cache
        return torch.Size((c._B, c._Hkv, c._n[self.layer], c._D))

    @property
    def dtype(self) -> torch.dtype:
        return self.cache._dtype

    @property
    def device(self) -> torch.device:
        return self.cache._device

    def materialize(self) -> torch.Tensor:
        return self.cache._materialize(self.layer, self.which)


class _LayerList(list):
    """List-like view whose items materialise one layer's K, V or salience."""

    def __init__(self, cache, which):
        super().__init__()
        self._cache, self._which = cache, which

    def __len__(self):
        return len(self._cache._n)

    def __iter__(self):
        for i in range(len(self)):
            yield self[i]

    def __getitem__(self, i):
        if isinstance(i, slice):
            return [self[j] for j in range(*i.indices(len(self)))]
        if i < 0:
            i += len(self)
        if i >= len(self) or self._cache._n[i] is None:
            return None
        return self._cache._materialize(i, self._which)

    def __bool__(self):
        return len(self) > 0


class PagedRazorKVCache(BaseCacheClass):
    # reorder_cache with the batch size unchanged (beam search) shares pages between sequences
    # through the row map; set False to move every live page's K/V rows instead, which keeps
    # the pool in sequence order for code that reads it without the row map
    share_pages_on_reorder: bool = True

    def __init__(self, config: Optional[RazorConfig] = None, num_layers: int = 32,
                 max_slots: Optional[int] = None):
        try:
            super().__init__()
        except Exception:
            pass
        self.config = config or RazorConfig()
        self.num_layers = num_layers
        self._seen_tokens = 0
        self._initial_slots = max_slots
        # pool (allocated on the first update, when B / Hkv / D / dtype / device are known)
        self._k = self._v = self._s = None
        self._free = None
        self._free_top = 0
        self._slots = 0
        # row map [slots, B] int32 (None = sequence b in row b): created by the first in-place
        # reorder_cache, which then shares pages between beams instead of copying them
        self._rowmap: Optional[torch.Tensor] = None
        self._B = self._Hkv = self._D = 0
        self._dtype = None
        self._device = None
        # per layer
        self._n: List[Optional[int]] = []
        self._pt: List[Optional[torch.Tensor]] = []
        self._layers: List[RazorLayerState] = []
        # selection hooks / diagnostics
        self.score_reducer: Optional[Callable[[torch.Tensor], torch.Tensor]] = None
        # KV-head sharding (razorkv_b200.distributed.HeadGroup): this cache holds only some kv
        # heads; every salience update goes through an exchange block combined over the group
        self.head_group = None
        self._xbuf: Optional[torch.Tensor] = None
        self._xpend = None   # (layer, block, Exchange, score_tokens, new_first, n_new)
        # with record_decisions set, every compaction appends a SelectionRecord (device
        # tensors, read when the caller syncs); kept_override(layer, index, kept, margin) may
        # return a replacement kept-page tensor (to follow an external decision trace)
        self.compactions = 0   # compactions run so far (all layers; prefill ones included)
        self.record_decisions = False
        self.decisions: List["SelectionRecord"] = []
        self.kept_override: Optional[Callable[[int, int, torch.Tensor], Optional[torch.Tensor]]] = None
        # decode steps of ``update`` return PagedKV handles instead of gathered K/V; the
        # engine's attention function then reads the pool directly
        self.return_handles = False
        # HF hook path with return_handles: the q_proj hook's pre-RoPE query of a decode step
        # is kept here (layer -> (q, tokens scored)) and scored by the attention pass
        self._pending: Dict[int, Tuple[torch.Tensor, int]] = {}
        # optional observer with before(layer, kv_bytes) / after() around every attention
        # launch of decode_step (used to time the decode kernel inside a running step)
        self.launch_observer = None
        # argument blocks reused by the decode fast path
        self._lib = None
        self._ratio_cache = {}
        self._lay_cache = {}
        self._ws = {}
        self._q_struct = Query()
        self._o_struct = Output()
        self._sal_struct = None
        self._elt = 0
        self._dtype_code = 0
        self._sal_init = 0

    # ---------------------------------------------------------------- HF / reference surface
    @property
    def seen_tokens(self) -> int:
        return self._seen_tokens

    @property
    def is_compileable(self) -> bool:
        return False

    @property
    def is_sliding(self) -> List[bool]:
        return [False] * len(self._n)

    @property
    def is_croppable(self) -> bool:
        return True

    @property
    def is_initialized(self) -> bool:
        return len(self._n) > 0 and self._n[0] is not None

    @property
    def batch_size(self) -> int:
        return self._B if self.is_initialized else 0

    @property
    def layers(self) -> List[RazorLayerState]:
        return self._layers

    @layers.setter
    def layers(self, value):   # the HF base class assigns an empty list in __init__
        pass

    @property
    def key_cache(self):
        return _LayerList(self, 0)

    @property
    def value_cache(self):
        return _LayerList(self, 1)

    @property
    def salience_scores(self):
        return _LayerList(self, 2)

    def __len__(self) -> int:
        return self._seen_tokens

    def __getitem__(self, layer_idx: int):
        if layer_idx < len(self._n) and self._n[layer_idx] is not None:
            return self._materialize(layer_idx, 0), self._materialize(layer_idx, 1)
        raise IndexError(f"Layer index {layer_idx} out of range ({len(self._n)} layers allocated).")

    def __iter__(self):
        for l in range(len(self._n)):
            if self._n[l] is not None:
                yield self._materialize(l, 0), self._materialize(l, 1)

    def get_seq_length(self, layer_idx: Optional[int] = 0) -> int:
        return self._seen_tokens

    def get_cached_seq_length(self, layer_idx: Optional[int] = 0) -> int:
        if layer_idx is None:
            layer_idx = 0
        if layer_idx >= len(self._n) or self._n[layer_idx] is None:
            return 0
        return self._n[layer_idx]

    def get_max_length(self) -> Optional[int]:
        return None

    def get_max_cache_shape(self, *args) -> Optional[int]:
        return None

    def get_usable_length(self, new_seq_len: int, layer_idx: Optional[int] = 0) -> int:
        return self._seen_tokens

    def get_mask_sizes(self, query_length, layer_idx: int = 0) -> Tuple[int, int]:
        if isinstance(query_length, torch.Tensor):
            q_len = query_length.shape[0] if query_length.ndim > 0 else int(query_length.item())
        else:
            q_len = int(query_length)
        return self.get_cached_seq_length(layer_idx) + q_len, 0

    def get_query_offset(self, layer_idx: int = 0) -> int:
        return self._seen_tokens

    # ------------------------------------------------------------------------ pool plumbing
    def _init_pool(self, k: torch.Tensor):
        require_cuda(k)
        self._B, self._Hkv, _, self._D = k.shape
        self._dtype = k.dtype
        self._device = k.device
        self._dtype_code = dtype_code(k.dtype)
        self._elt = k.element_size()
        self._sal_init = _lib.SAL_NORM if self.config.salience_init == "norm" else _lib.SAL_UNIFORM
        self._lib = _lib.load()
        self._grow(self._initial_slots or 64)

    def _slot_shape(self, n):
        return (n, self._B, self._Hkv, self.config.page_size, self._D)

    def _grow(self, min_slots: int):
        """Enlarge the pool to at least min_slots slots; existing slot ids stay valid."""
        new = max(min_slots, 2 * self._slots, 16)
        P = self.config.page_size
        dev = self._device
        k = torch.zeros(self._slot_shape(new), dtype=self._dtype, device=dev)
        v = torch.zeros(self._slot_shape(new), dtype=self._dtype, device=dev)
        s = torch.zeros((new, self._B, P), dtype=torch.float32, device=dev)
        free = torch.empty(new, dtype=torch.int64, device=dev)
        old = self._slots
        if old:
            k[:old].copy_(self._k)
            v[:old].copy_(self._v)
            s[:old].copy_(self._s)
            free[: self._free_top].copy_(self._free[: self._free_top])
        # new slots go under the existing free entries, highest id first, so pops continue in
        # ascending slot order
        added = torch.arange(new - 1, old - 1, -1, dtype=torch.int64, device=dev)
        if self._free_top:
            free[new - old: new - old + self._free_top].copy_(free[: self._free_top].clone())
        free[: new - old].copy_(added)
        self._k, self._v, self._s, self._free = k, v, s, free
        if self._rowmap is not None:
            rm = torch.arange(self._B, dtype=torch.int32, device=dev).repeat(new, 1)
            rm[:old].copy_(self._rowmap)
            self._rowmap = rm
        self._free_top += new - old
        self._slots = new
        self._pool_changed()

    def _pool_changed(self):
        """Pool tensors were replaced: drop argument blocks that point into them."""
        self._lay_cache.clear()
        self._sal_struct = self._salience()

    def _ensure_free(self, n_pages: int):
        if self._free_top < n_pages:
            self._grow(self._slots + (n_pages - self._free_top))

    def _ensure_layer(self, layer_idx: int):
        while len(self._n) <= layer_idx:
            self._n.append(None)
            self._pt.append(None)
            self._layers.append(RazorLayerState(self, len(self._layers)))

    def _ensure_pt(self, layer_idx: int, n_pages: int):
        pt = self._pt[layer_idx]
        if pt is None or pt.numel() < n_pages:
            cap = max(n_pages, 2 * (pt.numel() if pt is not None else 0), 64)
            new = torch.zeros(cap, dtype=torch.int64, device=self._device)
            if pt is not None:
                new[: pt.numel()].copy_(pt)
            self._pt[layer_idx] = new
            self._lay_cache.pop(layer_idx, None)

    def _layout(self, layer_idx: int, n_tokens: Optional[int] = None) -> KVLayout:
        k = self._k
        n = self._n[layer_idx] if n_tokens is None else n_tokens
        return KVLayout(k.data_ptr(), self._v.data_ptr(), dtype_code(self._dtype), self._D,
                        self._B, self._Hkv, k.stride(1), k.stride(2), k.stride(0), k.stride(3),
                        self.config.page_size, self._slots, self._pt[layer_idx].data_ptr(), 0, n,
                        self._rowmap.data_ptr() if self._rowmap is not None else None)

    def _salience(self) -> Salience:
        return Salience(self._s.data_ptr(), self._s.stride(1), self._s.stride(0))

    def _stream(self):
        return stream_ptr(self._device)

    def _pages(self, n_tokens: int) -> int:
        P = self.config.page_size
        return (n_tokens + P - 1) // P

    # ------------------------------------------------------------------------------ append
    def _append(self, layer_idx: int, k: torch.Tensor, v: torch.Tensor):
        lib = _lib.load()
        if k.dtype != self._dtype or k.shape[0] != self._B or k.shape[1] != self._Hkv or k.shape[3] != self._D:
            raise ValueError(f"key_states {tuple(k.shape)}/{k.dtype} does not match the cache "
                             f"[{self._B}, {self._Hkv}, *, {self._D}]/{self._dtype}")
        k = k if k.stride(-1) == 1 else k.contiguous()
        v = v if v.stride(-1) == 1 else v.contiguous()
        if k.stride() != v.stride():
            k, v = k.contiguous(), v.contiguous()
        n0 = self._n[layer_idx] or 0
        T = k.shape[2]
        new_pages = self._pages(n0 + T) - self._pages(n0)
        self._ensure_free(new_pages)
        self._ensure_pt(layer_idx, self._pages(n0 + T))
        lay = self._layout(layer_idx, n0)
        sal = self._salience()
        init = _lib.SAL_NORM if self.config.salience_init == "norm" else _lib.SAL_UNIFORM
        if self.head_group is not None:
            if self._xpend is None:   # an append outside update(): no scoring follows
                self._xbegin(layer_idx, score_tokens=0, new_first=n0, n_new=T)
            st = lib.rkv_append_partial(lay, k.data_ptr(), v.data_ptr(), k.stride(0), k.stride(1),
                                        k.stride(2), T, n0, self._pt[layer_idx].data_ptr(),
                                        self._free.data_ptr(), self._free_top, init,
                                        self._xpend[2], self._stream())
            check(st, "rkv_append_partial")
        else:
            st = lib.rkv_append(lay, sal, k.data_ptr(), v.data_ptr(), k.stride(0), k.stride(1),
                                k.stride(2), T, n0, self._pt[layer_idx].data_ptr(),
                                self._free.data_ptr(), self._free_top, init, self._stream())
            check(st, "rkv_append")
        self._free_top -= new_pages
        self._n[layer_idx] = n0 + T

    # ----------------------------------------------------------------------------- scoring
    def update_salience_with_query(self, query_states: torch.Tensor, layer_idx: int):
        """razorkv/cache.py:249-287 on the pool (scores every retained token).

        With ``return_handles`` set (the engine's paged attention), a single-row query is not
        scored here: it is kept and scored, over the same tokens, by the layer's attention
        pass of this step (``rkv_decode_scored``), which reads K once for both."""
        if layer_idx >= len(self._n) or self._n[layer_idx] is None:
            return
        require_cuda(query_states)
        q = query_states.to(self._device)
        if q.stride(-1) != 1:
            q = q.contiguous()
        if q.shape[1] % self._Hkv:
            raise ValueError("query heads must be a multiple of the cache's kv heads")
        self._flush_pending(layer_idx)
        if self.return_handles and q.shape[2] == 1 and q.dtype == self._dtype:
            self._pending[layer_idx] = (q, self._n[layer_idx])
            return
        self._score(q, layer_idx, self._n[layer_idx])

    # ----------------------------------------------------------------- KV-head sharding
    def _xbegin(self, layer_idx: int, score_tokens: int, new_first: int, n_new: int):
        """Open the exchange block of one salience update of a head-sharded layer: the keys
        of score_tokens tokens, then the kv-head norms of the n_new tokens from new_first."""
        H = self.head_group.num_kv_heads_total
        stride = score_tokens + n_new * H
        need = max(1, self._B * stride)
        if self._xbuf is None or self._xbuf.numel() < need:
            old = 0 if self._xbuf is None else self._xbuf.numel()
            self._xbuf = torch.empty(max(need, 2 * old), dtype=torch.int32, device=self._device)
        x = self._xbuf[: self._B * stride].view(self._B, stride)
        xc = Exchange(x.data_ptr(), stride, score_tokens, self.head_group.head0, H)
        self._xpend = (layer_idx, x, xc, score_tokens, new_first, n_new)

    def _settle(self):
        """Combine the open exchange block over the head group (all-reduce MAX) and update
        the salience from it."""
        if self._xpend is None:
            return
        layer_idx, x, xc, score_tokens, new_first, n_new = self._xpend
        self._xpend = None
        if x.numel():
            self.head_group.reduce(x)
        init = _lib.SAL_NORM if self.config.salience_init == "norm" else _lib.SAL_UNIFORM
        decay = self.config.salience_decay
        st = _lib.load().rkv_salience_apply(self._layout(layer_idx), self._salience(), xc,
                                            score_tokens, new_first, n_new, init, float(decay),
                                            float(1.0 - decay), self._stream())
        check(st, "rkv_salience_apply")

    def _score(self, q: torch.Tensor, layer_idx: int, n_tokens: int):
        lib = _lib.load()
        if self.head_group is not None:
            standalone = self._xpend is None
            if standalone:
                self._xbegin(layer_idx, score_tokens=n_tokens, new_first=n_tokens, n_new=0)
            elif self._xpend[3] != n_tokens:
                raise RuntimeError("head-sharded scoring: exchange opened for a different length")
            st = lib.rkv_score_partial(Query(q.data_ptr(), dtype_code(q.dtype), q.shape[1],
                                             q.shape[2], q.stride(0), q.stride(1), q.stride(2)),
                                       self._layout(layer_idx, n_tokens), self._xpend[2],
                                       self._stream())
            check(st, "rkv_score_partial")
            if standalone:
                self._settle()
            return
        decay = self.config.salience_decay
        st = lib.rkv_score(Query(q.data_ptr(), dtype_code(q.dtype), q.shape[1], q.shape[2],
                                 q.stride(0), q.stride(1), q.stride(2)),
                           self._layout(layer_idx, n_tokens), self._salience(), float(decay),
                           float(1.0 - decay), 1, self._stream())
        check(st, "rkv_score")

    def _flush_pending(self, layer_idx: Optional[int] = None):
        """Score a kept hook query now (before anything else reads or reshapes the layer)."""
        layers = list(self._pending) if layer_idx is None else [layer_idx]
        for l in layers:
            item = self._pending.pop(l, None)
            if item is not None:
                self._score(item[0], l, item[1])

    # -------------------------------------------------------------------------- compaction
    def _evict_layer(self, layer_idx: int, target_budget: int):
        """razorkv/cache.py:289-359 on the pool."""
        self._flush_pending(layer_idx)
        N = self._n[layer_idx]
        if N <= target_budget:
            return
        c = self.config
        P = c.page_size
        sink = min(c.sink_tokens, N)
        local = min(c.local_window, N - sink)
        hs, he = sink, N - local
        if he - hs <= 0:
            return
        hb = target_budget - sink - local
        if hb <= 0:
            self.compactions += 1
            if self.record_decisions:
                self.decisions.append(SelectionRecord(layer_idx, N, target_budget, "zones"))
            self._compact_copy(layer_idx, new_len=sink + local, sink=sink, kept=None, k=0,
                               hay_start=hs, tail_src_start=he)
            return
        num_pages = (he - hs) // P
        if num_pages <= 0:
            return
        k = max(1, min(num_pages, hb // P))
        self.compactions += 1
        kept, margin = self._select(layer_idx, hs, num_pages, k)
        if self.kept_override is not None:
            repl = self.kept_override(layer_idx, len(self.decisions), kept, margin)
            if repl is not None:
                kept = repl.to(device=self._device, dtype=torch.int64).contiguous()
        if self.record_decisions:
            self.decisions.append(SelectionRecord(layer_idx, N, target_budget, "pages", num_pages,
                                                  k, kept.clone(), margin))
        aligned_end = hs + num_pages * P
        new_len = sink + k * P + (N - aligned_end)
        if hs % P == 0:
            lib = _lib.load()
            sink_pages = hs // P
            st = lib.rkv_compact_pages(self._pt[layer_idx].data_ptr(), sink_pages, num_pages,
                                       kept.data_ptr(), k, sink_pages + num_pages,
                                       self._pages(N), self._free.data_ptr(), self._free_top,
                                       self._stream())
            check(st, "rkv_compact_pages")
            self._free_top += num_pages - k
            self._n[layer_idx] = new_len
        else:
            self._compact_copy(layer_idx, new_len=new_len, sink=sink, kept=kept, k=k,
                               hay_start=hs, tail_src_start=aligned_end)

    def _select(self, layer_idx: int, first_token: int, num_pages: int, k: int) -> torch.Tensor:
        lib = _lib.load()
        P = self.config.page_size
        scores = torch.empty(self._B, num_pages, dtype=torch.float32, device=self._device)
        st = lib.rkv_page_scores(self._layout(layer_idx), self._salience(), first_token,
                                 num_pages, P, scores.data_ptr(), self._stream())
        check(st, "rkv_page_scores")
        if self.score_reducer is not None:
            scores = self.score_reducer(scores).contiguous()
        kept = torch.empty(k, dtype=torch.int64, device=self._device)
        margin = torch.empty(1, dtype=torch.float32, device=self._device)
        ws_bytes = lib.rkv_select_pages_workspace_size(num_pages)
        ws = Workspace.get(self._device, ws_bytes)
        st = lib.rkv_select_pages(scores.data_ptr(), scores.shape[0], num_pages, k,
                                  kept.data_ptr(), margin.data_ptr(), ws.data_ptr(), ws.numel(),
                                  self._stream())
        check(st, "rkv_select_pages")
        return kept, margin

    def _compact_copy(self, layer_idx, new_len, sink, kept, k, hay_start, tail_src_start):
        lib = _lib.load()
        P = self.config.page_size
        N = self._n[layer_idx]
        old_pages = self._pages(N)
        new_pages = self._pages(new_len)
        self._ensure_free(new_pages)
        old_pt = self._pt[layer_idx]
        new_pt = torch.zeros(max(old_pt.numel(), 64), dtype=torch.int64, device=self._device)
        st = lib.rkv_compact_tokens(self._layout(layer_idx), self._salience(), new_pt.data_ptr(),
                                    self._free.data_ptr(), self._free_top, new_len, sink,
                                    kept.data_ptr() if kept is not None else None, k, P,
                                    hay_start, tail_src_start, self._stream())
        check(st, "rkv_compact_tokens")
        self._free_top -= new_pages
        st = lib.rkv_release_pages(old_pt.data_ptr(), old_pages, self._free.data_ptr(),
                                   self._free_top, self._stream())
        check(st, "rkv_release_pages")
        self._free_top += old_pages
        self._pt[layer_idx] = new_pt
        self._lay_cache.pop(layer_idx, None)
        self._n[layer_idx] = new_len

    # ------------------------------------------------------------------------------ update
    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int,
               cache_kwargs: Optional[Dict[str, Any]] = None):
        """razorkv/cache.py:361-414 on the pool."""
        require_cuda(key_states, value_states)
        self._ensure_layer(layer_idx)
        if self._k is None:
            self._init_pool(key_states)
        T = key_states.shape[-2]
        is_prefill = T > 1
        first = self._n[layer_idx] is None
        scored = cache_kwargs is not None and "query_states" in cache_kwargs
        if self.head_group is not None:
            if self.return_handles:
                raise NotImplementedError("KV-head sharding does not serve the HF engine path")
            n0 = self._n[layer_idx] or 0
            self._xbegin(layer_idx, score_tokens=n0 + T if scored else 0, new_first=n0, n_new=T)
        self._append(layer_idx, key_states, value_states)
        if layer_idx == 0:
            self._seen_tokens = T if first else self._seen_tokens + T
        self._sync_layer(layer_idx)
        if scored:
            self.update_salience_with_query(cache_kwargs["query_states"], layer_idx)
        self._settle()
        cur = self._n[layer_idx]
        budget = self._budget(layer_idx)
        if is_prefill:
            if first:
                ret = (key_states, value_states)
            else:
                ret = (self._materialize(layer_idx, 0), self._materialize(layer_idx, 1))
            if cur > budget:
                self._evict_layer(layer_idx, budget)
            return ret
        if cur > budget + self.config.page_size:
            self._evict_layer(layer_idx, budget)
        if self.return_handles:
            return PagedKV(self, layer_idx, 0), PagedKV(self, layer_idx, 1)
        return self._materialize(layer_idx, 0), self._materialize(layer_idx, 1)

    def _budget(self, layer_idx: int) -> int:
        num_layers = max(self.num_layers, len(self._n))
        total = max(self._seen_tokens, self._n[layer_idx])
        return self.config.get_layer_budget(layer_idx, num_layers, total)

    def _sync_layer(self, layer_idx: int):
        self._layers[layer_idx].cumulative_length = self._seen_tokens

    # ------------------------------------------------------------------------- decode step
    def decode_step(self, query_states: torch.Tensor, key_states: torch.Tensor,
                    value_states: torch.Tensor, layer_idx: int,
                    out: Optional[torch.Tensor] = None,
                    scaling: Optional[float] = None) -> torch.Tensor:
        """One decode step of one layer: ``update(k, v, l, {"query_states": q})`` followed by
        attention of q over the retained cache (the reference's step protocol,
        razorkv/cache.py:361-414 then razorkv/kernels/torch_sparse.py:15-61).

        q [B, Hq, 1, D]; k, v [B, Hkv, 1, D]; returns [B, Hq, 1, D] in q's dtype."""
        fast = self._decode_step_fast(query_states, key_states, value_states, layer_idx, out,
                                      scaling)
        if fast is not None:
            return fast
        fused = self._compact_step_fused(query_states, key_states, value_states, layer_idx, out,
                                         scaling)
        if fused is not None:
            return fused
        self._ensure_layer(layer_idx)
        if self._k is None:
            self._init_pool(key_states)
        if key_states.shape[-2] != 1:
            raise ValueError("decode_step takes exactly one new token")
        first = self._n[layer_idx] is None
        sharded = self.head_group is not None
        if sharded:
            n0 = self._n[layer_idx] or 0
            self._xbegin(layer_idx, score_tokens=n0 + 1, new_first=n0, n_new=1)
        self._append(layer_idx, key_states, value_states)
        if layer_idx == 0:
            self._seen_tokens = 1 if first else self._seen_tokens + 1
        self._sync_layer(layer_idx)
        q = query_states if query_states.stride(-1) == 1 else query_states.contiguous()
        if sharded:
            # head-sharded: the exchange-based salience update, then compaction (every rank
            # holds the same salience, so every rank keeps the same pages), then attention
            self.update_salience_with_query(q, layer_idx)
            self._settle()
        B, Hq, _, D = q.shape
        if out is None:
            out = torch.empty(B, Hq, 1, D, dtype=q.dtype, device=q.device)
        cur = self._n[layer_idx]
        budget = self._budget(layer_idx)
        lib = _lib.load()
        qs = Query(q.data_ptr(), dtype_code(q.dtype), Hq, 1, q.stride(0), q.stride(1), q.stride(2))
        os_ = Output(out.data_ptr(), dtype_code(out.dtype), 0, out.stride(0), out.stride(1),
                     out.stride(2))
        scale = float(scaling) if scaling else 0.0
        obs = self.launch_observer
        if sharded or cur > budget + self.config.page_size:
            if not sharded:
                self.update_salience_with_query(q, layer_idx)
            if cur > budget + self.config.page_size:
                self._evict_layer(layer_idx, budget)
            lay = self._layout(layer_idx)
            ws = Workspace.get(self._device, lib.rkv_decode_attention_workspace_size(qs, lay))
            if obs is not None:
                obs.before(layer_idx, self._kv_bytes(layer_idx))
            st = lib.rkv_decode_attention(qs, lay, scale, 0, os_, ws.data_ptr(), ws.numel(),
                                          self._stream())
            if obs is not None:
                obs.after()
            check(st, "rkv_decode_attention")
        else:
            lay = self._layout(layer_idx)
            decay = self.config.salience_decay
            ws = Workspace.get(self._device, lib.rkv_decode_fused_workspace_size(qs, lay))
            if obs is not None:
                obs.before(layer_idx, self._kv_bytes(layer_idx))
            st = lib.rkv_decode_fused(qs, lay, self._salience(), float(decay), float(1.0 - decay),
                                      scale, os_, ws.data_ptr(), ws.numel(), self._stream())
            if obs is not None:
                obs.after()
            check(st, "rkv_decode_fused")
        return out

    def _compact_step_fused(self, q, k, v, layer_idx, out, scaling):
        """A compacting decode step with a page-aligned sink (razorkv/cache.py:361-414 then
        the attention) in three launches: append + score + haystack page max-pool in one pass
        over K (``rkv_append_score_pool``), selection + pointer-only compaction in one launch
        (``rkv_select_compact_pages``), attention over the kept pages.  Returns None when the
        step needs the general path (head sharding, a kept-set hook, an unaligned sink, the
        no-haystack branch, or no compaction due)."""
        if (self._k is None or layer_idx >= len(self._n) or self.head_group is not None
                or self.kept_override is not None or self._pending):
            return None
        n0 = self._n[layer_idx]
        if n0 is None or n0 == 0 or k.shape[2] != 1 or k.dtype != self._dtype:
            return None
        c = self.config
        P = c.page_size
        cur = n0 + 1
        seen = self._seen_tokens + 1 if layer_idx == 0 else self._seen_tokens
        num_layers = max(self.num_layers, len(self._n))
        budget = c.get_layer_budget(layer_idx, num_layers, max(seen, cur))
        if cur <= budget + P:
            return None
        sink = min(c.sink_tokens, cur)
        local = min(c.local_window, cur - sink)
        hs, he = sink, cur - local
        hb = budget - sink - local
        num_pages = (he - hs) // P if he > hs else 0
        if hb <= 0 or num_pages <= 0 or hs % P:
            return None
        k_sel = max(1, min(num_pages, hb // P))
        lib = _lib.load()
        self._ensure_free(1)
        self._ensure_pt(layer_idx, self._pages(cur))
        q = q if q.stride(-1) == 1 else q.contiguous()
        k = k if k.stride(-1) == 1 else k.contiguous()
        v = v if v.stride(-1) == 1 else v.contiguous()
        if k.stride() != v.stride():
            k, v = k.contiguous(), v.contiguous()
        B, Hq, _, D = q.shape
        if out is None:
            out = torch.empty(B, Hq, 1, D, dtype=q.dtype, device=q.device)
        qs = Query(q.data_ptr(), dtype_code(q.dtype), Hq, 1, q.stride(0), q.stride(1), q.stride(2))
        pt = self._pt[layer_idx]
        stream = self._stream()
        scores = torch.empty(self._B, num_pages, dtype=torch.float32, device=self._device)
        decay = c.salience_decay
        init = _lib.SAL_NORM if c.salience_init == "norm" else _lib.SAL_UNIFORM
        st = lib.rkv_append_score_pool(self._layout(layer_idx, n0), self._salience(), k.data_ptr(),
                                       v.data_ptr(), k.stride(0), k.stride(1), pt.data_ptr(),
                                       self._free.data_ptr(), self._free_top, init, qs,
                                       float(decay), float(1.0 - decay), hs, num_pages,
                                       scores.data_ptr(), stream)
        check(st, "rkv_append_score_pool")
        if n0 % P == 0:
            self._free_top -= 1
        self._n[layer_idx] = cur
        self._seen_tokens = seen
        self._sync_layer(layer_idx)
        if self.score_reducer is not None:
            scores = self.score_reducer(scores).contiguous()
        kept = torch.empty(k_sel, dtype=torch.int64, device=self._device)
        margin = torch.empty(1, dtype=torch.float32, device=self._device)
        ws = Workspace.get(self._device, lib.rkv_select_pages_workspace_size(num_pages))
        sink_pages = hs // P
        st = lib.rkv_select_compact_pages(scores.data_ptr(), scores.shape[0], num_pages, k_sel,
                                          pt.data_ptr(), sink_pages, sink_pages + num_pages,
                                          self._pages(cur), self._free.data_ptr(),
                                          self._free_top, kept.data_ptr(), margin.data_ptr(),
                                          ws.data_ptr(), ws.numel(), stream)
        check(st, "rkv_select_compact_pages")
        self._free_top += num_pages - k_sel
        self._n[layer_idx] = sink + k_sel * P + (cur - (hs + num_pages * P))
        self.compactions += 1
        if self.record_decisions:
            self.decisions.append(SelectionRecord(layer_idx, cur, budget, "pages", num_pages,
                                                  k_sel, kept, margin))
        os_ = Output(out.data_ptr(), dtype_code(out.dtype), 0, out.stride(0), out.stride(1),
                     out.stride(2))
        lay = self._layout(layer_idx)
        ws = Workspace.get(self._device, lib.rkv_decode_attention_workspace_size(qs, lay))
        obs = self.launch_observer
        if obs is not None:
            obs.before(layer_idx, self._kv_bytes(layer_idx))
        st = lib.rkv_decode_attention(qs, lay, float(scaling) if scaling else 0.0, 0, os_,
                                      ws.data_ptr(), ws.numel(), stream)
        if obs is not None:
            obs.after()
        check(st, "rkv_decode_attention")
        return out

    def _decode_step_fast(self, q, k, v, layer_idx, out, scaling):
        """The common decode step -- no compaction, no pool or table growth -- in one library
        call with cached argument blocks.  Returns None when the step needs the general path."""
        if self._k is None or layer_idx >= len(self._n):
            return None
        n0 = self._n[layer_idx]
        if n0 is None or n0 == 0:
            return None
        P = self.config.page_size
        new_page = n0 % P == 0
        pt = self._pt[layer_idx]
        if (new_page and (self._free_top < 1 or pt.numel() < n0 // P + 1)):
            return None
        if (k.dtype != self._dtype or q.dtype != self._dtype or k.shape[2] != 1
                or k.shape[0] != self._B or k.shape[1] != self._Hkv or k.shape[3] != self._D
                or v.shape != k.shape or k.stride() != v.stride() or k.stride(3) != 1
                or q.stride(3) != 1 or not k.is_cuda):
            return None
        cur = n0 + 1
        seen = self._seen_tokens + 1 if layer_idx == 0 else self._seen_tokens
        T = max(seen, cur)
        floor = self.config.sink_tokens + self.config.local_window
        if T <= floor:
            budget = T
        else:
            num_layers = max(self.num_layers, len(self._n))
            key = (layer_idx, num_layers)
            ratio = self._ratio_cache.get(key)
            if ratio is None:
                ratio = self._ratio_cache[key] = self.config.get_layer_ratio(layer_idx, num_layers)
            budget = min(T, max(floor, int(T * ratio)))
        if cur > budget + P:
            return None
        B, Hq, _, D = q.shape
        if out is None:
            out = torch.empty(B, Hq, 1, D, dtype=q.dtype, device=q.device)
        lay = self._lay_cache.get(layer_idx)
        if lay is None:
            lay = self._lay_cache[layer_idx] = self._layout(layer_idx)
        lay.num_tokens = n0
        qs, os_ = self._q_struct, self._o_struct
        qs.q = q.data_ptr(); qs.dtype = self._dtype_code; qs.num_heads = Hq; qs.q_len = 1
        qs.stride_b = q.stride(0); qs.stride_h = q.stride(1); qs.stride_t = q.stride(2)
        os_.out = out.data_ptr(); os_.dtype = self._dtype_code
        os_.stride_b = out.stride(0); os_.stride_h = out.stride(1); os_.stride_t = out.stride(2)
        lay.num_tokens = cur
        ws_need = self._lib.rkv_decode_fused_workspace_size(qs, lay)
        lay.num_tokens = n0
        stream = stream_ptr(self._device)
        ws = self._ws.get(stream)
        if ws is None or ws.numel() < ws_need:
            ws = self._ws[stream] = Workspace.get(self._device, ws_need)
        decay = self.config.salience_decay
        obs = self.launch_observer
        if obs is not None:
            obs.before(layer_idx, 2 * B * self._Hkv * cur * D * self._elt)
        peer = None
        if self.head_group is not None:
            hg = self.head_group
            if hg.peer is not None and cur + hg.num_kv_heads_total <= hg.peer.stride:
                # head-sharded over NVLink: the kernel stores its share into every rank's
                # region; the update below waits on the ranks' flags (no collective)
                peer = hg.peer.next()
                xc = Exchange(0, hg.peer.stride, cur, hg.head0, hg.num_kv_heads_total)
                st = self._lib.rkv_append_decode_peer(
                    lay, k.data_ptr(), v.data_ptr(), k.stride(0), k.stride(1), pt.data_ptr(),
                    self._free.data_ptr(), self._free_top, self._sal_init, qs,
                    float(scaling) if scaling else 0.0, os_, xc, peer, ws.data_ptr(),
                    ws.numel(), stream)
                what = "rkv_append_decode_peer"
                if st == 2:   # not a fused-kernel shape: every rank takes the collective path
                    peer = None
            if peer is None:
                # head-sharded: keys and norms to the exchange block, then the MAX over the
                # group and the salience update (below, once the token count is advanced)
                self._xbegin(layer_idx, score_tokens=cur, new_first=n0, n_new=1)
                st = self._lib.rkv_append_decode_partial(
                    lay, k.data_ptr(), v.data_ptr(), k.stride(0), k.stride(1), pt.data_ptr(),
                    self._free.data_ptr(), self._free_top, self._sal_init, qs,
                    float(scaling) if scaling else 0.0, os_, self._xpend[2], ws.data_ptr(),
                    ws.numel(), stream)
                what = "rkv_append_decode_partial"
        else:
            st = self._lib.rkv_append_decode(
                lay, self._sal_struct, k.data_ptr(), v.data_ptr(), k.stride(0), k.stride(1),
                pt.data_ptr(), self._free.data_ptr(), self._free_top, self._sal_init, qs,
                decay, 1.0 - decay, float(scaling) if scaling else 0.0, os_, ws.data_ptr(),
                ws.numel(), stream)
            what = "rkv_append_decode"
        if obs is not None:
            obs.after()
        check(st, what)
        if new_page:
            self._free_top -= 1
        self._n[layer_idx] = cur
        self._seen_tokens = seen
        self._layers[layer_idx].cumulative_length = seen
        if peer is not None:
            st = self._lib.rkv_salience_apply_peer(
                self._layout(layer_idx), self._sal_struct, xc, peer, cur, n0, 1, self._sal_init,
                decay, 1.0 - decay, ws.data_ptr(), ws.numel(), stream)
            check(st, "rkv_salience_apply_peer")
        elif self.head_group is not None:
            self._settle()
        return out

    def check_errors(self) -> None:
        """Raise ``DeviceError`` if a decode kernel of this cache's device recorded a
        device-side error (a bounded wait that gave up, a page id outside the pool) since the
        last check, and clear the flags.  Synchronises the device."""
        if self._device is not None:
            Workspace.check_errors(self._device)

    def _kv_bytes(self, layer_idx: int) -> int:
        """Bytes of retained K and V one attention pass over the layer reads."""
        return 2 * self._B * self._Hkv * self._n[layer_idx] * self._D * self._elt

    def attention(self, query_states: torch.Tensor, layer_idx: int,
                  scaling: Optional[float] = None, is_causal: bool = False) -> torch.Tensor:
        """Attention of query_states [B, Hq, QL, D] over the retained cache of one layer.

        A hook query kept for this layer (see ``update_salience_with_query``) is scored in
        the same pass over K (``rkv_decode_scored``)."""
        lib = _lib.load()
        q = query_states if query_states.stride(-1) == 1 else query_states.contiguous()
        B, Hq, QL, D = q.shape
        out = torch.empty(B, Hq, QL, D, dtype=q.dtype, device=q.device)
        qs = Query(q.data_ptr(), dtype_code(q.dtype), Hq, QL, q.stride(0), q.stride(1), q.stride(2))
        os_ = Output(out.data_ptr(), dtype_code(out.dtype), 0, out.stride(0), out.stride(1),
                     out.stride(2))
        lay = self._layout(layer_idx)
        pending = self._pending.pop(layer_idx, None)
        if pending is not None:
            if QL != 1 or is_causal or pending[0].shape[1] != Hq:
                self._score(pending[0], layer_idx, pending[1])
            else:
                qp = pending[0]
                qps = Query(qp.data_ptr(), dtype_code(qp.dtype), Hq, 1, qp.stride(0),
                            qp.stride(1), qp.stride(2))
                decay = self.config.salience_decay
                ws = Workspace.get(self._device, lib.rkv_decode_scored_workspace_size(qs, lay))
                st = lib.rkv_decode_scored(qps, qs, lay, self._salience(), pending[1],
                                           float(decay), float(1.0 - decay),
                                           float(scaling) if scaling else 0.0, os_,
                                           ws.data_ptr(), ws.numel(), self._stream())
                check(st, "rkv_decode_scored")
                return out
        ws = Workspace.get(self._device, lib.rkv_decode_attention_workspace_size(qs, lay))
        st = lib.rkv_decode_attention(qs, lay, float(scaling) if scaling else 0.0,
                                      1 if (is_causal and QL > 1) else 0, os_, ws.data_ptr(),
                                      ws.numel(), self._stream())
        check(st, "rkv_decode_attention")
        return out

    # --------------------------------------------------------------------- materialisation
    def _materialize(self, layer_idx: int, which: int) -> Optional[torch.Tensor]:
        """Contiguous [B, Hkv, N, D] K (which=0) / V (1) or [B, N] fp32 salience (2)."""
        if layer_idx >= len(self._n) or self._n[layer_idx] is None:
            return None
        if which == 2:
            self._flush_pending(layer_idx)
        lib = _lib.load()
        N = self._n[layer_idx]
        lay = self._layout(layer_idx)
        if which == 2:
            dst = torch.empty(self._B, self._Hkv, N, self._D, dtype=self._dtype, device=self._device)
            sal = torch.empty(self._B, N, dtype=torch.float32, device=self._device)
            st = lib.rkv_gather_tokens(lay, 0, dst.data_ptr(), self._salience(), sal.data_ptr(),
                                       self._stream())
            check(st, "rkv_gather_tokens")
            return sal
        dst = torch.empty(self._B, self._Hkv, N, self._D, dtype=self._dtype, device=self._device)
        st = lib.rkv_gather_tokens(lay, which, dst.data_ptr(), None, None, self._stream())
        check(st, "rkv_gather_tokens")
        return dst

    def page_table(self, layer_idx: int) -> torch.Tensor:
        """Physical slot of every logical page of one layer (a copy)."""
        return self._pt[layer_idx][: self._pages(self._n[layer_idx])].clone()

    # ---------------------------------------------------------------- cache-level utilities
    def _crop_layer(self, layer_idx: int, tokens_to_remove: int):
        if tokens_to_remove <= 0 or self._n[layer_idx] is None:
            return
        N = self._n[layer_idx]
        new_n = max(0, N - tokens_to_remove)
        old_pages, new_pages = self._pages(N), self._pages(new_n)
        if old_pages > new_pages:
            lib = _lib.load()
            pt = self._pt[layer_idx]
            st = lib.rkv_release_pages(pt[new_pages:].data_ptr(), old_pages - new_pages,
                                       self._free.data_ptr(), self._free_top, self._stream())
            check(st, "rkv_release_pages")
            self._free_top += old_pages - new_pages
        self._n[layer_idx] = new_n
        if self._rowmap is not None and new_pages > 0:
            # the new last page will be written again: give every sequence its own rows
            last = self._pt[layer_idx][new_pages - 1: new_pages]
            self._reindex_rows(torch.arange(self._B, device=self._device), last, 1)

    def crop(self, tokens_to_remove: int = 0) -> None:
        """razorkv/cache.py:177-188: drop the most recent tokens of every layer."""
        if tokens_to_remove <= 0:
            return
        self._flush_pending()
        for l in range(len(self._n)):
            if self._n[l] is not None:
                self._crop_layer(l, tokens_to_remove)
                self._sync_layer(l)
        self._seen_tokens = max(0, self._seen_tokens - tokens_to_remove)

    def reset(self) -> None:
        """razorkv/cache.py:190-196."""
        self._pending.clear()
        self._n.clear()
        self._pt.clear()
        self._layers.clear()
        self._seen_tokens = 0
        self._lay_cache.clear()
        self._rowmap = None
        if self._k is not None:
            self._free = torch.arange(self._slots - 1, -1, -1, dtype=torch.int64, device=self._device)
            self._free_top = self._slots

    def _live_slots(self) -> Tuple[torch.Tensor, int]:
        """Physical slots that hold retained pages, each layer's last page first, and the number
        of those last pages.  Each slot appears once: no slot serves two layers."""
        last, rest = [], []
        for l, n in enumerate(self._n):
            if n:
                pages = self._pages(n)
                last.append(self._pt[l][pages - 1: pages])
                rest.append(self._pt[l][: pages - 1])
        if not last:
            return torch.empty(0, dtype=torch.int64, device=self._device), 0
        return torch.cat(last + rest), len(last)

    def _pool_layout(self, k, v, batch, rowmap) -> KVLayout:
        return KVLayout(k.data_ptr(), v.data_ptr(), dtype_code(self._dtype), self._D, batch,
                        self._Hkv, k.stride(1), k.stride(2), k.stride(0), k.stride(3),
                        self.config.page_size, self._slots, None, 0, 0,
                        rowmap.data_ptr() if rowmap is not None else None)

    def _reindex_rows(self, idx: torch.Tensor, slots: torch.Tensor, num_moved: int):
        """In-place ``rkv_reindex_batch`` over ``slots`` (the first ``num_moved`` move their
        K/V rows; the others only have their row map rewritten)."""
        lib = _lib.load()
        idx = idx.to(device=self._device, dtype=torch.int64).reshape(-1).contiguous()
        flag = Workspace._flag(Workspace.get(self._device, 1 << 20))
        lay = self._pool_layout(self._k, self._v, self._B, self._rowmap)
        sal = self._salience()
        st = lib.rkv_reindex_batch(lay, sal, lay, sal, idx.data_ptr(), slots.data_ptr(),
                                   slots.numel(), num_moved, flag.data_ptr(), self._stream())
        check(st, "rkv_reindex_batch")

    def _reindex_batch(self, index: torch.Tensor):
        """Sequence b becomes sequence index[b] (``rkv_reindex_batch`` over the live pages).

        The same batch size (beam search) is a page-table update: every full page keeps its
        K/V and the row map points each sequence at the row of the beam it continues; only
        the salience rows (every beam's EWMA diverges) and each layer's last page (it will be
        written again) move.  A new batch size gathers the live pages into a new pool.  Free
        slots are never copied.  An index outside [0, B) raises ``DeviceError`` at the next
        ``check_errors`` (that sequence keeps its old contents)."""
        self._flush_pending()
        idx = index.to(device=self._device, dtype=torch.int64).reshape(-1).contiguous()
        new_b = idx.numel()
        slots, n_last = self._live_slots()
        if new_b == self._B and not self.share_pages_on_reorder:
            self._reindex_rows(idx, slots, slots.numel())
            return
        if new_b == self._B:
            if self._rowmap is None:
                self._rowmap = torch.arange(self._B, dtype=torch.int32,
                                            device=self._device).repeat(self._slots, 1)
                self._pool_changed()
            self._reindex_rows(idx, slots, n_last)
            return
        lib = _lib.load()
        flag = Workspace._flag(Workspace.get(self._device, 1 << 20))
        P = self.config.page_size
        shape = (self._slots, new_b, self._Hkv, P, self._D)
        k = torch.zeros(shape, dtype=self._dtype, device=self._device)
        v = torch.zeros(shape, dtype=self._dtype, device=self._device)
        s = torch.zeros((self._slots, new_b, P), dtype=torch.float32, device=self._device)
        src = self._pool_layout(self._k, self._v, self._B, self._rowmap)
        dst = self._pool_layout(k, v, new_b, None)
        dst_sal = Salience(s.data_ptr(), s.stride(1), s.stride(0))
        st = lib.rkv_reindex_batch(src, self._salience(), dst, dst_sal, idx.data_ptr(),
                                   slots.data_ptr(), slots.numel(), slots.numel(),
                                   flag.data_ptr(), self._stream())
        check(st, "rkv_reindex_batch")
        self._k, self._v, self._s = k, v, s
        self._rowmap = None
        self._B = new_b
        self._pool_changed()

    def batch_repeat_interleave(self, repeats: int) -> None:
        """razorkv/cache.py:198-206 (page tables are shared by every sequence)."""
        if not self.is_initialized:
            return
        idx = torch.arange(self._B, device=self._device).repeat_interleave(repeats)
        self._reindex_batch(idx)

    def batch_select_indices(self, indices: torch.Tensor) -> None:
        """razorkv/cache.py:208-218."""
        if not self.is_initialized:
            return
        self._reindex_batch(indices)

    def reorder_cache(self, beam_idx: torch.LongTensor):
        """razorkv/cache.py:220-229."""
        if not self.is_initialized:
            return
        self._reindex_batch(beam_idx)

    def get_memory_stats(self) -> Dict[str, Any]:
        """razorkv/cache.py:416-436: bytes of the retained K and V of every layer."""
        total_elements = 0
        per_layer = []
        for n in self._n:
            if n is not None:
                total_elements += 2 * self._B * self._Hkv * n * self._D
                per_layer.append(n)
        elt = torch.tensor([], dtype=self._dtype).element_size() if self._dtype else 0
        total_bytes = total_elements * elt
        return {
            "total_bytes": total_bytes,
            "total_mb": total_bytes / (1024 * 1024),
            "total_elements": total_elements,
            "per_layer_tokens": per_layer,
            "seen_tokens": self._seen_tokens,
            "pool_slots": self._slots,
            "free_slots": self._free_top,
        }


# The reference's class name, for code that constructs the cache by name.
RazorKVCache = PagedRazorKVCache
