"""CPU oracle of the RazorKV decode path -- TEST INFRASTRUCTURE ONLY.

Only the test suite, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py``
import this module; the product package never does.  It restates the reference cache at
the reference's own (logical, contiguous) level:

* ``OracleCache.update``                     razorkv/cache.py:361-414
* ``OracleCache.update_salience_with_query`` razorkv/cache.py:249-287
* ``OracleCache._evict_layer``               razorkv/cache.py:289-359
* ``OracleCache._init_salience``             razorkv/cache.py:239-247
* ``budget``                                 razorkv/config.py:65-112
* ``page_pool``                              razorkv/kernels/torch_sparse.py:64-93
* ``attention``                              razorkv/kernels/torch_sparse.py:15-61

with three documented adjustments:

1. fp32 dot products, norms and the batch mean use the canonical summation order of
   ``oracle.c`` (shared with the CUDA kernels) instead of torch's ISA-dependent orders;
   the batch mean is a sequential fp32 sum over b followed by one fp32 division;
2. exact ties in the top-k page selection go to the lower page index (torch.topk does not
   promise any order among ties);
3. every token carries an integer id through appends and compactions, so a kept set can
   be compared without looking at the data, and every top-k decision records the gap
   between the k-th and (k+1)-th page score (the near-tie margin).

Arrays are numpy fp32 holding values exactly representable in the cache dtype (bf16 values
widened losslessly); ``elt_size`` (2 for bf16/fp16, 4 for fp32) selects the chunk width of
the canonical order.
"""

import ctypes
import math
import os
import subprocess
from dataclasses import dataclass, field
from typing import List, Optional

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None


def build_oracle(force: bool = False) -> str:
    """Compile oracle.c into oracle/_build/liboracle.so (gcc, OpenMP, no FP contraction)."""
    src = os.path.join(_HERE, "oracle.c")
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        os.makedirs(os.path.dirname(_LIB_PATH), exist_ok=True)
        subprocess.check_call(["make", "-s", "-C", _HERE])
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build_oracle()
        L = ctypes.CDLL(_LIB_PATH)
        P, I, F, D = ctypes.c_void_p, ctypes.c_int64, ctypes.c_float, ctypes.c_double
        L.orc_canon_dot.argtypes = [P, P, I, I]
        L.orc_canon_dot.restype = F
        L.orc_norm_salience.argtypes = [P, I, I, I, I, I, P]
        L.orc_resonance.argtypes = [P, P, I, I, I, I, I, I, I, F, P]
        L.orc_ewma.argtypes = [P, P, I, F, F]
        L.orc_attention.argtypes = [P, P, P, I, I, I, I, I, I, D, ctypes.c_int, P]
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctypes.c_void_p)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


# ------------------------------------------------------------------------------------------
# kernels
# ------------------------------------------------------------------------------------------
def canon_dot(a, b, elt_size: int) -> np.float32:
    a, b = _f32(a), _f32(b)
    return np.float32(lib().orc_canon_dot(_p(a), _p(b), a.shape[-1], 16 // elt_size))


def norm_salience(k: np.ndarray, elt_size: int) -> np.ndarray:
    """[B, H, T, D] -> [B, T] fp32 (razorkv/cache.py:241-243)."""
    k = _f32(k)
    B, H, T, D = k.shape
    out = np.empty((B, T), np.float32)
    lib().orc_norm_salience(_p(k), B, H, T, D, 16 // elt_size, _p(out))
    return out


def resonance(q: np.ndarray, k: np.ndarray, elt_size: int) -> np.ndarray:
    """max over (q head, q row) of (q*scale).k -> [B, N] fp32 (razorkv/cache.py:263-280)."""
    q, k = _f32(q), _f32(k)
    B, Hq, QL, D = q.shape
    _, Hkv, N, _ = k.shape
    scale = np.float32(1.0 / math.sqrt(D))
    R = np.empty((B, N), np.float32)
    lib().orc_resonance(_p(q), _p(k), B, Hq, Hkv, QL, N, D, 16 // elt_size, scale, _p(R))
    return R


def ewma(S: np.ndarray, R: np.ndarray, decay: float) -> np.ndarray:
    """decay*S + (1-decay)*R in fp32 without contraction (razorkv/cache.py:285)."""
    S = _f32(S).copy()
    R = _f32(R)
    lib().orc_ewma(_p(S), _p(R), S.size, np.float32(decay), np.float32(1.0 - decay))
    return S


def attention(q, k, v, scale: Optional[float] = None, causal: bool = False) -> np.ndarray:
    """softmax(q.k*scale).v with GQA grouping, fp64 (razorkv/kernels/torch_sparse.py:15-61)."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    B, Hq, QL, D = q.shape
    _, Hkv, N, _ = k.shape
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    out = np.empty((B, Hq, QL, D), np.float64)
    lib().orc_attention(_p(q), _p(k), _p(v), B, Hq, Hkv, QL, N, D, float(scale),
                        1 if (causal and QL > 1) else 0, _p(out))
    return out


def paged_attention(q, k_paged, v_paged, page_table, scale=None) -> np.ndarray:
    """Gather pages by table then attend (razorkv/kernels/triton_paged_sparse.py:124-139)."""
    k_paged, v_paged = _f32(k_paged), _f32(v_paged)
    B, Hkv, _, P, D = k_paged.shape
    pt = np.asarray(page_table, dtype=np.int64)
    K = np.stack([k_paged[b][:, pt[b]].reshape(Hkv, -1, D) for b in range(B)])
    V = np.stack([v_paged[b][:, pt[b]].reshape(Hkv, -1, D) for b in range(B)])
    return attention(q, K, V, scale)


def page_pool(S: np.ndarray, page_size: int, pool: str = "max"):
    """[B, N] -> ([B, n_pages], n_pages) (razorkv/kernels/torch_sparse.py:64-93)."""
    S = _f32(S)
    B, N = S.shape
    n = N // page_size
    if n == 0:
        return S.max(axis=-1, keepdims=True), 1
    r = S[:, : n * page_size].reshape(B, n, page_size)
    if pool == "max":
        return r.max(axis=-1), n
    if pool == "mean":
        acc = np.zeros((B, n), np.float32)
        for t in range(page_size):
            acc = (acc + r[:, :, t]).astype(np.float32)
        return (acc / np.float32(page_size)).astype(np.float32), n
    raise ValueError(f"Unknown pool_type: {pool}")


def batch_mean(scores: np.ndarray) -> np.ndarray:
    """Sequential fp32 sum over the batch, then one division (razorkv/cache.py:335-338)."""
    B = scores.shape[0]
    if B == 1:
        return scores[0].astype(np.float32)
    acc = scores[0].astype(np.float32).copy()
    for b in range(1, B):
        acc = (acc + scores[b]).astype(np.float32)
    return (acc / np.float32(B)).astype(np.float32)


def ordered_key(x: np.ndarray) -> np.ndarray:
    """Monotone uint32 key of fp32 values; every NaN maps above +inf."""
    u = _f32(x).view(np.uint32).astype(np.uint64)
    neg = (u >> 31) == 1
    key = np.where(neg, (~u) & 0xFFFFFFFF, u | 0x80000000)
    key = np.where(np.isnan(_f32(x)), 0xFFFFFFFF, key)
    return key.astype(np.uint64)


def canonical_topk(avg: np.ndarray, k: int):
    """Indices of the k largest values, ties to the lower index, returned ascending.

    Also returns the margin: avg[k-th] - avg[(k+1)-th] in the selection order (inf when
    every page is kept)."""
    key = ordered_key(avg)
    order = np.lexsort((np.arange(len(avg)), -key.astype(np.float64)))  # by key desc, index asc
    # lexsort on float64 of uint32 keys is exact (keys < 2**32)
    kept = np.sort(order[:k])
    if k < len(avg):
        margin = float(avg[order[k - 1]]) - float(avg[order[k]])
    else:
        margin = math.inf
    return kept.astype(np.int64), margin


# ------------------------------------------------------------------------------------------
# cache
# ------------------------------------------------------------------------------------------
@dataclass
class OracleConfig:
    """Independent restatement of the reference budget (razorkv/config.py:65-112)."""
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

    def ratio(self, layer: int, num_layers: int) -> float:
        if num_layers <= 1 or self.pyramid_mode == "uniform":
            return self.compression_ratio
        if self.pyramid_mode == "custom" and self.custom_layer_ratios is not None:
            return (self.custom_layer_ratios[layer] if layer < len(self.custom_layer_ratios)
                    else self.compression_ratio)
        x = layer / (num_layers - 1)
        lo, hi = self.pyramid_min_ratio, self.pyramid_max_ratio
        if self.pyramid_mode == "linear":
            return lo + x * (hi - lo)
        if self.pyramid_mode == "adaptive":
            raw = [lo + (i / (num_layers - 1)) ** 1.8 * (hi - lo) for i in range(num_layers)]
            s = self.compression_ratio / max(sum(raw) / len(raw), 1e-6)
            return max(0.05, min(1.0, (lo + x ** 1.8 * (hi - lo)) * s))
        return self.compression_ratio

    def budget(self, layer: int, num_layers: int, T: int) -> int:
        floor = self.sink_tokens + self.local_window
        if T <= floor:
            return T
        return min(T, max(floor, int(T * self.ratio(layer, num_layers))))


@dataclass
class Decision:
    layer: int
    seq_len: int
    budget: int
    kind: str                       # "pages" | "zones" (haystack budget <= 0)
    num_pages: int = 0
    kept: Optional[np.ndarray] = None
    margin: float = math.inf


class OracleCache:
    def __init__(self, cfg: OracleConfig, num_layers: int, elt_size: int):
        self.cfg = cfg
        self.num_layers = num_layers
        self.elt = elt_size
        self.K: List[Optional[np.ndarray]] = []
        self.V: List[Optional[np.ndarray]] = []
        self.S: List[Optional[np.ndarray]] = []
        self.ids: List[Optional[np.ndarray]] = []
        self.next_id: List[int] = []
        self.seen = 0
        self.decisions: List[Decision] = []
        # kept_override(layer, decision index, kept, margin) -> replacement kept pages or None
        # (lets a test follow another implementation's decision at a provable near-tie)
        self.kept_override = None

    def _init_salience(self, k):
        if self.cfg.salience_init == "norm":
            return norm_salience(k, self.elt)
        return np.ones((k.shape[0], k.shape[2]), np.float32)

    def update_salience_with_query(self, q, layer):
        if layer >= len(self.K) or self.K[layer] is None:
            return
        R = resonance(q, self.K[layer], self.elt)
        if self.S[layer] is not None:
            self.S[layer] = ewma(self.S[layer], R, self.cfg.salience_decay)
        else:
            self.S[layer] = R

    def _gather(self, layer, idx):
        self.K[layer] = np.ascontiguousarray(self.K[layer][:, :, idx, :])
        self.V[layer] = np.ascontiguousarray(self.V[layer][:, :, idx, :])
        self.S[layer] = np.ascontiguousarray(self.S[layer][:, idx])
        self.ids[layer] = self.ids[layer][idx]

    def _evict_layer(self, layer, budget):
        K, S = self.K[layer], self.S[layer]
        B, N = K.shape[0], K.shape[2]
        if N <= budget:
            return
        c = self.cfg
        sink = min(c.sink_tokens, N)
        local = min(c.local_window, N - sink)
        hs, he = sink, N - local
        if he - hs <= 0:
            return
        hb = budget - sink - local
        if hb <= 0:
            idx = np.concatenate([np.arange(0, sink), np.arange(he, N)])
            self.decisions.append(Decision(layer, N, budget, "zones"))
            self._gather(layer, idx)
            return
        P = c.page_size
        num_pages = (he - hs) // P
        if num_pages <= 0:
            return
        aligned = num_pages * P
        scores = S[:, hs: hs + aligned].reshape(B, num_pages, P).max(axis=-1)
        k = max(1, min(num_pages, hb // P))
        avg = batch_mean(scores)
        kept, margin = canonical_topk(avg, k)
        if self.kept_override is not None:
            repl = self.kept_override(layer, len(self.decisions), kept, margin)
            if repl is not None:
                kept = np.asarray(repl, dtype=np.int64)
        tok = (hs + kept[:, None] * P + np.arange(P)[None, :]).reshape(-1)
        parts = [np.arange(0, sink), tok]
        if aligned < he - hs:
            parts.append(np.arange(hs + aligned, he))
        parts.append(np.arange(he, N))
        self.decisions.append(Decision(layer, N, budget, "pages", num_pages, kept, margin))
        self._gather(layer, np.concatenate(parts).astype(np.int64))

    def update(self, k, v, layer, query_states=None):
        k, v = _f32(k), _f32(v)
        while len(self.K) <= layer:
            self.K.append(None); self.V.append(None); self.S.append(None)
            self.ids.append(None); self.next_id.append(0)
        new_s = self._init_salience(k)
        T = k.shape[2]
        is_prefill = T > 1
        new_ids = np.arange(self.next_id[layer], self.next_id[layer] + T, dtype=np.int64)
        self.next_id[layer] += T
        if self.K[layer] is None:
            self.K[layer], self.V[layer], self.S[layer] = k.copy(), v.copy(), new_s
            self.ids[layer] = new_ids
            if layer == 0:
                self.seen = T
        else:
            self.K[layer] = np.concatenate([self.K[layer], k], axis=2)
            self.V[layer] = np.concatenate([self.V[layer], v], axis=2)
            self.S[layer] = np.concatenate([self.S[layer], new_s], axis=1)
            self.ids[layer] = np.concatenate([self.ids[layer], new_ids])
            if layer == 0:
                self.seen += T
        if query_states is not None:
            self.update_salience_with_query(_f32(query_states), layer)
        cur = self.K[layer].shape[2]
        num_layers = max(self.num_layers, len(self.K))
        budget = self.cfg.budget(layer, num_layers, max(self.seen, cur))
        if is_prefill:
            ret = (self.K[layer], self.V[layer])
            if cur > budget:
                self._evict_layer(layer, budget)
            return ret
        if cur > budget + self.cfg.page_size:
            self._evict_layer(layer, budget)
        return self.K[layer], self.V[layer]
