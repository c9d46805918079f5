"""The reference's kernel operators, served by the CUDA library.

Same names, arguments, return values and error behaviour as ``razorkv.kernels``
(razorkv/kernels/__init__.py:5-13):

* ``triton_paged_sparse_attention(query, key_paged, value_paged, page_table, scale=None)``
  (razorkv/kernels/triton_paged_sparse.py:105-174) -- decode attention over the pages a
  per-sequence page table lists; ``AssertionError`` when q_len != 1.  ``paged_sparse_attention``
  is the same function under a name that does not mention Triton (none is used here).
* ``compacted_paged_sdpa(query_states, key_states, value_states, attention_mask=None,
  scaling=None, dropout_p=0.0, is_causal=False)`` (razorkv/kernels/torch_sparse.py:15-61).
* ``compute_page_salience_pool(salience_scores, page_size, pool_type="max")``
  (razorkv/kernels/torch_sparse.py:64-93).
* ``is_triton_available()`` (triton_paged_sparse.py:177-179) -- kept for callers that gate
  on it; True when the CUDA path can run (a CUDA device and the built library).

Every operator requires CUDA tensors and raises on anything it cannot run; there is no
CPU fallback.  All of them are also registered as ``torch.ops.razorkv.*`` custom ops.
"""

import math
import threading
from typing import Optional, Tuple

import torch

from . import _lib
from ._lib import KVLayout, Output, Query, check, dtype_code, require_cuda, stream_ptr

__all__ = [
    "triton_paged_sparse_attention",
    "paged_sparse_attention",
    "compacted_paged_sdpa",
    "compute_page_salience_pool",
    "is_triton_available",
    "check_device_errors",
    "Workspace",
]


class Workspace:
    """Caller-owned scratch memory for one (device, stream): grows, never shrinks.

    Zero-initialised, because the split-K merge counters inside it must start at zero (the
    kernels return them to zero after every launch)."""

    _pool = {}
    # error flags of workspaces replaced by larger ones (read by the next check)
    _retired = {}
    _lock = threading.Lock()

    @classmethod
    def get(cls, device: torch.device, nbytes: int) -> torch.Tensor:
        key = (device.index, stream_ptr(device))
        buf = cls._pool.get(key)
        if buf is None or buf.numel() < nbytes:
            size = max(nbytes, 1 << 20)
            with cls._lock:
                if buf is not None:
                    size = max(size, 2 * buf.numel())
                    # keep the old flag word until it has been checked
                    cls._retired.setdefault(device.index, []).append(cls._flag(buf).clone())
                buf = torch.zeros(size, dtype=torch.uint8, device=device)
                cls._pool[key] = buf
        return buf

    @staticmethod
    def _flag(buf: torch.Tensor) -> torch.Tensor:
        off = int(_lib.load().rkv_workspace_error_flag_offset())
        return buf[off: off + 4].view(torch.int32)

    @classmethod
    def check_errors(cls, device=None, clear: bool = True) -> None:
        """Raise ``DeviceError`` if a decode kernel flagged an error in any workspace of
        ``device`` (all devices when None) since the last check, and clear the flags.

        The decode kernels never stop the stream on a device-side error: a bounded wait that
        gave up (code 1) or a page-table entry outside the pool (code 2; the page is read as
        slot 0 instead) only sets the workspace's int32 error flag, so the result of that
        launch is wrong while the launch itself reports success.  This check reads the flags
        (one device synchronisation), so call it at sync points -- after a generation, at the
        end of a timed region, in tests -- not inside the decode loop."""
        codes = []
        want = None if device is None else torch.device(device).index
        with cls._lock:
            for (dev, _), buf in list(cls._pool.items()):
                if want is not None and dev != want:
                    continue
                flag = cls._flag(buf)
                code = int(flag.item())
                if code:
                    codes.append(code)
                    if clear:
                        flag.zero_()
            for dev in list(cls._retired):
                if want is not None and dev != want:
                    continue
                flags = cls._retired.pop(dev, []) if clear else cls._retired.get(dev, [])
                codes += [int(f.item()) for f in flags if int(f.item())]
        if codes:
            raise _lib.DeviceError(max(codes))


def check_device_errors(device=None) -> None:
    """Raise ``razorkv_b200._lib.DeviceError`` if a decode kernel recorded a device-side
    error on ``device`` (every device when None) since the last check; clears the flags.
    Synchronises the device: call it at sync points, not per step."""
    Workspace.check_errors(device)


def _query(q: torch.Tensor) -> Query:
    # q: [B, H, QL, D], last dim contiguous
    return Query(q.data_ptr(), dtype_code(q.dtype), q.shape[1], q.shape[2],
                 q.stride(0), q.stride(1), q.stride(2))


def _output(o: torch.Tensor) -> Output:
    return Output(o.data_ptr(), dtype_code(o.dtype), 0, o.stride(0), o.stride(1), o.stride(2))


def _last_dim_contiguous(t: torch.Tensor) -> torch.Tensor:
    return t if t.stride(-1) == 1 else t.contiguous()


def is_triton_available() -> bool:
    if not torch.cuda.is_available():
        return False
    try:
        _lib.load()
    except ImportError:
        return False
    return True


def _run_attention(q, layout: KVLayout, scale: Optional[float], causal: bool, out):
    lib = _lib.load()
    qs, os_ = _query(q), _output(out)
    ws_bytes = lib.rkv_decode_attention_workspace_size(qs, layout)
    ws = Workspace.get(q.device, ws_bytes)
    st = lib.rkv_decode_attention(qs, layout, float(scale) if scale else 0.0, 1 if causal else 0,
                                  os_, ws.data_ptr(), ws.numel(), stream_ptr(q.device))
    check(st, "rkv_decode_attention")


def triton_paged_sparse_attention(
    query: torch.Tensor,
    key_paged: torch.Tensor,
    value_paged: torch.Tensor,
    page_table: torch.Tensor,
    scale: Optional[float] = None,
    validate: bool = True,
) -> torch.Tensor:
    """Block-sparse paged decode attention.

    query [B, H, 1, D]; key_paged / value_paged [B, Hkv, MAXP, P, D]; page_table
    [B, n_active] integer page indices; returns [B, H, 1, D] in the query dtype.
    ``validate`` checks every table entry against MAXP on the host first (one device sync).
    """
    require_cuda(query, key_paged, value_paged, page_table)
    B, H, q_len, D = query.shape
    assert q_len == 1, "paged decode attention is defined for single-token decoding (q_len == 1)."
    _, Hkv, max_pages, P, Dk = key_paged.shape
    if Dk != D or value_paged.shape != key_paged.shape:
        raise ValueError("key_paged/value_paged must both be [B, Hkv, MAXP, P, D] matching the query")
    if H % Hkv != 0:
        raise ValueError(f"num_heads {H} is not a multiple of num_kv_heads {Hkv}")
    if key_paged.dtype != value_paged.dtype:
        raise TypeError("key_paged and value_paged must share a dtype")
    kp = _last_dim_contiguous(key_paged)
    vp = _last_dim_contiguous(value_paged)
    if kp.stride() != vp.stride():
        kp, vp = kp.contiguous(), vp.contiguous()
    if kp.stride(3) != D:
        kp, vp = kp.contiguous(), vp.contiguous()
    pt = page_table.to(torch.int64)
    if pt.dim() != 2 or pt.shape[0] != B:
        raise ValueError("page_table must be [B, n_active]")
    pt = pt.contiguous()
    n_active = pt.shape[1]
    if validate and pt.numel():
        lo, hi = int(pt.min()), int(pt.max())
        if lo < 0 or hi >= max_pages:
            raise IndexError(f"page_table entries must lie in [0, {max_pages}), got [{lo}, {hi}]")
    q = _last_dim_contiguous(query)
    out = torch.empty(B, H, 1, D, dtype=query.dtype, device=query.device)
    if n_active == 0 or B == 0:
        return out.zero_()
    layout = KVLayout(kp.data_ptr(), vp.data_ptr(), dtype_code(kp.dtype), D, B, Hkv,
                      kp.stride(0), kp.stride(1), kp.stride(2), kp.stride(3), P, max_pages,
                      pt.data_ptr(), pt.stride(0), n_active * P)
    _run_attention(q, layout, scale, False, out)
    return out


paged_sparse_attention = triton_paged_sparse_attention


def compacted_paged_sdpa(
    query_states: torch.Tensor,
    key_states: torch.Tensor,
    value_states: torch.Tensor,
    attention_mask: Optional[torch.Tensor] = None,
    scaling: Optional[float] = None,
    dropout_p: float = 0.0,
    is_causal: bool = False,
) -> torch.Tensor:
    """Attention over compacted contiguous K/V with GQA head grouping.

    query [B, H, QL, D]; key/value [B, Hkv, N, D]; returns [B, H, QL, D] in the query dtype.
    ``is_causal`` applies only when QL > 1 (upper-left aligned, as torch SDPA).  Masks and
    dropout are not implemented on this path and raise."""
    require_cuda(query_states, key_states, value_states)
    if attention_mask is not None:
        raise NotImplementedError("compacted_paged_sdpa: attention_mask is not supported on the CUDA path")
    if dropout_p:
        raise NotImplementedError("compacted_paged_sdpa: dropout is not supported on the CUDA path")
    B, H, QL, D = query_states.shape
    _, Hkv, N, Dk = key_states.shape
    if Dk != D or value_states.shape != key_states.shape:
        raise ValueError("key_states/value_states must be [B, Hkv, N, D] matching the query")
    if H % Hkv != 0:
        raise ValueError(f"num_heads {H} is not a multiple of num_kv_heads {Hkv}")
    k = _last_dim_contiguous(key_states)
    v = _last_dim_contiguous(value_states)
    if k.stride() != v.stride():
        k, v = k.contiguous(), v.contiguous()
    q = _last_dim_contiguous(query_states)
    out = torch.empty(B, H, QL, D, dtype=query_states.dtype, device=query_states.device)
    if B == 0 or QL == 0:
        return out
    if N == 0:
        return out.zero_()
    layout = KVLayout(k.data_ptr(), v.data_ptr(), dtype_code(k.dtype), D, B, Hkv,
                      k.stride(0), k.stride(1), 0, k.stride(2), 1, 0, None, 0, N)
    _run_attention(q, layout, scaling, bool(is_causal and QL > 1), out)
    return out


def compute_page_salience_pool(
    salience_scores: torch.Tensor,
    page_size: int,
    pool_type: str = "max",
) -> Tuple[torch.Tensor, int]:
    """Pools token salience [B, S] into page scores; returns (scores [B, n_pages], n_pages)."""
    require_cuda(salience_scores)
    if pool_type not in ("max", "mean"):
        raise ValueError(f"Unknown pool_type: {pool_type}")
    B, S = salience_scores.shape
    n_pages = S // page_size
    ret_pages = n_pages if n_pages > 0 else 1
    sal = salience_scores.to(torch.float32)
    if sal.stride(1) != 1:
        sal = sal.contiguous()
    out = torch.empty(B, ret_pages, dtype=torch.float32, device=sal.device)
    if B == 0 or S == 0:
        return out.to(salience_scores.dtype), ret_pages
    lib = _lib.load()
    st = lib.rkv_page_salience_pool(sal.data_ptr(), B, S, sal.stride(0), page_size,
                                    _lib.POOL_MEAN if pool_type == "mean" else _lib.POOL_MAX,
                                    out.data_ptr(), stream_ptr(sal.device))
    check(st, "rkv_page_salience_pool")
    return out.to(salience_scores.dtype), ret_pages


# ---- torch.ops.razorkv registration ---------------------------------------------------------
def _register_ops():
    lib = torch.library.Library("razorkv", "FRAGMENT")
    lib.define("paged_decode_attention(Tensor query, Tensor key_paged, Tensor value_paged, "
               "Tensor page_table, float scale=0.0) -> Tensor")
    lib.define("compacted_sdpa(Tensor query, Tensor key, Tensor value, float scale=0.0, "
               "bool is_causal=False) -> Tensor")
    lib.define("page_salience_pool(Tensor salience, int page_size, str pool_type='max') -> Tensor")

    def _paged(query, key_paged, value_paged, page_table, scale=0.0):
        return triton_paged_sparse_attention(query, key_paged, value_paged, page_table,
                                             scale or None)

    def _dense(query, key, value, scale=0.0, is_causal=False):
        return compacted_paged_sdpa(query, key, value, scaling=scale or None, is_causal=is_causal)

    def _pool(salience, page_size, pool_type="max"):
        return compute_page_salience_pool(salience, page_size, pool_type)[0]

    lib.impl("paged_decode_attention", _paged, "CUDA")
    lib.impl("compacted_sdpa", _dense, "CUDA")
    lib.impl("page_salience_pool", _pool, "CUDA")

    def _paged_meta(query, key_paged, value_paged, page_table, scale=0.0):
        return torch.empty_like(query)

    def _dense_meta(query, key, value, scale=0.0, is_causal=False):
        return torch.empty_like(query)

    def _pool_meta(salience, page_size, pool_type="max"):
        n = max(1, salience.shape[1] // page_size)
        return salience.new_empty(salience.shape[0], n)

    lib.impl("paged_decode_attention", _paged_meta, "Meta")
    lib.impl("compacted_sdpa", _dense_meta, "Meta")
    lib.impl("page_salience_pool", _pool_meta, "Meta")
    return lib


try:
    _TORCH_LIBRARY = _register_ops()
except RuntimeError:   # already registered in this process
    _TORCH_LIBRARY = None
