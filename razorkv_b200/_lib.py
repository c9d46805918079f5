"""ctypes binding of librazorkv_b200.so (the C ABI declared in include/razorkv_b200.h).

The library is loaded from razorkv_b200/_lib/ and nothing else: if it is missing the
import fails with an error that says how to build it.  There is no CPU fallback.
"""

import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "librazorkv_b200.so")

c_i64 = ctypes.c_int64
c_i32 = ctypes.c_int32
c_vp = ctypes.c_void_p
c_f32 = ctypes.c_float
c_sz = ctypes.c_size_t

F32, F16, BF16 = 0, 1, 2
POOL_MAX, POOL_MEAN = 0, 1
SAL_NORM, SAL_UNIFORM = 0, 1

_STATUS = {
    0: "ok", 1: "invalid argument", 2: "unsupported shape or dtype", 3: "workspace too small",
    4: "free page list exhausted", 5: "misaligned pointer or stride",
    6: "CUDA launch or runtime error", 7: "page index out of range",
}


class KVLayout(ctypes.Structure):
    _fields_ = [
        ("k", c_vp), ("v", c_vp), ("dtype", c_i32), ("head_dim", c_i32),
        ("batch", c_i64), ("num_kv_heads", c_i64),
        ("stride_b", c_i64), ("stride_h", c_i64), ("stride_p", c_i64), ("stride_t", c_i64),
        ("page_size", c_i64), ("num_slots", c_i64), ("page_table", c_vp),
        ("pt_stride_b", c_i64), ("num_tokens", c_i64), ("row_map", c_vp),
    ]


class Query(ctypes.Structure):
    _fields_ = [("q", c_vp), ("dtype", c_i32), ("num_heads", c_i32), ("q_len", c_i64),
                ("stride_b", c_i64), ("stride_h", c_i64), ("stride_t", c_i64)]


class Output(ctypes.Structure):
    _fields_ = [("out", c_vp), ("dtype", c_i32), ("reserved", c_i32),
                ("stride_b", c_i64), ("stride_h", c_i64), ("stride_t", c_i64)]


class Salience(ctypes.Structure):
    _fields_ = [("s", c_vp), ("stride_b", c_i64), ("stride_p", c_i64)]


class Exchange(ctypes.Structure):
    _fields_ = [("x", c_vp), ("stride_b", c_i64), ("norm_off", c_i64), ("head0", c_i32),
                ("num_kv_heads_total", c_i32)]


class PeerExchange(ctypes.Structure):
    _fields_ = [("regions", c_vp), ("flags", c_vp), ("my_region", c_vp), ("my_flags", c_vp),
                ("rank", c_i32), ("nranks", c_i32), ("sub", c_i64), ("buf_off", c_i64),
                ("epoch", ctypes.c_uint32), ("reserved", ctypes.c_uint32)]


P = ctypes.POINTER

# name -> (restype, argtypes); mirrors include/razorkv_b200.h
_SIGNATURES = {
    "rkv_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "rkv_abi_version": (ctypes.c_int, []),
    "rkv_launch_count": (ctypes.c_ulonglong, []),
    "rkv_workspace_error_flag_offset": (c_sz, []),
    "rkv_selftest_wait_timeout": (ctypes.c_int, [c_vp, ctypes.c_longlong, c_vp]),
    "rkv_decode_attention_workspace_size": (c_sz, [P(Query), P(KVLayout)]),
    "rkv_decode_attention": (ctypes.c_int, [P(Query), P(KVLayout), c_f32, ctypes.c_int,
                                            P(Output), c_vp, c_sz, c_vp]),
    "rkv_decode_attention_noalloc": (ctypes.c_int, [P(Query), P(KVLayout), c_f32, ctypes.c_int,
                                                    P(Output), c_vp]),
    "rkv_page_salience_pool": (ctypes.c_int, [c_vp, c_i64, c_i64, c_i64, c_i64, ctypes.c_int,
                                              c_vp, c_vp]),
    "rkv_append": (ctypes.c_int, [P(KVLayout), P(Salience), c_vp, c_vp, c_i64, c_i64, c_i64,
                                  c_i64, c_i64, c_vp, c_vp, c_i64, ctypes.c_int, c_vp]),
    "rkv_score": (ctypes.c_int, [P(Query), P(KVLayout), P(Salience), c_f32, c_f32,
                                 ctypes.c_int, c_vp]),
    "rkv_decode_fused_workspace_size": (c_sz, [P(Query), P(KVLayout)]),
    "rkv_decode_fused": (ctypes.c_int, [P(Query), P(KVLayout), P(Salience), c_f32, c_f32,
                                        c_f32, P(Output), c_vp, c_sz, c_vp]),
    "rkv_append_decode": (ctypes.c_int, [P(KVLayout), P(Salience), c_vp, c_vp, c_i64, c_i64,
                                         c_vp, c_vp, c_i64, ctypes.c_int, P(Query), c_f32, c_f32,
                                         c_f32, P(Output), c_vp, c_sz, c_vp]),
    "rkv_decode_scored_workspace_size": (c_sz, [P(Query), P(KVLayout)]),
    "rkv_decode_scored": (ctypes.c_int, [P(Query), P(Query), P(KVLayout), P(Salience), c_i64,
                                         c_f32, c_f32, c_f32, P(Output), c_vp, c_sz, c_vp]),
    "rkv_page_scores": (ctypes.c_int, [P(KVLayout), P(Salience), c_i64, c_i64, c_i64, c_vp,
                                       c_vp]),
    "rkv_select_pages_workspace_size": (c_sz, [c_i64]),
    "rkv_select_pages": (ctypes.c_int, [c_vp, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp, c_sz,
                                        c_vp]),
    "rkv_compact_pages": (ctypes.c_int, [c_vp, c_i64, c_i64, c_vp, c_i64, c_i64, c_i64, c_vp,
                                         c_i64, c_vp]),
    "rkv_compact_tokens": (ctypes.c_int, [P(KVLayout), P(Salience), c_vp, c_vp, c_i64, c_i64,
                                          c_i64, c_vp, c_i64, c_i64, c_i64, c_i64, c_vp]),
    "rkv_release_pages": (ctypes.c_int, [c_vp, c_i64, c_vp, c_i64, c_vp]),
    "rkv_gather_tokens": (ctypes.c_int, [P(KVLayout), ctypes.c_int, c_vp, P(Salience), c_vp,
                                         c_vp]),
    "rkv_reindex_batch": (ctypes.c_int, [P(KVLayout), P(Salience), P(KVLayout), P(Salience),
                                         c_vp, c_vp, c_i64, c_i64, c_vp, c_vp]),
    "rkv_append_partial": (ctypes.c_int, [P(KVLayout), c_vp, c_vp, c_i64, c_i64, c_i64, c_i64,
                                          c_i64, c_vp, c_vp, c_i64, ctypes.c_int, P(Exchange),
                                          c_vp]),
    "rkv_score_partial": (ctypes.c_int, [P(Query), P(KVLayout), P(Exchange), c_vp]),
    "rkv_append_decode_partial": (ctypes.c_int, [P(KVLayout), c_vp, c_vp, c_i64, c_i64, c_vp,
                                                 c_vp, c_i64, ctypes.c_int, P(Query), c_f32,
                                                 P(Output), P(Exchange), c_vp, c_sz, c_vp]),
    "rkv_salience_apply": (ctypes.c_int, [P(KVLayout), P(Salience), P(Exchange), c_i64, c_i64,
                                          c_i64, ctypes.c_int, c_f32, c_f32, c_vp]),
    "rkv_ipc_export": (ctypes.c_int, [c_vp, c_vp, P(c_i64)]),
    "rkv_ipc_import": (ctypes.c_int, [c_vp, c_i64, P(c_vp)]),
    "rkv_ipc_release": (ctypes.c_int, [c_vp, c_i64]),
    "rkv_append_decode_peer": (ctypes.c_int, [P(KVLayout), c_vp, c_vp, c_i64, c_i64, c_vp, c_vp,
                                              c_i64, ctypes.c_int, P(Query), c_f32, P(Output),
                                              P(Exchange), P(PeerExchange), c_vp, c_sz, c_vp]),
    "rkv_salience_apply_peer": (ctypes.c_int, [P(KVLayout), P(Salience), P(Exchange),
                                               P(PeerExchange), c_i64, c_i64, c_i64, ctypes.c_int,
                                               c_f32, c_f32, c_vp, c_sz, c_vp]),
    "rkv_append_score_pool": (ctypes.c_int, [P(KVLayout), P(Salience), c_vp, c_vp, c_i64, c_i64,
                                             c_vp, c_vp, c_i64, ctypes.c_int, P(Query), c_f32,
                                             c_f32, c_i64, c_i64, c_vp, c_vp]),
    "rkv_select_compact_pages": (ctypes.c_int, [c_vp, c_i64, c_i64, c_i64, c_vp, c_i64, c_i64,
                                                c_i64, c_vp, c_i64, c_vp, c_vp, c_vp, c_sz,
                                                c_vp]),
}

EXPORTED = tuple(_SIGNATURES)

_lib = None


def load():
    """Load the library (once) and declare every entry point's signature."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing; build it with `python -m razorkv_b200.build` "
            "(the decode path has no CPU fallback)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


class RazorKVError(RuntimeError):
    pass


# Codes a decode kernel leaves in a workspace's error flag (read by Workspace.check_errors).
DEVICE_ERRORS = {
    1: "a bounded wait inside a decode kernel gave up (the launch's output is incomplete)",
    2: "a page-table entry lies outside the page pool (that page was read as slot 0), or a "
       "batch reindex named a slot or a row outside the pool (that slot or row was left as it was)",
}


class DeviceError(RazorKVError):
    """A device-side error that a decode kernel recorded in its workspace flag."""

    def __init__(self, code: int):
        self.code = code
        super().__init__(f"device error {code}: {DEVICE_ERRORS.get(code, 'unknown code')}")


def check(status: int, what: str):
    if status != 0:
        raise RazorKVError(f"{what}: {_STATUS.get(status, status)} (status {status})")


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float32:
        return F32
    if dt == torch.float16:
        return F16
    if dt == torch.bfloat16:
        return BF16
    raise TypeError(f"unsupported dtype {dt}; expected float32, float16 or bfloat16")


def stream_ptr(device) -> int:
    """Raw handle of torch's current stream on `device` (cheap: no Stream object)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    return torch._C._cuda_getCurrentRawStream(idx)


def require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError(
                "razorkv_b200 runs on CUDA tensors only; got a tensor on "
                f"{t.device} (there is no CPU path)")
