"""rkv_decode_attention_noalloc: decode attention for callers that cannot allocate (GPU).

Callers such as a framework that owns the whole device heap, or a decode loop that must not
enter the driver's allocator between steps, call the variant that takes no workspace; its
scratch is a fixed array inside the library.  These tests call it through the C ABI twice in
a row (the second call finds the first call's leftovers in the shared array) and compare each
result with rkv_decode_attention given its own workspace, within the tolerance of the dtype.
The file is named to run last so that a run stopping at the first failure has already run
every other test.
"""

import numpy as np
import pytest
import torch

from razorkv_b200 import _lib
from razorkv_b200._lib import KVLayout, Output, Query, dtype_code
from razorkv_b200.kernels import Workspace

pytestmark = pytest.mark.gpu

TOL = {torch.bfloat16: (2e-2, 1e-2), torch.float32: (1e-5, 1e-5)}


def _paged_case(B, Hq, Hkv, D, N, P, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    n_pages = (N + P - 1) // P
    slots = n_pages + 5
    kpool = torch.randn(slots, B, Hkv, P, D, generator=g).to(dtype).cuda()
    vpool = torch.randn(slots, B, Hkv, P, D, generator=g).to(dtype).cuda()
    pt = torch.randperm(slots, generator=g)[:n_pages].to(torch.int64).cuda()
    q = torch.randn(B, Hq, 1, D, generator=g).to(dtype).cuda()
    lay = KVLayout(kpool.data_ptr(), vpool.data_ptr(), dtype_code(dtype), D, B, Hkv,
                   kpool.stride(1), kpool.stride(2), kpool.stride(0), kpool.stride(3), P, slots,
                   pt.data_ptr(), 0, N)
    return (kpool, vpool, pt, q), lay


def _query(q):
    return Query(q.data_ptr(), dtype_code(q.dtype), q.shape[1], q.shape[2], q.stride(0),
                 q.stride(1), q.stride(2))


def _output(o):
    return Output(o.data_ptr(), dtype_code(o.dtype), 0, o.stride(0), o.stride(1), o.stride(2))


@pytest.mark.parametrize("B,Hq,Hkv,D,N,P,dtype", [
    (8, 32, 8, 128, 3000, 16, torch.bfloat16),   # sm_100a fused kernel + merge
    (1, 28, 4, 128, 9001, 16, torch.bfloat16),   # GQA 7, many partials per sequence
    (2, 8, 2, 64, 777, 5, torch.float32),        # shape-general kernels (page size 5, fp32)
])
def test_noalloc_matches_workspace_entry_point(B, Hq, Hkv, D, N, P, dtype):
    lib = _lib.load()
    keep, lay = _paged_case(B, Hq, Hkv, D, N, P, dtype, seed=N)
    q = keep[3]
    qs = _query(q)
    stream = torch.cuda.current_stream().cuda_stream
    ref = torch.empty_like(q)
    ws = Workspace.get(q.device, lib.rkv_decode_attention_workspace_size(qs, lay))
    assert lib.rkv_decode_attention(qs, lay, 0.0, 0, _output(ref), ws.data_ptr(), ws.numel(),
                                    stream) == 0
    atol, rtol = TOL[dtype]
    for _ in range(2):   # the second call starts from the first call's scratch contents
        out = torch.full_like(q, float("nan"))
        assert lib.rkv_decode_attention_noalloc(qs, lay, 0.0, 0, _output(out), stream) == 0
        torch.cuda.synchronize()
        np.testing.assert_allclose(out.float().cpu().numpy(), ref.float().cpu().numpy(),
                                   atol=atol, rtol=rtol)


def test_noalloc_rejects_oversized_request():
    """A request whose scratch would exceed the fixed array fails with the workspace status
    and launches nothing."""
    lib = _lib.load()
    B, Hq, Hkv, QL, N, D = 64, 64, 8, 16, 4096, 256
    k = torch.zeros(B, Hkv, N, D, device="cuda")
    q = torch.zeros(B, Hq, QL, D, device="cuda")
    lay = KVLayout(k.data_ptr(), k.data_ptr(), dtype_code(k.dtype), D, B, Hkv, k.stride(0),
                   k.stride(1), 0, k.stride(2), 1, 0, None, 0, N)
    qs = _query(q)
    assert lib.rkv_decode_attention_workspace_size(qs, lay) > (16 << 20)
    out = torch.zeros_like(q)
    before = lib.rkv_launch_count()
    st = lib.rkv_decode_attention_noalloc(qs, lay, 0.0, 0, _output(out),
                                          torch.cuda.current_stream().cuda_stream)
    assert st == 3   # RKV_ERR_WORKSPACE_TOO_SMALL
    assert lib.rkv_launch_count() == before
