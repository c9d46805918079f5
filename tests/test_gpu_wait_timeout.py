"""Failure detection without a GPU fault: every spin in the kernels is a bounded wait that
gives up, sets an error flag the host reads and lets the CTA finish.  The self-test waits on
a barrier nothing arrives on with a ~1 ms limit; afterwards the context still runs a decode."""

import pytest
import torch

from razorkv_b200 import _lib
from razorkv_b200._lib import KVLayout, Output, Query, dtype_code
from razorkv_b200.kernels import Workspace

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_reports():
    lib = _lib.load()
    result = torch.zeros(3, dtype=torch.int32, device="cuda")
    st = lib.rkv_selftest_wait_timeout(result.data_ptr(), 2_000_000,
                                       torch.cuda.current_stream().cuda_stream)
    assert st == 0
    torch.cuda.synchronize()
    assert result.cpu().tolist() == [1, 0, 1]
    assert lib.rkv_selftest_wait_timeout(result.data_ptr(), 0, None) != 0   # rejected limit

    # the context is intact: a decode attention launch right after runs and is error-free
    B, Hq, Hkv, D, P, N = 2, 8, 2, 128, 16, 300
    slots = (N + P - 1) // P
    k = torch.randn(slots, B, Hkv, P, D, device="cuda", dtype=torch.bfloat16)
    v = torch.randn_like(k)
    pt = torch.arange(slots, device="cuda", dtype=torch.int64)
    q = torch.randn(B, Hq, 1, D, device="cuda", dtype=torch.bfloat16)
    out = torch.empty_like(q)
    lay = KVLayout(k.data_ptr(), v.data_ptr(), dtype_code(k.dtype), D, B, Hkv, k.stride(1),
                   k.stride(2), k.stride(0), k.stride(3), P, slots, pt.data_ptr(), 0, N)
    qs = Query(q.data_ptr(), dtype_code(q.dtype), Hq, 1, q.stride(0), q.stride(1), q.stride(2))
    os_ = Output(out.data_ptr(), dtype_code(out.dtype), 0, out.stride(0), out.stride(1), out.stride(2))
    ws = Workspace.get(q.device, lib.rkv_decode_attention_workspace_size(qs, lay))
    assert lib.rkv_decode_attention(qs, lay, 0.0, 0, os_, ws.data_ptr(), ws.numel(),
                                    torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    assert int(ws[:4].view(torch.int32)[0]) == 0
    assert torch.isfinite(out.float()).all()
