"""The ctypes binding printed in INTEGRATION.md section 2, run as printed (GPU).

A maintainer of the reference routes the CUDA branch of
``razorkv.kernels.triton_paged_sparse.triton_paged_sparse_attention``
(razorkv/kernels/triton_paged_sparse.py:141-174) to this library by pasting that stub and
calling ``_paged_attention_cuda(query, key_paged, value_paged, page_table, scale)`` where the
Triton launch was.  This test extracts the stub's code block from INTEGRATION.md, executes it
with only the library path filled in, and runs it on the case of the reference's own paged
attention test (razorkv tests/test_kernels.py:49-82: batch 2, 4 query / 2 kv heads, 6 pages
of 8 tokens, head_dim 32, page table [[0, 2, 4], [1, 3, 5]], fp32, tolerance 1e-5) and on a
bf16 case of the cache's page shape (16-token pages, head_dim 128: the sm_100a kernel).
The expected output is the reference test's own recipe: gather the listed pages per
sequence, then softmax(q.k / sqrt(D)).v with each kv head serving G query heads.
"""

import os
import re

import pytest
import torch

from razorkv_b200 import _lib

pytestmark = pytest.mark.gpu

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))


def _stub():
    with open(os.path.join(ROOT, "INTEGRATION.md")) as f:
        text = f.read()
    blocks = re.findall(r"```python\n(.*?)```", text, flags=re.S)
    code = [b for b in blocks if "_paged_attention_cuda" in b]
    assert len(code) == 1, "INTEGRATION.md must print exactly one ctypes stub"
    src = code[0].replace('ctypes.CDLL("librazorkv_b200.so")', f'ctypes.CDLL({_lib.LIB_PATH!r})')
    ns = {}
    exec(compile(src, "INTEGRATION.md:stub", "exec"), ns)
    return ns["_paged_attention_cuda"]


def _expected(q, k_paged, v_paged, page_table, scale=None):
    B, H, _, D = q.shape
    Hkv = k_paged.shape[1]
    G = H // Hkv
    ks = torch.stack([k_paged[b][:, page_table[b]].reshape(Hkv, -1, D) for b in range(B)])
    vs = torch.stack([v_paged[b][:, page_table[b]].reshape(Hkv, -1, D) for b in range(B)])
    ks = ks.double().repeat_interleave(G, dim=1)
    vs = vs.double().repeat_interleave(G, dim=1)
    s = (q.double() @ ks.transpose(-1, -2)) * (scale if scale else D ** -0.5)
    return torch.softmax(s, dim=-1) @ vs


@pytest.mark.parametrize("dtype,P,D,maxp,pt,atol,rtol", [
    (torch.float32, 8, 32, 6, [[0, 2, 4], [1, 3, 5]], 1e-5, 1e-5),
    (torch.bfloat16, 16, 128, 40, [[3, 7, 11, 0, 39, 20], [1, 2, 5, 8, 13, 21]], 2e-2, 1e-2),
])
def test_stub_runs_the_reference_paged_attention_case(dtype, P, D, maxp, pt, atol, rtol):
    run = _stub()
    g = torch.Generator().manual_seed(P * 100 + D)
    B, H, Hkv = 2, 4, 2
    q = torch.randn(B, H, 1, D, generator=g).to(dtype)
    kp = torch.randn(B, Hkv, maxp, P, D, generator=g).to(dtype)
    vp = torch.randn(B, Hkv, maxp, P, D, generator=g).to(dtype)
    table = torch.tensor(pt, dtype=torch.long)
    out = run(q.cuda(), kp.cuda(), vp.cuda(), table.cuda())
    assert out.shape == (B, H, 1, D) and out.dtype == dtype
    ref = _expected(q, kp, vp, table)
    torch.testing.assert_close(out.double().cpu(), ref, atol=atol, rtol=rtol)
    # an explicit scale is passed through
    out2 = run(q.cuda(), kp.cuda(), vp.cuda(), table.cuda(), scale=0.05)
    torch.testing.assert_close(out2.double().cpu(), _expected(q, kp, vp, table, 0.05),
                               atol=atol, rtol=rtol)
