"""CUDA operators against the oracle (GPU).  Every call goes through the C ABI."""

import math

import numpy as np
import pytest
import torch

from oracle import razorkv_oracle as O
import razorkv_b200 as R
from razorkv_b200 import _lib
from razorkv_b200._lib import KVLayout, Query, Salience, dtype_code
from razorkv_b200.kernels import Workspace

pytestmark = pytest.mark.gpu

TOL = {torch.float32: (1e-5, 1e-5), torch.bfloat16: (2e-2, 1e-2), torch.float16: (2e-3, 1e-3)}


def _rand(*shape, dtype=torch.float32, seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g).to(dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(2, 4, 2, 1, 128, 64), (1, 8, 2, 1, 1216, 64),
                                   (3, 28, 4, 1, 777, 128), (2, 4, 4, 3, 50, 32),
                                   (1, 8, 1, 1, 5, 256)])
def test_compacted_paged_sdpa(dtype, shape):
    B, H, Hkv, QL, N, D = shape
    q, k, v = (_rand(B, H, QL, D, dtype=dtype, seed=1), _rand(B, Hkv, N, D, dtype=dtype, seed=2),
               _rand(B, Hkv, N, D, dtype=dtype, seed=3))
    out = R.compacted_paged_sdpa(q.cuda(), k.cuda(), v.cuda())
    ref = O.attention(q.float().numpy(), k.float().numpy(), v.float().numpy())
    atol, rtol = TOL[dtype]
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, atol=atol, rtol=rtol)
    assert out.dtype == dtype and out.shape == (B, H, QL, D)


def test_compacted_paged_sdpa_causal():
    q, k, v = _rand(1, 4, 6, 32, seed=4), _rand(1, 2, 6, 32, seed=5), _rand(1, 2, 6, 32, seed=6)
    out = R.compacted_paged_sdpa(q.cuda(), k.cuda(), v.cuda(), is_causal=True)
    ref = O.attention(q.numpy(), k.numpy(), v.numpy(), causal=True)
    np.testing.assert_allclose(out.cpu().numpy(), ref, atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_paged_sparse_attention_reference_case(dtype):
    # razorkv tests/test_kernels.py:49-82: page table [[0,2,4],[1,3,5]], page 8, D 32
    B, H, Hkv, MAXP, P, D = 2, 4, 2, 6, 8, 32
    q = _rand(B, H, 1, D, dtype=dtype, seed=7)
    kp = _rand(B, Hkv, MAXP, P, D, dtype=dtype, seed=8)
    vp = _rand(B, Hkv, MAXP, P, D, dtype=dtype, seed=9)
    pt = torch.tensor([[0, 2, 4], [1, 3, 5]], dtype=torch.long)
    out = R.triton_paged_sparse_attention(q.cuda(), kp.cuda(), vp.cuda(), pt.cuda())
    assert out.shape == (B, H, 1, D)
    ref = O.paged_attention(q.float().numpy(), kp.float().numpy(), vp.float().numpy(), pt.numpy())
    atol, rtol = TOL[dtype]
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, atol=atol, rtol=rtol)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("P,D,H,Hkv", [(16, 128, 32, 8), (16, 64, 8, 2), (16, 128, 28, 4)])
def test_paged_sparse_attention_pool_layout(dtype, P, D, H, Hkv):
    B, MAXP, n_active = 3, 40, 29
    q = _rand(B, H, 1, D, dtype=dtype, seed=10)
    kp = _rand(B, Hkv, MAXP, P, D, dtype=dtype, seed=11)
    vp = _rand(B, Hkv, MAXP, P, D, dtype=dtype, seed=12)
    g = torch.Generator().manual_seed(13)
    pt = torch.stack([torch.randperm(MAXP, generator=g)[:n_active] for _ in range(B)])
    out = R.triton_paged_sparse_attention(q.cuda(), kp.cuda(), vp.cuda(), pt.cuda())
    ref = O.paged_attention(q.float().numpy(), kp.float().numpy(), vp.float().numpy(), pt.numpy())
    atol, rtol = TOL[dtype]
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, atol=atol, rtol=rtol)


def test_paged_sparse_attention_errors():
    q = torch.zeros(1, 2, 2, 16, device="cuda")
    kp = torch.zeros(1, 1, 4, 8, 16, device="cuda")
    pt = torch.zeros(1, 2, dtype=torch.long, device="cuda")
    with pytest.raises(AssertionError):
        R.triton_paged_sparse_attention(q, kp, kp, pt)
    with pytest.raises(IndexError):
        R.triton_paged_sparse_attention(q[:, :, :1], kp, kp, pt + 7)
    with pytest.raises(RuntimeError):
        R.triton_paged_sparse_attention(q[:, :, :1].cpu(), kp.cpu(), kp.cpu(), pt.cpu())


def test_page_salience_pool_known_answer():
    # razorkv tests/test_kernels.py:35-46
    s = torch.tensor([[1.0, 5.0, 2.0, 3.0, 8.0, 2.0, 1.0, 4.0]], device="cuda")
    mx, n = R.compute_page_salience_pool(s, 4, "max")
    assert n == 2 and mx.cpu().tolist() == [[5.0, 8.0]]
    mn, n = R.compute_page_salience_pool(s, 4, "mean")
    assert n == 2 and torch.allclose(mn.cpu(), torch.tensor([[2.75, 3.75]]))
    sh, n = R.compute_page_salience_pool(s[:, :3], 4)
    assert n == 1 and sh.cpu().tolist() == [[5.0]]
    x = _rand(5, 1000, seed=14).cuda()
    mx, n = R.compute_page_salience_pool(x, 16)
    ref, rn = O.page_pool(x.cpu().numpy(), 16)
    assert n == rn and np.array_equal(mx.cpu().numpy(), ref)


def _contig_layout(k, v=None):
    B, Hkv, N, D = k.shape
    return KVLayout(k.data_ptr(), v.data_ptr() if v is not None else None, dtype_code(k.dtype), D,
                    B, Hkv, k.stride(0), k.stride(1), 0, k.stride(2), 1, 0, None, 0, N)


@pytest.mark.parametrize("dtype,D,Hq,Hkv,QL", [(torch.float32, 64, 8, 2, 1), (torch.bfloat16, 128, 32, 8, 1),
                                               (torch.bfloat16, 128, 28, 4, 1), (torch.float32, 32, 6, 3, 3),
                                               (torch.bfloat16, 20, 4, 2, 2)])
def test_score_bit_exact(dtype, D, Hq, Hkv, QL):
    B, N = 3, 517
    q = _rand(B, Hq, QL, D, dtype=dtype, seed=20)
    k = _rand(B, Hkv, N, D, dtype=dtype, seed=21)
    S0 = (torch.rand(B, N, generator=torch.Generator().manual_seed(22)) * 10).float()
    lib = _lib.load()
    qd, kd, Sd = q.cuda(), k.cuda(), S0.clone().cuda()
    qs = Query(qd.data_ptr(), dtype_code(dtype), Hq, QL, qd.stride(0), qd.stride(1), qd.stride(2))
    sal = Salience(Sd.data_ptr(), Sd.stride(0), 0)
    st = lib.rkv_score(qs, _contig_layout(kd), sal, 0.98, 1.0 - 0.98, 1,
                       torch.cuda.current_stream().cuda_stream)
    assert st == 0
    elt = torch.tensor([], dtype=dtype).element_size()
    R_ = O.resonance(q.float().numpy(), k.float().numpy(), elt)
    expect = O.ewma(S0.numpy(), R_, 0.98)
    got = Sd.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), expect.view(np.uint32))


@pytest.mark.parametrize("B,n,k", [(1, 222, 66), (8, 1400, 700), (2, 5, 5), (3, 8192, 1000),
                                   (1, 1, 1), (4, 3000, 1),
                                   # keys in shared memory up to 11264 pages, global above
                                   (1, 11264, 5000), (2, 11265, 3), (2, 20000, 7000)])
def test_select_pages_exact(B, n, k):
    g = torch.Generator().manual_seed(n + k)
    scores = (torch.randn(B, n, generator=g) * 2 + 10).float()
    # plant exact ties around the boundary
    scores[:, 3:9] = scores[:, 3:4]
    lib = _lib.load()
    sd = scores.cuda()
    kept = torch.empty(k, dtype=torch.int64, device="cuda")
    margin = torch.empty(1, device="cuda")
    ws = Workspace.get(sd.device, lib.rkv_select_pages_workspace_size(n))
    st = lib.rkv_select_pages(sd.data_ptr(), B, n, k, kept.data_ptr(), margin.data_ptr(),
                              ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)
    assert st == 0
    avg = O.batch_mean(scores.numpy())
    ek, em = O.canonical_topk(avg, k)
    assert kept.cpu().numpy().tolist() == ek.tolist()
    m = float(margin.cpu())
    assert (m == em) or (math.isinf(m) and math.isinf(em))


def test_select_pages_all_tied():
    lib = _lib.load()
    sd = torch.ones(2, 37, device="cuda")
    kept = torch.empty(10, dtype=torch.int64, device="cuda")
    ws = Workspace.get(sd.device, lib.rkv_select_pages_workspace_size(37))
    st = lib.rkv_select_pages(sd.data_ptr(), 2, 37, 10, kept.data_ptr(), None, ws.data_ptr(),
                              ws.numel(), torch.cuda.current_stream().cuda_stream)
    assert st == 0 and kept.cpu().tolist() == list(range(10))


def test_capi_rejects_bad_arguments():
    lib = _lib.load()
    s = torch.cuda.current_stream().cuda_stream
    assert lib.rkv_select_pages(None, 1, 4, 2, None, None, None, 0, s) == 1
    k = torch.zeros(1, 1, 4, 16, device="cuda")
    lay = _contig_layout(k, k)
    lay.head_dim = 512
    q = torch.zeros(1, 1, 1, 512, device="cuda")
    qs = Query(q.data_ptr(), 0, 1, 1, q.stride(0), q.stride(1), q.stride(2))
    assert lib.rkv_decode_attention(qs, lay, 0.0, 0, None, None, 0, s) == 2
    assert lib.rkv_compact_pages(None, 0, 1, None, 1, 1, 1, None, 0, s) == 1
