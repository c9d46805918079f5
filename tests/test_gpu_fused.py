"""The sm_100a fused decode kernel (score + attention in one pass) against the oracle (GPU).

A random page pool in the cache layout [slots, B, Hkv, 16, D] with a shuffled page table is
scored and attended through the C ABI; the salience must equal the oracle's canonical-order
EWMA bit for bit and the output must match fp64 attention within the bf16 tolerance.
"""

import numpy as np
import pytest
import torch

from oracle import razorkv_oracle as O
from razorkv_b200 import _lib
from razorkv_b200._lib import KVLayout, Output, Query, Salience, dtype_code
from razorkv_b200.kernels import Workspace

pytestmark = pytest.mark.gpu

P = 16


def _setup(B, Hq, Hkv, D, N, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    n_pages = (N + P - 1) // P
    slots = n_pages + 7
    kpool = torch.randn(slots, B, Hkv, P, D, generator=g).to(dtype)
    vpool = torch.randn(slots, B, Hkv, P, D, generator=g).to(dtype)
    spool = (torch.rand(slots, B, P, generator=g) * 10 + 1).float()
    pt = torch.randperm(slots, generator=g)[:n_pages].to(torch.int64)
    q = torch.randn(B, Hq, 1, D, generator=g).to(dtype)
    return kpool, vpool, spool, pt, q


def _logical(pool, pt, N):
    # [slots, B, Hkv, P, D] -> [B, Hkv, N, D] in logical token order
    x = pool[pt].permute(1, 2, 0, 3, 4).reshape(pool.shape[1], pool.shape[2], -1, pool.shape[4])
    return x[:, :, :N]


def _sal_logical(spool, pt, N):
    return spool[pt].permute(1, 0, 2).reshape(spool.shape[1], -1)[:, :N]


def _layout(kd, vd, ptd, N):
    return KVLayout(kd.data_ptr(), vd.data_ptr() if vd is not None else None, dtype_code(kd.dtype),
                    kd.shape[4], kd.shape[1], kd.shape[2], kd.stride(1), kd.stride(2), kd.stride(0),
                    kd.stride(3), P, kd.shape[0], ptd.data_ptr(), 0, N)


SHAPES = [
    # B, Hq, Hkv, D, N
    (8, 32, 8, 128, 1000),     # Llama-8B-like heads, ragged last page
    (1, 28, 4, 128, 5003),     # Qwen-like GQA 7 (padded to 8 heads per kv head)
    (2, 64, 8, 128, 777),      # GQA 8
    (3, 8, 2, 128, 64),        # 2 kv heads, 4 tiles per stage
    (2, 4, 1, 128, 300),       # 1 kv head, 8 tiles per stage
    (4, 16, 4, 64, 513),       # head_dim 64
    (1, 8, 8, 128, 16),        # one page, G = 1
    (5, 40, 8, 128, 3),        # fewer tokens than a page
    (2, 6, 2, 128, 900),       # G = 3: the second query-head slice has one live head
    (3, 16, 8, 128, 1500),     # G = 2
    (2, 16, 2, 64, 700),       # G = 8 over 2 kv heads: query heads split over two warps
    (3, 6, 1, 128, 333),       # G = 6, 1 kv head: split, second warp with 2 live heads
    # a CTA on every SM, CTA ranges crossing sequence boundaries, tens of partials a row
    (4, 32, 8, 128, 2000),     # ~37 partials a row
    (8, 16, 4, 64, 4000),      # head_dim 64, 2 tiles per stage
    (16, 8, 8, 128, 700),      # G = 1, 16 sequences
    # batch 1, hundreds of partials a row: the merge spreads each row over a CTA cluster
    (1, 16, 2, 64, 20000),     # ~560 partials a row: clusters of 8
    (1, 28, 4, 128, 20000),    # ~280 partials a row: clusters of 7
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,Hq,Hkv,D,N", SHAPES)
def test_fused_matches_oracle(B, Hq, Hkv, D, N, dtype):
    kpool, vpool, spool, pt, q = _setup(B, Hq, Hkv, D, N, dtype, seed=B * 131 + N)
    kd, vd, sd, ptd, qd = (t.cuda() for t in (kpool, vpool, spool, pt, q))
    out = torch.empty_like(qd)
    lib = _lib.load()
    lay = _layout(kd, vd, ptd, N)
    qs = Query(qd.data_ptr(), dtype_code(dtype), Hq, 1, qd.stride(0), qd.stride(1), qd.stride(2))
    os_ = Output(out.data_ptr(), dtype_code(dtype), 0, out.stride(0), out.stride(1), out.stride(2))
    sal = Salience(sd.data_ptr(), sd.stride(1), sd.stride(0))
    ws = Workspace.get(qd.device, lib.rkv_decode_fused_workspace_size(qs, lay))
    st = lib.rkv_decode_fused(qs, lay, sal, 0.98, 1.0 - 0.98, 0.0, os_, ws.data_ptr(), ws.numel(),
                              torch.cuda.current_stream().cuda_stream)
    assert st == 0
    torch.cuda.synchronize()
    assert int(ws[:4].view(torch.int32)[0]) == 0, "device wait gave up"
    K = _logical(kpool, pt, N).float().numpy()
    V = _logical(vpool, pt, N).float().numpy()
    S0 = _sal_logical(spool, pt, N).numpy()
    R = O.resonance(q.float().numpy(), K, 2)
    expect_S = O.ewma(S0, R, 0.98)
    got_S = _sal_logical(sd.cpu(), pt, N).numpy()
    assert np.array_equal(got_S.view(np.uint32), expect_S.view(np.uint32))
    # salience of slots outside the table is untouched
    untouched = torch.ones(spool.shape[0], dtype=torch.bool)
    untouched[pt] = False
    assert torch.equal(sd.cpu()[untouched], spool[untouched])
    ref = O.attention(q.float().numpy(), K, V)
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, atol=2e-2, rtol=1e-2)
    # counters returned to zero
    assert int(ws[256:256 + 4 * B].view(torch.int32).abs().sum()) == 0


@pytest.mark.parametrize("B,Hq,Hkv,D,N", SHAPES[:4])
def test_fast_score_only_matches_oracle(B, Hq, Hkv, D, N):
    kpool, vpool, spool, pt, q = _setup(B, Hq, Hkv, D, N, torch.bfloat16, seed=7 + N)
    kd, sd, ptd, qd = (t.cuda() for t in (kpool, spool, pt, q))
    lib = _lib.load()
    lay = _layout(kd, None, ptd, N)
    qs = Query(qd.data_ptr(), dtype_code(torch.bfloat16), Hq, 1, qd.stride(0), qd.stride(1), qd.stride(2))
    sal = Salience(sd.data_ptr(), sd.stride(1), sd.stride(0))
    st = lib.rkv_score(qs, lay, sal, 0.98, 1.0 - 0.98, 1, torch.cuda.current_stream().cuda_stream)
    assert st == 0
    K = _logical(kpool, pt, N).float().numpy()
    expect_S = O.ewma(_sal_logical(spool, pt, N).numpy(), O.resonance(q.float().numpy(), K, 2), 0.98)
    got_S = _sal_logical(sd.cpu(), pt, N).numpy()
    assert np.array_equal(got_S.view(np.uint32), expect_S.view(np.uint32))


def test_fused_repeated_launches_are_stable():
    """Counters self-reset: back-to-back launches give identical outputs."""
    B, Hq, Hkv, D, N = 8, 32, 8, 128, 4000
    kpool, vpool, spool, pt, q = _setup(B, Hq, Hkv, D, N, torch.bfloat16, seed=99)
    kd, vd, ptd, qd = (t.cuda() for t in (kpool, vpool, pt, q))
    lib = _lib.load()
    lay = _layout(kd, vd, ptd, N)
    qs = Query(qd.data_ptr(), dtype_code(torch.bfloat16), Hq, 1, qd.stride(0), qd.stride(1), qd.stride(2))
    outs = []
    for _ in range(3):
        out = torch.empty_like(qd)
        os_ = Output(out.data_ptr(), dtype_code(torch.bfloat16), 0, out.stride(0), out.stride(1), out.stride(2))
        ws = Workspace.get(qd.device, lib.rkv_decode_attention_workspace_size(qs, lay))
        st = lib.rkv_decode_attention(qs, lay, 0.0, 0, os_, ws.data_ptr(), ws.numel(),
                                      torch.cuda.current_stream().cuda_stream)
        assert st == 0
        outs.append(out)
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,Hq,Hkv,D,N", SHAPES)
def test_attention_only_matches_oracle(B, Hq, Hkv, D, N, dtype):
    """rkv_decode_attention on the fast path: logits on tensor cores, no scoring."""
    kpool, vpool, spool, pt, q = _setup(B, Hq, Hkv, D, N, dtype, seed=B * 17 + N)
    kd, vd, ptd, qd = (t.cuda() for t in (kpool, vpool, pt, q))
    out = torch.empty_like(qd)
    lib = _lib.load()
    lay = _layout(kd, vd, ptd, N)
    qs = Query(qd.data_ptr(), dtype_code(dtype), Hq, 1, qd.stride(0), qd.stride(1), qd.stride(2))
    os_ = Output(out.data_ptr(), dtype_code(dtype), 0, out.stride(0), out.stride(1), out.stride(2))
    ws = Workspace.get(qd.device, lib.rkv_decode_attention_workspace_size(qs, lay))
    assert lib.rkv_decode_attention(qs, lay, 0.0, 0, os_, ws.data_ptr(), ws.numel(),
                                    torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    assert int(ws[:4].view(torch.int32)[0]) == 0
    ref = O.attention(q.float().numpy(), _logical(kpool, pt, N).float().numpy(),
                      _logical(vpool, pt, N).float().numpy())
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, atol=2e-2, rtol=1e-2)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,Hq,Hkv,D,N", SHAPES)
def test_scored_matches_oracle(B, Hq, Hkv, D, N, dtype):
    """rkv_decode_scored (the HF hook step): the salience of the tokens before score_tokens
    takes the EWMA of q_score's resonance bit for bit, later tokens keep theirs, and the
    output is q_attn's attention over every token."""
    kpool, vpool, spool, pt, q = _setup(B, Hq, Hkv, D, N, dtype, seed=B * 29 + N)
    q_attn = torch.randn(B, Hq, 1, D, generator=torch.Generator().manual_seed(N)).to(dtype)
    score_tokens = max(0, N - 1 - N % 3)
    kd, vd, sd, ptd, qd, qad = (t.cuda() for t in (kpool, vpool, spool, pt, q, q_attn))
    out = torch.empty_like(qd)
    lib = _lib.load()
    lay = _layout(kd, vd, ptd, N)
    mk = lambda t: Query(t.data_ptr(), dtype_code(dtype), Hq, 1, t.stride(0), t.stride(1), t.stride(2))
    qs, qas = mk(qd), mk(qad)
    os_ = Output(out.data_ptr(), dtype_code(dtype), 0, out.stride(0), out.stride(1), out.stride(2))
    sal = Salience(sd.data_ptr(), sd.stride(1), sd.stride(0))
    ws = Workspace.get(qd.device, lib.rkv_decode_scored_workspace_size(qas, lay))
    assert lib.rkv_decode_scored(qs, qas, lay, sal, score_tokens, 0.98, 1.0 - 0.98, 0.0, os_,
                                 ws.data_ptr(), ws.numel(),
                                 torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    assert int(ws[:4].view(torch.int32)[0]) == 0
    K = _logical(kpool, pt, N).float().numpy()
    V = _logical(vpool, pt, N).float().numpy()
    S0 = _sal_logical(spool, pt, N).numpy()
    expect_S = S0.copy()
    if score_tokens:
        R = O.resonance(q.float().numpy(), K[:, :, :score_tokens], 2)
        expect_S[:, :score_tokens] = O.ewma(S0[:, :score_tokens], R, 0.98)
    got_S = _sal_logical(sd.cpu(), pt, N).numpy()
    assert np.array_equal(got_S.view(np.uint32), expect_S.view(np.uint32))
    ref = O.attention(q_attn.float().numpy(), K, V)
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, atol=2e-2, rtol=1e-2)


def _tied_queries(q, Hkv, kind, seed):
    """Query heads of each kv group made (nearly) equal, so that several heads of a token
    fall inside the tensor-core screen's error window and take the canonical recompute."""
    B, Hq, _, D = q.shape
    G = Hq // Hkv
    g = torch.Generator().manual_seed(seed)
    base = q.float().view(B, Hkv, G, 1, D)[:, :, :1].expand(B, Hkv, G, 1, D).clone()
    if kind == "tied":          # identical heads: every head is a candidate
        x = base
    elif kind == "near":        # heads one bf16 step apart in a few dimensions
        x = base.clone()
        bump = (torch.rand(B, Hkv, G, 1, D, generator=g) < 0.03).float()
        x = x + bump * x.abs().clamp(min=1e-2) * (2.0 ** -7)
    else:                       # "scaled": heads differ by powers of two
        x = base * (2.0 ** torch.arange(G, dtype=torch.float32)).view(1, 1, G, 1, 1)
    return x.reshape(B, Hq, 1, D).to(q.dtype)


@pytest.mark.parametrize("kind", ["tied", "near", "scaled"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,Hq,Hkv,D,N", [(1, 28, 4, 128, 5003), (2, 64, 8, 128, 777),
                                          (3, 6, 1, 128, 333), (2, 16, 2, 64, 700)])
def test_screened_resonance_with_tied_heads(B, Hq, Hkv, D, N, dtype, kind):
    """5-8 query heads per kv head: the resonance comes from a tensor-core screen plus the
    canonical dot of the candidate heads; with (nearly) tied heads many tokens have several
    candidates and the salience must still equal the canonical max bit for bit."""
    kpool, vpool, spool, pt, q = _setup(B, Hq, Hkv, D, N, dtype, seed=B * 7 + N)
    q = _tied_queries(q, Hkv, kind, seed=N)
    kd, vd, sd, ptd, qd = (t.cuda() for t in (kpool, vpool, spool, pt, q))
    out = torch.empty_like(qd)
    lib = _lib.load()
    lay = _layout(kd, vd, ptd, N)
    qs = Query(qd.data_ptr(), dtype_code(dtype), Hq, 1, qd.stride(0), qd.stride(1), qd.stride(2))
    os_ = Output(out.data_ptr(), dtype_code(dtype), 0, out.stride(0), out.stride(1), out.stride(2))
    sal = Salience(sd.data_ptr(), sd.stride(1), sd.stride(0))
    ws = Workspace.get(qd.device, lib.rkv_decode_fused_workspace_size(qs, lay))
    assert lib.rkv_decode_fused(qs, lay, sal, 0.98, 1.0 - 0.98, 0.0, os_, ws.data_ptr(),
                                ws.numel(), torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    assert int(ws[:4].view(torch.int32)[0]) == 0
    K = _logical(kpool, pt, N).float().numpy()
    V = _logical(vpool, pt, N).float().numpy()
    expect_S = O.ewma(_sal_logical(spool, pt, N).numpy(), O.resonance(q.float().numpy(), K, 2), 0.98)
    got_S = _sal_logical(sd.cpu(), pt, N).numpy()
    assert np.array_equal(got_S.view(np.uint32), expect_S.view(np.uint32))
    ref = O.attention(q.float().numpy(), K, V)
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, atol=2e-2, rtol=1e-2)
