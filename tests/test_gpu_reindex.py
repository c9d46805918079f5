"""rkv_reindex_batch through the C ABI: the batch reindex behind reorder_cache,
batch_select_indices and batch_repeat_interleave (razorkv/cache.py:198-229) on the live slots
of a cache pool, checked bit for bit against torch's index_select of the same pool."""

import numpy as np
import pytest
import torch

from razorkv_b200 import PagedRazorKVCache, RazorConfig, _lib
from razorkv_b200._lib import KVLayout, Salience, dtype_code, stream_ptr
from razorkv_b200.kernels import Workspace

pytestmark = pytest.mark.gpu


def _pool(slots, B, Hkv, P, D, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    k = torch.randn(slots, B, Hkv, P, D, generator=g).to(dtype).cuda()
    v = torch.randn(slots, B, Hkv, P, D, generator=g).to(dtype).cuda()
    s = torch.randn(slots, B, P, generator=g).cuda()
    return k, v, s


def _layout(k, v, row_map=None):
    slots, B, Hkv, P, D = k.shape
    return KVLayout(k.data_ptr(), v.data_ptr(), dtype_code(k.dtype), D, B, Hkv, k.stride(1),
                    k.stride(2), k.stride(0), k.stride(3), P, slots, None, 0, 0,
                    row_map.data_ptr() if row_map is not None else None)


def _sal(s):
    return Salience(s.data_ptr(), s.stride(1), s.stride(0))


def _flag():
    f = Workspace._flag(Workspace.get(torch.device("cuda", torch.cuda.current_device()), 1 << 20))
    f.zero_()
    return f


def _reindex(src, dst, index, slots, flag=None, row_map=None, num_moved=None):
    lib = _lib.load()
    idx = torch.as_tensor(index, dtype=torch.int64).cuda()
    sl = torch.as_tensor(slots, dtype=torch.int64).cuda()
    moved = sl.numel() if num_moved is None else num_moved
    st = lib.rkv_reindex_batch(_layout(*src[:2], row_map), _sal(src[2]),
                               _layout(*dst[:2], row_map if dst is src else None), _sal(dst[2]),
                               idx.data_ptr(), sl.data_ptr(), sl.numel(), moved,
                               flag.data_ptr() if flag is not None else None,
                               stream_ptr(torch.device("cuda")))
    torch.cuda.synchronize()
    return st


def _expected(before, index, slots):
    exp = [t.clone() for t in before]
    sl = torch.as_tensor(slots, dtype=torch.int64).cuda()
    idx = torch.as_tensor(index, dtype=torch.int64).cuda()
    for e, b in zip(exp, before):
        e[sl] = b[sl].index_select(1, idx)
    return exp


SHAPES = [
    # slots, B, Hkv, P, D, dtype         (access width the call picks)
    (40, 8, 8, 16, 128, torch.bfloat16),   # 16-byte rows
    (33, 5, 2, 5, 64, torch.float32),      # 20-byte salience rows: 4-byte accesses
    (17, 3, 1, 5, 3, torch.bfloat16),      # 30-byte K rows: 2-byte accesses
    (12, 64, 8, 16, 128, torch.bfloat16),  # batch 64: 512-byte chunks
]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s[:5])) + str(s[5])[-4:])
def test_in_place_permutation_matches_index_select(shape):
    slots, B, Hkv, P, D, dt = shape
    rng = np.random.default_rng(slots * B)
    pool = _pool(slots, B, Hkv, P, D, dt, seed=B)
    live = rng.permutation(slots)[: (2 * slots) // 3]
    for index in (rng.permutation(B), rng.integers(0, B, size=B), np.arange(B),
                  np.concatenate([[B - 1], np.arange(B - 1)])):
        before = [t.clone() for t in pool]
        exp = _expected(before, index, live)
        flag = _flag()
        assert _reindex(pool, pool, index, live, flag) == 0
        assert int(flag.item()) == 0
        for got, want in zip(pool, exp):
            assert torch.equal(got, want)


@pytest.mark.parametrize("new_rows", ["repeat3", "select2", "expand_one"])
def test_gather_into_new_batch(new_rows):
    slots, B, Hkv, P, D, dt = 30, 4, 4, 16, 128, torch.bfloat16
    src = _pool(slots, B, Hkv, P, D, dt, seed=7)
    index = {"repeat3": np.repeat(np.arange(B), 3), "select2": np.array([3, 1]),
             "expand_one": np.zeros(9, dtype=np.int64)}[new_rows]
    nb = len(index)
    dst = [torch.zeros(slots, nb, Hkv, P, D, dtype=dt, device="cuda"),
           torch.zeros(slots, nb, Hkv, P, D, dtype=dt, device="cuda"),
           torch.zeros(slots, nb, P, device="cuda")]
    live = list(range(0, slots, 2))
    before = [t.clone() for t in src]
    assert _reindex(src, dst, index, live) == 0
    idx = torch.as_tensor(index).cuda()
    sl = torch.as_tensor(live).cuda()
    for got, s0, s1 in zip(dst, before, src):
        assert torch.equal(s1, s0)   # source untouched
        assert torch.equal(got[sl], s0[sl].index_select(1, idx))
        rest = torch.ones(slots, dtype=torch.bool, device="cuda")
        rest[sl] = False
        assert torch.count_nonzero(got[rest]) == 0   # unlisted slots not written


def test_out_of_range_index_and_slot_set_the_flag():
    slots, B, Hkv, P, D, dt = 10, 4, 2, 16, 64, torch.bfloat16
    pool = _pool(slots, B, Hkv, P, D, dt, seed=3)
    before = [t.clone() for t in pool]
    flag = _flag()
    # row 1 names a row outside the batch: it keeps its contents, the others move
    assert _reindex(pool, pool, [2, 9, 0, 3], [1, 4], flag) == 0
    assert int(flag.item()) == 2
    exp = _expected(before, [2, 1, 0, 3], [1, 4])
    for got, want in zip(pool, exp):
        assert torch.equal(got, want)
    flag.zero_()
    before = [t.clone() for t in pool]
    assert _reindex(pool, pool, [1, 0, 2, 3], [slots + 5, 2], flag) == 0
    assert int(flag.item()) == 2
    exp = _expected(before, [1, 0, 2, 3], [2])
    for got, want in zip(pool, exp):
        assert torch.equal(got, want)
    flag.zero_()


def test_rejected_calls_launch_nothing():
    lib = _lib.load()
    k, v, s = _pool(4, 2, 1, 16, 64, torch.bfloat16, seed=1)
    k2, v2, s2 = _pool(4, 2, 1, 16, 64, torch.bfloat16, seed=2)
    idx = torch.zeros(2, dtype=torch.int64, device="cuda")
    sl = torch.zeros(1, dtype=torch.int64, device="cuda")
    n0 = lib.rkv_launch_count()
    # K in place but V not
    bad = _layout(k, v2)
    assert lib.rkv_reindex_batch(_layout(k, v), _sal(s), bad, _sal(s2), idx.data_ptr(),
                                 sl.data_ptr(), 1, 1, None, None) == 1
    # non-contiguous (slot, sequence) planes
    lay = _layout(k, v)
    lay.stride_h = lay.stride_h * 2
    assert lib.rkv_reindex_batch(lay, _sal(s), _layout(k2, v2), _sal(s2), idx.data_ptr(),
                                 sl.data_ptr(), 1, 1, None, None) == 2
    # a destination batch too large for the staging buffer
    big = _layout(k2, v2)
    big.batch = 100000
    assert lib.rkv_reindex_batch(_layout(k, v), _sal(s), big, _sal(s2), idx.data_ptr(),
                                 sl.data_ptr(), 1, 1, None, None) == 2
    assert lib.rkv_launch_count() == n0


def test_cache_reorder_touches_live_pages_only():
    """reorder_cache keeps the pool tensors (in place); batch_repeat_interleave builds a new
    pool whose live pages hold the repeated rows."""
    rc = RazorConfig(compression_ratio=0.3, sink_tokens=32, local_window=64, page_size=16,
                     pyramid_mode="uniform")
    cache = PagedRazorKVCache(rc, 2)
    g = torch.Generator().manual_seed(11)
    for l in range(2):
        k = torch.randn(3, 2, 500, 64, generator=g).to(torch.bfloat16).cuda()
        v = torch.randn(3, 2, 500, 64, generator=g).to(torch.bfloat16).cuda()
        cache.update(k, v, l, {"query_states": torch.randn(3, 4, 1, 64, generator=g)
                               .to(torch.bfloat16).cuda()})
    K0 = [cache.key_cache[l].clone() for l in range(2)]
    S0 = [cache.salience_scores[l].clone() for l in range(2)]
    ptr = cache._k.data_ptr()
    pool0 = cache._k.clone()
    full = torch.cat([cache.page_table(l)[:-1] for l in range(2)])
    cache.reorder_cache(torch.tensor([2, 2, 0]))
    assert cache._k.data_ptr() == ptr
    # full pages keep their K (only the row map changed); the salience moved
    assert torch.equal(cache._k[full], pool0[full])
    assert torch.equal(cache._rowmap[full].cpu(), torch.tensor([[2, 2, 0]] * full.numel(),
                                                               dtype=torch.int32))
    for l in range(2):
        assert torch.equal(cache.key_cache[l], K0[l][[2, 2, 0]])
        assert torch.equal(cache.salience_scores[l], S0[l][[2, 2, 0]])
    cache.batch_repeat_interleave(2)
    assert cache.batch_size == 6
    for l in range(2):
        assert torch.equal(cache.key_cache[l], K0[l][[2, 2, 2, 2, 0, 0]])
    cache.check_errors()


def test_row_map_moves_listed_pages_and_rewrites_the_rest():
    """In place with a row map: the first num_moved slots get their K/V rows gathered through
    the map (and identity entries); the others keep K/V and compose their map entries; the
    salience of every listed slot moves."""
    slots, B, Hkv, P, D, dt = 24, 6, 2, 16, 128, torch.bfloat16
    rng = np.random.default_rng(5)
    pool = _pool(slots, B, Hkv, P, D, dt, seed=4)
    rm0 = torch.as_tensor(rng.integers(0, B, size=(slots, B)), dtype=torch.int32).cuda()
    rm = rm0.clone()
    live = rng.permutation(slots)[:15]
    moved, kept = live[:4], live[4:]
    index = rng.integers(0, B, size=B)
    before = [t.clone() for t in pool]
    flag = _flag()
    assert _reindex(pool, pool, index, live, flag, row_map=rm, num_moved=len(moved)) == 0
    assert int(flag.item()) == 0
    k0, v0, s0 = before
    idx = torch.as_tensor(index).cuda()
    for sl in moved:
        rows = rm0[sl].long()[idx]
        assert torch.equal(pool[0][sl], k0[sl][rows])
        assert torch.equal(pool[1][sl], v0[sl][rows])
        assert torch.equal(rm[sl].cpu(), torch.arange(B, dtype=torch.int32))
    for sl in kept:
        assert torch.equal(pool[0][sl], k0[sl]) and torch.equal(pool[1][sl], v0[sl])
        assert torch.equal(rm[sl], rm0[sl][idx])
    for sl in live:
        assert torch.equal(pool[2][sl], s0[sl][idx])
    rest = np.setdiff1d(np.arange(slots), live)
    for t, t0 in zip(pool, before):
        assert torch.equal(t[rest], t0[rest])
    assert torch.equal(rm[rest], rm0[rest])
    # out of place through the map: the new pool holds the mapped rows as its own rows
    dst = [torch.zeros(slots, 3, Hkv, P, D, dtype=dt, device="cuda"),
           torch.zeros(slots, 3, Hkv, P, D, dtype=dt, device="cuda"),
           torch.zeros(slots, 3, P, device="cuda")]
    assert _reindex(pool, dst, [5, 0, 5], live, row_map=rm) == 0
    sel = torch.tensor([5, 0, 5]).cuda()
    for sl in live:
        rows = rm[sl].long()[sel]
        assert torch.equal(dst[0][sl], pool[0][sl][rows])
        assert torch.equal(dst[2][sl], pool[2][sl][sel])


@pytest.mark.parametrize("Hq", [8, 14], ids=["gqa4", "gqa7_screened"])
def test_beam_search_on_shared_pages_matches_oracle(Hq):
    """reorder_cache as a page-table update across decode steps, compactions and a crop: the
    cache keeps the oracle's K, V and salience (the oracle copies rows) bit for bit, on the
    4-head instance and on the screened instance of 5-8 query heads per kv head."""
    from oracle import razorkv_oracle as O
    layers, B, Hkv, D = 2, 4, 2, 128
    dt = torch.bfloat16
    rc = RazorConfig(compression_ratio=0.30, sink_tokens=32, local_window=64, page_size=16,
                     pyramid_mode="uniform")
    cache = PagedRazorKVCache(rc, layers)
    oc = O.OracleCache(O.OracleConfig(compression_ratio=0.30, sink_tokens=32, local_window=64,
                                      page_size=16, pyramid_mode="uniform"), layers, 2)

    def randn(*shape, seed):
        return torch.randn(*shape, generator=torch.Generator().manual_seed(seed)).to(dt).cuda()

    def check(where):
        for l in range(layers):
            assert np.array_equal(cache.key_cache[l].float().cpu().numpy(), oc.K[l]), where
            assert np.array_equal(cache.value_cache[l].float().cpu().numpy(), oc.V[l]), where
            S = cache.salience_scores[l].cpu().numpy()
            assert np.array_equal(S.view(np.uint32), oc.S[l].view(np.uint32)), where

    for l in range(layers):
        k, v = randn(B, Hkv, 600, D, seed=l), randn(B, Hkv, 600, D, seed=40 + l)
        q = randn(B, Hq, 1, D, seed=80 + l)
        cache.update(k, v, l, {"query_states": q})
        oc.update(k.float().cpu().numpy(), v.float().cpu().numpy(), l, q.float().cpu().numpy())
    rng = np.random.default_rng(9)
    seed = 1000
    compactions0 = cache.compactions
    for step in range(48):
        for l in range(layers):
            seed += 3
            q = randn(B, Hq, 1, D, seed=seed)
            k, v = randn(B, Hkv, 1, D, seed=seed + 1), randn(B, Hkv, 1, D, seed=seed + 2)
            out = cache.decode_step(q, k, v, l)
            Kc, Vc = oc.update(k.float().cpu().numpy(), v.float().cpu().numpy(), l,
                               q.float().cpu().numpy())
            ref = O.attention(q.float().cpu().numpy(), Kc, Vc)
            np.testing.assert_allclose(out.float().cpu().numpy(), ref, atol=2e-2, rtol=1e-2)
        beam = np.sort(rng.integers(0, B, size=B))
        cache.reorder_cache(torch.as_tensor(beam))
        for l in range(layers):
            for arr in (oc.K, oc.V, oc.S):
                arr[l] = np.ascontiguousarray(arr[l][beam])
        if step == 20:
            cache.crop(3)
            for l in range(layers):
                oc.K[l], oc.V[l] = oc.K[l][:, :, :-3].copy(), oc.V[l][:, :, :-3].copy()
                oc.S[l] = oc.S[l][:, :-3].copy()
                oc.ids[l] = oc.ids[l][:-3]
            oc.seen -= 3
        if step % 8 == 0:
            check(f"step {step}")
    check("end")
    assert cache.compactions > compactions0   # pages were dropped while shared
    cache.check_errors()


def test_row_map_bad_index_keeps_the_sequence():
    """An index outside the batch sets the error flag and leaves that sequence as it was, on
    moved slots (its own row is gathered into place) and on rewritten ones (its entry stays)."""
    slots, B, Hkv, P, D, dt = 6, 4, 2, 16, 128, torch.bfloat16
    rng = np.random.default_rng(8)
    pool = _pool(slots, B, Hkv, P, D, dt, seed=9)
    rm0 = torch.as_tensor(rng.integers(0, B, size=(slots, B)), dtype=torch.int32).cuda()
    rm = rm0.clone()
    index = [1, 9, 0, 3]
    ok = [0, 2, 3]
    before = [t.clone() for t in pool]
    flag = _flag()
    assert _reindex(pool, pool, index, list(range(slots)), flag, row_map=rm, num_moved=2) == 0
    assert int(flag.item()) == 2
    flag.zero_()
    k0, _, s0 = before
    for sl in range(slots):
        for b in range(B):
            src = index[b] if b in ok else b
            assert torch.equal(pool[2][sl][b], s0[sl][src])
            if sl < 2:
                assert torch.equal(pool[0][sl][b], k0[sl][int(rm0[sl][src])])
                assert int(rm[sl][b]) == b
            else:
                assert torch.equal(pool[0][sl], k0[sl])
                assert int(rm[sl][b]) == int(rm0[sl][src])
