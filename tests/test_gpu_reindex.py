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


def _layout(k, v):
    slots, B, Hkv, P, D = k.shape
    return KVLayout(k.data_ptr(), v.data_ptr(), dtype_code(k.dtype), D, B, Hkv, k.stride(1),
                    k.stride(2), k.stride(0), k.stride(3), P, slots, None, 0, 0)


def _sal(s):
    return Salience(s.data_ptr(), s.stride(1), s.stride(0))


def _flag():
    f = Workspace._flag(Workspace.get(torch.device("cuda", torch.cuda.current_device()), 1 << 20))
    f.zero_()
    return f


def _reindex(src, dst, index, slots, flag=None):
    lib = _lib.load()
    idx = torch.as_tensor(index, dtype=torch.int64).cuda()
    sl = torch.as_tensor(slots, dtype=torch.int64).cuda()
    st = lib.rkv_reindex_batch(_layout(*src[:2]), _sal(src[2]), _layout(*dst[:2]), _sal(dst[2]),
                               idx.data_ptr(), sl.data_ptr(), sl.numel(),
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
                                 sl.data_ptr(), 1, None, None) == 1
    # non-contiguous (slot, sequence) planes
    lay = _layout(k, v)
    lay.stride_h = lay.stride_h * 2
    assert lib.rkv_reindex_batch(lay, _sal(s), _layout(k2, v2), _sal(s2), idx.data_ptr(),
                                 sl.data_ptr(), 1, None, None) == 2
    # a destination batch too large for the staging buffer
    big = _layout(k2, v2)
    big.batch = 100000
    assert lib.rkv_reindex_batch(_layout(k, v), _sal(s), big, _sal(s2), idx.data_ptr(),
                                 sl.data_ptr(), 1, None, None) == 2
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
    cache.reorder_cache(torch.tensor([2, 2, 0]))
    assert cache._k.data_ptr() == ptr
    for l in range(2):
        assert torch.equal(cache.key_cache[l], K0[l][[2, 2, 0]])
        assert torch.equal(cache.salience_scores[l], S0[l][[2, 2, 0]])
    cache.batch_repeat_interleave(2)
    assert cache.batch_size == 6
    for l in range(2):
        assert torch.equal(cache.key_cache[l], K0[l][[2, 2, 2, 2, 0, 0]])
    cache.check_errors()
