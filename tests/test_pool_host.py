"""Host-side pool bookkeeping of PagedRazorKVCache on CPU tensors (no kernel runs): growing a
pool keeps every slot's data, free-stack order and row-map entries, and gives new slots
identity rows; reset drops the row map."""

import torch

from razorkv_b200 import PagedRazorKVCache, RazorConfig


def _cache(B=3, Hkv=1, D=8):
    cache = PagedRazorKVCache(RazorConfig(), 1)
    cache._B, cache._Hkv, cache._D = B, Hkv, D
    cache._dtype, cache._device = torch.float32, torch.device("cpu")
    cache._grow(4)
    return cache


def test_grow_keeps_slots_and_free_order():
    cache = _cache()
    n0 = cache._slots
    assert n0 == 16 and cache._free_top == 16
    # pops take ascending slot ids from the top of the stack
    assert cache._free[:16].tolist() == list(range(15, -1, -1))
    cache._k.normal_()
    k0 = cache._k.clone()
    cache._free_top = 5                       # 11 slots in use
    top0 = cache._free[:5].clone()
    cache._grow(40)
    assert cache._slots == 40
    assert torch.equal(cache._k[:n0], k0)
    assert torch.count_nonzero(cache._k[n0:]) == 0
    # the new slots sit under the old free entries, highest id first
    assert cache._free_top == 5 + 24
    assert cache._free[:24].tolist() == list(range(39, 15, -1))
    assert torch.equal(cache._free[24:29], top0)


def test_grow_extends_the_row_map_with_identity_rows():
    cache = _cache(B=3)
    rm = torch.randint(0, 3, (cache._slots, 3), dtype=torch.int32)
    cache._rowmap = rm.clone()
    cache._pool_changed()
    cache._grow(40)
    assert cache._rowmap.shape == (40, 3)
    assert torch.equal(cache._rowmap[:16], rm)
    assert torch.equal(cache._rowmap[16:], torch.arange(3, dtype=torch.int32).repeat(24, 1))
    cache.reset()
    assert cache._rowmap is None and cache._free_top == 40
