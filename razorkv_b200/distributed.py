"""Sharding of the cache across ranks (one process per GPU): by sequence and by kv head.

Batch sharding.  Each rank holds all kv heads of its own B_local sequences, so scoring and
attention need no communication.  Page selection does: the reference averages page scores
over the *whole* batch before its top-k (razorkv/cache.py:335-341).  To keep the kept-page set
identical to a single process holding the global batch, every rank all-gathers its
[B_local, pages] page scores in rank order (global batch order), and every rank then runs the
same sequential-sum mean and top-k on the same data.  The exchange happens only on
compaction steps (about 64 KB per rank per compacting layer).

KV-head sharding.  Each rank holds kv heads [head0, head0 + Hkv_local) of every sequence
(and their query heads), so attention is local but a token's salience is not: the resonance
is a max over every query head (razorkv/cache.py:280) and the initial salience a mean of
||k|| over every kv head (razorkv/cache.py:241-243).  Every scoring call therefore writes this
rank's share as order-preserving int32 keys into an exchange block, the ranks of the head
group take the element-wise MAX (an all-reduce MAX: exact, so the result does not depend on
the order of the ranks), and the salience update runs on the combined block, bit for bit as
one process holding every head.  The exchange is one all-reduce of B * (tokens + kv heads)
int32 per scored layer step.  Every rank then holds the same salience and selects the same
pages with no further collective.
"""

from typing import Callable, Optional

import torch
import torch.distributed as dist


def batch_sharded_score_reducer(group: Optional[dist.ProcessGroup] = None
                                ) -> Callable[[torch.Tensor], torch.Tensor]:
    """Returns f(scores [B_local, pages]) -> [world * B_local, pages] in rank order.

    Install it as ``PagedRazorKVCache.score_reducer``.  All ranks must hold the same number
    of sequences and compact the same layers at the same steps (they do: the budgets depend
    only on token counts)."""
    world = dist.get_world_size(group)

    def reduce(scores: torch.Tensor) -> torch.Tensor:
        scores = scores.contiguous()
        if world == 1:
            return scores
        parts = [torch.empty_like(scores) for _ in range(world)]
        dist.all_gather(parts, scores, group=group)
        return torch.cat(parts, dim=0)

    return reduce


class HeadGroup:
    """This rank's place in a KV-head shard group: it holds global kv heads
    [head0, head0 + num_kv_heads_local) of num_kv_heads_total.  Install it as
    ``PagedRazorKVCache.head_group``; ``reduce`` combines an exchange block over the group."""

    def __init__(self, head0: int, num_kv_heads_local: int, num_kv_heads_total: int,
                 group: Optional[dist.ProcessGroup] = None):
        if head0 < 0 or num_kv_heads_local < 1 or head0 + num_kv_heads_local > num_kv_heads_total:
            raise ValueError("kv head range outside the layer's heads")
        self.head0 = head0
        self.num_kv_heads_local = num_kv_heads_local
        self.num_kv_heads_total = num_kv_heads_total
        self.group = group
        self.peer = None   # PeerExchange once enable_peer_exchange has run

    def reduce(self, x: torch.Tensor) -> None:
        """Element-wise MAX of the int32 exchange block over the ranks of the group, in place."""
        dist.all_reduce(x, op=dist.ReduceOp.MAX, group=self.group)

    def enable_peer_exchange(self, device, batch: int, max_tokens: int) -> "PeerExchange":
        """Set up the exchange without a collective for decode steps of up to max_tokens
        tokens per layer (a collective call: every rank of the group calls it).  Each rank
        allocates a region of two buffers x world sub-blocks of batch x (max_tokens + kv heads)
        int32 plus world flags, and maps every other rank's region into this process through
        CUDA IPC; the decode kernel then stores its share straight into every rank's region
        over NVLink and the salience update waits on the flags instead of an all-reduce.
        Steps longer than max_tokens fall back to ``reduce``."""
        self.peer = PeerExchange(self, torch.device(device), batch, max_tokens)
        return self.peer


class PeerExchange:
    """The ranks' exchange regions mapped into this process (see HeadGroup)."""

    def __init__(self, hg: HeadGroup, device: torch.device, batch: int, max_tokens: int):
        import ctypes

        from . import _lib
        from ._lib import PeerExchange as PX

        lib = _lib.load()
        world = dist.get_world_size(hg.group)
        rank = dist.get_rank(hg.group)
        self.world, self.rank = world, rank
        self.stride = max_tokens + hg.num_kv_heads_total
        self.sub = batch * self.stride
        n_data = 2 * world * self.sub
        self.flag_off = (n_data + 63) // 64 * 64          # int32 elements
        self.region = torch.zeros(self.flag_off + 64 * ((world + 63) // 64), dtype=torch.int32,
                                  device=device)
        torch.cuda.synchronize(device)
        handle = (ctypes.c_ubyte * 64)()
        offset = ctypes.c_int64(0)
        _lib.check(lib.rkv_ipc_export(self.region.data_ptr(), handle, ctypes.byref(offset)),
                   "rkv_ipc_export")
        shared = [None] * world
        dist.all_gather_object(shared, (bytes(handle), offset.value), group=hg.group)
        # map every peer's region into this rank's device context (peer access over NVLink)
        self._imported = []
        base = []
        with torch.cuda.device(device):
            for r in range(world):
                if r == rank:
                    base.append(self.region.data_ptr())
                    continue
                h = (ctypes.c_ubyte * 64).from_buffer_copy(shared[r][0])
                ptr = ctypes.c_void_p()
                _lib.check(lib.rkv_ipc_import(h, shared[r][1], ctypes.byref(ptr)),
                           "rkv_ipc_import")
                self._imported.append((ptr.value, shared[r][1]))
                base.append(ptr.value)
        self.regions = torch.tensor(base, dtype=torch.int64, device=device)
        self.flags = torch.tensor([b + 4 * self.flag_off for b in base], dtype=torch.int64,
                                  device=device)
        self.epoch = 0
        self.px = PX(self.regions.data_ptr(), self.flags.data_ptr(), self.region.data_ptr(),
                     self.region.data_ptr() + 4 * self.flag_off, rank, world, self.sub, 0, 0, 0)
        torch.cuda.synchronize(device)
        dist.barrier(group=hg.group)

    def next(self):
        """The descriptor of the next exchange (epoch + 1, the other buffer)."""
        self.epoch += 1
        self.px.epoch = self.epoch & 0xFFFFFFFF
        self.px.buf_off = (self.epoch & 1) * self.world * self.sub
        return self.px

    def close(self):
        """Unmap the peers' regions (every rank, before the regions are freed)."""
        from . import _lib
        lib = _lib.load()
        for ptr, off in self._imported:
            lib.rkv_ipc_release(ptr, off)
        self._imported = []


def kv_head_shard(num_kv_heads: int, group: Optional[dist.ProcessGroup] = None) -> HeadGroup:
    """The HeadGroup of this rank when a layer's kv heads are split evenly over ``group``
    (rank r holds heads [r * Hkv / world, (r + 1) * Hkv / world))."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if num_kv_heads % world:
        raise ValueError(f"{num_kv_heads} kv heads do not split over {world} ranks")
    local = num_kv_heads // world
    return HeadGroup(rank * local, local, num_kv_heads, group)
