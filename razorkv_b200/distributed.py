"""Batch sharding of the cache across ranks (one process per GPU).

Each rank holds all kv heads of its own B_local sequences, so scoring and attention need no
communication.  Page selection does: the reference averages page scores over the *whole*
batch before its top-k (razorkv/cache.py:335-341).  To keep the kept-page set identical to a
single process holding the global batch, every rank all-gathers its [B_local, pages] page
scores in rank order (global batch order), and every rank then runs the same
sequential-sum mean and top-k on the same data.  The exchange happens only on compaction
steps (about 64 KB per rank per compacting layer).
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
