"""Batch-sharded page selection over 2 gloo ranks (CPU): the kept pages equal those of one
process holding the whole batch, and every rank keeps the same pages."""

import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import razorkv_oracle as O


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _scores(B=8, pages=1400, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, pages, generator=g) * 0.4 + 12.0
    x[:, 100:140] = x[:, 100:101]          # exact ties across a block of pages
    return x.float()


def _worker(rank, world, port, k, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from razorkv_b200.distributed import batch_sharded_score_reducer
        full = _scores()
        per = full.shape[0] // world
        local = full[rank * per:(rank + 1) * per].clone()
        gathered = batch_sharded_score_reducer()(local)
        kept, margin = O.canonical_topk(O.batch_mean(gathered.numpy()), k)
        q.put((rank, gathered.numpy(), kept))
    finally:
        dist.destroy_process_group()


def test_two_rank_selection_matches_single_process():
    world, k = 2, 550
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, k, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    full = _scores().numpy()
    expect, _ = O.canonical_topk(O.batch_mean(full), k)
    for rank, gathered, kept in results:
        assert np.array_equal(gathered, full), f"rank {rank}: gather is not in global batch order"
        assert np.array_equal(kept, expect), f"rank {rank}: kept pages differ"
