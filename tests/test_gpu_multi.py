"""Batch sharding over 2 GPUs (NCCL, one process per GPU) against one process holding the
whole batch: every rank decodes its own sequences, page selection averages the page scores
of the global batch through the all-gather score reducer, and NCCL gathers the page tables,
salience and outputs to rank 0 for verification.  Skipped with fewer than 2 GPUs."""

import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

LAYERS, B, HQ, HKV, D, T, STEPS = 2, 4, 8, 2, 128, 1500, 24


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(kind, layer, step):
    """Global-batch tensors, identical on every rank (seeded on the CPU)."""
    g = torch.Generator().manual_seed(1000 * layer + step * 7 + (0 if kind == "prefill" else 3))
    if kind == "prefill":
        return (torch.randn(B, HKV, T, D, generator=g).bfloat16(),
                torch.randn(B, HKV, T, D, generator=g).bfloat16(),
                torch.randn(B, HQ, 1, D, generator=g).bfloat16())
    return (torch.randn(B, HQ, 1, D, generator=g).bfloat16(),
            torch.randn(B, HKV, 1, D, generator=g).bfloat16(),
            torch.randn(B, HKV, 1, D, generator=g).bfloat16())


def _run(cache, dev, sl):
    outs = []
    for l in range(LAYERS):
        k, v, q = (t[sl].to(dev) for t in _inputs("prefill", l, 0))
        cache.update(k, v, l, {"query_states": q})
    for s in range(STEPS):
        for l in range(LAYERS):
            q, k, v = (t[sl].to(dev) for t in _inputs("decode", l, s + 1))
            outs.append(cache.decode_step(q, k, v, l))
    return outs


def _config():
    from razorkv_b200 import RazorConfig
    return RazorConfig(compression_ratio=0.30, sink_tokens=32, local_window=128, page_size=16,
                       pyramid_mode="linear", pyramid_min_ratio=0.2, pyramid_max_ratio=0.5)


def _worker(rank, world, port, q):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=dev)
    try:
        from razorkv_b200 import PagedRazorKVCache
        from razorkv_b200.distributed import batch_sharded_score_reducer
        per = B // world
        cache = PagedRazorKVCache(_config(), LAYERS)
        cache.score_reducer = batch_sharded_score_reducer()
        outs = torch.stack(_run(cache, dev, slice(rank * per, (rank + 1) * per)))
        torch.cuda.synchronize()
        # verification only: gather everything to rank 0
        gathered = [torch.empty_like(outs) for _ in range(world)]
        dist.all_gather(gathered, outs)
        sal = [cache.salience_scores[l] for l in range(LAYERS)]
        sal_all = []
        for s in sal:
            parts = [torch.empty_like(s) for _ in range(world)]
            dist.all_gather(parts, s.contiguous())
            sal_all.append(torch.cat(parts, 0).cpu())
        keys_all = []
        for l in range(LAYERS):
            k = cache.key_cache[l].contiguous()
            parts = [torch.empty_like(k) for _ in range(world)]
            dist.all_gather(parts, k)
            keys_all.append(torch.cat(parts, 0).cpu())
        tables = [cache.page_table(l) for l in range(LAYERS)]
        table_sets = []
        for t in tables:
            parts = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(parts, t)
            table_sets.append([p.cpu() for p in parts])
        if rank == 0:
            single = PagedRazorKVCache(_config(), LAYERS)
            ref = torch.stack(_run(single, dev, slice(0, B))).cpu()
            q.put(("ok", torch.cat([g.cpu() for g in gathered], 1), ref, sal_all,
                   [single.salience_scores[l].cpu() for l in range(LAYERS)], table_sets,
                   keys_all, [single.key_cache[l].cpu() for l in range(LAYERS)],
                   [cache.get_cached_seq_length(l) for l in range(LAYERS)],
                   [single.get_cached_seq_length(l) for l in range(LAYERS)]))
        dist.barrier()
    except Exception as exc:   # report to the parent, then leave the group cleanly
        q.put(("error", repr(exc)))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_batch_sharding_matches_one_process():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = q.get(timeout=600)
    for p in procs:
        p.join(timeout=120)
    assert res[0] == "ok", res
    _, outs, ref, sal, sal_ref, tables, keys, keys_ref, n_shard, n_single = res
    assert n_shard == n_single
    for l in range(LAYERS):
        assert torch.equal(tables[l][0], tables[l][1]), "ranks kept different pages"
        assert torch.equal(keys[l], keys_ref[l]), "retained tokens differ from one process"
        assert np.array_equal(sal[l].numpy().view(np.uint32), sal_ref[l].numpy().view(np.uint32))
    np.testing.assert_allclose(outs.float().numpy(), ref.float().numpy(), atol=2e-2, rtol=1e-2)
    for p in procs:
        assert p.exitcode == 0
