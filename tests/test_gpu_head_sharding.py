"""KV-head sharding against one process holding every head (GPU).

Each rank holds some kv heads of every sequence (and their query heads).  A token's salience
needs every head -- the resonance is a max over all query heads, the initial salience a mean
of ||k|| over all kv heads -- so every scoring call writes the rank's share into an exchange
block, the ranks combine the blocks with an element-wise MAX, and the salience update runs on
the result.  The salience must come out bit for bit as in one process holding every head, so
every rank keeps the same pages as that process; each rank's attention output is the one
process's output for its own query heads.

* On one GPU the ranks are emulated by threads in lockstep (one CUDA stream each); their
  ``reduce`` is an element-wise torch.maximum over the ranks' blocks, which is what the
  all-reduce MAX computes.
* On two GPUs the ranks are processes, exchanging either by NCCL's all-reduce MAX
  (razorkv_b200.distributed.kv_head_shard) or by the decode kernel's stores into every rank's
  region over NVLink with flags (``HeadGroup.enable_peer_exchange``; compactions and the
  prefill still use the all-reduce); skipped with fewer than 2 GPUs.
"""

import os
import socket
import threading

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

LAYERS, T, STEPS = 2, 1500, 24


def _config():
    from razorkv_b200 import RazorConfig
    return RazorConfig(compression_ratio=0.30, sink_tokens=32, local_window=128, page_size=16,
                       pyramid_mode="linear", pyramid_min_ratio=0.2, pyramid_max_ratio=0.5)


def _inputs(shape, kind, layer, step):
    """Tensors with every head, identical for every rank (seeded on the CPU)."""
    B, HQ, HKV, D = shape
    g = torch.Generator().manual_seed(1000 * layer + step * 7 + (0 if kind == "prefill" else 3))
    if kind == "prefill":
        return (torch.randn(B, HKV, T, D, generator=g).bfloat16(),
                torch.randn(B, HKV, T, D, generator=g).bfloat16(),
                torch.randn(B, HQ, 1, D, generator=g).bfloat16())
    return (torch.randn(B, HQ, 1, D, generator=g).bfloat16(),
            torch.randn(B, HKV, 1, D, generator=g).bfloat16(),
            torch.randn(B, HKV, 1, D, generator=g).bfloat16())


def _run(cache, shape, dev, h0, hkv):
    """Prefill and decode with kv heads [h0, h0 + hkv) and their query heads."""
    B, HQ, HKV, D = shape
    G = HQ // HKV
    kv_sl, q_sl = slice(h0, h0 + hkv), slice(h0 * G, (h0 + hkv) * G)
    outs = []
    for l in range(LAYERS):
        k, v, q = _inputs(shape, "prefill", l, 0)
        cache.update(k[:, kv_sl].contiguous().to(dev), v[:, kv_sl].contiguous().to(dev), l,
                     {"query_states": q[:, q_sl].contiguous().to(dev)})
    for s in range(STEPS):
        for l in range(LAYERS):
            q, k, v = _inputs(shape, "decode", l, s + 1)
            outs.append(cache.decode_step(q[:, q_sl].contiguous().to(dev),
                                          k[:, kv_sl].contiguous().to(dev),
                                          v[:, kv_sl].contiguous().to(dev), l))
    return torch.stack(outs)


class _LockstepGroup:
    """Element-wise MAX of the exchange blocks of ranks run as threads on one GPU."""

    def __init__(self, world):
        self.world = world
        self.blocks = [None] * world
        self.barrier = threading.Barrier(world, timeout=120)

    def member(self, rank, head0, local, total):
        from razorkv_b200.distributed import HeadGroup
        group = self

        class Member(HeadGroup):
            def reduce(self, x):
                group.blocks[rank] = x
                group.barrier.wait()
                torch.cuda.synchronize()      # every rank's block is written
                m = group.blocks[0].clone()
                for other in group.blocks[1:]:
                    m = torch.maximum(m, other)
                torch.cuda.synchronize()
                group.barrier.wait()          # every rank has read every block
                x.copy_(m)
                torch.cuda.synchronize()

        return Member(head0, local, total)


def _compare(shape, outs, sal, tables, keys, lens, single_outs, single, world):
    B, HQ, HKV, D = shape
    G, local = HQ // HKV, HKV // world
    for l in range(LAYERS):
        s_ref = single.salience_scores[l].cpu().numpy()
        t_ref = single.page_table(l).cpu()
        k_ref = single.key_cache[l].cpu()
        for r in range(world):
            assert lens[r][l] == single.get_cached_seq_length(l)
            assert np.array_equal(sal[r][l].view(np.uint32), s_ref.view(np.uint32)), (r, l)
            assert torch.equal(tables[r][l], t_ref), (r, l)
            assert torch.equal(keys[r][l], k_ref[:, r * local:(r + 1) * local]), (r, l)
    for r in range(world):
        ref = single_outs[:, :, r * local * G:(r + 1) * local * G]
        np.testing.assert_allclose(outs[r].float().numpy(), ref.float().numpy(), atol=2e-2,
                                   rtol=1e-2)


@pytest.mark.parametrize("shape", [(1, 28, 4, 128), (2, 8, 2, 128), (2, 16, 2, 64)])
def test_head_sharding_matches_one_process_on_one_gpu(shape):
    """Two ranks in lockstep threads on one GPU (GQA 7 exercises the screened instance)."""
    from razorkv_b200 import PagedRazorKVCache
    B, HQ, HKV, D = shape
    world = 2
    local = HKV // world
    dev = torch.device("cuda", 0)
    group = _LockstepGroup(world)
    res = [None] * world
    errors = []

    def rank_main(r):
        try:
            stream = torch.cuda.Stream(device=dev)
            with torch.cuda.stream(stream):
                cache = PagedRazorKVCache(_config(), LAYERS)
                cache.head_group = group.member(r, r * local, local, HKV)
                outs = _run(cache, shape, dev, r * local, local)
                torch.cuda.synchronize()
                cache.check_errors()
                res[r] = (outs.cpu(),
                          [cache.salience_scores[l].cpu().numpy() for l in range(LAYERS)],
                          [cache.page_table(l).cpu() for l in range(LAYERS)],
                          [cache.key_cache[l].cpu() for l in range(LAYERS)],
                          [cache.get_cached_seq_length(l) for l in range(LAYERS)])
        except Exception as exc:   # noqa: BLE001 - reported below
            errors.append(repr(exc))
            group.barrier.abort()

    threads = [threading.Thread(target=rank_main, args=(r,)) for r in range(world)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=600)
    assert not errors, errors
    single = PagedRazorKVCache(_config(), LAYERS)
    single_outs = _run(single, shape, dev, 0, HKV).cpu()
    _compare(shape, [x[0] for x in res], [x[1] for x in res], [x[2] for x in res],
             [x[3] for x in res], [x[4] for x in res], single_outs, single, world)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, shape, peer, q):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=dev)
    try:
        from razorkv_b200 import PagedRazorKVCache
        from razorkv_b200.distributed import kv_head_shard
        B, HQ, HKV, D = shape
        cache = PagedRazorKVCache(_config(), LAYERS)
        cache.head_group = kv_head_shard(HKV)
        hg = cache.head_group
        if peer:   # the exchange by peer stores over NVLink instead of the all-reduce
            hg.enable_peer_exchange(dev, B, T + STEPS + 64)
        outs = _run(cache, shape, dev, hg.head0, hg.num_kv_heads_local)
        torch.cuda.synchronize()
        cache.check_errors()
        q.put((rank, outs.cpu(), [cache.salience_scores[l].cpu().numpy() for l in range(LAYERS)],
               [cache.page_table(l).cpu() for l in range(LAYERS)],
               [cache.key_cache[l].cpu() for l in range(LAYERS)],
               [cache.get_cached_seq_length(l) for l in range(LAYERS)]))
        dist.barrier()
        if peer:
            hg.peer.close()
    except Exception as exc:
        q.put((rank, "error", repr(exc)))
        raise
    finally:
        dist.destroy_process_group()


def _collect(procs, q, world):
    """The workers' results; fails as soon as a worker exits without one."""
    import queue
    import time
    got, deadline = [], time.monotonic() + 600
    while len(got) < world:
        try:
            got.append(q.get(timeout=5))
            continue
        except queue.Empty:
            pass
        dead = [p.exitcode for p in procs if p.exitcode not in (None, 0)]
        if dead or time.monotonic() > deadline:
            for p in procs:
                p.join(timeout=60)
            pytest.fail(f"worker exit codes {[p.exitcode for p in procs]}, results {len(got)}")
    return sorted(got, key=lambda x: x[0])


def _spawn_and_compare(world, peer):
    import torch.multiprocessing as mp
    from razorkv_b200 import PagedRazorKVCache
    shape = (1, 28, 4, 128)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, shape, peer, q))
             for r in range(world)]
    for p in procs:
        p.start()
    got = _collect(procs, q, world)
    for p in procs:
        p.join(timeout=120)
    for g in got:
        assert g[1] != "error", g
    single = PagedRazorKVCache(_config(), LAYERS)
    single_outs = _run(single, shape, torch.device("cuda", 0), 0, shape[2]).cpu()
    _compare(shape, [g[1] for g in got], [g[2] for g in got], [g[3] for g in got],
             [g[4] for g in got], [g[5] for g in got], single_outs, single, world)
    for p in procs:
        assert p.exitcode == 0


def test_peer_exchange_one_rank_matches_one_process():
    """The peer-store exchange path (regions, flags, epochs, the waiting salience update) with
    a group of one rank on one GPU: the update waits only on the flag its own preceding decode
    launch released, so no launch waits on a concurrent one."""
    _spawn_and_compare(1, True)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("peer", [False, True], ids=["all_reduce", "peer_stores"])
def test_two_gpu_head_sharding_matches_one_process(peer):
    _spawn_and_compare(2, peer)
