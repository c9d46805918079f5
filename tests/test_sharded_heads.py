"""KV-head sharding over 2 gloo ranks (CPU): the exchange-block decomposition of the salience
update is exact.

Each rank holds half of the kv heads (and their query heads).  It computes, with the oracle,
the resonance of every token over its own query heads and the norms of the new tokens' rows
of its own kv heads, encodes them as signed keys into an exchange block (INT32_MIN where it
holds no head), and the ranks combine the blocks with ``HeadGroup.reduce`` (an all-reduce MAX
over gloo).  Decoding the block and applying the update -- initial salience = sequential fp32
sum of the kv-head norms / Hkv, then the EWMA with the combined resonance -- must give the
single-process oracle's salience bit for bit, on every rank.
"""

import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import razorkv_oracle as O

B, HQ, HKV, D, N0, NEW = 2, 28, 4, 64, 300, 5   # GQA 7
ELT = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _data():
    g = torch.Generator().manual_seed(5)
    K = torch.randn(B, HKV, N0 + NEW, D, generator=g).bfloat16().float().numpy()
    q = torch.randn(B, HQ, 1, D, generator=g).bfloat16().float().numpy()
    S0 = (torch.rand(B, N0, generator=g) * 10 + 1).float().numpy()
    return K, q, S0


def signed_key(x):
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    key = np.where((u >> 31) == 1, (~u) & 0xFFFFFFFF, u | 0x80000000)
    return (key ^ 0x80000000).astype(np.uint32).view(np.int32)


def from_signed_key(k):
    u = (np.asarray(k, np.int32).view(np.uint32).astype(np.uint64) ^ 0x80000000)
    bits = np.where((u & 0x80000000) != 0, u & 0x7FFFFFFF, (~u) & 0xFFFFFFFF)
    return bits.astype(np.uint32).view(np.float32)


def _apply(x, S0, n_tok, decay=0.98):
    """The salience update from a combined block: keys [B, n_tok], then NEW x HKV norms."""
    f32 = np.float32
    R = from_signed_key(x[:, :n_tok])
    norms = from_signed_key(x[:, n_tok:]).reshape(B, NEW, HKV)
    init = np.zeros((B, NEW), np.float32)
    for h in range(HKV):
        init = (init + norms[:, :, h]).astype(np.float32)
    init = (init / f32(HKV)).astype(np.float32)
    old = np.concatenate([S0, init], axis=1)
    return O.ewma(old, R, decay)


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from razorkv_b200.distributed import kv_head_shard
        hg = kv_head_shard(HKV)
        K, qq, S0 = _data()
        G = HQ // HKV
        h0, hl = hg.head0, hg.num_kv_heads_local
        n_tok = N0 + NEW
        x = np.full((B, n_tok + NEW * HKV), np.iinfo(np.int32).min, np.int32)
        Kl = np.ascontiguousarray(K[:, h0:h0 + hl])
        ql = np.ascontiguousarray(qq[:, h0 * G:(h0 + hl) * G])
        x[:, :n_tok] = signed_key(O.resonance(ql, Kl, ELT))
        for i in range(NEW):
            for h in range(h0, h0 + hl):
                nrm = O.norm_salience(np.ascontiguousarray(K[:, h:h + 1, N0 + i:N0 + i + 1]), ELT)
                x[:, n_tok + i * HKV + h] = signed_key(nrm[:, 0])
        xt = torch.from_numpy(x)
        hg.reduce(xt)
        q.put((rank, _apply(xt.numpy(), S0, n_tok)))
    finally:
        dist.destroy_process_group()


def test_two_rank_head_sharded_salience_matches_one_process():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    K, qq, S0 = _data()
    init = O.norm_salience(np.ascontiguousarray(K[:, :, N0:]), ELT)          # all kv heads
    expect = O.ewma(np.concatenate([S0, init], axis=1), O.resonance(qq, K, ELT), 0.98)
    for rank, got in results:
        assert np.array_equal(got.view(np.uint32), expect.view(np.uint32)), f"rank {rank}"


def test_signed_keys_order_like_floats():
    v = np.array([-np.inf, -3.5, -1e-30, -0.0, 0.0, 1e-30, 2.0, np.inf], np.float32)
    k = signed_key(v)
    assert np.all(np.diff(k.astype(np.int64)) >= 0)
    assert np.array_equal(from_signed_key(k).view(np.uint32)[[0, 1, 2, 4, 5, 6, 7]],
                          v.view(np.uint32)[[0, 1, 2, 4, 5, 6, 7]])
