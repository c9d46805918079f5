#!/usr/bin/env python
"""Decode throughput of the RazorKV sparse decode path (score + select + compact + attend).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
    python -m torch.distributed.run --nproc-per-node N bench.py --gpus N ...

Workload (default): the Llama-3.1-8B-shaped cache -- 32 layers, 32 query / 8 KV heads,
head_dim 128, bf16, batch 8 per GPU, 32768-token prefill in 16-token pages, sink 32,
window 512, linear layer pyramid 15 % -> 70 %, 1 % planted query-aligned pages, seeded
synthetic N(0, 1) data.  A *step* is one decode step of all layers for the whole batch:
per layer, append the new token, score every retained token, compact when the hysteresis
threshold is crossed, and attend over the retained pages.  Tokens/s = batch / step time.

* ``value``   : device time (CUDA events, max over ranks) of K steps with inputs resident
                in HBM; the retained KV read per step (~14.6 GB) exceeds the 126 MB L2.
* ``e2e``     : the same steps driven through the public ``PagedRazorKVCache.decode_step``
                with every step's q / k / v copied from pinned host memory and the step's
                outputs copied back, inside the timed region; as in a serving loop the copies
                run on two copy streams (double-buffered) while the previous step decodes.
* ``roofline``: the decode kernel's algorithmic bytes (retained K + V of each launch) over
                its CUDA-event duration, against the measured HBM copy bandwidth.
* ``cpu_baseline`` : the CPU oracle (a restatement of the reference algorithm) timed on a
                bounded sample of the same workload on this host's cores.
* ``--impl reference``: the reference algorithm's CPU path (the oracle port; the reference
                itself is Python and is not installed here) on the host cores, same metric.

Multi-GPU: one process per GPU, weak scaling (batch 8 per GPU, different sequences per
rank).  Page selection averages page scores over the global batch, so on compaction steps
the ranks all-gather their [B_local, pages] scores (NCCL) before the identical top-k.
"""

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode attention tokens/s/GPU and HBM GB/s (% of peak) at 32k ctx; 1/2/4/8 GPU"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="llama8b-b8-32k-bf16")
    ap.add_argument("--e2e-steps", type=int, default=32)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--only-layer", type=int, default=-1,
                    help="run a single layer of the workload (budget as in the full model); "
                         "a small case for profiling")
    ap.add_argument("--context", type=int, default=0, help="override the prefill length (profiling)")
    ap.add_argument("--layers", type=int, default=0,
                    help="time K evenly spaced layers of the model only (for caches larger "
                         "than one GPU's memory); the JSON config records the subset")
    ap.add_argument("--shard", default="auto", choices=["auto", "batch", "split", "heads"],
                    help="multi-GPU split: 'batch' gives every GPU the workload's batch of its "
                         "own sequences (weak scaling); 'split' divides the workload's batch "
                         "over the GPUs (strong scaling); 'heads' gives every GPU some kv heads "
                         "of the same sequences (strong scaling); auto splits heads when the "
                         "batch is smaller than the GPU count, else 'batch'")
    ap.add_argument("--no-peer-exchange", action="store_true",
                    help="with --shard heads, exchange salience shares by NCCL all-reduce "
                         "instead of peer stores over NVLink")
    ap.add_argument("--event-every", type=int, default=8,
                    help="record per-launch CUDA events on every k-th timed step")
    return ap.parse_args()


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ---------------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap,uuid")

    def __init__(self, gpu_index, uuid=None):
        # nvidia-smi lists the GPUs by their index on the machine, whatever CUDA_VISIBLE_DEVICES
        # says, so this process's GPU is found by its UUID (by index only when that is unknown)
        self.gpu = gpu_index
        self.uuid = str(uuid).lower().removeprefix("gpu-") if uuid else None
        self.proc = None
        self.path = os.path.join(tempfile.gettempdir(), f"rkv_clocks_{os.getpid()}_{gpu_index}.csv")

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        sm, mx, reasons = [], 0.0, set()
        with open(self.path) as f:
            lines = f.readlines()
        try:
            os.remove(self.path)
        except OSError:
            pass
        for line in lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10 or not parts[0].isdigit():
                continue
            if self.uuid is not None:
                if parts[9].lower().removeprefix("gpu-") != self.uuid:
                    continue
            elif int(parts[0]) != self.gpu:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------- helpers
def pool_slots(w, cfg, steps, layers):
    P = w.page_size
    T_end = w.context + steps + 1
    slots = 0
    for l in layers:
        b = cfg.get_layer_budget(l, w.num_layers, T_end)
        slots += (b + 2 * P) // P + 2
    return slots + (w.context + P - 1) // P + 64


class KernelTimer:
    """Counts the retained K/V bytes of every decode-kernel launch of decode_step inside the
    timed region, and records CUDA events around the launches of the sampled steps.

    An event recorded between two launches ends the programmatic overlap of the second
    launch's start with the first one's tail, so events go only around the launches of every
    ``every``-th timed step; the other steps run as a user's would."""

    def __init__(self, torch, every=1):
        self.torch = torch
        self.pairs = []
        self.enabled = False      # inside the timed region
        self.sampling = False     # this step's launches get events
        self.every = max(1, every)
        self.all_bytes = 0
        self.all_launches = 0
        self.pool = []

    def prepare(self, n):
        """Create the events up front so recording costs the host as little as possible."""
        mk = lambda: self.torch.cuda.Event(enable_timing=True)
        self.pool = [(mk(), mk()) for _ in range(n)]

    def before(self, layer, kv_bytes):
        if not self.enabled:
            return
        self.all_bytes += kv_bytes
        self.all_launches += 1
        if not self.sampling:
            return
        i = len(self.pairs)
        e0, e1 = self.pool[i] if i < len(self.pool) else (
            self.torch.cuda.Event(enable_timing=True), self.torch.cuda.Event(enable_timing=True))
        e0.record()
        self.pairs.append([e0, e1, kv_bytes])

    def after(self):
        if not (self.enabled and self.sampling):
            return
        self.pairs[-1][1].record()

    def summary(self):
        ms = sum(a.elapsed_time(b) for a, b, _ in self.pairs)
        nbytes = sum(n for _, _, n in self.pairs)
        return len(self.pairs), ms, nbytes


def traffic_per_byte():
    """DRAM bytes per algorithmic byte of the decode kernel from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "decode_kernel_llama8b_layer.md")
    try:
        with open(path) as f:
            for line in f:
                if line.startswith("dram_bytes_per_algorithmic_byte:"):
                    return float(line.split(":")[1])
    except OSError:
        pass
    return None


# ---------------------------------------------------------------------------- CPU oracle arm
def oracle_sample(w, steps, warmup=0, threads=None, parity_dev=None):
    """Time the CPU oracle (reference algorithm) on a bounded sample of workload w and, with
    ``parity_dev``, run the GPU cache beside it on the same CPU-drawn inputs.

    Sample: the shallowest and deepest layers (0 and L-1) at the full batch after a full
    prefill (which compacts every layer to its budget); every decode step runs
    update(k, v, l, q) + attention on those two layers.  A full step's time is extrapolated:
    the measured seconds per retained token of the sampled layers times the retained tokens
    of all L layers (the sampled layers' measured counts, the budget for the others).

    Parity (GPU cache vs oracle, same inputs): the kept pages of every compaction decision,
    the salience of the sampled layers after the last step (bit for bit), the largest
    absolute difference of the attention outputs, and the smallest top-k margin met."""
    import numpy as np
    import torch
    from oracle import razorkv_oracle as O
    from razorkv_b200.workload import decode_inputs, layer_prefill

    if threads:
        os.environ["ORACLE_THREADS"] = str(threads)
    O.lib()
    cores = int(os.environ.get("ORACLE_THREADS", os.cpu_count() or 1))
    cfg = w.razor_config()
    ocfg = O.OracleConfig(compression_ratio=cfg.compression_ratio, sink_tokens=cfg.sink_tokens,
                          local_window=cfg.local_window, page_size=cfg.page_size,
                          pyramid_mode=cfg.pyramid_mode, pyramid_min_ratio=cfg.pyramid_min_ratio,
                          pyramid_max_ratio=cfg.pyramid_max_ratio)
    L = w.num_layers
    layers = sorted({0, L - 1})
    elt = torch.tensor([], dtype=w.dtype).element_size()
    cache = O.OracleCache(ocfg, L, elt)
    gcache = None
    if parity_dev is not None:
        from razorkv_b200 import PagedRazorKVCache
        gcache = PagedRazorKVCache(cfg, L)
        gcache.record_decisions = True
    for l in layers:
        K, V, q0 = layer_prefill(w, l, "cpu")
        cache.update(K.float().numpy(), V.float().numpy(), l, q0.float().numpy())
        if gcache is not None:
            gcache.update(K.to(parity_dev), V.to(parity_dev), l, {"query_states": q0.to(parity_dev)})
        del K, V
    n_prefill_dec = len(cache.decisions)
    tot_time, tot_tokens = 0.0, 0
    max_err = 0.0
    for step in range(warmup + steps):
        t_step, n_step = 0.0, 0
        for l in layers:
            q, k, v = decode_inputs(w, step, l, "cpu")
            qn, kn, vn = q.float().numpy(), k.float().numpy(), v.float().numpy()
            t0 = time.perf_counter()
            Kc, Vc = cache.update(kn, vn, l, qn)
            ref = O.attention(qn, Kc, Vc)
            t_step += time.perf_counter() - t0
            n_step += Kc.shape[2]
            if gcache is not None:
                out = gcache.decode_step(q.to(parity_dev), k.to(parity_dev), v.to(parity_dev), l)
                max_err = max(max_err, float(np.max(np.abs(out.float().cpu().numpy() - ref))))
        if step >= warmup:
            tot_time += t_step
            tot_tokens += n_step
    sec_per_token = tot_time / max(tot_tokens, 1)
    T = cache.seen
    retained = sum(cache.K[l].shape[2] if l in layers else ocfg.budget(l, L, T) for l in range(L))
    est_step = sec_per_token * retained
    decode_evictions = len(cache.decisions) - n_prefill_dec
    res = {
        "value": w.batch / est_step,
        "unit": "tokens/s",
        "cores": cores,
        "kind": "port",
        "sample": (f"layers {layers} of {L}, batch {w.batch}, {w.context}-token prefill "
                   f"(untimed), {steps} timed decode steps with {decode_evictions} decode-time "
                   f"compactions; the full-step time is EXTRAPOLATED from the sampled layers' "
                   f"seconds per retained token to {retained} retained tokens over {L} layers"),
        "ms_per_step_est": est_step * 1e3,
        "sampled_seconds": tot_time,
        "decode_evictions_in_sample": decode_evictions,
    }
    if gcache is not None:
        torch.cuda.synchronize(parity_dev)
        gcache.check_errors()
        kept_equal = len(gcache.decisions) == len(cache.decisions)
        margins = []
        for gd, od in zip(gcache.decisions, cache.decisions):
            if gd.kind == "pages":
                kept_equal &= gd.layer == od.layer and np.array_equal(gd.kept.cpu().numpy(), od.kept)
                margins.append(float(gd.margin.item()))
            else:
                kept_equal &= od.kind == "zones"
        sal_equal = all(
            np.array_equal(gcache.salience_scores[l].cpu().numpy().view(np.uint32),
                           cache.S[l].view(np.uint32)) for l in layers)
        res["parity"] = {
            "kept_pages_equal": bool(kept_equal),
            "salience_bitexact": bool(sal_equal),
            "max_abs_err": max_err,
            "tolerance": "2e-2 abs / 1e-2 rel (bf16)" if w.dtype == torch.bfloat16 else "1e-5 rel (fp32)",
            "min_topk_margin": min(margins) if margins else None,
            "decisions": len(cache.decisions),
            "against": "oracle (CPU restatement pinned to the reference's decisions on this "
                       "workload's layers 0 and L-1 by tests/test_oracle_scale.py)",
            "sample": f"layers {layers}, CPU-drawn inputs, prefill + {warmup + steps} decode steps",
        }
        del gcache
    return res


def reference_calibration(workload_name):
    """The reference's own CPU path timed beside the oracle port on one host
    (tests/golden/time_reference.py; the reference cannot travel to this host).  Returns the
    record for the workload, or None."""
    path = os.path.join(ROOT, "tests", "golden", "reference_timing.json")
    try:
        with open(path) as f:
            rec = json.load(f)
    except OSError:
        return None
    wl = rec.get("workloads", {}).get(workload_name)
    if not wl:
        return None
    return {
        "what": "the unmodified reference torch path (RazorKVCache.update + compacted_paged_sdpa) "
                "and the oracle port timed on the same sample and the same host",
        "host_cores": rec.get("cores"), "torch": rec.get("torch"),
        "reference_torch_tokens_per_s": wl["reference_torch"]["tokens_per_s"],
        "oracle_port_tokens_per_s": wl["oracle_port"]["tokens_per_s"],
        "port_over_reference": wl["port_over_reference"],
        "sample": wl["sample"],
    }


def run_reference(args):
    import torch
    from razorkv_b200.workload import WORKLOADS
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    w = WORKLOADS[args.workload]
    if args.context:
        w = w.scaled(context=args.context)
    steps = max(1, min(args.steps, 4))
    warm = min(args.warmup, 1)
    res = oracle_sample(w, steps, warm, threads=os.cpu_count())
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": res["value"],
        "unit": "tokens/s",
        "n_gpus": args.gpus,
        "steps": steps,
        "warmup": warm,
        "ms_per_step": res["ms_per_step_est"],
        "ms_per_step_kind": "extrapolated from the sampled layers (see cpu_baseline.sample)",
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16" if w.dtype == torch.bfloat16 else "fp32",
        "data": "synthetic: seeded N(0,1) K/V/q with planted query-aligned pages",
        "config": workload_config(w, args.gpus),
        "cpu_baseline": dict({k: res[k] for k in ("value", "unit", "cores", "kind", "sample")},
                             reference_torch_calibration=reference_calibration(w.name)),
        "e2e": {"value": res["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def workload_config(w, n, shard="batch"):
    heads = shard == "heads" and n > 1
    return {
        "workload": w.name, "layers": w.num_layers, "q_heads": w.num_q_heads,
        "kv_heads": w.num_kv_heads, "head_dim": w.head_dim,
        "batch_per_gpu": w.batch, "global_batch": w.batch if heads else w.batch * n,
        "kv_heads_per_gpu": w.num_kv_heads // n if heads else w.num_kv_heads,
        "shard": shard,
        "context": w.context, "page_size": w.page_size,
        "sink": w.sink_tokens, "window": w.local_window,
        "pyramid": f"{w.pyramid_mode} {w.pyramid_min_ratio}->{w.pyramid_max_ratio}",
        "parallelism": (f"kv-head-sharded x{n}" if heads else
                        f"batch-split x{n}" if shard == "split" else f"batch-sharded x{n}")
                       if n > 1 else "single GPU",
        "l2": "inputs larger than L2 (retained KV per step >> 126 MB)",
    }


# ---------------------------------------------------------------------------- GPU arm
HF_WORKLOAD = "hf-llama24l-b4-16k"


def run_hf_generate(args):
    """End-to-end HF generate through RazorEngine.patch_model: a random-init Llama-architecture
    model (24 layers, hidden 2048, 16/4 heads, head_dim 128, vocab 32000, bf16), batch 4,
    16384-token prompt of uniform random ids, greedy decoding.  Decode throughput is
    B * (n - 1) / (t(generate n tokens) - t(generate 1 token)), both CUDA-event timed; the stock
    HF path (DynamicCache + SDPA, no eviction) is timed the same way on the same model."""
    import torch
    from transformers import LlamaConfig, LlamaForCausalLM

    from razorkv_b200 import RazorConfig, RazorEngine, _lib

    torch.cuda.set_device(0)
    B, T = 4, args.context or 16384
    new = args.steps if args.steps != 256 else 1024
    cfg = LlamaConfig(vocab_size=32000, hidden_size=2048, num_hidden_layers=24,
                      num_attention_heads=16, num_key_value_heads=4, head_dim=128,
                      max_position_embeddings=max(32768, T + new + 16))
    torch.manual_seed(0)
    model = LlamaForCausalLM(cfg).to(device="cuda", dtype=torch.bfloat16).eval()
    prompt = torch.randint(0, 32000, (B, T), generator=torch.Generator().manual_seed(1)).cuda()
    mask = torch.ones_like(prompt)

    def timed_generate(n):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        with torch.no_grad():
            out = model.generate(prompt, attention_mask=mask, max_new_tokens=n, min_new_tokens=n,
                                 do_sample=False, eos_token_id=None, pad_token_id=0,
                                 return_dict_in_generate=True)
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / 1e3, out

    def measure():
        timed_generate(2)   # warm-up (kernels, allocator)
        t1, _ = timed_generate(1)
        tn, out = timed_generate(new)
        return t1, tn, out

    rcfg = RazorConfig()
    RazorEngine.patch_model(model, config=rcfg)
    lib = _lib.load()
    l0 = lib.rkv_launch_count()
    t1, tn, out = measure()
    launches = lib.rkv_launch_count() - l0
    cache = out.past_key_values
    stats = cache.get_memory_stats()
    razor_tokens = out.sequences[:, T:].cpu()
    RazorEngine.unpatch_model(model)
    d1, dn, dout = measure()
    dense_kv = 2 * cfg.num_hidden_layers * B * cfg.num_key_value_heads * (T + new) * 128 * 2
    del dout
    line = {
        "metric": "HF generate decode tokens/s (RazorEngine drop-in, paged cache)",
        "value": B * (new - 1) / (tn - t1), "unit": "tokens/s", "n_gpus": 1,
        "steps": new, "warmup": 1, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: random-init weights (seed 0), uniform random prompt ids (seed 1)",
        "config": {"workload": HF_WORKLOAD, "model": "Llama-architecture 24L, hidden 2048, "
                   "16/4 heads, head_dim 128, vocab 32000, intermediate 11008 (LlamaConfig "
                   "default)", "batch": B, "prompt": T, "new_tokens": new,
                   "razor_config": "RazorConfig() defaults: 30 % adaptive pyramid, sink 32, "
                                   "window 512, page 16"},
        "impl": "b200",
        "prefill_s": t1,
        "ms_per_token_step": (tn - t1) / (new - 1) * 1e3,
        "dense_hf": {"value": B * (new - 1) / (dn - d1), "prefill_s": d1,
                     "ms_per_token_step": (dn - d1) / (new - 1) * 1e3,
                     "kv_bytes": dense_kv},
        "retained_kv_bytes": stats["total_bytes"],
        "pool_slots": stats["pool_slots"],
        "gpu_launches": int(launches),
        "first_tokens": razor_tokens[0, :8].tolist(),
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse_args()
    if args.workload == HF_WORKLOAD:
        return run_hf_generate(args)
    if args.impl == "reference":
        return run_reference(args)

    import torch
    import torch.distributed as dist

    from razorkv_b200 import PagedRazorKVCache, _lib
    from razorkv_b200.workload import WORKLOADS, decode_inputs, layer_prefill

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    w = WORKLOADS[args.workload]
    if args.context:
        w = w.scaled(context=args.context)
    shard = args.shard
    if shard == "auto":
        shard = "heads" if (world > 1 and w.batch < world
                            and w.num_kv_heads % world == 0) else "batch"
    if world == 1:
        shard = "none"
    if shard == "heads":
        # every rank decodes the same sequences with its own kv heads (strong scaling)
        wr = w
        h0 = rank * (w.num_kv_heads // world)
        hkv = w.num_kv_heads // world
    elif shard == "split":
        # the workload's batch divided over the ranks (strong scaling); each rank draws its own
        # sequences, and selection still averages over the whole batch (all-gather)
        if w.batch % world:
            raise SystemExit(f"--shard split: batch {w.batch} does not divide over {world} GPUs")
        w = w.scaled(batch=w.batch // world)
        wr = w.scaled(seed=w.seed + 1000 * rank)
        h0, hkv = 0, w.num_kv_heads
    else:
        # each rank holds its own sequences (weak scaling): a distinct seed per rank
        wr = w.scaled(seed=w.seed + 1000 * rank)
        h0, hkv = 0, w.num_kv_heads
    G = w.group
    kv_sl, q_sl = slice(h0, h0 + hkv), slice(h0 * G, (h0 + hkv) * G)
    cfg = w.razor_config()
    L, B = w.num_layers, w.batch
    if args.only_layer >= 0:
        layers = [args.only_layer]
    elif 0 < args.layers < L:
        layers = sorted({round(i * (L - 1) / (args.layers - 1)) for i in range(args.layers)}) \
            if args.layers > 1 else [0]
    else:
        layers = list(range(L))
    total_steps = args.warmup + args.steps + args.e2e_steps
    cache = PagedRazorKVCache(cfg, L, max_slots=pool_slots(w, cfg, total_steps, layers))

    if shard in ("batch", "split"):
        from razorkv_b200.distributed import batch_sharded_score_reducer
        cache.score_reducer = batch_sharded_score_reducer()
    elif shard == "heads":
        from razorkv_b200.distributed import kv_head_shard
        cache.head_group = kv_head_shard(w.num_kv_heads)
        if not args.no_peer_exchange:
            # decode steps exchange by peer stores over NVLink (no collective); the bound
            # covers every layer's retained tokens over the run
            cache.head_group.enable_peer_exchange(dev, B, w.context + total_steps + 64)

    def local(q, k, v):
        """This rank's heads of one step's (or the prefill's) tensors."""
        return (q[:, q_sl].contiguous(), k[:, kv_sl].contiguous(), v[:, kv_sl].contiguous())

    # ---- prefill (untimed)
    t0 = time.time()
    for l in layers:
        K, V, q0 = layer_prefill(wr, l, dev)
        q0, K, V = local(q0, K, V)
        cache.update(K, V, l, {"query_states": q0})
        del K, V, q0
    torch.cuda.synchronize()
    prefill_s = time.time() - t0

    # ---- decode inputs for every step, resident in HBM
    n_dev_steps = args.warmup + args.steps
    inputs = [{l: local(*decode_inputs(wr, s, l, dev)) for l in layers} for s in range(n_dev_steps)]
    Hq_l = hkv * G
    outs = {l: torch.empty(B, Hq_l, 1, w.head_dim, dtype=w.dtype, device=dev) for l in layers}
    timer = KernelTimer(torch, every=args.event_every)
    cache.launch_observer = timer

    single = len(layers) == 1 and layers[0] != 0
    if single:
        # the cache counts logical tokens on layer 0 (as the reference does); a single-layer
        # profiling run keeps that count as the full model would
        cache._seen_tokens = w.context

    def step(s):
        timer.sampling = (s - args.warmup) % timer.every == 0
        if single:
            cache._seen_tokens += 1
        for l in layers:
            q, k, v = inputs[s][l]
            cache.decode_step(q, k, v, l, out=outs[l])

    for s in range(args.warmup):
        step(s)
    torch.cuda.synchronize()
    lib = _lib.load()
    # every rank samples its own GPU's clocks; the samplers start before the barrier so that
    # no rank enters the timed region while another is still setting up
    try:
        gpu_uuid = torch.cuda.get_device_properties(dev).uuid
    except Exception:   # noqa: BLE001 - fall back to the index
        gpu_uuid = None
    clocks = ClockSampler(local, gpu_uuid)
    clocks.start()
    time.sleep(0.4)
    timer.prepare(-(-args.steps // timer.every) * len(layers) + 8)
    if world > 1:
        dist.barrier()
    timer.enabled = True
    launches0 = lib.rkv_launch_count()
    compactions0 = cache.compactions
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    h0 = time.perf_counter()
    for s in range(args.warmup, n_dev_steps):
        step(s)
    host_ms = (time.perf_counter() - h0) * 1e3   # time to enqueue the steps (host side)
    ev1.record()
    torch.cuda.synchronize()
    launches = lib.rkv_launch_count() - launches0
    timed_compactions = cache.compactions - compactions0
    timer.enabled = False
    clock_info = clocks.stop() if clocks else None
    ms = ev0.elapsed_time(ev1)
    n_launch, kern_ms, kern_bytes = timer.summary()
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        infos = [None] * world
        dist.all_gather_object(infos, clock_info)
        infos = [i for i in infos if i]
        if infos:
            clock_info = {
                "sm_mhz": statistics.median(i["sm_mhz"] for i in infos),
                "sm_max_mhz": max(i["sm_max_mhz"] for i in infos),
                "reasons": sorted(set(r for i in infos for r in i["reasons"])),
                "samples": sum(i["samples"] for i in infos),
                "gpus": len(infos),
            }
        dist.barrier()

    # sequences decoded by the whole job per step: every rank's own batch when sharding by
    # sequence, one shared batch when sharding by kv head
    seq_shards = 1 if shard == "heads" else world

    # ---- end to end: host inputs, public API, outputs back to the host
    e2e = None
    if args.e2e_steps > 0:
        Hq, Hkv, D = Hq_l, hkv, w.head_dim     # this rank's heads
        per_layer = B * (Hq + 2 * Hkv) * D
        host_in = []
        nl = len(layers)
        for s in range(n_dev_steps, total_steps):
            buf = torch.empty(nl, per_layer, dtype=w.dtype).pin_memory()
            for i, l in enumerate(layers):
                q, k, v = local(*decode_inputs(wr, s, l, "cpu"))
                buf[i] = torch.cat([q.reshape(-1), k.reshape(-1), v.reshape(-1)])
            host_in.append(buf)
        host_out = torch.empty(nl, B, Hq, 1, D, dtype=w.dtype).pin_memory()
        # A serving loop's copies overlap the decode: step s+1's inputs go up on one copy
        # stream and step s's outputs come down on another while step s computes, into
        # double-buffered device inputs and outputs ordered by events.
        dev_in = [torch.empty(nl, per_layer, dtype=w.dtype, device=dev) for _ in range(2)]
        dev_out = [torch.empty(nl, B, Hq, 1, D, dtype=w.dtype, device=dev) for _ in range(2)]
        comp = torch.cuda.current_stream(dev)
        h2d, d2h = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
        in_ready = [torch.cuda.Event() for _ in range(2)]
        in_free = [torch.cuda.Event() for _ in range(2)]
        out_ready = [torch.cuda.Event() for _ in range(2)]
        out_free = [torch.cuda.Event() for _ in range(2)]
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(comp)

        def upload(s):
            j = s % 2
            h2d.wait_event(e0)
            if s >= 2:
                h2d.wait_event(in_free[j])          # step s-2 is done reading this buffer
            with torch.cuda.stream(h2d):
                dev_in[j].copy_(host_in[s], non_blocking=True)
            in_ready[j].record(h2d)

        upload(0)
        for s in range(len(host_in)):
            j = s % 2
            if s + 1 < len(host_in):
                upload(s + 1)
            comp.wait_event(in_ready[j])
            if s >= 2:
                comp.wait_event(out_free[j])        # step s-2's outputs have left the GPU
            for i, l in enumerate(layers):
                x = dev_in[j][i]
                q = x[: B * Hq * D].view(B, Hq, 1, D)
                k = x[B * Hq * D: B * (Hq + Hkv) * D].view(B, Hkv, 1, D)
                v = x[B * (Hq + Hkv) * D:].view(B, Hkv, 1, D)
                cache.decode_step(q, k, v, l, out=dev_out[j][i])
            in_free[j].record(comp)
            out_ready[j].record(comp)
            d2h.wait_event(out_ready[j])
            with torch.cuda.stream(d2h):
                host_out.copy_(dev_out[j], non_blocking=True)
            out_free[j].record(d2h)
        comp.wait_event(out_free[(len(host_in) - 1) % 2])
        e1.record(comp)
        torch.cuda.synchronize()
        e_ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([e_ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e_ms = float(t.item())
        elt = torch.tensor([], dtype=w.dtype).element_size()
        e2e = {"value": seq_shards * B * args.e2e_steps / (e_ms / 1e3), "unit": "tokens/s",
               "steps": args.e2e_steps, "ms_per_step": e_ms / args.e2e_steps,
               "h2d_bytes_per_step": nl * per_layer * elt,
               "d2h_bytes_per_step": nl * B * Hq * D * elt,
               "copies": "pinned host buffers; step s+1 up and step s down on two copy "
                         "streams while step s decodes (double-buffered)"}

    # device-side errors of every launch above (bounded waits, page ids) surface here
    cache.check_errors()
    if world > 1:
        dist.barrier()
        if cache.head_group is not None and cache.head_group.peer is not None:
            cache.head_group.peer.close()   # every rank is past its last peer store
        dist.destroy_process_group()
    if rank != 0:
        return 0

    peak, peak_kind = peaks()
    achieved = (kern_bytes / n_launch) / ((kern_ms / n_launch) / 1e3) / 1e9 if n_launch else 0.0
    tpb = traffic_per_byte()
    step_bytes = timer.all_bytes / max(args.steps, 1)
    value = seq_shards * B * args.steps / (ms / 1e3)
    line = {
        "metric": METRIC,
        "value": value,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms / args.steps,
        "higher_is_better": True,
        "scaling": "strong" if shard in ("heads", "split") else "weak",
        "vs_baseline": None,
        "dtype": "bf16" if w.dtype == torch.bfloat16 else "fp32",
        "data": "synthetic: seeded N(0,1) K/V/q, 1% planted query-aligned pages per head",
        "config": dict(workload_config(w, world, shard), **({} if len(layers) == L else {
            "layer_subset": f"{len(layers)} of {L} layers ({layers[0]}..{layers[-1]}, evenly "
                            f"spaced); tokens/s counts the timed layers only"})),
        "impl": "b200",
        "tokens_per_s_per_gpu": value / world,
        "retained_kv_gb_per_step": step_bytes / 1e9,
        "step_hbm_gbs": step_bytes / (ms / args.steps / 1e3) / 1e9,
        "roofline": {
            "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
            "frac": achieved / peak, "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
            "kernel": "rkv::sm100::decode_kernel (score+attend, and attend-only on compaction steps)",
            "launches": n_launch, "kernel_ms_total": kern_ms,
            "event_bracket": "each bracket holds the decode launch, its merge launch and the "
                             "gap to the next launch (an event also ends the programmatic "
                             "overlap of consecutive launches), so achieved is a lower bound "
                             "on the kernel's own rate",
            "timed_launches": f"CUDA events around each decode launch of every {timer.every}-th "
                              f"timed step ({n_launch} of {timer.all_launches} launches)",
            "traffic": (tpb * kern_bytes / n_launch) if (tpb and n_launch) else None,
        },
        "gpu_launches": int(launches),
        "compactions_timed": int(timed_compactions),
        "compactions_note": f"{timed_compactions} layer compactions in the {args.steps} timed "
                            f"steps x {len(layers)} layers (steady state: ~1 in 20-85 "
                            f"layer-steps, by layer depth)",
        "prefill_s": prefill_s,
        "host_enqueue_ms_per_step": host_ms / args.steps,
        "e2e": e2e,
        "clocks": clock_info,
    }
    if world == 1 and not args.no_cpu_baseline:
        try:
            del inputs
            res = oracle_sample(w, steps=2, warmup=0, threads=os.cpu_count(), parity_dev=dev)
            line["cpu_baseline"] = {k: res[k] for k in ("value", "unit", "cores", "kind", "sample")}
            line["cpu_baseline"]["ms_per_step_extrapolated"] = res["ms_per_step_est"]
            line["cpu_baseline"]["reference_torch_calibration"] = reference_calibration(w.name)
            line["parity"] = res.get("parity")
        except Exception as exc:  # report, never hide
            line["cpu_baseline"] = {"error": repr(exc)}
    print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
