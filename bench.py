"""Decode-step benchmark of the strict Top-K speculative path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--method saved|light|compact|repair_fused|signed_fused] [--overlap 0.9]

Headline workload: one request, 32 query / 8 KV heads,
head dim 128, bf16, 65,536-token context in 32-token blocks (2,048 blocks),
K = 64, predicted list = true Top-K with round((1 - overlap) * 64) IDs swapped
for seeded-random unselected blocks. Synthetic seeded inputs (Q ~ N(0,1);
K = N(0,1) + per-block N(0, 0.5^2) bias; V ~ N(0,1)); metadata lo/hi is the
per-block min/max of K, built outside timing.

A step is one full speculative decode step (strict Top-K selection and
predicted-block attention, then repair). The timed region runs exactly K steps
(``--steps``) bracketed by a barrier and a device synchronisation; it is
repeated until the repeats cover >= 200 ms, and the line reports the median
repeat (``repeats`` gives the count). Steps rotate over ``--sets``
independent input sets (default 8 x ~272 MiB, far above the 126 MB L2), so no
step finds its KV in L2.

With N > 1 (torchrun, one process per GPU) every rank decodes its own config-1
request (weak scaling, no collective in the data path); times are the max over
ranks. The same line also carries, measured at the same N:
  * ``batched``: BASELINE config 3, a batch of 64 paged requests split across
    the N ranks by LPT (strong scaling, no collective), strict and relaxed
    (max_extra_mass = 0.01);
  * ``hierarchical``: BASELINE config 2 (96 q / 8 KV heads, 4-token blocks,
    K 512 shared per group) through the gqa_hierarchical API, per call;
  * ``context_parallel``: BASELINE config 4, one 524,288-token request whose
    blocks are split across the N ranks, exchanged with two NCCL all-gathers,
    with its IDs checked bit for bit against single-GPU selection.
"""
from __future__ import annotations

import argparse
import csv
import io
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

HQ, HKV, D, BLOCKS, B, TOPK = 32, 8, 128, 2048, 32, 64
METRIC = "decode-step µs (score+topk+spec attn+repair) vs serial; HBM GB/s % of peak"
# Kernel launches per step: the fused step (saved / light, one persistent
# launch) and the launch chains of the other methods.
LAUNCHES_PER_STEP = {"saved": 1, "light": 1, "compact": 8, "repair_fused": 5, "signed_fused": 5}
MIN_TIMED_MS = 200.0


def parse():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--method", default="saved")
    ap.add_argument("--overlap", type=float, default=0.9)
    ap.add_argument("--sets", type=int, default=8)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--sweep", action="store_true", help="also time every method at overlap 1.0/0.9/0.75")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-batched", action="store_true", help="skip the config-3 object")
    ap.add_argument("--no-cp", action="store_true", help="skip the config-4 object")
    ap.add_argument("--no-c2", action="store_true", help="skip the config-2 object")
    ap.add_argument("--quick", action="store_true",
                    help="short run for profiler captures: no clock window, repeats, e2e, sweep, CPU baseline, "
                         "config-3 or config-4 objects")
    ap.add_argument("--graph-steps", type=int, default=8,
                    help="decode steps per CUDA graph in the timed loops (one per input set, like the attention "
                         "calls of consecutive layers of one token step); 1 = one graph per step")
    ap.add_argument("--workload", choices=("c1", "c2", "batched", "cp", "kernels"), default="c1",
                    help="c1: BASELINE config 1 (default, the headline, with the config-2, -3 and -4 objects); "
                         "c2 / batched / cp: only the config-2 / -3 / -4 measurement, as its own line; "
                         "kernels: one untimed eager pass over every kernel family (for profiler captures)")
    ap.add_argument("--requests", type=int, default=64, help="config 3: requests in the whole batch")
    ap.add_argument("--eager", action="store_true",
                    help="launch each step's kernels directly instead of replaying a CUDA graph (for per-kernel "
                         "profiler launch lists)")
    return ap.parse_args()


# ----------------------------------------------------------------------------- plumbing

def dist_setup(backend):
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        from datetime import timedelta
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        # NCCL writes its debug output (its version banner included) to stdout;
        # rank 0's stdout is the JSON line only.
        os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
        if backend == "nccl":
            torch.cuda.set_device(local)
            dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
        else:
            dist.init_process_group("gloo", timeout=timedelta(seconds=600))
    elif backend == "nccl":
        torch.cuda.set_device(local)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def all_reduce(x, world, device, op="max"):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op={"max": dist.ReduceOp.MAX, "min": dist.ReduceOp.MIN, "sum": dist.ReduceOp.SUM}[op])
    return float(t.item())


def max_over_ranks(x, world, device):
    return all_reduce(x, world, device, "max")


class ClockSampler:
    """nvidia-smi clock / throttle sampling (every 100 ms) around the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        if self.gpu < 0:
            return self
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.text = ""
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.text = self.proc.communicate(timeout=5)[0]
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.text = ""

    def summary(self):
        rows = []
        for r in csv.reader(io.StringIO(getattr(self, "text", ""))):
            if len(r) < 9:
                continue
            try:
                rows.append({"sm": float(r[1]), "max": float(r[2]), "power": float(r[3]),
                             "hw": r[5].strip(), "hwt": r[6].strip(), "swt": r[7].strip(), "pcap": r[8].strip()})
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        peak_power = max(r["power"] for r in rows)
        loaded = [r for r in rows if r["power"] >= 0.5 * peak_power] or rows
        reasons = set()
        for r in loaded:
            for key, name in (("hw", "hw_slowdown"), ("hwt", "hw_thermal_slowdown"), ("swt", "sw_thermal_slowdown"),
                              ("pcap", "sw_power_cap")):
                if r[key].lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r["sm"] for r in loaded), "sm_max_mhz": max(r["max"] for r in rows),
                "reasons": sorted(reasons), "samples": len(loaded), "power_w_max": peak_power}


def traffic_of(kernel):
    """DRAM bytes per launch of `kernel` from the committed ncu capture
    (profiles/roofline_traffic.json), or None."""
    p = ROOT / "profiles" / "roofline_traffic.json"
    try:
        return json.loads(p.read_text())[kernel]["dram_bytes_per_launch"]
    except (OSError, KeyError, ValueError):
        return None


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        j = json.loads(p.read_text())
        return float(j["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def time_loop(fn, steps, device, stream=None):
    """CUDA-event time (ms) of fn(0) .. fn(steps - 1), synchronised on both sides."""
    import torch
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(device)
    start.record(stream)
    for i in range(steps):
        fn(i)
    end.record(stream)
    end.synchronize()
    return start.elapsed_time(end)


def timed_repeats(run_k, world, device, min_ms=MIN_TIMED_MS, max_repeats=1000, quick=False):
    """Time run_k() (which runs exactly the K timed steps) bracketed by a
    barrier and a device synchronisation on both sides, max over ranks;
    repeat until the repeats cover min_ms. Every rank sees the same maxima,
    so every rank takes the same number of repeats (and collectives)."""
    import torch
    reps = []
    while True:
        barrier(world)
        torch.cuda.synchronize(device)
        ms = time_loop(lambda _: run_k(), 1, device)
        barrier(world)
        reps.append(max_over_ranks(ms, world, device))
        if quick or sum(reps) >= min_ms or len(reps) >= max_repeats:
            return reps


# ----------------------------------------------------------------------------- workload

def make_set(seed, overlap, device):
    """One seeded C1 input set on `device`, with its predicted list."""
    import torch
    from strict_topk import gqa
    g = torch.Generator(device=device).manual_seed(seed)
    q = torch.randn(HQ, D, device=device, generator=g).to(torch.bfloat16)
    k = torch.randn(HKV, BLOCKS, B, D, device=device, generator=g)
    k += torch.randn(HKV, BLOCKS, 1, D, device=device, generator=g) * 0.5
    k = k.to(torch.bfloat16)
    v = torch.randn(HKV, BLOCKS, B, D, device=device, generator=g).to(torch.bfloat16)
    lo, hi = k.amin(dim=2).float(), k.amax(dim=2).float()
    a = gqa.select_blocks(q, lo, hi, TOPK).cpu()
    p = swap_rows(a, BLOCKS, round((1 - overlap) * TOPK), seed + 7919).to(device)
    return {"q": q, "k": k, "v": v, "lo": lo, "hi": hi, "p": p, "a": a}


def swap_rows(a, n_blocks, nswap, seed, blocks_of_row=None):
    """Predicted list: each row of ``a`` with ``nswap`` IDs replaced by
    seeded-random unselected blocks of the row's request."""
    import torch
    gen = torch.Generator().manual_seed(seed)
    rows = []
    for i, row in enumerate(a.tolist()):
        n = blocks_of_row(i) if blocks_of_row else n_blocks
        ns = nswap(i) if callable(nswap) else nswap
        chosen = set(row)
        cand = torch.randperm(n, generator=gen).tolist()
        repl = [x for x in cand if x not in chosen][:ns]
        for j, x in zip(torch.randperm(len(row), generator=gen)[:ns].tolist(), repl):
            row[j] = x
        rows.append(row)
    return torch.tensor(rows, dtype=torch.int32)


def unique_blocks(ids, g):
    """Sum over KV heads of unique block IDs used by its query heads."""
    import torch
    total = 0
    for kv in range(ids.shape[0] // g):
        total += torch.unique(ids[kv * g:(kv + 1) * g].reshape(-1)).numel()
    return total


def graph_of(fn, device):
    """Warm fn up on a side stream, then capture it in a CUDA graph; returns (graph, fn's result)."""
    import torch
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize(device)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = fn()
    return g, out


# ----------------------------------------------------------------------------- reference arm

def run_reference(args):
    """Time the reference's CPU torch path (oracle/cpu_path.py) on this host."""
    import torch
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    torch.set_num_threads(os.cpu_count() or 1)
    from oracle.cpu_path import serial_step
    sys.path.insert(0, str(ROOT / "tests" / "golden"))
    import cases as C
    q, k, v, lo, hi = C.synthetic_kv(HQ, HKV, BLOCKS, B, D, torch.bfloat16, seed=args.seed)
    t0 = time.perf_counter()
    serial_step(q, k, v, lo, hi, TOPK)
    full = time.perf_counter() - t0
    budget_s = 60.0
    frac = min(1.0, budget_s / max(1e-9, (args.steps + args.warmup) * full))
    nh = max(1, min(HQ, int(math.floor(frac * HQ))))
    heads = list(range(nh))
    for _ in range(args.warmup):
        serial_step(q, k, v, lo, hi, TOPK, heads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        serial_step(q, k, v, lo, hi, TOPK, heads)
    dt = time.perf_counter() - t0
    step_s = dt / args.steps * (HQ / nh)  # full-step equivalent
    value = 1.0 / step_s
    sample = f"{nh}/{HQ} query heads per step, scaled to the full step; serial strict path (FP32 scores + topk, FP64 attention)"
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "decode-steps/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_s * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "BASELINE config 1: 32q/8kv, D128, 65536 tokens, 32-token blocks, K=64, bf16",
                       "path": "reference torch CPU path (benchmarks/run_benchmark.py:44-51 + critical_path.py:16-25)"},
            "cpu_baseline": {"value": value, "unit": "decode-steps/s", "cores": torch.get_num_threads(),
                             "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "decode-steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------- config 3 (batched)

def measure_batched(args, rank, world, device, quick=False):
    """a batch of ``--requests`` requests (context
    U[8192, 32768] tokens, multiple of 32; 16 query / 8 KV heads, D 128, bf16;
    paged KV, page 16, 32-token blocks; K 64; per-request predicted overlap ~
    Beta(8, 2)). Requests are split across ranks by greedy LPT on context
    length (paged.shard_requests); each rank builds its own page pool and
    decodes its requests, with no collective in the data path. A step is one
    batched decode step of the whole batch (one CUDA graph per rank); the
    serial step is selection then exact attention. Strict: saved speculation
    + saved repair; relaxed: hybrid speculation + fused repair with
    max_extra_mass = 0.01. Each rank's KV (~5 GB at N=1) is far above L2.
    Returns the object for the JSON line (rank 0) with times as max over ranks."""
    import torch
    from strict_topk_overlap_b200 import paged
    HQB, PAGE = 16, 16
    gen = torch.Generator().manual_seed(args.seed + 3)
    lengths = [int(x) // 32 * 32 for x in (8192 + torch.rand(args.requests, generator=gen) * (32768 - 8192)).tolist()]
    import numpy as np
    overlaps = np.random.default_rng(args.seed + 5).beta(8.0, 2.0, args.requests).tolist()
    mine = paged.shard_requests(lengths, world)[rank]
    ks, vs, qs = [], [], []
    for r in mine:
        g = torch.Generator(device=device).manual_seed(args.seed * 1000 + r)
        n = lengths[r] // B
        k = torch.randn(HKV, n, B, D, device=device, generator=g)
        k += torch.randn(HKV, n, 1, D, device=device, generator=g) * 0.5
        ks.append(k.to(torch.bfloat16))
        vs.append(torch.randn(HKV, n, B, D, device=device, generator=g).to(torch.bfloat16))
        qs.append(torch.randn(HQB, D, device=device, generator=g).to(torch.bfloat16))
        del k
    cache = paged.build_paged_cache(ks, vs, PAGE, generator=torch.Generator().manual_seed(args.seed + 11),
                                    device=device)
    del ks, vs
    q = torch.cat(qs, 0).contiguous()
    a = paged.select_blocks(q, cache, TOPK).cpu()
    p = swap_rows(a, 0, lambda i: round((1 - overlaps[mine[i // HQB]]) * TOPK), args.seed + 17,
                  blocks_of_row=lambda i: lengths[mine[i // HQB]] // B).to(device)
    eps = 0.01
    # Both speculative steps run as one launch chain over the whole batch
    # (paged.speculative_step: selection -> predicted states -> repair).
    ws_saved = paged.speculative_step_workspace(q, cache, p, "saved")
    ws_hybrid = paged.speculative_step_workspace(q, cache, p, "repair_fused")

    def spec():
        return paged.speculative_step(q, cache, p, TOPK, workspace=ws_saved)[0]

    def relaxed():
        return paged.speculative_step(q, cache, p, TOPK, variant="repair_fused", max_extra_mass=eps,
                                      workspace=ws_hybrid)[0]

    def serial():
        return paged.exact(q, cache, paged.select_blocks(q, cache, TOPK))

    graphs = {name: graph_of(fn, device) for name, fn in (("spec", spec), ("relaxed", relaxed), ("serial", serial))}
    for g, _ in graphs.values():
        g.replay()
    torch.cuda.synchronize(device)
    assert (graphs["spec"][1] - graphs["serial"][1]).abs().max().item() <= 2e-3
    steps = 5 if quick else 50
    times = {}
    for name, (g, _) in graphs.items():
        for _ in range(3):
            g.replay()

        def run_k(g=g):
            for _ in range(steps):
                g.replay()
        reps = timed_repeats(run_k, world, device, min_ms=50.0, quick=quick)
        times[name] = statistics.median(reps) / steps
    # Algorithmic bytes of the whole batch's speculative step (sum over ranks).
    blk = B * D * 2
    total_blocks = sum(lengths[r] // B for r in mine)
    ap = a.numpy()
    pn = p.cpu().numpy()
    g_ = HQB // HKV
    upred = unique_blocks(torch.from_numpy(pn), g_)
    miss = sum(len(set(x) - set(y)) for x, y in zip(ap.tolist(), pn.tolist()))
    step_bytes = 2 * HKV * total_blocks * D * 4 + 2 * blk * upred + 2 * blk * miss + q.numel() * 2 + q.numel() * 4
    step_bytes = all_reduce(step_bytes, world, device, "sum")
    hbm_peak, _ = peaks()
    tokens = sum(lengths[r] for r in mine)
    tok_max = all_reduce(tokens, world, device, "max")
    out = {
        "workload": f"BASELINE config 3: {args.requests} paged requests, context U[8192, 32768] tokens, 16q/8kv, "
                    "D128, page 16, 32-token blocks, K=64, overlap ~ Beta(8,2), bf16",
        "parallelism": f"requests split across {world} rank(s) by LPT, no collective", "ranks": world,
        "scaling": "strong", "steps_per_repeat": steps,
        "requests_per_s": args.requests / (times["spec"] / 1e3),
        "us_per_step": times["spec"] * 1e3, "serial_us_per_step": times["serial"] * 1e3,
        "speedup_vs_serial": times["serial"] / times["spec"],
        "relaxed": {"max_extra_mass": eps, "us_per_step": times["relaxed"] * 1e3,
                    "requests_per_s": args.requests / (times["relaxed"] / 1e3),
                    "speedup_vs_serial": times["serial"] / times["relaxed"]},
        "step_algorithmic_bytes": step_bytes,
        "hbm_frac": step_bytes / (times["spec"] * 1e-3) / 1e9 / (world * hbm_peak),
        "max_rank_tokens": int(tok_max),
    }
    graphs.clear()
    return out


# ----------------------------------------------------------------------------- config 4 (context parallel)

def measure_cp(args, rank, world, device, quick=False):
    """one request of 524,288 tokens (8192 blocks of 64),
    32 query / 8 KV heads, D 128, bf16, K 256, predicted overlap 0.7, its
    blocks split evenly across the ranks (context_parallel.decode_step:
    shard-local candidates -> NCCL all-gather -> global Top-K -> owned
    states -> NCCL all-gather -> merge). Every rank generates the whole
    request from one seed, keeps its shard and the full metadata, and checks
    the step's IDs bit for bit against a single-GPU selection of the whole
    request. Times: µs per step (max over ranks) and the two all-gathers of a
    step timed alone."""
    import torch
    from strict_topk import gqa
    from strict_topk_overlap_b200.context_parallel import ProcessGroupComm, decode_step, shard_range
    hq, hkv, n, b, d, topk = 32, 8, 8192, 64, 128, 256
    g = torch.Generator(device=device).manual_seed(args.seed + 4444)
    q = torch.randn(hq, d, device=device, generator=g).to(torch.bfloat16)
    s, e = shard_range(n, rank, world)
    ks, vs, los, his = [], [], [], []
    for h in range(hkv):  # one KV head at a time keeps the FP32 temporaries small
        kh = torch.randn(n, b, d, device=device, generator=g)
        kh += torch.randn(n, 1, d, device=device, generator=g) * 0.5
        kh = kh.to(torch.bfloat16)
        vh = torch.randn(n, b, d, device=device, generator=g).to(torch.bfloat16)
        los.append(kh.amin(dim=1).float())
        his.append(kh.amax(dim=1).float())
        ks.append(kh[s:e].clone())
        vs.append(vh[s:e].clone())
        del kh, vh
    k = torch.stack(ks).contiguous()
    v = torch.stack(vs).contiguous()
    lo_full = torch.stack(los).contiguous()
    hi_full = torch.stack(his).contiguous()
    del ks, vs, los, his
    lo, hi = lo_full[:, s:e].contiguous(), hi_full[:, s:e].contiguous()
    single = gqa.select_blocks(q, lo_full, hi_full, topk)
    pred = swap_rows(single.cpu(), n, round(0.3 * topk), args.seed + 45).to(device)
    comm = ProcessGroupComm()
    side = torch.cuda.Stream(device)
    out, sel = decode_step(q, k, v, lo, hi, topk, n, predicted=pred, comm=comm, side_stream=side)
    torch.cuda.synchronize(device)
    exact_ids = all_reduce(float(torch.equal(sel, single)), world, device, "min") == 1.0
    steps = 5 if quick else 20

    def run_k(strict=False):
        for _ in range(steps):
            decode_step(q, k, v, lo, hi, topk, n, predicted=None if strict else pred, comm=comm, side_stream=side)
    for _ in range(3):
        run_k()
    reps = timed_repeats(run_k, world, device, min_ms=50.0, quick=quick)
    us = statistics.median(reps) / steps * 1e3
    reps_s = timed_repeats(lambda: run_k(strict=True), world, device, min_ms=50.0, quick=quick)
    us_strict = statistics.median(reps_s) / steps * 1e3
    # The step's exchanges alone: candidates (keys int64 + IDs int32) and states (m, l, u FP32).
    keys = torch.zeros((hq, topk), dtype=torch.int64, device=device)
    ids = torch.zeros((hq, topk), dtype=torch.int32, device=device)
    ms_, ls_ = torch.zeros(hq, device=device), torch.zeros(hq, device=device)
    us_ = torch.zeros((hq, d), device=device)

    def exchange():
        for _ in range(steps):
            for t in (keys, ids, ms_, ls_, us_):
                comm.all_gather(t)
    exchange()
    reps_c = timed_repeats(exchange, world, device, min_ms=20.0, quick=quick)
    coll_us = statistics.median(reps_c) / steps * 1e3
    return {
        "workload": "BASELINE config 4: 1 request, 524288 tokens in 8192 blocks of 64, 32q/8kv, D128, K=256, "
                    "overlap 0.7, bf16",
        "parallelism": f"context split over {world} rank(s), NCCL all-gathers of candidates and (m, l, u) states",
        "ranks": world, "scaling": "strong", "steps_per_repeat": steps,
        "us_per_step": us, "strict_us_per_step": us_strict,
        "collective_us_per_step": coll_us if world > 1 else 0.0,
        "ids_bit_exact_vs_1gpu": bool(exact_ids),
        "launch": "eager (host-orchestrated; each all-gather is one NCCL call per tensor)",
    }


# ----------------------------------------------------------------------------- config 2 (wide GQA, tiny blocks)

def measure_c2(args, device, quick=False):
    """96 query / 8 KV heads (12 per group), D 128, bf16,
    32,768 tokens in 8192 blocks of 4, K = 512 blocks shared per group,
    predicted overlap 0.8, through the reference's gqa_hierarchical API:
    shared selection, partials over P, repair_saved_shared (the speculative
    step's parts), exact over A (the serial step's attention), and the
    tensor-core exact_shared. Each call is timed alone in a CUDA graph of
    `nset` calls on rotating input sets (> L2), CUDA events."""
    import torch
    from strict_topk import gqa_hierarchical as GH
    hq, hkv, n, b, d, topk = 96, 8, 8192, 4, 128, 512
    g = hq // hkv
    nset = 4
    sets = []
    for i in range(nset):
        gen = torch.Generator(device=device).manual_seed(args.seed + 200 + i)
        q = torch.randn(hq, d, device=device, generator=gen).to(torch.bfloat16)
        k = (torch.randn(hkv, n, b, d, device=device, generator=gen)
             + torch.randn(hkv, n, 1, d, device=device, generator=gen) * 0.5).to(torch.bfloat16)
        v = torch.randn(hkv, n, b, d, device=device, generator=gen).to(torch.bfloat16)
        lo, hi = k.amin(dim=2).float(), k.amax(dim=2).float()
        a = GH.select_blocks_shared(q, lo, hi, topk)
        pg = swap_rows(a[::g].cpu(), n, round(0.2 * topk), args.seed + 300 + i)
        p = pg.repeat_interleave(g, dim=0).contiguous().to(device)
        sets.append(dict(q=q, k=k, v=v, lo=lo, hi=hi, a=a, p=p, ag=a[::g].contiguous(),
                         st=GH.partials(q, k, v, p)))
    calls = {
        "select_shared": lambda s: GH.select_blocks_shared(s["q"], s["lo"], s["hi"], topk),
        "partials": lambda s: GH.partials(s["q"], s["k"], s["v"], s["p"]),
        "repair_saved_shared": lambda s: GH.repair_saved_shared(s["q"], s["k"], s["v"], s["a"], s["p"], s["st"]),
        "exact": lambda s: GH.exact(s["q"], s["k"], s["v"], s["a"]),
        "exact_shared": lambda s: GH.exact_shared(s["q"], s["k"], s["v"], s["ag"]),
    }
    res = {}
    for name, fn in calls.items():
        gr, _ = graph_of(lambda: [fn(s) for s in sets], device)
        for _ in range(3):
            gr.replay()
        nrep = 3 if quick else 30
        ms = time_loop(lambda i: gr.replay(), nrep, device)
        res[name] = ms * 1e3 / (nrep * nset)
        del gr
    hbm_peak, _ = peaks()
    meta = 2 * hkv * n * d * 4
    kv_sel = 2 * hkv * topk * b * d * 2  # unique K+V of the group-shared selection
    miss = sum(len(set(x) - set(y)) for x, y in zip(sets[0]["ag"].tolist(), sets[0]["p"][::g].tolist()))
    out = {"workload": "BASELINE config 2: 96q/8kv, D128, 8192 blocks of 4 tokens, K=512 shared per group, "
                       "overlap 0.8, bf16", "us": {k: round(v, 2) for k, v in res.items()},
           "algorithmic_bytes": {"select_shared": meta, "exact": kv_sel, "partials": kv_sel,
                                 "repair_saved_shared": 2 * b * d * 2 * miss},
           "hbm_frac": {"select_shared": meta / (res["select_shared"] * 1e-6) / 1e9 / hbm_peak,
                        "exact": kv_sel / (res["exact"] * 1e-6) / 1e9 / hbm_peak,
                        "exact_shared": kv_sel / (res["exact_shared"] * 1e-6) / 1e9 / hbm_peak},
           # The serial step's attention over the shared lists is the tensor-core group tile
           # (exact_shared); the per-head exact is reported beside it.
           "step_us": {"speculative": res["select_shared"] + max(0.0, res["partials"]) + res["repair_saved_shared"],
                       "serial": res["select_shared"] + res["exact_shared"],
                       "serial_per_head": res["select_shared"] + res["exact"]},
           "timing": f"each call alone, CUDA graph of {nset} calls on rotating inputs (> L2), CUDA events"}
    del sets
    return out


def run_kernels(args, device):
    """One eager pass over every kernel family of the library, on config-1
    inputs (and small config-2 / -3 / -4 shapes), for profiler launch lists
    and captures: the fused step, the saved, hybrid (fused and signed fused)
    and compact speculation with their repairs, the split repair, the
    hierarchical (config 2) calls with the tensor-core group attention, the
    batched paged chain, metadata building and token append, and the
    context-parallel candidate and state merges. Nothing is timed."""
    import torch
    from strict_topk import gqa, gqa_hierarchical as GH, kernels
    from strict_topk_overlap_b200 import context_parallel, decode, metadata, paged
    ran = []
    s = make_set(args.seed, 0.9, device)
    q, k, v, lo, hi, p = s["q"], s["k"], s["v"], s["lo"], s["hi"], s["p"]
    decode.decode_step(q, k, v, lo, hi, TOPK, p)
    decode.decode_step(q, k, v, lo, hi, TOPK, None)
    ran += ["decode_step (speculative, serial)"]
    decode.speculative_step(q, k, v, lo, hi, p, TOPK)
    for variant in ("repair_fused", "signed_fused"):
        decode.speculative_step_hybrid(q, k, v, lo, hi, p, TOPK, variant=variant, max_extra_mass=0.01)
    ran += ["speculative_step", "speculative_step_hybrid (repair_fused, signed_fused)"]
    a = gqa.select_blocks(q, lo, hi, TOPK)
    pc = kernels.speculate(q, k, v, p, mode="compact", mass_threshold=0.1)
    kernels.repair(q, k, v, a, p, pc)
    gqa.exact(q, k, v, a)
    ran += ["compact speculation + split repair", "exact"]
    lo2, hi2 = metadata.build_metadata(k)
    metadata.append_token(k.clone(), v.clone(), lo2, hi2, k[:, 0, 0].contiguous(), v[:, 0, 0].contiguous(), 5)
    ran += ["build_metadata", "append_token"]
    del s, q, k, v, lo, hi, p, a, pc, lo2, hi2
    torch.cuda.empty_cache()  # a profiler saves and restores what stays allocated
    # Config 2 (one input set): the hierarchical API and the tensor-core group attention.
    hq2, hkv2, n2, b2, d2, k2 = 96, 8, 8192, 4, 128, 512
    gen = torch.Generator(device=device).manual_seed(args.seed + 200)
    q2 = torch.randn(hq2, d2, device=device, generator=gen).to(torch.bfloat16)
    kk = (torch.randn(hkv2, n2, b2, d2, device=device, generator=gen)
          + torch.randn(hkv2, n2, 1, d2, device=device, generator=gen) * 0.5).to(torch.bfloat16)
    vv = torch.randn(hkv2, n2, b2, d2, device=device, generator=gen).to(torch.bfloat16)
    lo2, hi2 = kk.amin(dim=2).float(), kk.amax(dim=2).float()
    a2 = GH.select_blocks_shared(q2, lo2, hi2, k2)
    g2 = hq2 // hkv2
    p2 = swap_rows(a2[::g2].cpu(), n2, round(0.2 * k2), args.seed + 300).repeat_interleave(g2, 0).contiguous().to(device)
    st2 = GH.partials(q2, kk, vv, p2)
    GH.repair_saved_shared(q2, kk, vv, a2, p2, st2)
    GH.exact(q2, kk, vv, a2)
    GH.exact_shared(q2, kk, vv, a2[::g2].contiguous())
    ran += ["config 2: select_blocks_shared, partials, repair_saved_shared, exact, exact_shared"]
    del q2, kk, vv, lo2, hi2, a2, p2, st2
    torch.cuda.empty_cache()
    # Config 3 shape, 8 requests: the batched paged chain, strict and relaxed.
    gen = torch.Generator().manual_seed(args.seed + 3)
    lengths = [int(x) // 32 * 32 for x in (8192 + torch.rand(8, generator=gen) * (32768 - 8192)).tolist()]
    ks, vs, qs = [], [], []
    for r, ln in enumerate(lengths):
        gd = torch.Generator(device=device).manual_seed(r)
        kt = torch.randn(HKV, ln // B, B, D, device=device, generator=gd)
        kt += torch.randn(HKV, ln // B, 1, D, device=device, generator=gd) * 0.5
        ks.append(kt.to(torch.bfloat16))
        vs.append(torch.randn(HKV, ln // B, B, D, device=device, generator=gd).to(torch.bfloat16))
        qs.append(torch.randn(16, D, device=device, generator=gd).to(torch.bfloat16))
    cache = paged.build_paged_cache(ks, vs, 16, generator=torch.Generator().manual_seed(11), device=device)
    q3 = torch.cat(qs, 0).contiguous()
    a3 = paged.select_blocks(q3, cache, TOPK).cpu()
    p3 = swap_rows(a3, 0, 8, args.seed + 17, blocks_of_row=lambda i: lengths[i // 16] // B).to(device)
    paged.speculative_step(q3, cache, p3, TOPK)
    paged.speculative_step(q3, cache, p3, TOPK, variant="repair_fused", max_extra_mass=0.01)
    paged.exact(q3, cache, paged.select_blocks(q3, cache, TOPK))
    ran += ["config 3 (8 requests): paged speculative_step saved / repair_fused, exact"]
    del ks, vs, qs, cache, q3
    torch.cuda.empty_cache()
    # Config 4 shape on one rank: shard candidates, candidate merge, state reduce and merge.
    cp = measure_cp(args, 0, 1, device, quick=True)
    ran += [f"config 4 (one rank): {cp['workload']}"]
    torch.cuda.synchronize(device)
    return {"ran": ran}


def run_single_workload(args):
    import torch
    rank, world, local = dist_setup("nccl")
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if args.workload == "kernels":
        obj = run_kernels(args, device)
    elif args.workload == "c2":
        obj = measure_c2(args, device, quick=args.quick)
    else:
        fn = measure_batched if args.workload == "batched" else measure_cp
        obj = fn(args, rank, world, device, quick=args.quick)
    if rank == 0:
        print(json.dumps({"workload": args.workload, "n_gpus": world, **obj}), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


# ----------------------------------------------------------------------------- config 1 (headline)

def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    if args.workload != "c1":
        return run_single_workload(args)
    import torch
    rank, world, local = dist_setup("nccl")
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    from strict_topk_overlap_b200 import _lib
    _lib.load()
    from strict_topk import gqa
    from strict_topk_overlap_b200.decode import SpeculativeDecoder, StepSpec, capture_steps

    nsets = args.sets
    sets = [make_set(args.seed + 1000 * rank + i, args.overlap, device) for i in range(nsets)]
    spec = StepSpec(topk=TOPK, method=args.method, max_extra_mass=0.0)
    graph = not args.eager
    dec = [SpeculativeDecoder(s["q"], s["k"], s["v"], s["lo"], s["hi"], s["p"], spec, graph=graph) for s in sets]
    ser = [SpeculativeDecoder(s["q"], s["k"], s["v"], s["lo"], s["hi"], s["p"], spec, serial=True, graph=graph,
                              fused=True) for s in sets]
    # The same steps as launch chains (scorer -> Top-K -> states / exact ->
    # repair): the serial baseline is the faster of the two serial forms.
    ser_chain = [SpeculativeDecoder(s["q"], s["k"], s["v"], s["lo"], s["hi"], s["p"], spec, serial=True, graph=graph,
                                    fused=False) for s in sets]
    dec_chain = [SpeculativeDecoder(s["q"], s["k"], s["v"], s["lo"], s["hi"], s["p"], spec, graph=graph, fused=False)
                 for s in sets]
    # Correctness gate before timing: speculative == serial within bf16 tolerance, IDs identical.
    for d_, s_, c_, e_ in zip(dec, ser, ser_chain, dec_chain):
        o1 = d_.step().clone()
        o2 = s_.step().clone()
        o3 = c_.step().clone()
        o4 = e_.step().clone()
        torch.cuda.synchronize()
        for x in (s_, c_, e_):
            assert torch.equal(d_.selected.cpu(), x.selected.cpu())
        for o in (o2, o3, o4):
            assert (o1 - o).abs().max().item() <= 2e-3, "speculative and serial outputs differ"

    # Exactly K steps per timed region: K // gsteps graphs of `gsteps`
    # consecutive decode steps (one per input set), then K % gsteps
    # single-step graphs, continuing the rotation.
    gsteps = max(1, min(args.graph_steps, nsets)) if graph else 1
    K = max(1, args.steps)
    def graphs_of(decs):
        return [capture_steps([decs[(j + i) % nsets] for i in range(gsteps)])[0] for j in range(0, nsets, gsteps)]

    if gsteps > 1:
        gspec, gser, gser_chain, gspec_chain = graphs_of(dec), graphs_of(ser), graphs_of(ser_chain), graphs_of(dec_chain)
    else:
        gspec = gser = gser_chain = gspec_chain = None

    def run_steps(decs, graphs, count):
        full, rest = divmod(count, gsteps) if graphs else (0, count)
        for i in range(full):
            graphs[i % len(graphs)].replay()
        for i in range(rest):
            decs[(full * gsteps + i) % nsets].step()

    hbm_peak, peak_kind = peaks()
    run_steps(dec, gspec, max(args.warmup, 3 * gsteps))
    torch.cuda.synchronize()
    with ClockSampler(local if not args.quick else -1) as clk:
        t_end = time.perf_counter() + (0.0 if args.quick else 1.0)
        while time.perf_counter() < t_end:
            run_steps(dec, gspec, 200)
            torch.cuda.synchronize()
        reps = timed_repeats(lambda: run_steps(dec, gspec, K), world, device, quick=args.quick)
    ms = statistics.median(reps)
    us_step = ms * 1e3 / K
    value = world * K / (ms / 1e3)
    clocks = clk.summary()

    # Serial baselines with the same kernels (same rotation and repeats):
    # the fused serial step and the serial launch chain; the faster one is
    # the baseline. The speculative launch chain is reported beside them.
    variants = {}
    for name, decs, gr in (("serial_fused", ser, gser), ("serial_chained", ser_chain, gser_chain),
                           ("speculative_chained", dec_chain, gspec_chain)):
        run_steps(decs, gr, 3 * gsteps)
        rp = timed_repeats(lambda: run_steps(decs, gr, K), world, device, quick=args.quick)
        variants[name] = statistics.median(rp) * 1e3 / K
    variants["speculative_fused"] = us_step
    us_ser = min(variants["serial_fused"], variants["serial_chained"])
    # Context: one CUDA graph per step (graph-launch cost paid every step).
    single = {}
    if graph and gsteps > 1 and not args.quick:
        n1 = min(K * 10, 2000)
        single = {"spec_us": time_loop(lambda i: dec[i % nsets].step(), n1, device) * 1e3 / n1,
                  "serial_us": min(time_loop(lambda i: ser[i % nsets].step(), n1, device),
                                   time_loop(lambda i: ser_chain[i % nsets].step(), n1, device)) * 1e3 / n1}

    # Roofline of the dominant kernel: predicted-block attention (block states over P).
    g = HQ // HKV
    blk = B * D * 2
    pstates = [None] * nsets

    # The dominant kernel timed alone: one CUDA graph of `nsets` launches
    # (one per input set, so no launch finds its KV in L2), replayed; CUDA
    # events on the launching stream around the replays.
    def partials_all():
        for i in range(nsets):
            s = sets[i]
            pstates[i] = gqa.partials(s["q"], s["k"], s["v"], s["p"])

    if graph:
        partials_all()
        torch.cuda.synchronize()
        gpart = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gpart):
            partials_all()
        run_part = lambda i: gpart.replay()  # noqa: E731
    else:
        run_part = lambda i: partials_all()  # noqa: E731
    for i in range(5):
        run_part(i)
    nrep = 3 if args.quick else max(50, min(K // nsets, 1000))
    ms_part = time_loop(run_part, nrep, device, torch.cuda.current_stream())
    us_part = ms_part * 1e3 / (nrep * nsets)
    upred = statistics.mean(unique_blocks(s["p"].cpu(), g) for s in sets)
    # Algorithmic bytes: unique (KV head, block) K+V of P, Q and the IDs read;
    # the per-block states written are intermediate and not counted.
    part_bytes = 2 * blk * upred + HQ * D * 2 + HQ * TOPK * 4
    achieved = part_bytes / (us_part * 1e-6) / 1e9

    # Whole-step algorithmic bytes (score + predicted + misses), for context.
    score_bytes = 2 * HKV * BLOCKS * D * 4 + HQ * D * 2 + HQ * TOPK * 4
    ua = statistics.mean(unique_blocks(torch.as_tensor(s["a"]), g) for s in sets)
    miss = statistics.mean(
        sum(len(set(a_) - set(p_)) for a_, p_ in zip(s["a"].tolist(), s["p"].cpu().tolist())) for s in sets)
    step_bytes = score_bytes + 2 * blk * upred + 2 * blk * miss + HQ * D * 4
    serial_bytes = score_bytes + 2 * blk * ua + HQ * D * 4

    # End to end through the public API with host buffers: every step copies
    # its q and P in from pinned host memory and its output back to pinned
    # host memory (decode.capture_host_steps: the graphs hold `gsteps` such
    # steps, one per input set); the host reads every step's output, double-
    # buffered (it reads one graph's outputs while the next graph runs).
    e2e_value = None
    if graph and not args.quick:
        from strict_topk_overlap_b200.decode import capture_host_steps
        hq_pin = [s["q"].cpu().pin_memory() for s in sets]
        hp_pin = [s["p"].cpu().pin_memory() for s in sets]
        houts = [[torch.empty(HQ, D, dtype=torch.float32).pin_memory() for _ in range(gsteps)] for _ in range(2)]
        hgraphs = [capture_host_steps([dec[j % nsets] for j in range(gsteps)], hq_pin[:gsteps], hp_pin[:gsteps],
                                      houts[b]) for b in range(2)]
        evs = [torch.cuda.Event() for _ in range(2)]

        def e2e_steps(count):
            sink = 0.0
            for i in range(count // gsteps):
                b = i % 2
                hgraphs[b].replay()
                evs[b].record()
                if i > 0:
                    evs[1 - b].synchronize()
                    sink += sum(float(h[0, 0]) for h in houts[1 - b])
            torch.cuda.current_stream().synchronize()
            return sink

        e2e_steps(4 * gsteps)
        n_e2e = max(200, min(K, 5000)) // gsteps * gsteps
        barrier(world)
        t0 = time.perf_counter()
        e2e_steps(n_e2e)
        e2e_s = max_over_ranks(time.perf_counter() - t0, world, device)
        e2e_value = world * n_e2e / e2e_s
        del hgraphs
        torch.cuda.synchronize()

    sweep = {}
    if args.sweep and not args.quick:
        for method in ("saved", "light", "compact", "repair_fused", "signed_fused"):
            for ov in (1.0, 0.9, 0.75):
                ss = [make_set(args.seed + 500 + i, ov, device) for i in range(4)]
                dd = [SpeculativeDecoder(s["q"], s["k"], s["v"], s["lo"], s["hi"], s["p"],
                                         StepSpec(topk=TOPK, method=method)) for s in ss]
                rr = [SpeculativeDecoder(s["q"], s["k"], s["v"], s["lo"], s["hi"], s["p"],
                                         StepSpec(topk=TOPK, method=method), serial=True) for s in ss]
                n = 2000
                for i in range(100):
                    dd[i % 4].graph.replay()
                a_ = time_loop(lambda i: dd[i % 4].graph.replay(), n, device) * 1e3 / n
                b_ = time_loop(lambda i: rr[i % 4].graph.replay(), n, device) * 1e3 / n
                sweep[f"{method}@{ov:g}"] = {"spec_us": round(a_, 2), "serial_us": round(b_, 2),
                                              "speedup": round(b_ / a_, 3)}
                del dd, rr, ss

    # Config 2 on each rank's own GPU (rank 0 reports it); config 3 and
    # config 4 at the same N (every rank takes part).
    c2 = None
    if not args.quick and not args.no_c2:
        del pstates
        pstates = None
        c2 = measure_c2(args, device)
        torch.cuda.empty_cache()
    batched = cp = None
    if not args.quick and not args.no_batched:
        batched = measure_batched(args, rank, world, device)
        torch.cuda.empty_cache()
    if not args.quick and not args.no_cp:
        cp = measure_cp(args, rank, world, device)
        torch.cuda.empty_cache()

    cpu = None
    if rank == 0 and not args.no_cpu_baseline and not args.quick:
        from oracle.cpu_path import serial_step as cpu_step
        s0 = sets[0]
        torch.set_num_threads(os.cpu_count() or 1)
        cq, ck, cv, clo, chi = (s0[x].cpu() for x in ("q", "k", "v", "lo", "hi"))
        cpu_step(cq, ck, cv, clo, chi, TOPK)
        t0 = time.perf_counter()
        nc = 0
        while time.perf_counter() - t0 < 10.0 and nc < 200:
            cpu_step(cq, ck, cv, clo, chi, TOPK)
            nc += 1
        cdt = (time.perf_counter() - t0) / nc
        cpu = {"value": 1.0 / cdt, "unit": "decode-steps/s", "cores": torch.get_num_threads(), "kind": "port",
               "sample": f"{nc} full C1 serial strict steps (FP32 bound scores + topk, FP64 attention) on input set 0"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "decode-steps/s", "n_gpus": world, "steps": K,
            "warmup": args.warmup, "ms_per_step": ms / K, "us_per_step": us_step,
            "repeats": len(reps), "timed_ms_total": sum(reps), "repeat_ms_min_max": [min(reps), max(reps)],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded; BASELINE config 1 distribution)",
            "config": {"workload": "BASELINE config 1: 1 request, 32q/8kv, D128, 65536 tokens, 32-token blocks, "
                                   "K=64, bf16", "method": args.method, "predicted_overlap": args.overlap,
                       "l2": f"{nsets} rotating input sets x {(2 * HKV * BLOCKS * B * D * 2 + 2 * HKV * BLOCKS * D * 4) / 2**20:.0f} MiB (> 126 MB L2)",
                       "parallelism": f"request replicas x{world} (no collective in the data path)",
                       "timing": (f"each repeat: exactly {K} steps between barrier + synchronize, CUDA events, max "
                                  f"over ranks; repeated to >= {MIN_TIMED_MS:.0f} ms, median reported"),
                       "graph": (f"{gsteps} decode steps per CUDA graph (one per input set, replayed; each step one "
                                 "launch chain)") if gsteps > 1 else "one CUDA graph per step"},
            "serial_us_per_step": us_ser, "speedup_vs_serial": us_ser / us_step,
            "us_per_step_variants": variants,
            "one_graph_per_step_us": single or None,
            "step_algorithmic_bytes": step_bytes, "serial_algorithmic_bytes": serial_bytes,
            "step_hbm_frac": step_bytes / (us_step * 1e-6) / 1e9 / hbm_peak,
            "serial_hbm_frac": serial_bytes / (us_ser * 1e-6) / 1e9 / hbm_peak,
            # The step is one launch of the fused kernel: its algorithmic bytes
            # (metadata, predicted and missed K/V, q, IDs, output) over the
            # step time (graph-replayed, launch gaps included).
            "roofline": {"bound": "hbm", "kernel": "decode_step_kernel (fused speculative step: scoring, Top-K, "
                                                   "predicted-block states, saved repair)",
                         "achieved": step_bytes / (us_step * 1e-6) / 1e9, "peak": hbm_peak, "unit": "GB/s",
                         "frac": step_bytes / (us_step * 1e-6) / 1e9 / hbm_peak, "peak_kind": peak_kind,
                         "us_per_launch": us_step, "bytes_per_launch": step_bytes,
                         "traffic": traffic_of("decode_step_kernel")},
            # The predicted-block attention kernel of the launch-chain path
            # (gqa.partials) timed alone.
            "roofline_attention": {"bound": "hbm", "kernel": "jobs_fast_kernel (predicted-block attention, "
                                                             "gqa.partials)",
                                   "achieved": achieved, "peak": hbm_peak, "unit": "GB/s", "frac": achieved / hbm_peak,
                                   "peak_kind": peak_kind, "us_per_launch": us_part, "bytes_per_launch": part_bytes,
                                   "traffic": traffic_of("jobs_fast_kernel")},
            "clocks": clocks,
            "e2e": {"value": e2e_value, "unit": "decode-steps/s", "h2d_bytes_per_step": HQ * D * 2 + HQ * TOPK * 4,
                    "d2h_bytes_per_step": HQ * D * 4,
                    "path": "decode.capture_host_steps: per step the pinned H2D of q and P, the step and the D2H of "
                            "its output, graphs of consecutive steps with the copies on side streams (step i's copies "
                            "overlap the other steps); the host reads every step's output"},
            "gpu_launches": LAUNCHES_PER_STEP.get(args.method, 4) * K * len(reps),
            "cpu_baseline": cpu,
        }
        if c2:
            line["hierarchical"] = c2
        if batched:
            line["batched"] = batched
        if cp:
            line["context_parallel"] = cp
        if sweep:
            line["sweep"] = sweep
        print(json.dumps(line), flush=True)
    for d_ in dec + ser + ser_chain + dec_chain:
        d_.close()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
