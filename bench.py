"""Decode-step benchmark of the strict Top-K speculative path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--method saved|light|compact|repair_fused|signed_fused] [--overlap 0.9]

Workload: one request, 32 query / 8 KV heads, head dim
128, bf16, 65,536-token context in 32-token blocks (2,048 blocks), K = 64,
predicted list = true Top-K with round((1 - overlap) * 64) IDs swapped for
seeded-random unselected blocks. Synthetic seeded inputs (Q ~ N(0,1);
K = N(0,1) + per-block N(0, 0.5^2) bias; V ~ N(0,1)); metadata lo/hi is the
per-block min/max of K, built outside timing.

A step is one full speculative decode step (strict Top-K selection ||
predicted-block attention, then repair), replayed as one CUDA graph. Steps
rotate over ``--sets`` independent input sets (default 8 x ~272 MiB, far
above the 126 MB L2), so no step finds its KV in L2.

With N > 1 (torchrun, one process per GPU) every rank decodes its own
request (weak scaling, no collective in the data path); the timed region is
bracketed by barriers and the reported time is the max over ranks.
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
LAUNCHES_PER_STEP = {"saved": 4, "light": 4, "compact": 8, "repair_fused": 5, "signed_fused": 5}


def parse():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=200)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--method", default="saved")
    ap.add_argument("--overlap", type=float, default=0.9)
    ap.add_argument("--sets", type=int, default=8)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--sweep", action="store_true", help="also time every method at overlap 1.0/0.9/0.75")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--quick", action="store_true",
                    help="short run for profiler captures: no clock window, e2e, sweep or CPU baseline")
    ap.add_argument("--graph-steps", type=int, default=8,
                    help="decode steps per CUDA graph in the timed loops (one per input set, like the attention "
                         "calls of consecutive layers of one token step); 1 = one graph per step")
    ap.add_argument("--workload", choices=("c1", "batched"), default="c1",
                    help="c1: BASELINE config 1 (default, the headline); batched: BASELINE config 3, a batch of "
                         "paged requests split across the ranks")
    ap.add_argument("--requests", type=int, default=64, help="batched workload: requests in the whole batch")
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


def max_over_ranks(x, world, device):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


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
    nswap = round((1 - overlap) * TOPK)
    gen = torch.Generator().manual_seed(seed + 7919)
    rows = []
    for row in a.tolist():
        chosen = set(row)
        pool = [x for x in range(BLOCKS) if x not in chosen]
        repl = [pool[i] for i in torch.randperm(len(pool), generator=gen)[:nswap].tolist()]
        pos = torch.randperm(TOPK, generator=gen)[:nswap].tolist()
        for j, r in zip(pos, repl):
            row[j] = r
        rows.append(row)
    p = torch.tensor(rows, dtype=torch.int32, device=device)
    return {"q": q, "k": k, "v": v, "lo": lo, "hi": hi, "p": p, "a": a}


def unique_blocks(ids, g):
    """Sum over KV heads of unique block IDs used by its query heads."""
    import torch
    total = 0
    for kv in range(ids.shape[0] // g):
        total += torch.unique(ids[kv * g:(kv + 1) * g].reshape(-1)).numel()
    return total


def time_loop(fn, steps, device, stream=None):
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


# ----------------------------------------------------------------------------- our arm

def run_batched(args):
    """a batch of `--requests` requests (context U[8192, 32768]
    tokens, multiple of 32; 16 query / 8 KV heads, D 128, bf16; paged KV, page
    16, 32-token blocks; K 64; per-request predicted overlap ~ Beta(8, 2)).
    Requests are split across ranks by greedy LPT on context length
    (paged.shard_requests); each rank builds its own page pool and decodes its
    requests, with no collective in the data path. A step is one batched
    speculative step (selection || predicted-block states, then saved repair,
    one CUDA graph); the serial step is selection then exact attention. Each
    rank's KV (~5 GB at N=1) is far above L2. value = requests decoded per
    second over the whole job (all ranks), from the max over ranks."""
    import torch
    rank, world, local = dist_setup("nccl")
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    from strict_topk_overlap_b200 import paged
    from strict_topk_overlap_b200.decode import overlap_run
    HQB, PAGE = 16, 16
    gen = torch.Generator().manual_seed(args.seed + 3)
    lengths = [int(x) // 32 * 32 for x in (8192 + torch.rand(args.requests, generator=gen) * (32768 - 8192)).tolist()]
    torch.manual_seed(args.seed + 5)
    overlaps = torch.distributions.Beta(8.0, 2.0).sample((args.requests,)).tolist()
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
    pg = torch.Generator().manual_seed(args.seed + 17)
    rows = []
    for i, row in enumerate(a.tolist()):
        r = mine[i // HQB]
        n = lengths[r] // B
        nswap = round((1 - overlaps[r]) * TOPK)
        chosen = set(row)
        cand = torch.randperm(n, generator=pg).tolist()
        repl = [x for x in cand if x not in chosen][:nswap]
        for j, x in zip(torch.randperm(TOPK, generator=pg)[:nswap].tolist(), repl):
            row[j] = x
        rows.append(row)
    p = torch.tensor(rows, dtype=torch.int32, device=device)
    s_sel = torch.cuda.Stream(device, priority=-1)
    s_pred = torch.cuda.Stream(device)

    def spec():
        return overlap_run(lambda: paged.select_blocks(q, cache, TOPK), lambda: paged.partials(q, cache, p),
                           lambda sel, st: paged.repair_saved(q, cache, sel, p, st), s_sel, s_pred)

    def serial():
        return paged.exact(q, cache, paged.select_blocks(q, cache, TOPK))

    graphs = {}
    for name, fn in (("spec", spec), ("serial", serial)):
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(2):
                fn()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            out = fn()
        graphs[name] = (g, out)
    graphs["spec"][0].replay()
    graphs["serial"][0].replay()
    torch.cuda.synchronize()
    assert (graphs["spec"][1] - graphs["serial"][1]).abs().max().item() <= 2e-3
    steps = max(1, min(args.steps, 400))
    for i in range(max(args.warmup, 3)):
        graphs["spec"][0].replay()
    with ClockSampler(local if not args.quick else -1) as clk:
        barrier(world)
        ms = time_loop(lambda i: graphs["spec"][0].replay(), steps, device)
        barrier(world)
    ms = max_over_ranks(ms, world, device)
    for i in range(3):
        graphs["serial"][0].replay()
    barrier(world)
    ms_ser = max_over_ranks(time_loop(lambda i: graphs["serial"][0].replay(), steps, device), world, device)
    hbm_peak, peak_kind = peaks()
    tokens = sum(lengths[r] for r in mine)
    if rank == 0:
        line = {
            "metric": "batched decode steps (score+topk+spec attn+repair), requests decoded per second",
            "value": args.requests * steps / (ms / 1e3), "unit": "requests/s", "n_gpus": world, "steps": steps,
            "warmup": args.warmup, "ms_per_step": ms / steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded; BASELINE config 3 distribution)",
            "config": {"workload": f"BASELINE config 3: {args.requests} paged requests, context U[8192, 32768], "
                                   "16q/8kv, D128, page 16, 32-token blocks, K=64, overlap ~ Beta(8,2), bf16",
                       "parallelism": f"requests split across {world} rank(s) by LPT, no collective",
                       "l2": f"rank 0 holds {tokens} tokens of KV ({tokens * HKV * D * 4 / 2**30:.1f} GiB, > L2)",
                       "graph": "one CUDA graph per batched step"},
            "serial_ms_per_step": ms_ser / steps, "speedup_vs_serial": ms_ser / ms,
            "clocks": clk.summary(), "peak_gbs": hbm_peak, "peak_kind": peak_kind,
        }
        print(json.dumps(line), flush=True)
    graphs.clear()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "batched":
        return run_batched(args)
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
    ser = [SpeculativeDecoder(s["q"], s["k"], s["v"], s["lo"], s["hi"], s["p"], spec, serial=True, graph=graph)
           for s in sets]
    # Correctness gate before timing: speculative == serial within bf16 tolerance, IDs identical.
    for d_, s_ in zip(dec, ser):
        o1 = d_.step().clone()
        o2 = s_.step().clone()
        torch.cuda.synchronize()
        assert torch.equal(d_.selected.cpu(), s_.selected.cpu())
        assert (o1 - o2).abs().max().item() <= 2e-3, "speculative and serial outputs differ"

    # Timed loops: graphs of `gsteps` consecutive decode steps (one per input
    # set); a call of spec_step / serial_step runs one such graph.
    gsteps = max(1, min(args.graph_steps, nsets)) if graph else 1
    if gsteps > 1:
        gspec = [capture_steps([dec[(j + i) % nsets] for i in range(gsteps)])[0] for j in range(0, nsets, gsteps)]
        gser = [capture_steps([ser[(j + i) % nsets] for i in range(gsteps)])[0] for j in range(0, nsets, gsteps)]

        def spec_step(i):
            gspec[i % len(gspec)].replay()

        def serial_step(i):
            gser[i % len(gser)].replay()
    else:
        def spec_step(i):
            dec[i % nsets].step()

        def serial_step(i):
            ser[i % nsets].step()
    ncalls = max(1, args.steps // gsteps)
    args.steps = ncalls * gsteps

    hbm_peak, peak_kind = peaks()
    # Warm-up (untimed), then a ~1 s load window so clock samples see steady state.
    for i in range(max(args.warmup // gsteps, 3)):
        spec_step(i)
    torch.cuda.synchronize()
    with ClockSampler(local if not args.quick else -1) as clk:
        t_end = time.perf_counter() + (0.0 if args.quick else 1.0)
        while time.perf_counter() < t_end:
            for i in range(200 // gsteps + 1):
                spec_step(i)
            torch.cuda.synchronize()
        barrier(world)
        ms = time_loop(spec_step, ncalls, device)
        barrier(world)
    ms = max_over_ranks(ms, world, device)
    us_step = ms * 1e3 / args.steps
    value = world * args.steps / (ms / 1e3)
    clocks = clk.summary()

    # Serial baseline with the same kernels (same rotation), outside the main region.
    for i in range(3):
        serial_step(i)
    ms_ser = max_over_ranks(time_loop(serial_step, ncalls, device), world, device)
    us_ser = ms_ser * 1e3 / args.steps
    # Context: one CUDA graph per step (graph-launch cost paid every step).
    single = {}
    if graph and gsteps > 1 and not args.quick:
        n1 = min(args.steps, 2000)
        single = {"spec_us": time_loop(lambda i: dec[i % nsets].step(), n1, device) * 1e3 / n1,
                  "serial_us": time_loop(lambda i: ser[i % nsets].step(), n1, device) * 1e3 / n1}

    # Roofline of the dominant kernel: predicted-block attention (block states over P).
    s0 = sets[0]
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
    nrep = 3 if args.quick else max(50, min(args.steps // nsets, 1000))
    ms_part = time_loop(run_part, nrep, device, torch.cuda.current_stream())
    us_part = ms_part * 1e3 / (nrep * nsets)
    upred = statistics.mean(unique_blocks(s["p"].cpu(), g) for s in sets)
    part_bytes = 2 * blk * upred + HQ * D * 2 + HQ * TOPK * 4 + HQ * TOPK * (D + 2) * 4
    achieved = part_bytes / (us_part * 1e-6) / 1e9

    # Whole-step algorithmic bytes (score + predicted + misses), for context.
    score_bytes = 2 * HKV * BLOCKS * D * 4 + HQ * D * 2 + HQ * TOPK * 4
    ua = statistics.mean(unique_blocks(torch.as_tensor(s["a"]), g) for s in sets)
    miss = statistics.mean(
        sum(len(set(a_) - set(p_)) for a_, p_ in zip(s["a"].tolist(), s["p"].cpu().tolist())) for s in sets)
    step_bytes = score_bytes + 2 * blk * upred + 2 * blk * miss + HQ * D * 4
    serial_bytes = score_bytes + 2 * blk * ua + HQ * D * 4

    # End to end through the public API with host buffers: pinned q and P in,
    # output back to the host every step.
    hq_pin = [s["q"].cpu().pin_memory() for s in sets]
    hp_pin = [s["p"].cpu().pin_memory() for s in sets]
    hout = torch.empty(HQ, D, dtype=torch.float32).pin_memory()

    def e2e_step(i):
        j = i % nsets
        dec[j].q.copy_(hq_pin[j], non_blocking=True)
        dec[j].predicted.copy_(hp_pin[j], non_blocking=True)
        out = dec[j].step()
        hout.copy_(out, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    for i in range(20):
        e2e_step(i)
    n_e2e = 20 if args.quick else max(100, min(args.steps, 5000))
    t0 = time.perf_counter()
    for i in range(n_e2e):
        e2e_step(i)
    e2e_s = max_over_ranks(time.perf_counter() - t0, world, device)
    e2e_value = world * n_e2e / e2e_s

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

    cpu = None
    if rank == 0 and not args.no_cpu_baseline and not args.quick:
        from oracle.cpu_path import serial_step as cpu_step
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
            "metric": METRIC, "value": value, "unit": "decode-steps/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "us_per_step": us_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded; BASELINE config 1 distribution)",
            "config": {"workload": "BASELINE config 1: 1 request, 32q/8kv, D128, 65536 tokens, 32-token blocks, "
                                   "K=64, bf16", "method": args.method, "predicted_overlap": args.overlap,
                       "l2": f"{nsets} rotating input sets x {(2 * HKV * BLOCKS * B * D * 2 + 2 * HKV * BLOCKS * D * 4) / 2**20:.0f} MiB (> 126 MB L2)",
                       "parallelism": f"request replicas x{world} (no collective in the data path)",
                       "graph": (f"{gsteps} decode steps per CUDA graph (one per input set, replayed; each step one "
                                 "launch chain: scorer, Top-K, predicted-block states, repair)") if gsteps > 1 else
                                "one CUDA graph per step (scorer, Top-K, predicted-block states, repair)"},
            "serial_us_per_step": us_ser, "speedup_vs_serial": us_ser / us_step,
            "one_graph_per_step_us": single or None,
            "step_algorithmic_bytes": step_bytes, "serial_algorithmic_bytes": serial_bytes,
            "step_hbm_frac": step_bytes / (us_step * 1e-6) / 1e9 / hbm_peak,
            "serial_hbm_frac": serial_bytes / (us_ser * 1e-6) / 1e9 / hbm_peak,
            "roofline": {"bound": "hbm", "kernel": "jobs_fast_kernel (predicted-block attention, gqa.partials)",
                         "achieved": achieved, "peak": hbm_peak, "unit": "GB/s", "frac": achieved / hbm_peak,
                         "peak_kind": peak_kind, "us_per_launch": us_part, "bytes_per_launch": part_bytes,
                         "traffic": traffic_of("jobs_fast_kernel")},
            "clocks": clocks,
            "e2e": {"value": e2e_value, "unit": "decode-steps/s", "h2d_bytes_per_step": HQ * D * 2 + HQ * TOPK * 4,
                    "d2h_bytes_per_step": HQ * D * 4},
            "gpu_launches": LAUNCHES_PER_STEP.get(args.method, 4) * args.steps,
            "cpu_baseline": cpu,
        }
        if sweep:
            line["sweep"] = sweep
        print(json.dumps(line), flush=True)
    for d_ in dec + ser:
        d_.close()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
