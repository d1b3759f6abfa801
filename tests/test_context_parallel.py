"""Context-parallel decode of one long request (reduced
sizes): the exchange logic of strict_topk_overlap_b200.context_parallel.

CPU: gloo ranks (world size 2 and 4, uneven shards, cross-shard score ties)
run decode_step with the oracle's per-shard compute; the selection must equal
the unsharded strict Top-K bit for bit and the output the unsharded FP64
oracle. A rank that never reaches the step ends the others' step with an
error (short process-group timeout), not a hang.

GPU: ranks emulated as threads on one device (host-side all-gather between
threads, each rank on its own stream) run decode_step with the sm_100a
library; the selection must equal single-GPU selection bit for bit and the
output the FP64 oracle within the bf16 bar."""
from __future__ import annotations

import datetime
import os
import socket
import threading

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from strict_topk_overlap_b200.context_parallel import decode_step, shard_range


def test_shard_range_partitions():
    for n in (37, 64, 8192):
        for world in (1, 2, 3, 4, 8):
            spans = [shard_range(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


def _case(seed, hq=8, hkv=2, n=37, b=8, d=32, ties=False):
    import cases as C
    q, k, v, lo, hi = C.synthetic_kv(hq, hkv, n, b, d, torch.float32, seed=seed)
    if ties:
        # Every block repeats one of 5 blocks: exact score ties across shards.
        idx = torch.arange(n) % 5
        k, lo, hi = k[:, idx].contiguous(), lo[:, idx].contiguous(), hi[:, idx].contiguous()
    return q, k, v, lo, hi


def _predicted(ids, n, overlap, seed):
    import cases as C
    topk = ids.shape[1]
    return C.swap_prediction(torch.as_tensor(ids), n, int(round((1 - overlap) * topk)), seed)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cp_worker(rank, world, port, spec, out):
    from oracle.context_parallel import OracleShard
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        res = []
        for seed, n, topk, ties, pred in spec:
            q, k, v, lo, hi = _case(seed, n=n, ties=ties)
            s, e = shard_range(n, rank, world)
            o, sel = decode_step(q, k[:, s:e].contiguous(), v[:, s:e].contiguous(), lo[:, s:e].contiguous(),
                                 hi[:, s:e].contiguous(), topk, n, predicted=pred, backend=OracleShard)
            res.append((o.numpy(), sel.numpy()))
        out.put((rank, res))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_context_parallel_over_gloo_matches_unsharded(world):
    from oracle import attention as OA
    from oracle import selection as OS
    spec = []
    for seed, n, topk, ties in [(0, 37, 6, False), (1, 64, 8, True), (2, 41, 5, False)]:
        q, k, v, lo, hi = _case(seed, n=n, ties=ties)
        ids = OS.select_blocks(q.numpy(), lo.numpy(), hi.numpy(), topk)
        spec.append((seed, n, topk, ties, None))
        spec.append((seed, n, topk, ties, _predicted(ids, n, 0.7, seed)))
    ctx = mp.get_context("spawn")
    qu = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_cp_worker, args=(r, world, port, spec, qu)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(qu.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for i, (seed, n, topk, ties, pred) in enumerate(spec):
        q, k, v, lo, hi = _case(seed, n=n, ties=ties)
        ids = OS.select_blocks(q.numpy(), lo.numpy(), hi.numpy(), topk)
        assert np.array_equal(ids, OS.shard_select(q.numpy(), lo.numpy(), hi.numpy(), topk, world))
        ref = OA.attention_fp64(q.numpy(), k.numpy(), v.numpy(), ids)
        for r in range(world):
            o, sel = results[r][i]
            assert np.array_equal(sel, ids), (i, r)
            np.testing.assert_allclose(o, ref, rtol=1e-10, atol=1e-12)


def _missing_worker(rank, world, port, out):
    from oracle.context_parallel import OracleShard
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    try:
        if rank == 1:
            # This rank fails before the step: it never joins the exchange.
            out.put((rank, "left"))
            return
        q, k, v, lo, hi = _case(0, n=40)
        s, e = shard_range(40, rank, world)
        try:
            decode_step(q, k[:, s:e].contiguous(), v[:, s:e].contiguous(), lo[:, s:e].contiguous(),
                        hi[:, s:e].contiguous(), 4, 40, backend=OracleShard)
            out.put((rank, "completed"))
        except Exception as exc:  # the expected path: a collective error
            out.put((rank, "error:" + type(exc).__name__))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_missing_rank_gives_error_not_hang():
    ctx = mp.get_context("spawn")
    qu = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_missing_worker, args=(r, 2, port, qu)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(qu.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert got[1] == "left"
    assert got[0].startswith("error:"), got[0]


class ThreadComm:
    """All-gather between threads of one process (one thread per emulated
    rank); each rank's device work runs on the thread's own stream."""

    def __init__(self, shared, rank, world):
        self.shared, self.rank, self.world = shared, rank, world

    def all_gather(self, t):
        torch.cuda.current_stream().synchronize()
        slots, bar = self.shared["slots"], self.shared["barrier"]
        slots[self.rank] = t
        bar.wait()
        out = torch.stack([x.to(t.device) for x in slots], 0)
        torch.cuda.current_stream().synchronize()
        bar.wait()
        return out


def _emulated_ranks(world, q, k, v, lo, hi, topk, predicted=None):
    n = lo.shape[1]
    shared = {"slots": [None] * world, "barrier": threading.Barrier(world, timeout=120)}
    results, errors = [None] * world, []

    def run(rank):
        try:
            s, e = shard_range(n, rank, world)
            stream = torch.cuda.Stream()
            side = torch.cuda.Stream()
            with torch.cuda.stream(stream):
                sh = [t[:, s:e].contiguous() for t in (k, v, lo, hi)]
                o, sel = decode_step(q, *sh, topk, n, predicted=predicted, comm=ThreadComm(shared, rank, world),
                                     side_stream=side)
                stream.synchronize()
            results[rank] = (o.cpu(), sel.cpu())
        except Exception as exc:  # pragma: no cover - reported below
            errors.append(exc)
            shared["barrier"].abort()

    threads = [threading.Thread(target=run, args=(r,)) for r in range(world)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=300)
    if errors:
        raise errors[0]
    return results


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4])
def test_context_parallel_device_emulated_ranks(world):
    import cases as C
    from oracle import attention as OA
    from oracle import selection as OS
    from strict_topk import gqa
    hq, hkv, n, b, d, topk = 32, 8, 512, 64, 128, 64
    q, k, v, lo, hi = C.synthetic_kv(hq, hkv, n, b, d, torch.bfloat16, seed=4)
    ids = OS.select_blocks(q.float().numpy(), lo.numpy(), hi.numpy(), topk)
    ref = OA.attention_fp64(q.float().numpy(), k.float().numpy(), v.float().numpy(), ids)
    dev = [t.cuda() for t in (q, k, v, lo, hi)]
    single = gqa.select_blocks(dev[0], dev[3], dev[4], topk).cpu().numpy()
    assert np.array_equal(single, ids)
    strict = _emulated_ranks(world, *dev, topk)
    pred = _predicted(ids, n, 0.7, seed=4).cuda()
    spec = _emulated_ranks(world, *dev, topk, predicted=pred)
    for r in range(world):
        o, sel = strict[r]
        assert np.array_equal(sel.numpy(), ids)
        err = np.abs(o.numpy() - ref)
        assert (err <= 2e-3 + 1e-2 * np.abs(ref)).all(), err.max()
        assert torch.equal(o, strict[0][0])
        so, ssel = spec[r]
        assert np.array_equal(ssel.numpy(), ids)
        assert (so - o).abs().max().item() <= 1e-5


def _nccl_worker(rank, world, port, out):
    import cases as C
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        hq, hkv, n, b, d, topk = 32, 8, 512, 64, 128, 64
        q, k, v, lo, hi = C.synthetic_kv(hq, hkv, n, b, d, torch.bfloat16, seed=4)
        s, e = shard_range(n, rank, world)
        dev = torch.device("cuda", rank)
        sh = [t[:, s:e].contiguous().to(dev) for t in (k, v, lo, hi)]
        o, sel = decode_step(q.to(dev), *sh, topk, n)
        torch.cuda.synchronize()
        out.put((rank, o.cpu().numpy(), sel.cpu().numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_context_parallel_over_nccl_two_gpus():
    """Two processes, one GPU each, exchanging candidates and states with NCCL:
    selection bit-identical to single-GPU selection on both ranks, output
    within the bf16 bar of the FP64 oracle."""
    import cases as C
    from oracle import attention as OA
    from oracle import selection as OS
    hq, hkv, n, b, d, topk = 32, 8, 512, 64, 128, 64
    q, k, v, lo, hi = C.synthetic_kv(hq, hkv, n, b, d, torch.bfloat16, seed=4)
    ids = OS.select_blocks(q.float().numpy(), lo.numpy(), hi.numpy(), topk)
    ref = OA.attention_fp64(q.float().numpy(), k.float().numpy(), v.float().numpy(), ids)
    ctx = mp.get_context("spawn")
    qu = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, 2, port, qu)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(2):
        r, o, sel = qu.get(timeout=240)
        got[r] = (o, sel)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(2):
        o, sel = got[r]
        assert np.array_equal(sel, ids)
        assert (np.abs(o - ref) <= 2e-3 + 1e-2 * np.abs(ref)).all()
