"""Request sharding for batched decode (BASELINE config 3 across GPUs): the
greedy longest-processing-time split, and its use by CPU ranks over gloo
(world size 2): every rank decodes only its own requests (here with the CPU
oracle standing in for the device kernels) and the gathered per-request
results equal a single-process run. No collective is needed in the data
path; the gather exists only to check the result."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from strict_topk_overlap_b200.paged import shard_requests


def test_lpt_partitions_and_balances():
    rng = np.random.default_rng(0)
    lengths = (rng.integers(8192, 32769, 64) // 32 * 32).tolist()
    for world in (1, 2, 4, 8):
        shards = shard_requests(lengths, world)
        flat = sorted(i for s in shards for i in s)
        assert flat == list(range(64))
        loads = [sum(lengths[i] for i in s) for s in shards]
        # LPT bound: max load <= mean + the longest request.
        assert max(loads) <= sum(lengths) / world + max(lengths)
    assert shard_requests([5, 5, 5], 2) == [[0, 2], [1]]
    assert shard_requests([], 3) == [[], [], []]
    with pytest.raises(ValueError):
        shard_requests([1], 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _decode_request(r):
    """Oracle decode of request r: strict selection + FP64 attention (CPU)."""
    import cases as C
    from oracle import attention as OA
    from oracle import selection as OS
    n = 40 + 8 * r
    q, k, v, lo, hi = C.synthetic_kv(4, 2, n, 8, 32, torch.float32, seed=100 + r)
    ids = OS.select_blocks(q.numpy(), lo.numpy(), hi.numpy(), 6)
    return OA.attention_fp64(q.numpy(), k.numpy(), v.numpy(), ids)


def _worker(rank, world, port, lengths, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = shard_requests(lengths, world)[rank]
        res = {r: _decode_request(r) for r in mine}
        gathered = [None] * world
        dist.all_gather_object(gathered, res)
        if rank == 0:
            merged = {}
            for g in gathered:
                merged.update(g)
            out.put(merged)
    finally:
        dist.destroy_process_group()


def test_sharded_decode_over_gloo_matches_single_process():
    lengths = [300, 120, 500, 80, 220, 410]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, lengths, q)) for r in range(2)]
    for p in procs:
        p.start()
    merged = q.get(timeout=300)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert sorted(merged) == list(range(len(lengths)))
    for r in range(len(lengths)):
        assert np.array_equal(merged[r], _decode_request(r))
