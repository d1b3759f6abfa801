"""Context-parallel strict decode of one very long request.

New (the reference decodes on one GPU only). The request's blocks are split
evenly across the R ranks of a process group: rank r owns global blocks
[start_r, end_r) = shard_range(n_blocks, r, R) of every KV head, with their
K/V and min/max metadata. One decode step:

  1. shard-local bound scores and strict Top-K candidates per query row:
     (64-bit score order key, global block ID), IDs ascending;
  2. all-gather of the candidates (8 B per candidate — 64 KiB per rank at
     32 rows x K 256);
  3. the global strict Top-K from the R*K candidates per row, ties to the
     lower global ID. Every shard's candidates are ascending and shards own
     increasing ID ranges, so candidate position order is global ID order,
     and the result is bit-identical to single-GPU selection on every rank;
  4. the FP32 softmax states of the selected blocks this rank owns, reduced
     to one unnormalised (m, l, u) per row. With a predicted list, the states
     of the owned predicted blocks are computed on a second stream while
     steps 1-3 run, and step 4 computes only the owned misses (selected, not
     predicted) and merges them with the predicted states that were selected
     (the saved repair of kernels.py:504-550, restricted to owned blocks);
  5. all-gather of those states (~(D + 2) * 4 B per row) and their LSE merge
     into the output, identically on every rank.

The exchange is latency-bound (tens of KiB), so the two all-gathers are the
whole communication; no rank reads another rank's memory.

The device work goes through ``DeviceShard`` (the sm_100a library) and the
exchange through a ``Comm`` (``ProcessGroupComm``: torch.distributed, NCCL on
GPUs). ``decode_step`` takes both as arguments, so that the same
orchestration runs on CPU ranks (gloo) with a CPU compute stand-in in the
tests; the product path uses ``DeviceShard``.
"""
from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as dist

from . import _lib as L


def shard_range(n_blocks: int, rank: int, world: int):
    """Blocks [start, end) owned by ``rank`` of ``world`` (even split, the
    first n_blocks % world ranks one block longer)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank / world")
    base, extra = divmod(n_blocks, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


class ProcessGroupComm:
    """All-gather over a torch.distributed process group (rank order).

    Give the group a short timeout: a rank that never reaches a step's
    all-gather then ends the others' with an error instead of a hang."""

    def __init__(self, group=None):
        self.group = group
        if dist.is_available() and dist.is_initialized():
            self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        else:
            self.world, self.rank = 1, 0

    def all_gather(self, t: torch.Tensor) -> torch.Tensor:
        """[world, *t.shape] with rank r's tensor at index r."""
        if self.world == 1:
            return t.unsqueeze(0)
        parts = [torch.empty_like(t) for _ in range(self.world)]
        dist.all_gather(parts, t.contiguous(), group=self.group)
        return torch.stack(parts, 0)


class DeviceShard:
    """The per-shard device work of a context-parallel step (sm_100a library)."""

    @staticmethod
    def local_candidates(q, lo, hi, topk, id_base):
        """Shard-local strict Top-K of every query row: (order keys int64
        [rows, topk], global IDs int32 [rows, topk]), IDs ascending."""
        hq, d = q.shape
        hm, n, _ = lo.shape
        ids = torch.empty((hq, topk), device=q.device, dtype=torch.int32)
        keys = torch.empty((hq, topk), device=q.device, dtype=torch.int64)
        lib = L.load()
        ws_bytes = lib.stk_select_workspace_bytes(hq, n)
        ws = torch.empty((ws_bytes,), device=q.device, dtype=torch.uint8)
        rc = lib.stk_select_topk(q.data_ptr(), L.dtype_code(q), lo.data_ptr(), hi.data_ptr(), 1, hq, hm, n, None, n, n,
                                 d, topk, 0, int(id_base), ids.data_ptr(), keys.data_ptr(), ws.data_ptr(), ws_bytes,
                                 L.status_ptr(), L.stream_of(q))
        L.check(rc, "select_topk (shard)")
        return keys, ids

    @staticmethod
    def merge_candidates(keys, ids, topk):
        """Global strict Top-K (IDs ascending) from per-row candidates whose
        position order is ascending ID order."""
        rows, ncand = ids.shape
        out = torch.empty((rows, topk), device=ids.device, dtype=torch.int32)
        rc = L.load().stk_merge_candidates(keys.data_ptr(), ids.data_ptr(), rows, ncand, topk, out.data_ptr(),
                                           L.status_ptr(), L.stream_of(ids))
        L.check(rc, "merge_candidates")
        return out

    @staticmethod
    def block_states(q, k, v, ids, pred=None):
        """Per-slot states (m, l [rows, s], u [rows, s, D]) of local block IDs
        [rows, s]; -1 slots give (-inf, 0, 0). With ``pred`` (local IDs
        [rows, sp]), slots whose block is in the row's pred are skipped
        (their states are left unwritten) and the 4th result holds each
        slot's position in pred (-1 = miss)."""
        hq, d = q.shape
        rows, s = ids.shape
        m = torch.empty((rows, s), device=q.device, dtype=torch.float32)
        lsum = torch.empty_like(m)
        u = torch.empty((rows, s, d), device=q.device, dtype=torch.float32)
        slot = None if pred is None else torch.empty((rows, s), device=q.device, dtype=torch.int32)
        kv = L.kv_struct(k, v)
        rc = L.load().stk_block_states(C.byref(kv), q.data_ptr(), L.dtype_code(q), rows, hq, ids.data_ptr(),
                                       L.id_is64(ids), s, None, 0, 0, L.ptr(pred),
                                       0 if pred is None else L.id_is64(pred), 0 if pred is None else pred.shape[1],
                                       L.ptr(slot), L.MODE_FULL, None, m.data_ptr(), lsum.data_ptr(), u.data_ptr(),
                                       None, L.status_ptr(), L.stream_of(q))
        L.check(rc, "block_states (shard)")
        return m, lsum, u, slot

    @staticmethod
    def reduce_states(m, l, u, include=None):
        """One unnormalised state per row from per-slot states."""
        rows, s, d = u.shape
        mo = torch.empty((rows,), device=u.device, dtype=torch.float32)
        lo = torch.empty_like(mo)
        uo = torch.empty((rows, d), device=u.device, dtype=torch.float32)
        inc = None if include is None else include.to(torch.uint8).contiguous()
        rc = L.load().stk_reduce_states(m.data_ptr(), l.data_ptr(), u.data_ptr(), L.ptr(inc), rows, s, d,
                                        mo.data_ptr(), lo.data_ptr(), uo.data_ptr(), L.stream_of(u))
        L.check(rc, "reduce_states")
        return mo, lo, uo

    @staticmethod
    def merge_states(m, l, u):
        """LSE merge of per-shard states [rows, R] / [rows, R, D] -> FP32 [rows, D]."""
        rows, s, d = u.shape
        out = torch.empty((rows, d), device=u.device, dtype=torch.float32)
        rc = L.load().stk_merge_states(m.data_ptr(), l.data_ptr(), u.data_ptr(), None, rows, s, d, out.data_ptr(),
                                       L.stream_of(u))
        L.check(rc, "merge_states")
        return out


def _localise(ids, start, end):
    """Global IDs -> this shard's local IDs, -1 where another shard owns the block."""
    own = (ids >= start) & (ids < end)
    return torch.where(own, ids - start, torch.full_like(ids, -1))


def decode_step(q, k, v, lo, hi, topk, n_blocks, *, predicted=None, comm=None, backend=DeviceShard,
                side_stream=None):
    """One strict context-parallel decode step.

    q [Hq, D] (the same on every rank); k/v [Hkv, n_r, B, D] and lo/hi
    [Hkv, n_r, D] are this rank's shard of the request (global blocks
    shard_range(n_blocks, rank, world)); every shard must hold >= topk blocks.
    predicted: optional global block IDs [Hq, sp] (the same on every rank),
    whose owned blocks' states are computed before the selection is known
    (on ``side_stream`` when given, overlapping steps 1-3).
    Returns (output FP32 [Hq, D], selected global block IDs int32 [Hq, topk]),
    identical on every rank."""
    comm = comm if comm is not None else ProcessGroupComm()
    world, rank = comm.world, comm.rank
    start, end = shard_range(n_blocks, rank, world)
    if end - start != lo.shape[1] or k.shape[1] != end - start:
        raise ValueError(f"rank {rank} holds {lo.shape[1]} blocks, expected {end - start} (global [{start}, {end}))")
    if n_blocks // world < topk:
        raise ValueError("every shard must hold at least topk blocks")
    hq = q.shape[0]
    pstates = None
    if predicted is not None:
        ploc = _localise(predicted.to(torch.int32), start, end)
        if side_stream is not None:
            side_stream.wait_stream(torch.cuda.current_stream(q.device))
            with torch.cuda.stream(side_stream):
                pstates = backend.block_states(q, k, v, ploc)
        else:
            pstates = backend.block_states(q, k, v, ploc)
    # 1-3: candidates, exchange, global Top-K.
    keys, ids = backend.local_candidates(q, lo, hi, topk, start)
    all_keys = comm.all_gather(keys)  # [R, Hq, K]
    all_ids = comm.all_gather(ids)
    cand_keys = all_keys.permute(1, 0, 2).reshape(hq, world * topk).contiguous()
    cand_ids = all_ids.permute(1, 0, 2).reshape(hq, world * topk).contiguous()
    selected = backend.merge_candidates(cand_keys, cand_ids, topk)
    # 4: owned blocks' states.
    aloc = _localise(selected, start, end)
    if predicted is None:
        m, l, u, _ = backend.block_states(q, k, v, aloc)
        ms, ls, us = backend.reduce_states(m, l, u, None)
    else:
        if side_stream is not None:
            torch.cuda.current_stream(q.device).wait_stream(side_stream)
        pm, pl, pu, _ = pstates
        # Misses: owned selected blocks not in the predicted list.
        mm, ml, mu, slot = backend.block_states(q, k, v, aloc, ploc)
        miss = (aloc >= 0) & (slot < 0)
        hit = (ploc >= 0) & (ploc.unsqueeze(2) == aloc.unsqueeze(1)).any(2)
        ms, ls, us = backend.reduce_states(torch.cat([pm, mm], 1), torch.cat([pl, ml], 1), torch.cat([pu, mu], 1),
                                           torch.cat([hit, miss], 1))
    # 5: exchange and merge.
    all_m = comm.all_gather(ms)  # [R, Hq]
    all_l = comm.all_gather(ls)
    all_u = comm.all_gather(us)  # [R, Hq, D]
    out = backend.merge_states(all_m.t().contiguous(), all_l.t().contiguous(), all_u.permute(1, 0, 2).contiguous())
    return out, selected
