"""Batched, paged-KV speculative decode and request sharding.

New entry points (the reference decodes one request over a dense
[Hkv, N, B, D] cache, kernels.py:1-6): a batch of R requests whose KV lives in
a shared page pool [pages, Hkv, page_size, D]. Request r owns the global
blocks block_offsets[r] .. block_offsets[r+1] (its local block j is global
block block_offsets[r] + j); block g is made of the pages
page_table[g * (B / page_size) + i], i < B / page_size. Min/max metadata is
per global block, [Hkv, total_blocks, D] FP32. Query rows are request-major,
row = r * Hq + h, and every ID is a request-local block index, so each row of
the batched calls has exactly the meaning of a row of the single-request API.

Every call is one launch sequence on the current stream with no host
synchronisation, like the rest of the library; the page table and block
offsets stay on the device.

Multi-GPU: requests are independent, so ``shard_requests`` splits a batch
across ranks (greedy longest-processing-time on context length) and each rank
decodes its own requests from its own cache — there is no collective in the
data path.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _lib as L
from .kernels import (PartialState, Prediction, RepairResult, _allocate_state, _prediction_struct,
                      compact_capacity)


@dataclass
class PagedKVCache:
    """A batch's KV page pool, page table, block offsets and block metadata."""
    k_pages: torch.Tensor        # [pages, Hkv, page_size, D]
    v_pages: torch.Tensor        # [pages, Hkv, page_size, D]
    page_table: torch.Tensor     # int32 [total_blocks * (block_size // page_size)]
    block_offsets: torch.Tensor  # int32 [R + 1], device
    lo: torch.Tensor             # FP32 [Hkv, total_blocks, D]
    hi: torch.Tensor             # FP32 [Hkv, total_blocks, D]
    block_size: int
    page_size: int
    max_blocks: int              # blocks of the longest request (host int)

    @property
    def requests(self) -> int:
        return self.block_offsets.shape[0] - 1

    @property
    def hkv(self) -> int:
        return self.k_pages.shape[1]

    @property
    def dim(self) -> int:
        return self.k_pages.shape[3]

    @property
    def total_blocks(self) -> int:
        return self.lo.shape[1]

    def kv(self) -> L.StkKV:
        return L.kv_struct(self.k_pages, self.v_pages, page_table=self.page_table,
                           block_offsets=self.block_offsets, page_size=self.page_size, hkv=self.hkv, n=0,
                           b=self.block_size, d=self.dim)


def build_paged_cache(ks, vs, page_size, *, generator=None, device=None) -> PagedKVCache:
    """Pack per-request dense caches K/V [Hkv, n_r, B, D] into one page pool.

    Pages are placed in a seeded random order (``generator``), as a serving
    system's allocator would leave them. Metadata lo/hi is each block's
    token-wise min/max of K in FP32 (built once here, outside any timing)."""
    if not ks or len(ks) != len(vs):
        raise ValueError("expected one K and one V tensor per request")
    hkv, _, b, d = ks[0].shape
    if b % page_size:
        raise ValueError(f"page size {page_size} must divide the block size {b}")
    device = device or ks[0].device
    ppb = b // page_size
    nblk = [k.shape[1] for k in ks]
    total = sum(nblk)
    npages = total * ppb
    perm = torch.randperm(npages, generator=generator).to(torch.int32)
    k_pages = torch.empty((npages, hkv, page_size, d), dtype=ks[0].dtype, device=device)
    v_pages = torch.empty_like(k_pages)
    offsets = [0]
    for n in nblk:
        offsets.append(offsets[-1] + n)
    for r, (k, v) in enumerate(zip(ks, vs)):
        g0 = offsets[r]
        # [hkv, n, b, d] -> [n * ppb, hkv, page, d] in (block, page) order
        kp = k.reshape(hkv, k.shape[1], ppb, page_size, d).permute(1, 2, 0, 3, 4).reshape(-1, hkv, page_size, d)
        vp = v.reshape(hkv, v.shape[1], ppb, page_size, d).permute(1, 2, 0, 3, 4).reshape(-1, hkv, page_size, d)
        dst = perm[g0 * ppb:(g0 + k.shape[1]) * ppb].long().to(device)
        k_pages[dst] = kp.to(device)
        v_pages[dst] = vp.to(device)
    lo = torch.cat([k.amin(dim=2).float() for k in ks], dim=1).to(device)
    hi = torch.cat([k.amax(dim=2).float() for k in ks], dim=1).to(device)
    return PagedKVCache(k_pages, v_pages, perm.to(device), torch.tensor(offsets, dtype=torch.int32, device=device),
                        lo.contiguous(), hi.contiguous(), b, page_size, max(nblk))


def _check_q(q, cache):
    if q.ndim != 2 or q.shape[1] != cache.dim or q.shape[0] % cache.requests:
        raise ValueError("q must be [R * Hq, D] with R the cache's request count")
    hq = q.shape[0] // cache.requests
    if hq % cache.hkv:
        raise ValueError("query heads must be a multiple of KV heads")
    if not q.is_cuda or not q.is_contiguous() or q.device != cache.k_pages.device:
        raise ValueError("q must be contiguous on the cache's CUDA device")
    return hq


def _check_ids(ids, q):
    if ids.ndim != 2 or ids.shape[0] != q.shape[0] or ids.dtype not in (torch.int32, torch.int64):
        raise ValueError("ids must be an int32/int64 matrix with one row per query row")
    if not ids.is_contiguous() or ids.device != q.device:
        raise ValueError("ids must be contiguous on the query's device")


def select_blocks(q, cache: PagedKVCache, topk, *, group_select=False):
    """Strict min/max-bound Top-K per query row of every request (ties to
    the lower block index, ascending request-local IDs). Returns int32
    [R * Hq, topk] (or [R * Hkv, topk] with ``group_select``)."""
    hq = _check_q(q, cache)
    if topk <= 0:
        raise ValueError("topk must be positive")
    R = cache.requests
    rows = R * (cache.hkv if group_select else hq)
    ids = torch.empty((rows, topk), device=q.device, dtype=torch.int32)
    lib = L.load()
    ws_bytes = lib.stk_select_workspace_bytes(cache.hkv if group_select else hq, cache.total_blocks)
    ws = torch.empty((max(ws_bytes, 1),), device=q.device, dtype=torch.uint8)
    rc = lib.stk_select_topk(q.data_ptr(), L.dtype_code(q), cache.lo.data_ptr(), cache.hi.data_ptr(), R, hq, cache.hkv,
                             0, cache.block_offsets.data_ptr(), cache.total_blocks, cache.max_blocks, cache.dim, topk,
                             int(group_select), 0, ids.data_ptr(), None, ws.data_ptr(), ws_bytes, L.status_ptr(),
                             L.stream_of(q))
    L.check(rc, "select_topk (batched)")
    return ids


def partials(q, cache: PagedKVCache, ids):
    """Per (row, slot) FP32 softmax state of the listed blocks."""
    hq = _check_q(q, cache)
    _check_ids(ids, q)
    rows, s = ids.shape
    state = _allocate_state(rows, s, cache.dim, q.device)
    kv = cache.kv()
    rc = L.load().stk_block_states(C.byref(kv), q.data_ptr(), L.dtype_code(q), rows, hq, ids.data_ptr(),
                                   L.id_is64(ids), s, None, 0, 0, None, 0, 0, None, L.MODE_FULL, None,
                                   state.m.data_ptr(), state.l.data_ptr(), state.u.data_ptr(), None, L.status_ptr(),
                                   L.stream_of(q))
    L.check(rc, "block_states (batched)")
    return state


def speculate(q, cache: PagedKVCache, predicted, mode="saved", mass_threshold=0.1, *, keep_mass=False):
    """Speculation over each row's predicted blocks (semantics of
    kernels.speculate, per row)."""
    if mode not in ("saved", "hybrid", "compact"):
        raise ValueError(mode)
    if not 0 <= mass_threshold <= 1:
        raise ValueError("mass_threshold must be in [0,1]")
    hq = _check_q(q, cache)
    _check_ids(predicted, q)
    rows, s = predicted.shape
    d = cache.dim
    dev = q.device
    pmode = L.PRED_MODES[mode]
    sc = compact_capacity(s, mass_threshold) if mode == "compact" else s
    state = _allocate_state(rows, sc, d, dev)
    high = low = low_abs = rids = overflow = pm = pl = None
    if mode != "saved":
        high = torch.empty((rows, s), device=dev, dtype=torch.bool)
        low = _allocate_state(rows, 1, d, dev)
        low_abs = torch.empty((rows, d), device=dev, dtype=torch.float32)
    if mode == "compact":
        rids = torch.empty((rows, sc), device=dev, dtype=predicted.dtype)
        overflow = torch.empty((rows,), device=dev, dtype=torch.bool)
        pm = torch.empty((rows, s), device=dev, dtype=torch.float32)
        pl = torch.empty_like(pm)
    lib = L.load()
    ws_bytes = lib.stk_speculate_workspace_bytes(rows, s, d, pmode)
    ws = torch.empty((max(ws_bytes, 1),), device=dev, dtype=torch.uint8)
    kv = cache.kv()
    rc = lib.stk_speculate(
        C.byref(kv), q.data_ptr(), L.dtype_code(q), rows, hq, predicted.data_ptr(), L.id_is64(predicted), s, pmode,
        float(mass_threshold), sc, state.m.data_ptr(), state.l.data_ptr(), state.u.data_ptr(), L.ptr(high),
        L.ptr(rids), L.ptr(low.m) if low else None, L.ptr(low.l) if low else None, L.ptr(low.u) if low else None,
        L.ptr(low_abs), L.ptr(overflow), L.ptr(pm), L.ptr(pl), ws.data_ptr(), ws_bytes, L.status_ptr(),
        L.stream_of(q))
    L.check(rc, "speculate (batched)")
    if mode == "compact":
        return Prediction(state, "compact", high, low, rids, overflow, low_abs,
                          pm if keep_mass else None, pl if keep_mass else None)
    mass_m, mass_l = (state.m, state.l) if keep_mass else (None, None)
    if mode == "saved":
        return Prediction(state, mode, mass_m=mass_m, mass_l=mass_l)
    return Prediction(state, mode, high, low, low_abs=low_abs, mass_m=mass_m, mass_l=mass_l)


def _repair(q, cache, selected, predicted, prediction, variant, *, min_remaining=1e-3, cancellation_tol=1e-5,
            max_extra_mass=0., want_approx=False, want_jobs=False):
    hq = _check_q(q, cache)
    _check_ids(selected, q)
    if predicted is not None:
        _check_ids(predicted, q)
    rows, d = q.shape
    dev = q.device
    out = torch.empty((rows, d), device=dev, dtype=torch.float32)
    fallback = torch.empty((rows,), device=dev, dtype=torch.bool)
    remaining = torch.empty((rows,), device=dev, dtype=torch.float32)
    approx = torch.empty_like(fallback) if want_approx else None
    extra = torch.empty_like(remaining) if want_approx else None
    pos = torch.empty((rows,), device=dev, dtype=torch.int32) if want_jobs else None
    total = torch.empty_like(pos) if want_jobs else None
    kv = cache.kv()
    ps = _prediction_struct(prediction)
    ro = L.StkRepairOut(out.data_ptr(), fallback.data_ptr(), remaining.data_ptr(), L.ptr(approx), L.ptr(extra),
                        L.ptr(pos), L.ptr(total))
    sp = predicted.shape[1] if predicted is not None else 0
    rc = L.load().stk_repair(
        C.byref(kv), q.data_ptr(), L.dtype_code(q), rows, hq, selected.data_ptr(), L.id_is64(selected),
        selected.shape[1], L.ptr(predicted), L.id_is64(predicted) if predicted is not None else 0, sp, C.byref(ps),
        variant, float(min_remaining), float(cancellation_tol), float(max_extra_mass), cache.max_blocks,
        C.byref(ro), L.status_ptr(), L.stream_of(q))
    L.check(rc, "repair (batched)")
    if want_jobs:
        return out, fallback, remaining, approx, extra, pos, total
    return out, fallback, remaining, approx, extra


def exact(q, cache: PagedKVCache, selected):
    """Strict attention of every row over its selected blocks -> FP32 [rows, D]."""
    return _repair(q, cache, selected, None, None, L.VAR_SAVED)[0]


def repair_saved(q, cache: PagedKVCache, selected, predicted, state: PartialState):
    """Saved-state repair: reuse predicted hits, compute the misses."""
    return _repair(q, cache, selected, predicted, Prediction(state, "saved"), L.VAR_SAVED)[0]


def repair_fused(q, cache: PagedKVCache, selected, predicted, prediction, min_remaining=1.e-3,
                 cancellation_tol=1.e-5, max_extra_mass=0.):
    """Guarded one-launch repair (semantics of fused.repair_fused, per row),
    relaxed by ``max_extra_mass`` when it is positive."""
    if not 0 <= max_extra_mass <= 1:
        raise ValueError("max_extra_mass must be in [0, 1]")
    if max_extra_mass > 0 and prediction.mode != "saved" and prediction.mass_m is None:
        raise ValueError("positive max_extra_mass requires speculate(..., keep_mass=True)")
    out, fallback, remaining, approx, extra = _repair(
        q, cache, selected, predicted, prediction, L.VAR_FUSED, min_remaining=min_remaining,
        cancellation_tol=cancellation_tol, max_extra_mass=max_extra_mass, want_approx=max_extra_mass > 0)
    res = RepairResult(out, fallback, remaining)
    if max_extra_mass > 0:
        res.approximate_heads = approx
        res.extra_mass_bound = extra
    return res


def repair_signed_fused(q, cache: PagedKVCache, selected, predicted, prediction, min_remaining=1.e-3,
                        cancellation_tol=1.e-5, max_extra_mass=0.):
    """Signed add/erase repair with inline strict fallback (semantics of
    signed_fused.repair_signed_fused, per row), relaxed by ``max_extra_mass``
    when it is positive; also returns the positive / total job counts."""
    from .signed_repair import SignedRepairResult
    if not 0 <= max_extra_mass <= 1:
        raise ValueError("max_extra_mass must be in [0, 1]")
    if max_extra_mass > 0 and prediction.mode != "saved" and prediction.mass_m is None:
        raise ValueError("positive max_extra_mass requires speculate(..., keep_mass=True)")
    out, fallback, remaining, approx, extra, pos, total = _repair(
        q, cache, selected, predicted, prediction, L.VAR_SIGNED_FUSED, min_remaining=min_remaining,
        cancellation_tol=cancellation_tol, max_extra_mass=max_extra_mass, want_approx=max_extra_mass > 0,
        want_jobs=True)
    return SignedRepairResult(out, fallback, remaining, approx, extra, pos, total)


# ----------------------------------------------------------------------------- sharding

def shard_requests(lengths, world):
    """Split requests across ``world`` ranks by greedy longest-processing-time
    on context length: longest request first, each to the least-loaded rank
    (ties to the lower rank). Returns one ascending index list per rank; the
    lists partition range(len(lengths))."""
    if world <= 0:
        raise ValueError("world must be positive")
    order = sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i))
    load = [0] * world
    shards = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda j: (load[j], j))
        shards[r].append(i)
        load[r] += int(lengths[i])
    return [sorted(s) for s in shards]

_STEP_VARIANTS = {"saved": L.VAR_SAVED, "repair_fused": L.VAR_FUSED, "signed_fused": L.VAR_SIGNED_FUSED}


def speculative_step_workspace(q, cache: PagedKVCache, predicted, variant="saved"):
    """Workspace for ``speculative_step`` (selection scratch, the predicted
    blocks' states and, for the hybrid variants, the grouping's mask and low
    aggregate)."""
    hq = _check_q(q, cache)
    need = L.load().stk_speculative_step_batched_workspace_bytes(
        cache.requests, hq, cache.total_blocks, predicted.shape[1], cache.dim, int(variant != "saved"))
    return torch.empty((max(need, 1),), device=q.device, dtype=torch.uint8)


def speculative_step(q, cache: PagedKVCache, predicted, topk, *, variant="saved", mass_threshold=0.1,
                     min_remaining=1.e-3, cancellation_tol=1.e-5, max_extra_mass=0., workspace=None):
    """One speculative decode step of the whole batch as one chain of
    dependent launches on the current stream (stk_speculative_step_batched):
    strict Top-K selection, the predicted blocks' states while the selection
    finishes, then the saved repair (``variant="saved"``: equal to
    select_blocks, partials and repair_saved in sequence) or the hybrid
    grouping and the guarded repair (``"repair_fused"`` / ``"signed_fused"``:
    equal to select_blocks, speculate(mode="hybrid", keep_mass=True) and
    repair_fused / the signed fused repair, relaxed by ``max_extra_mass``).
    Returns (output FP32 [rows, D], selected int32 [rows, topk])."""
    hq = _check_q(q, cache)
    _check_ids(predicted, q)
    if variant not in _STEP_VARIANTS:
        raise ValueError(f"variant must be one of {sorted(_STEP_VARIANTS)}")
    if not 0 <= max_extra_mass <= 1:
        raise ValueError("max_extra_mass must be in [0, 1]")
    rows, d = q.shape
    dev = q.device
    if workspace is None:
        workspace = speculative_step_workspace(q, cache, predicted, variant)
    selected = torch.empty((rows, topk), device=dev, dtype=torch.int32)
    out = torch.empty((rows, d), device=dev, dtype=torch.float32)
    flags = torch.empty((rows,), device=dev, dtype=torch.bool)
    remaining = torch.empty((rows,), device=dev, dtype=torch.float32)
    approx = torch.empty_like(flags)
    extra = torch.empty_like(remaining)
    ro = L.StkRepairOut(out.data_ptr(), flags.data_ptr(), remaining.data_ptr(), approx.data_ptr(), extra.data_ptr(),
                        None, None)
    kv = cache.kv()
    rc = L.load().stk_speculative_step_batched(
        C.byref(kv), q.data_ptr(), L.dtype_code(q), cache.lo.data_ptr(), cache.hi.data_ptr(), cache.requests, hq,
        cache.total_blocks, cache.max_blocks, topk, predicted.data_ptr(), L.id_is64(predicted), predicted.shape[1],
        float(mass_threshold), _STEP_VARIANTS[variant], float(min_remaining), float(cancellation_tol),
        float(max_extra_mass), selected.data_ptr(), C.byref(ro), workspace.data_ptr(), workspace.numel(),
        L.status_ptr(), L.stream_of(q))
    L.check(rc, "speculative_step (batched)")
    return out, selected
