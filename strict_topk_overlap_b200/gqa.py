"""Split-block sparse attention for native grouped-query KV layouts.

Drop-in for ``strict_topk.gqa`` (reference gqa.py:1-193). Q is
[query_heads, dim]; K and V are [kv_heads, blocks, tokens, dim]; adjacent
query heads share a KV head. Each row of IDs holds a nonempty set of unique,
valid block IDs. Inputs are contiguous and finite.
"""
from __future__ import annotations

import torch

from . import _lib as L
from .kernels import PartialState, Prediction, _allocate_state, _block_states, _run_repair, merge_partials
from .selector import topk_from_metadata


def _validate_ids(q, ids):
    if (ids.ndim != 2 or ids.shape[0] != q.shape[0] or ids.shape[1] == 0
            or ids.dtype not in (torch.int32, torch.int64)):
        raise ValueError("ids must be a nonempty int32/int64 matrix with one row per query head")
    if ids.device != q.device or not ids.is_contiguous():
        raise ValueError("ids must be contiguous and on the query's CUDA device")


def _shape(q, k, v, ids):
    """Contract of gqa.py:115-125 (ValueError on violation)."""
    if q.ndim != 2 or k.ndim != 4 or k.shape != v.shape:
        raise ValueError("expected Q[Hq,D] and K/V[Hkv,N,B,D]")
    hkv, n, b, d = k.shape
    hq, qd = q.shape
    if min(hq, hkv, n, b, d) <= 0 or qd != d or hq % hkv != 0:
        raise ValueError("expected nonempty shapes, matching head dimensions and Hq divisible by Hkv")
    if not q.is_cuda or any(x.device != q.device or not x.is_contiguous() for x in (q, k, v)):
        raise ValueError("Q/K/V must be contiguous and on the same CUDA device")
    _validate_ids(q, ids)
    return hq, n, b, d, hq // hkv, ids.shape[1]


def partials(q, k, v, ids):
    """Compute one FP32 softmax partial per query head and block."""
    hq, n, b, d, group, sa = _shape(q, k, v, ids)
    state = _allocate_state(hq, sa, d, q.device)
    return _block_states(q, k, v, ids, out=state)


def exact(q, k, v, selected):
    """Attend to the selected blocks: per-block partials merged on chip, in one
    launch (the reference's partials + merge, gqa.py:140-142)."""
    _shape(q, k, v, selected)
    out, *_ = _run_repair(q, k, v, selected, None, None, L.VAR_SAVED)
    return out


def select_blocks(q, lo, hi, topk):
    """Select min/max bound Top-K using native FP32 metadata [Hkv,N,D]
    (ties to the lower block index, ascending IDs)."""
    if q.ndim != 2 or lo.ndim != 3 or hi.shape != lo.shape:
        raise ValueError("expected Q[Hq,D] and LO/HI[Hkv,N,D]")
    hkv, n, d = lo.shape
    hq, qd = q.shape
    if min(hq, hkv, n, d) <= 0 or qd != d or hq % hkv != 0:
        raise ValueError("expected nonempty shapes, matching head dimensions and Hq divisible by Hkv")
    if lo.dtype != torch.float32 or hi.dtype != torch.float32:
        raise ValueError("lo and hi must be FP32")
    if not q.is_cuda or any(x.device != q.device or not x.is_contiguous() for x in (q, lo, hi)):
        raise ValueError("Q/LO/HI must be contiguous and on the same CUDA device")
    return topk_from_metadata(q, lo, hi, topk)


def select_blocks_shared(q, lo, hi, topk):
    """Shared per-group selection: each KV head is scored by the FP64 sum of
    its query heads' bound scores (ascending query head), and every query
    head of the group receives the group's Top-K row. Returns [Hq, topk]."""
    if q.ndim != 2 or lo.ndim != 3 or hi.shape != lo.shape:
        raise ValueError("expected Q[Hq,D] and LO/HI[Hkv,N,D]")
    hkv = lo.shape[0]
    hq = q.shape[0]
    if hq % hkv:
        raise ValueError("expected nonempty shapes, matching head dimensions and Hq divisible by Hkv")
    rows = topk_from_metadata(q, lo, hi, topk, group_select=True)
    return rows.repeat_interleave(hq // hkv, dim=0)


def _check_state(q, d, predicted, state):
    hq = q.shape[0]
    sp = predicted.shape[1]
    if state.m.shape != (hq, sp) or state.l.shape != (hq, sp) or state.u.shape != (hq, sp, d):
        raise ValueError("state must contain a softmax partial for every predicted block")


def _repair(q, k, v, selected, predicted, state, union):
    hq, n, b, d, group, sa = _shape(q, k, v, selected)
    _validate_ids(q, predicted)
    _check_state(q, d, predicted, state)
    pred = Prediction(state, "saved")
    out, *_ = _run_repair(q, k, v, selected, predicted, pred, L.VAR_UNION if union else L.VAR_SAVED)
    return out


def repair_saved(q, k, v, selected, predicted, state):
    """Reuse predicted hits and compute only selected misses."""
    return _repair(q, k, v, selected, predicted, state, union=False)


def repair_union(q, k, v, selected, predicted, state):
    """Attend to the union of selected and predicted blocks, once each."""
    return _repair(q, k, v, selected, predicted, state, union=True)
