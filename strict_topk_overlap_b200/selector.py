"""Fused min/max bound block scoring and strict Top-K selection on sm_100a.

Drop-in for ``strict_topk.selector`` (reference selector.py:1-43). Scores are
summed in FP64 in one fixed order (see csrc/select.cu) and the Top-K breaks
ties toward the lower block index; IDs are returned in ascending order.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib as L


def _validate(q, lo, hi):
    """Argument checks of selector.py:23-33 (same ValueError messages)."""
    if lo.ndim != 3 or hi.shape != lo.shape:
        raise ValueError("lo and hi must have the same [heads, blocks, dim] shape")
    h, n, d = lo.shape
    if q.shape != (h, d) or min(h, n, d) <= 0:
        raise ValueError("q must have shape [heads, dim], with nonempty input dimensions")
    if lo.dtype != torch.float32 or hi.dtype != torch.float32:
        raise ValueError("lo and hi must be FP32")
    if not q.is_cuda or any(x.device != q.device or not x.is_contiguous() for x in (q, lo, hi)):
        raise ValueError("q, lo and hi must be contiguous on the same CUDA device")
    return h, n, d


def bound_scores(q, lo, hi):
    """FP32-rounded FP64 bound scores for per-head ([H,N,D]) or shared
    ([Hkv,N,D], Hq % Hkv == 0) metadata."""
    hq, d = q.shape
    hm, n, _ = lo.shape
    scores = torch.empty((hq, n), device=q.device, dtype=torch.float32)
    rc = L.load().stk_bound_scores(q.data_ptr(), L.dtype_code(q), lo.data_ptr(), hi.data_ptr(), hq, hm, n, d,
                                   scores.data_ptr(), L.stream_of(q))
    L.check(rc, "bound_scores")
    return scores


def block_scores(q, lo, hi):
    """Compute FP32 min/max bound scores for contiguous CUDA inputs."""
    _validate(q, lo, hi)
    return bound_scores(q, lo, hi)


def topk_from_metadata(q, lo, hi, topk, *, group_select=False, id_base=0, keys_out=None):
    """Score + strict Top-K. ``group_select`` scores each KV head by the sum of
    its query heads' scores and returns one row per KV head."""
    hq, d = q.shape
    hm, n, _ = lo.shape
    rows = hm if group_select else hq
    if topk > n:
        raise RuntimeError(f"selected index k out of range (k={topk}, blocks={n})")
    if topk == 0:
        return torch.empty((rows, 0), device=q.device, dtype=torch.int32)
    ids = torch.empty((rows, topk), device=q.device, dtype=torch.int32)
    lib = L.load()
    ws_bytes = lib.stk_select_workspace_bytes(rows, n)
    ws = torch.empty((ws_bytes,), device=q.device, dtype=torch.uint8)
    rc = lib.stk_select_topk(q.data_ptr(), L.dtype_code(q), lo.data_ptr(), hi.data_ptr(), 1, hq, hm, n, None, n, n, d,
                             topk, int(group_select), int(id_base), ids.data_ptr(), L.ptr(keys_out), ws.data_ptr(),
                             ws_bytes, L.status_ptr(), L.stream_of(q))
    L.check(rc, "select_topk")
    return ids


def select_blocks(q, lo, hi, topk):
    """Return the int32 block IDs of the strict Top-K bound scores
    (ties to the lower index, ascending IDs)."""
    _validate(q, lo, hi)
    return topk_from_metadata(q, lo, hi, topk)
