"""FP64 bound scores in the library's fixed order, and strict Top-K.

Score formula: reference selector.py:8-20 / gqa.py:15-26 and the FP64 form of
tests/check_selector.py:14-15; the summation order is the one the sm_100a
kernel fixes (lane-contiguous dims summed left to right, then an xor
butterfly over 32 lanes with offsets 16, 8, 4, 2, 1). Ties in Top-K go to the
lower block index (a stricter contract than the reference's torch.topk,
whose tie order is unspecified, tests/check_gqa.py:46).
"""
from __future__ import annotations

import numpy as np


def bound_scores_fp64(q, lo, hi):
    """q [Hq, D] (any float), lo/hi [Hm, N, D] float32 with Hq % Hm == 0 -> [Hq, N] float64."""
    q64 = np.asarray(q, dtype=np.float64)
    lo64 = np.asarray(lo, dtype=np.float64)
    hi64 = np.asarray(hi, dtype=np.float64)
    hq, d = q64.shape
    hm, n, _ = lo64.shape
    g = hq // hm
    c = (d + 31) // 32
    idx = np.arange(32)
    out = np.empty((hq, n), dtype=np.float64)
    for h in range(hq):
        prod = np.where(q64[h] >= 0, hi64[h // g], lo64[h // g]) * q64[h]  # exact in FP64
        pad = np.zeros((n, 32 * c))
        pad[:, :d] = prod
        lanes = pad.reshape(n, 32, c)
        part = np.zeros((n, 32))
        for j in range(c):
            part = part + lanes[:, :, j]
        for off in (16, 8, 4, 2, 1):
            part = part + part[:, idx ^ off]
        out[h] = part[:, 0]
    return out


def group_scores_fp64(scores, group):
    """Per-KV-head score = FP64 sum over its query heads in ascending order."""
    hq, n = scores.shape
    out = np.zeros((hq // group, n))
    for g in range(group):
        out = out + scores[g::group]
    return out


def stable_topk(scores, k):
    """Top-k per row by (score desc, index asc); returned ascending by index."""
    scores = np.asarray(scores, dtype=np.float64)
    rows, n = scores.shape
    ids = np.broadcast_to(np.arange(n), (rows, n))
    order = np.lexsort((ids, -scores), axis=1)
    return np.sort(order[:, :k], axis=1).astype(np.int32)


def select_blocks(q, lo, hi, k, *, shared=False):
    s = bound_scores_fp64(q, lo, hi)
    if shared:
        g = s.shape[0] // lo.shape[0]
        rows = stable_topk(group_scores_fp64(s, g), k)
        return np.repeat(rows, g, axis=0)
    return stable_topk(s, k)


def shard_select(q, lo, hi, k, shards):
    """Context-parallel selection: each shard owns a contiguous block range,
    picks its local top-k (score, global id), and the candidates merge to the
    global strict top-k. Equal to select_blocks by construction."""
    s = bound_scores_fp64(q, lo, hi)
    n = s.shape[1]
    bounds = np.linspace(0, n, shards + 1).astype(int)
    cand_ids, cand_scores = [], []
    for r in range(shards):
        a, b = bounds[r], bounds[r + 1]
        loc = stable_topk(s[:, a:b], min(k, b - a)) + a
        cand_ids.append(loc)
        cand_scores.append(np.take_along_axis(s, loc, axis=1))
    ids = np.concatenate(cand_ids, axis=1)
    sc = np.concatenate(cand_scores, axis=1)
    pick = np.lexsort((ids, -sc), axis=1)[:, :k]
    return np.sort(np.take_along_axis(ids, pick, axis=1), axis=1).astype(np.int32)


def order_keys(scores):
    """64-bit order keys of FP64 scores: unsigned-integer order equals score
    order (-0 folded to +0). The candidate exchange format of the
    context-parallel path (new; the reference selects on one GPU)."""
    b = (np.asarray(scores, dtype=np.float64) + 0.0).view(np.uint64)
    neg = (b >> np.uint64(63)) != 0
    return np.where(neg, ~b, b | np.uint64(1 << 63))
