"""CPU restatement of the reference's next-step predictor policies — TEST
INFRASTRUCTURE (the checker of strict_topk_overlap_b200.predictor).

Follows experiments/hisparse_cache_trace.py:40-57 ``predict`` (previous_step,
previous_layer, rank_interleave) and experiments/predictor_rank_trace.py:37-48
``interleave``, on ranked lists (best first). ``rank_by_keys`` turns a
selection row plus its 64-bit order keys into that ranking (descending key,
ties to the lower position), as the reference's stable descending argsort of
scores does (predictor_rank_trace.py:26-27). Where the reference raises
because an interleave source ran out, this restatement — like the device
kernel — lets the other source fill the slot and pads with -1.
"""
from __future__ import annotations

import numpy as np


def rank_by_keys(ids, keys):
    ids = list(ids)
    if keys is None:
        return ids
    keys = np.asarray(keys).view(np.uint64)
    order = sorted(range(len(ids)), key=lambda i: (-int(keys[i]), i))
    return [ids[i] for i in order]


def predict(policy, previous_step, previous_layer, budget):
    """One row: previous_step / previous_layer are ranked ID lists."""
    if policy == "previous_step":
        return list(previous_step[:budget]) + [-1] * max(0, budget - len(previous_step))
    if policy == "previous_layer":
        return list(previous_layer[:budget]) + [-1] * max(0, budget - len(previous_layer))
    if policy != "rank_interleave":
        raise ValueError(f"unknown policy: {policy}")
    sources = (list(previous_step), list(previous_layer))
    pos = [0, 0]
    seen, out = set(), []

    def take(s):
        while pos[s] < len(sources[s]):
            b = sources[s][pos[s]]
            pos[s] += 1
            if b not in seen:
                seen.add(b)
                return b
        return None

    for slot in range(budget):
        b = take(slot % 2)
        if b is None:
            b = take(1 - slot % 2)
        out.append(-1 if b is None else b)
    return out
