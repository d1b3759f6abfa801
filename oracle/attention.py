"""FP64 strict attention over selected blocks — the reference's own test oracle.

Restates tests/check_correctness.py:12-17 (expanded KV), tests/check_gqa.py:10-17
and benchmarks/critical_path.py:16-25 (native GQA, optional include mask).
"""
from __future__ import annotations

import numpy as np


def attention_fp64(q, k, v, ids, include=None):
    """q [H, D], k/v [Hkv, N, B, D], ids [H, S] -> [H, D] float64."""
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k)
    v = np.asarray(v)
    ids = np.asarray(ids).astype(np.int64)
    h, d = q.shape
    g = h // k.shape[0]
    out = np.empty((h, d))
    for i in range(h):
        ks = k[i // g][ids[i]].astype(np.float64)  # [S, B, D]
        vs = v[i // g][ids[i]].astype(np.float64)
        logits = ks @ q[i] / np.sqrt(d)  # [S, B]
        if include is not None:
            logits = np.where(np.asarray(include)[i][:, None], logits, -np.inf)
        flat = logits.reshape(-1)
        w = np.exp(flat - flat.max())
        w = (w / w.sum()).reshape(logits.shape)
        out[i] = np.einsum("sb,sbd->d", w, vs)
    return out


def union_ids(selected, predicted):
    """Row-wise union, predicted first then selected misses (gqa.repair_union semantics)."""
    rows = []
    for a, p in zip(np.asarray(selected).tolist(), np.asarray(predicted).tolist()):
        ps = set(p)
        rows.append(list(p) + [x for x in a if x not in ps])
    width = max(len(r) for r in rows)
    assert all(len(r) == width for r in rows), "union rows must have equal length"
    return np.array(rows, dtype=np.int64)
