"""The reference's serial strict decode step on the host CPU (timed baseline).

Restates, with torch CPU tensors and all intra-op threads, the reference's
own torch code path for one decode step:
  selection  benchmarks/run_benchmark.py:44-51  torch.where(q >= 0, hi*q, lo*q).sum(-1).topk(K)
             (native GQA metadata indexed by h // G, as gqa.py:15-26)
  attention  benchmarks/critical_path.py:16-25  FP64 softmax attention over the selected blocks
This is test / benchmark infrastructure: bench.py's cpu_baseline and
``--impl reference`` legs time it; the product never calls it.
"""
from __future__ import annotations

import math

import torch


def serial_step(q, k, v, lo, hi, topk, heads=None):
    """One strict decode step for query heads ``heads`` (default: all)."""
    hq = q.shape[0]
    g = hq // lo.shape[0]
    hs = torch.arange(hq) if heads is None else torch.as_tensor(heads)
    kvh = hs // g
    qf = q[hs].float()[:, None, :]
    lo_h, hi_h = lo[kvh], hi[kvh]
    scores = torch.where(qf >= 0, hi_h * qf, lo_h * qf).sum(-1)
    ids = scores.topk(topk, sorted=False).indices
    keys = k[kvh[:, None], ids].double()
    values = v[kvh[:, None], ids].double()
    logits = torch.einsum("hd,hsbd->hsb", q[hs].double(), keys) / math.sqrt(q.shape[1])
    w = logits.flatten(1).softmax(-1).view_as(logits)
    return torch.einsum("hsb,hsbd->hd", w, values), ids
