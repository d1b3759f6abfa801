"""CPU stand-in for the per-shard device work of the context-parallel decode
step — TEST INFRASTRUCTURE (the checker of strict_topk_overlap_b200's
context_parallel orchestration; never the product).

Implements the ``DeviceShard`` interface of the context-parallel module in
FP64 NumPy on torch CPU tensors, so that CPU ranks (gloo) run the very same
exchange logic:
  local_candidates  fixed-order FP64 bound scores (selection.py) and stable
                    Top-K, plus order keys (selection.order_keys)
  merge_candidates  Top-K by (key desc, candidate position asc)
  block_states      per-block (m, l, u) of kernels.py:42-71 (_partial), FP64
  reduce_states     LSE reduction to one unnormalised state (kernels.py:74-91)
  merge_states      LSE merge and normalisation (kernels.py:74-91, _merge)
"""
from __future__ import annotations

import numpy as np
import torch

from . import selection as S


class OracleShard:
    @staticmethod
    def local_candidates(q, lo, hi, topk, id_base):
        s = S.bound_scores_fp64(q.numpy(), lo.numpy(), hi.numpy())
        loc = S.stable_topk(s, topk)
        keys = S.order_keys(np.take_along_axis(s, loc.astype(np.int64), axis=1)).view(np.int64)
        return torch.from_numpy(keys.copy()), torch.from_numpy((loc + id_base).astype(np.int32))

    @staticmethod
    def merge_candidates(keys, ids, topk):
        k = keys.numpy().view(np.uint64)
        rows, n = k.shape
        out = np.empty((rows, topk), dtype=np.int32)
        pos = np.arange(n)
        for r in range(rows):
            # Descending key, ascending position: sort ascending on (~key, pos).
            pick = np.lexsort((pos, ~k[r]))[:topk]
            out[r] = np.sort(ids.numpy()[r][pick])
        return torch.from_numpy(out)

    @staticmethod
    def block_states(q, k, v, ids, pred=None):
        qn = q.double().numpy()
        kn, vn = k.double().numpy(), v.double().numpy()
        idn = ids.numpy().astype(np.int64)
        rows, s = idn.shape
        d = qn.shape[1]
        g = rows // kn.shape[0]
        m = np.full((rows, s), -np.inf)
        lsum = np.zeros((rows, s))
        u = np.zeros((rows, s, d))
        slot = None if pred is None else np.full((rows, s), -1, dtype=np.int32)
        for r in range(rows):
            for j in range(s):
                b = idn[r, j]
                if b < 0:
                    continue
                if pred is not None:
                    hits = np.nonzero(pred.numpy()[r] == b)[0]
                    if hits.size:
                        slot[r, j] = hits.max()
                        m[r, j], lsum[r, j], u[r, j] = np.nan, np.nan, np.nan  # unwritten, like the device
                        continue
                x = kn[r // g, b] @ qn[r] / np.sqrt(d)
                m[r, j] = x.max()
                w = np.exp(x - m[r, j])
                lsum[r, j] = w.sum()
                u[r, j] = w @ vn[r // g, b]
        return (torch.from_numpy(m), torch.from_numpy(lsum), torch.from_numpy(u),
                None if slot is None else torch.from_numpy(slot))

    @staticmethod
    def reduce_states(m, l, u, include=None):
        mn, ln, un = m.numpy(), l.numpy(), u.numpy()
        inc = np.ones(mn.shape, bool) if include is None else include.numpy().astype(bool)
        inc = inc & (mn != -np.inf)
        M = np.where(inc, mn, -np.inf).max(1)
        with np.errstate(invalid="ignore"):
            w = np.where(inc, np.exp(np.where(inc, mn, 0.0) - np.where(np.isfinite(M), M, 0.0)[:, None]), 0.0)
        lo = (w * np.where(inc, ln, 0.0)).sum(1)
        uo = np.einsum("rs,rsd->rd", w, np.where(inc[:, :, None], un, 0.0))
        return torch.from_numpy(M), torch.from_numpy(lo), torch.from_numpy(uo)

    @staticmethod
    def merge_states(m, l, u):
        mn, ln, un = m.numpy(), l.numpy(), u.numpy()
        M = mn.max(1)
        M = np.where(np.isfinite(M), M, 0.0)
        w = np.exp(mn - M[:, None])
        z = (w * ln).sum(1)
        return torch.from_numpy(np.einsum("rs,rsd->rd", w, un) / z[:, None])
