"""On-device prediction of the next step's block list.

The reference's predictor policies (experiments/hisparse_cache_trace.py:40-57
``predict``; experiments/predictor_rank_trace.py:37-48 ``interleave``;
experiments/trace_replay.py:74-75,111 feeds the previous step's selection back
as the next prediction) as one kernel, stk_predict, so a decode loop never
leaves the GPU between steps:

* ``previous_step``  — the first ``budget`` IDs of the previous step's ranking;
* ``previous_layer`` — the first ``budget`` IDs of the previous layer's ranking;
* ``rank_interleave`` — slots alternate between the two rankings (the step's
  first), each slot taking its source's next ID not already taken.

A ranking is a selection row, best first, ties to the lower block ID. Pass the
order keys that selection can write (``selector.topk_from_metadata(...,
keys_out=...)``) to rank a row by score; without keys the row is used in its
given order. Where an interleave source runs out (the reference raises), the
other source fills the slot; slots that no source can fill are -1, which every
kernel of this library treats as an empty slot.
"""
from __future__ import annotations

import torch

from . import _lib as L

POLICIES = {"previous_step": L.PREDICT_PREVIOUS_STEP, "previous_layer": L.PREDICT_PREVIOUS_LAYER,
            "rank_interleave": L.PREDICT_RANK_INTERLEAVE}


def _rows(ids, keys, name):
    if ids is None:
        return None, None, 0
    if ids.ndim != 2 or ids.dtype != torch.int32 or not ids.is_cuda or not ids.is_contiguous():
        raise ValueError(f"{name} must be a contiguous CUDA int32 [rows, k] tensor")
    if keys is not None and (keys.shape != ids.shape or keys.dtype != torch.int64 or not keys.is_contiguous()):
        raise ValueError(f"{name} keys must be int64 order keys shaped like the IDs")
    return ids, keys, ids.shape[1]


def predict(policy: str, budget: int, n_blocks: int, *, previous_step=None, previous_step_keys=None,
            previous_layer=None, previous_layer_keys=None, out=None):
    """Predicted IDs [rows, budget] int32 for the next step."""
    if policy not in POLICIES:
        raise ValueError(f"unknown policy: {policy}")
    s_ids, s_keys, ks = _rows(previous_step, previous_step_keys, "previous_step")
    l_ids, l_keys, kl = _rows(previous_layer, previous_layer_keys, "previous_layer")
    ref = s_ids if s_ids is not None else l_ids
    if ref is None:
        raise ValueError("a previous selection is required")
    rows = ref.shape[0]
    if s_ids is not None and l_ids is not None and s_ids.shape[0] != l_ids.shape[0]:
        raise ValueError("previous_step and previous_layer must have the same rows")
    if out is None:
        out = torch.empty((rows, budget), device=ref.device, dtype=torch.int32)
    rc = L.load().stk_predict(POLICIES[policy], L.ptr(s_ids), L.ptr(s_keys), ks, L.ptr(l_ids), L.ptr(l_keys), kl,
                              rows, int(n_blocks), int(budget), out.data_ptr(), L.status_ptr(), L.stream_of(ref))
    L.check(rc, "predict")
    return out
