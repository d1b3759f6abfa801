"""Tiny-block GQA attention with bounded on-chip merging.

Drop-in for ``strict_topk.gqa_hierarchical`` (reference
gqa_hierarchical.py:1-144). Per-block states keep the reference's layout;
exact and repair reductions merge on chip inside one launch.
"""
from __future__ import annotations

from . import _lib as L
from . import gqa
from .kernels import Prediction, _run_repair, merge_partials


def partials(q, k, v, selected):
    return gqa.partials(q, k, v, selected)


def exact(q, k, v, selected):
    """Attention over the selected blocks. Tiny blocks (<= 8 tokens: the
    shape this module serves) take the reference's own structure,
    per-block states then one merge (gqa_hierarchical.py:111-112, 99-109), where the
    state kernel keeps eight blocks in flight per warp; larger blocks use the
    one-launch attention."""
    h, n, b, d, group, sa = gqa._shape(q, k, v, selected)
    if b <= 8:
        return merge_partials(gqa.partials(q, k, v, selected))
    out, *_ = _run_repair(q, k, v, selected, None, None, L.VAR_SAVED)
    return out


def _repair(q, k, v, selected, predicted, state, shared):
    h, n, b, d, group, sa = gqa._shape(q, k, v, selected)
    gqa._validate_ids(q, predicted)
    sp = predicted.shape[1]
    if state.u.shape != (h, sp, d) or state.m.shape != (h, sp) or state.l.shape != (h, sp):
        raise ValueError('prediction state shape does not match predicted blocks')
    out, *_ = _run_repair(q, k, v, selected, predicted, Prediction(state, "saved"), L.VAR_SAVED)
    return out


def repair_saved(q, k, v, selected, predicted, state):
    return _repair(q, k, v, selected, predicted, state, False)


def repair_saved_shared(q, k, v, selected, predicted, state):
    """Shared selection: every head has identical ordered IDs (caller-validated
    contract). Membership is resolved per row on chip, so the result equals
    repair_saved; attention states stay independent for every query head."""
    return _repair(q, k, v, selected, predicted, state, True)


select_blocks_shared = gqa.select_blocks_shared
