"""Single-launch saved-state repair for native GQA with few late misses.

Drop-in for ``strict_topk.gqa_light`` (reference gqa_light.py:1-92). On
sm_100a both schedules of the reference run through the same one-launch
repair kernel; the static dispatch of ``repair_saved_auto`` is kept.
"""
from __future__ import annotations

from . import gqa


def repair_saved_light(q, k, v, selected, predicted, state):
    """Repair the strict selected set with one CTA per query head."""
    return gqa.repair_saved(q, k, v, selected, predicted, state)


def repair_saved_auto(q, k, v, selected, predicted, state, expected_miss_fraction):
    """Choose a repair schedule using an external estimate from past steps.

    The threshold of two expected misses per head and at least 16 query heads
    is the reference's static scheduling hypothesis (gqa_light.py:80-92). Both
    schedules compute the strict selected set whatever the estimate.
    """
    if not 0 <= expected_miss_fraction <= 1:
        raise ValueError("expected_miss_fraction must be in [0, 1]")
    if (q.ndim == 2 and q.shape[0] >= 16 and selected.ndim == 2
            and selected.shape[1] * expected_miss_fraction <= 2):
        return repair_saved_light(q, k, v, selected, predicted, state)
    return gqa.repair_saved(q, k, v, selected, predicted, state)
