"""Signed corrections for saved, hybrid and compact prediction states.

Drop-in for ``strict_topk.signed_repair`` (reference signed_repair.py:1-232):
misses are added (+) and wrong low blocks subtracted (-) from the low group;
here the queue, the signed block work, the guarded merge and the fallback
share one launch.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib as L
from .kernels import RepairResult, _run_repair, _shape


@dataclass
class SignedRepairResult(RepairResult):
    positive_jobs: torch.Tensor | None = None
    total_jobs: torch.Tensor | None = None


def _signed(q, k, v, selected, predicted, prediction, min_remaining, cancellation_tol, max_extra_mass, variant):
    _shape(q, k, v, selected)
    _shape(q, k, v, predicted)
    hybrid = prediction.mode in ("hybrid", "compact")
    if not 0 <= max_extra_mass <= 1:
        raise ValueError("max_extra_mass must be in [0, 1]")
    if hybrid and max_extra_mass > 0 and (prediction.mass_m is None or prediction.mass_l is None):
        raise ValueError("positive max_extra_mass requires speculate(..., keep_mass=True)")
    out, bad, remain, approx, extra, pos, total = _run_repair(
        q, k, v, selected, predicted, prediction, variant, min_remaining=min_remaining,
        cancellation_tol=cancellation_tol, max_extra_mass=max_extra_mass, want_approx=max_extra_mass > 0,
        want_jobs=True)
    return SignedRepairResult(out, bad, remain, approx, extra, pos, total)


def repair_signed(q, k, v, selected, predicted, prediction, min_remaining=1.e-3,
                  cancellation_tol=1.e-5, max_extra_mass=0.):
    """Repair with one signed correction queue (misses first, then wrong low
    blocks); wrong blocks enter as block-local states rescaled to the low
    group's frame. Positive and total job counts describe the queue before
    fallback."""
    return _signed(q, k, v, selected, predicted, prediction, min_remaining, cancellation_tol, max_extra_mass,
                   L.VAR_SIGNED)
