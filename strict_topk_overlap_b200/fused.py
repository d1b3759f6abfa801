"""Single-launch repair for the prediction states of ``kernels.speculate``.

Drop-in for ``strict_topk.fused`` (reference fused.py:1-220).
"""
from __future__ import annotations

from . import _lib as L
from .kernels import RepairResult, _run_repair, _shape


def repair_fused(q, k, v, selected, predicted, prediction,
                 min_remaining=1.e-3, cancellation_tol=1.e-5,
                 max_extra_mass=0.):
    """Repair finite Q/K/V with valid, unique IDs in one launch.

    The cancellation and remaining-mass guards operate in the original
    low-group exponent frame; wrong low blocks are re-evaluated per token at
    the low group's maximum. A positive max_extra_mass opts into retaining
    wrong low blocks if their estimated share of the output softmax is within
    that budget (reference fused.py:176-220).
    """
    h, n, b, d, sa = _shape(q, k, v, selected)
    _shape(q, k, v, predicted)
    hybrid = prediction.mode in ("hybrid", "compact")
    if not 0 <= max_extra_mass <= 1:
        raise ValueError("max_extra_mass must be in [0, 1]")
    if hybrid and max_extra_mass > 0 and (prediction.mass_m is None or prediction.mass_l is None):
        raise ValueError("positive max_extra_mass requires speculate(..., keep_mass=True)")
    out, fallback, remaining, approx, extra, _, _ = _run_repair(
        q, k, v, selected, predicted, prediction, L.VAR_FUSED, min_remaining=min_remaining,
        cancellation_tol=cancellation_tol, max_extra_mass=max_extra_mass, want_approx=max_extra_mass > 0)
    return RepairResult(out, fallback, remaining, approx, extra)
