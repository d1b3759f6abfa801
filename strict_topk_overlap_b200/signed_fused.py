"""Signed block correction with a shared low-group scale and inline fallback.

Drop-in for ``strict_topk.signed_fused`` (reference signed_fused.py:1-193).
Hybrid negatives are evaluated block-locally and rescaled to the low frame
(reproducing the preparation's underflow order); compact negatives use the
low frame per token.
"""
from __future__ import annotations

from . import _lib as L
from .signed_repair import SignedRepairResult, _signed

__all__ = ["SignedRepairResult", "repair_signed_fused"]


def repair_signed_fused(q, k, v, selected, predicted, prediction, min_remaining=1.e-3,
                        cancellation_tol=1.e-5, max_extra_mass=0.):
    """One shared add/erase KV pass followed by guarded finalization, with the
    strict fallback inline (one launch here, three in the reference)."""
    return _signed(q, k, v, selected, predicted, prediction, min_remaining, cancellation_tol, max_extra_mass,
                   L.VAR_SIGNED_FUSED)
