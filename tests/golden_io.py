"""Fixture loading shared by the CPU and GPU parity tests."""
from __future__ import annotations

from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name: str):
    return np.load(GOLDEN / f"{name}.npz", allow_pickle=False)


def field(fx, key, default=None):
    return fx[key] if key in fx.files else default


def ref_tol_ok(out, expected, atol=3e-4, rtol=3e-4):
    """Reference tolerance (tests/check_correctness.py:20-32): |err| <= atol + rtol*|ref| and finite."""
    out = np.asarray(out, dtype=np.float64)
    expected = np.asarray(expected, dtype=np.float64)
    return bool(np.isfinite(out).all() and (np.abs(out - expected) <= atol + rtol * np.abs(expected)).all())


MODES = [("saved", 0.1), ("hybrid", 0.05), ("hybrid", 0.2), ("hybrid", 1.0),
         ("compact", 0.05), ("compact", 0.2), ("compact", 1.0)]
VARIANTS = [("split", "split", 0.), ("fused", "fused", 0.), ("signed", "signed", 0.),
            ("signed_fused", "signed_fused", 0.), ("fused_eps", "fused", 0.01), ("signed_eps", "signed", 0.01),
            ("signed_fused_eps", "signed_fused", 0.01)]
