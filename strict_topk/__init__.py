"""Drop-in alias: ``strict_topk`` resolves to the sm_100a implementation.

Code written against the reference package (``from strict_topk import gqa``,
``from strict_topk.fused import repair_fused`` ...) runs unchanged; each
submodule below is the corresponding module of ``strict_topk_overlap_b200``.
"""
import importlib
import sys

from strict_topk_overlap_b200 import *  # noqa: F401,F403
from strict_topk_overlap_b200 import __all__  # noqa: F401

for _name in ("kernels", "selector", "fused", "gqa", "gqa_light", "gqa_hierarchical",
              "signed_repair", "signed_fused"):
    _mod = importlib.import_module(f"strict_topk_overlap_b200.{_name}")
    sys.modules[f"{__name__}.{_name}"] = _mod
    globals()[_name] = _mod
del importlib, sys, _name, _mod
