"""B200-native (sm_100a) strict Top-K speculative block-sparse decode.

The public API mirrors the reference ``strict_topk`` package module by
module; ``import strict_topk`` (the top-level alias package) resolves to
these modules. Device work runs in libstk_sm100.so through its C ABI
(include/strict_topk_b200.h); there is no CPU or Triton fallback.
"""
from .kernels import (PartialState, Prediction, RepairResult, block_partials, exact_attention,  # noqa: F401
                      merge_partials, repair, speculate, touch_kv)

__all__ = ["PartialState", "Prediction", "RepairResult", "block_partials",
           "merge_partials", "exact_attention", "speculate", "repair", "touch_kv"]
