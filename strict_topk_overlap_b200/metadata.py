"""Block metadata: per-block min / max of K, built once and kept current.

Replaces the prefill-time ``lo, hi = k.amin(dim=2).float(), k.amax(dim=2).float()``
of the reference (benchmarks/run_benchmark.py:42-43, experiments/trace_replay.py:68)
with ``build_metadata`` (stk_build_metadata), and adds ``append_token``
(stk_append_token): the decode-loop step that writes one new token per
request into the KV cache and folds its key into the block's bounds, so the
metadata is never rebuilt. Both are bit-identical to recomputing amin/amax
over the block's filled tokens.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib as L


def build_metadata(k: torch.Tensor):
    """lo, hi [Hkv, N, D] FP32 for a dense K [Hkv, N, B, D] (any of f32/f16/bf16)."""
    if k.ndim != 4 or not k.is_cuda or not k.is_contiguous():
        raise ValueError("expected a contiguous CUDA K [Hkv, N, B, D]")
    hkv, n, b, d = k.shape
    lo = torch.empty((hkv, n, d), device=k.device, dtype=torch.float32)
    hi = torch.empty_like(lo)
    kv = L.kv_struct(k, k)
    rc = L.load().stk_build_metadata(C.byref(kv), 1, n, lo.data_ptr(), hi.data_ptr(), L.status_ptr(), L.stream_of(k))
    L.check(rc, "build_metadata")
    return lo, hi


def append_token(k: torch.Tensor, v: torch.Tensor, lo: torch.Tensor, hi: torch.Tensor, k_new: torch.Tensor,
                 v_new: torch.Tensor, position: int | torch.Tensor):
    """Write token `position` of a dense single-request cache K/V [Hkv, N, B, D]
    from k_new / v_new [Hkv, D] and update lo/hi [Hkv, N, D] in place.
    `position` may be a one-element int32 CUDA tensor (graph-capturable)."""
    hkv, n, b, d = k.shape
    if k_new.shape != (hkv, d) or v_new.shape != (hkv, d) or k_new.dtype != k.dtype or v_new.dtype != v.dtype:
        raise ValueError("k_new / v_new must be [Hkv, D] in the cache's dtype")
    if lo.shape != (hkv, n, d) or hi.shape != lo.shape:
        raise ValueError("lo / hi must be [Hkv, N, D] FP32")
    if not isinstance(position, torch.Tensor):
        if not 0 <= int(position) < n * b:
            raise ValueError(f"position {position} outside the cache's {n * b} tokens")
        position = torch.tensor([int(position)], dtype=torch.int32, device=k.device)
    kv = L.kv_struct(k, v)
    rc = L.load().stk_append_token(C.byref(kv), 1, n, k_new.contiguous().data_ptr(), v_new.contiguous().data_ptr(),
                                   position.data_ptr(), lo.data_ptr(), hi.data_ptr(), L.status_ptr(),
                                   L.stream_of(k))
    L.check(rc, "append_token")
