"""Tiny-block GQA attention with bounded on-chip merging.

Drop-in for ``strict_topk.gqa_hierarchical`` (reference
gqa_hierarchical.py:1-144). Per-block states keep the reference's layout;
exact and repair reductions merge on chip inside one launch.
"""
from __future__ import annotations

import ctypes as C

import torch

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


def _group_tile_ok(q, k, selected, predicted):
    """Shapes the tensor-core group repair takes: q and K/V in one 16-bit
    dtype, D 64 or 128, blocks dividing 64 tokens, a dense tile of 8..16
    query heads per KV head, int32 contiguous lists."""
    hq, d = q.shape
    hkv, n, b, _ = k.shape
    g = hq // hkv
    return (q.dtype == k.dtype and q.dtype in (torch.bfloat16, torch.float16) and d in (64, 128)
            and 64 % b == 0 and 8 <= g <= 16 and hq % hkv == 0
            and selected.dtype == torch.int32 and predicted.dtype == torch.int32
            and selected.is_contiguous() and predicted.is_contiguous())


def repair_saved_shared(q, k, v, selected, predicted, state):
    """Shared selection: every head of a KV group has identical ordered IDs
    (caller-validated contract, as in the reference; membership is taken from
    each group's first row). Where the group forms a dense tensor-core tile
    (8..16 query heads per KV head, 16-bit q and K/V, D 64 or 128), the
    misses are attended on the group's MMA tile, each missed block read once
    per group, and every head folds its own saved states of the hits
    (stk_group_repair_saved); other shapes resolve membership per row on
    chip. Attention states stay independent for every query head."""
    h, n, b, d, group, sa = gqa._shape(q, k, v, selected)
    gqa._validate_ids(q, predicted)
    sp = predicted.shape[1]
    if state.u.shape != (h, sp, d) or state.m.shape != (h, sp) or state.l.shape != (h, sp):
        raise ValueError('prediction state shape does not match predicted blocks')
    if not _group_tile_ok(q, k, selected, predicted):
        return _repair(q, k, v, selected, predicted, state, True)
    lib = L.load()
    out = torch.empty((h, d), device=q.device, dtype=torch.float32)
    ws_bytes = lib.stk_group_repair_saved_workspace_bytes(h, k.shape[0], sa, sp, b, d)
    ws = torch.empty((ws_bytes,), device=q.device, dtype=torch.uint8)
    kv = L.kv_struct(k, v)
    rc = lib.stk_group_repair_saved(C.byref(kv), q.data_ptr(), L.dtype_code(q), h, selected.data_ptr(), sa,
                                    predicted.data_ptr(), sp, state.m.contiguous().data_ptr(),
                                    state.l.contiguous().data_ptr(), state.u.contiguous().data_ptr(), out.data_ptr(),
                                    ws.data_ptr(), ws_bytes, L.status_ptr(), L.stream_of(q))
    L.check(rc, "group_repair_saved")
    return out


select_blocks_shared = gqa.select_blocks_shared


def exact_shared(q, k, v, group_selected):
    """Attention of every query head over its KV group's shared block list
    group_selected [Hkv, S] (the rows select_blocks_shared repeats per head),
    on the tensor cores: the Hq / Hkv (<= 16) heads of a group form one MMA
    tile, so each listed block is read once per group. q and K/V both bf16 or
    both f16, D 64 or 128. Equals exact(q, k, v, group rows repeated per
    head) within FP32 rounding."""
    if group_selected.ndim != 2 or group_selected.dtype != torch.int32 or not group_selected.is_contiguous():
        raise ValueError("group_selected must be a contiguous int32 [Hkv, S] tensor")
    hq, d = q.shape
    hkv, n, b, _ = k.shape
    if group_selected.shape[0] != hkv or q.dtype != k.dtype or q.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError("expected one list per KV head and q, K, V of one 16-bit dtype")
    sa = group_selected.shape[1]
    out = torch.empty((hq, d), device=q.device, dtype=torch.float32)
    lib = L.load()
    ws_bytes = lib.stk_group_attention_workspace_bytes(hq, sa, b, d)
    ws = torch.empty((ws_bytes,), device=q.device, dtype=torch.uint8)
    kv = L.kv_struct(k, v)
    rc = lib.stk_group_attention(C.byref(kv), q.data_ptr(), L.dtype_code(q), hq, group_selected.data_ptr(), sa,
                                 out.data_ptr(), ws.data_ptr(), ws_bytes, L.status_ptr(), L.stream_of(q))
    L.check(rc, "group_attention")
    return out
