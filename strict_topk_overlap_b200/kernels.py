"""Per-block FP32 softmax states, speculation and split repair on sm_100a.

Drop-in for ``strict_topk.kernels`` (reference kernels.py:1-560). Inputs are
contiguous Q[H,D] and K/V[Hkv,N,B,D] on one CUDA device, with H a multiple
of Hkv (Hkv == H is the reference's expanded layout; Hkv < H reads shared
GQA heads natively, query head h using KV head h // (H // Hkv)). ID rows are
unique, valid, int32 or int64, without padding. Every call is asynchronous on
the current CUDA stream and capturable in a CUDA graph; the caller orders KV
writes before either stream of an overlapped step.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _lib as L


@dataclass
class PartialState:
    """FP32 block states: m = max logit, l = sum exp(s-m), u = sum exp(s-m) v."""
    m: torch.Tensor
    l: torch.Tensor
    u: torch.Tensor


@dataclass
class Prediction:
    """Speculative states for predicted IDs (reference kernels.py:20-30)."""
    state: PartialState
    mode: str
    high: torch.Tensor | None = None
    low: PartialState | None = None
    retained_ids: torch.Tensor | None = None
    overflow: torch.Tensor | None = None
    low_abs: torch.Tensor | None = None
    mass_m: torch.Tensor | None = None
    mass_l: torch.Tensor | None = None


@dataclass
class RepairResult:
    output: torch.Tensor
    fallback: torch.Tensor
    remaining: torch.Tensor
    approximate_heads: torch.Tensor | None = None
    extra_mass_bound: torch.Tensor | None = None


def _shape(q, k, v, ids):
    """Shape contract of kernels.py:410-417 (AssertionError on violation),
    widened to native GQA: Q heads must be a multiple of K/V heads."""
    assert q.is_cuda and k.is_cuda and v.is_cuda and ids.is_cuda
    assert q.ndim == 2 and k.ndim == 4 and v.shape == k.shape
    hkv, n, b, d = k.shape
    h = q.shape[0]
    assert q.shape[1] == d and h % hkv == 0 and ids.ndim == 2 and ids.shape[0] == h
    assert ids.dtype in (torch.int32, torch.int64) and ids.shape[1] > 0
    assert all(x.is_contiguous() for x in (q, k, v, ids))
    assert all(x.device == q.device for x in (k, v, ids))
    return h, n, b, d, ids.shape[1]


def _allocate_state(h, s, d, device):
    m = torch.empty((h, s), device=device, dtype=torch.float32)
    return PartialState(m, torch.empty_like(m), torch.empty((h, s, d), device=device, dtype=torch.float32))


def _block_states(q, k, v, ids, *, active=None, active_invert=False, mode=L.MODE_FULL, frame=None,
                  pred=None, slot_out=None, out=None, uabs=None):
    """Launch the per-block job kernel; returns ``out`` (a PartialState)."""
    h = q.shape[0]
    s = ids.shape[1]
    kv = L.kv_struct(k, v)
    active_mode = 0 if active is None else (1 if active.ndim == 1 else 2)
    lib = L.load()
    rc = lib.stk_block_states(
        C.byref(kv), q.data_ptr(), L.dtype_code(q), h, h, ids.data_ptr(), L.id_is64(ids), s,
        L.ptr(active), active_mode, int(active_invert), L.ptr(pred),
        L.id_is64(pred) if pred is not None else 0, pred.shape[1] if pred is not None else 0,
        L.ptr(slot_out), mode, L.ptr(frame), L.ptr(out.m) if out is not None else None,
        L.ptr(out.l) if out is not None else None, L.ptr(out.u) if out is not None else None, L.ptr(uabs),
        L.status_ptr(), L.stream_of(q))
    L.check(rc, "block_states")
    return out


def block_partials(q, k, v, ids, active=None):
    """Each block's m, sum exp(logit-m), sum exp(logit-m)*V (all FP32).

    ``active`` ([H] or [H,S] bool) marks blocks to compute; inactive slots hold
    (-inf, 0, 0) (reference kernels.py:425-434)."""
    h, n, b, d, s = _shape(q, k, v, ids)
    state = _allocate_state(h, s, d, q.device)
    if active is not None:
        assert active.is_contiguous() and active.shape in ((h,), (h, s)) and active.dtype == torch.bool
    return _block_states(q, k, v, ids, active=active, out=state)


def merge_partials(state, include=None):
    """LSE merge of states [H,S] (+ optional include mask) -> FP32 [H,D]
    (reference kernels.py:437-442)."""
    h, s, d = state.u.shape
    out = torch.empty((h, d), device=state.u.device, dtype=torch.float32)
    if include is not None:
        assert include.shape == (h, s) and include.dtype == torch.bool and include.is_contiguous()
    rc = L.load().stk_merge_states(state.m.data_ptr(), state.l.data_ptr(), state.u.data_ptr(), L.ptr(include),
                                   h, s, d, out.data_ptr(), L.stream_of(state.u))
    L.check(rc, "merge_states")
    return out


def exact_attention(q, k, v, selected):
    """Split-block, selected-set baseline, with the same FP32 accumulation:
    per-block partials merged on chip in one launch (kernels.py:445-447)."""
    _shape(q, k, v, selected)
    out, *_ = _run_repair(q, k, v, selected, None, None, L.VAR_SAVED)
    return out


def compact_capacity(s: int, mass_threshold: float) -> int:
    """Retained-slot capacity of compact mode (reference kernels.py:485)."""
    return s if mass_threshold <= 1 / s else min(s, int(1 / mass_threshold) + 1)


def speculate(q, k, v, predicted, mode='saved', mass_threshold=0.1, *, keep_mass=False):
    """Speculate using CURRENT Q. Threshold uses actual predicted-set mass.

    saved: per-block states; hybrid: per-block states plus high mask and a
    low-mass aggregate with its absolute numerator envelope; compact: a
    K-only statistics pass, capacity-bounded retained states and a per-token
    low aggregate (reference kernels.py:450-501). ``keep_mass`` exposes the
    per-block maxima and normalizers in predicted order.
    """
    if mode not in ('saved', 'hybrid', 'compact'):
        raise ValueError(mode)
    if not 0 <= mass_threshold <= 1:
        raise ValueError('mass_threshold must be in [0,1]')
    h, n, b, d, s = _shape(q, k, v, predicted)
    dev = q.device
    kv = L.kv_struct(k, v)
    pmode = L.PRED_MODES[mode]
    sc = compact_capacity(s, mass_threshold) if mode == 'compact' else s
    state = _allocate_state(h, sc, d, dev)
    high = low = low_abs = rids = overflow = pm = pl = None
    if mode != 'saved':
        high = torch.empty((h, s), device=dev, dtype=torch.bool)
        low = _allocate_state(h, 1, d, dev)
        low_abs = torch.empty((h, d), device=dev, dtype=torch.float32)
    if mode == 'compact':
        rids = torch.empty((h, sc), device=dev, dtype=predicted.dtype)
        overflow = torch.empty((h,), device=dev, dtype=torch.bool)
        pm = torch.empty((h, s), device=dev, dtype=torch.float32)
        pl = torch.empty_like(pm)
    lib = L.load()
    ws_bytes = lib.stk_speculate_workspace_bytes(h, s, d, pmode)
    ws = torch.empty((max(ws_bytes, 1),), device=dev, dtype=torch.uint8)
    rc = lib.stk_speculate(
        C.byref(kv), q.data_ptr(), L.dtype_code(q), h, h, predicted.data_ptr(), L.id_is64(predicted), s, pmode,
        float(mass_threshold), sc, state.m.data_ptr(), state.l.data_ptr(), state.u.data_ptr(), L.ptr(high),
        L.ptr(rids), L.ptr(low.m) if low else None, L.ptr(low.l) if low else None, L.ptr(low.u) if low else None,
        L.ptr(low_abs), L.ptr(overflow), L.ptr(pm), L.ptr(pl), ws.data_ptr(), ws_bytes, L.status_ptr(),
        L.stream_of(q))
    L.check(rc, "speculate")
    if mode == 'compact':
        mass_m, mass_l = (pm, pl) if keep_mass else (None, None)
        return Prediction(state, 'compact', high, low, rids, overflow, low_abs, mass_m, mass_l)
    mass_m, mass_l = (state.m, state.l) if keep_mass else (None, None)
    if mode == 'saved':
        return Prediction(state, mode, mass_m=mass_m, mass_l=mass_l)
    return Prediction(state, mode, high, low, low_abs=low_abs, mass_m=mass_m, mass_l=mass_l)


def _prediction_struct(prediction):
    if prediction is None:
        return L.StkPrediction(L.PRED_NONE, 0)
    st, low = prediction.state, prediction.low
    rids = prediction.retained_ids
    return L.StkPrediction(
        L.PRED_MODES[prediction.mode], st.m.shape[1], st.m.data_ptr(), st.l.data_ptr(), st.u.data_ptr(),
        L.ptr(prediction.high), L.ptr(rids), L.id_is64(rids) if rids is not None else 0,
        L.ptr(low.m) if low is not None else None, L.ptr(low.l) if low is not None else None,
        L.ptr(low.u) if low is not None else None, L.ptr(prediction.low_abs), L.ptr(prediction.mass_m),
        L.ptr(prediction.mass_l))


def _run_repair(q, k, v, selected, predicted, prediction, variant, *, min_remaining=1e-3, cancellation_tol=1e-5,
                max_extra_mass=0., want_approx=False, want_jobs=False, max_blocks=None, kv=None, rows_hq=None):
    """One launch of the unified repair kernel; returns the output tensors."""
    h, d = q.shape[0], q.shape[1]
    dev = q.device
    out = torch.empty((h, d), device=dev, dtype=torch.float32)
    fallback = torch.empty((h,), device=dev, dtype=torch.bool)
    remaining = torch.empty((h,), device=dev, dtype=torch.float32)
    approx = torch.empty_like(fallback) if want_approx else None
    extra = torch.empty_like(remaining) if want_approx else None
    pos = torch.empty((h,), device=dev, dtype=torch.int32) if want_jobs else None
    total = torch.empty_like(pos) if want_jobs else None
    if kv is None:
        kv = L.kv_struct(k, v)
    ps = _prediction_struct(prediction)
    ro = L.StkRepairOut(out.data_ptr(), fallback.data_ptr(), remaining.data_ptr(), L.ptr(approx), L.ptr(extra),
                        L.ptr(pos), L.ptr(total))
    sp = predicted.shape[1] if predicted is not None else 0
    rc = L.load().stk_repair(
        C.byref(kv), q.data_ptr(), L.dtype_code(q), h, rows_hq or h, selected.data_ptr(), L.id_is64(selected),
        selected.shape[1], L.ptr(predicted), L.id_is64(predicted) if predicted is not None else 0, sp, C.byref(ps),
        variant, float(min_remaining), float(cancellation_tol), float(max_extra_mass),
        int(max_blocks or k.shape[1]), C.byref(ro), L.status_ptr(), L.stream_of(q))
    L.check(rc, "repair")
    return out, fallback, remaining, approx, extra, pos, total


def repair(q, k, v, selected, predicted, prediction, min_remaining=1.e-3, cancellation_tol=1.e-5):
    """Restore exact selected-set semantics; conservative guards recompute QKV.

    Remaining is the residual low-group denominator over the original one, in
    the merge's common exponent frame (reference kernels.py:504-550). A wholly
    rejected low group is discarded directly without subtraction. Single launch.
    """
    h, n, b, d, sa = _shape(q, k, v, selected)
    _shape(q, k, v, predicted)
    out, fallback, remaining, *_ = _run_repair(q, k, v, selected, predicted, prediction, L.VAR_SPLIT,
                                               min_remaining=min_remaining, cancellation_tol=cancellation_tol)
    return RepairResult(out, fallback, remaining)


def touch_kv(k, v, predicted):
    """Read predicted KV with a checksum side effect; cache residency not assured."""
    hkv, n, b, d = k.shape
    h, s = predicted.shape
    nt = (b * d + 1023) // 1024
    scratch = torch.empty((h, s, nt), device=k.device, dtype=torch.float32)
    kv = L.kv_struct(k, v)
    rc = L.load().stk_touch_kv(C.byref(kv), h, h, predicted.data_ptr(), L.id_is64(predicted), s,
                               scratch.data_ptr(), L.stream_of(k))
    L.check(rc, "touch_kv")
    return scratch
