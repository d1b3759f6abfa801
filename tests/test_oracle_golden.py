"""Pin the CPU oracle to the reference: every oracle function is checked
against golden fixtures that the reference implementation itself produced
(tests/golden/make_golden.py). No GPU needed."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import cases as C
from golden_io import MODES, VARIANTS, field, load, ref_tol_ok
from oracle import attention as OA
from oracle import selection as OS
from oracle import speculative as OP

DECISIONS = ("fallback", "approx", "pos", "total")


def _np(t):
    return C.as_np(t)


def _check_result(fx, key, got, fp64, exp_tol=1e-4):
    ref_out = fx[f"{key}/output"]
    assert np.allclose(got["output"], ref_out, atol=exp_tol, rtol=exp_tol), key
    assert ref_tol_ok(got["output"], fp64) or ref_tol_ok(ref_out, fp64) is False, key
    for name in DECISIONS:
        ref = field(fx, f"{key}/{name}")
        if ref is None:
            continue
        assert np.array_equal(np.asarray(got[name]).astype(ref.dtype), ref), (key, name, got[name], ref)
    rem = fx[f"{key}/remaining"]
    assert np.allclose(np.asarray(got["remaining"], np.float32), rem, rtol=1e-4, atol=1e-6, equal_nan=True), key
    ext = field(fx, f"{key}/extra")
    if ext is not None:
        assert np.allclose(np.asarray(got["extra"], np.float32), ext, rtol=1e-4, atol=1e-7), key


@pytest.mark.parametrize("dtype,tag", [(torch.float16, "fp16"), (torch.bfloat16, "bf16")])
def test_correctness_cases(dtype, tag):
    fx = load(f"correctness_{tag}")
    for name, q, k, v, p, a in C.correctness_cases(dtype):
        assert str(fx[f"{name}/sha256"]) == C.digest(q, k, v, p, a), f"input drift in {name}"
        qn, kn, vn, pn, an = _np(q), _np(k), _np(v), p.numpy(), a.numpy()
        fp64 = fx[f"{name}/fp64"]
        assert np.allclose(OA.attention_fp64(qn, kn, vn, an), fp64, atol=1e-12, rtol=1e-10)
        for mode, tau in MODES:
            key = f"{name}/{mode}_{tau:g}"
            pred = OP.speculate(qn, kn, vn, pn, mode, tau, keep_mass=True)
            for f_ in ("high", "overflow", "retained_ids"):
                ref = field(fx, f"{key}/pred/{f_}")
                if ref is not None:
                    assert np.array_equal(pred[f_].astype(ref.dtype), ref), (key, f_)
            assert np.allclose(pred["m"], fx[f"{key}/pred/state_m"], atol=1e-5, rtol=1e-5), key
            assert np.allclose(pred["l"], fx[f"{key}/pred/state_l"], atol=1e-5, rtol=1e-5), key
            for label, variant, eps in VARIANTS:
                got = OP.repair(variant, qn, kn, vn, an, pn, pred, max_extra_mass=eps)
                _check_result(fx, f"{key}/{label}", got, fp64)


def test_budget_kats():
    fx = load("kats")
    q, k, v, p, a, extra_set = C.budget_case()
    assert str(fx["budget/sha256"]) == C.digest(q, k, v, p, a)
    qn, kn, vn, pn, an = _np(q), _np(k), _np(v), p.numpy(), a.numpy()
    strict = fx["budget/strict_fp64"]
    with_extra = fx["budget/extra_fp64"]
    extra_mass = float(fx["budget/extra_mass"])
    assert np.allclose(OA.attention_fp64(qn, kn, vn, an), strict)
    for mode in ("hybrid", "compact"):
        pred = OP.speculate(qn, kn, vn, pn, mode, .2, keep_mass=True)
        for impl in ("signed", "signed_fused"):
            low = OP.repair(impl, qn, kn, vn, an, pn, pred, max_extra_mass=.01)
            high = OP.repair(impl, qn, kn, vn, an, pn, pred, max_extra_mass=.1)
            forced = OP.repair(impl, qn, kn, vn, an, pn, pred, cancellation_tol=2., max_extra_mass=.1)
            # tests/check_signed_repair.py:41-56 known answers
            assert not low["approx"][0] and low["extra"][0] == 0. and low["pos"][0] == 1 and low["total"][0] == 2
            assert ref_tol_ok(low["output"], strict)
            assert high["approx"][0] and extra_mass <= high["extra"][0] <= .1
            assert high["pos"][0] == 1 and high["total"][0] == 1 and ref_tol_ok(high["output"], with_extra)
            assert forced["fallback"][0] and not forced["approx"][0] and forced["extra"][0] == 0.
            assert ref_tol_ok(forced["output"], strict)
            for label, got in (("low", low), ("high", high), ("forced", forced)):
                _check_result(fx, f"budget/{mode}/{impl}/{label}", got, strict if label != "high" else with_extra)
        for eps in (.01, .1):
            got = OP.repair("fused", qn, kn, vn, an, pn, pred, max_extra_mass=eps)
            _check_result(fx, f"budget/{mode}/fused/eps{eps:g}", got, strict if eps == .01 else with_extra)
        got = OP.repair("fused", qn, kn, vn, an, pn, pred, cancellation_tol=2., max_extra_mass=.1)
        _check_result(fx, f"budget/{mode}/fused/forced", got, strict)


def test_underflow_regression():
    """tests/check_signed_fused.py:17-30: hybrid erasure must reproduce the
    preparation's underflow order; the reference falls back (fallback True)."""
    fx = load("kats")
    q, k, v, p, a = C.underflow_case()
    assert str(fx["underflow/sha256"]) == C.digest(q, k, v, p, a)
    qn, kn, vn, pn, an = _np(q), _np(k), _np(v), p.numpy(), a.numpy()
    pred = OP.speculate(qn, kn, vn, pn, "hybrid", 1.)
    got = OP.repair("signed_fused", qn, kn, vn, an, pn, pred)
    assert got["fallback"][0]
    assert ref_tol_ok(got["output"], fx["underflow/fp64"])
    _check_result(fx, "underflow/signed_fused", got, fx["underflow/fp64"])


def test_config0_selection_and_methods():
    fx = load("config0")
    q, k, v, lo, hi, topk, nswap = C.baseline_config0()
    assert str(fx["c0/sha256"]) == C.digest(q, k, v, lo, hi)
    qn, kn, vn = _np(q), _np(k), _np(v)
    s = OS.bound_scores_fp64(qn, lo.numpy(), hi.numpy())
    assert np.allclose(s, fx["c0/scores_fp64"], rtol=1e-13, atol=1e-12)
    a = OS.select_blocks(qn, lo.numpy(), hi.numpy(), topk)
    assert np.array_equal(a, fx["c0/selected"])
    p = C.swap_prediction(torch.from_numpy(a), k.shape[1], nswap, seed=0).numpy()
    assert np.array_equal(p, fx["c0/predicted"])
    fp64 = fx["c0/fp64"]
    assert np.allclose(OA.attention_fp64(qn, kn, vn, a), fp64, atol=1e-12)
    pred = OP.speculate(qn, kn, vn, p, "saved")
    got = OP.repair("saved", qn, kn, vn, a, p, pred)["output"]
    assert np.allclose(got, fx["c0/gqa_repair_saved"], atol=1e-5) and ref_tol_ok(got, fp64, 1e-5, 1e-5)
    for mode in ("saved", "hybrid", "compact"):
        pred = OP.speculate(qn, kn, vn, p, mode, 0.1, keep_mass=True)
        for label, variant, eps in (("split", "split", 0.), ("fused", "fused", 0.),
                                    ("signed_fused", "signed_fused", 0.), ("signed_fused_eps", "signed_fused", .01)):
            got = OP.repair(variant, qn, kn, vn, a, p, pred, max_extra_mass=eps)
            _check_result(fx, f"c0/{mode}/{label}", got, fp64, exp_tol=1e-5)


def test_gqa_cases():
    fx = load("gqa")
    for name, q, k, v, p, a in C.gqa_cases() + C.gqa_light_cases():
        assert str(fx[f"{name}/sha256"]) == C.digest(q, k, v, p, a), name
        qn, kn, vn, pn, an = _np(q), _np(k), _np(v), p.numpy(), a.numpy()
        fp64 = fx[f"{name}/fp64"]
        assert np.allclose(OA.attention_fp64(qn, kn, vn, an), fp64, atol=1e-10)
        pred = OP.speculate(qn, kn, vn, pn, "saved")
        assert np.allclose(pred["m"], fx[f"{name}/partials_m"], atol=1e-5, rtol=1e-5)
        saved = OP.repair("saved", qn, kn, vn, an, pn, pred)["output"]
        union = OP.repair("union", qn, kn, vn, an, pn, pred)["output"]
        for ref_key in ("repair_saved", "light", "exact"):
            assert np.allclose(saved, fx[f"{name}/{ref_key}"], atol=1e-4, rtol=1e-4), (name, ref_key)
        assert np.allclose(union, fx[f"{name}/repair_union"], atol=1e-4, rtol=1e-4), name
        assert ref_tol_ok(saved, fp64) and ref_tol_ok(union, fx[f"{name}/fp64_union"])
        u_ids = OA.union_ids(an, pn)
        assert np.allclose(OA.attention_fp64(qn, kn, vn, u_ids), fx[f"{name}/fp64_union"], atol=1e-10)


def test_selector_scores_and_ties():
    fx = load("gqa")
    q, lo, hi, ks = C.selector_case()
    assert str(fx["select/sha256"]) == C.digest(q, lo, hi)
    s = OS.bound_scores_fp64(_np(q), lo.numpy(), hi.numpy())
    assert np.allclose(s, fx["select/scores_fp64"], rtol=1e-13, atol=1e-13)
    # The reference's FP32 kernel agrees with FP64 within its own tolerance.
    assert np.allclose(fx["select/scores_ref_fp32"], s, atol=2e-5, rtol=2e-6)
    for k in ks:
        ids = OS.select_blocks(_np(q), lo.numpy(), hi.numpy(), k)
        assert np.array_equal(ids, fx[f"select/ids_stable_k{k}"])
        assert (np.diff(ids, axis=1) > 0).all()
    # Row 0 has q == 0: every score ties at 0 and the lowest IDs win.
    assert np.array_equal(OS.select_blocks(_np(q), lo.numpy(), hi.numpy(), 11)[0], np.arange(11))
    q, lo, hi, k = C.gqa_selector_case()
    assert str(fx["gqa_select/sha256"]) == C.digest(q, lo, hi)
    ids = OS.select_blocks(_np(q), lo.numpy(), hi.numpy(), k)
    assert np.array_equal(ids, fx["gqa_select/ids_stable"])


@pytest.mark.parametrize("tag,dtype", [("fp16", torch.float16), ("bf16", torch.bfloat16)])
def test_hierarchical_cases(tag, dtype):
    try:
        fx = load(f"hierarchical_{tag}")
    except FileNotFoundError:
        pytest.skip("fixture not generated")
    for name, q, k, v, p, a, shared in C.hierarchical_cases(dtype, large=False):
        assert str(fx[f"{name}/sha256"]) == C.digest(q, k, v, p, a), name
        qn, kn, vn, pn, an = _np(q), _np(k), _np(v), p.numpy(), a.numpy()
        pred = OP.speculate(qn, kn, vn, pn, "saved")
        got = OP.repair("saved", qn, kn, vn, an, pn, pred)["output"]
        assert np.allclose(got, fx[f"{name}/repair"], atol=1e-4, rtol=1e-4), name
        assert ref_tol_ok(got, fx[f"{name}/fp64"]), name


def test_shard_select_equals_global():
    """Context-parallel selection merges shard candidates into the global Top-K."""
    q, k, v, lo, hi = C.synthetic_kv(8, 2, 256, 8, 64, torch.bfloat16, seed=3)
    qn = _np(q)
    full = OS.select_blocks(qn, lo.numpy(), hi.numpy(), 24)
    for shards in (2, 4, 8):
        assert np.array_equal(OS.shard_select(qn, lo.numpy(), hi.numpy(), 24, shards), full)
