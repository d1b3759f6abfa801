"""Generate golden fixtures by running the REFERENCE implementation on the CPU.

Run once, in a container that has the reference checkout (read-only), with
``STK_REFERENCE`` naming its directory::

    STK_REFERENCE=<reference checkout> python tests/golden/make_golden.py

The reference is pure Python + Triton. Its kernels execute on the CPU under
Triton's interpreter (``TRITON_INTERPRET=1``); only its CUDA-device shape
assertions are bypassed, and one interpreter quirk (a Python ``bool``
combined with a mask tensor by ``&``) is coerced to NumPy bool arithmetic,
which is what the compiled kernel does with such a mask. The fixtures hold,
per case, the reference outputs and every discrete decision it makes
(fallback, remaining fraction, approximation flags, job counts, the
prediction's high mask / retained IDs / overflow), plus the reference's own
FP64 oracle output. Inputs are NOT stored: they are regenerated from
``cases.py`` and checked against the stored SHA-256.

Nothing at test time imports the reference; the GPU box never sees it.
"""
from __future__ import annotations

import math
import os
import sys
import time
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"
REF = os.environ.get("STK_REFERENCE")
if not REF:
    raise SystemExit("set STK_REFERENCE to the reference checkout's directory")
sys.path.insert(0, REF)
sys.path.insert(0, str(Path(__file__).resolve().parent))

import numpy as np  # noqa: E402
import torch  # noqa: E402
from triton.runtime import interpreter as _ti  # noqa: E402

import cases as C  # noqa: E402


def _bitop(op):
    def f(self, lhs, rhs):
        l, r = lhs.data, rhs.data
        if l.dtype == np.bool_ and r.dtype != np.bool_:
            r = r != 0
        if r.dtype == np.bool_ and l.dtype != np.bool_:
            l = l != 0
        return _ti.TensorHandle(op(l, r), lhs.dtype.scalar)
    return f


_ti.InterpreterBuilder.create_and = _bitop(np.bitwise_and)
_ti.InterpreterBuilder.create_or = _bitop(np.bitwise_or)

from strict_topk import (fused, gqa, gqa_hierarchical, gqa_light, kernels,  # noqa: E402
                         selector, signed_fused, signed_repair)


def _shape_cpu(q, k, v, ids):
    assert q.ndim == 2 and k.ndim == 4 and v.shape == k.shape
    h, n, b, d = k.shape
    assert q.shape == (h, d) and ids.ndim == 2 and ids.shape[0] == h
    return h, n, b, d, ids.shape[1]


def _gqa_shape_cpu(q, k, v, ids):
    hkv, n, b, d = k.shape
    hq = q.shape[0]
    return hq, n, b, d, hq // hkv, ids.shape[1]


for mod in (kernels, fused, signed_repair, signed_fused):
    mod._shape = _shape_cpu
gqa._shape = _gqa_shape_cpu


def ref_fp64(q, k, v, ids, include=None):
    """tests/check_correctness.py:12-17 and benchmarks/critical_path.py:16-25."""
    group = q.shape[0] // k.shape[0]
    kvh = torch.arange(q.shape[0])[:, None] // group
    ks, vs = k[kvh, ids.long()].double(), v[kvh, ids.long()].double()
    logits = torch.einsum("hd,hkbd->hkb", q.double(), ks) / math.sqrt(q.shape[-1])
    if include is not None:
        logits = logits.masked_fill(~include[:, :, None], -torch.inf)
    w = logits.flatten(1).softmax(-1).view_as(logits)
    return torch.einsum("hkb,hkbd->hd", w, vs)


def block_scores_ref(q, lo, hi):
    """selector.block_scores without its CUDA-device check (selector.py:23-38)."""
    import triton
    h, n, d = lo.shape
    scores = torch.empty((h, n), dtype=torch.float32)
    dd = triton.next_power_of_2(d)
    nn = max(1, min(32, 2048 // dd))
    selector._score[(h, triton.cdiv(n, nn))](q, lo, hi, scores, n, d, nn, dd, num_warps=4)
    return scores


def bound_scores_fp64(q, lo, hi):
    """FP64 bound score, as in tests/check_selector.py:14-15 / check_gqa.py:50-51."""
    group = q.shape[0] // lo.shape[0]
    kvh = torch.arange(q.shape[0]) // group
    qd = q.double()[:, None, :]
    return (torch.where(qd >= 0, hi[kvh].double(), lo[kvh].double()) * qd).sum(-1)


def stable_topk(scores, k):
    """Descending score, ties to the lower block index; returned ascending by ID."""
    order = np.lexsort((np.arange(scores.shape[1])[None, :].repeat(scores.shape[0], 0),
                        -scores), axis=1)
    return np.sort(order[:, :k], axis=1).astype(np.int32)


class Sink:
    def __init__(self):
        self.data = {}

    def put(self, key, value):
        if value is None:
            return
        if isinstance(value, torch.Tensor):
            value = value.detach()
            if value.dtype == torch.bfloat16 or value.dtype == torch.float16:
                value = value.float()
            value = value.numpy()
        self.data[key] = np.asarray(value)

    def save(self, path):
        np.savez_compressed(path, **self.data)
        print(f"wrote {path} ({len(self.data)} arrays, {Path(path).stat().st_size} bytes)", flush=True)


def _put_prediction(sink, key, pred):
    sink.put(f"{key}/state_m", pred.state.m)
    sink.put(f"{key}/state_l", pred.state.l)
    sink.put(f"{key}/state_u", pred.state.u)
    sink.put(f"{key}/high", pred.high)
    if pred.low is not None:
        sink.put(f"{key}/low_m", pred.low.m)
        sink.put(f"{key}/low_l", pred.low.l)
        sink.put(f"{key}/low_u", pred.low.u)
    sink.put(f"{key}/low_abs", pred.low_abs)
    sink.put(f"{key}/retained_ids", pred.retained_ids)
    sink.put(f"{key}/overflow", pred.overflow)


def _put_result(sink, key, res):
    sink.put(f"{key}/output", res.output)
    sink.put(f"{key}/fallback", res.fallback)
    sink.put(f"{key}/remaining", res.remaining)
    sink.put(f"{key}/approx", getattr(res, "approximate_heads", None))
    sink.put(f"{key}/extra", getattr(res, "extra_mass_bound", None))
    sink.put(f"{key}/pos", getattr(res, "positive_jobs", None))
    sink.put(f"{key}/total", getattr(res, "total_jobs", None))


MODES = [("saved", 0.1), ("hybrid", 0.05), ("hybrid", 0.2), ("hybrid", 1.0),
         ("compact", 0.05), ("compact", 0.2), ("compact", 1.0)]
EPS = 0.01


def run_expanded(sink, name, q, k, v, p, a):
    """All expanded-layout speculate/repair variants for one case."""
    sink.put(f"{name}/sha256", np.array(C.digest(q, k, v, p, a)))
    sink.put(f"{name}/fp64", ref_fp64(q, k, v, a))
    sink.put(f"{name}/exact/output", kernels.exact_attention(q, k, v, a))
    for mode, tau in MODES:
        key = f"{name}/{mode}_{tau:g}"
        pred = kernels.speculate(q, k, v, p, mode=mode, mass_threshold=tau)
        _put_prediction(sink, f"{key}/pred", pred)
        _put_result(sink, f"{key}/split", kernels.repair(q, k, v, a, p, pred))
        _put_result(sink, f"{key}/fused", fused.repair_fused(q, k, v, a, p, pred))
        _put_result(sink, f"{key}/signed", signed_repair.repair_signed(q, k, v, a, p, pred))
        _put_result(sink, f"{key}/signed_fused", signed_fused.repair_signed_fused(q, k, v, a, p, pred))
        pk = kernels.speculate(q, k, v, p, mode=mode, mass_threshold=tau, keep_mass=True)
        sink.put(f"{key}/pred/mass_m", pk.mass_m)
        sink.put(f"{key}/pred/mass_l", pk.mass_l)
        _put_result(sink, f"{key}/fused_eps", fused.repair_fused(q, k, v, a, p, pk, max_extra_mass=EPS))
        _put_result(sink, f"{key}/signed_eps",
                    signed_repair.repair_signed(q, k, v, a, p, pk, max_extra_mass=EPS))
        _put_result(sink, f"{key}/signed_fused_eps",
                    signed_fused.repair_signed_fused(q, k, v, a, p, pk, max_extra_mass=EPS))


def make_correctness(out_dir):
    for dtype, tag in [(torch.float16, "fp16"), (torch.bfloat16, "bf16")]:
        sink = Sink()
        names = []
        for name, q, k, v, p, a in C.correctness_cases(dtype):
            t = time.time()
            run_expanded(sink, name, q, k, v, p, a)
            names.append(name)
            print(f"  {tag} {name}: {time.time() - t:.1f}s", flush=True)
        sink.put("cases", np.array(names))
        sink.save(out_dir / f"correctness_{tag}.npz")


def run_gqa_case(sink, name, q, k, v, p, a):
    sink.put(f"{name}/sha256", np.array(C.digest(q, k, v, p, a)))
    sink.put(f"{name}/fp64", ref_fp64(q, k, v, a))
    hit = (a[:, :, None] == p[:, None, :]).any(-1)
    union = torch.cat((p.long(), a.long()), 1)
    inc = torch.cat((torch.ones_like(p, dtype=torch.bool), ~hit), 1)
    sink.put(f"{name}/fp64_union", ref_fp64(q, k, v, union, inc))
    state = gqa.partials(q, k, v, p)
    sink.put(f"{name}/partials_m", state.m)
    sink.put(f"{name}/partials_l", state.l)
    sink.put(f"{name}/partials_u", state.u)
    sink.put(f"{name}/exact", gqa.exact(q, k, v, a))
    sink.put(f"{name}/repair_saved", gqa.repair_saved(q, k, v, a, p, state))
    sink.put(f"{name}/repair_union", gqa.repair_union(q, k, v, a, p, state))
    sink.put(f"{name}/light", gqa_light.repair_saved_light(q, k, v, a, p, state))


def make_gqa(out_dir):
    sink = Sink()
    names = []
    for name, q, k, v, p, a in C.gqa_cases() + C.gqa_light_cases():
        run_gqa_case(sink, name, q, k, v, p, a)
        names.append(name)
        print(f"  gqa {name}", flush=True)
    sink.put("cases", np.array(names))
    # Tied GQA selection (tests/check_gqa.py:46-54).
    q, lo, hi, k = C.gqa_selector_case()
    s64 = bound_scores_fp64(q, lo, hi).numpy()
    sink.put("gqa_select/sha256", np.array(C.digest(q, lo, hi)))
    sink.put("gqa_select/scores_fp64", s64)
    sink.put("gqa_select/ids_stable", stable_topk(s64, k))
    # Per-head selector (tests/check_selector.py:8-27).
    q, lo, hi, ks = C.selector_case()
    s64 = bound_scores_fp64(q, lo, hi).numpy()
    sink.put("select/sha256", np.array(C.digest(q, lo, hi)))
    sink.put("select/scores_fp64", s64)
    sink.put("select/scores_ref_fp32", block_scores_ref(q, lo, hi))
    for k in ks:
        sink.put(f"select/ids_stable_k{k}", stable_topk(s64, k))
    sink.save(out_dir / "gqa.npz")


def make_hierarchical(out_dir):
    for dtype, tag in [(torch.float16, "fp16"), (torch.bfloat16, "bf16")]:
        sink = Sink()
        names = []
        for name, q, k, v, p, a, shared in C.hierarchical_cases(dtype):
            t = time.time()
            sink.put(f"{name}/sha256", np.array(C.digest(q, k, v, p, a)))
            sink.put(f"{name}/fp64", ref_fp64(q, k, v, a))
            if "hit0" in name and not shared:
                sink.put(f"{name}/exact", gqa_hierarchical.exact(q, k, v, a))
            state = gqa_hierarchical.partials(q, k, v, p)
            fn = gqa_hierarchical.repair_saved_shared if shared else gqa_hierarchical.repair_saved
            sink.put(f"{name}/repair", fn(q, k, v, a, p, state))
            names.append(name)
            print(f"  hier {tag} {name}: {time.time() - t:.1f}s", flush=True)
        sink.put("cases", np.array(names))
        sink.save(out_dir / f"hierarchical_{tag}.npz")


def make_kats(out_dir):
    sink = Sink()
    q, k, v, p, a, extra_set = C.budget_case()
    sink.put("budget/sha256", np.array(C.digest(q, k, v, p, a)))
    sink.put("budget/strict_fp64", ref_fp64(q, k, v, a))
    sink.put("budget/extra_fp64", ref_fp64(q, k, v, extra_set))
    sink.put("budget/extra_mass",
             np.array(k[0, extra_set[0].long(), 0, 0].double().softmax(dim=0)[-1].item()))
    for mode in ("hybrid", "compact"):
        state = kernels.speculate(q, k, v, p, mode=mode, mass_threshold=.2, keep_mass=True)
        for impl_name, impl in [("signed", signed_repair.repair_signed),
                                ("signed_fused", signed_fused.repair_signed_fused)]:
            _put_result(sink, f"budget/{mode}/{impl_name}/low", impl(q, k, v, a, p, state, max_extra_mass=.01))
            _put_result(sink, f"budget/{mode}/{impl_name}/high", impl(q, k, v, a, p, state, max_extra_mass=.1))
            _put_result(sink, f"budget/{mode}/{impl_name}/forced",
                        impl(q, k, v, a, p, state, cancellation_tol=2., max_extra_mass=.1))
        for eps in (.01, .1):
            _put_result(sink, f"budget/{mode}/fused/eps{eps:g}",
                        fused.repair_fused(q, k, v, a, p, state, max_extra_mass=eps))
        _put_result(sink, f"budget/{mode}/fused/forced",
                    fused.repair_fused(q, k, v, a, p, state, cancellation_tol=2., max_extra_mass=.1))
    q, k, v, p, a = C.underflow_case()
    sink.put("underflow/sha256", np.array(C.digest(q, k, v, p, a)))
    sink.put("underflow/fp64", ref_fp64(q, k, v, a))
    pred = kernels.speculate(q, k, v, p, mode="hybrid", mass_threshold=1.)
    _put_result(sink, "underflow/signed_fused", signed_fused.repair_signed_fused(q, k, v, a, p, pred))
    sink.save(out_dir / "kats.npz")


def make_config0(out_dir):
    """BASELINE config 0 through the reference torch/FP64 path and its kernels."""
    sink = Sink()
    q, k, v, lo, hi, topk, nswap = C.baseline_config0()
    s64 = bound_scores_fp64(q, lo, hi).numpy()
    a = torch.from_numpy(stable_topk(s64, topk))
    p = C.swap_prediction(a, k.shape[1], nswap, seed=0)
    sink.put("c0/sha256", np.array(C.digest(q, k, v, lo, hi)))
    sink.put("c0/scores_fp64", s64)
    sink.put("c0/selected", a)
    sink.put("c0/predicted", p)
    sink.put("c0/fp64", ref_fp64(q, k, v, a))
    state = gqa.partials(q, k, v, p)
    sink.put("c0/gqa_repair_saved", gqa.repair_saved(q, k, v, a, p, state))
    sink.put("c0/gqa_light", gqa_light.repair_saved_light(q, k, v, a, p, state))
    sink.put("c0/gqa_exact", gqa.exact(q, k, v, a))
    # Expanded-KV methods (the reference's kernels.py family needs K/V[Hq,...]).
    g = q.shape[0] // k.shape[0]
    ke, ve = k.repeat_interleave(g, 0).contiguous(), v.repeat_interleave(g, 0).contiguous()
    for mode, tau in [("saved", 0.1), ("hybrid", 0.1), ("compact", 0.1)]:
        pred = kernels.speculate(q, ke, ve, p, mode=mode, mass_threshold=tau, keep_mass=True)
        _put_result(sink, f"c0/{mode}/split", kernels.repair(q, ke, ve, a, p, pred))
        _put_result(sink, f"c0/{mode}/fused", fused.repair_fused(q, ke, ve, a, p, pred))
        _put_result(sink, f"c0/{mode}/signed_fused",
                    signed_fused.repair_signed_fused(q, ke, ve, a, p, pred))
        _put_result(sink, f"c0/{mode}/signed_fused_eps",
                    signed_fused.repair_signed_fused(q, ke, ve, a, p, pred, max_extra_mass=EPS))
    sink.save(out_dir / "config0.npz")


def main():
    out_dir = Path(__file__).resolve().parent
    which = sys.argv[1:] or ["kats", "config0", "gqa", "correctness", "hierarchical"]
    for w in which:
        t = time.time()
        globals()[f"make_{w}"](out_dir)
        print(f"{w}: {time.time() - t:.1f}s", flush=True)


if __name__ == "__main__":
    main()
