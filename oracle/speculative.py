"""FP32 restatement of the reference's speculation and repair algorithms.

Each function follows the cited reference kernel line by line in FP32
(NumPy float32), per head, so the discrete decisions — high masks, compact
packing and overflow, fallback, remaining fraction, approximation flag,
extra-mass bound, positive / total job counts — reproduce the reference's on
the golden cases. Outputs are FP32 and agree with the FP64 oracle within the
reference's tolerance. Summation orders inside a block differ from Triton's;
decisions that sit exactly on a threshold may therefore differ, which the
golden cases avoid (as the reference's own tests do).

Reference files (paths within 6Mikao9/strict-topk-overlap):
  strict_topk/kernels.py         speculate / repair (split)
  strict_topk/fused.py           repair_fused
  strict_topk/signed_repair.py   repair_signed (+ _schedule)
  strict_topk/signed_fused.py    repair_signed_fused
  strict_topk/gqa.py, gqa_light.py, gqa_hierarchical.py   saved / union repair
"""
from __future__ import annotations

import numpy as np

F = np.float32
NEG_INF = F(-np.inf)


def _f(x):
    return np.asarray(x, dtype=np.float32)


def _exp(x):
    with np.errstate(over="ignore", under="ignore", invalid="ignore"):
        return np.exp(_f(x)).astype(np.float32)


class Inputs:
    """q [H, D], k/v [Hkv, N, B, D] widened to FP32; query head h reads KV head h // g."""

    def __init__(self, q, k, v):
        self.q = _f(q)
        self.k = _f(k)
        self.v = _f(v)
        self.h, self.d = self.q.shape
        self.g = self.h // self.k.shape[0]
        self.scale = F(self.d ** -0.5)

    def logits(self, h, bid):
        kb = self.k[h // self.g, int(bid)]
        return ((kb @ self.q[h]).astype(np.float32) * self.scale).astype(np.float32)

    def values(self, h, bid):
        return self.v[h // self.g, int(bid)]


def block_state(X, h, bid):
    """kernels.py:42-71 (_partial): (m, l, u) of one block."""
    s = X.logits(h, bid)
    m = F(s.max())
    w = _exp(s - m)
    return m, F(w.sum(dtype=np.float32)), (w[:, None] * X.values(h, bid)).sum(0, dtype=np.float32)


def fixed_frame_sums(X, h, bids, frame, with_abs=False):
    """Per-token weights exp(s - frame) summed over blocks in order
    (kernels.py:324-334 compact low aggregate, :384-407 _wrong_aggregate,
    fused.py:22-44 FIXED_M accumulation)."""
    z = F(0.)
    u = np.zeros(X.d, dtype=np.float32)
    a = np.zeros(X.d, dtype=np.float32)
    for bid in bids:
        w = _exp(X.logits(h, bid) - F(frame))
        wv = w[:, None] * X.values(h, bid)
        z = F(z + w.sum(dtype=np.float32))
        u = (u + wv.sum(0, dtype=np.float32)).astype(np.float32)
        if with_abs:
            a = (a + np.abs(wv).sum(0, dtype=np.float32)).astype(np.float32)
    return z, u, a


def online(X, h, bids, m=NEG_INF, z=F(0.), u=None):
    """Online softmax over blocks in order (kernels.py:223-247, fused.py:22-44)."""
    u = np.zeros(X.d, dtype=np.float32) if u is None else _f(u).copy()
    m, z = F(m), F(z)
    for bid in bids:
        s = X.logits(h, bid)
        nm = F(max(m, s.max()))
        al = _exp(m - nm)
        w = _exp(s - nm)
        u = (u * al + (w[:, None] * X.values(h, bid)).sum(0, dtype=np.float32)).astype(np.float32)
        z = F(z * al + w.sum(dtype=np.float32))
        m = nm
    return m, z, u


def compact_capacity(s, tau):
    """kernels.py:485."""
    return s if tau <= 1 / s else min(s, int(1 / tau) + 1)


# --------------------------------------------------------------------------- speculate

def speculate(q, k, v, predicted, mode="saved", tau=0.1, keep_mass=False):
    """kernels.py:450-501. Returns a dict of FP32/bool/int arrays."""
    X = Inputs(q, k, v)
    P = np.asarray(predicted).astype(np.int64)
    h, s = P.shape
    d = X.d
    T = F(tau)
    out = {"mode": mode}
    if mode in ("saved", "hybrid"):
        M = np.empty((h, s), np.float32)
        Lm = np.empty((h, s), np.float32)
        U = np.empty((h, s, d), np.float32)
        for i in range(h):
            for j in range(s):
                M[i, j], Lm[i, j], U[i, j] = block_state(X, i, P[i, j])
        out.update(m=M, l=Lm, u=U, sc=s)
        if keep_mass:
            out.update(mass_m=M, mass_l=Lm)
        if mode == "hybrid":  # _group, kernels.py:94-117
            high = np.zeros((h, s), bool)
            LM = np.zeros(h, np.float32)
            LL = np.zeros(h, np.float32)
            LU = np.zeros((h, d), np.float32)
            LA = np.zeros((h, d), np.float32)
            for i in range(h):
                gm = M[i].max()
                mass = _exp(M[i] - gm) * Lm[i]
                total = F(mass.sum(dtype=np.float32))
                hi = mass >= T * total
                high[i] = hi
                low = ~hi
                lm = M[i][low].max() if low.any() else NEG_INF
                lm = F(0.) if lm == NEG_INF else F(lm)
                alpha = np.where(low, _exp(M[i] - lm), F(0.)).astype(np.float32)
                LM[i] = lm
                LL[i] = (alpha * Lm[i]).sum(dtype=np.float32)
                LU[i] = (alpha[:, None] * U[i]).sum(0, dtype=np.float32)
                LA[i] = (alpha[:, None] * np.abs(U[i])).sum(0, dtype=np.float32)
            out.update(high=high, low_m=LM, low_l=LL, low_u=LU, low_abs=LA)
        return out
    if mode != "compact":
        raise ValueError(mode)
    c = compact_capacity(s, tau)
    pm = np.empty((h, s), np.float32)
    pl = np.empty((h, s), np.float32)
    for i in range(h):
        for j in range(s):
            sc = X.logits(i, P[i, j])
            pm[i, j] = sc.max()
            pl[i, j] = _exp(sc - pm[i, j]).sum(dtype=np.float32)
    high = np.zeros((h, s), bool)
    rids = np.full((h, c), -1, np.int64)
    overflow = np.zeros(h, bool)
    LM = np.zeros(h, np.float32)
    LL = np.zeros(h, np.float32)
    for i in range(h):  # _compact_group, kernels.py:281-309
        mass = _exp(pm[i] - pm[i].max()) * pl[i]
        hi = mass >= T * F(mass.sum(dtype=np.float32))
        rank = np.cumsum(hi)
        count = int(hi.sum())
        overflow[i] = count > c
        hi = hi & (rank <= c)
        high[i] = hi
        for cc in range(min(count, c)):
            rids[i, cc] = P[i][np.nonzero(hi & (rank == cc + 1))[0][0]]
        low = ~hi
        lm = pm[i][low].max() if low.any() else NEG_INF
        lm = F(0.) if lm == NEG_INF else F(lm)
        LM[i] = lm
        LL[i] = np.where(low, _exp(pm[i] - lm) * pl[i], F(0.)).sum(dtype=np.float32)
    M = np.full((h, c), NEG_INF, np.float32)
    Lc = np.zeros((h, c), np.float32)
    U = np.zeros((h, c, d), np.float32)
    LU = np.zeros((h, d), np.float32)
    LA = np.zeros((h, d), np.float32)
    for i in range(h):  # _compact_values, kernels.py:312-356
        _, LU[i], LA[i] = fixed_frame_sums(X, i, [P[i, j] for j in range(s) if not high[i, j]], LM[i], True)
        for cc in range(c):
            if rids[i, cc] >= 0:
                M[i, cc], Lc[i, cc], U[i, cc] = block_state(X, i, rids[i, cc])
    out.update(m=M, l=Lc, u=U, sc=c, high=high, retained_ids=rids, overflow=overflow, low_m=LM, low_l=LL,
               low_u=LU, low_abs=LA)
    if keep_mass:
        out.update(mass_m=pm, mass_l=pl)
    return out


# --------------------------------------------------------------------------- repair

def _membership(A, P):
    hit = np.isin(P, A)
    miss = ~np.isin(A, P)
    return hit, miss


def _keep(pred, i, A, hit, high):
    """Retained states that enter the merge (fused.py:82-89, signed_repair.py:47-55)."""
    if pred["mode"] == "compact":
        r = pred["retained_ids"][i]
        return (r >= 0) & np.isin(r, A)
    if pred["mode"] == "hybrid":
        return hit & high
    return hit


def _eps_decision(pred, i, keep, wrong, lm, eps):
    """fused.py:104-112 / signed_repair.py:60-73."""
    pm = np.where(keep, pred["m"][i], NEG_INF)
    pl = np.where(keep, pred["l"][i], F(0.))
    ref = F(max(pm.max() if pm.size else NEG_INF, lm))
    wm = np.where(wrong, pred["mass_m"][i], NEG_INF)
    wl = np.where(wrong, pred["mass_l"][i], F(0.))
    wrong_mass = (_exp(wm - ref) * wl).sum(dtype=np.float32)
    denom = F(_exp(lm - ref) * pred["low_l"][i]) + (_exp(pm - ref) * pl).sum(dtype=np.float32)
    extra = F(wrong_mass / denom)
    return bool(extra <= F(eps)), extra


def _guard_margin(fraction=None, mn=None, residual=None, scale=None, tol=None, extra=None, eps=None):
    """How close a row's guard inputs sit to their thresholds: the smallest of
    |fraction - min_remaining|, min over dims with scale > 0 of
    | |residual| - tol * scale | / scale, and |extra - eps| / eps (each only
    where the guard was evaluated); inf when no guard applies. Summation
    orders differ between this restatement and any kernel, so a decision
    whose margin is within a few FP32 roundings may legitimately differ."""
    m = np.inf
    if fraction is not None and np.isfinite(fraction):
        m = min(m, abs(float(fraction) - float(mn)))
    if residual is not None:
        sc = np.asarray(scale, np.float64)
        pos = sc > 0
        if pos.any():
            r = np.abs(np.asarray(residual, np.float64)[pos])
            m = min(m, float((np.abs(r - float(tol) * sc[pos]) / sc[pos]).min()))
    if extra is not None and eps is not None and eps > 0:
        m = min(m, abs(float(extra) - float(eps)) / float(eps))
    return m


def repair(variant, q, k, v, selected, predicted, pred, min_remaining=1e-3, cancellation_tol=1e-5,
           max_extra_mass=0.):
    """Dispatch to one variant: 'split' | 'fused' | 'signed' | 'signed_fused' | 'saved' | 'union'."""
    X = Inputs(q, k, v)
    A = np.asarray(selected).astype(np.int64)
    P = np.asarray(predicted).astype(np.int64)
    fn = {"split": _repair_split, "fused": _repair_fused, "signed": _repair_signed,
          "signed_fused": _repair_signed, "saved": _repair_saved, "union": _repair_saved}[variant]
    res = {k_: [] for k_ in ("output", "fallback", "remaining", "approx", "extra", "pos", "total", "margin")}
    for i in range(X.h):
        r = fn(X, i, A[i], P[i], pred, F(min_remaining), F(cancellation_tol), F(max_extra_mass), variant)
        for k_ in res:
            res[k_].append(r.get(k_, np.inf if k_ == "margin" else 0))
    out = {k_: np.array(v_) for k_, v_ in res.items()}
    out["output"] = out["output"].astype(np.float32)
    return out


def _merge_states(states):
    """LSE merge of (m, l, u) states (kernels.py:74-91 without the include mask)."""
    ms = np.array([s[0] for s in states], np.float32)
    m = ms.max()
    m = F(0.) if m == NEG_INF else m
    a = _exp(ms - m)
    z = F(sum((F(a_ * s[1]) for a_, s in zip(a, states)), F(0.)))
    u = np.zeros_like(states[0][2])
    for a_, s in zip(a, states):
        u = (u + a_ * s[2]).astype(np.float32)
    return u, z


def _repair_saved(X, i, A, P, pred, mn, tol, eps, variant):
    """gqa.py:62-104 (_merge_repair): saved gathers hit states, union keeps all P."""
    hit, miss = _membership(A, P)
    states = []
    for j in range(len(P)):
        if variant == "union" or hit[j]:
            states.append((F(pred["m"][i, j]), F(pred["l"][i, j]), _f(pred["u"][i, j])))
    for a_ in A[miss]:
        states.append(block_state(X, i, a_))
    u, z = _merge_states(states)
    return {"output": (u / z).astype(np.float32), "fallback": False, "remaining": 1.0}


def _strict(X, i, A):
    _, z, u = online(X, i, A)
    return (u / z).astype(np.float32)


def _repair_split(X, i, A, P, pred, mn, tol, eps, variant):
    """kernels.py:504-550: membership, miss partials, merge in the common frame, fallback."""
    hit_p, miss = _membership(A, P)
    mode = pred["mode"]
    if mode == "saved":  # _saved_merge, kernels.py:196-218
        states = [(F(pred["m"][i, j]), F(pred["l"][i, j]), _f(pred["u"][i, j])) for j in range(len(P)) if hit_p[j]]
        states += [block_state(X, i, a_) for a_ in A[miss]]
        ms = np.array([s[0] for s in states], np.float32)
        m = ms.max()
        a = _exp(ms - m)
        z = F(sum((F(x * s[1]) for x, s in zip(a, states)), F(0.)))
        u = np.zeros(X.d, np.float32)
        for x, s in zip(a, states):
            u = (u + x * s[2]).astype(np.float32)
        return {"output": (u / z).astype(np.float32), "fallback": False, "remaining": 1.0}
    high = pred["high"][i]
    low_hit = bool((hit_p & ~high).any())
    wrong = (~hit_p) & (~high) & low_hit
    if mode == "compact":  # _compact_membership, kernels.py:359-381
        r = pred["retained_ids"][i]
        hit_s = (r >= 0) & np.isin(r, A)
    else:
        hit_s = hit_p & high
    lm = F(pred["low_m"][i])
    # wrong states: per-block (hybrid) or one per-token aggregate at LM (compact)
    if mode == "compact":
        wz, wu, _ = fixed_frame_sums(X, i, [P[j] for j in range(len(P)) if wrong[j]], lm)
        wstates = [(lm, wz, wu)] if low_hit else []
    else:
        wstates = [block_state(X, i, P[j]) for j in range(len(P)) if wrong[j]] if low_hit else []
    astates = [block_state(X, i, a_) for a_ in A[miss]]
    pm = [F(pred["m"][i, c]) for c in range(len(hit_s)) if hit_s[c]]
    m = F(max(pm + [s[0] for s in astates] + ([lm] if low_hit else []) + [NEG_INF]))
    lowalpha = _exp(lm - m) if low_hit else F(0.)
    ll = F(pred["low_l"][i] * lowalpha) if low_hit else F(0.)
    removed = F(0.)
    removed_u = np.zeros(X.d, np.float32)
    for wm, wl, wu_ in wstates:
        aw = _exp(wm - m)
        removed = F(removed + aw * wl)
        removed_u = (removed_u + aw * wu_).astype(np.float32)
    remaining = F(ll - removed)
    fraction = F(remaining / max(ll, F(1e-30))) if ll > 0 else F(1.)
    z = remaining
    u = ((pred["low_u"][i] * lowalpha if low_hit else np.zeros(X.d, np.float32)) - removed_u).astype(np.float32)
    residual = u.copy()
    for c in range(len(hit_s)):
        if hit_s[c]:
            ap = _exp(F(pred["m"][i, c]) - m)
            z = F(z + ap * F(pred["l"][i, c]))
            u = (u + ap * _f(pred["u"][i, c])).astype(np.float32)
    for am, al, au in astates:
        ax = _exp(am - m)
        z = F(z + ax * al)
        u = (u + ax * au).astype(np.float32)
    low_abs = (pred["low_abs"][i] * lowalpha if low_hit else np.zeros(X.d, np.float32)).astype(np.float32)
    scale = (low_abs + np.abs(removed_u)).astype(np.float32)
    cancel = low_hit and bool(((np.abs(residual) < tol * scale) & (scale > 0)).any())
    with np.errstate(all="ignore"):
        out = (u / max(z, F(1e-30))).astype(np.float32)
    bad = bool(z <= 0 or fraction < mn or np.isnan(fraction) or np.isinf(z) or cancel
               or (~np.isfinite(out)).any())
    margin = _guard_margin(fraction, mn, residual, scale, tol) if low_hit else np.inf
    if bad:
        out = _strict(X, i, A)
    return {"output": out, "fallback": bad, "remaining": float(fraction), "margin": margin}


def _repair_fused(X, i, A, P, pred, mn, tol, eps, variant):
    """fused.py:48-173 (one CTA per head)."""
    hybrid = pred["mode"] in ("hybrid", "compact")
    hit, missing = _membership(A, P)
    high = pred["high"][i] if hybrid else np.zeros(len(P), bool)
    low_hit = bool((hit & ~high).any()) if hybrid else False
    keep = _keep(pred, i, A, hit, high)
    pm = np.where(keep, pred["m"][i], NEG_INF).astype(np.float32)
    pl = np.where(keep, pred["l"][i], F(0.)).astype(np.float32)
    retained_m = F(pm.max()) if pm.size else NEG_INF
    fraction, bad, mass, lm, skip, extra = F(1.), False, F(0.), NEG_INF, False, F(0.)
    residual = np.zeros(X.d, np.float32)
    margin = np.inf
    if hybrid and low_hit:
        lm = F(pred["low_m"][i])
        ll = F(pred["low_l"][i])
        wrong = ~hit & ~high
        removed, removed_u = F(0.), np.zeros(X.d, np.float32)
        if eps > 0 and wrong.any():
            skip, extra = _eps_decision(pred, i, keep, wrong, lm, eps)
        if wrong.any() and not skip:
            removed, removed_u, _ = fixed_frame_sums(X, i, [P[j] for j in range(len(P)) if wrong[j]], lm)
        mass = F(ll - removed)
        residual = (pred["low_u"][i] - removed_u).astype(np.float32)
        fraction = F(mass / ll)
        scale = (pred["low_abs"][i] + np.abs(removed_u)).astype(np.float32)
        cancel = bool(((np.abs(residual) < tol * scale) & (scale > 0)).any())
        bad = bool(fraction < mn or np.isnan(fraction) or cancel)
        margin = _guard_margin(fraction, mn, residual, scale, tol, extra if eps > 0 and wrong.any() else None, eps)
    m = F(max(retained_m, lm))
    ref = F(0.) if m == NEG_INF else m
    alpha = _exp(pm - ref)
    low_alpha = _exp(lm - ref)
    z = F((alpha * pl).sum(dtype=np.float32) + low_alpha * mass)
    u = ((alpha[:, None] * np.where(keep[:, None], pred["u"][i], F(0.))).sum(0, dtype=np.float32)
         + low_alpha * residual).astype(np.float32)
    todo = A[missing]
    if hybrid and bad:
        todo, m, z, u = A, NEG_INF, F(0.), np.zeros(X.d, np.float32)
    if len(todo):
        m, z, u = online(X, i, todo, m, z, u)
    with np.errstate(all="ignore"):
        out = (u / z).astype(np.float32)
    if hybrid:
        bad_output = bool(z <= 0 or np.isinf(z) or (~np.isfinite(out)).any())
        if bad_output and not bad:
            out = _strict(X, i, A)
        bad = bad or bad_output
    approx = skip and not bad
    return {"output": out, "fallback": bad, "remaining": float(fraction), "approx": approx,
            "extra": float(extra) if approx else 0.0, "margin": margin}


def _repair_signed(X, i, A, P, pred, mn, tol, eps, variant):
    """signed_repair.py:18-172 (+ _fallback) and signed_fused.py:30-145."""
    hybrid = pred["mode"] in ("hybrid", "compact")
    compact = pred["mode"] == "compact"
    hit, miss = _membership(A, P)
    high = pred["high"][i] if hybrid else np.zeros(len(P), bool)
    low_hit = bool((hit & ~high).any()) if hybrid else False
    wrong = low_hit & ~hit & ~high
    keep = _keep(pred, i, A, hit, high)
    skip, extra = False, F(0.)
    lm = F(pred["low_m"][i]) if hybrid else NEG_INF
    decided = bool(hybrid and eps > 0 and wrong.any())
    if decided:
        skip, extra = _eps_decision(pred, i, keep, wrong, lm, eps)
        wrong = wrong & (not skip)
    pos = int(miss.sum())
    queue = [(a_, +1) for a_ in A[miss]] + ([(P[j], -1) for j in range(len(P)) if wrong[j]] if hybrid else [])
    total = len(queue)
    jobs = []
    for bid, sign in queue:
        if variant == "signed_fused" and sign < 0 and compact:
            z_, u_, _ = fixed_frame_sums(X, i, [bid], lm)
            jobs.append((lm, F(-z_), (-u_).astype(np.float32), sign))
        else:
            bm, bl, bu = block_state(X, i, bid)
            if sign < 0 and variant == "signed_fused":
                f = _exp(bm - lm)
                jobs.append((lm, F(-(bl * f)), (-(bu * f)).astype(np.float32), sign))
            else:
                jobs.append((bm, F(sign * bl), (sign * bu).astype(np.float32), sign))
    pm = np.where(keep, pred["m"][i], NEG_INF).astype(np.float32)
    pl = np.where(keep, pred["l"][i], F(0.)).astype(np.float32)
    pu = np.where(keep[:, None], pred["u"][i], F(0.)).astype(np.float32)
    fraction, bad = F(1.), False
    margin = np.inf
    low_m, low_z, low_u = NEG_INF, F(0.), np.zeros(X.d, np.float32)
    if hybrid and low_hit:
        low_m = lm
        oz = F(pred["low_l"][i])
        delta_u = np.zeros(X.d, np.float32)
        dz = F(0.)
        for cm, cl, cu, sign in jobs:
            if sign < 0:
                wx = _exp(cm - low_m)  # signed_fused negatives are already at low_m: wx == 1
                delta_u = (delta_u + wx * cu).astype(np.float32)
                dz = F(dz + wx * cl)
        low_z = F(oz + dz)
        low_u = (pred["low_u"][i] + delta_u).astype(np.float32)
        fraction = F(low_z / oz)
        scale = (pred["low_abs"][i] + np.abs(delta_u)).astype(np.float32)
        cancel = bool(((np.abs(low_u) < tol * scale) & (scale > 0)).any())
        bad = bool(fraction < mn or np.isnan(fraction) or cancel)
        margin = _guard_margin(fraction, mn, low_u, scale, tol, extra if eps > 0 and decided else None, eps)
    posm = [cm for cm, _, _, sg in jobs if sg > 0]
    m = F(max([pm.max() if pm.size else NEG_INF] + posm + [low_m]))
    px = _exp(pm - m)
    z = F((px * pl).sum(dtype=np.float32))
    u = (px[:, None] * pu).sum(0, dtype=np.float32)
    for cm, cl, cu, sg in jobs:
        if sg > 0:
            ax = _exp(cm - m)
            z = F(z + ax * cl)
            u = (u + ax * cu).astype(np.float32)
    lx = _exp(low_m - m)
    z = F(z + lx * low_z)
    u = (u + lx * low_u).astype(np.float32)
    with np.errstate(all="ignore"):
        out = (u / z).astype(np.float32)
    if hybrid:
        bad = bad or bool(z <= 0 or np.isinf(z) or (~np.isfinite(out)).any())
        if bad:
            out = _strict(X, i, A)
    approx = skip and not bad
    return {"output": out, "fallback": bad, "remaining": float(fraction), "approx": approx,
            "extra": float(extra) if approx else 0.0, "pos": pos, "total": total, "margin": margin}
