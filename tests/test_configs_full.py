"""GPU parity at the BASELINE configurations' own sizes.

The library (through the drop-in API and its C ABI) against the CPU oracle on
identical seeded inputs:

* config 1 (32 q / 8 KV heads, D 128, 2048 blocks of 32, K 64, bf16): seeds
  0/1/2 x predicted overlap 1.0/0.9/0.75 x every method the bench runs
  (saved, gqa_light, compact, repair_fused, signed_fused), strict and with
  max_extra_mass = 0.01. Block IDs bit-exact; outputs within the north-star
  bf16 bar (|err| <= 2e-3 + 1e-2 |ref|) of the FP64 oracle over the strict
  set (or, for rows the relaxed repair approximates, over the strict set plus
  the retained wrong-low blocks); and the discrete decisions equal the
  oracle's: high masks, compact packing and overflow, fallback, approximation
  flags, extra-mass bounds and signed job counts. A decision may differ only
  where the oracle's guard input lies within a few FP32 roundings of its
  threshold (the summation orders differ), and such rows are reported;
* config 2 (96 q / 8 KV heads, 8192 blocks of 4 tokens, K 512 shared per
  group, 80 % overlap) through gqa_hierarchical (partials ->
  repair_saved_shared, exact) and the tensor-core exact_shared;
* config 3 (paged requests with U[8192, 32768]-token contexts, 16 q / 8 KV,
  page 16, K 64, overlap ~ Beta(8, 2)) in relaxed mode, against the relaxed
  oracle of benchmarks/signed_benchmark.py:21-33 and the FP64 mass check of
  benchmarks/pareto_benchmark.py:15-28;
* config 4 (32 q / 8 KV, 8192 blocks of 64, K 256, overlap 0.7) as 2, 4 and 8
  ranks emulated on one GPU: IDs bit-identical to single-GPU selection and to
  the oracle, outputs within the bf16 bar.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import cases as C
from oracle import attention as OA
from oracle import selection as OS
from oracle import speculative as OP

pytestmark = pytest.mark.gpu

DEV = "cuda"
BORDER = 1e-5  # guard inputs this close (relative) to a threshold may round either way


def _bar(out, ref):
    out = out.cpu().numpy() if isinstance(out, torch.Tensor) else np.asarray(out)
    err = np.abs(out - ref)
    return bool((err <= 2e-3 + 1e-2 * np.abs(ref)).all()), float(err.max())


def _fp64_rows_gqa(q, k, v, heads, rows_ids, g):
    """FP64 oracle for query heads ``heads`` of q, head h over its own block
    list rows_ids[j] (lists may differ in length); k/v torch CPU
    [Hkv, N, B, D]. Returns [len(heads), D]."""
    qn = q.float().numpy()
    out = np.empty((len(rows_ids), qn.shape[1]))
    for j, (h, ids) in enumerate(zip(heads, rows_ids)):
        idx = torch.as_tensor(np.asarray(ids, np.int64))
        kk = k[h // g][idx].float().numpy()[None]
        vv = v[h // g][idx].float().numpy()[None]
        out[j] = OA.attention_fp64(qn[h:h + 1], kk, vv, np.arange(len(ids))[None])[0]
    return out


def _high_margin(m, l, tau):
    """Relative distance of every slot's mass share to the high threshold
    (kernels.py:100-117: mass = e^(m - max m) l, high = mass >= tau * sum)."""
    m = np.asarray(m, np.float64)
    l = np.asarray(l, np.float64)
    mass = np.exp(m - m.max(axis=1, keepdims=True)) * l
    tot = mass.sum(axis=1, keepdims=True)
    return np.abs(mass - tau * tot) / np.maximum(tot, 1e-300)


def _decisions_equal(name, got, want, margin, tag):
    """Boolean decisions equal, except where the oracle's margin says the
    decision sits on its threshold; returns the borderline rows."""
    got = np.asarray(got, bool)
    want = np.asarray(want, bool)
    diff = got != want
    border = diff & (np.asarray(margin) <= BORDER)
    assert not (diff & ~border).any(), (tag, name, np.argwhere(diff & ~border)[:8].tolist())
    return np.argwhere(border).tolist()


# ----------------------------------------------------------------------------- config 1

C1 = dict(hq=32, hkv=8, n=2048, b=32, d=128, k=64)
METHODS = ("saved", "gqa_light", "compact", "repair_fused", "signed_fused")


@pytest.fixture(scope="module")
def status_word():
    import strict_topk_overlap_b200._lib as L
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    L.set_status_tensor(st)
    yield st
    torch.cuda.synchronize()
    L.set_status_tensor(None)
    assert st.item() == 0, f"device status {st.item()}"


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_config1_every_method_and_decision(seed, status_word):
    from strict_topk import fused, gqa, gqa_light, kernels, signed_fused
    from strict_topk_overlap_b200.decode import SpeculativeDecoder, StepSpec
    hq, hkv, n, b, d, topk = (C1[x] for x in ("hq", "hkv", "n", "b", "d", "k"))
    g = hq // hkv
    q, k, v, lo, hi = C.synthetic_kv(hq, hkv, n, b, d, torch.bfloat16, seed=seed)
    qn, kn, vn = C.as_np(q), C.as_np(k), C.as_np(v)
    want_ids = OS.select_blocks(qn, lo.numpy(), hi.numpy(), topk)
    qd, kd, vd, lod, hid = (t.to(DEV) for t in (q, k, v, lo, hi))
    a = gqa.select_blocks(qd, lod, hid, topk)
    assert np.array_equal(a.cpu().numpy(), want_ids), "C1 selection differs from the FP64 oracle"
    strict_ref = OA.attention_fp64(qn, kn, vn, want_ids)
    border_rows = []
    for overlap in (1.0, 0.9, 0.75):
        nswap = round((1 - overlap) * topk)
        p = C.swap_prediction(torch.from_numpy(want_ids), n, nswap, seed=seed * 10 + nswap)
        pn = p.numpy()
        pd = p.to(DEV)
        tag = f"seed {seed} overlap {overlap}"
        for method in METHODS:
            mtag = f"{tag} {method}"
            if method in ("saved", "gqa_light"):
                st = gqa.partials(qd, kd, vd, pd)
                out = (gqa.repair_saved if method == "saved" else gqa_light.repair_saved_light)(qd, kd, vd, a, pd, st)
                ok, err = _bar(out, strict_ref)
                assert ok, (mtag, err)
                want = OP.repair("saved", qn, kn, vn, want_ids, pn, OP.speculate(qn, kn, vn, pn, "saved"))
                assert np.abs(out.cpu().numpy() - want["output"]).max() <= 1e-4, mtag
                continue
            mode = "compact" if method == "compact" else "hybrid"
            pred = kernels.speculate(qd, kd, vd, pd, mode=mode, mass_threshold=0.1, keep_mass=True)
            want_pred = OP.speculate(qn, kn, vn, pn, mode, 0.1, keep_mass=True)
            mm = want_pred["mass_m"]
            ml = want_pred["mass_l"]
            hmargin = _high_margin(mm, ml, 0.1)
            border_rows += _decisions_equal("high", pred.high.cpu().numpy(), want_pred["high"], hmargin, mtag)
            rows_ok = ~(pred.high.cpu().numpy() != want_pred["high"]).any(axis=1)
            if mode == "compact":
                ov_g, ov_w = pred.overflow.cpu().numpy(), want_pred["overflow"]
                assert np.array_equal(ov_g[rows_ok], ov_w[rows_ok]), (mtag, "overflow")
                rg = pred.retained_ids.cpu().numpy().astype(np.int64)
                assert np.array_equal(rg[rows_ok], want_pred["retained_ids"][rows_ok]), (mtag, "retained_ids")
            for eps in (0.0, 0.01):
                if method == "signed_fused":
                    res = signed_fused.repair_signed_fused(qd, kd, vd, a, pd, pred, max_extra_mass=eps)
                    want = OP.repair("signed_fused", qn, kn, vn, want_ids, pn, want_pred, max_extra_mass=eps)
                else:
                    res = fused.repair_fused(qd, kd, vd, a, pd, pred, max_extra_mass=eps)
                    want = OP.repair("fused", qn, kn, vn, want_ids, pn, want_pred, max_extra_mass=eps)
                etag = f"{mtag} eps {eps}"
                margin = np.where(rows_ok, want["margin"], 0.0)
                border_rows += _decisions_equal("fallback", res.fallback.cpu().numpy(), want["fallback"], margin, etag)
                approx = res.approximate_heads.cpu().numpy() if res.approximate_heads is not None else np.zeros(hq, bool)
                border_rows += _decisions_equal("approx", approx, want["approx"], margin, etag)
                same = rows_ok & (res.fallback.cpu().numpy() == want["fallback"]) & (approx == want["approx"])
                if res.extra_mass_bound is not None:
                    eb = res.extra_mass_bound.cpu().numpy()
                    assert np.allclose(eb[same], np.asarray(want["extra"], np.float32)[same], rtol=1e-4, atol=1e-7), \
                        (etag, "extra_mass_bound")
                    assert (eb[approx] <= eps + 1e-7).all() and (eb[~approx] == 0).all(), etag
                rem = res.remaining.cpu().numpy()
                assert np.allclose(rem[same], np.asarray(want["remaining"], np.float32)[same], rtol=1e-4, atol=1e-6), \
                    (etag, "remaining")
                if method == "signed_fused":
                    assert np.array_equal(res.positive_jobs.cpu().numpy()[same], want["pos"][same]), (etag, "pos")
                    assert np.array_equal(res.total_jobs.cpu().numpy()[same], want["total"][same]), (etag, "total")
                # Output: strict rows against the strict set; approximated rows
                # against the strict set plus the retained wrong-low blocks.
                out = res.output.cpu().numpy()
                ref = strict_ref.copy()
                if approx.any():
                    high = pred.high.cpu().numpy()
                    rows_ids = []
                    for h in np.nonzero(approx)[0]:
                        extra = [int(x) for x, hh in zip(pn[h], high[h]) if not hh and x not in set(want_ids[h])]
                        rows_ids.append(list(want_ids[h]) + extra)
                    ref[approx] = _fp64_rows_gqa(q, k, v, np.nonzero(approx)[0], rows_ids, g)
                ok, err = _bar(out, ref)
                assert ok, (etag, "output", err)
        # The chained decode steps the bench times give the same results.
        for method in ("saved", "repair_fused", "signed_fused"):
            dec = SpeculativeDecoder(qd, kd, vd, lod, hid, pd, StepSpec(topk=topk, method=method), graph=False)
            out = dec.step()
            torch.cuda.synchronize()
            assert torch.equal(dec.selected.cpu(), a.cpu()), (tag, method, "chained IDs")
            ok, err = _bar(out, strict_ref)
            assert ok, (tag, method, "chained", err)
    if border_rows:
        print(f"seed {seed}: {len(border_rows)} decision(s) on a threshold boundary: {border_rows[:8]}")


# ----------------------------------------------------------------------------- config 2

def test_config2_hierarchical_full_size(status_word):
    from strict_topk import gqa_hierarchical as GH
    hq, hkv, n, b, d, topk = 96, 8, 8192, 4, 128, 512
    g = hq // hkv
    q, k, v, lo, hi = C.synthetic_kv(hq, hkv, n, b, d, torch.bfloat16, seed=2)
    qn = C.as_np(q)
    want = OS.select_blocks(qn, lo.numpy(), hi.numpy(), topk, shared=True)  # [Hq, K], group rows repeated
    qd, kd, vd, lod, hid = (t.to(DEV) for t in (q, k, v, lo, hi))
    a = GH.select_blocks_shared(qd, lod, hid, topk)
    assert np.array_equal(a.cpu().numpy(), want), "C2 shared selection differs from the FP64 oracle"
    ref = OA.attention_fp64(qn, C.as_np(k), C.as_np(v), want)
    # Predicted list per group: 80 % overlap, one list shared by the group's heads.
    group_a = torch.from_numpy(want[::g].copy())
    p_group = C.swap_prediction(group_a, n, round(0.2 * topk), seed=21)
    p = p_group.repeat_interleave(g, dim=0).contiguous().to(DEV)
    st = GH.partials(qd, kd, vd, p)
    out_shared = GH.repair_saved_shared(qd, kd, vd, a, p, st)
    out_saved = GH.repair_saved(qd, kd, vd, a, p, st)
    out_exact = GH.exact(qd, kd, vd, a)
    out_mma = GH.exact_shared(qd, kd, vd, a[::g].contiguous())
    for name, out in (("repair_saved_shared", out_shared), ("repair_saved", out_saved), ("exact", out_exact),
                      ("exact_shared", out_mma)):
        ok, err = _bar(out, ref)
        assert ok, (name, err)
    assert (out_shared - out_saved).abs().max().item() <= 1e-6


# ----------------------------------------------------------------------------- config 3

def test_config3_relaxed_decisions(status_word):
    """Relaxed mode (max_extra_mass = 0.01) on a batch of paged requests with
    config 3's context distribution, request by request against the oracle."""
    from strict_topk_overlap_b200 import paged
    HQ, HKV, D, B, PAGE, TOPK, EPS = 16, 8, 128, 32, 16, 64, 0.01
    gen = torch.Generator().manual_seed(33)
    lengths = [int(x) // 32 * 32 for x in (8192 + torch.rand(6, generator=gen) * (32768 - 8192)).tolist()]
    torch.manual_seed(35)
    overlaps = torch.distributions.Beta(8.0, 2.0).sample((len(lengths),)).tolist()
    qs, ks, vs = [], [], []
    for r, tokens in enumerate(lengths):
        q, k, v, _, _ = C.synthetic_kv(HQ, HKV, tokens // B, B, D, torch.bfloat16, seed=300 + r)
        qs.append(q)
        ks.append(k)
        vs.append(v)
    cache = paged.build_paged_cache(ks, vs, PAGE, generator=torch.Generator().manual_seed(37),
                                    device=torch.device(DEV))
    q = torch.cat(qs, 0).contiguous()
    qd = q.to(DEV)
    a = paged.select_blocks(qd, cache, TOPK)
    a_cpu = a.cpu().numpy()
    preds = []
    for r, k in enumerate(ks):
        lo, hi = k.amin(dim=2).float(), k.amax(dim=2).float()
        want_ids = OS.select_blocks(C.as_np(qs[r]), lo.numpy(), hi.numpy(), TOPK)
        assert np.array_equal(a_cpu[r * HQ:(r + 1) * HQ], want_ids), f"request {r}: IDs"
        nswap = round((1 - overlaps[r]) * TOPK)
        preds.append(C.swap_prediction(torch.from_numpy(want_ids), k.shape[1], nswap, seed=400 + r))
    p = torch.cat(preds, 0).contiguous().to(DEV)
    pred = paged.speculate(qd, cache, p, mode="hybrid", mass_threshold=0.1, keep_mass=True)
    results = {"fused": paged.repair_fused(qd, cache, a, p, pred, max_extra_mass=EPS),
               "signed_fused": paged.repair_signed_fused(qd, cache, a, p, pred, max_extra_mass=EPS)}
    torch.cuda.synchronize()
    high_all = pred.high.cpu().numpy()
    n_approx = 0
    for variant, res in results.items():
        approx_all = res.approximate_heads.cpu().numpy()
        extra_all = res.extra_mass_bound.cpu().numpy()
        fb_all = res.fallback.cpu().numpy()
        out_all = res.output.cpu().numpy()
        for r, (k, v) in enumerate(zip(ks, vs)):
            sl = slice(r * HQ, (r + 1) * HQ)
            qn, kn, vn = C.as_np(qs[r]), C.as_np(k), C.as_np(v)
            pn = preds[r].numpy()
            ids = a_cpu[sl]
            wp = OP.speculate(qn, kn, vn, pn, "hybrid", 0.1, keep_mass=True)
            hmargin = _high_margin(wp["mass_m"], wp["mass_l"], 0.1)
            _decisions_equal("high", high_all[sl], wp["high"], hmargin, f"C3 request {r}")
            rows_ok = ~(high_all[sl] != wp["high"]).any(axis=1)
            want = OP.repair(variant, qn, kn, vn, ids, pn, wp, max_extra_mass=EPS)
            margin = np.where(rows_ok, want["margin"], 0.0)
            tag = f"C3 {variant} request {r}"
            _decisions_equal("approx", approx_all[sl], want["approx"], margin, tag)
            _decisions_equal("fallback", fb_all[sl], want["fallback"], margin, tag)
            same = rows_ok & (approx_all[sl] == want["approx"]) & (fb_all[sl] == want["fallback"])
            assert np.allclose(extra_all[sl][same], np.asarray(want["extra"], np.float32)[same], rtol=1e-4,
                               atol=1e-7), tag
            # Relaxed oracle: strict set plus the retained wrong-low blocks for approximated rows.
            rows_ids = []
            for h in range(HQ):
                row = list(ids[h])
                if approx_all[sl][h]:
                    sel = set(row)
                    row += [int(x) for x, hh in zip(pn[h], high_all[sl][h]) if not hh and int(x) not in sel]
                rows_ids.append(row)
            ref = _fp64_rows_gqa(qs[r], k, v, range(HQ), rows_ids, HQ // HKV)
            ok, err = _bar(out_all[sl], ref)
            assert ok, (tag, err)
            # FP64 probability mass of the extra blocks stays within the budget.
            for h in np.nonzero(approx_all[sl])[0]:
                n_approx += 1
                extra = rows_ids[h][TOPK:]
                if not extra:
                    continue
                kk = k[h // (HQ // HKV)]
                qq = qs[r][h].double()
                chosen = (kk[torch.as_tensor(ids[h], dtype=torch.long)].double().reshape(-1, D) @ qq) / D ** 0.5
                ext = (kk[torch.as_tensor(extra, dtype=torch.long)].double().reshape(-1, D) @ qq) / D ** 0.5
                mass = torch.exp(torch.logsumexp(ext, 0) - torch.logsumexp(torch.cat([chosen, ext]), 0)).item()
                assert mass <= EPS * (1 + 1e-3), (tag, h, mass)
    print(f"C3 relaxed: {n_approx} approximated rows checked")


# ----------------------------------------------------------------------------- config 4

@pytest.mark.parametrize("world", [2, 4, 8])
def test_config4_context_parallel_full_size(world, status_word):
    from strict_topk import gqa
    from test_context_parallel import _emulated_ranks
    hq, hkv, n, b, d, topk = 32, 8, 8192, 64, 128, 256
    g = hq // hkv
    cg = torch.Generator(device=DEV).manual_seed(44)
    qd = torch.randn(hq, d, device=DEV, generator=cg).to(torch.bfloat16)
    kd = (torch.randn(hkv, n, b, d, device=DEV, generator=cg)
          + torch.randn(hkv, n, 1, d, device=DEV, generator=cg) * 0.5).to(torch.bfloat16)
    vd = torch.randn(hkv, n, b, d, device=DEV, generator=cg).to(torch.bfloat16)
    lod, hid = kd.amin(dim=2).float(), kd.amax(dim=2).float()
    ids = OS.select_blocks(qd.float().cpu().numpy(), lod.cpu().numpy(), hid.cpu().numpy(), topk)
    single = gqa.select_blocks(qd, lod, hid, topk).cpu().numpy()
    assert np.array_equal(single, ids), "C4 single-GPU selection differs from the FP64 oracle"
    # FP64 oracle over each row's selected blocks only (gathered on the device, then copied).
    ref = np.empty((hq, d))
    qn = qd.float().cpu().numpy()
    for h in range(hq):
        idx = torch.as_tensor(ids[h], dtype=torch.long, device=DEV)
        kk = kd[h // g][idx].float().cpu().numpy()[None]
        vv = vd[h // g][idx].float().cpu().numpy()[None]
        ref[h] = OA.attention_fp64(qn[h:h + 1], kk, vv, np.arange(topk)[None])[0]
    pred = C.swap_prediction(torch.from_numpy(ids), n, round(0.3 * topk), seed=45).to(DEV)
    strict = _emulated_ranks(world, qd, kd, vd, lod, hid, topk)
    spec = _emulated_ranks(world, qd, kd, vd, lod, hid, topk, predicted=pred)
    for r in range(world):
        o, sel = strict[r]
        assert np.array_equal(sel.numpy(), ids), (world, r, "strict IDs")
        ok, err = _bar(o, ref)
        assert ok, (world, r, err)
        assert torch.equal(o, strict[0][0])
        so, ssel = spec[r]
        assert np.array_equal(ssel.numpy(), ids), (world, r, "speculative IDs")
        ok, err = _bar(so, ref)
        assert ok, (world, r, "speculative", err)
