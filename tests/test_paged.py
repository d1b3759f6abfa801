"""Batched paged-KV decode (BASELINE config 3 shape, reduced sizes): the
sm_100a library through the batched entry points against the CPU oracle,
request by request, on identical seeded inputs.

Bars: block IDs bit-exact (ties to the lower index) against the FP64
stable-sorted oracle of each request; strict outputs within the north-star
bf16 tolerance (max-abs 2e-3 / rel 1e-2) of the FP64 oracle; the batched
saved / fused repairs equal the batched exact attention; rows the relaxed
repair approximates carry an extra-mass bound <= max_extra_mass and stay within
the error that bound allows."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import cases as C
from oracle import attention as OA
from oracle import selection as OS

pytestmark = pytest.mark.gpu

DEV = "cuda"
HQ, HKV, D, B, PAGE, TOPK = 16, 8, 128, 32, 16, 16


def _batch(seed=0, lengths=(40, 64, 97, 128)):
    """Per-request dense caches with the BASELINE distribution, and their paged pool."""
    from strict_topk_overlap_b200 import paged
    qs, ks, vs = [], [], []
    for r, n in enumerate(lengths):
        q, k, v, _, _ = C.synthetic_kv(HQ, HKV, n, B, D, torch.bfloat16, seed=seed * 100 + r)
        qs.append(q)
        ks.append(k)
        vs.append(v)
    gen = torch.Generator().manual_seed(seed + 12345)
    cache = paged.build_paged_cache(ks, vs, PAGE, generator=gen, device=torch.device(DEV))
    q = torch.cat(qs, 0).contiguous()
    return q, ks, vs, cache


def _oracle_ids(q, ks):
    rows = []
    for r, k in enumerate(ks):
        lo, hi = k.amin(dim=2).float(), k.amax(dim=2).float()
        rows.append(OS.select_blocks(q[r * HQ:(r + 1) * HQ].float().numpy(), lo.numpy(), hi.numpy(), TOPK))
    return np.concatenate(rows, 0)


def _oracle_out(q, ks, vs, ids):
    outs = []
    for r, (k, v) in enumerate(zip(ks, vs)):
        outs.append(OA.attention_fp64(q[r * HQ:(r + 1) * HQ].float().numpy(), k.float().numpy(),
                                      v.float().numpy(), ids[r * HQ:(r + 1) * HQ]))
    return np.concatenate(outs, 0)


def _close(out, ref):
    """North-star bf16 bar: |err| <= 2e-3 + 1e-2 |ref| elementwise."""
    out = out.cpu().numpy() if isinstance(out, torch.Tensor) else out
    return bool((np.abs(out - ref) <= 2e-3 + 1e-2 * np.abs(ref)).all())


def _predicted(ids, lengths, overlap, seed):
    """Per-row predicted lists: true Top-K with round((1-overlap)*K) IDs swapped
    for seeded-random unselected blocks of the row's request."""
    rng = np.random.default_rng(seed)
    rows = []
    for i, row in enumerate(ids.tolist()):
        n = lengths[i // HQ]
        chosen = set(row)
        pool = np.array([x for x in range(n) if x not in chosen])
        nswap = int(round((1 - overlap) * TOPK))
        pos = rng.choice(TOPK, nswap, replace=False)
        repl = rng.choice(pool, nswap, replace=False)
        row = list(row)
        for j, x in zip(pos, repl):
            row[j] = int(x)
        rows.append(row)
    return torch.tensor(rows, dtype=torch.int32)


@pytest.fixture(scope="module")
def batch():
    lengths = (40, 64, 97, 128)
    q, ks, vs, cache = _batch(0, lengths)
    return lengths, q, ks, vs, cache


def test_paged_selection_bit_exact(batch):
    from strict_topk_overlap_b200 import paged
    lengths, q, ks, vs, cache = batch
    ids = paged.select_blocks(q.to(DEV), cache, TOPK)
    torch.cuda.synchronize()
    assert np.array_equal(ids.cpu().numpy(), _oracle_ids(q, ks))


def test_paged_exact_and_saved_repair(batch):
    from strict_topk_overlap_b200 import paged
    lengths, q, ks, vs, cache = batch
    qd = q.to(DEV)
    a = paged.select_blocks(qd, cache, TOPK)
    ref = _oracle_out(q, ks, vs, a.cpu().numpy())
    out = paged.exact(qd, cache, a)
    assert _close(out, ref)
    for overlap in (1.0, 0.75, 0.5):
        p = _predicted(a.cpu().numpy(), lengths, overlap, seed=int(overlap * 10)).to(DEV)
        st = paged.partials(qd, cache, p)
        rep = paged.repair_saved(qd, cache, a, p, st)
        torch.cuda.synchronize()
        assert (rep - out).abs().max().item() <= 1e-4, overlap


def test_paged_fused_strict_and_relaxed(batch):
    from strict_topk_overlap_b200 import paged
    lengths, q, ks, vs, cache = batch
    qd = q.to(DEV)
    a = paged.select_blocks(qd, cache, TOPK)
    exact = paged.exact(qd, cache, a)
    vmax = max(float(v.float().abs().max()) for v in vs)
    for overlap in (0.9, 0.75):
        p = _predicted(a.cpu().numpy(), lengths, overlap, seed=7).to(DEV)
        pred = paged.speculate(qd, cache, p, mode="hybrid", mass_threshold=0.1, keep_mass=True)
        strict = paged.repair_fused(qd, cache, a, p, pred)
        assert (strict.output - exact).abs().max().item() <= 2e-3
        eps = 0.01
        rel = paged.repair_fused(qd, cache, a, p, pred, max_extra_mass=eps)
        torch.cuda.synchronize()
        approx = rel.approximate_heads.cpu().numpy()
        bound = rel.extra_mass_bound.cpu().numpy()
        err = (rel.output - exact).abs().amax(dim=1).cpu().numpy()
        assert (bound[approx] <= eps + 1e-7).all()
        assert (bound[~approx] == 0).all()
        assert (err[~approx] <= 2e-3).all()
        # An approximated row keeps extra mass <= eps of its normaliser: its
        # output moves by at most ~2 eps max|v|.
        assert (err[approx] <= 2 * eps * vmax + 2e-3).all()


def test_paged_equals_dense_per_request(batch):
    """The batched paged path and the single-request dense path agree."""
    from strict_topk import gqa
    from strict_topk_overlap_b200 import paged
    lengths, q, ks, vs, cache = batch
    qd = q.to(DEV)
    a = paged.select_blocks(qd, cache, TOPK)
    out = paged.exact(qd, cache, a)
    for r, (k, v) in enumerate(zip(ks, vs)):
        qr = q[r * HQ:(r + 1) * HQ].to(DEV)
        kd, vd = k.to(DEV), v.to(DEV)
        lo, hi = k.amin(dim=2).float().to(DEV), k.amax(dim=2).float().to(DEV)
        ar = gqa.select_blocks(qr, lo, hi, TOPK)
        assert torch.equal(ar, a[r * HQ:(r + 1) * HQ])
        o = gqa.exact(qr, kd, vd, ar)
        assert (o - out[r * HQ:(r + 1) * HQ]).abs().max().item() <= 1e-5


@pytest.mark.parametrize("variant", ["saved", "repair_fused", "signed_fused"])
def test_batched_chained_step_equals_separate_calls(variant):
    """paged.speculative_step (one launch chain for the whole batch) against
    the separate batched calls it replaces, and its IDs against the oracle;
    the strict variants' outputs within the bf16 bar of FP64."""
    from strict_topk_overlap_b200 import paged
    q, ks, vs, cache = _batch(seed=7)
    qd = q.to(DEV)
    ids = _oracle_ids(q, ks)
    lengths = [k.shape[1] for k in ks]
    p = _predicted(ids, lengths, 0.75, seed=3).to(DEV).contiguous()
    out, sel = paged.speculative_step(qd, cache, p, TOPK, variant=variant)
    a = paged.select_blocks(qd, cache, TOPK)
    if variant == "saved":
        ref = paged.repair_saved(qd, cache, a, p, paged.partials(qd, cache, p))
    else:
        pr = paged.speculate(qd, cache, p, mode="hybrid", mass_threshold=0.1, keep_mass=True)
        if variant == "repair_fused":
            ref = paged.repair_fused(qd, cache, a, p, pr).output
        else:
            ref = paged._repair(qd, cache, a, p, pr, 3)[0]
    torch.cuda.synchronize()
    assert np.array_equal(sel.cpu().numpy(), ids)
    assert (out - ref).abs().max().item() <= 1e-5
    assert _close(out, _oracle_out(q, ks, vs, ids))
