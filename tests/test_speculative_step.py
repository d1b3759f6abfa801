"""The one-stream speculative step (stk_speculative_step: scorer -> Top-K ->
predicted-block states launched behind Top-K -> saved repair) against the
same kernels called one by one (gqa.select_blocks, gqa.partials,
gqa.repair_saved) and against the FP64 oracle, at BASELINE config 1 and at a
small shape, across prediction overlaps, eagerly and replayed from a CUDA
graph with new inputs copied in between; and the hybrid methods' chained
step (stk_speculative_step_hybrid) against speculate(mode='hybrid') plus the
fused / signed fused repair called one by one."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import cases as C
from oracle import attention as OA
from oracle import selection as OS

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def status_word():
    import strict_topk_overlap_b200._lib as L
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    L.set_status_tensor(st)
    yield st
    torch.cuda.synchronize()
    L.set_status_tensor(None)
    assert st.item() == 0, f"device status {st.item()}"


def _case(hq, hkv, n, b, d, topk, overlap, seed, dtype=torch.bfloat16):
    q, k, v, lo, hi = C.synthetic_kv(hq, hkv, n, b, d, dtype, seed=seed)
    ids = OS.select_blocks(C.as_np(q), lo.numpy(), hi.numpy(), topk)
    p = C.swap_prediction(torch.from_numpy(ids), n, int(round((1 - overlap) * topk)), seed)
    return [t.to(DEV) for t in (q, k, v, lo, hi, p.to(torch.int32))], ids


@pytest.mark.parametrize("shape", [(8, 2, 96, 16, 64, 12), (32, 8, 2048, 32, 128, 64)])
@pytest.mark.parametrize("overlap", [1.0, 0.75, 0.5])
def test_step_equals_separate_calls(shape, overlap):
    from strict_topk import gqa
    from strict_topk_overlap_b200.decode import speculative_step
    hq, hkv, n, b, d, topk = shape
    (q, k, v, lo, hi, p), ids = _case(hq, hkv, n, b, d, topk, overlap, seed=int(overlap * 10) + n)
    out, sel = speculative_step(q, k, v, lo, hi, p, topk)
    a = gqa.select_blocks(q, lo, hi, topk)
    st = gqa.partials(q, k, v, p)
    ref = gqa.repair_saved(q, k, v, a, p, st)
    torch.cuda.synchronize()
    assert torch.equal(sel, a)
    assert np.array_equal(sel.cpu().numpy(), ids)
    assert torch.equal(out, ref)
    want = OA.attention_fp64(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(), ids)
    assert (np.abs(out.cpu().numpy() - want) <= 2e-3 + 1e-2 * np.abs(want)).all()


def test_step_in_graph_with_new_inputs():
    from strict_topk_overlap_b200.decode import SpeculativeDecoder, StepSpec
    hq, hkv, n, b, d, topk = 16, 4, 256, 32, 128, 16
    cases = [_case(hq, hkv, n, b, d, topk, 0.75, seed=s) for s in range(3)]
    (q0, k, v, lo, hi, p0), _ = cases[0]
    q_buf, p_buf = q0.clone(), p0.clone()
    dec = SpeculativeDecoder(q_buf, k, v, lo, hi, p_buf, StepSpec(topk=topk, method="saved"))
    assert dec.chained and dec.graph is not None
    for s in range(3):
        # Same K/V cache, new query and prediction each step.
        qs = C.synthetic_kv(hq, hkv, n, b, d, torch.bfloat16, seed=50 + s)[0].to(DEV)
        ids = OS.select_blocks(C.as_np(qs.cpu()), lo.cpu().numpy(), hi.cpu().numpy(), topk)
        ps = C.swap_prediction(torch.from_numpy(ids), n, 4, 70 + s).to(torch.int32).to(DEV)
        q_buf.copy_(qs)
        p_buf.copy_(ps)
        out = dec.step()
        torch.cuda.synchronize()
        assert np.array_equal(dec.selected.cpu().numpy(), ids)
        want = OA.attention_fp64(qs.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(), ids)
        assert (np.abs(out.cpu().numpy() - want) <= 2e-3 + 1e-2 * np.abs(want)).all()
    dec.close()


@pytest.mark.parametrize("variant", ["repair_fused", "signed_fused"])
@pytest.mark.parametrize("shape", [(8, 2, 96, 16, 64, 12), (32, 8, 2048, 32, 128, 64)])
@pytest.mark.parametrize("overlap,eps", [(1.0, 0.0), (0.75, 0.0), (0.75, 0.01)])
def test_hybrid_step_equals_separate_calls(variant, shape, overlap, eps):
    """stk_speculative_step_hybrid against gqa.select_blocks,
    kernels.speculate(mode='hybrid', keep_mass=True) and the fused / signed
    fused repair called one by one: same IDs, same output bits; strict mode
    also against the FP64 oracle."""
    from strict_topk import fused, gqa, kernels, signed_fused
    from strict_topk_overlap_b200.decode import speculative_step_hybrid
    hq, hkv, n, b, d, topk = shape
    (q, k, v, lo, hi, p), ids = _case(hq, hkv, n, b, d, topk, overlap, seed=int(overlap * 10) + n + 3)
    out, sel = speculative_step_hybrid(q, k, v, lo, hi, p, topk, variant=variant, max_extra_mass=eps)
    a = gqa.select_blocks(q, lo, hi, topk)
    pred = kernels.speculate(q, k, v, p, mode="hybrid", mass_threshold=0.1, keep_mass=True)
    rep = fused.repair_fused if variant == "repair_fused" else signed_fused.repair_signed_fused
    ref = rep(q, k, v, a, p, pred, 1e-3, 1e-5, eps).output
    torch.cuda.synchronize()
    assert torch.equal(sel, a)
    assert np.array_equal(sel.cpu().numpy(), ids)
    assert torch.equal(out, ref)
    if eps == 0.0:
        want = OA.attention_fp64(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(), ids)
        assert (np.abs(out.cpu().numpy() - want) <= 2e-3 + 1e-2 * np.abs(want)).all()


def test_hybrid_step_in_graph_with_new_inputs():
    from strict_topk_overlap_b200.decode import SpeculativeDecoder, StepSpec
    hq, hkv, n, b, d, topk = 16, 4, 256, 32, 128, 16
    (q0, k, v, lo, hi, p0), _ = _case(hq, hkv, n, b, d, topk, 0.75, seed=0)
    q_buf, p_buf = q0.clone(), p0.clone()
    dec = SpeculativeDecoder(q_buf, k, v, lo, hi, p_buf, StepSpec(topk=topk, method="repair_fused"))
    assert dec.chained and dec.graph is not None
    for s in range(3):
        qs = C.synthetic_kv(hq, hkv, n, b, d, torch.bfloat16, seed=80 + s)[0].to(DEV)
        ids = OS.select_blocks(C.as_np(qs.cpu()), lo.cpu().numpy(), hi.cpu().numpy(), topk)
        ps = C.swap_prediction(torch.from_numpy(ids), n, 4, 90 + s).to(torch.int32).to(DEV)
        q_buf.copy_(qs)
        p_buf.copy_(ps)
        out = dec.step()
        torch.cuda.synchronize()
        assert np.array_equal(dec.selected.cpu().numpy(), ids)
        want = OA.attention_fp64(qs.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(), ids)
        assert (np.abs(out.cpu().numpy() - want) <= 2e-3 + 1e-2 * np.abs(want)).all()
    dec.close()
