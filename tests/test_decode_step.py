"""The fused decode step (stk_decode_step: one persistent, cooperative launch
per step) against the CPU oracle and the launch-chain path it replaces.

Bars: selected block IDs bit-exact against the FP64 stable-sorted oracle
(ties to the lower index); outputs within the north-star bf16 bar
(|err| <= 2e-3 + 1e-2 |ref|) of the FP64 oracle over the strict set (fp16
inputs: the same bar); speculative and serial steps agree with the chained
launches (stk_speculative_step, gqa.exact) within 1e-5. Shapes cover config 1,
a config-0-sized request, ragged block counts (metadata items shorter than 16
blocks), the larger-request selection path (> 2048 blocks), wide groups
(8 query heads per KV head), predicted lists of other lengths than K, full
and zero overlap, repeated calls on one workspace (the control block must
come back to zero) and CUDA-graph replay with new inputs."""
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


def _bar(out, ref):
    err = np.abs(out.cpu().numpy() - ref)
    return bool((err <= 2e-3 + 1e-2 * np.abs(ref)).all()), float(err.max())


def _case(hq, hkv, n, topk, overlap, seed, dtype=torch.bfloat16, sp=None):
    """Seeded config-shaped inputs, the oracle's strict IDs and a predicted
    list (true Top-K with round((1 - overlap) * topk) IDs swapped), cut to
    its first ``sp`` entries when sp < topk."""
    q, k, v, lo, hi = C.synthetic_kv(hq, hkv, n, 32, 128, dtype, seed=seed)
    ids = OS.select_blocks(C.as_np(q), lo.numpy(), hi.numpy(), topk)
    p = C.swap_prediction(torch.from_numpy(ids), n, round((1 - overlap) * topk), seed=seed + 1)
    if sp is not None:
        p = p[:, :sp]
    return q, k, v, lo, hi, ids, p.to(torch.int32).contiguous()


SHAPES = [
    # hq, hkv, n, topk, overlap, sp
    (32, 8, 2048, 64, 0.9, None),   # config 1
    (32, 8, 2048, 64, 1.0, None),
    (32, 8, 2048, 64, 0.0, None),
    (8, 2, 128, 16, 0.75, None),    # config-0 sized
    (16, 8, 200, 16, 0.75, None),   # ragged: 200 blocks (last metadata item holds 8)
    (32, 8, 3000, 32, 0.9, None),   # > 2048 blocks
    (32, 4, 512, 48, 0.8, None),    # 8 query heads per KV head
    (16, 4, 1024, 64, 0.75, 40),    # shorter predicted list
]


@pytest.mark.parametrize("hq,hkv,n,topk,overlap,sp", SHAPES)
def test_fused_step_matches_oracle_and_chain(hq, hkv, n, topk, overlap, sp):
    from strict_topk import gqa
    from strict_topk_overlap_b200.decode import decode_step, speculative_step
    q, k, v, lo, hi, ids, p = _case(hq, hkv, n, topk, overlap, seed=n + hq, sp=sp)
    qd, kd, vd, lod, hid, pd = (t.to(DEV) for t in (q, k, v, lo, hi, p))
    ref = OA.attention_fp64(C.as_np(q), C.as_np(k), C.as_np(v), ids)
    out_s, sel_s = decode_step(qd, kd, vd, lod, hid, topk, pd)
    out_r, sel_r = decode_step(qd, kd, vd, lod, hid, topk, None)
    torch.cuda.synchronize()
    assert np.array_equal(sel_s.cpu().numpy(), ids), "speculative fused step: IDs"
    assert np.array_equal(sel_r.cpu().numpy(), ids), "serial fused step: IDs"
    for name, out in (("speculative", out_s), ("serial", out_r)):
        ok, err = _bar(out, ref)
        assert ok, (name, err)
    chain, _ = speculative_step(qd, kd, vd, lod, hid, pd, topk)
    exact = gqa.exact(qd, kd, vd, sel_r)
    torch.cuda.synchronize()
    assert (out_s - chain).abs().max().item() <= 1e-5
    assert (out_r - exact).abs().max().item() <= 1e-5


def test_fused_step_f16():
    from strict_topk_overlap_b200.decode import decode_step
    q, k, v, lo, hi, ids, p = _case(16, 4, 512, 32, 0.75, seed=5, dtype=torch.float16)
    qd, kd, vd, lod, hid, pd = (t.to(DEV) for t in (q, k, v, lo, hi, p))
    ref = OA.attention_fp64(C.as_np(q), C.as_np(k), C.as_np(v), ids)
    for pred in (pd, None):
        out, sel = decode_step(qd, kd, vd, lod, hid, 32, pred)
        torch.cuda.synchronize()
        assert np.array_equal(sel.cpu().numpy(), ids)
        ok, err = _bar(out, ref)
        assert ok, err


def test_fused_step_reuses_workspace_and_replays_in_graph():
    """Steps on one workspace in a row (the control block returns to zero
    after each), then a CUDA graph of the step replayed with new q and P
    copied into its static inputs."""
    from strict_topk_overlap_b200.decode import decode_step, decode_step_workspace
    hq, hkv, n, topk = 32, 8, 2048, 64
    q, k, v, lo, hi, ids, p = _case(hq, hkv, n, topk, 0.9, seed=11)
    qd, kd, vd, lod, hid, pd = (t.to(DEV) for t in (q, k, v, lo, hi, p))
    ws = decode_step_workspace(qd, kd, topk, pd)
    out = torch.empty((hq, 128), device=DEV)
    sel = torch.empty((hq, topk), device=DEV, dtype=torch.int32)
    for _ in range(3):
        decode_step(qd, kd, vd, lod, hid, topk, pd, out=out, selected=sel, workspace=ws)
    torch.cuda.synchronize()
    assert np.array_equal(sel.cpu().numpy(), ids)
    first = out.clone()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        decode_step(qd, kd, vd, lod, hid, topk, pd, out=out, selected=sel, workspace=ws)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, first)
    # New inputs through the captured graph: another query and prediction.
    q2 = C.synthetic_kv(hq, hkv, 1, 32, 128, torch.bfloat16, seed=77)[0]
    ids2 = OS.select_blocks(C.as_np(q2), lo.numpy(), hi.numpy(), topk)
    p2 = C.swap_prediction(torch.from_numpy(ids2), n, 16, seed=78)
    qd.copy_(q2.to(DEV))
    pd.copy_(p2.to(DEV))
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    assert np.array_equal(sel.cpu().numpy(), ids2)
    ok, err = _bar(out, OA.attention_fp64(C.as_np(q2), C.as_np(k), C.as_np(v), ids2))
    assert ok, err
    del g


def test_fused_step_rejects_shapes_outside_its_plan():
    from strict_topk_overlap_b200.decode import decode_step
    q, k, v, lo, hi = C.synthetic_kv(8, 2, 64, 16, 128, torch.bfloat16, seed=1)  # 16-token blocks
    qd, kd, vd, lod, hid = (t.to(DEV) for t in (q, k, v, lo, hi))
    assert decode_step(qd, kd, vd, lod, hid, 8, None, strict=False) is None
    with pytest.raises(RuntimeError, match="32-token blocks"):
        decode_step(qd, kd, vd, lod, hid, 8, None)


def test_decoder_uses_fused_step():
    """SpeculativeDecoder runs the saved method through the fused kernel
    where the shape fits, and the serial step through it on request (its
    default is the launch chain), with the same results."""
    from strict_topk_overlap_b200.decode import SpeculativeDecoder, StepSpec
    q, k, v, lo, hi, ids, p = _case(32, 8, 2048, 64, 0.75, seed=21)
    qd, kd, vd, lod, hid, pd = (t.to(DEV) for t in (q, k, v, lo, hi, p))
    spec = SpeculativeDecoder(qd, kd, vd, lod, hid, pd, StepSpec(topk=64))
    ser = SpeculativeDecoder(qd, kd, vd, lod, hid, pd, StepSpec(topk=64), serial=True, fused=True)
    chain = SpeculativeDecoder(qd, kd, vd, lod, hid, pd, StepSpec(topk=64), serial=True)
    assert spec.fused and ser.fused and not chain.fused
    o1, o2, o3 = spec.step().clone(), ser.step().clone(), chain.step().clone()
    torch.cuda.synchronize()
    for d in (spec, ser, chain):
        assert np.array_equal(d.selected.cpu().numpy(), ids)
    assert (o1 - o2).abs().max().item() <= 1e-5
    assert (o1 - o3).abs().max().item() <= 1e-5
    spec.close()
    ser.close()
    chain.close()


def test_capture_host_steps_copies_inputs_and_outputs():
    """capture_host_steps: one graph of several steps, each with its pinned
    host inputs copied in and its output copied out; new host inputs are
    picked up on replay and every step's output reaches its host buffer."""
    from strict_topk_overlap_b200.decode import SpeculativeDecoder, StepSpec, capture_host_steps
    decs, hq_pin, hp_pin, refs = [], [], [], []
    for seed in (31, 32):
        q, k, v, lo, hi, ids, p = _case(16, 4, 512, 32, 0.75, seed=seed)
        qd, kd, vd, lod, hid, pd = (t.to(DEV) for t in (q, k, v, lo, hi, p))
        decs.append(SpeculativeDecoder(torch.zeros_like(qd), kd, vd, lod, hid, torch.zeros_like(pd),
                                       StepSpec(topk=32), graph=False))
        hq_pin.append(q.pin_memory())
        hp_pin.append(p.pin_memory())
        refs.append(OA.attention_fp64(C.as_np(q), C.as_np(k), C.as_np(v), ids))
    # The first decoder again, with another query: its second step's input
    # copy must wait for its first step, and that step for its output copy.
    q0, k0, v0, lo0, hi0, _, p0 = _case(16, 4, 512, 32, 0.75, seed=31)
    q2 = torch.randn(16, 128, generator=torch.Generator().manual_seed(77)).to(q0.dtype)
    ids2 = OS.select_blocks(C.as_np(q2), lo0.numpy(), hi0.numpy(), 32)
    decs.append(decs[0])
    hq_pin.append(q2.pin_memory())
    hp_pin.append(p0.pin_memory())
    refs.append(OA.attention_fp64(C.as_np(q2), C.as_np(k0), C.as_np(v0), ids2))
    outs = [torch.empty(16, 128, dtype=torch.float32).pin_memory() for _ in decs]
    g = capture_host_steps(decs, hq_pin, hp_pin, outs)
    for _ in range(2):
        for o in outs:
            o.zero_()
        g.replay()
        torch.cuda.synchronize()
        for o, ref in zip(outs, refs):
            ok, err = _bar(o, ref)
            assert ok, err
    del g
