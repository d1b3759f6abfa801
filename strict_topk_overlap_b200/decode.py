"""Speculative decode-step orchestration: selector || speculation, then repair.

``overlap_run`` is the drop-in for the reference's two-stream harness
(benchmarks/run_benchmark.py:99-118): the selector runs on one side stream,
speculation over the predicted IDs on another, the caller's stream joins both
and runs the repair. ``speculative_step`` is the B200 form of the same step
for the saved method: one stream, one chain of programmatically dependent
launches (scorer -> Top-K -> predicted-block states -> repair) in which the
predicted K/V stream starts while Top-K runs and the repair needs no stream
join. ``SpeculativeDecoder`` packages one full decode step for fixed shapes
and captures it in a CUDA graph, so a step is one graph launch; ``serial``
steps run select -> attention on one stream with the same kernels, which is
the baseline the speculative path must beat.
"""
from __future__ import annotations

from dataclasses import dataclass

import ctypes as C

import torch

from . import _lib as L
from . import fused, gqa, gqa_light, kernels, signed_fused

# method -> (prediction mode, repair entry point)
METHODS = {
    "saved": ("saved", "gqa"),                  # gqa.partials + gqa.repair_saved
    "light": ("saved", "light"),                # gqa.partials + gqa_light.repair_saved_light
    "compact": ("compact", "fused"),            # compact speculation + repair_fused
    "repair_fused": ("hybrid", "fused"),        # hybrid speculation + repair_fused
    "signed_fused": ("hybrid", "signed_fused"), # hybrid speculation + repair_signed_fused
}


def overlap_run(selector, speculative, finish, select_stream, predict_stream):
    """Run selector() and speculative() concurrently, then finish(selected, state)
    (reference benchmarks/run_benchmark.py:99-118); the current stream waits
    for the result.

    The finish runs on the selector's stream, directly behind the Top-K
    kernel: the repair kernel is launched for programmatic dependent launch,
    so it starts while Top-K drains instead of paying a kernel-boundary gap
    (its dependency on the speculation stream stays an ordinary one)."""
    main = torch.cuda.current_stream()
    select_stream.wait_stream(main)
    predict_stream.wait_stream(main)
    with torch.cuda.stream(select_stream):
        a = selector()
    with torch.cuda.stream(predict_stream):
        state = speculative()

    def record(obj, stream):
        if isinstance(obj, torch.Tensor):
            obj.record_stream(stream)
        elif hasattr(obj, "__dict__"):
            for value in vars(obj).values():
                record(value, stream)
    with torch.cuda.stream(select_stream):
        select_stream.wait_stream(predict_stream)
        record(state, select_stream)
        out = finish(a, state)
    main.wait_stream(select_stream)
    record(out, main)
    a.record_stream(main)
    return out


def speculative_step(q, k, v, lo, hi, predicted, topk, *, out=None, selected=None, workspace=None):
    """One saved-method speculative step on the current stream in one launch
    chain (stk_speculative_step): returns (output FP32 [Hq, D], selected
    int32 [Hq, topk]). Equal to gqa.select_blocks, gqa.partials and
    gqa.repair_saved in sequence."""
    hq, d = q.shape
    hkv, n, b, _ = k.shape
    sp = predicted.shape[1]
    lib = L.load()
    if out is None:
        out = torch.empty((hq, d), device=q.device, dtype=torch.float32)
    if selected is None:
        selected = torch.empty((hq, topk), device=q.device, dtype=torch.int32)
    need = lib.stk_speculative_step_workspace_bytes(hq, n, sp, d)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty((need,), device=q.device, dtype=torch.uint8)
    kv = L.kv_struct(k, v)
    rc = lib.stk_speculative_step(C.byref(kv), q.data_ptr(), L.dtype_code(q), lo.data_ptr(), hi.data_ptr(), hq, topk,
                                  predicted.data_ptr(), L.id_is64(predicted), sp, selected.data_ptr(), out.data_ptr(),
                                  workspace.data_ptr(), need, L.status_ptr(), L.stream_of(q))
    L.check(rc, "speculative_step")
    return out, selected


def speculative_step_hybrid(q, k, v, lo, hi, predicted, topk, *, variant="repair_fused", mass_threshold=0.1,
                            min_remaining=1e-3, cancellation_tol=1e-5, max_extra_mass=0.0, out=None, selected=None,
                            workspace=None):
    """One hybrid-method speculative step on the current stream in one launch
    chain (stk_speculative_step_hybrid): returns (output FP32 [Hq, D],
    selected int32 [Hq, topk]). ``variant`` "repair_fused" equals
    gqa.select_blocks, kernels.speculate(mode='hybrid', keep_mass=True) and
    fused.repair_fused in sequence; "signed_fused" ends with
    signed_fused.repair_signed_fused instead."""
    hq, d = q.shape
    hkv, n, b, _ = k.shape
    sp = predicted.shape[1]
    var = {"repair_fused": L.VAR_FUSED, "signed_fused": L.VAR_SIGNED_FUSED}[variant]
    lib = L.load()
    if out is None:
        out = torch.empty((hq, d), device=q.device, dtype=torch.float32)
    if selected is None:
        selected = torch.empty((hq, topk), device=q.device, dtype=torch.int32)
    need = lib.stk_speculative_step_hybrid_workspace_bytes(hq, n, sp, d)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty((need,), device=q.device, dtype=torch.uint8)
    kv = L.kv_struct(k, v)
    res = L.StkRepairOut(out.data_ptr(), None, None, None, None, None, None)
    rc = lib.stk_speculative_step_hybrid(
        C.byref(kv), q.data_ptr(), L.dtype_code(q), lo.data_ptr(), hi.data_ptr(), hq, topk, predicted.data_ptr(),
        L.id_is64(predicted), sp, float(mass_threshold), var, float(min_remaining), float(cancellation_tol),
        float(max_extra_mass), selected.data_ptr(), C.byref(res), workspace.data_ptr(), need, L.status_ptr(),
        L.stream_of(q))
    L.check(rc, "speculative_step_hybrid")
    return out, selected


STK_ESMEM = -2


def decode_step_workspace(q, k, topk, predicted=None):
    """A zeroed workspace for ``decode_step`` (its control block, score slots
    and tags must start at zero; every call leaves them zero again)."""
    slots = predicted.shape[1] if predicted is not None else topk
    need = L.load().stk_decode_step_workspace_bytes(q.shape[0], k.shape[0], k.shape[1], slots, q.shape[1])
    return torch.zeros((max(need, 1),), device=q.device, dtype=torch.uint8)


def decode_step(q, k, v, lo, hi, topk, predicted=None, *, out=None, selected=None, workspace=None, strict=True):
    """One decode step as one persistent, cooperative launch (stk_decode_step).

    With ``predicted`` [Hq, P]: the speculative saved step — equal to
    gqa.select_blocks, gqa.partials and gqa.repair_saved in sequence (and to
    ``speculative_step``). Without it: the serial step, equal to
    gqa.exact(q, k, v, gqa.select_blocks(q, lo, hi, topk)). Returns (output
    FP32 [Hq, D], selected int32 [Hq, topk]). ``workspace`` must come from
    ``decode_step_workspace`` (zeroed) or have been used by an earlier call
    of the same shape. Shapes outside the fused kernel's plan (see
    stk_decode_step) raise RuntimeError, or return None with strict=False."""
    hq, d = q.shape
    hkv, n, b, _ = k.shape
    sp = predicted.shape[1] if predicted is not None else 0
    lib = L.load()
    if out is None:
        out = torch.empty((hq, d), device=q.device, dtype=torch.float32)
    if selected is None:
        selected = torch.empty((hq, topk), device=q.device, dtype=torch.int32)
    if workspace is None:
        workspace = decode_step_workspace(q, k, topk, predicted)
    kv = L.kv_struct(k, v)
    rc = lib.stk_decode_step(C.byref(kv), q.data_ptr(), L.dtype_code(q), lo.data_ptr(), hi.data_ptr(), hq, topk,
                             L.ptr(predicted), L.id_is64(predicted) if predicted is not None else 0, sp,
                             selected.data_ptr(), out.data_ptr(), workspace.data_ptr(), workspace.numel(),
                             L.status_ptr(), L.stream_of(q))
    if rc == STK_ESMEM and not strict:
        return None
    L.check(rc, "decode_step")
    return out, selected


@dataclass
class StepSpec:
    """One decode step's configuration."""
    topk: int
    method: str = "saved"
    mass_threshold: float = 0.1
    max_extra_mass: float = 0.0
    min_remaining: float = 1e-3
    cancellation_tol: float = 1e-5


def _speculate_fn(spec, q, k, v, p):
    mode, _ = METHODS[spec.method]
    if mode == "saved":
        return lambda: gqa.partials(q, k, v, p)
    keep = spec.max_extra_mass > 0
    return lambda: kernels.speculate(q, k, v, p, mode=mode, mass_threshold=spec.mass_threshold, keep_mass=keep)


def _finish_fn(spec, q, k, v, p):
    _, rep = METHODS[spec.method]
    if rep == "gqa":
        return lambda a, st: gqa.repair_saved(q, k, v, a, p, st)
    if rep == "light":
        return lambda a, st: gqa_light.repair_saved_light(q, k, v, a, p, st)
    if rep == "fused":
        return lambda a, pred: fused.repair_fused(q, k, v, a, p, pred, spec.min_remaining, spec.cancellation_tol,
                                                  spec.max_extra_mass).output
    return lambda a, pred: signed_fused.repair_signed_fused(q, k, v, a, p, pred, spec.min_remaining,
                                                            spec.cancellation_tol, spec.max_extra_mass).output


class SpeculativeDecoder:
    """One speculative decode step over a fixed KV cache and static input
    buffers ``q`` [Hq, D] and ``predicted`` [Hq, P] (copy new values into
    them between steps). ``step()`` returns the FP32 output buffer [Hq, D];
    ``selected`` holds the step's strict Top-K IDs.

    With ``graph=True`` the whole step (both concurrent branches and the
    repair) is captured once and replayed as one CUDA-graph launch."""

    def __init__(self, q, k, v, lo, hi, predicted, spec: StepSpec, *, graph: bool = True, serial: bool = False,
                 chained: bool = True, fused: bool | None = None):
        self.q, self.k, self.v, self.lo, self.hi, self.predicted = q, k, v, lo, hi, predicted
        self.spec = spec
        self.serial = serial
        # The saved method runs as one persistent launch (decode_step) where
        # the shape fits its plan. The serial step takes the launch chain by
        # default (selection, then exact attention: measured faster than the
        # fused serial launch at config 1); fused=True asks for the fused one.
        if fused is None:
            fused = not serial
        self.fused = fused and (serial or spec.method in ("saved", "light"))
        self._fws = decode_step_workspace(q, k, spec.topk, None if serial else predicted) if self.fused else None
        # The saved and hybrid (repair_fused, signed_fused) methods run as one
        # launch chain on one stream; compact (and chained=False) uses the
        # two-stream harness.
        self.chained = chained and spec.method in ("saved", "light", "repair_fused", "signed_fused")
        self._ws = None
        if self.chained:
            ws_fn = (L.load().stk_speculative_step_workspace_bytes if spec.method in ("saved", "light")
                     else L.load().stk_speculative_step_hybrid_workspace_bytes)
            need = ws_fn(q.shape[0], k.shape[1], predicted.shape[1], q.shape[1])
            self._ws = torch.empty((need,), device=q.device, dtype=torch.uint8)
        # The selector is the critical path (score -> Top-K -> repair): its
        # stream gets the higher priority when both branches want SMs.
        self._sel_stream = torch.cuda.Stream(q.device, priority=-1)
        self._pred_stream = torch.cuda.Stream(q.device)
        self._selector = lambda: gqa.select_blocks(q, lo, hi, spec.topk)
        self._spec = _speculate_fn(spec, q, k, v, predicted)
        self._finish = _finish_fn(spec, q, k, v, predicted)
        self.graph = None
        self.host_graph = None
        self.out = None
        self.selected = None
        if graph:
            self._capture()

    def _run(self):
        if self.fused:
            res = decode_step(self.q, self.k, self.v, self.lo, self.hi, self.spec.topk,
                              None if self.serial else self.predicted, workspace=self._fws, strict=False)
            if res is not None:
                return res
            self.fused = False  # outside the fused kernel's plan: the launch chains below
        if self.serial:
            a = self._selector()
            return gqa.exact(self.q, self.k, self.v, a), a
        if self.chained and self.spec.method in ("repair_fused", "signed_fused"):
            sp = self.spec
            return speculative_step_hybrid(self.q, self.k, self.v, self.lo, self.hi, self.predicted, sp.topk,
                                           variant=sp.method, mass_threshold=sp.mass_threshold,
                                           min_remaining=sp.min_remaining, cancellation_tol=sp.cancellation_tol,
                                           max_extra_mass=sp.max_extra_mass, workspace=self._ws)
        if self.chained:
            return speculative_step(self.q, self.k, self.v, self.lo, self.hi, self.predicted, self.spec.topk,
                                    workspace=self._ws)
        sel_box = {}

        def finish(a, st):
            sel_box["a"] = a
            return self._finish(a, st)
        out = overlap_run(self._selector, self._spec, finish, self._sel_stream, self._pred_stream)
        return out, sel_box["a"]

    def _capture(self):
        side = torch.cuda.Stream(self.q.device)
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(2):
                self._run()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize(self.q.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out, self.selected = self._run()

    def step(self):
        if self.graph is not None:
            self.graph.replay()
            return self.out
        self.out, self.selected = self._run()
        return self.out

    def bind_host(self, q_host, predicted_host, out_host):
        """Capture the step together with its host I/O: copies of ``q_host``
        and ``predicted_host`` (pinned host tensors shaped like ``q`` and
        ``predicted``) into the device inputs, the step, and a copy of the
        output into the pinned ``out_host``, as one CUDA graph that
        ``step_host()`` replays. The copies are stream-ordered; the host
        reads ``out_host`` after synchronising with the stream (or an event
        recorded after ``step_host()``)."""
        for t, want in ((q_host, self.q), (predicted_host, self.predicted)):
            if t.shape != want.shape or t.dtype != want.dtype or t.is_cuda or not t.is_pinned():
                raise ValueError("host inputs must be pinned CPU tensors shaped like the device inputs")
        if out_host.is_cuda or not out_host.is_pinned() or out_host.dtype != torch.float32 or \
                out_host.shape != (self.q.shape[0], self.q.shape[1]):
            raise ValueError("out_host must be a pinned FP32 CPU tensor [Hq, D]")

        def run():
            self.q.copy_(q_host, non_blocking=True)
            self.predicted.copy_(predicted_host, non_blocking=True)
            out, sel = self._run()
            out_host.copy_(out, non_blocking=True)
            return out, sel
        side = torch.cuda.Stream(self.q.device)
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            run()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize(self.q.device)
        self.host_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.host_graph):
            self.host_out, self.host_selected = run()

    def step_host(self):
        """Replay the graph captured by ``bind_host``."""
        self.host_graph.replay()

    def close(self):
        self.graph = None
        self.host_graph = None


def capture_steps(decoders):
    """One CUDA graph that runs one decode step of every decoder in turn (for
    example the attention of consecutive layers of one token step, which a
    model replays as one graph). Returns (graph, outputs, selections): the
    buffers this graph writes, one per decoder. The decoders' own single-step
    graphs and buffers are left as they were."""
    dev = decoders[0].q.device
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            for d in decoders:
                d._run()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    outs, sels = [], []
    with torch.cuda.graph(graph):
        for d in decoders:
            out, sel = d._run()
            outs.append(out)
            sels.append(sel)
    return graph, outs, sels

def capture_host_steps(decoders, q_hosts, predicted_hosts, out_hosts):
    """One CUDA graph that runs, for every decoder in turn, the copy of its
    pinned host inputs (``q_hosts[i]``, ``predicted_hosts[i]``, shaped like
    its ``q`` and ``predicted``) into its device inputs, its decode step and
    the copy of the step's output into the pinned ``out_hosts[i]`` (FP32
    [Hq, D]): the host-facing form of ``capture_steps``. The host reads
    ``out_hosts`` after synchronising with the stream (or an event recorded
    after the replay).

    The copies run on two side streams inside the graph: step i's inputs
    only have to land before step i starts and its output copy only waits
    for step i, so the copies of the other steps overlap the decode steps.
    A decoder listed twice gets the extra orderings its shared buffers need
    (its next input copy waits for its previous step, its next step for its
    previous output copy)."""
    for d, qh, ph, oh in zip(decoders, q_hosts, predicted_hosts, out_hosts):
        for t, want in ((qh, d.q), (ph, d.predicted)):
            if t.shape != want.shape or t.dtype != want.dtype or t.is_cuda or not t.is_pinned():
                raise ValueError("host inputs must be pinned CPU tensors shaped like the device inputs")
        if oh.is_cuda or not oh.is_pinned() or oh.dtype != torch.float32 or oh.shape != (d.q.shape[0], d.q.shape[1]):
            raise ValueError("out_hosts must be pinned FP32 CPU tensors [Hq, D]")
    dev = decoders[0].q.device
    copy_in = torch.cuda.Stream(dev)
    copy_out = torch.cuda.Stream(dev)

    def run():
        main = torch.cuda.current_stream(dev)
        copy_in.wait_stream(main)
        copy_out.wait_stream(main)
        last_step, last_out = {}, {}  # per decoder: events of its latest step / output copy
        for d, qh, ph, oh in zip(decoders, q_hosts, predicted_hosts, out_hosts):
            key = id(d)
            landed = torch.cuda.Event()
            with torch.cuda.stream(copy_in):
                if key in last_step:
                    copy_in.wait_event(last_step[key])
                d.q.copy_(qh, non_blocking=True)
                d.predicted.copy_(ph, non_blocking=True)
                landed.record(copy_in)
            main.wait_event(landed)
            if key in last_out:
                main.wait_event(last_out[key])
            out, _ = d._run()
            stepped = torch.cuda.Event()
            stepped.record(main)
            last_step[key] = stepped
            copied = torch.cuda.Event()
            with torch.cuda.stream(copy_out):
                copy_out.wait_event(stepped)
                oh.copy_(out, non_blocking=True)
                copied.record(copy_out)
            last_out[key] = copied
        main.wait_stream(copy_in)
        main.wait_stream(copy_out)

    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        run()
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        run()
    return graph
