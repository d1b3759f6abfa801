"""Failure detection without a GPU fault: a bounded device wait that runs out.

Every bulk-copy wait in the library's kernels gives up after a runtime limit
(stk_set_wait_limit_ns, default 2 s), records STK_STATUS_WAIT_TIMEOUT in the
call's status word, drains its barrier (bounded as well) and returns, so the
context stays usable. stk_check_wait_timeout waits on a barrier armed for bytes
that no copy delivers; with a 1 ms limit it must return promptly and leave
status 1. Afterwards, with the default limit back, the library's kernels still
run and give correct results (the context survived). No trap, fault or
unbounded loop is involved."""
from __future__ import annotations

import time

import numpy as np
import pytest
import torch

import cases as C
from oracle import selection as OS

pytestmark = pytest.mark.gpu

STATUS_WAIT_TIMEOUT = 1
DEFAULT_NS = 2_000_000_000


def test_wait_runs_out_and_reports_status():
    from strict_topk_overlap_b200 import _lib as L
    lib = L.load()
    torch.cuda.set_device(0)
    torch.cuda.synchronize()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert lib.stk_set_wait_limit_ns(1_000_000) == 0, lib.stk_last_error()
    try:
        t0 = time.perf_counter()
        rc = lib.stk_check_wait_timeout(status.data_ptr(), torch.cuda.current_stream().cuda_stream)
        assert rc == 0, lib.stk_last_error()
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
    finally:
        torch.cuda.synchronize()
        assert lib.stk_set_wait_limit_ns(DEFAULT_NS) == 0, lib.stk_last_error()
    assert status.item() == STATUS_WAIT_TIMEOUT
    assert elapsed < 1.0, elapsed  # two 1 ms waits, not the 2 s default
    # The context is intact: a selection after the timeout is exact.
    q, k, v, lo, hi = C.synthetic_kv(8, 2, 256, 32, 128, torch.bfloat16, seed=9)
    from strict_topk import gqa
    ok_status = torch.zeros(1, dtype=torch.int32, device="cuda")
    L.set_status_tensor(ok_status)
    try:
        ids = gqa.select_blocks(q.cuda(), lo.cuda(), hi.cuda(), 16)
        torch.cuda.synchronize()
    finally:
        L.set_status_tensor(None)
    assert ok_status.item() == 0
    assert np.array_equal(ids.cpu().numpy(), OS.select_blocks(C.as_np(q), lo.numpy(), hi.numpy(), 16))


def test_default_limit_does_not_fire():
    """With the default limit a wait that completes never records a timeout."""
    from strict_topk_overlap_b200 import _lib as L
    from strict_topk import gqa
    q, k, v, lo, hi = C.synthetic_kv(8, 2, 256, 32, 128, torch.bfloat16, seed=10)
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    L.set_status_tensor(st)
    try:
        a = gqa.select_blocks(qd, lo.cuda(), hi.cuda(), 16)
        gqa.exact(qd, kd, vd, a)
        torch.cuda.synchronize()
    finally:
        L.set_status_tensor(None)
    assert st.item() == 0
