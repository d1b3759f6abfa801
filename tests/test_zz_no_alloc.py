"""stk_select_topk_static: strict Top-K selection for callers that cannot
allocate device memory (a decode loop that must not call cudaMalloc, or a
plugin host that only passes inputs and outputs). Its FP64 scores live in the
library's own static device array instead of a caller workspace.

Called through the C ABI and checked against stk_select_topk with a
caller-provided workspace: block IDs and order keys must be bit-identical
(the bar for every selection test here), on two calls in a row with
different inputs, since every call shares the one array and finds the
previous call's scores in it. This file is named to be collected last."""
from __future__ import annotations

import ctypes as C

import pytest
import torch

import cases

pytestmark = pytest.mark.gpu

STK_EWS = -4


def _select(lib, q, lo, hi, topk, group_select, static):
    from strict_topk_overlap_b200 import _lib as L
    hq, d = q.shape
    hm, n, _ = lo.shape
    rows = hm if group_select else hq
    ids = torch.full((rows, topk), -1, device=q.device, dtype=torch.int32)
    keys = torch.zeros((rows, topk), device=q.device, dtype=torch.int64)
    stream = torch.cuda.current_stream(q.device).cuda_stream
    if static:
        rc = lib.stk_select_topk_static(q.data_ptr(), L.dtype_code(q), lo.data_ptr(), hi.data_ptr(), 1, hq, hm, n,
                                        None, n, n, d, topk, int(group_select), 0, ids.data_ptr(), keys.data_ptr(),
                                        None, stream)
    else:
        ws_bytes = lib.stk_select_workspace_bytes(rows, n)
        ws = torch.empty((ws_bytes,), device=q.device, dtype=torch.uint8)
        rc = lib.stk_select_topk(q.data_ptr(), L.dtype_code(q), lo.data_ptr(), hi.data_ptr(), 1, hq, hm, n, None, n,
                                 n, d, topk, int(group_select), 0, ids.data_ptr(), keys.data_ptr(), ws.data_ptr(),
                                 ws_bytes, None, stream)
    assert rc == 0, lib.stk_last_error().decode()
    return ids, keys


@pytest.mark.parametrize("group_select", [False, True])
def test_static_select_matches_workspace_select(group_select):
    from strict_topk_overlap_b200 import _lib as L
    lib = L.load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    # BASELINE config 1 shapes (32 query / 8 KV heads, 2048 blocks, K = 64), two seeds back to back.
    for seed in (0, 1):
        q, k, v, lo, hi = cases.synthetic_kv(32, 8, 2048, 32, 128, torch.bfloat16, seed=seed)
        qd, lod, hid = q.to(dev), lo.to(dev), hi.to(dev)
        want_ids, want_keys = _select(lib, qd, lod, hid, 64, group_select, static=False)
        got_ids, got_keys = _select(lib, qd, lod, hid, 64, group_select, static=True)
        torch.cuda.synchronize()
        assert torch.equal(got_ids.cpu(), want_ids.cpu()), f"seed {seed}: IDs differ"
        assert torch.equal(got_keys.cpu(), want_keys.cpu()), f"seed {seed}: order keys differ"
        assert int(got_ids.min()) >= 0


def test_static_select_allocates_nothing():
    """After the first call (which looks up the array's address), further
    calls leave the device's free memory unchanged: the library allocates
    nothing for them. Outputs are allocated before the measurement."""
    from strict_topk_overlap_b200 import _lib as L
    lib = L.load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    q, k, v, lo, hi = cases.synthetic_kv(32, 8, 2048, 32, 128, torch.bfloat16, seed=3)
    qd, lod, hid = q.to(dev), lo.to(dev), hi.to(dev)
    ids = torch.empty((32, 64), device=dev, dtype=torch.int32)
    stream = torch.cuda.current_stream(dev).cuda_stream

    def call():
        rc = lib.stk_select_topk_static(qd.data_ptr(), L.dtype_code(qd), lod.data_ptr(), hid.data_ptr(), 1, 32, 8,
                                        2048, None, 2048, 2048, 128, 64, 0, 0, ids.data_ptr(), None, None, stream)
        assert rc == 0, lib.stk_last_error().decode()

    call()
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info(dev)
    for _ in range(2):
        call()
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info(dev)
    assert free_after == free_before, (free_before, free_after)


def test_static_select_rejects_oversize():
    from strict_topk_overlap_b200 import _lib as L
    lib = L.load()
    cap = 1 << 20
    q = torch.zeros((8, 128), device="cuda", dtype=torch.float32)
    ids = torch.empty((8, 4), device="cuda", dtype=torch.int32)
    n = cap // 8 + 1  # 8 rows x n blocks is one score slot over the capacity
    rc = lib.stk_select_topk_static(q.data_ptr(), 0, C.c_void_p(q.data_ptr()), C.c_void_p(q.data_ptr()), 1, 8, 8,
                                    n, None, n, n, 128, 4, 0, 0, ids.data_ptr(), None, None,
                                    torch.cuda.current_stream().cuda_stream)
    assert rc == STK_EWS
    assert b"static scratch" in lib.stk_last_error()
