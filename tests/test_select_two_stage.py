"""Two-stage strict Top-K (FP32 score intervals, exact FP64 scores only for
the blocks that straddle the K-th boundary) against the FP64 fixed-order
oracle, on inputs built to defeat the intervals: one-ulp near-ties,
duplicated blocks (exact ties, so every block straddles), infinite
metadata, per-KV-group selection at the wide-GQA size, head dims 64 / 128 /
256, and batches of requests shorter than one scorer tile. The bar is the
same as everywhere: block IDs bit-exact, ties to the lower index."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import cases as C
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


def _select(q, lo, hi, k, shared=False, keys=False):
    from strict_topk_overlap_b200 import selector
    rows = lo.shape[0] if shared else q.shape[0]
    ko = torch.empty((rows, k), dtype=torch.int64, device=DEV) if keys else None
    ids = selector.topk_from_metadata(q.to(DEV), lo.to(DEV), hi.to(DEV), k, group_select=shared,
                                      keys_out=None if ko is None else ko.view(torch.int64))
    torch.cuda.synchronize()
    return ids.cpu().numpy(), (None if ko is None else ko.cpu().numpy().view(np.uint64))


def _want(q, lo, hi, k, shared=False):
    """Oracle IDs, one row per selection row (a KV head when shared)."""
    ids = OS.select_blocks(C.as_np(q), lo.numpy(), hi.numpy(), k, shared=shared)
    return ids[:: q.shape[0] // lo.shape[0]] if shared else ids


def _near_tie_metadata(hkv, n, d, seed):
    """Blocks in pairs whose second member differs from the first in one
    dimension by one FP32 ulp (or not at all): FP64 scores that differ in
    their last bits or tie exactly."""
    g = torch.Generator().manual_seed(seed)
    base = torch.randn(hkv, n // 2, d, generator=g)
    lo = base.repeat_interleave(2, dim=1).clone()
    hi = (lo + torch.rand(hkv, n, d, generator=g)).clone()
    lo_np, hi_np = lo.numpy(), hi.numpy()
    hi[:, 1::2] = hi[:, 0::2]
    rng = np.random.default_rng(seed)
    for h in range(hkv):
        for j in range(1, n, 2):
            dd = rng.integers(d)
            step = rng.integers(-1, 2)
            if step:
                hi_np[h, j, dd] = np.nextafter(hi_np[h, j, dd], np.float32(np.inf * step))
                lo_np[h, j, dd] = min(lo_np[h, j, dd], hi_np[h, j, dd])
    return torch.from_numpy(lo_np), torch.from_numpy(hi_np)


@pytest.mark.parametrize("d", [64, 128, 256])
def test_near_ties_bit_exact(d):
    hq, hkv, n = 8, 2, 512
    lo, hi = _near_tie_metadata(hkv, n, d, seed=d)
    q = torch.randn(hq, d, generator=torch.Generator().manual_seed(d + 1)).to(torch.bfloat16)
    for k in (1, 7, 64, 255, 511):
        assert np.array_equal(_select(q, lo, hi, k)[0], _want(q, lo, hi, k)), k
        assert np.array_equal(_select(q, lo, hi, k, shared=True)[0], _want(q, lo, hi, k, shared=True)), k


@pytest.mark.parametrize("hq", [24, 32])
def test_near_ties_wide_group_selection(hq):
    """Group selection with 12 and 16 query heads per KV head (the group
    scorer's one dot product with the summed positive and negative q parts)
    on near-tie metadata: IDs bit-exact."""
    hkv, n, d = 2, 512, 128
    lo, hi = _near_tie_metadata(hkv, n, d, seed=hq)
    q = torch.randn(hq, d, generator=torch.Generator().manual_seed(hq + 1)).to(torch.bfloat16)
    for k in (1, 7, 64, 255, 511):
        assert np.array_equal(_select(q, lo, hi, k, shared=True)[0], _want(q, lo, hi, k, shared=True)), k


def test_duplicated_blocks_take_the_lower_index():
    """Every block repeats one of 7: whole classes tie exactly and straddle
    the boundary (more than the ranked list holds)."""
    hq, hkv, n, d = 4, 2, 2000, 128
    q, _, _, lo, hi = C.synthetic_kv(hq, hkv, n, 4, d, torch.float32, seed=3)
    idx = torch.arange(n) % 7
    lo, hi = lo[:, idx].contiguous(), hi[:, idx].contiguous()
    for k in (5, 300, 1000, 1999):
        assert np.array_equal(_select(q, lo, hi, k)[0], _want(q, lo, hi, k)), k
        assert np.array_equal(_select(q, lo, hi, k, shared=True)[0], _want(q, lo, hi, k, shared=True)), k


def test_keys_out_are_exact_order_keys():
    hq, hkv, n, d, k = 16, 4, 1500, 128, 40
    q, _, _, lo, hi = C.synthetic_kv(hq, hkv, n, 4, d, torch.bfloat16, seed=5)
    ids, keys = _select(q, lo, hi, k, keys=True)
    scores = OS.bound_scores_fp64(C.as_np(q), lo.numpy(), hi.numpy())
    assert np.array_equal(ids, OS.stable_topk(scores, k))
    assert np.array_equal(keys, OS.order_keys(np.take_along_axis(scores, ids.astype(np.int64), axis=1)))
    ids, keys = _select(q, lo, hi, k, shared=True, keys=True)
    grp = OS.group_scores_fp64(scores, hq // hkv)
    assert np.array_equal(ids, OS.stable_topk(grp, k))
    assert np.array_equal(keys, OS.order_keys(np.take_along_axis(grp, ids.astype(np.int64), axis=1)))


def test_infinite_metadata():
    """A block with +inf upper bounds scores +inf for an all-positive query
    and is selected; its interval is (-inf, +inf), resolved exactly."""
    hq, hkv, n, d = 4, 4, 300, 64
    q, _, _, lo, hi = C.synthetic_kv(hq, hkv, n, 4, d, torch.float32, seed=6)
    q[0] = q[0].abs() + 0.1
    hi[0, 17, :] = float("inf")
    want = _want(q, lo, hi, 9)
    got = _select(q, lo, hi, 9)[0]
    assert 17 in got[0]
    assert np.array_equal(got, want)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_wide_gqa_group_selection(dtype):
    """BASELINE config 2 shape: 96 query / 8 KV heads (group 12), 8192 blocks, K 512, shared per group."""
    hq, hkv, n, d, k = 96, 8, 8192, 128, 512
    q, _, _, lo, hi = C.synthetic_kv(hq, hkv, n, 4, d, dtype, seed=7)
    assert np.array_equal(_select(q, lo, hi, k, shared=True)[0], _want(q, lo, hi, k, shared=True))


def test_short_requests_batch():
    """Requests shorter than one scorer tile: tiles span many requests and
    read q from global memory."""
    import strict_topk_overlap_b200._lib as L
    hq, hkv, d, k = 8, 4, 128, 2
    lengths = [5, 3, 17, 2, 9, 40, 2, 70, 4, 33]
    qs, los, his = [], [], []
    for r, n in enumerate(lengths):
        q, _, _, lo, hi = C.synthetic_kv(hq, hkv, n, 4, d, torch.bfloat16, seed=100 + r)
        qs.append(q)
        los.append(lo)
        his.append(hi)
    q = torch.cat(qs, 0).to(DEV)
    lo = torch.cat(los, 1).contiguous().to(DEV)
    hi = torch.cat(his, 1).contiguous().to(DEV)
    offs = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int32, device=DEV)
    total, R = int(sum(lengths)), len(lengths)
    for shared in (False, True):
        rows = hkv if shared else hq
        ids = torch.empty((R, rows, k), dtype=torch.int32, device=DEV)
        lib = L.load()
        ws_bytes = lib.stk_select_workspace_bytes(rows, total)
        ws = torch.empty((ws_bytes,), dtype=torch.uint8, device=DEV)
        rc = lib.stk_select_topk(q.data_ptr(), L.dtype_code(q), lo.data_ptr(), hi.data_ptr(), R, hq, hkv, 0,
                                 offs.data_ptr(), total, max(lengths), d, k, int(shared), 0, ids.data_ptr(), None,
                                 ws.data_ptr(), ws_bytes, L.status_ptr(), L.stream_of(q))
        L.check(rc, "select_topk")
        got = ids.cpu().numpy()
        for r in range(R):
            want = _want(qs[r], los[r], his[r], k, shared=shared)
            assert np.array_equal(got[r], want), (r, shared)
