"""Tensor-core group attention (stk_group_attention, gqa_hierarchical.exact_shared)
against the per-head path on the same shared lists and the FP64 oracle:
BASELINE config 2's shape (12 query heads per KV head, 4-token blocks,
K 512 shared per group), a head dim of 64 with 8 heads per group and
8-token blocks, a list that ends inside a CTA's token range, and f16."""
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


@pytest.mark.parametrize("hq,hkv,n,b,d,k,dtype", [
    (96, 8, 8192, 4, 128, 512, torch.bfloat16),
    (16, 2, 300, 8, 64, 37, torch.bfloat16),
    (24, 2, 500, 4, 128, 100, torch.float16),
])
def test_group_attention_matches_per_head_and_oracle(hq, hkv, n, b, d, k, dtype):
    from strict_topk import gqa, gqa_hierarchical as gh
    q, kk, vv, lo, hi = C.synthetic_kv(hq, hkv, n, b, d, dtype, seed=hq + n)
    ids = OS.select_blocks(C.as_np(q), lo.numpy(), hi.numpy(), k, shared=True)  # [hq, k], repeated per group
    g = hq // hkv
    grp = torch.from_numpy(np.ascontiguousarray(ids[::g])).to(torch.int32).to(DEV)
    qd, kd, vd = q.to(DEV), kk.to(DEV), vv.to(DEV)
    out = gh.exact_shared(qd, kd, vd, grp)
    per_head = gqa.exact(qd, kd, vd, grp.repeat_interleave(g, 0).contiguous())
    torch.cuda.synchronize()
    assert (out - per_head).abs().max().item() <= 1e-4
    ref = OA.attention_fp64(q.float().numpy(), kk.float().numpy(), vv.float().numpy(), ids)
    assert (np.abs(out.cpu().numpy() - ref) <= 2e-3 + 1e-2 * np.abs(ref)).all()


@pytest.mark.parametrize("hq,hkv,n,b,d,k,sp,nswap,dtype", [
    (96, 8, 2048, 4, 128, 256, 256, 51, torch.bfloat16),   # config-2 shape, reduced context, 80 % overlap
    (64, 8, 700, 4, 64, 100, 90, 30, torch.float16),        # 8 heads per group, shorter predicted list
    (32, 2, 400, 8, 128, 50, 50, 0, torch.bfloat16),        # full overlap: no misses
])
def test_group_repair_saved_shared_matches_per_row_and_oracle(hq, hkv, n, b, d, k, sp, nswap, dtype):
    """repair_saved_shared on the tensor-core group tile (misses once per
    group, hits per head) against the per-row saved repair on the same
    inputs and the FP64 oracle over the strict set."""
    from strict_topk import gqa_hierarchical as gh
    q, kk, vv, lo, hi = C.synthetic_kv(hq, hkv, n, b, d, dtype, seed=hq + n + 1)
    ids = OS.select_blocks(C.as_np(q), lo.numpy(), hi.numpy(), k, shared=True)
    g = hq // hkv
    pg = C.swap_prediction(torch.from_numpy(np.ascontiguousarray(ids[::g])), n, nswap, seed=hq + 2)[:, :sp]
    p = pg.repeat_interleave(g, 0).to(torch.int32).contiguous().to(DEV)
    a = torch.from_numpy(ids).to(torch.int32).contiguous().to(DEV)
    qd, kd, vd = q.to(DEV), kk.to(DEV), vv.to(DEV)
    st = gh.partials(qd, kd, vd, p)
    assert gh._group_tile_ok(qd, kd, a, p)
    out = gh.repair_saved_shared(qd, kd, vd, a, p, st)
    per_row = gh.repair_saved(qd, kd, vd, a, p, st)
    torch.cuda.synchronize()
    assert (out - per_row).abs().max().item() <= 1e-4
    ref = OA.attention_fp64(q.float().numpy(), kk.float().numpy(), vv.float().numpy(), ids)
    assert (np.abs(out.cpu().numpy() - ref) <= 2e-3 + 1e-2 * np.abs(ref)).all()


@pytest.mark.parametrize("hq,hkv,n,b,d,dtype", [
    (24, 2, 300, 4, 128, torch.bfloat16),   # config-2 group (12 heads) and block size
    (32, 2, 150, 4, 128, torch.bfloat16),   # 16 heads per group
    (16, 2, 200, 8, 64, torch.float16),
    (6, 3, 100, 2, 128, torch.float32),     # 2 heads per group
])
def test_tiny_block_group_states(hq, hkv, n, b, d, dtype):
    """Per-block states of tiny blocks (the group kernel: a block shared by a
    KV group is read once, a head with its own ID reads its own block, -1
    gives (-inf, 0, 0)) against the oracle's per-block state, on lists that
    are shared per group with some heads' slots replaced or emptied."""
    from strict_topk import kernels
    from oracle import speculative as OP
    q, kk, vv, _, _ = C.synthetic_kv(hq, hkv, n, b, d, dtype, seed=hq + b)
    g, s = hq // hkv, 40
    gen = torch.Generator().manual_seed(hq + d)
    ids = torch.stack([torch.randperm(n, generator=gen)[:s] for _ in range(hkv)]).repeat_interleave(g, 0)
    own = torch.rand(hq, s, generator=gen) < 0.2
    ids[own] = torch.randint(0, n, (int(own.sum()),), generator=gen)
    ids[torch.rand(hq, s, generator=gen) < 0.05] = -1
    ids[0::g, 3] = -1  # the group's first head has no block at slot 3: the others still do
    ids[1::g, 5] = -1
    ids = ids.to(torch.int32).contiguous()
    st = kernels.block_partials(q.to(DEV), kk.to(DEV), vv.to(DEV), ids.to(DEV))
    torch.cuda.synchronize()
    m, l, u = st.m.cpu().numpy(), st.l.cpu().numpy(), st.u.cpu().numpy()
    X = OP.Inputs(C.as_np(q), C.as_np(kk), C.as_np(vv))
    for h in range(hq):
        for j in range(s):
            bid = int(ids[h, j])
            if bid < 0:
                assert np.isneginf(m[h, j]) and l[h, j] == 0 and not u[h, j].any(), (h, j)
                continue
            mm, ll, uu = OP.block_state(X, h, bid)
            assert np.isclose(m[h, j], mm, rtol=1e-5, atol=1e-5), (h, j)
            assert np.isclose(l[h, j], ll, rtol=1e-5), (h, j)
            assert np.allclose(u[h, j], uu, rtol=1e-4, atol=1e-4), (h, j)
