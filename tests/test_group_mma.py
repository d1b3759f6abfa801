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
