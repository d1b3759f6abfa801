"""Block metadata builder and decode-loop append (stk_build_metadata,
stk_append_token) against torch amin / amax over the filled tokens: dense
caches in f32 / f16 / bf16, the paged pool, and a sequence of appended
tokens crossing block boundaries; bit-exact (min / max involve no rounding)."""
from __future__ import annotations

import ctypes as C

import pytest
import torch

import cases as CS

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_build_metadata_dense(dtype):
    from strict_topk_overlap_b200 import metadata
    _, k, _, lo, hi = CS.synthetic_kv(8, 4, 37, 32, 128, dtype, seed=11)
    glo, ghi = metadata.build_metadata(k.to(DEV))
    torch.cuda.synchronize()
    assert torch.equal(glo.cpu(), lo) and torch.equal(ghi.cpu(), hi)


def test_build_metadata_paged():
    import strict_topk_overlap_b200._lib as L
    from strict_topk_overlap_b200 import paged
    ks, vs, los, his = [], [], [], []
    for r, n in enumerate((5, 9, 3)):
        _, k, v, lo, hi = CS.synthetic_kv(4, 2, n, 32, 64, torch.bfloat16, seed=20 + r)
        ks.append(k)
        vs.append(v)
        los.append(lo)
        his.append(hi)
    cache = paged.build_paged_cache(ks, vs, 16, generator=torch.Generator().manual_seed(1), device=torch.device(DEV))
    total = sum(k.shape[1] for k in ks)
    lo = torch.empty((2, total, 64), device=DEV)
    hi = torch.empty_like(lo)
    kv = cache.kv()
    rc = L.load().stk_build_metadata(C.byref(kv), 3, total, lo.data_ptr(), hi.data_ptr(), None,
                                     L.stream_of(lo))
    L.check(rc, "build_metadata")
    torch.cuda.synchronize()
    assert torch.equal(lo.cpu(), torch.cat(los, 1)) and torch.equal(hi.cpu(), torch.cat(his, 1))


def test_append_tokens_across_blocks():
    from strict_topk_overlap_b200 import metadata
    hkv, n, b, d = 2, 4, 8, 64
    gen = torch.Generator().manual_seed(5)
    full_k = torch.randn(hkv, n, b, d, generator=gen).to(torch.bfloat16)
    full_v = torch.randn(hkv, n, b, d, generator=gen).to(torch.bfloat16)
    k = torch.zeros_like(full_k, device=DEV)
    v = torch.zeros_like(full_v, device=DEV)
    lo = torch.full((hkv, n, d), float("nan"), device=DEV)
    hi = torch.full_like(lo, float("nan"))
    pos = torch.zeros(1, dtype=torch.int32, device=DEV)
    for p in range(n * b - 3):
        j, t = divmod(p, b)
        pos.fill_(p)
        metadata.append_token(k, v, lo, hi, full_k[:, j, t].to(DEV), full_v[:, j, t].to(DEV), pos)
        torch.cuda.synchronize()
        filled = full_k[:, j, : t + 1].float()
        assert torch.equal(lo[:, j].cpu(), filled.amin(1)) and torch.equal(hi[:, j].cpu(), filled.amax(1))
    assert torch.equal(k[:, :3].cpu(), full_k[:, :3]) and torch.equal(v[:, :3].cpu(), full_v[:, :3])
    with pytest.raises(ValueError):
        metadata.append_token(k, v, lo, hi, full_k[:, 0, 0].to(DEV), full_v[:, 0, 0].to(DEV), n * b)
