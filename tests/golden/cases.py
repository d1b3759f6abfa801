"""Seeded CPU input cases shared by the golden-fixture script and the parity tests.

Every generator builds its tensors on the CPU with ``torch.Generator`` so the
golden script (run once, beside the reference) and the tests (run anywhere,
including the GPU box, where the reference is absent) see bit-identical
inputs. Each fixture stores a SHA-256 of its inputs so a drift in the
generator is a loud failure rather than a silent mismatch.

The case shapes and adversarial constructions restate the reference's own
test inputs:

* ``correctness_cases``  -> tests/check_correctness.py:35-104
* ``gqa_cases``          -> tests/check_gqa.py:35-70
* ``gqa_light_cases``    -> tests/check_gqa_light.py:23-48
* ``hierarchical_cases`` -> tests/check_gqa_hierarchical.py:12-37
* ``selector_case``      -> tests/check_selector.py:8-27
* ``budget_case``        -> tests/check_signed_repair.py:29-56
* ``underflow_case``     -> tests/check_signed_fused.py:17-30
* ``baseline_config0``   -> BASELINE config 0 (CPU plumbing, FP32)
"""
from __future__ import annotations

import hashlib
import math

import numpy as np
import torch


def digest(*tensors) -> str:
    """SHA-256 over the raw bytes of the given tensors (order matters)."""
    h = hashlib.sha256()
    for t in tensors:
        t = t.contiguous()
        h.update(str(t.dtype).encode())
        h.update(str(tuple(t.shape)).encode())
        h.update(t.view(torch.uint8).numpy().tobytes() if t.dtype in (torch.float16, torch.bfloat16)
                 else t.numpy().tobytes())
    return h.hexdigest()


def correctness_cases(dtype):
    """Random, ragged, and adversarial cases (tests/check_correctness.py:35-104)."""
    gen = torch.Generator().manual_seed(20261103)
    out = []
    for h, n, b, d, count in [(1, 19, 16, 32, 5), (4, 32, 32, 64, 8), (8, 24, 64, 128, 8)]:
        q = torch.randn(h, d, generator=gen, dtype=dtype)
        k = torch.randn(h, n, b, d, generator=gen, dtype=dtype)
        v = torch.randn(h, n, b, d, generator=gen, dtype=dtype)
        p = torch.arange(count, dtype=torch.int32).expand(h, -1).contiguous()
        for overlap in [0, count // 2, count]:
            a = torch.arange(count - overlap, 2 * count - overlap, dtype=torch.int32)
            out.append((f"random_h{h}_b{b}_d{d}_overlap{overlap}of{count}", q, k, v, p,
                        a.expand(h, -1).contiguous()))

    # Non-power-of-two tiles, |P| != |A|, unsorted unique IDs per head.
    h, n, b, d = 4, 31, 17, 48
    q = torch.randn(h, d, generator=gen, dtype=dtype)
    k = torch.randn(h, n, b, d, generator=gen, dtype=dtype)
    v = torch.randn(h, n, b, d, generator=gen, dtype=dtype)
    for sp, sa, overlap in [(8, 5, 0), (8, 5, 2), (8, 5, 5), (3, 7, 2)]:
        preds, sels = [], []
        for _ in range(h):
            perm = torch.randperm(n, generator=gen)
            pi = perm[:sp]
            ai = torch.cat((pi[:overlap], perm[sp:sp + sa - overlap]))
            preds.append(pi[torch.randperm(sp, generator=gen)])
            sels.append(ai[torch.randperm(sa, generator=gen)])
        p, a = torch.stack(preds).int(), torch.stack(sels).int()
        out.append((f"random_unordered_b17_d48_p{sp}_a{sa}_hit{overlap}", q, k, v, p, a))

    for name in ["high_wrong_mass", "many_low_wrong_mass", "signed_value_cancellation",
                 "extreme_wrong_logits"]:
        h, n, b, d, count = 2, 24, 16, 32, 8
        q = torch.zeros(h, d, dtype=dtype)
        q[:, 0] = 1
        logits = torch.zeros(h, n)
        if name == "high_wrong_mass":
            logits[:, 0] = 20
        elif name == "many_low_wrong_mass":
            logits.fill_(-8)
            logits[:, :7] = 10
        elif name == "extreme_wrong_logits":
            logits.fill_(-40)
            logits[:, :7] = 80
        k = torch.zeros(h, n, b, d, dtype=dtype)
        k[..., 0] = (logits * math.sqrt(d))[:, :, None]
        v = torch.randn(h, n, b, d, generator=gen, dtype=dtype)
        if name == "signed_value_cancellation":
            signs = torch.where(torch.arange(d) % 2 == 0, 1., -1.)
            v[:] = signs * .01
            v[:, :7] = signs * 60000.
        p = torch.arange(count, dtype=torch.int32).expand(h, -1).contiguous()
        a = torch.arange(7, 15, dtype=torch.int32).expand(h, -1).contiguous()
        out.append((name, q, k, v, p, a))

    # Removed blocks cancel exactly; only the absolute envelope sees the loss.
    q = torch.ones(1, 1, dtype=dtype)
    k = torch.zeros(1, 4, 1, 1, dtype=dtype)
    v = torch.tensor([60000., .01, -60000., 1.], dtype=dtype).view_as(k)
    p = torch.tensor([[0, 1, 2]], dtype=torch.int32)
    a = torch.tensor([[1]], dtype=torch.int32)
    out.append(("signed_low_aggregate_cancellation", q, k, v, p, a))

    # A fully rejected low group with a huge maximum must be discarded.
    k = k.clone()
    k[:, :3] = 100
    a = torch.tensor([[3]], dtype=torch.int32)
    out.append(("discard_high_logit_low_group", q, k, v, p, a))
    return out


def gqa_cases():
    """Native-GQA cases (tests/check_gqa.py:35-70); returns (name, q, k, v, p, a)."""
    gen = torch.Generator().manual_seed(20261103)
    q = torch.randn((6, 13), dtype=torch.float16, generator=gen)
    k = torch.randn((2, 23, 7, 13), dtype=torch.float16, generator=gen)
    v = torch.randn(k.shape, dtype=torch.float16, generator=gen)
    perms = torch.stack([torch.randperm(23, generator=gen) for _ in range(6)])
    out = []
    for sp, sa, overlap in [(6, 6, 0), (6, 6, 3), (6, 6, 6), (7, 5, 2), (3, 7, 2)]:
        p = perms[:, :sp].contiguous()
        a = torch.cat((perms[:, :overlap], perms[:, sp:sp + sa - overlap]), dim=1)
        out.append((f"gqa_p{sp}_a{sa}_hit{overlap}", q, k, v, p, a.flip(1).int().contiguous()))
    q2 = q.clone()
    q2.zero_()
    q2[:, 0] = 1
    k2 = k.clone()
    k2[..., 0] = -5000
    k2[:, 1, :, 0] = 2000
    k2[:, 3, :, 0] = 5000
    p = torch.tensor([[0, 3, 2]] * 6, dtype=torch.int32)
    a = torch.tensor([[2, 1, 0]] * 6, dtype=torch.int64)
    out.append(("gqa_extreme_logits", q2, k2, v, p, a))
    q3 = torch.ones((2, 1), dtype=torch.float16)
    k3 = torch.tensor([[[[2.]], [[-3.]]]], dtype=torch.float16)
    v3 = torch.tensor([[[[8.]], [[-5.]]]], dtype=torch.float16)
    p3 = torch.tensor([[0], [1]], dtype=torch.int32)
    out.append(("gqa_tiny_hit", q3, k3, v3, p3, p3.clone()))
    out.append(("gqa_tiny_miss", q3, k3, v3, p3, (1 - p3).contiguous()))
    return out


def gqa_selector_case():
    """Tied-score GQA selection (tests/check_gqa.py:46-54): q[0] is zero."""
    gen = torch.Generator().manual_seed(20261103)
    q = torch.randn((6, 13), dtype=torch.float16, generator=gen)
    k = torch.randn((2, 23, 7, 13), dtype=torch.float16, generator=gen)
    q[0].zero_()
    lo, hi = k.amin(2).float(), k.amax(2).float()
    return q, lo, hi, 5


def gqa_light_cases():
    """Light-repair cases (tests/check_gqa_light.py:23-48)."""
    gen = torch.Generator().manual_seed(20261103)
    q = torch.randn((16, 13), dtype=torch.float16, generator=gen)
    k = torch.randn((4, 23, 7, 13), dtype=torch.float16, generator=gen)
    v = torch.randn(k.shape, dtype=torch.float16, generator=gen)
    perms = torch.stack([torch.randperm(23, generator=gen) for _ in range(16)])
    out = []
    for sp, sa, overlap in [(6, 6, 0), (6, 6, 3), (6, 6, 5), (6, 6, 6), (7, 5, 2), (3, 7, 2)]:
        p = perms[:, :sp].contiguous()
        a = torch.cat((perms[:, :overlap], perms[:, sp:sp + sa - overlap]), dim=1)
        out.append((f"light_p{sp}_a{sa}_hit{overlap}", q, k, v, p, a.flip(1).int().contiguous()))
    q2 = q.clone()
    q2.zero_()
    q2[:, 0] = 1
    k2 = k.clone()
    k2[..., 0] = -5000
    k2[:, 1, :, 0] = 2000
    k2[:, 3, :, 0] = 5000
    p = torch.tensor([[0, 3, 2]] * 16, dtype=torch.int32)
    a = torch.tensor([[2, 1, 0]] * 16, dtype=torch.int64)
    out.append(("light_extreme_logits", q2, k2, v, p, a))
    return out


def _prediction(selected, blocks, predict_k, hits):
    """benchmarks/critical_path.py:170-176: first ``hits`` selected + lowest unselected."""
    rows = []
    for row in selected.tolist():
        chosen = set(row)
        wrong = [blk for blk in range(blocks) if blk not in chosen]
        rows.append(row[:hits] + wrong[:predict_k - hits])
    return torch.tensor(rows, dtype=selected.dtype)


def hierarchical_cases(dtype, large=True):
    """Tiny-block GQA cases (tests/check_gqa_hierarchical.py:12-37).

    Returns (name, q, k, v, p, a, shared) tuples; ``shared`` rows repeat row 0.
    """
    gen = torch.Generator().manual_seed(317)
    shapes = [(24, 2, 1024, 4, 256, 512), (6, 2, 96, 5, 96, 37)]
    out = []
    for h, hkv, n, b, d, sa in shapes:
        q = torch.randn((h, d), dtype=dtype, generator=gen)
        k = torch.randn((hkv, n, b, d), dtype=dtype, generator=gen)
        v = torch.randn(k.shape, dtype=dtype, generator=gen)
        a = torch.stack([torch.randperm(n, generator=gen)[:sa] for _ in range(h)]).int()
        for hit in [0, sa // 2, sa - 1, sa]:
            p = _prediction(a, n, sa, hit)
            out.append((f"hier_h{h}_b{b}_d{d}_hit{hit}", q, k, v, p, a, False))
        shared = a[:1].expand(h, -1).contiguous()
        for hit in (0, sa // 2, sa):
            pred = _prediction(shared, n, max(1, sa // 2), min(hit, sa // 2))
            out.append((f"hier_shared_h{h}_b{b}_d{d}_hit{hit}", q, k, v, pred, shared, True))
    if not large:  # the RNG stream is consumed for every shape; only the return is filtered
        out = [c for c in out if "_h24_" not in c[0]]
    return out


def selector_case():
    """Per-head fused-score selector case (tests/check_selector.py:8-27)."""
    gen = torch.Generator().manual_seed(20261103)
    q = torch.randn((3, 70), dtype=torch.float16, generator=gen)
    keys = torch.randn((3, 37, 7, 70), dtype=torch.float16, generator=gen)
    lo, hi = keys.amin(dim=2).float(), keys.amax(dim=2).float()
    q[0].zero_()
    return q, lo, hi, (1, 11, 37)


def budget_case():
    """max_extra_mass known-answer case (tests/check_signed_repair.py:29-56)."""
    q = torch.ones((1, 1), dtype=torch.float16)
    k = torch.tensor([3., 0., -3., 0.], dtype=q.dtype).view(1, 4, 1, 1)
    v = torch.tensor([100., 1., 8., 2.], dtype=q.dtype).view_as(k)
    p = torch.tensor([[0, 1, 2]], dtype=torch.int64)
    a = torch.tensor([[1, 3]], dtype=torch.int32)
    extra_set = torch.tensor([[1, 3, 2]], dtype=torch.int32)
    return q, k, v, p, a, extra_set


def underflow_case():
    """BF16 hybrid-erasure underflow regression (tests/check_signed_fused.py:17-30)."""
    q = torch.ones((1, 1), dtype=torch.bfloat16)
    k = torch.full((1, 3, 8192, 1), -200., dtype=q.dtype)
    k[:, :, 0, 0] = 0.
    k[:, 2, :, 0] = -104.
    k[:, 2, 0, 0] = -80.
    v = torch.zeros_like(k)
    v[:, 2, 1:, 0] = 3.e38
    p = torch.tensor([[0, 1, 2]], dtype=torch.int32)
    a = torch.tensor([[0, 1]], dtype=torch.int32)
    return q, k, v, p, a


def synthetic_kv(hq, hkv, blocks, block_size, dim, dtype, seed, bias_std=0.5):
    """BASELINE input distribution: Q ~ N(0,1); K = N(0,1) + per-block bias; V ~ N(0,1).

    The bias is one N(0, bias_std^2) vector of length ``dim`` per (KV head,
    block), shared by the block's tokens. Metadata lo/hi are the per-block
    token-wise min/max of K, in FP32.
    """
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(hq, dim, generator=gen)
    k = torch.randn(hkv, blocks, block_size, dim, generator=gen)
    bias = torch.randn(hkv, blocks, 1, dim, generator=gen) * bias_std
    k = k + bias
    v = torch.randn(hkv, blocks, block_size, dim, generator=gen)
    q, k, v = q.to(dtype), k.to(dtype), v.to(dtype)
    lo, hi = k.amin(dim=2).float(), k.amax(dim=2).float()
    return q, k, v, lo, hi


def swap_prediction(selected, blocks, n_swap, seed):
    """Predicted list = true Top-K with ``n_swap`` IDs per row replaced by
    seeded-random unselected blocks (same position, so row order is kept)."""
    gen = torch.Generator().manual_seed(seed)
    rows = []
    for row in selected.tolist():
        chosen = set(row)
        pool = torch.tensor([b for b in range(blocks) if b not in chosen])
        repl = pool[torch.randperm(len(pool), generator=gen)[:n_swap]].tolist()
        pos = torch.randperm(len(row), generator=gen)[:n_swap].tolist()
        new = list(row)
        for j, r in zip(pos, repl):
            new[j] = r
        rows.append(new)
    return torch.tensor(rows, dtype=torch.int32)


def baseline_config0():
    """batch 1, 8 query / 2 KV heads, D=128, 4096 tokens in
    32-token blocks (128 blocks), K=16, FP32, seed 0; 4 of 16 IDs swapped."""
    q, k, v, lo, hi = synthetic_kv(8, 2, 128, 32, 128, torch.float32, seed=0)
    return q, k, v, lo, hi, 16, 4


def as_np(t):
    """Tensor -> numpy, widening half types to float32 exactly."""
    if t.dtype in (torch.float16, torch.bfloat16):
        return t.float().numpy()
    return t.numpy()


def np_f32(t) -> np.ndarray:
    return as_np(t).astype(np.float32)
