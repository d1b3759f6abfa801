"""Next-step predictor (previous_step / previous_layer / rank_interleave).

CPU: the oracle restatement against golden vectors produced by the
reference's own experiments/hisparse_cache_trace.py predict()
(tests/golden/make_predictor_golden.py), and key ranking ties.
GPU: stk_predict against the oracle, with and without order keys, including
sources that run out (the reference raises there; the device fills from the
other source, then -1)."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import predictor as OP

GOLDEN = json.loads((Path(__file__).resolve().parent / "golden" / "predictor.json").read_text())


def test_oracle_matches_reference_golden():
    checked = 0
    for c in GOLDEN["cases"]:
        for policy, rows in c["expected"].items():
            for i, want in enumerate(rows):
                if want is None:  # the reference raised: a source ran out
                    continue
                b = len(want)
                got = OP.predict(policy, c["previous_step"][i], c["previous_layer"][i], b)
                assert got == want, (policy, i)
                checked += 1
    assert checked >= 200


def test_rank_by_keys_ties_to_lower_position():
    ids = [5, 9, 2, 7]
    keys = np.array([3, 8, 8, 1], dtype=np.uint64).view(np.int64)
    assert OP.rank_by_keys(ids, keys) == [9, 2, 5, 7]
    assert OP.rank_by_keys(ids, None) == ids


@pytest.mark.gpu
def test_device_predict_matches_oracle():
    from strict_topk_overlap_b200 import predictor
    import strict_topk_overlap_b200._lib as L
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    L.set_status_tensor(st)
    try:
        for c in GOLDEN["cases"]:
            step = torch.tensor(c["previous_step"], dtype=torch.int32, device="cuda")
            layer = torch.tensor(c["previous_layer"], dtype=torch.int32, device="cuda")
            for policy in ("previous_step", "previous_layer", "rank_interleave"):
                for budget in (c["budget"], 2 * c["k"] + 3):
                    got = predictor.predict(policy, budget, c["n_blocks"], previous_step=step,
                                            previous_layer=layer).cpu().tolist()
                    for i in range(step.shape[0]):
                        want = OP.predict(policy, c["previous_step"][i], c["previous_layer"][i], budget)
                        assert got[i] == want, (policy, budget, i)
        # Ranked by order keys (random keys with ties).
        gen = torch.Generator().manual_seed(3)
        ids = torch.stack([torch.randperm(500, generator=gen)[:40] for _ in range(4)]).to(torch.int32)
        keys = torch.randint(0, 5, (4, 40), generator=gen, dtype=torch.int64)
        lay = torch.stack([torch.randperm(500, generator=gen)[:40] for _ in range(4)]).to(torch.int32)
        lkeys = torch.randint(0, 1 << 40, (4, 40), generator=gen, dtype=torch.int64)
        got = predictor.predict("rank_interleave", 50, 500, previous_step=ids.cuda(), previous_step_keys=keys.cuda(),
                                previous_layer=lay.cuda(), previous_layer_keys=lkeys.cuda()).cpu().tolist()
        for i in range(4):
            rs = OP.rank_by_keys(ids[i].tolist(), keys[i].numpy())
            rl = OP.rank_by_keys(lay[i].tolist(), lkeys[i].numpy())
            assert got[i] == OP.predict("rank_interleave", rs, rl, 50)
        torch.cuda.synchronize()
        assert st.item() == 0
    finally:
        L.set_status_tensor(None)
