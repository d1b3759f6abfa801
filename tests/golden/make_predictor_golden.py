"""Golden vectors for the next-step predictor, produced by the reference
itself: experiments/hisparse_cache_trace.py `predict` (pure Python) is
imported from the reference checkout and run on seeded ranked lists.

Run once beside the reference (it is not on the GPU box):
    python tests/golden/make_predictor_golden.py /path/to/strict-topk-overlap
writes tests/golden/predictor.json. Cases avoid source exhaustion, where the
reference raises."""
from __future__ import annotations

import importlib.util
import json
import random
import sys
from pathlib import Path


def main(ref_root):
    spec = importlib.util.spec_from_file_location("hisparse_cache_trace",
                                                  Path(ref_root) / "experiments" / "hisparse_cache_trace.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    rng = random.Random(20261202)
    cases = []
    for i in range(24):
        n_blocks = rng.choice([64, 200, 2048])
        k = min(rng.choice([4, 8, 16, 64]), n_blocks // 2)
        budget = rng.choice([k // 2, k, 2 * k if i % 3 == 0 else k])
        overlap = rng.random()
        rows_step, rows_layer, expected = [], [], {p: [] for p in mod.POLICIES}
        for _ in range(3):
            step = rng.sample(range(n_blocks), k)
            shared = [b for b in step if rng.random() < overlap]
            rest = [b for b in range(n_blocks) if b not in step]
            layer = shared + rng.sample(rest, k - len(shared))
            rng.shuffle(layer)
            rows_step.append(step)
            rows_layer.append(layer)
            for p in mod.POLICIES:
                b = min(budget, k) if p != "rank_interleave" else budget
                try:
                    expected[p].append(list(mod.predict(p, tuple(step), tuple(layer), b)))
                except (StopIteration, RuntimeError):  # a source ran out: the reference raises
                    expected[p].append(None)
        cases.append({"n_blocks": n_blocks, "k": k, "budget": budget, "previous_step": rows_step,
                      "previous_layer": rows_layer, "expected": expected})
    out = Path(__file__).resolve().parent / "predictor.json"
    out.write_text(json.dumps({"source": "experiments/hisparse_cache_trace.py predict()", "cases": cases}) + "\n")
    print(out, len(cases))


if __name__ == "__main__":
    if len(sys.argv) < 2:
        raise SystemExit("usage: make_predictor_golden.py <reference checkout directory>")
    main(sys.argv[1])
