"""CPU oracle for the strict Top-K speculative decode path — TEST INFRASTRUCTURE.

This package restates, in NumPy, the reference algorithms
(6Mikao9/strict-topk-overlap, strict_topk/*.py) that the sm_100a library
replaces. It is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` import it. Nothing in ``strict_topk_overlap_b200`` may.

Parity is pinned: ``tests/test_oracle_golden.py`` checks every function here
against golden fixtures produced by running the reference implementation
itself (its Triton kernels under the Triton CPU interpreter, and its torch
FP64 oracles) — see ``tests/golden/make_golden.py``.

Modules
  selection   fixed-order FP64 bound scores, stable Top-K, shard candidate merge
  attention   FP64 strict / union attention (the reference's test oracle)
  speculative FP32 restatement of speculate() and every repair variant,
              reproducing their guard / budget / job-count decisions
"""
