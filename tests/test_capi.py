"""The C-ABI library loads on a CPU-only host and exports exactly the
symbols include/strict_topk_b200.h declares; host-side validation rejects bad
arguments before any device work."""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "strict_topk_b200.h"


def _declared():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"STK_API\s+(?:int|size_t|const char\*)\s+(stk_\w+)\(", text)))


@pytest.fixture(scope="module")
def lib():
    from strict_topk_overlap_b200 import _lib as L
    from strict_topk_overlap_b200.build import build_library
    build_library()
    return L.load()


def test_header_matches_binding():
    from strict_topk_overlap_b200 import _lib as L
    assert _declared() == sorted(L.SYMBOLS)


def test_library_exports_every_symbol(lib):
    for name in _declared():
        assert hasattr(lib, name), name
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", str(ROOT / "strict_topk_overlap_b200/_lib/libstk_sm100.so")],
                         capture_output=True, text=True).stdout
    exported = sorted(set(re.findall(r" T (stk_\w+)", out)))
    assert exported == _declared()


def test_host_validation_without_gpu(lib):
    assert lib.stk_abi_version() == 1
    assert lib.stk_select_workspace_bytes(4, 100) == 4 * 100 * 8
    assert lib.stk_speculate_workspace_bytes(2, 8, 128, 2) == 2 * 8 * 128 * 4 * 2
    assert lib.stk_speculate_workspace_bytes(2, 8, 128, 0) == 0
    # Null pointers / bad shapes are rejected on the host with STK_EINVAL (-1).
    assert lib.stk_bound_scores(None, 0, None, None, 1, 1, 1, 1, None, None) == -1
    assert b"null" in lib.stk_last_error()
    assert lib.stk_merge_states(None, None, None, None, 1, 1, 1, None, None) == -1
    from strict_topk_overlap_b200 import _lib as L
    kv = L.StkKV(1, 1, 2, 2, 10, 32, 2048, None, None, 0, 0)
    rc = lib.stk_touch_kv(C.byref(kv), 4, 4, 1, 0, 1, 1, None)
    assert rc == -3 and b"1024" in lib.stk_last_error()
    kv = L.StkKV(1, 1, 2, 3, 10, 32, 128, None, None, 0, 0)
    assert lib.stk_touch_kv(C.byref(kv), 4, 4, 1, 0, 1, 1, None) == -1  # 4 % 3 != 0
    assert b"divisible" in lib.stk_last_error()
    # The wait-limit setter and the wait probe validate before touching a device.
    assert lib.stk_set_wait_limit_ns(0) == -1 and b"positive" in lib.stk_last_error()
    assert lib.stk_check_wait_timeout(None, None) == -1


def test_no_cpu_fallback_in_product():
    """The product package never imports the oracle or Triton."""
    for p in (ROOT / "strict_topk_overlap_b200").rglob("*.py"):
        src = p.read_text()
        assert "import oracle" not in src and "from oracle" not in src, p
        assert "import triton" not in src, p
