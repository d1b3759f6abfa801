"""ctypes binding of libstk_sm100.so (the C ABI in include/strict_topk_b200.h).

The library is loaded lazily on the first device call. There is no CPU or
Triton fallback: when the shared library is missing or fails to load, every
entry point raises ``RuntimeError`` naming the build command.
"""
from __future__ import annotations

import ctypes as C
import os
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libstk_sm100.so"

STK_F32, STK_F16, STK_BF16 = 0, 1, 2
MODE_FULL, MODE_MASS, MODE_FIXED = 0, 1, 2
PREDICT_PREVIOUS_STEP, PREDICT_PREVIOUS_LAYER, PREDICT_RANK_INTERLEAVE = 0, 1, 2
PRED_SAVED, PRED_HYBRID, PRED_COMPACT, PRED_NONE = 0, 1, 2, 3
VAR_SPLIT, VAR_FUSED, VAR_SIGNED, VAR_SIGNED_FUSED, VAR_SAVED, VAR_UNION = 0, 1, 2, 3, 4, 5
PRED_MODES = {"saved": PRED_SAVED, "hybrid": PRED_HYBRID, "compact": PRED_COMPACT}

_DTYPES = {torch.float32: STK_F32, torch.float16: STK_F16, torch.bfloat16: STK_BF16}

# Exported symbols, exactly those declared in include/strict_topk_b200.h.
SYMBOLS = (
    "stk_abi_version", "stk_last_error", "stk_device_sm_count", "stk_set_wait_limit_ns", "stk_check_wait_timeout",
    "stk_bound_scores",
    "stk_select_workspace_bytes", "stk_select_topk", "stk_select_topk_static", "stk_merge_candidates", "stk_block_states",
    "stk_merge_states", "stk_reduce_states", "stk_speculate_workspace_bytes", "stk_speculate", "stk_repair",
    "stk_speculative_step_workspace_bytes", "stk_speculative_step", "stk_speculative_step_hybrid_workspace_bytes",
    "stk_speculative_step_hybrid", "stk_speculative_step_batched_workspace_bytes", "stk_speculative_step_batched",
    "stk_decode_step_workspace_bytes", "stk_decode_step", "stk_build_metadata", "stk_append_token",
    "stk_predict", "stk_group_repair_saved_workspace_bytes", "stk_group_repair_saved",
    "stk_group_attention_workspace_bytes", "stk_group_attention", "stk_touch_kv",
)


class StkKV(C.Structure):
    _fields_ = [("k", C.c_void_p), ("v", C.c_void_p), ("kv_dtype", C.c_int), ("hkv", C.c_int), ("n", C.c_int),
                ("b", C.c_int), ("d", C.c_int), ("page_table", C.c_void_p), ("block_offsets", C.c_void_p),
                ("page_size", C.c_int), ("kv_request_stride", C.c_longlong)]


class StkPrediction(C.Structure):
    _fields_ = [("mode", C.c_int), ("sc", C.c_int), ("m", C.c_void_p), ("l", C.c_void_p), ("u", C.c_void_p),
                ("high", C.c_void_p), ("retained_ids", C.c_void_p), ("retained_ids64", C.c_int),
                ("low_m", C.c_void_p), ("low_l", C.c_void_p), ("low_u", C.c_void_p), ("low_abs", C.c_void_p),
                ("mass_m", C.c_void_p), ("mass_l", C.c_void_p)]


class StkRepairOut(C.Structure):
    _fields_ = [("out", C.c_void_p), ("fallback", C.c_void_p), ("remaining", C.c_void_p), ("approx", C.c_void_p),
                ("extra", C.c_void_p), ("positive_jobs", C.c_void_p), ("total_jobs", C.c_void_p)]


_P = C.c_void_p
_I = C.c_int
_F = C.c_float
_SZ = C.c_size_t
_SIGS = {
    "stk_abi_version": (_I, []),
    "stk_last_error": (C.c_char_p, []),
    "stk_device_sm_count": (_I, [_I]),
    "stk_set_wait_limit_ns": (_I, [C.c_ulonglong]),
    "stk_check_wait_timeout": (_I, [_P, _P]),
    "stk_bound_scores": (_I, [_P, _I, _P, _P, _I, _I, _I, _I, _P, _P]),
    "stk_select_workspace_bytes": (_SZ, [_I, _I]),
    "stk_select_topk": (_I, [_P, _I, _P, _P, _I, _I, _I, _I, _P, _I, _I, _I, _I, _I, _I, _P, _P, _P, _SZ, _P, _P]),
    "stk_select_topk_static": (_I, [_P, _I, _P, _P, _I, _I, _I, _I, _P, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P]),
    "stk_merge_candidates": (_I, [_P, _P, _I, _I, _I, _P, _P, _P]),
    "stk_block_states": (_I, [C.POINTER(StkKV), _P, _I, _I, _I, _P, _I, _I, _P, _I, _I, _P, _I, _I, _P, _I, _P,
                              _P, _P, _P, _P, _P, _P]),
    "stk_merge_states": (_I, [_P, _P, _P, _P, _I, _I, _I, _P, _P]),
    "stk_reduce_states": (_I, [_P, _P, _P, _P, _I, _I, _I, _P, _P, _P, _P]),
    "stk_speculate_workspace_bytes": (_SZ, [_I, _I, _I, _I]),
    "stk_speculate": (_I, [C.POINTER(StkKV), _P, _I, _I, _I, _P, _I, _I, _I, _F, _I, _P, _P, _P, _P, _P, _P, _P,
                           _P, _P, _P, _P, _P, _P, _SZ, _P, _P]),
    "stk_repair": (_I, [C.POINTER(StkKV), _P, _I, _I, _I, _P, _I, _I, _P, _I, _I, C.POINTER(StkPrediction), _I, _F,
                        _F, _F, _I, C.POINTER(StkRepairOut), _P, _P]),
    "stk_speculative_step_workspace_bytes": (_SZ, [_I, _I, _I, _I]),
    "stk_speculative_step": (_I, [C.POINTER(StkKV), _P, _I, _P, _P, _I, _I, _P, _I, _I, _P, _P, _P, _SZ, _P, _P]),
    "stk_speculative_step_hybrid_workspace_bytes": (_SZ, [_I, _I, _I, _I]),
    "stk_speculative_step_hybrid": (_I, [C.POINTER(StkKV), _P, _I, _P, _P, _I, _I, _P, _I, _I, _F, _I, _F, _F, _F, _P,
                                         C.POINTER(StkRepairOut), _P, _SZ, _P, _P]),
    "stk_speculative_step_batched_workspace_bytes": (_SZ, [_I, _I, _I, _I, _I, _I]),
    "stk_speculative_step_batched": (_I, [C.POINTER(StkKV), _P, _I, _P, _P, _I, _I, _I, _I, _I, _P, _I, _I, _F, _I, _F,
                                          _F, _F, _P, C.POINTER(StkRepairOut), _P, _SZ, _P, _P]),
    "stk_decode_step_workspace_bytes": (_SZ, [_I, _I, _I, _I, _I]),
    "stk_decode_step": (_I, [C.POINTER(StkKV), _P, _I, _P, _P, _I, _I, _P, _I, _I, _P, _P, _P, _SZ, _P, _P]),
    "stk_build_metadata": (_I, [C.POINTER(StkKV), _I, _I, _P, _P, _P, _P]),
    "stk_append_token": (_I, [C.POINTER(StkKV), _I, _I, _P, _P, _P, _P, _P, _P, _P]),
    "stk_predict": (_I, [_I, _P, _P, _I, _P, _P, _I, _I, _I, _I, _P, _P, _P]),
    "stk_group_repair_saved_workspace_bytes": (_SZ, [_I, _I, _I, _I, _I, _I]),
    "stk_group_repair_saved": (_I, [C.POINTER(StkKV), _P, _I, _I, _P, _I, _P, _I, _P, _P, _P, _P, _P, _SZ, _P, _P]),
    "stk_group_attention_workspace_bytes": (_SZ, [_I, _I, _I, _I]),
    "stk_group_attention": (_I, [C.POINTER(StkKV), _P, _I, _I, _P, _I, _P, _P, _SZ, _P, _P]),
    "stk_touch_kv": (_I, [C.POINTER(StkKV), _I, _I, _P, _I, _I, _P, _P]),
}

_lock = threading.Lock()
_lib = None
_status = None  # optional device status word (int32 tensor) passed to every call


def load(path: str | os.PathLike | None = None):
    """Load (once) and return the shared library handle."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = Path(path) if path else LIB_PATH
        if not p.exists():
            raise RuntimeError(
                f"libstk_sm100.so not found at {p}. Build it with `python -m strict_topk_overlap_b200.build` "
                "(needs nvcc); there is no CPU fallback.")
        lib = C.CDLL(str(p))
        for name, (res, args) in _SIGS.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.stk_abi_version() != 1:
            raise RuntimeError("libstk_sm100.so ABI version mismatch")
        _lib = lib
        return lib


def set_status_tensor(t: torch.Tensor | None):
    """Route device-detected data faults of later calls into ``t`` (int32, >= 1 element)."""
    global _status
    if t is not None and (t.dtype != torch.int32 or not t.is_cuda):
        raise ValueError("status tensor must be a CUDA int32 tensor")
    _status = t


def status_ptr() -> int | None:
    return _status.data_ptr() if _status is not None else None


def check(rc: int, what: str):
    if rc != 0:
        msg = load().stk_last_error().decode(errors="replace")
        raise RuntimeError(f"{what} failed (code {rc}): {msg}")


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {t.dtype}; expected float32, float16 or bfloat16") from None


def id_is64(t: torch.Tensor) -> int:
    if t.dtype == torch.int64:
        return 1
    if t.dtype == torch.int32:
        return 0
    raise ValueError("block ids must be int32 or int64")


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def kv_struct(k: torch.Tensor, v: torch.Tensor, *, page_table=None, block_offsets=None, page_size=0,
              hkv=None, n=None, b=None, d=None, kv_request_stride=0) -> StkKV:
    """Describe a dense [Hkv, N, B, D] or paged [pages, Hkv, page, D] KV cache."""
    if k.dtype != v.dtype:
        raise ValueError("K and V must share a dtype")
    if page_table is None:
        hkv_, n_, b_, d_ = k.shape[-4:]
    else:
        hkv_, n_, b_, d_ = k.shape[1], 0, b, k.shape[3]
    return StkKV(k.data_ptr(), v.data_ptr(), dtype_code(k), int(hkv if hkv is not None else hkv_),
                 int(n if n is not None else n_), int(b if b is not None else b_), int(d if d is not None else d_),
                 ptr(page_table), ptr(block_offsets), int(page_size), int(kv_request_stride))


def sm_count(device: torch.device) -> int:
    return load().stk_device_sm_count(device.index if device.index is not None else torch.cuda.current_device())
