"""ctypes binding of libcsaq_b200.so, the C ABI declared in include/csaq_b200.h.

The shared library is built in-tree (``python csaq-quant_b200/build.py``) and
loaded from ``csaq/lib/libcsaq_b200.so``. There is no fallback: a missing
library, a CPU-only process or a failing launch raises.
"""

from __future__ import annotations

import ctypes
import os
import threading
from typing import Iterable, List, Optional, Sequence

import torch

# CSAQ_LIB=checked loads the checked build (index guards, csaq_guard_report)
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib",
                        "libcsaq_b200_checked.so" if os.environ.get("CSAQ_LIB") == "checked" else "libcsaq_b200.so")

CSAQ_OK = 0
DT_F32, DT_F16, DT_BF16 = 0, 1, 2
MAX_TIERS = 16

_DTYPES = {torch.float32: DT_F32, torch.float16: DT_F16, torch.bfloat16: DT_BF16}

c_i64 = ctypes.c_int64
c_int = ctypes.c_int
c_vp = ctypes.c_void_p


class CsaqTier(ctypes.Structure):
    """Mirror of ``csaq_tier`` (include/csaq_b200.h)."""

    _fields_ = [
        ("bits", ctypes.c_int32),
        ("n_rows", ctypes.c_int32),
        ("group_size", ctypes.c_int32),
        ("n_groups", ctypes.c_int32),
        ("row_bytes", c_i64),
        ("codes", c_vp),
        ("scales", c_vp),
        ("zps", c_vp),
        ("out_rows", c_vp),
        ("blocks", c_vp),
        ("y", c_vp),
        ("ldy", c_i64),
        ("bias", c_vp),
        ("residual", c_vp),
        ("ldr", c_i64),
    ]


class CsaqGemvExt(ctypes.Structure):
    """Mirror of ``csaq_gemv_ext`` (include/csaq_b200.h)."""

    _fields_ = [
        ("silu_tiers", ctypes.c_uint32),
        ("x_mul", c_vp),
    ]


MAX_RANKS = 8
IPC_HANDLE_BYTES = 64


class CsaqP2PGroup(ctypes.Structure):
    """Mirror of ``csaq_p2p_group`` (include/csaq_b200.h)."""

    _fields_ = [
        ("n_ranks", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("parts", c_vp * MAX_RANKS),
        ("flags", c_vp * MAX_RANKS),
        ("seq", c_vp),
        ("ticket", c_vp),
        ("err", c_vp),
    ]


# name -> (restype, argtypes)
_SIGNATURES = {
    "csaq_version": (ctypes.c_char_p, []),
    "csaq_status_string": (ctypes.c_char_p, [c_int]),
    "csaq_last_cuda_error": (c_int, []),
    "csaq_checked_build": (c_int, []),
    "csaq_guard_report": (c_int, [c_vp, c_vp, c_vp, c_vp]),
    "csaq_guard_clear": (c_int, []),
    "csaq_packed_row_bytes": (c_i64, [c_i64, c_int]),
    "csaq_group_scales": (c_int, [c_vp, c_int, c_i64, c_i64, c_i64, c_int, c_i64, c_vp, c_vp, c_vp, c_vp]),
    "csaq_quant_pack_rows": (c_int, [c_vp, c_int, c_i64, c_i64, c_i64, c_int, c_i64, c_vp, c_vp, c_i64,
                                     c_int, c_vp, c_int, c_vp, c_vp]),
    "csaq_quant_pack": (c_int, [c_vp, c_int, c_i64, c_i64, c_i64, c_int, c_i64, c_vp, c_vp, c_vp, c_vp]),
    "csaq_cast_f16": (c_int, [c_vp, c_int, c_i64, c_i64, c_i64, c_vp, c_vp]),
    "csaq_pack": (c_int, [c_vp, c_int, c_i64, c_i64, c_vp, c_vp]),
    "csaq_unpack": (c_int, [c_vp, c_int, c_i64, c_i64, c_vp, c_vp]),
    "csaq_float_to_int": (c_int, [c_vp, c_vp, c_vp, c_int, c_i64, c_i64, c_vp, c_vp]),
    "csaq_dequant": (c_int, [c_vp, c_vp, c_vp, c_int, c_i64, c_i64, c_i64, c_int, c_int, c_vp, c_vp]),
    "csaq_qgemv_wait_timeouts": (c_int, [ctypes.POINTER(c_i64)]),
    "csaq_qgemm": (c_int, [ctypes.POINTER(CsaqTier), c_int, c_i64, c_vp, c_int, c_i64, c_i64, c_vp]),
    "csaq_qgemm_wait_timeouts": (c_int, [ctypes.POINTER(c_i64)]),
    "csaq_qgemv": (c_int, [ctypes.POINTER(CsaqTier), c_int, c_i64, c_vp, c_int, c_i64, c_i64, c_vp]),
    "csaq_qgemv_simt": (c_int, [ctypes.POINTER(CsaqTier), c_int, c_i64, c_vp, c_int, c_i64, c_i64, c_vp]),
    "csaq_qgemv_ext": (c_int, [ctypes.POINTER(CsaqTier), c_int, c_i64, c_vp, c_int, c_i64, c_i64,
                               ctypes.POINTER(CsaqGemvExt), c_vp]),
    "csaq_tile_blocks_bytes": (c_i64, [c_int, c_i64, c_i64]),
    "csaq_repack_tiles": (c_int, [ctypes.POINTER(CsaqTier), c_i64, c_vp, c_vp]),
    "csaq_act_mask": (c_int, [c_vp, c_int, c_i64, c_i64, c_i64, c_int, ctypes.c_float, c_i64, c_vp, c_vp,
                              c_i64, c_i64, c_vp]),
    "csaq_coact_counts": (c_int, [c_vp, c_i64, c_i64, c_i64, c_vp, c_i64, c_vp, c_vp]),
    "csaq_jaccard_bits": (c_int, [c_vp, c_i64, c_vp, c_i64, ctypes.c_float, c_vp, c_i64, c_vp]),
    "csaq_greedy_cliques": (c_int, [c_vp, c_i64, c_i64, c_vp, c_vp, c_vp]),
    "csaq_salience_accum": (c_int, [c_vp, c_vp, c_int, c_i64, c_vp, c_vp]),
    "csaq_salience_finalize": (c_int, [c_vp, c_i64, c_i64, c_vp]),
    "csaq_rmsnorm": (c_int, [c_vp, c_i64, c_vp, c_vp, c_i64, c_i64, c_i64, ctypes.c_float, c_int, c_vp]),
    "csaq_rope_kv": (c_int, [c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_i64, c_i64, c_i64, c_i64,
                             c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_int, c_vp]),
    "csaq_attention_workspace_floats": (c_i64, [c_i64, c_i64, c_i64, c_i64, c_i64, c_i64]),
    "csaq_decode_attention": (c_int, [c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64,
                                      ctypes.c_float, c_vp, c_vp, c_vp, c_int, c_vp]),
    "csaq_decode_attention_rope": (c_int, [c_vp, c_vp, c_vp, c_i64, c_vp, c_i64, c_i64, c_i64, c_i64, c_i64,
                                           c_vp, c_vp, c_vp, c_vp, c_i64, ctypes.c_float, c_vp, c_vp, c_vp,
                                           c_int, c_vp]),
    "csaq_decode_attention_static": (c_int, [c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64,
                                             ctypes.c_float, c_vp, c_int, c_vp]),
    "csaq_rank_sum": (c_int, [c_vp, c_int, c_i64, c_i64, c_vp, c_i64, c_i64, c_i64, c_int, c_int, c_vp]),
    "csaq_argmax_parts": (c_int, [c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_vp, c_int, c_vp]),
    "csaq_sample_rows": (c_int, [c_vp, c_int, c_i64, c_i64, c_i64, c_i64, ctypes.c_float, ctypes.c_float,
                                 ctypes.c_uint64, c_vp, c_vp, c_int, c_vp]),
    "csaq_spec_sample_verify": (c_int, [c_vp, c_vp, c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_i64,
                                        ctypes.c_float, ctypes.c_float, ctypes.c_uint64, c_vp, c_vp, c_int, c_vp]),
    "csaq_p2p_alloc": (c_int, [c_i64, ctypes.POINTER(c_vp)]),
    "csaq_p2p_free": (c_int, [c_vp]),
    "csaq_ipc_handle": (c_int, [c_vp, c_vp]),
    "csaq_ipc_open": (c_int, [c_vp, ctypes.POINTER(c_vp)]),
    "csaq_ipc_close": (c_int, [c_vp]),
    "csaq_tp_exchange_sum": (c_int, [ctypes.POINTER(CsaqP2PGroup), c_i64, c_i64, c_vp, c_i64, c_i64, c_i64, c_int,
                                     c_vp]),
    "csaq_tp_exchange_sum_rmsnorm": (c_int, [ctypes.POINTER(CsaqP2PGroup), c_i64, c_i64, c_vp, c_i64, c_i64, c_i64,
                                             c_vp, c_vp, c_i64, ctypes.c_float, c_int, c_vp]),
    "csaq_p2p_errors": (c_int, [ctypes.POINTER(CsaqP2PGroup), ctypes.POINTER(c_i64)]),
    "csaq_p2p_set_spin_limit": (c_int, [c_i64]),
    "csaq_silu_mul": (c_int, [c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_i64, c_i64, c_int, c_vp]),
    "csaq_spec_accept": (c_int, [c_vp, c_vp, c_i64, c_i64, c_vp, c_vp, c_vp, c_i64, c_vp, c_vp, c_vp, c_vp, c_vp]),
    "csaq_greedy_commit": (c_int, [c_vp, c_i64, c_vp, c_vp, c_vp, c_i64, c_vp, c_vp, c_vp]),
}

_lib = None
_lock = threading.Lock()


def exported_symbols() -> List[str]:
    return list(_SIGNATURES)


def lib() -> ctypes.CDLL:
    """Load the library once; raise if it is missing or incomplete."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"csaq-b200: native library not found at {LIB_PATH}. Build it with "
                "`python csaq-quant_b200/build.py` (nvcc, sm_100a). There is no CPU fallback.")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
        return L


def register(name: str, restype, argtypes) -> None:
    """Declare an additional entry point (used by modules with their own kernels)."""
    _SIGNATURES[name] = (restype, argtypes)
    if _lib is not None:
        fn = getattr(_lib, name)
        fn.restype = restype
        fn.argtypes = argtypes


class CsaqError(RuntimeError):
    pass


def check(rc: int, what: str) -> None:
    if rc != CSAQ_OK:
        L = lib()
        msg = L.csaq_status_string(rc).decode()
        cu = L.csaq_last_cuda_error()
        raise CsaqError(f"csaq-b200 {what} failed: {msg} (status {rc}, cudaError {cu})")


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPES[dt]
    except KeyError:
        raise TypeError(f"csaq-b200: unsupported dtype {dt}") from None


def require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("csaq-b200 kernels run on CUDA tensors only (no CPU path)")


def cuda_device() -> torch.device:
    if not torch.cuda.is_available():
        raise RuntimeError("csaq-b200 needs a CUDA device (B200, sm_100a); none is available")
    return torch.device("cuda", torch.cuda.current_device())


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def tier_array(tiers: Sequence[CsaqTier]):
    if not 1 <= len(tiers) <= MAX_TIERS:
        raise ValueError(f"csaq-b200: 1..{MAX_TIERS} tiers per launch, got {len(tiers)}")
    arr = (CsaqTier * len(tiers))()
    for i, t in enumerate(tiers):
        arr[i] = t
    return arr


def qgemv(descs, K: int, x: torch.Tensor, M: int, stream: int = None) -> None:
    """Launch csaq_qgemv on a list of ctypes tier descriptors."""
    arr = tier_array(descs) if isinstance(descs, list) else descs
    st = stream if stream is not None else stream_of(x)
    check(lib().csaq_qgemv(arr, len(descs), K, x.data_ptr(), dtype_code(x.dtype), M, x.stride(0), st), "qgemv")


def qgemm(descs, K: int, x: torch.Tensor, M: int, stream: int = None) -> None:
    """Launch csaq_qgemm (the many-token tensor-core path) on tier descriptors."""
    arr = tier_array(descs) if isinstance(descs, list) else descs
    st = stream if stream is not None else stream_of(x)
    check(lib().csaq_qgemm(arr, len(descs), K, x.data_ptr(), dtype_code(x.dtype), M, x.stride(0), st), "qgemm")
