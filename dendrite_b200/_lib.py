"""ctypes binding of ``libdendrite_b200.so`` (the C ABI in include/dendrite_b200.h).

The library is loaded from the package directory. There is no fallback: if
the shared library is missing or fails to load, importing this module raises,
so no CPU path can stand in for the CUDA kernels.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

# DENDRITE_B200_LIB may point at another build of the same library (e.g. one
# compiled with different flags for an experiment).
_LIB_PATH = Path(os.environ.get("DENDRITE_B200_LIB") or
                 Path(__file__).resolve().parent / "libdendrite_b200.so")

# dd_status -> exception class; mirrors FfiError (crates/dendrite-ffi/src/error.rs:9-30).
DD_OK = 0
DD_ERR_INVALID_ARGUMENT = 1
DD_ERR_CUDA = 2
DD_ERR_NOT_AVAILABLE = 3
DD_ERR_ALLOCATION = 4
DD_ERR_WORKSPACE = 5

DTYPE_F16, DTYPE_BF16, DTYPE_F32, DTYPE_E4M3, DTYPE_MXFP8 = 0, 1, 2, 3, 4
GQA_TILED, GQA_GROUPED = 0, 1


class FfiError(RuntimeError):
    """Base of the errors the C ABI reports (FfiError in the reference)."""

    status = -1


class InvalidArgument(FfiError, ValueError):
    status = DD_ERR_INVALID_ARGUMENT


class CudaError(FfiError):
    status = DD_ERR_CUDA


class NotAvailable(FfiError):
    status = DD_ERR_NOT_AVAILABLE


class AllocationFailed(FfiError, MemoryError):
    status = DD_ERR_ALLOCATION


class WorkspaceTooSmall(InvalidArgument):
    status = DD_ERR_WORKSPACE


_ERRORS = {c.status: c for c in (InvalidArgument, CudaError, NotAvailable, AllocationFailed,
                                 WorkspaceTooSmall)}


class AttnConfig(C.Structure):
    _fields_ = [("num_qo_heads", C.c_int32), ("num_kv_heads", C.c_int32),
                ("head_dim", C.c_int32), ("page_size", C.c_int32), ("kv_dtype", C.c_int32),
                ("q_dtype", C.c_int32), ("gqa_map", C.c_int32), ("num_pages", C.c_int32),
                ("scale", C.c_float)]


class PlanOptions(C.Structure):
    _fields_ = [("share_prefixes", C.c_int32), ("max_chunk_pages", C.c_int32),
                ("use_tensor_cores", C.c_int32), ("cta_pairs", C.c_int32), ("tc_sms", C.c_int32)]


class PlanInfo(C.Structure):
    _fields_ = [("batch_size", C.c_int32), ("num_nodes", C.c_int32), ("num_items", C.c_int32),
                ("max_depth", C.c_int32), ("kv_tokens", C.c_int64),
                ("kv_tokens_flat", C.c_int64), ("workspace_bytes", C.c_size_t),
                ("device_bytes", C.c_size_t), ("kv_tokens_by_kernel", C.c_int64 * 5),
                ("tc_row_tokens", C.c_int64), ("tc_ctas", C.c_int32)]


class QuantConfig(C.Structure):
    _fields_ = [("format", C.c_int32), ("src_dtype", C.c_int32), ("num_kv_heads", C.c_int32),
                ("head_dim", C.c_int32), ("page_size", C.c_int32), ("scale_mode", C.c_int32)]


_VP = C.c_void_p
_I32P = C.POINTER(C.c_int32)
_U32P = C.POINTER(C.c_uint32)
_CFGP = C.POINTER(AttnConfig)
_QCP = C.POINTER(QuantConfig)

# name -> (restype, argtypes). Every symbol declared in include/dendrite_b200.h.
SIGNATURES = {
    "dd_version": (C.c_char_p, []),
    "dd_last_error": (C.c_char_p, []),
    "dd_validate_config": (C.c_int, [_CFGP]),
    "dd_plan_create": (C.c_int, [_CFGP, C.c_int32, _I32P, _U32P, _I32P,
                                 C.POINTER(PlanOptions), C.POINTER(_VP)]),
    "dd_plan_create_prefill": (C.c_int, [_CFGP, C.c_int32, _I32P, _U32P, _I32P, _I32P,
                                         C.POINTER(PlanOptions), C.POINTER(_VP)]),
    "dd_plan_destroy": (None, [_VP]),
    "dd_plan_rebuild": (C.c_int, [C.c_void_p, C.c_int32, _I32P, _U32P, _I32P]),
    "dd_plan_advance": (C.c_int, [C.c_void_p, _I32P, _U32P]),
    "dd_selftest_wait": (C.c_int, [_VP, C.c_uint64, _VP]),
    "dd_plan_get_info": (C.c_int, [_VP, C.POINTER(PlanInfo)]),
    "dd_plan_upload": (C.c_int, [_VP, _VP, C.c_size_t, _VP]),
    "dd_plan_export_nodes": (C.c_int, [_VP, _I32P, _I32P, _I32P, _I32P, _I32P, _I32P, _U32P,
                                       _I32P]),
    "dd_cascade_decode": (C.c_int, [_CFGP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, C.c_size_t, _VP]),
    "dd_cascade_decode_shards": (C.c_int, [_CFGP, _VP, _VP, _VP, _VP, _VP, C.c_int32, C.c_int32,
                                           C.c_int32, C.c_int32, _VP, _VP, C.c_size_t, _VP]),
    "dd_decode_paged_workspace_size": (C.c_size_t, [_CFGP, C.c_int32, C.c_int32]),
    "dd_decode_paged": (C.c_int, [_CFGP, C.c_int32, C.c_int32, _VP, _VP, _VP, _VP, _VP, _VP,
                                  _VP, _VP, _VP, C.c_size_t, _VP]),
    "dd_workspace_status": (C.c_int, [_VP, _VP, _U32P, _U32P]),
    "dd_decode_paged_static": (C.c_int, [_CFGP, C.c_int32, C.c_int32, _VP, _VP, _VP, _VP, _VP, _VP,
                                         _VP, _VP, _VP]),
    "dd_decode_paged_static_status": (C.c_int, [_VP, _U32P, _U32P]),
    "dd_merge_states": (C.c_int, [C.c_int32, C.c_int32, _VP, _VP, _VP, _VP, _VP, _VP, _VP]),
    "dd_append_kv": (C.c_int, [_CFGP, _VP, C.c_uint32, C.c_int32, C.c_int32, _VP, _VP, _VP]),
    "dd_quantize_workspace_size": (C.c_size_t, [_QCP]),
    "dd_quantize_kv_pages": (C.c_int, [_QCP, _VP, C.c_int64, _VP, _VP, _VP, C.c_size_t, _VP]),
    "dd_dequantize_kv_pages": (C.c_int, [_QCP, _VP, _VP, C.c_int64, _VP, C.c_int32, _VP]),
    "dd_append_kv_batch": (C.c_int, [_CFGP, _VP, _VP, C.c_int32, _VP, _VP, _VP, _VP, C.c_int32, _VP, _VP]),
    "dd_copy_pages": (C.c_int, [_CFGP, _VP, _VP, C.c_int32, _VP, _VP, _VP, _VP]),
    "dd_scatter_head_shards": (C.c_int, [_CFGP, C.c_int32, C.c_int32, _VP, _VP, _VP]),
    "dd_allgather_heads": (C.c_int, [_VP, _CFGP, C.c_int32, C.c_int32, _VP, _VP, _VP, _VP]),
    "dd_tc_available": (C.c_int, []),
    "dd_launch_count": (C.c_uint64, []),
    "dd_profile_enable": (None, [C.c_int]),
    "dd_profile_read": (C.c_int, [C.POINTER(C.c_double), C.POINTER(C.c_int64), C.c_int32]),
}

PROFILE_KINDS = ("attn_simple", "attn_mma", "attn_tc", "merge", "quant", "other")


def _load() -> C.CDLL:
    if not _LIB_PATH.exists():
        raise ImportError(
            f"{_LIB_PATH.name} is not built: run `python dendrite_b200/build.py` "
            "(the CUDA extension is required; there is no CPU fallback)")
    lib = C.CDLL(str(_LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def check(rc: int, what: str = "") -> None:
    """Raise the FfiError subclass matching a non-zero dd_status."""
    if rc == DD_OK:
        return
    msg = lib.dd_last_error().decode(errors="replace")
    raise _ERRORS.get(rc, FfiError)(f"{what}: {msg}" if what else msg)


def version() -> str:
    return lib.dd_version().decode()


def launch_count() -> int:
    """Kernels launched by the library since it was loaded."""
    return int(lib.dd_launch_count())


def profile_enable(on: bool = True) -> None:
    lib.dd_profile_enable(1 if on else 0)


def profile_read() -> dict:
    """{kernel family: (total ms, launches)} since the previous read."""
    n = len(PROFILE_KINDS)
    ms = (C.c_double * n)()
    cnt = (C.c_int64 * n)()
    check(lib.dd_profile_read(ms, cnt, n), "dd_profile_read")
    return {k: (ms[i], cnt[i]) for i, k in enumerate(PROFILE_KINDS)}
