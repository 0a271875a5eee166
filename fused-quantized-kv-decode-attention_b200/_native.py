"""ctypes binding of ``libfqkv_b200.so`` (the C ABI in ``include/fqkv_b200.h``).

The library is built in-tree by ``build.py`` next to this file.  There is no
CPU fallback: if the library is missing or fails to load, every operator
raises ``NativeLibraryError``.
"""
from __future__ import annotations

import ctypes
import pathlib
import threading

LIB_PATH = pathlib.Path(__file__).resolve().with_name("libfqkv_b200.so")

# status codes (fqkv_status_t)
OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_MISALIGNED = 2
ERR_CUDA = 3
ERR_UNSUPPORTED_DEVICE = 4
ERR_DEVICE_TIMEOUT = 5
ERR_PEER = 6

KV_F16, KV_INT8, KV_INT4 = 0, 1, 2

# fqkv_set_split_mode
SPLIT_AUTO, SPLIT_COMBINE, SPLIT_CLUSTER = 0, 1, 2

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_SZ = ctypes.c_size_t
_INT = ctypes.c_int

TP_MAX_RANKS = 8


class TpOut(ctypes.Structure):
    """fqkv_tp_out_t: where a tensor-parallel decode call sends its output."""
    _fields_ = [("world", ctypes.c_int32), ("rank", ctypes.c_int32), ("dst_offset", ctypes.c_int64),
                ("dst", ctypes.c_void_p * TP_MAX_RANKS), ("counters", ctypes.c_void_p * TP_MAX_RANKS)]


# name -> (restype, argtypes); the same set of symbols the header declares.
SIGNATURES = {
    "fqkv_last_error": (ctypes.c_char_p, []),
    "fqkv_version": (ctypes.c_char_p, []),
    "fqkv_device_status": (_INT, [ctypes.POINTER(_INT), _INT]),
    "fqkv_set_wait_timeout_ms": (None, [ctypes.c_uint32]),
    "fqkv_debug_skip_loads": (None, [_INT]),
    "fqkv_set_split_mode": (_INT, [_INT]),
    "fqkv_decode_workspace_bytes": (_SZ, [_INT, _I64, _I64, _I64, _I64, _I64]),
    "fqkv_device_info": (_INT, [ctypes.POINTER(ctypes.c_int32), ctypes.c_int32]),
    "fqkv_decode_plan": (_INT, [_INT, _I64, _I64, _I64, _I64, _I64, _SZ, ctypes.POINTER(ctypes.c_int32)]),
    "fqkv_decode_attn_fp16_mw": (_INT, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _P, _SZ, _P]),
    "fqkv_decode_attn_int8_mw": (_INT, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _P, _SZ, _P]),
    "fqkv_decode_attn_int4": (_INT, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _P, _SZ, _P]),
    "fqkv_decode_attn_gqa": (_INT, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _SZ, _P]),
    "fqkv_decode_attn_gqa_kvcache": (_INT, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P, _SZ, _P]),
    "fqkv_decode_attn_gqa_int8": (_INT, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P, _SZ, _P]),
    "fqkv_decode_attn_gqa_int8_kvcache": (_INT, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P,
                                                 _SZ, _P]),
    "fqkv_quantize_int8_into_cache": (_INT, [_P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P, _P]),
    "fqkv_quantize_int4_into_cache": (_INT, [_P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P, _P]),
    "fqkv_gqa_sk_fast": (_INT, [_P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _P]),
    "fqkv_gqa_sk_fast_static_scratch": (_INT, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _P]),
    "fqkv_quantize_int8_per_token": (_INT, [_P, _P, _P, _I64, _I64, _P]),
    "fqkv_quantize_int4_per_token": (_INT, [_P, _P, _P, _I64, _I64, _P]),
    "fqkv_rope_qkv_append": (_INT, [ctypes.c_int32, ctypes.c_int32, _P, _I64, _P, _P, _I64, _I64, _P, _P, _P, _P, _P,
                                    _P, _I64, _I64, _I64, _I64, _I64, _P]),
    "fqkv_add_rmsnorm": (_INT, [ctypes.c_int32, _P, _P, _P, _P, _I64, _I64, ctypes.c_float, _P]),
    "fqkv_silu_mul": (_INT, [ctypes.c_int32, _P, _P, _I64, _I64, _I64, _P]),
    "fqkv_gemv": (_INT, [ctypes.c_int32, ctypes.c_int32, _P, _P, _P, _P, _I64, _I64, _I64, _P]),
    "fqkv_gemv_swiglu": (_INT, [ctypes.c_int32, _P, _P, _P, _P, _I64, _I64, _I64, _P]),
    "fqkv_gemv_rope_append": (_INT, [ctypes.c_int32, _P, _P, _P, _I64, _P, _P, _I64, _I64, _P, _P, _P, _P,
                                     _I64, _I64, _I64, _I64, _P]),
    "fqkv_argmax_scratch_bytes": (_SZ, [_I64]),
    "fqkv_argmax": (_INT, [ctypes.c_int32, _P, _I64, _I64, _P, _P, _P]),
    "fqkv_decode_attn_kvcache_out": (_INT, [ctypes.c_int32, ctypes.c_int32, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64,
                                            _I64, _I64, _I64, _P, _P, _SZ, _P]),
    "fqkv_decode_attn_kvcache_tp": (_INT, [ctypes.c_int32, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _P,
                                           _P, _SZ, ctypes.POINTER(TpOut), _P]),
    "fqkv_tp_arrivals": (_I64, [ctypes.c_int32, _I64, _I64, _I64, _I64, _I64, _SZ]),
    "fqkv_tp_wait": (_INT, [_P, ctypes.c_int32, ctypes.c_uint64, _P, _P]),
    "fqkv_ipc_alloc": (_INT, [_SZ, ctypes.POINTER(_P), _P]),
    "fqkv_ipc_open": (_INT, [_P, ctypes.POINTER(_P)]),
    "fqkv_ipc_close": (_INT, [_P]),
    "fqkv_ipc_free": (_INT, [_P]),
}


class NativeLibraryError(RuntimeError):
    """The native library is missing or could not be loaded."""


_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise NativeLibraryError(
                    f"{LIB_PATH.name} is not built; run build.py in {LIB_PATH.parent} "
                    "(there is no CPU fallback)")
            try:
                handle = ctypes.CDLL(str(LIB_PATH))
            except OSError as exc:  # pragma: no cover - depends on the box
                raise NativeLibraryError(f"cannot load {LIB_PATH}: {exc}") from exc
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def last_error() -> str:
    msg = lib().fqkv_last_error()
    return msg.decode() if msg else ""


def check(rc: int, op: str) -> None:
    """Raise RuntimeError (as the reference's TORCH_CHECK does) on a non-zero status."""
    if rc != OK:
        raise RuntimeError(f"{op}: {last_error()} [fqkv status {rc}]")
