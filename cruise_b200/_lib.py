"""ctypes binding of ``libcruise_epoch.so`` (the C ABI in include/cruise_epoch.h).

The library is built in-tree by :mod:`cruise_b200.build`.  There is no
fallback: if the shared library is missing or fails to load, every engine
call raises.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

from .model_config import CruiseModelConfigC

LIBRARY_ENV = "VLLM_ASCEND_RESIDENT_EPOCH_LIBRARY"
_DEFAULT = Path(__file__).resolve().parent / "libcruise_epoch.so"

i32p = ctypes.POINTER(ctypes.c_int32)
i64p = ctypes.POINTER(ctypes.c_int64)
u8p = ctypes.POINTER(ctypes.c_uint8)
f32p = ctypes.POINTER(ctypes.c_float)

# symbol -> (restype, argtypes); the exported surface of include/cruise_epoch.h
SIGNATURES = {
    "resident_epoch_create": (
        ctypes.c_void_p,
        [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p, i32p],
    ),
    "resident_epoch_execute": (
        ctypes.c_int32,
        [
            ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32,
            i64p, i64p, i32p, i32p, i32p,
            i64p, i32p, i32p,
            i32p, i32p, i32p, i32p, i32p, i32p,
            i64p, i64p, i64p, i64p,
            ctypes.c_char_p, ctypes.c_uint64, ctypes.c_void_p,
        ],
    ),
    "resident_epoch_destroy": (None, [ctypes.c_void_p]),
    "resident_epoch_prefill": (ctypes.c_int32, [ctypes.c_void_p, i64p, i32p, ctypes.c_int32]),
    "cruise_epoch_preset": (ctypes.c_int32, [ctypes.c_char_p, ctypes.POINTER(CruiseModelConfigC)]),
    "cruise_epoch_create": (ctypes.c_void_p, [ctypes.POINTER(CruiseModelConfigC), ctypes.c_int32, i32p]),
    "cruise_epoch_destroy": (None, [ctypes.c_void_p]),
    "cruise_epoch_create_tp": (
        ctypes.c_void_p, [ctypes.POINTER(CruiseModelConfigC), ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, i32p]
    ),
    "cruise_epoch_tp_handle": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_void_p]),
    "cruise_epoch_tp_connect": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_void_p]),
    "cruise_epoch_tp_shard": (
        ctypes.c_int32, [ctypes.POINTER(CruiseModelConfigC), ctypes.c_int32, ctypes.c_int32, i32p]
    ),
    "cruise_epoch_init_synthetic": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_double]),
    "cruise_epoch_set_weight": (
        ctypes.c_int32, [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_void_p, ctypes.c_uint64]
    ),
    "cruise_epoch_get_weight": (
        ctypes.c_int32, [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_void_p, ctypes.c_uint64]
    ),
    "cruise_epoch_set_rope_table": (
        ctypes.c_int32, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint64]
    ),
    "cruise_epoch_read_kv": (
        ctypes.c_int32, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint64]
    ),
    "cruise_epoch_write_kv": (
        ctypes.c_int32, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint64]
    ),
    "cruise_epoch_run": (
        ctypes.c_int32,
        [
            ctypes.c_void_p, i64p, i64p, i32p, i32p, i32p, i32p, u8p, i32p,
            ctypes.c_void_p, ctypes.c_uint64, i64p, i64p, i32p, f32p,
        ],
    ),
    "cruise_epoch_run_noalloc": (
        ctypes.c_int32, [ctypes.c_void_p, i64p, i64p, i32p, i32p, i32p, i32p, i32p, i64p, i32p],
    ),
    "cruise_decoder_step": (
        ctypes.c_int32,
        [ctypes.c_void_p, i64p, i64p, i32p, ctypes.c_void_p, i32p, i32p, i32p, ctypes.c_void_p, u8p, f32p, i64p],
    ),
    "cruise_epoch_last_timing": (
        ctypes.c_int32, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_double), i32p]
    ),
    "cruise_epoch_set_trace": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_int32]),
    "cruise_epoch_read_trace": (
        ctypes.c_int32, [ctypes.c_void_p, ctypes.c_int32, ctypes.POINTER(ctypes.c_uint64), ctypes.c_int32]
    ),
    "cruise_epoch_read_trace_cta": (
        ctypes.c_int32, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint32), ctypes.c_int32, i32p]
    ),
    "cruise_epoch_last_error": (ctypes.c_char_p, [ctypes.c_void_p]),
    "cruise_epoch_prefill": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32]),
    "cruise_epoch_stream_enable": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_int32]),
    "cruise_epoch_stream_next_id": (ctypes.c_uint32, [ctypes.c_void_p]),
    "cruise_epoch_stream_poll": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p]),
}

_LIB: ctypes.CDLL | None = None


def library_path() -> Path:
    override = os.getenv(LIBRARY_ENV)
    return Path(override).resolve() if override else _DEFAULT


def load() -> ctypes.CDLL:
    """Loads and binds the engine library (raises if it is missing)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    path = library_path()
    if not path.is_file():
        raise RuntimeError(
            f"CUDA engine library {path} is missing: build it with `python -m cruise_b200.build` "
            "(there is no CPU fallback)"
        )
    lib = ctypes.CDLL(str(path))
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    _LIB = lib
    return lib
