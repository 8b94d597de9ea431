"""The C-ABI library loads without a GPU and exports every declared symbol."""

import re
from pathlib import Path

from cruise_b200 import _lib

INCLUDE = Path(__file__).resolve().parents[1] / "include"


def declared_functions() -> set[str]:
    names = set()
    for header in INCLUDE.glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
        names.update(re.findall(r"\b((?:resident_epoch|cruise_epoch|cruise_decoder)_\w+)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    declared = declared_functions()
    assert "resident_epoch_execute" in declared and "cruise_epoch_run" in declared
    for name in sorted(declared):
        assert hasattr(lib, name), name
    assert set(_lib.SIGNATURES) == declared


def test_engine_creation_without_gpu_fails_cleanly():
    import ctypes

    import torch

    if torch.cuda.is_available():
        return
    lib = _lib.load()
    from cruise_b200.model_config import TINY

    status = ctypes.c_int32(-1)
    cfg = TINY.to_c()
    handle = lib.cruise_epoch_create(ctypes.byref(cfg), 0, ctypes.byref(status))
    assert not handle and status.value == 3
    reason = lib.cruise_epoch_last_error(None).decode()
    assert reason.startswith(("cudaSetDevice", "cudaGetDeviceProperties")), reason
