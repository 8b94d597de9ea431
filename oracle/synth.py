"""Seeded weight generator, CPU restatement (test infrastructure only).

The engine generates synthetic weights on the GPU; this module produces the
identical bf16 bit patterns on the CPU so the oracle and the engine run on the
same model.  The algorithm is integer-only up to one correctly rounded fp32
multiply, so it is bit-reproducible on any IEEE machine:

  key_t   = mix(seed * GAMMA + (tensor_id + 1) * KEYMUL)        (mod 2**64)
  h_i     = mix(key_t + (i + 1) * GAMMA)                         (mod 2**64)
  s_i     = sum of the four 16-bit lanes of h_i                  (Irwin-Hall(4))
  value_i = bf16_rne( float32(2 * s_i - 262140) * SCALE_F32 )

``mix`` is the splitmix64 finaliser (Steele, Lea, Flood, "Fast splittable
pseudorandom number generators", OOPSLA 2014).  SCALE_F32 maps the centred sum
to standard deviation ``std`` (0.02 for every tensor, as the workload asks).
The sum of four uniforms approximates N(0, std) (bounded at +-3.46 sigma).
"""

from __future__ import annotations

import math

import numpy as np

GAMMA = np.uint64(0x9E3779B97F4A7C15)
KEYMUL = np.uint64(0xD1B54A32D192ED03)
C1 = np.uint64(0xBF58476D1CE4E5B9)
C2 = np.uint64(0x94D049BB133111EB)
CENTER = 262140  # 4 * 65535


def scale_f32(std: float = 0.02) -> np.float32:
    sigma_centred = 2.0 * math.sqrt(4.0 * (65536.0**2 - 1.0) / 12.0)
    return np.float32(std / sigma_centred)


def _mix(z: np.ndarray) -> np.ndarray:
    z = z ^ (z >> np.uint64(30))
    z = z * C1
    z = z ^ (z >> np.uint64(27))
    z = z * C2
    return z ^ (z >> np.uint64(31))


def tensor_key(seed: int, tensor_id: int) -> np.uint64:
    with np.errstate(over="ignore"):
        z = np.array(
            [np.uint64(seed) * GAMMA + np.uint64(tensor_id + 1) * KEYMUL],
            dtype=np.uint64,
        )
        return _mix(z)[0]


def f32_to_bf16_bits(values: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 (finite inputs)."""
    bits = np.ascontiguousarray(values, dtype=np.float32).view(np.uint32)
    rounding = ((bits >> np.uint32(16)) & np.uint32(1)) + np.uint32(0x7FFF)
    return ((bits + rounding) >> np.uint32(16)).astype(np.uint16)


def synth_bf16_bits(
    seed: int, tensor_id: int, count: int, std: float = 0.02, start: int = 0
) -> np.ndarray:
    """bf16 bit patterns of elements ``start .. start+count`` of one tensor."""
    key = tensor_key(seed, tensor_id)
    index = np.arange(start + 1, start + count + 1, dtype=np.uint64)
    with np.errstate(over="ignore"):
        h = _mix(key + index * GAMMA)
    lanes = (
        (h & np.uint64(0xFFFF))
        + ((h >> np.uint64(16)) & np.uint64(0xFFFF))
        + ((h >> np.uint64(32)) & np.uint64(0xFFFF))
        + (h >> np.uint64(48))
    ).astype(np.int64)
    centred = (2 * lanes - CENTER).astype(np.float32)
    return f32_to_bf16_bits(centred * scale_f32(std))


# -- the same generator in C (oracle/csynth.c), for full-depth models ----------
_CSYNTH = None


def csynth_library():
    """oracle/libcsynth.so, compiled with gcc (OpenMP) when missing or older
    than its source.  Raises when no C compiler is available."""
    global _CSYNTH
    if _CSYNTH is not None:
        return _CSYNTH
    import ctypes
    import os
    import shutil
    import subprocess
    from pathlib import Path

    here = Path(__file__).resolve().parent
    src, lib = here / "csynth.c", here / "libcsynth.so"
    if not lib.exists() or lib.stat().st_mtime < src.stat().st_mtime:
        cc = shutil.which("gcc") or shutil.which("cc")
        if cc is None:
            raise RuntimeError("oracle/csynth.c needs a C compiler (gcc)")
        tmp = lib.with_name(f"libcsynth.so.tmp{os.getpid()}")
        subprocess.run([cc, "-O3", "-fopenmp", "-shared", "-fPIC", "-o", str(tmp), str(src)], check=True)
        os.replace(tmp, lib)
    handle = ctypes.CDLL(str(lib))
    handle.cruise_oracle_synth.argtypes = [ctypes.c_uint64, ctypes.c_int32, ctypes.c_int64, ctypes.c_int64,
                                           ctypes.c_float, ctypes.c_void_p, ctypes.c_int32]
    handle.cruise_oracle_synth.restype = None
    _CSYNTH = handle
    return handle


def synth_bf16_bits_c(seed: int, tensor_id: int, count: int, std: float = 0.02, start: int = 0,
                      threads: int | None = None) -> np.ndarray:
    """:func:`synth_bf16_bits` computed by oracle/csynth.c on ``threads`` host
    threads (default: every core this process may use)."""
    import os

    out = np.empty(count, dtype=np.uint16)
    n = threads or len(os.sched_getaffinity(0))
    csynth_library().cruise_oracle_synth(seed, tensor_id, start, count, float(scale_f32(std)),
                                         out.ctypes.data, n)
    return out
