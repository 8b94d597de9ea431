"""Canary-padded output buffers: an epoch writes exactly its documented
outputs and nothing past them, through both C entry points.  Every output
buffer is over-allocated, the tail filled with a canary pattern, and checked
after the call (host-side overrun detection in place of a sanitizer, which
is closed on this pool)."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from scenario import decode_inputs, make_scenario, prefill_epochs

pytestmark = pytest.mark.gpu

PAD = 64
_CTYPES = {np.dtype(np.int64): ctypes.c_int64, np.dtype(np.int32): ctypes.c_int32,
           np.dtype(np.float32): ctypes.c_float, np.dtype(np.uint8): ctypes.c_uint8}


def _p(a: np.ndarray):
    """A typed ctypes pointer to a numpy buffer."""
    return a.ctypes.data_as(ctypes.POINTER(_CTYPES[a.dtype]))


def _padded(shape, dtype, fill):
    n = int(np.prod(shape))
    buf = np.full(n + PAD, fill, dtype=dtype)
    return buf, buf[:n].reshape(shape)


def test_cruise_epoch_run_stays_inside_its_outputs(cuda_ok):
    from cruise_b200.engine import EpochEngine
    from cruise_b200.model_config import TINY

    engine = EpochEngine("tiny")
    engine.init_synthetic(0)
    sc = make_scenario(vocab=TINY.vocab, seed=9, active_rows=(1, 1, 0, 1), k=8, budget=(8, 8))
    for inputs in prefill_epochs(sc, TINY.block_size, TINY.vocab):
        assert engine.run(**inputs).status == 0
    inp = decode_inputs(sc, TINY.block_size)
    canary_i64, canary_i32, canary_f32 = np.int64(0x5A5A5A5A5A5A5A5A), np.int32(0x3C3C3C3C), np.float32(-7.25e30)
    hist_buf, _ = _padded((8, 4), np.int64, canary_i64)
    ctrl_buf, _ = _padded((28,), np.int32, canary_i32)
    logit_buf, _ = _padded((8, 4, TINY.vocab), np.float32, canary_f32)
    args = [np.ascontiguousarray(inp[k]) for k in ("token", "position", "seq_len", "slot", "active", "block_table")]
    control = np.ascontiguousarray(inp["control"])
    rc = engine.lib.cruise_epoch_run(engine.handle, *(_p(a) for a in args), None, _p(control), None, 0, None,
                                     _p(hist_buf), _p(ctrl_buf), _p(logit_buf))
    assert rc == 0 and ctrl_buf[3] == 0
    assert (hist_buf[32:] == canary_i64).all() and (ctrl_buf[28:] == canary_i32).all()
    assert (logit_buf[8 * 4 * TINY.vocab:] == canary_f32).all()
    engine.close()


def test_bridge_execute_stays_inside_its_outputs(cuda_ok):
    from cruise_b200 import _lib

    lib = _lib.load()
    status = ctypes.c_int32(-1)
    handle = lib.resident_epoch_create(b"tiny", None, None, b"synthetic:0", None, ctypes.byref(status))
    assert handle and status.value == 0
    try:
        i64, i32 = np.int64, np.int32
        tokens, _ = _padded((4, 8), i64, i64(0x1111111111111111))
        executed, _ = _padded((4,), i32, i32(0x22222222))
        gens_out, _ = _padded((4,), i32, i32(0x33333333))
        scalars = {name: _padded((1,), i32, i32(0x44444444))[0] for name in
                   ("calls", "status", "feed", "fetch", "commit", "checksum")}
        wides = {name: _padded((1,), i64, i64(0x5555555555555555))[0] for name in ("wall", "cpu", "din", "dout")}
        tok_in = np.array([7, 8, 9, 0], dtype=i64)
        pos_in = np.zeros(4, dtype=i64)
        len_in = np.array([1, 1, 1, 0], dtype=i32)
        eos_in = np.full(4, 4095, dtype=i32)
        gen_in = np.array([1, 2, 3, 0], dtype=i32)
        p = _p
        rc = lib.resident_epoch_execute(
            handle, 3, 8, p(tok_in), p(pos_in), p(len_in), p(eos_in), p(gen_in), p(tokens), p(executed), p(gens_out),
            p(scalars["calls"]), p(scalars["status"]), p(scalars["feed"]), p(scalars["fetch"]), p(scalars["commit"]),
            p(scalars["checksum"]), p(wides["wall"]), p(wides["cpu"]), p(wides["din"]), p(wides["dout"]),
            None, 0, None)
        assert rc == 0 and scalars["status"][0] == 0 and scalars["commit"][0] == 2
        assert (tokens[32:] == i64(0x1111111111111111)).all()
        assert (executed[4:] == i32(0x22222222)).all() and (gens_out[4:] == i32(0x33333333)).all()
        for buf in scalars.values():
            assert (buf[1:] == i32(0x44444444)).all()
        for buf in wides.values():
            assert (buf[1:] == i64(0x5555555555555555)).all()
    finally:
        lib.resident_epoch_destroy(handle)
