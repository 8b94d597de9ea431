"""The allocation-free epoch entry point against the regular one.

``cruise_epoch_run_noalloc`` is for callers that must not allocate device
memory once they serve (a worker that handed its HBM to its own KV pool at
start-up, or a runtime that forbids allocation after warm-up).  It runs the
same epoch kernel with its scratch in the library's static device array
instead of the engine's allocation.  Two engines with the same seeded weights
and the same prefilled prompts run two greedy epochs in a row, one through
``cruise_epoch_run`` and one through the allocation-free call (C ABI via
ctypes): token history, the 28-word control output and both KV caches must be
bit-identical (the same deterministic kernel on the same inputs), and the
device's free memory must not move across an allocation-free call.  Both the
tiny model and the 7B geometry (two layers; its scratch is about 300 KB of
the 1 MiB array) are run.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from scenario import BATCH, compute_slot, decode_inputs, make_scenario, prefill_epochs

pytestmark = pytest.mark.gpu


def _p(arr: np.ndarray, ctype):
    return arr.ctypes.data_as(ctypes.POINTER(ctype))


def run_noalloc(engine, inputs: dict) -> tuple[int, np.ndarray, np.ndarray]:
    cfg = engine.config
    token = np.ascontiguousarray(np.asarray(inputs["token"], dtype=np.int64).reshape(BATCH))
    position = np.ascontiguousarray(np.asarray(inputs["position"], dtype=np.int64).reshape(BATCH))
    seq_len = np.ascontiguousarray(np.asarray(inputs["seq_len"], dtype=np.int32).reshape(BATCH))
    slot = np.ascontiguousarray(np.asarray(inputs["slot"], dtype=np.int32).reshape(BATCH))
    active = np.ascontiguousarray(np.asarray(inputs["active"], dtype=np.int32).reshape(BATCH))
    block_table = np.ascontiguousarray(
        np.asarray(inputs["block_table"], dtype=np.int32).reshape(BATCH * cfg.blocks_per_row))
    control = np.ascontiguousarray(np.asarray(inputs["control"], dtype=np.int32).reshape(11))
    history = np.empty((8, BATCH), dtype=np.int64)
    control_out = np.empty(28, dtype=np.int32)
    rc = engine.lib.cruise_epoch_run_noalloc(
        engine.handle, _p(token, ctypes.c_int64), _p(position, ctypes.c_int64), _p(seq_len, ctypes.c_int32),
        _p(slot, ctypes.c_int32), _p(active, ctypes.c_int32), _p(block_table, ctypes.c_int32),
        _p(control, ctypes.c_int32), _p(history, ctypes.c_int64), _p(control_out, ctypes.c_int32),
    )
    return rc, history, control_out


def next_epoch(inputs: dict, history: np.ndarray, block_size: int, block_table: np.ndarray, eos: list[int]):
    """Inputs of the epoch that continues every row after ``history``."""
    token = np.array(inputs["token"], dtype=np.int64)
    position = np.array(inputs["position"], dtype=np.int64)
    active = np.array(inputs["active"], dtype=np.int32)
    for row in range(BATCH):
        if not active[row]:
            continue
        emitted = [int(t) for t in history[:, row] if t >= 0]
        token[row] = emitted[-1]
        position[row] += len(emitted)
        if emitted[-1] == eos[row]:
            active[row] = 0
    seq_len = (position + 1).astype(np.int32)
    for row in range(BATCH):
        if not inputs["active"][row]:
            seq_len[row] = inputs["seq_len"][row]
    slot = np.array([compute_slot(block_table, block_size, r, int(position[r])) for r in range(BATCH)],
                    dtype=np.int32)
    control = np.array(inputs["control"], dtype=np.int32)
    return dict(token=token, position=position, seq_len=seq_len, slot=slot, active=active,
                block_table=inputs["block_table"], control=control)


def _free_bytes(device: int) -> int:
    return int(torch.cuda.mem_get_info(device)[0])


def _match_two_epochs(config, seed: int, k: int) -> None:
    from cruise_b200.engine import EpochEngine

    regular = EpochEngine(config)
    static = EpochEngine(config)
    cfg = regular.config
    for engine in (regular, static):
        engine.init_synthetic(0)
    sc = make_scenario(vocab=cfg.vocab, seed=seed, k=k, token_high=min(cfg.vocab, 151643))
    for inputs in prefill_epochs(sc, cfg.block_size, cfg.vocab):
        for engine in (regular, static):
            assert engine.run(**inputs).status == 0

    inputs = decode_inputs(sc, cfg.block_size)
    _free_bytes(static.device)   # the first query sets up torch's view of the device
    for call in range(2):
        expect = regular.run(**inputs)
        free_before = _free_bytes(static.device)
        rc, history, control_out = run_noalloc(static, inputs)
        free_after = _free_bytes(static.device)
        assert rc == 0, static.lib.cruise_epoch_last_error(static.handle)
        assert free_after == free_before, f"call {call}: device free memory moved by {free_before - free_after} B"
        assert expect.status == 0 and int(control_out[3]) == 0, f"call {call}"
        np.testing.assert_array_equal(history, expect.history, err_msg=f"call {call}")
        np.testing.assert_array_equal(control_out, expect.control_out, err_msg=f"call {call}")
        device_us, launches = static.last_timing()
        assert launches == 1 and device_us > 0.0
        for name, a, b in zip(("key", "value"), static.read_kv(), regular.read_kv()):
            assert torch.equal(a.view(torch.int16), b.view(torch.int16)), f"call {call}: {name} cache differs"
        inputs = next_epoch(inputs, expect.history, cfg.block_size, sc.block_table, sc.eos)
    regular.close()
    static.close()


def test_noalloc_epochs_match_regular_entry_point(cuda_ok):
    _match_two_epochs("tiny", seed=4, k=4)


def test_noalloc_epochs_match_regular_entry_point_7b_geometry(cuda_ok):
    from dataclasses import replace

    from cruise_b200.model_config import QWEN25_7B

    _match_two_epochs(replace(QWEN25_7B, name="qwen2.5-7b-2l", num_layers=2), seed=5, k=2)


def test_noalloc_rejects_oversized_scratch_and_imports(cuda_ok):
    from cruise_b200.engine import EpochEngine
    from cruise_b200.model_config import ModelConfig

    # 4 rows x 131072 intermediate activations alone exceed the 1 MiB static scratch
    wide = ModelConfig(name="wide", num_layers=1, hidden=256, num_heads=4, num_kv_heads=2, head_dim=64,
                       intermediate=131072, vocab=256, block_size=32, blocks_per_row=2, num_blocks=8,
                       configured_eos=255)
    engine = EpochEngine(wide)
    engine.init_synthetic(0)
    sc = make_scenario(vocab=wide.vocab, seed=0, blocks_per_row=2)
    rc, _, _ = run_noalloc(engine, decode_inputs(sc, wide.block_size))
    assert rc == -2
    message = engine.lib.cruise_epoch_last_error(engine.handle).decode()
    assert "bytes of scratch" in message and str(1 << 20) in message
    engine.close()

    tiny = EpochEngine("tiny")
    tiny.init_synthetic(0)
    sc = make_scenario(vocab=tiny.config.vocab, seed=0)
    rc, _, _ = run_noalloc(tiny, decode_inputs(sc, tiny.config.block_size, importing=True))
    assert rc == -3
    assert "import" in tiny.lib.cruise_epoch_last_error(tiny.handle).decode()
    tiny.close()
