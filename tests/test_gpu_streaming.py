"""Streaming token egress: each decode step's tokens reach the host while the
epoch is still running, and they are exactly the epoch's token history."""

from __future__ import annotations

import time

import numpy as np
import pytest

from scenario import decode_inputs, make_scenario, prefill_epochs

pytestmark = pytest.mark.gpu


def _prefilled(engine, cfg, seed, k, token_high=None):
    sc = make_scenario(vocab=cfg.vocab, seed=seed, active_rows=(1, 1, 0, 1), prompt_len=(2, 5), k=k,
                       budget=(8, 8), token_high=token_high)
    for inputs in prefill_epochs(sc, cfg.block_size, cfg.vocab):
        assert engine.run(**inputs).status == 0
    return sc


def test_tiny_stream_equals_history(cuda_ok):
    from cruise_b200.engine import EpochEngine
    from cruise_b200.model_config import TINY

    engine = EpochEngine("tiny")
    engine.init_synthetic(0)
    # egress allocated but off: the prefill epochs publish nothing
    assert engine.lib.cruise_epoch_stream_enable(engine.handle, 1) == 0
    assert engine.lib.cruise_epoch_stream_enable(engine.handle, 0) == 0
    first = engine.lib.cruise_epoch_stream_next_id(engine.handle)
    sc = _prefilled(engine, TINY, seed=2, k=8)
    buf = np.zeros((8, 4), dtype=np.int64)
    last = engine.lib.cruise_epoch_stream_next_id(engine.handle) - 1
    assert last >= first
    for launch in range(first, last + 1):
        assert engine.lib.cruise_epoch_stream_poll(engine.handle, launch, buf.ctypes.data) == 0
    steps = []
    out = engine.run_streaming(lambda step, tokens: steps.append((step, tokens)),
                               **decode_inputs(sc, TINY.block_size))
    assert out.status == 0 and out.model_calls == 8
    assert [s for s, _ in steps] == list(range(out.model_calls))
    np.testing.assert_array_equal(np.stack([t for _, t in steps]), out.history[: out.model_calls])
    assert (out.history[: out.model_calls, 2] == -1).all()   # the inactive row
    engine.close()


def test_qwen7b_steps_arrive_during_the_epoch(cuda_ok):
    from cruise_b200.engine import EpochEngine
    from cruise_b200.model_config import QWEN25_7B

    engine = EpochEngine(QWEN25_7B)
    engine.init_synthetic(0)
    sc = _prefilled(engine, QWEN25_7B, seed=7, k=8, token_high=151643)
    arrivals = []
    out = engine.run_streaming(lambda step, tokens: arrivals.append((time.perf_counter(), tokens)),
                               **decode_inputs(sc, QWEN25_7B.block_size))
    assert out.status == 0 and out.model_calls == 8
    np.testing.assert_array_equal(np.stack([t for _, t in arrivals]), out.history[:8])
    # the 8 steps of a ~23 ms epoch arrive spread over its run, not at its end
    spread_us = (arrivals[-1][0] - arrivals[0][0]) * 1e6
    assert spread_us > 0.5 * out.device_us * 7 / 8, (spread_us, out.device_us)
    engine.close()
