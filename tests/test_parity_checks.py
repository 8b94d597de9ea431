"""The parity checker itself (scenario.check_epoch), on the CPU: the oracle's
own epoch passes, and mistakes planted in a copy of the oracle's output are
caught -- a control word, a token, logits and KV beyond the tolerance, a
block outside the block table that changed -- also for rows that did not
diverge when another row diverged at a near-tie."""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import pytest
import torch

from oracle.decoder import OracleDecoder
from oracle.epoch import EpochTrace, OracleEpochController
from oracle.model import TINY, seeded_weights
from scenario import check_epoch, decode_inputs, make_scenario, prefill_epochs


@dataclass
class Fake:
    history: np.ndarray
    control_out: np.ndarray
    logits: np.ndarray | None


@pytest.fixture(scope="module")
def epoch():
    weights = seeded_weights(TINY, seed=0)
    oracle = OracleEpochController(OracleDecoder(TINY, weights))
    sc = make_scenario(vocab=TINY.vocab, seed=2, k=4, budget=(4, 4))
    for inputs in prefill_epochs(sc, TINY.block_size, TINY.vocab):
        oracle.run(**inputs)
    inputs = decode_inputs(sc, TINY.block_size)
    trace = EpochTrace()
    history, control = oracle.run(**inputs, trace=trace)
    logits = np.zeros((8, 4, TINY.vocab), dtype=np.float32)
    for s, lg in enumerate(trace.logits):
        logits[s] = lg.numpy()
    return inputs, history, control, trace, logits, oracle.key.clone(), oracle.value.clone()


def _run(epoch, history=None, control=None, logits=None, key=None, value=None, **kw):
    inputs, h, c, trace, lg, k, v = epoch
    out = Fake(h.copy() if history is None else history, c.copy() if control is None else control,
               lg.copy() if logits is None else logits)
    return check_epoch(out, h, c, trace, inputs, kv=(k.clone() if key is None else key, v.clone() if value is None else value, k, v),
                       block_size=TINY.block_size, label="planted", record=False, **kw)


def test_identical_outputs_pass(epoch):
    check = _run(epoch)
    assert check.diverged == {} and check.logits_err == 0.0 and check.kv_err == 0.0


def test_a_wrong_control_word_is_caught(epoch):
    control = epoch[2].copy()
    control[18] += 1   # row 0's finish reason
    with pytest.raises(AssertionError, match="control word 18"):
        _run(epoch, control=control)


def test_a_token_off_a_near_tie_is_caught(epoch):
    inputs, h, c, trace, *_ = epoch
    row, step = 0, 0
    history = h.copy()
    history[step, row] = (history[step, row] + 1) % TINY.vocab
    if trace.margins[step][row] < 2e-2:
        pytest.skip("seeded step is a near-tie")
    with pytest.raises(AssertionError, match="top-2 margin"):
        _run(epoch, history=history)


def test_logits_beyond_tolerance_are_caught(epoch):
    logits = epoch[4].copy()
    logits[1, 2] *= 1.05
    with pytest.raises(AssertionError, match="logits rel err"):
        _run(epoch, logits=logits)


def test_kv_beyond_tolerance_and_untouched_blocks_are_caught(epoch):
    inputs, *_, k, v = epoch
    bt = np.asarray(inputs["block_table"]).reshape(4, -1)
    key = k.clone()
    key[1, int(bt[0, 0]), 0, 0] *= 1.1
    with pytest.raises(AssertionError, match="key cache"):
        _run(epoch, key=key)
    outside = sorted(set(range(TINY.num_blocks)) - {int(b) for b in bt.reshape(-1)})
    if outside:
        value = v.clone()
        value[0, outside[0], 3, 1, 5] = 1.0
        with pytest.raises(AssertionError, match="in no row of the block table"):
            _run(epoch, value=value)


def test_a_near_tie_divergence_keeps_the_other_rows_checked(epoch):
    """Pretend row 1 diverged at a near-tie at step 1: its later tokens and KV
    slots are exempt, row 0's control words and KV are still compared."""
    inputs, h, c, trace, lg, k, v = epoch
    margins = [list(m) for m in trace.margins]
    margins[1][1] = 0.0
    forged = EpochTrace(trace.logits, trace.active, margins)
    history = h.copy()
    history[1, 1] = (history[1, 1] + 1) % TINY.vocab
    n = int(c[15])   # row 1's executed steps
    history[2:n, 1] = (history[2:n, 1] + 7) % TINY.vocab
    # row 1's slots after position p0 + 1 hold other values on the device side
    key = k.clone()
    bt = np.asarray(inputs["block_table"]).reshape(4, -1)
    p = int(inputs["position"][1]) + 2
    key[:, int(bt[1, p // TINY.block_size]), p % TINY.block_size] += 1.0
    out = Fake(history, c.copy(), lg.copy())
    check = check_epoch(out, h, c, forged, inputs, kv=(key, v.clone(), k, v), block_size=TINY.block_size, record=False)
    assert check.diverged == {1: 1}
    control = c.copy()
    control[14] += 1   # row 0's executed count is still compared
    with pytest.raises(AssertionError, match="control word 14"):
        check_epoch(Fake(history, control, lg.copy()), h, c, forged, inputs, kv=(key, v.clone(), k, v),
                    block_size=TINY.block_size, record=False)
    key0 = key.clone()
    p0 = int(inputs["position"][0])
    key0[:, int(bt[0, p0 // TINY.block_size]), p0 % TINY.block_size] *= 1.5   # row 0's KV is still compared
    with pytest.raises(AssertionError, match="key cache"):
        check_epoch(Fake(history, c.copy(), lg.copy()), h, c, forged, inputs, kv=(key0, v.clone(), k, v),
                    block_size=TINY.block_size, record=False)
