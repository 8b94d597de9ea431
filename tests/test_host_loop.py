"""The host-loop route (cruise_b200.host_loop, the reference's host runner
g4c_b4_epoch_runner.cpp:245-382) on the CPU: driven by the oracle's decoder
step, K host-driven calls compute exactly what one resident K-step epoch of
the oracle controller computes -- the reference's case matrix (K 1/2/4/8,
empty and finished rows, independent early EOS): same tokens, executed counts,
reasons, model calls, and the same KV cache."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from cruise_b200.host_loop import HostLoopError, host_loop_epoch
from oracle.decoder import OracleDecoder
from oracle.epoch import OracleEpochController
from oracle.model import TINY, seeded_weights
from scenario import prefill_epochs
from test_oracle_epoch import CASE_MATRIX, case_matrix_inputs


@pytest.fixture(scope="module")
def weights():
    return seeded_weights(TINY, seed=0)


class OracleStep:
    """The oracle decoder as the 9-in / 4-out step the host loop calls,
    holding the caches between calls (they stay on the device in the engine)."""

    def __init__(self, controller: OracleEpochController) -> None:
        self.c = controller

    def __call__(self, token, position, seq_len, slot, active, block_table):
        bt = torch.from_numpy(np.asarray(block_table, dtype=np.int32).reshape(4, -1).copy())
        logits, key, value, nxt = self.c.decoder.step(
            torch.from_numpy(token.copy()), torch.from_numpy(position.copy()), torch.from_numpy(seq_len.copy()),
            bt, torch.from_numpy(slot.copy()), self.c.key, self.c.value, torch.from_numpy(active.copy()))
        self.c.key, self.c.value = key, value
        return logits.numpy(), nxt.numpy()


@pytest.mark.parametrize("name, k, pattern", CASE_MATRIX, ids=[c[0] for c in CASE_MATRIX])
def test_host_loop_equals_resident_epoch(weights, name, k, pattern):
    sc, inputs = case_matrix_inputs(weights, name, k, pattern)
    epoch = OracleEpochController(OracleDecoder(TINY, weights))
    loop = OracleEpochController(OracleDecoder(TINY, weights))
    for prefill in prefill_epochs(sc, TINY.block_size, TINY.vocab):
        epoch.run(**prefill)
        loop.run(**prefill)
    want_history, want = epoch.run(**inputs)
    history, got = host_loop_epoch(OracleStep(loop), inputs, TINY.block_size, TINY.capacity)
    np.testing.assert_array_equal(history, want_history)
    same = [0, 3, 4, *range(6, 24)]   # all but sampling/variant/checksum words and the generations
    np.testing.assert_array_equal(got[same], want[same])
    assert torch.equal(loop.key, epoch.key) and torch.equal(loop.value, epoch.value)


def test_host_loop_fails_on_non_finite_logits():
    def step(token, position, seq_len, slot, active, block_table):
        logits = np.zeros((4, 8), dtype=np.float32)
        logits[0, 3] = np.nan
        return logits, position + active

    inputs = dict(token=np.zeros(4, np.int64), position=np.zeros(4, np.int64), seq_len=np.ones(4, np.int32),
                  slot=np.zeros(4, np.int32), active=np.array([1, 0, 0, 0], np.int32),
                  block_table=np.arange(8, dtype=np.int32), control=np.array([2, 7, 7, 7, 7, 0, 0, 1, 0, 0, 0]))
    with pytest.raises(HostLoopError) as err:
        host_loop_epoch(step, inputs, block_size=16, capacity=32)
    assert err.value.code == 23
