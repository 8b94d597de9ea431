"""bench.py's teacher-forced baseline (all rows of a cohort forced together)
prefills exactly what the row-by-row helper does: same KV cache, same
resident state, checked on the CPU oracle (tiny model)."""

from __future__ import annotations

import numpy as np
import torch

import bench
from oracle.decoder import OracleDecoder
from oracle.epoch import OracleEpochController
from oracle.model import TINY as ORACLE_TINY, seeded_weights
from scenario import decode_inputs, make_scenario, prefill_epochs


def test_all_rows_forcing_matches_row_by_row_prefill():
    from cruise_b200.model_config import TINY

    weights = seeded_weights(ORACLE_TINY, seed=0)
    sc = make_scenario(vocab=TINY.vocab, seed=4, active_rows=(1, 1, 1, 1), prompt_len=(3, 14), k=2)
    serial = OracleEpochController(OracleDecoder(ORACLE_TINY, weights))
    for inputs in prefill_epochs(sc, TINY.block_size, TINY.vocab):
        serial.run(**inputs)
    batched = OracleEpochController(OracleDecoder(ORACLE_TINY, weights))
    epochs = list(bench.forced_epochs_all_rows(sc, TINY, generation_offset=0))
    for inputs in epochs:
        _, control = batched.run(**inputs)
        assert int(control[3]) == 0
    assert torch.equal(serial.key, batched.key) and torch.equal(serial.value, batched.value)
    # both leave every row ready for the same decode epoch
    h1, c1 = serial.run(**decode_inputs(sc, TINY.block_size))
    h2, c2 = batched.run(**decode_inputs(sc, TINY.block_size))
    np.testing.assert_array_equal(h1, h2)
    np.testing.assert_array_equal(c1, c2)
