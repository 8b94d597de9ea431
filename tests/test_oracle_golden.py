"""The oracle is pinned to the reference's own decoder module.

``tests/golden/decoder_tiny.npz`` was produced by ``tests/golden/make_golden.py``,
which runs ``PagedQwenDecoderStep`` from the reference
(``history/attempts/g4c-attempt69c-b4-air/batched_decoder_step.py``) with tiny
geometry; the oracle must reproduce it bit for bit.
"""

from pathlib import Path

import numpy as np
import torch

from oracle.decoder import OracleDecoder
from oracle.model import TINY, seeded_weights

GOLDEN = Path(__file__).resolve().parent / "golden" / "decoder_tiny.npz"


def _bf16(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16)


def test_oracle_step_matches_reference_module_bit_exactly():
    g = np.load(GOLDEN)
    decoder = OracleDecoder(TINY, seeded_weights(TINY, int(g["seed"])))
    logits, key, value, next_position = decoder.step(
        torch.from_numpy(g["token"]), torch.from_numpy(g["position"]), torch.from_numpy(g["seq_len"]),
        torch.from_numpy(g["block_table"]), torch.from_numpy(g["slot"]),
        _bf16(g["key_cache_in"]), _bf16(g["value_cache_in"]), torch.from_numpy(g["active"]),
    )
    np.testing.assert_array_equal(logits.numpy(), g["logits"])
    np.testing.assert_array_equal(key.view(torch.int16).numpy().view(np.uint16), g["key_cache_out"])
    np.testing.assert_array_equal(value.view(torch.int16).numpy().view(np.uint16), g["value_cache_out"])
    np.testing.assert_array_equal(next_position.numpy(), g["next_position"])
