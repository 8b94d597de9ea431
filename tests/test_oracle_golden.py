"""The oracle is pinned to the reference's own decoder module.

The fixtures in ``tests/golden/`` were produced by
``tests/golden/make_golden.py``, which runs ``PagedQwenDecoderStep`` from the
reference (``history/attempts/g4c-attempt69c-b4-air/batched_decoder_step.py``).
``decoder_tiny.npz`` has the tiny geometry: 2 layers, 2 query heads per KV
head, head size 64.  ``decoder_gqa7_d128.npz`` has the 7B model's attention
shape: 7 query heads per KV head, head size 128.  The oracle must reproduce
both bit for bit.
"""

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle.decoder import OracleDecoder
from oracle.model import GQA7_D128, TINY, seeded_weights

GOLDEN = Path(__file__).resolve().parent / "golden"


def _bf16(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16)


@pytest.mark.parametrize("cfg, fixture", [(TINY, "decoder_tiny.npz"), (GQA7_D128, "decoder_gqa7_d128.npz")],
                         ids=["tiny", "gqa7_d128"])
def test_oracle_step_matches_reference_module_bit_exactly(cfg, fixture):
    g = np.load(GOLDEN / fixture)
    decoder = OracleDecoder(cfg, seeded_weights(cfg, int(g["seed"])))
    logits, key, value, next_position = decoder.step(
        torch.from_numpy(g["token"]), torch.from_numpy(g["position"]), torch.from_numpy(g["seq_len"]),
        torch.from_numpy(g["block_table"]), torch.from_numpy(g["slot"]),
        _bf16(g["key_cache_in"]), _bf16(g["value_cache_in"]), torch.from_numpy(g["active"]),
    )
    np.testing.assert_array_equal(logits.numpy(), g["logits"])
    np.testing.assert_array_equal(key.view(torch.int16).numpy().view(np.uint16), g["key_cache_out"])
    np.testing.assert_array_equal(value.view(torch.int16).numpy().view(np.uint16), g["value_cache_out"])
    np.testing.assert_array_equal(next_position.numpy(), g["next_position"])
