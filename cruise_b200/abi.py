"""Byte ledger of the epoch ABIs (src/vllm_ascend_resident_epoch/abi.py:18-76).

The minimal 8-input / 2-output epoch ABI moves 260 bytes in and 368 bytes out
per epoch; the reference's earlier 10/10 ABI shipped the whole paged K/V and
the logits history (58,720,516 / 78,184,928 bytes at the 7B capacity-8
geometry).  The engine implements the 8/2 ABI; the old ledger is kept for the
comparison the reference reports.
"""

from __future__ import annotations

from dataclasses import dataclass
from math import prod


@dataclass(frozen=True)
class TensorSpec:
    name: str
    shape: tuple[int, ...]
    element_bytes: int

    @property
    def nbytes(self) -> int:
        return prod(self.shape) * self.element_bytes


EPOCH_INPUTS = (
    TensorSpec("token", (4, 1), 8),
    TensorSpec("position", (4,), 8),
    TensorSpec("sequence_length", (4, 1), 4),
    TensorSpec("slot_mapping", (4,), 4),
    TensorSpec("active_mask", (4,), 4),
    TensorSpec("block_table", (4, 2), 4),
    TensorSpec("tiling", (72,), 1),
    TensorSpec("control", (11,), 4),
)
TOKEN_HISTORY = TensorSpec("token_history", (8, 4), 8)
CONTROL_OUTPUT = TensorSpec("control_output", (28,), 4)
EPOCH_OUTPUTS = (TOKEN_HISTORY, CONTROL_OUTPUT)

# decoder-step ABI (config/graph_config.json): 9 inputs, 4 outputs, 7B capacity-8 shapes
KEY_CACHE = TensorSpec("key_cache", (28, 8, 128, 4, 128), 2)
VALUE_CACHE = TensorSpec("value_cache", (28, 8, 128, 4, 128), 2)
OLD_INPUTS = EPOCH_INPUTS[:3] + (KEY_CACHE,) + EPOCH_INPUTS[3:6] + (VALUE_CACHE,) + EPOCH_INPUTS[6:]
OLD_OUTPUTS = (
    TensorSpec("logits_history", (8, 4, 1, 152064), 4),
    TOKEN_HISTORY,
    KEY_CACHE,
    VALUE_CACHE,
    TensorSpec("final_token", (4, 1), 8),
    TensorSpec("final_position", (4,), 8),
    TensorSpec("final_length", (4, 1), 4),
    TensorSpec("final_slot", (4,), 4),
    TensorSpec("final_active", (4,), 4),
    CONTROL_OUTPUT,
)


def total_bytes(specs) -> int:
    return sum(spec.nbytes for spec in specs)


ABI_BYTES = {
    "old": {"input": total_bytes(OLD_INPUTS), "output": total_bytes(OLD_OUTPUTS)},
    "new": {"input": total_bytes(EPOCH_INPUTS), "output": total_bytes(EPOCH_OUTPUTS)},
}
NEW_TOTAL_BYTES = ABI_BYTES["new"]["input"] + ABI_BYTES["new"]["output"]
OLD_TOTAL_BYTES = ABI_BYTES["old"]["input"] + ABI_BYTES["old"]["output"]
TOTAL_REDUCTION_BYTES = OLD_TOTAL_BYTES - NEW_TOTAL_BYTES
