"""The host-loop route: an epoch driven from the host, one decoder call per
token (the reference's host runner, ``RunHostCase`` in
``history/attempts/g4c-attempt69e-r4-b4-resident-epoch-storage-guard/host/g4c_b4_epoch_runner.cpp:245-382``).

Each step calls the 9-in / 4-out decoder ABI (``EpochEngine.decoder_step``),
copies the logits to the host and decides there what the resident epoch
decides on the device: the greedy token (first maximum, non-finite logits
fail), the position progress check, the next slot (-1 at capacity), EOS and
the finish reasons.  It is the baseline of the resident epoch: both compute
the same tokens, KV and accounting, and the epoch saves the per-token host
round trips.
"""

from __future__ import annotations

from typing import Callable

import numpy as np

from .model_config import BATCH, MAX_STEPS

FINISH_NONE, FINISH_EOS, FINISH_MAX_STEPS, FINISH_EMPTY, FINISH_ALREADY_FINISHED = 0, 1, 2, 4, 5


class HostLoopError(RuntimeError):
    """The runner's failure codes: 22 an inactive row moved, 23 non-finite
    logits or no position progress, 24 no slot for the next position."""

    def __init__(self, code: int, message: str) -> None:
        super().__init__(f"host loop failed ({code}): {message}")
        self.code = code


def first_max(logits_row: np.ndarray) -> int | None:
    """Index of the first maximum; None when any value is not finite."""
    if not np.isfinite(logits_row).all():
        return None
    return int(np.argmax(logits_row))   # numpy returns the first occurrence


def row_slot(block_table: np.ndarray, block_size: int, row: int, position: int) -> int:
    blocks = block_table.reshape(BATCH, -1)
    if position < 0 or position >= block_size * blocks.shape[1]:
        return -1
    return int(blocks[row, position // block_size]) * block_size + position % block_size


def host_loop_epoch(step: Callable, inputs: dict, block_size: int, capacity: int
                    ) -> tuple[np.ndarray, np.ndarray]:
    """One epoch of ``inputs`` (the 8-in epoch ABI: token, position, seq_len,
    slot, active, block_table, control) as K host-driven decoder calls.
    ``step(token, position, seq_len, slot, active, block_table)`` returns
    (logits f32 [4, V], next_position i64 [4]).  Returns the token history
    i64 [8][4] and the runner's control words i32[28] (status 0; generation
    words 0, the runner does not report them)."""
    control = np.asarray(inputs["control"], dtype=np.int32)
    max_steps = int(control[0])
    eos = [int(v) for v in control[1:1 + BATCH]]
    token = np.array(inputs["token"], dtype=np.int64).reshape(BATCH)
    position = np.array(inputs["position"], dtype=np.int64).reshape(BATCH)
    length = np.array(inputs["seq_len"], dtype=np.int32).reshape(BATCH)
    slot = np.array(inputs["slot"], dtype=np.int32).reshape(BATCH)
    active = np.array(inputs["active"], dtype=np.int32).reshape(BATCH)
    block_table = np.array(inputs["block_table"], dtype=np.int32).reshape(-1)
    initial = active.copy()
    executed = [0] * BATCH
    reason = [FINISH_NONE] * BATCH
    for r in range(BATCH):
        if initial[r] == 0:
            reason[r] = FINISH_EMPTY if length[r] == 0 else FINISH_ALREADY_FINISHED
    history = np.full((MAX_STEPS, BATCH), -1, dtype=np.int64)
    calls = 0
    while calls < max_steps and active.any():
        before = active.copy()
        logits, next_position = step(token, position, length, slot, active, block_table)
        for r in range(BATCH):
            if before[r] == 0:
                if next_position[r] != position[r]:
                    raise HostLoopError(22, f"inactive row {r} moved")
                continue
            generated = first_max(logits[r])
            if generated is None or next_position[r] != position[r] + 1:
                raise HostLoopError(23, f"row {r}: non-finite logits or no position progress")
            history[calls, r] = generated
            executed[r] += 1
            token[r] = generated
            length[r] = next_position[r] + 1
            if next_position[r] == capacity:
                slot[r] = -1
            else:
                slot[r] = row_slot(block_table, block_size, r, int(next_position[r]))
                if slot[r] < 0:
                    raise HostLoopError(24, f"row {r}: no slot for position {int(next_position[r])}")
            if generated == eos[r]:
                active[r] = 0
                reason[r] = FINISH_EOS
        position = next_position.astype(np.int64).copy()
        calls += 1
    for r in range(BATCH):
        if initial[r] == 1 and reason[r] == FINISH_NONE:
            reason[r] = FINISH_MAX_STEPS
    out = np.zeros(28, dtype=np.int32)
    out[0] = max_steps
    out[4] = calls
    for r in range(BATCH):
        out[6 + r] = eos[r]
        out[10 + r] = initial[r]
        out[14 + r] = executed[r]
        out[18 + r] = reason[r]
    out[22] = int(np.count_nonzero(initial))
    out[23] = int(np.count_nonzero(active))
    return history, out
