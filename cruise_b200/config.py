"""Resident-epoch configuration (src/vllm_ascend_resident_epoch/config.py:17-42).

Environment names are the reference's operator surface:
``VLLM_ASCEND_RESIDENT_EPOCH_STEPS`` (K per epoch, one of 1/2/4/8) and
``VLLM_ASCEND_RESIDENT_EPOCH_CAPACITY`` (logical tokens per row).  The
reference fixes capacity at 8 tokens; here it defaults to the paged layout's
``blocks_per_row * block_size`` of the served preset
(``VLLM_ASCEND_RESIDENT_EPOCH_MODEL``; 256 for the 7B preset).
``VLLM_ASCEND_RESIDENT_EPOCH_DEVICE_PREFILL`` (1: prefill new prompts on the
device) extends the reference's surface.
"""

from __future__ import annotations

import os
from dataclasses import dataclass

STEP_CHOICES = (1, 2, 4, 8)


def _env_int(name: str, default: int) -> int:
    raw = os.getenv(name)
    if raw is None:
        return default
    try:
        return int(raw)
    except ValueError as exc:
        raise ValueError(f"{name} must be an integer, got {raw!r}") from exc


@dataclass(frozen=True)
class ResidentEpochConfig:
    max_steps: int = 8
    logical_capacity: int = 256
    physical_blocks: int = 8
    blocks_per_request: int = 2
    block_size: int = 128
    max_batch_size: int = 4
    # VLLM_ASCEND_RESIDENT_EPOCH_DEVICE_PREFILL=1 (no reference counterpart):
    # new prompts of 2..block_size tokens are prefilled by the engine on the
    # device inside their first epoch instead of on the host lane
    device_prefill: bool = False

    @classmethod
    def from_env(cls) -> "ResidentEpochConfig":
        """The paged geometry of the served preset (VLLM_ASCEND_RESIDENT_EPOCH_MODEL,
        default the 7B one) with the step and capacity overrides."""
        from .model_config import PRESETS

        preset = PRESETS[os.getenv("VLLM_ASCEND_RESIDENT_EPOCH_MODEL", "qwen2.5-7b")]
        config = cls(
            max_steps=_env_int("VLLM_ASCEND_RESIDENT_EPOCH_STEPS", 8),
            logical_capacity=_env_int("VLLM_ASCEND_RESIDENT_EPOCH_CAPACITY", preset.capacity),
            physical_blocks=preset.num_blocks,
            blocks_per_request=preset.blocks_per_row,
            block_size=preset.block_size,
            device_prefill=_env_int("VLLM_ASCEND_RESIDENT_EPOCH_DEVICE_PREFILL", 0) != 0,
        )
        config.validate()
        return config

    def validate(self) -> None:
        if self.max_steps not in STEP_CHOICES:
            raise ValueError("resident epoch steps must be one of 1, 2, 4, 8")
        if self.logical_capacity < self.max_steps:
            raise ValueError("logical capacity must be at least max_steps")
        if self.logical_capacity > self.blocks_per_request * self.block_size:
            raise ValueError("logical capacity exceeds the blocks a row owns")
        if self.max_batch_size != 4:
            raise ValueError("the resident epoch has a fixed maximum B=4")


def epoch_steps(budget: int) -> int:
    """Largest K in {1, 2, 4, 8} not above ``budget`` (scheduler.py:244-247)."""
    if budget < 1:
        raise ValueError("an epoch needs a budget of at least one step")
    return max(k for k in STEP_CHOICES if k <= budget)
