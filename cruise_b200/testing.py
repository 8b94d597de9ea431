"""A control-plane stand-in for the native engine: scheduler, worker and
engine-core tests run against it without a GPU.  It never touches a device and
is never evidence of device execution.

What it answers is the contract of the reference's test double
(src/vllm_ascend_resident_epoch/testing.py:6-78), which vLLM-facing tests
match on:

* every planned request emits ``plan.max_steps`` tokens, each the id after
  the previous one, wrapping at the 152,064-token vocabulary (step s emits
  ``(input token + s + 1) mod 152064``);
* warm-up and every epoch report one submission and one completion and the
  8-in / 2-out byte ledger of the epoch ABI (260 bytes in, 368 out);
* an import epoch declares its payload plus a 212-byte header and reports the
  snapshot's checksum; a device transfer reports checksum 1 and the
  ``device_ipc`` transfer mode, a device prefill checksum 1 and the
  ``device_prefill`` mode (the last has no counterpart in the reference's
  double).
"""

from __future__ import annotations

from .abi import EPOCH_INPUTS, EPOCH_OUTPUTS, total_bytes
from .backend import NativeEpochOutput, NativeWarmupOutput
from .contract import ResidentEpochPlan
from .kv_transfer import DeviceKVTransfer, ResidentKVSnapshot

VOCAB = 152064
EPOCH_IN_BYTES = total_bytes(EPOCH_INPUTS)     # 260
EPOCH_OUT_BYTES = total_bytes(EPOCH_OUTPUTS)   # 368
IMPORT_HEADER_BYTES = 212


def counting_tokens(first: int, steps: int) -> list[int]:
    """The stand-in's decoding rule: each token is the id after the previous
    one, modulo the vocabulary, starting after ``first``."""
    tokens, current = [], first
    for _ in range(steps):
        current = (current + 1) % VOCAB
        tokens.append(current)
    return tokens


class DeterministicTestEngine:
    """The ``NativeEpochEngine`` surface (warm_up, execute, execute_with_import,
    execute_with_device_transfer) with counted calls."""

    def __init__(self) -> None:
        self.warmup_calls = 0
        self.execute_calls = 0
        self.prefill_calls = 0

    def warm_up(self) -> NativeWarmupOutput:
        self.warmup_calls += 1
        return NativeWarmupOutput(status=0, model_calls=1, feed_calls=1, fetch_calls=1, wall_us=10,
                                  native_cpu_us=1, declared_input_bytes=EPOCH_IN_BYTES,
                                  declared_output_bytes=EPOCH_OUT_BYTES)

    def _epoch(self, plan: ResidentEpochPlan, **overrides) -> NativeEpochOutput:
        self.execute_calls += 1
        record = {
            "status": 0,
            "model_calls": plan.max_steps,
            "token_ids": {r.req_id: counting_tokens(r.token_id, plan.max_steps) for r in plan.requests},
            "row_generations": plan.row_generations,
            "wall_us": 10,
            "native_cpu_us": 1,
            "declared_input_bytes": EPOCH_IN_BYTES,
            "declared_output_bytes": EPOCH_OUT_BYTES,
        }
        record.update(overrides)
        return NativeEpochOutput(**record)

    def execute(self, plan: ResidentEpochPlan) -> NativeEpochOutput:
        return self._epoch(plan)

    def execute_with_import(self, plan: ResidentEpochPlan, snapshot: ResidentKVSnapshot) -> NativeEpochOutput:
        snapshot.validate()
        return self._epoch(plan, kv_imported=True, kv_import_checksum=snapshot.checksum,
                           declared_input_bytes=len(snapshot.payload) + IMPORT_HEADER_BYTES)

    def execute_with_device_transfer(self, plan: ResidentEpochPlan, transfer: DeviceKVTransfer) -> NativeEpochOutput:
        transfer.validate()
        return self._epoch(plan, kv_imported=True, kv_import_checksum=1, kv_transfer_mode="device_ipc")

    def execute_with_device_prefill(self, plan: ResidentEpochPlan) -> NativeEpochOutput:
        self.prefill_calls += 1
        return self._epoch(plan, kv_imported=True, kv_import_checksum=1, kv_transfer_mode="device_prefill")


def create_test_engine() -> DeterministicTestEngine:
    return DeterministicTestEngine()
