"""Control-plane test double (src/vllm_ascend_resident_epoch/testing.py:6-78).

``DeterministicTestEngine`` answers every epoch with tokens
``(token + step + 1) % vocab`` and never touches a GPU; it lets scheduler and
worker integration run without the CUDA engine.  It is never evidence of
device execution.
"""

from __future__ import annotations

from dataclasses import replace

from .backend import NativeEpochOutput, NativeWarmupOutput
from .contract import ResidentEpochPlan
from .kv_transfer import DeviceKVTransfer, ResidentKVSnapshot

VOCAB = 152064


class DeterministicTestEngine:
    def __init__(self) -> None:
        self.warmup_calls = 0
        self.execute_calls = 0

    def warm_up(self) -> NativeWarmupOutput:
        self.warmup_calls += 1
        return NativeWarmupOutput(
            status=0, model_calls=1, feed_calls=1, fetch_calls=1, wall_us=10, native_cpu_us=1,
            declared_input_bytes=260, declared_output_bytes=368,
        )

    def execute(self, plan: ResidentEpochPlan) -> NativeEpochOutput:
        self.execute_calls += 1
        token_ids = {
            r.req_id: [(r.token_id + step + 1) % VOCAB for step in range(plan.max_steps)] for r in plan.requests
        }
        return NativeEpochOutput(
            status=0, model_calls=plan.max_steps, token_ids=token_ids, row_generations=plan.row_generations,
            wall_us=10, native_cpu_us=1, declared_input_bytes=260, declared_output_bytes=368,
        )

    def execute_with_import(self, plan: ResidentEpochPlan, snapshot: ResidentKVSnapshot) -> NativeEpochOutput:
        snapshot.validate()
        return replace(
            self.execute(plan), kv_imported=True, kv_import_checksum=snapshot.checksum,
            declared_input_bytes=len(snapshot.payload) + 212,
        )

    def execute_with_device_transfer(self, plan: ResidentEpochPlan, transfer: DeviceKVTransfer) -> NativeEpochOutput:
        transfer.validate()
        return replace(self.execute(plan), kv_imported=True, kv_import_checksum=1, kv_transfer_mode="device_ipc")


def create_test_engine() -> DeterministicTestEngine:
    return DeterministicTestEngine()
