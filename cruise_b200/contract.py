"""The resident-epoch contract between scheduler, worker and engine.

Restates ``src/vllm_ascend_resident_epoch/contract.py`` (plan ``:52-113``,
result ``:116-214``, commit states ``:13-17``, execution error ``:20-34``,
attach/get ``:217-237``) with the same names and rules, so a scheduler and a
worker written against the reference drive this engine unchanged.  The one
generalisation: the logical capacity of a row is a plan field checked against
``position + max_steps`` (the reference's graph fixes it at 8 tokens).

Commit states: an epoch is PREPARED until it is submitted to the GPU,
EXECUTING while it may have changed device state, and COMMITTED once its
outputs were validated.  Only a PREPARED failure is input-preserving, i.e. the
host may replay the step.
"""

from __future__ import annotations

from dataclasses import dataclass
from enum import IntEnum
from typing import Any, Literal

from .version import PYTHON_CONTRACT_VERSION

PLAN_ATTR = "_ascend_resident_epoch_plan"
RESULT_ATTR = "_ascend_resident_epoch_result"
CONTRACT_VERSION = PYTHON_CONTRACT_VERSION


class EpochCommitState(IntEnum):
    PREPARED = 0
    EXECUTING = 1
    COMMITTED = 2


class ResidentEpochExecutionError(RuntimeError):
    def __init__(self, message: str, *, commit_state: EpochCommitState, status: int | None = None) -> None:
        super().__init__(message)
        self.commit_state = commit_state
        self.status = status

    @property
    def input_preserving(self) -> bool:
        return self.commit_state == EpochCommitState.PREPARED


@dataclass(frozen=True)
class ResidentEpochRequest:
    req_id: str
    row: int
    generation: int
    token_id: int
    position: int
    sequence_length: int
    eos_token_id: int
    scheduler_block_ids: tuple[int, ...]
    device_block_ids: tuple[int, int]
    state_owner: Literal["host", "device"] = "host"
    kv_import_required: bool = False
    # Device prefill (no reference counterpart; the reference prefills on the
    # host): the whole prompt, whose K/V at positions 0..len-2 the engine
    # computes and imports before this epoch decodes from position len-1.
    # Empty for a request whose KV already exists.
    prompt_token_ids: tuple[int, ...] = ()


def _fail(message: str) -> None:
    raise ValueError(message)


@dataclass(frozen=True)
class ResidentEpochPlan:
    version: int
    graph_batch_size: Literal[1, 2, 4]
    max_steps: int
    logical_capacity: int
    requests: tuple[ResidentEpochRequest, ...]
    active_mask: tuple[int, ...]
    sampling_mode: int = 0
    graph_variant: int = 0

    @property
    def req_ids(self) -> tuple[str, ...]:
        return tuple(r.req_id for r in self.requests)

    @property
    def row_generations(self) -> tuple[int, ...]:
        generations = [0] * self.graph_batch_size
        for r in self.requests:
            generations[r.row] = r.generation
        return tuple(generations)

    @property
    def host_replay_safe(self) -> bool:
        return all(r.state_owner == "host" for r in self.requests)

    def validate(self) -> None:
        if self.version != CONTRACT_VERSION:
            _fail(f"unsupported resident epoch contract {self.version}")
        if self.graph_batch_size not in (1, 2, 4):
            _fail("graph batch size must be 1, 2, or 4")
        if not 1 <= len(self.requests) <= self.graph_batch_size:
            _fail("request count does not fit the static graph")
        if len(self.active_mask) != self.graph_batch_size:
            _fail("active mask does not match graph batch size")
        if any(v not in (0, 1) for v in self.active_mask):
            _fail("active mask must contain only zero or one")
        if len(set(self.req_ids)) != len(self.requests):
            _fail("request IDs must be unique")
        rows = [r.row for r in self.requests]
        if len(set(rows)) != len(rows):
            _fail("resident rows must be unique")
        generations = [r.generation for r in self.requests]
        if min(generations) <= 0:
            _fail("resident generations must be positive")
        if len(set(generations)) != len(generations):
            _fail("resident generations must be unique")
        expected = [0] * self.graph_batch_size
        for r in self.requests:
            if not 0 <= r.row < self.graph_batch_size:
                _fail("resident row is outside the static graph")
            expected[r.row] = 1
            if r.sequence_length != r.position + 1:
                _fail("sequence length and position disagree")
            if r.state_owner not in ("host", "device"):
                _fail("resident request has an invalid state owner")
            if r.kv_import_required and r.state_owner != "host":
                _fail("KV import requires Host-owned request state")
            if r.position + self.max_steps > self.logical_capacity:
                _fail("epoch exceeds logical capacity")
            if r.prompt_token_ids:
                if len(r.prompt_token_ids) < 2:
                    _fail("a device prefill needs a prompt of at least two tokens")
                if not r.kv_import_required or r.state_owner != "host":
                    _fail("a device prefill imports Host-owned request state")
                if r.position != len(r.prompt_token_ids) - 1 or r.token_id != r.prompt_token_ids[-1]:
                    _fail("a device prefill decodes from the last prompt token")
        if tuple(expected) != tuple(self.active_mask):
            _fail("active mask does not match resident rows")


@dataclass(frozen=True)
class ResidentEpochResult:
    version: int
    route: Literal["device", "host_fallback"]
    status: int
    model_calls: int
    computed_steps: dict[str, int]
    row_generations: tuple[int, ...] = ()
    commit_state: EpochCommitState = EpochCommitState.COMMITTED
    fallback_safe: bool = False
    feed_calls: int = 1
    fetch_calls: int = 1
    wall_us: int = 0
    native_cpu_us: int = 0
    declared_input_bytes: int = 0
    declared_output_bytes: int = 0
    socket_send_calls: int = 1
    socket_receive_calls: int = 1
    kv_imported: bool = False
    kv_import_checksum: int = 0
    kv_snapshot_checksum: int = 0
    kv_transfer_mode: Literal["none", "host_snapshot", "device_ipc", "device_prefill"] = "none"

    def _check_device_route(self, plan: ResidentEpochPlan) -> None:
        if self.status != 0:
            _fail("failed device execution cannot be committed")
        if self.commit_state != EpochCommitState.COMMITTED:
            _fail("device execution result is not committed")
        if self.feed_calls != 1 or self.fetch_calls != 1:
            _fail("device epoch must use exactly one Feed and one Fetch")
        if self.row_generations != plan.row_generations:
            _fail("device resident generations disagree with the plan")
        if any(r.kv_import_required for r in plan.requests) and not self.kv_imported:
            _fail("device result did not commit the requested KV import")

    def _check_transfer(self) -> None:
        mode = "host_snapshot" if self.kv_imported and self.kv_transfer_mode == "none" else self.kv_transfer_mode
        if self.kv_imported:
            if self.kv_import_checksum == 0 or mode not in ("host_snapshot", "device_ipc", "device_prefill"):
                _fail("device result did not prove an imported KV transfer")
            if mode == "host_snapshot" and (
                self.kv_snapshot_checksum == 0 or self.kv_import_checksum != self.kv_snapshot_checksum
            ):
                _fail("device result did not prove equivalent imported KV from the Host snapshot")
        elif mode != "none":
            _fail("KV transfer mode is set without an import")

    def _check_fallback_route(self, plan: ResidentEpochPlan) -> None:
        if not self.fallback_safe:
            _fail("host fallback must be declared input-preserving")
        if self.commit_state != EpochCommitState.PREPARED:
            _fail("host fallback requires a prepared device state")
        if not plan.host_replay_safe:
            _fail("Host no longer owns every request state")
        if self.feed_calls != 0 or self.fetch_calls != 0:
            _fail("Host fallback result cannot claim DataFlow calls")

    def validate_against(self, plan: ResidentEpochPlan, sampled_token_ids: dict[str, list[int]]) -> None:
        if self.version != plan.version:
            _fail("resident epoch result version mismatch")
        if set(self.computed_steps) != set(plan.req_ids):
            _fail("resident epoch result request set mismatch")
        if set(sampled_token_ids) != set(plan.req_ids):
            _fail("resident epoch output request set mismatch")
        device = self.route == "device"
        if device:
            self._check_device_route(plan)
        self._check_transfer()
        if self.route == "host_fallback":
            self._check_fallback_route(plan)
        for r in plan.requests:
            steps = self.computed_steps[r.req_id]
            tokens = sampled_token_ids[r.req_id]
            if not 1 <= steps <= plan.max_steps:
                _fail("computed step count is outside the epoch")
            if len(tokens) != steps:
                _fail("sampled token count and computed steps disagree")
            if self.route == "host_fallback" and steps != 1:
                _fail("host fallback must retain one-step vLLM semantics")
            if device and steps < plan.max_steps and (not tokens or tokens[-1] != r.eos_token_id):
                _fail("a short device epoch must terminate at EOS")
        if device and self.model_calls != max(self.computed_steps.values()):
            _fail("device model-call count disagrees with executed steps")


def attach_plan(scheduler_output: Any, plan: ResidentEpochPlan) -> None:
    plan.validate()
    setattr(scheduler_output, PLAN_ATTR, plan)


def get_plan(scheduler_output: Any) -> ResidentEpochPlan | None:
    value = getattr(scheduler_output, PLAN_ATTR, None)
    if value is not None and not isinstance(value, ResidentEpochPlan):
        raise TypeError("invalid resident epoch plan attached to SchedulerOutput")
    return value


def attach_result(model_runner_output: Any, result: ResidentEpochResult) -> None:
    setattr(model_runner_output, RESULT_ATTR, result)


def get_result(model_runner_output: Any) -> ResidentEpochResult | None:
    value = getattr(model_runner_output, RESULT_ATTR, None)
    if value is not None and not isinstance(value, ResidentEpochResult):
        raise TypeError("invalid resident epoch result attached to ModelRunnerOutput")
    return value
