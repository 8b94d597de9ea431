"""Backend adapter between the vLLM worker and a native epoch engine.

Restates ``src/vllm_ascend_resident_epoch/backend.py`` (``:20-221``): the
``NativeEpochEngine`` protocol, output records, plan/output validation and
the mapping of failures to commit states, plus the host-replay rule of
``plugin.py:23-57`` (``execute_with_fallback``).  The engine is chosen by
``VLLM_ASCEND_RESIDENT_EPOCH_BACKEND_FACTORY=module:factory``; the CUDA engine
is ``cruise_b200.cuda_backend:create_cuda_engine``.
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from importlib import import_module
from typing import Any, Callable, Protocol

from .contract import (
    CONTRACT_VERSION,
    EpochCommitState,
    ResidentEpochExecutionError,
    ResidentEpochPlan,
    ResidentEpochResult,
    attach_result,
)
from .kv_transfer import DeviceKVTransfer, ResidentKVSnapshot

FACTORY_ENV = "VLLM_ASCEND_RESIDENT_EPOCH_BACKEND_FACTORY"


@dataclass(frozen=True)
class NativeEpochOutput:
    status: int
    model_calls: int
    token_ids: dict[str, list[int]]
    row_generations: tuple[int, ...]
    commit_state: EpochCommitState = EpochCommitState.COMMITTED
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
    kv_transfer_mode: str = "none"


@dataclass(frozen=True)
class NativeWarmupOutput:
    status: int
    model_calls: int
    feed_calls: int
    fetch_calls: int
    wall_us: int
    commit_state: EpochCommitState = EpochCommitState.COMMITTED
    native_cpu_us: int = 0
    declared_input_bytes: int = 0
    declared_output_bytes: int = 0
    socket_send_calls: int = 1
    socket_receive_calls: int = 1


class NativeEpochEngine(Protocol):
    def warm_up(self) -> NativeWarmupOutput: ...

    def execute(self, plan: ResidentEpochPlan) -> NativeEpochOutput: ...

    def execute_with_import(self, plan: ResidentEpochPlan, snapshot: ResidentKVSnapshot) -> NativeEpochOutput: ...

    def execute_with_device_transfer(
        self, plan: ResidentEpochPlan, transfer: DeviceKVTransfer
    ) -> NativeEpochOutput: ...

    # Optional (no reference counterpart): prefill the plan's prompts
    # (requests with prompt_token_ids) on the device, then run the epoch that
    # imports them.
    def execute_with_device_prefill(self, plan: ResidentEpochPlan) -> NativeEpochOutput: ...


def _model_runner_output(req_ids: list[str], sampled: list[list[int]]) -> Any:
    try:
        from vllm.v1.outputs import ModelRunnerOutput
    except Exception:   # vLLM absent: a plain record with the same fields
        from types import SimpleNamespace

        return SimpleNamespace(
            req_ids=req_ids, req_id_to_index={r: i for i, r in enumerate(req_ids)}, sampled_token_ids=sampled
        )
    return ModelRunnerOutput(
        req_ids=req_ids, req_id_to_index={r: i for i, r in enumerate(req_ids)}, sampled_token_ids=sampled
    )


class ResidentEpochBackend:
    def __init__(self, engine: NativeEpochEngine) -> None:
        self.engine = engine

    def warm_up(self) -> NativeWarmupOutput:
        output = self.engine.warm_up()
        if output.status != 0:
            raise RuntimeError(f"native resident warmup returned {output.status}")
        if (output.model_calls, output.feed_calls, output.fetch_calls) != (1, 1, 1) or (
            output.commit_state != EpochCommitState.COMMITTED
        ):
            raise RuntimeError("resident warmup must execute one complete decoder step")
        return output

    def close(self) -> None:
        close = getattr(self.engine, "close", None)
        if callable(close):
            close()

    def _run_native(self, plan, snapshot, device_transfer) -> NativeEpochOutput:
        if any(r.prompt_token_ids for r in plan.requests):
            run = getattr(self.engine, "execute_with_device_prefill", None)
            if not callable(run) or snapshot is not None or device_transfer is not None:
                raise ResidentEpochExecutionError(
                    "resident backend cannot prefill on the device", commit_state=EpochCommitState.PREPARED
                )
            return run(plan)
        if device_transfer is not None:
            run = getattr(self.engine, "execute_with_device_transfer", None)
            if not callable(run):
                raise ResidentEpochExecutionError(
                    "resident backend does not support direct Device KV transfer",
                    commit_state=EpochCommitState.PREPARED,
                )
            return run(plan, device_transfer)
        if snapshot is not None:
            run = getattr(self.engine, "execute_with_import", None)
            if not callable(run):
                raise ResidentEpochExecutionError(
                    "resident backend does not support KV import", commit_state=EpochCommitState.PREPARED
                )
            return run(plan, snapshot)
        return self.engine.execute(plan)

    def execute(
        self,
        plan: ResidentEpochPlan,
        snapshot: ResidentKVSnapshot | None = None,
        device_transfer: DeviceKVTransfer | None = None,
    ):
        if snapshot is not None and device_transfer is not None:
            raise ValueError("resident epoch cannot use two KV transfer modes")
        try:
            plan.validate()
        except Exception as exc:
            raise ResidentEpochExecutionError(
                f"resident epoch plan validation failed: {exc}", commit_state=EpochCommitState.PREPARED
            ) from exc
        try:
            native = self._run_native(plan, snapshot, device_transfer)
        except ResidentEpochExecutionError:
            raise
        except Exception as exc:
            raise ResidentEpochExecutionError(
                "native resident epoch failed without commit-state proof", commit_state=EpochCommitState.EXECUTING
            ) from exc
        if native.status != 0:
            raise ResidentEpochExecutionError(
                f"native resident epoch returned status {native.status}",
                commit_state=native.commit_state,
                status=native.status,
            )
        committed = EpochCommitState.COMMITTED
        if native.commit_state != committed:
            raise ResidentEpochExecutionError(
                "successful native resident epoch was not committed", commit_state=native.commit_state
            )
        if snapshot is not None and native.kv_import_checksum != snapshot.checksum:
            raise ResidentEpochExecutionError(
                "resident KV import checksum disagrees with the Host snapshot", commit_state=committed
            )
        if device_transfer is not None and native.kv_import_checksum == 0:
            raise ResidentEpochExecutionError(
                "direct Device KV transfer did not return an import checksum", commit_state=committed
            )
        device_prefill = any(r.prompt_token_ids for r in plan.requests)
        if device_prefill and (not native.kv_imported or native.kv_import_checksum == 0):
            raise ResidentEpochExecutionError(
                "device prefill did not return an import checksum", commit_state=committed
            )
        if set(native.token_ids) != set(plan.req_ids):
            raise ResidentEpochExecutionError(
                "native resident epoch returned the wrong request set", commit_state=committed
            )
        req_ids = list(plan.req_ids)
        sampled = {r: native.token_ids[r] for r in req_ids}
        result = ResidentEpochResult(
            version=CONTRACT_VERSION,
            route="device",
            status=0,
            model_calls=native.model_calls,
            computed_steps={r: len(sampled[r]) for r in req_ids},
            row_generations=native.row_generations,
            commit_state=native.commit_state,
            feed_calls=native.feed_calls,
            fetch_calls=native.fetch_calls,
            wall_us=native.wall_us,
            native_cpu_us=native.native_cpu_us,
            declared_input_bytes=native.declared_input_bytes,
            declared_output_bytes=native.declared_output_bytes,
            socket_send_calls=native.socket_send_calls,
            socket_receive_calls=native.socket_receive_calls,
            kv_imported=native.kv_imported,
            kv_import_checksum=native.kv_import_checksum,
            kv_snapshot_checksum=snapshot.checksum if snapshot is not None else 0,
            kv_transfer_mode=(
                "device_ipc" if device_transfer is not None else "host_snapshot" if snapshot is not None
                else "device_prefill" if device_prefill else "none"
            ),
        )
        try:
            result.validate_against(plan, sampled)
        except Exception as exc:
            raise ResidentEpochExecutionError(
                f"committed resident epoch result is invalid: {exc}", commit_state=committed
            ) from exc
        output = _model_runner_output(req_ids, [sampled[r] for r in req_ids])
        attach_result(output, result)
        return output


def load_backend_from_env() -> ResidentEpochBackend:
    target = os.getenv(FACTORY_ENV)
    if not target or ":" not in target:
        raise RuntimeError(f"{FACTORY_ENV} must name a module:factory for the native epoch backend")
    module_name, factory_name = target.split(":", 1)
    return ResidentEpochBackend(getattr(import_module(module_name), factory_name)())


def host_fallback_result(req_ids: tuple[str, ...]) -> ResidentEpochResult:
    """Accounting record of a proven zero-model-call host replay (plugin.py:91-113)."""
    return ResidentEpochResult(
        version=CONTRACT_VERSION,
        route="host_fallback",
        status=0,
        model_calls=1,
        computed_steps={r: 1 for r in req_ids},
        commit_state=EpochCommitState.PREPARED,
        fallback_safe=True,
        feed_calls=0,
        fetch_calls=0,
    )


def execute_with_fallback(
    backend: ResidentEpochBackend | None,
    plan: ResidentEpochPlan,
    host_execute: Callable[[], Any],
    snapshot: ResidentKVSnapshot | None = None,
    device_transfer: DeviceKVTransfer | None = None,
):
    """Runs the epoch on the device; replays one host step only when the
    failure is input-preserving (PREPARED) and the host still owns every
    request (plugin.py:23-57).  Anything else propagates."""
    if backend is None:
        if not plan.host_replay_safe:
            raise RuntimeError("no resident backend and the device owns request state")
        output = host_execute()
        attach_result(output, host_fallback_result(plan.req_ids))
        return output
    try:
        return backend.execute(plan, snapshot=snapshot, device_transfer=device_transfer)
    except ResidentEpochExecutionError as exc:
        if not exc.input_preserving or not plan.host_replay_safe:
            raise
        output = host_execute()
        attach_result(output, host_fallback_result(plan.req_ids))
        return output

