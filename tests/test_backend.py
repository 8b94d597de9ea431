"""Backend commit-state handling and host replay (reference tests/test_commit_fallback.py:42-87)."""

from types import SimpleNamespace

import pytest

from cruise_b200.backend import NativeEpochOutput, ResidentEpochBackend, execute_with_fallback
from cruise_b200.contract import (
    CONTRACT_VERSION, EpochCommitState, ResidentEpochExecutionError, ResidentEpochPlan, ResidentEpochRequest,
    get_result,
)
from cruise_b200.testing import DeterministicTestEngine


def plan(owner="host", steps=2):
    return ResidentEpochPlan(
        version=CONTRACT_VERSION, graph_batch_size=4, max_steps=steps, logical_capacity=256,
        requests=(ResidentEpochRequest(req_id="r0", row=0, generation=1, token_id=1, position=0, sequence_length=1,
                                       eos_token_id=9, scheduler_block_ids=(4,), device_block_ids=(0, 1),
                                       state_owner=owner),),
        active_mask=(1, 0, 0, 0),
    )


class FailingEngine:
    def __init__(self, state):
        self.state = state

    def execute(self, plan):
        raise ResidentEpochExecutionError("injected failure", commit_state=self.state)


def host_output():
    return SimpleNamespace(req_ids=["r0"], req_id_to_index={"r0": 0}, sampled_token_ids=[[7]])


def test_device_epoch_through_test_engine():
    engine = DeterministicTestEngine()
    out = ResidentEpochBackend(engine).execute(plan(steps=4))
    result = get_result(out)
    assert out.sampled_token_ids == [[2, 3, 4, 5]]
    assert result.route == "device" and result.model_calls == 4 and engine.execute_calls == 1


def test_prepared_failure_replays_when_host_still_owns_state():
    out = execute_with_fallback(ResidentEpochBackend(FailingEngine(EpochCommitState.PREPARED)), plan(), host_output)
    result = get_result(out)
    assert result.route == "host_fallback" and result.commit_state == EpochCommitState.PREPARED
    assert result.fallback_safe


@pytest.mark.parametrize("owner,state", [
    ("device", EpochCommitState.PREPARED), ("host", EpochCommitState.EXECUTING), ("host", EpochCommitState.COMMITTED),
])
def test_ambiguous_or_device_owned_failure_never_replays(owner, state):
    with pytest.raises(ResidentEpochExecutionError) as caught:
        execute_with_fallback(ResidentEpochBackend(FailingEngine(state)), plan(owner), host_output)
    assert caught.value.commit_state == state


def test_engine_exception_without_proof_is_executing():
    class Broken:
        def execute(self, plan):
            raise OSError("socket gone")

    with pytest.raises(ResidentEpochExecutionError) as caught:
        ResidentEpochBackend(Broken()).execute(plan())
    assert caught.value.commit_state == EpochCommitState.EXECUTING and not caught.value.input_preserving


def test_device_status_is_not_input_preserving():
    class Status:
        def execute(self, plan):
            return NativeEpochOutput(status=209, model_calls=1, token_ids={"r0": [1]}, row_generations=(1, 0, 0, 0))

    with pytest.raises(ResidentEpochExecutionError) as caught:
        ResidentEpochBackend(Status()).execute(plan())
    assert caught.value.status == 209 and caught.value.commit_state == EpochCommitState.COMMITTED


def test_invalid_plan_is_prepared():
    bad = ResidentEpochPlan(**{**plan().__dict__, "active_mask": (0, 1, 0, 0)})
    with pytest.raises(ResidentEpochExecutionError) as caught:
        ResidentEpochBackend(DeterministicTestEngine()).execute(bad)
    assert caught.value.input_preserving


def test_warmup_requires_one_complete_step():
    backend = ResidentEpochBackend(DeterministicTestEngine())
    assert backend.warm_up().model_calls == 1


def test_backend_factory_from_env(monkeypatch):
    from cruise_b200.backend import load_backend_from_env

    monkeypatch.setenv("VLLM_ASCEND_RESIDENT_EPOCH_BACKEND_FACTORY", "cruise_b200.testing:create_test_engine")
    assert isinstance(load_backend_from_env().engine, DeterministicTestEngine)
    monkeypatch.setenv("VLLM_ASCEND_RESIDENT_EPOCH_BACKEND_FACTORY", "nocolon")
    with pytest.raises(RuntimeError):
        load_backend_from_env()


def prefill_plan():
    return ResidentEpochPlan(
        version=CONTRACT_VERSION, graph_batch_size=4, max_steps=2, logical_capacity=256,
        requests=(ResidentEpochRequest(req_id="r0", row=0, generation=1, token_id=7, position=2, sequence_length=3,
                                       eos_token_id=9, scheduler_block_ids=(4,), device_block_ids=(0, 1),
                                       kv_import_required=True, prompt_token_ids=(5, 6, 7)),),
        active_mask=(1, 0, 0, 0),
    )


def test_device_prefill_plans_route_to_the_engine_prefill():
    """A plan whose requests carry prompts goes to execute_with_device_prefill
    and must come back with an import proof; an engine without that method
    (the sidecar's, say) or a second transfer source fails before any device
    work, so the host may replay."""
    engine = DeterministicTestEngine()
    out = ResidentEpochBackend(engine).execute(prefill_plan())
    result = get_result(out)
    assert engine.prefill_calls == 1 and engine.execute_calls == 1
    assert result.kv_imported and result.kv_transfer_mode == "device_prefill"
    assert out.sampled_token_ids[0] == [8, 9]

    class NoPrefill:
        def execute(self, plan):
            raise AssertionError("a prefill plan must not run as a plain epoch")

    with pytest.raises(ResidentEpochExecutionError) as caught:
        ResidentEpochBackend(NoPrefill()).execute(prefill_plan())
    assert caught.value.input_preserving

    class NoProof(DeterministicTestEngine):
        def execute_with_device_prefill(self, plan):
            return self._epoch(plan)   # no import checksum

    with pytest.raises(ResidentEpochExecutionError, match="import checksum"):
        ResidentEpochBackend(NoProof()).execute(prefill_plan())
