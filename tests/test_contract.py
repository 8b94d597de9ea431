"""Epoch contract rules (reference tests/test_contract.py:98-271)."""

from types import SimpleNamespace

import pytest

from cruise_b200.contract import (
    CONTRACT_VERSION, EpochCommitState, ResidentEpochExecutionError, ResidentEpochPlan, ResidentEpochRequest,
    ResidentEpochResult, attach_plan, get_plan,
)
from cruise_b200.eligibility import request_rejection_reason
from cruise_b200.config import ResidentEpochConfig, epoch_steps


def make_request(**overrides):
    params = SimpleNamespace(
        temperature=0.0, top_p=1.0, top_k=0, min_p=0.0, presence_penalty=0.0, frequency_penalty=0.0,
        repetition_penalty=1.0, min_tokens=0, ignore_eos=False, eos_token_id=151645, stop=[], stop_token_ids=[],
        logprobs=None, prompt_logprobs=None, logit_bias=None, allowed_token_ids=None, bad_words=[],
        repetition_detection=None, extra_args=None,
    )
    request = SimpleNamespace(pooling_params=None, mm_features=[], lora_request=None, prompt_embeds=None,
                              use_structured_output=False, sampling_params=params)
    for key, value in overrides.items():
        setattr(params if hasattr(params, key) else request, key, value)
    return request


def make_plan(owner="host", import_required=False, capacity=8) -> ResidentEpochPlan:
    return ResidentEpochPlan(
        version=CONTRACT_VERSION, graph_batch_size=1, max_steps=4, logical_capacity=capacity,
        requests=(ResidentEpochRequest(req_id="r0", row=0, generation=1, token_id=1, position=0, sequence_length=1,
                                       eos_token_id=9, scheduler_block_ids=(17,), device_block_ids=(0, 1),
                                       state_owner=owner, kv_import_required=import_required),),
        active_mask=(1,),
    )


def device_result(plan, steps, **kw):
    return ResidentEpochResult(version=CONTRACT_VERSION, route="device", status=0, model_calls=steps,
                               computed_steps={"r0": steps}, row_generations=plan.row_generations, **kw)


def test_greedy_request_is_eligible():
    assert request_rejection_reason(make_request()) is None


@pytest.mark.parametrize(("field", "value", "reason"), [
    ("temperature", 0.8, "non-greedy-temperature"), ("top_k", 8, "unsupported-sampling-filter"),
    ("presence_penalty", 0.1, "sampling-penalty"), ("min_tokens", 2, "min-tokens"), ("ignore_eos", True, "ignore-eos"),
    ("stop_token_ids", [7], "extra-stop-condition"), ("logprobs", 1, "logprobs"),
    ("allowed_token_ids", [1, 2], "logit-processor"), ("lora_request", object(), "lora"),
])
def test_unsupported_semantics_are_rejected(field, value, reason):
    assert request_rejection_reason(make_request(**{field: value})) == reason


def test_short_device_result_requires_eos():
    plan = make_plan()
    with pytest.raises(ValueError, match="terminate at EOS"):
        device_result(plan, 2).validate_against(plan, {"r0": [3, 4]})
    device_result(plan, 2).validate_against(plan, {"r0": [3, 9]})


def test_host_fallback_keeps_one_step_accounting():
    plan = make_plan()
    result = ResidentEpochResult(version=CONTRACT_VERSION, route="host_fallback", status=0, model_calls=1,
                                 computed_steps={"r0": 1}, commit_state=EpochCommitState.PREPARED, fallback_safe=True,
                                 feed_calls=0, fetch_calls=0)
    result.validate_against(plan, {"r0": [3]})
    with pytest.raises(ValueError, match="Host no longer owns"):
        result.validate_against(make_plan(owner="device"), {"r0": [3]})


@pytest.mark.parametrize("state", [EpochCommitState.PREPARED, EpochCommitState.EXECUTING])
def test_device_result_requires_committed_state(state):
    plan = make_plan()
    with pytest.raises(ValueError, match="not committed"):
        device_result(plan, 4, commit_state=state).validate_against(plan, {"r0": [2, 3, 4, 5]})


def test_only_prepared_execution_error_is_input_preserving():
    assert ResidentEpochExecutionError("x", commit_state=EpochCommitState.PREPARED).input_preserving
    assert not ResidentEpochExecutionError("x", commit_state=EpochCommitState.EXECUTING).input_preserving
    assert not ResidentEpochExecutionError("x", commit_state=EpochCommitState.COMMITTED).input_preserving


def test_kv_import_requires_host_ownership_and_commit_acknowledgement():
    plan = make_plan(import_required=True)
    plan.validate()
    with pytest.raises(ValueError, match="did not commit"):
        device_result(plan, 4).validate_against(plan, {"r0": [2, 3, 4, 5]})
    proven = device_result(plan, 4, kv_imported=True, kv_import_checksum=123, kv_snapshot_checksum=123)
    proven.validate_against(plan, {"r0": [2, 3, 4, 5]})
    with pytest.raises(ValueError, match="equivalent imported KV"):
        device_result(plan, 4, kv_imported=True, kv_import_checksum=124, kv_snapshot_checksum=123).validate_against(
            plan, {"r0": [2, 3, 4, 5]})
    with pytest.raises(ValueError, match="Host-owned"):
        make_plan(owner="device", import_required=True).validate()


def test_plan_capacity_is_the_row_capacity():
    with pytest.raises(ValueError, match="logical capacity"):
        ResidentEpochPlan(**{**make_plan().__dict__, "requests": (ResidentEpochRequest(**{
            **make_plan().requests[0].__dict__, "position": 6, "sequence_length": 7}),)}).validate()
    make_plan(capacity=256).validate()


def test_attach_and_get_plan_round_trip():
    holder = SimpleNamespace()
    plan = make_plan()
    attach_plan(holder, plan)
    assert get_plan(holder) is plan
    holder._ascend_resident_epoch_plan = "junk"
    with pytest.raises(TypeError):
        get_plan(holder)


def test_epoch_steps_and_config():
    assert [epoch_steps(b) for b in (1, 2, 3, 4, 7, 8, 20)] == [1, 2, 2, 4, 4, 8, 8]
    ResidentEpochConfig().validate()
    with pytest.raises(ValueError):
        ResidentEpochConfig(max_steps=3).validate()


def prefill_plan(prompt, **request_overrides) -> ResidentEpochPlan:
    fields = dict(req_id="r0", row=0, generation=1, token_id=prompt[-1], position=len(prompt) - 1,
                  sequence_length=len(prompt), eos_token_id=9, scheduler_block_ids=(17,), device_block_ids=(0, 1),
                  state_owner="host", kv_import_required=True, prompt_token_ids=tuple(prompt))
    fields.update(request_overrides)
    return ResidentEpochPlan(version=CONTRACT_VERSION, graph_batch_size=1, max_steps=4, logical_capacity=256,
                             requests=(ResidentEpochRequest(**fields),), active_mask=(1,))


def test_device_prefill_request_rules():
    """A device-prefilled request (an extension over the reference) carries its
    whole prompt, imports Host-owned state and decodes from the last prompt
    token; its result proves the import like a device transfer does."""
    plan = prefill_plan([5, 6, 7])
    plan.validate()
    for bad, message in (
        (prefill_plan([5]), "at least two tokens"),
        (prefill_plan([5, 6, 7], kv_import_required=False), "imports Host-owned"),
        (prefill_plan([5, 6, 7], state_owner="device", kv_import_required=False), "imports Host-owned"),
        (prefill_plan([5, 6, 7], token_id=6), "last prompt token"),
        (prefill_plan([5, 6, 7], position=1, sequence_length=2), "last prompt token"),
    ):
        with pytest.raises(ValueError, match=message):
            bad.validate()
    good = device_result(plan, 4, kv_imported=True, kv_import_checksum=7, kv_transfer_mode="device_prefill")
    good.validate_against(plan, {"r0": [1, 2, 3, 4]})
    with pytest.raises(ValueError, match="did not commit the requested KV import"):
        device_result(plan, 4).validate_against(plan, {"r0": [1, 2, 3, 4]})
    with pytest.raises(ValueError, match="did not prove an imported KV transfer"):
        device_result(plan, 4, kv_imported=True, kv_transfer_mode="device_prefill").validate_against(
            plan, {"r0": [1, 2, 3, 4]})
