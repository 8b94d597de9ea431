"""vLLM 0.22's V1 ``EngineCore`` built directly (uniprocess executor) with the
resident epoch scheduler and dedicated worker on the deterministic test
engine (tokens ``token + step + 1``, no GPU work), after the reference's
tests/test_engine_core_runner.py:

* the engine core resolves the resident scheduler and worker, brings up and
  tears down torch.distributed, warms the backend up once, and runs one
  K-step epoch for a two-request cohort;
* a dynamic cohort A -> [A, B] -> [A, C] (B finishes, C takes its row with a
  new generation), checked plan by plan: rows, generations, positions, input
  tokens, the tokens of every epoch and the number of epochs executed.

Without a GPU vLLM resolves no device platform and refuses an empty device
string; the control path needs no device, so the tests give vLLM's device
config the CUDA device type it would resolve on a GPU host.
"""

from __future__ import annotations

import time

import pytest

pytest.importorskip("vllm")

from test_vllm_scheduler import hf_config_dir  # noqa: E402

WORKER = "cruise_b200.worker.ResidentEpochWorker"
SCHEDULER = "cruise_b200.scheduler.ResidentEpochScheduler"


@pytest.fixture
def cuda_device_type(monkeypatch):
    """vLLM's device config resolves an unset device to CUDA, as on a GPU host."""
    from vllm.config import DeviceConfig

    post_init = DeviceConfig.__post_init__

    def resolve(self):
        if not self.device or self.device == "auto":
            self.device = "cuda"
        post_init(self)

    monkeypatch.setattr(DeviceConfig, "__post_init__", resolve)


def make_engine_core(model_dir, preset, max_model_len, prefix_caching=True):
    from vllm.engine.arg_utils import EngineArgs
    from vllm.v1.engine.core import EngineCore
    from vllm.v1.executor.uniproc_executor import UniProcExecutor

    config = EngineArgs(model=str(model_dir), skip_tokenizer_init=True, max_model_len=max_model_len,
                        block_size=preset.block_size, max_num_seqs=4, async_scheduling=False,
                        enforce_eager=True, dtype="bfloat16", worker_cls=WORKER, scheduler_cls=SCHEDULER,
                        enable_prefix_caching=prefix_caching).create_engine_config()
    return EngineCore(vllm_config=config, executor_class=UniProcExecutor, log_stats=True)


def add_request(core, req_id, client, token, max_tokens, eos):
    from vllm import SamplingParams
    from vllm.v1.engine import EngineCoreRequest

    params = SamplingParams(temperature=0.0, max_tokens=max_tokens, detokenize=False)
    params.update_from_generation_config({}, eos)
    req, wave = core.preprocess_add_request(EngineCoreRequest(
        request_id=req_id, prompt_token_ids=[token], mm_features=None, sampling_params=params,
        pooling_params=None, arrival_time=time.time(), lora_request=None, cache_salt=None,
        data_parallel_rank=None, client_index=client))
    core.add_request(req, wave)


class PlanRecorder:
    """Keeps the resident plan of every schedule() the engine core makes."""

    def __init__(self, scheduler):
        from cruise_b200.contract import get_plan

        self.plans = []
        inner = scheduler.schedule

        def schedule():
            output = inner()
            self.plans.append(get_plan(output))
            return output

        scheduler.schedule = schedule


def epoch(core):
    """One engine-core step: the tokens each request received."""
    outputs, executed = core.step()
    core.post_step(executed)
    tokens = {}
    for client_outputs in outputs.values():
        for out in client_outputs.outputs:
            tokens.setdefault(out.request_id, []).extend(out.new_token_ids)
    return tokens


def run_dynamic_cohort(core, token, eos):
    recorder = PlanRecorder(core.scheduler)
    add_request(core, "A", 0, token, 6, eos)
    epochs = [epoch(core)]
    add_request(core, "B", 1, token, 2, eos)
    epochs.append(epoch(core))
    add_request(core, "C", 2, token, 2, eos)
    epochs.append(epoch(core))
    assert epoch(core) == {} and not core.scheduler.has_requests()
    return epochs, recorder.plans[:3]


def check_dynamic_cohort(epochs, plans, token, want):
    assert epochs == [{"A": want[0:2]}, {"A": want[2:4], "B": want[0:2]}, {"A": want[4:6], "C": want[0:2]}]
    expected_plans = [
        {"A": (0, 1, 0, token)},
        {"A": (0, 1, 2, want[1]), "B": (1, 2, 0, token)},
        {"A": (0, 1, 4, want[3]), "C": (1, 3, 0, token)},
    ]
    expected_generations = [(1, 0, 0, 0), (1, 2, 0, 0), (1, 3, 0, 0)]
    for plan, expected, generations in zip(plans, expected_plans, expected_generations):
        assert plan is not None and plan.max_steps == 2
        assert {r.req_id: (r.row, r.generation, r.position, r.token_id) for r in plan.requests} == expected
        assert plan.row_generations == generations


def test_engine_core_resolves_resident_scheduler_worker_and_epoch(cuda_device_type, tmp_path, monkeypatch):
    import torch
    from vllm.v1.executor.uniproc_executor import UniProcExecutor

    from cruise_b200.model_config import QWEN25_7B
    from cruise_b200.scheduler import ResidentEpochScheduler
    from cruise_b200.worker import ResidentEpochWorker

    monkeypatch.setenv("VLLM_ASCEND_RESIDENT_EPOCH_BACKEND_FACTORY", "cruise_b200.testing:create_test_engine")
    monkeypatch.setenv("VLLM_ASCEND_RESIDENT_EPOCH_MODEL", QWEN25_7B.name)
    monkeypatch.setenv("VLLM_ASCEND_RESIDENT_EPOCH_STEPS", "4")
    monkeypatch.setenv("VLLM_ASCEND_RESIDENT_EPOCH_CAPACITY", "8")
    monkeypatch.setenv("VLLM_ENABLE_V1_MULTIPROCESSING", "0")
    core = make_engine_core(hf_config_dir(tmp_path, QWEN25_7B), QWEN25_7B, 8)
    try:
        worker = core.model_executor.driver_worker.worker
        assert isinstance(core.scheduler, ResidentEpochScheduler)
        assert isinstance(core.model_executor, UniProcExecutor)
        assert isinstance(worker, ResidentEpochWorker)
        assert torch.distributed.is_initialized()
        assert worker.warmup_output is not None and worker.warmup_output.model_calls == 1
        assert worker.backend.engine.warmup_calls == 1

        recorder = PlanRecorder(core.scheduler)
        for i, req_id in enumerate(("0", "1")):
            add_request(core, req_id, i, 11690, 4, QWEN25_7B.configured_eos)
        tokens = epoch(core)
        assert tokens == {"0": [11691, 11692, 11693, 11694], "1": [11691, 11692, 11693, 11694]}
        plan = recorder.plans[0]
        assert plan is not None and plan.max_steps == 4 and plan.row_generations == (1, 2, 0, 0)
        assert worker.backend.engine.execute_calls == 1
        assert epoch(core) == {} and not core.scheduler.has_requests()
    finally:
        core.shutdown()
    assert not torch.distributed.is_initialized()


def test_engine_core_dynamic_cohort_on_the_test_engine(cuda_device_type, tmp_path, monkeypatch):
    import torch

    from cruise_b200.model_config import QWEN25_7B

    monkeypatch.setenv("VLLM_ASCEND_RESIDENT_EPOCH_BACKEND_FACTORY", "cruise_b200.testing:create_test_engine")
    monkeypatch.setenv("VLLM_ASCEND_RESIDENT_EPOCH_MODEL", QWEN25_7B.name)
    monkeypatch.setenv("VLLM_ASCEND_RESIDENT_EPOCH_STEPS", "2")
    monkeypatch.setenv("VLLM_ASCEND_RESIDENT_EPOCH_CAPACITY", "8")
    monkeypatch.setenv("VLLM_ENABLE_V1_MULTIPROCESSING", "0")
    core = make_engine_core(hf_config_dir(tmp_path, QWEN25_7B), QWEN25_7B, 8)
    try:
        worker = core.model_executor.driver_worker.worker
        assert worker.warmup_output.model_calls == 1 and worker.backend.engine.warmup_calls == 1
        epochs, plans = run_dynamic_cohort(core, 11690, QWEN25_7B.configured_eos)
        check_dynamic_cohort(epochs, plans, 11690, [11690 + 1 + i for i in range(6)])
        assert worker.backend.engine.execute_calls == 3
    finally:
        core.shutdown()
    assert not torch.distributed.is_initialized()


def test_engine_core_device_prefill_on_the_test_engine(cuda_device_type, tmp_path, monkeypatch):
    """VLLM_ASCEND_RESIDENT_EPOCH_DEVICE_PREFILL=1: multi-token prompts go
    straight into the first resident epoch (the engine prefills them on the
    device); the stand-in counts on from each last prompt token."""
    import time as _time

    from vllm import SamplingParams
    from vllm.v1.engine import EngineCoreRequest

    from cruise_b200.model_config import QWEN25_7B

    monkeypatch.setenv("VLLM_ASCEND_RESIDENT_EPOCH_BACKEND_FACTORY", "cruise_b200.testing:create_test_engine")
    monkeypatch.setenv("VLLM_ASCEND_RESIDENT_EPOCH_MODEL", QWEN25_7B.name)
    monkeypatch.setenv("VLLM_ASCEND_RESIDENT_EPOCH_STEPS", "4")
    monkeypatch.setenv("VLLM_ASCEND_RESIDENT_EPOCH_DEVICE_PREFILL", "1")
    monkeypatch.setenv("VLLM_ENABLE_V1_MULTIPROCESSING", "0")
    core = make_engine_core(hf_config_dir(tmp_path, QWEN25_7B), QWEN25_7B, 256, prefix_caching=False)
    try:
        recorder = PlanRecorder(core.scheduler)
        prompts = {"p": [9707, 11, 358, 374], "q": [500, 501]}
        for client, (req_id, prompt) in enumerate(prompts.items()):
            params = SamplingParams(temperature=0.0, max_tokens=6, detokenize=False)
            params.update_from_generation_config({}, QWEN25_7B.configured_eos)
            req, wave = core.preprocess_add_request(EngineCoreRequest(
                request_id=req_id, prompt_token_ids=prompt, mm_features=None, sampling_params=params,
                pooling_params=None, arrival_time=_time.time(), lora_request=None, cache_salt=None,
                data_parallel_rank=None, client_index=client))
            core.add_request(req, wave)
        first = epoch(core)
        assert first == {"p": [375, 376, 377, 378], "q": [502, 503, 504, 505]}
        plan = recorder.plans[0]
        assert {r.req_id: r.prompt_token_ids for r in plan.requests} == {k: tuple(v) for k, v in prompts.items()}
        assert core.model_executor.driver_worker.worker.backend.engine.prefill_calls == 1
        second = epoch(core)
        assert second == {"p": [379, 380], "q": [506, 507]}
        assert all(not r.prompt_token_ids and r.state_owner == "device" for r in recorder.plans[1].requests)
        assert epoch(core) == {} and not core.scheduler.has_requests()
    finally:
        core.shutdown()
