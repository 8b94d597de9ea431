"""The resident epoch scheduler and dedicated worker inside vLLM 0.22's real V1
scheduler (CPU; no model runs).  Scenarios follow the reference's
tests/test_real_scheduler.py: fixed-graph plans for 1-4 greedy requests, the
host-prefill -> import -> device-owned transition, continuous admission with
an isolated host lane, rejection reasons, and the scheduler -> worker ->
scheduler control path through a deterministic native engine."""

from __future__ import annotations

import json

import pytest

vllm = pytest.importorskip("vllm")

from vllm import SamplingParams  # noqa: E402
from vllm.sampling_params import RequestOutputKind  # noqa: E402
from vllm.v1.outputs import ModelRunnerOutput  # noqa: E402
from vllm.v1.request import Request, RequestStatus  # noqa: E402

from cruise_b200.config import ResidentEpochConfig  # noqa: E402
from cruise_b200.contract import CONTRACT_VERSION, ResidentEpochResult, attach_result, get_plan  # noqa: E402
from cruise_b200.model_config import QWEN25_7B  # noqa: E402

EOS = QWEN25_7B.configured_eos


def hf_config_dir(tmp_path, preset=QWEN25_7B):
    """A Hugging Face config directory with an engine preset's geometry."""
    path = tmp_path / f"{preset.name}-config"
    path.mkdir(exist_ok=True)
    (path / "config.json").write_text(json.dumps({
        "architectures": ["Qwen2ForCausalLM"], "model_type": "qwen2", "hidden_size": preset.hidden,
        "intermediate_size": preset.intermediate, "num_hidden_layers": preset.num_layers,
        "num_attention_heads": preset.num_heads, "num_key_value_heads": preset.num_kv_heads,
        "vocab_size": preset.vocab, "max_position_embeddings": 32768, "rms_norm_eps": 1e-6,
        "rope_theta": 1000000.0, "torch_dtype": "bfloat16", "tie_word_embeddings": False,
        "hidden_act": "silu", "eos_token_id": preset.configured_eos,
    }))
    # the EOS vLLM gives requests when it has no tokenizer comes from here
    (path / "generation_config.json").write_text(json.dumps({"eos_token_id": preset.configured_eos}))
    return path


def make_scheduler(tmp_path, batch_size, config=None, preset=QWEN25_7B, max_model_len=256, adopt=True,
                   prefix_caching=True, num_blocks=16, max_batched_tokens=512):
    """vLLM's own V1 scheduler for the preset, turned into the resident one."""
    from vllm.config import CacheConfig, DeviceConfig, ModelConfig, SchedulerConfig, VllmConfig
    from vllm.v1.core.sched.scheduler import Scheduler
    from vllm.v1.kv_cache_interface import FullAttentionSpec, KVCacheConfig, KVCacheGroupSpec
    from vllm.v1.structured_output import StructuredOutputManager
    import torch

    from cruise_b200.scheduler import ResidentEpochScheduler

    model = ModelConfig(model=str(hf_config_dir(tmp_path, preset)), skip_tokenizer_init=True,
                        max_model_len=max_model_len, dtype="bfloat16")
    cache = CacheConfig(block_size=preset.block_size, enable_prefix_caching=prefix_caching)
    cache.num_gpu_blocks = num_blocks
    sched = SchedulerConfig(max_num_seqs=batch_size, max_num_batched_tokens=max_batched_tokens,
                            max_model_len=max_model_len,
                            is_encoder_decoder=False, async_scheduling=False)
    vc = VllmConfig(model_config=model, cache_config=cache, scheduler_config=sched,
                    device_config=DeviceConfig(device="cuda"))
    spec = FullAttentionSpec(block_size=preset.block_size, num_kv_heads=preset.num_kv_heads,
                             head_size=preset.head_dim, dtype=torch.bfloat16)
    kv = KVCacheConfig(num_blocks=num_blocks, kv_cache_tensors=[],
                       kv_cache_groups=[KVCacheGroupSpec([f"model.layers.{i}.self_attn" for i in
                                                          range(preset.num_layers)], spec)])
    cls = Scheduler if adopt else ResidentEpochScheduler
    scheduler = cls(vllm_config=vc, kv_cache_config=kv, log_stats=False,
                    structured_output_manager=StructuredOutputManager(vc), block_size=preset.block_size)
    if adopt:
        ResidentEpochScheduler.adopt(scheduler, config or ResidentEpochConfig(
            logical_capacity=min(256, 2 * preset.block_size), block_size=preset.block_size))
    return scheduler


def request(req_id, prompt, max_tokens, temperature=0.0, eos=EOS):
    params = SamplingParams(temperature=temperature, max_tokens=max_tokens)
    params.update_from_generation_config({}, eos)
    return Request(request_id=req_id, client_index=0, prompt_token_ids=list(prompt), sampling_params=params,
                   pooling_params=None)


def host_step(scheduler, output, tokens):
    ids = list(tokens)
    scheduler.update_from_output(output, ModelRunnerOutput(req_ids=ids, req_id_to_index={r: i for i, r in enumerate(ids)},
                                                           sampled_token_ids=[tokens[r] for r in ids]))


def commit_device_epoch(scheduler, output, tokens):
    plan = get_plan(output)
    assert plan is not None
    ids = list(plan.req_ids)
    runner = ModelRunnerOutput(req_ids=ids, req_id_to_index={r: i for i, r in enumerate(ids)},
                               sampled_token_ids=[tokens[r] for r in ids])
    importing = any(r.kv_import_required for r in plan.requests)
    attach_result(runner, ResidentEpochResult(
        version=CONTRACT_VERSION, route="device", status=0, model_calls=plan.max_steps,
        computed_steps={r: len(tokens[r]) for r in ids}, row_generations=plan.row_generations,
        kv_imported=importing, kv_import_checksum=1 if importing else 0, kv_snapshot_checksum=1 if importing else 0))
    scheduler.update_from_output(output, runner)
    return plan


@pytest.mark.parametrize("batch", [1, 2, 3, 4])
def test_fixed_graph_plan_and_commit(tmp_path, batch):
    scheduler = make_scheduler(tmp_path, batch)
    reqs = [request(str(i), [5 + i], max_tokens=8) for i in range(batch)]
    for r in reqs:
        scheduler.add_request(r)
    output = scheduler.schedule()
    plan = get_plan(output)
    assert plan is not None and plan.graph_batch_size == 4 and plan.max_steps == 8
    assert plan.active_mask == (1,) * batch + (0,) * (4 - batch)
    assert all(v == 1 for v in output.num_scheduled_tokens.values())
    assert all(len(r.scheduler_block_ids) == 1 for r in plan.requests)
    assert [r.generation for r in plan.requests] == list(range(1, batch + 1))
    commit_device_epoch(scheduler, output, {r: [100 + s for s in range(8)] for r in plan.req_ids})
    for r in reqs:
        assert (r.num_computed_tokens, r.num_tokens, r.num_output_tokens) == (8, 9, 8)
        assert r.status == RequestStatus.FINISHED_LENGTH_CAPPED


def test_unsupported_sampling_stays_on_the_host_path(tmp_path):
    scheduler = make_scheduler(tmp_path, 1)
    scheduler.add_request(request("0", [5], max_tokens=8, temperature=0.8))
    output = scheduler.schedule()
    assert get_plan(output) is None and scheduler.last_rejection == "non-greedy-temperature"
    assert scheduler.num_lookahead_tokens == 0


def test_delta_output_kind_allows_a_multi_token_epoch(tmp_path):
    scheduler = make_scheduler(tmp_path, 2, ResidentEpochConfig(max_steps=4))
    reqs = [request(str(i), [5 + i], max_tokens=6) for i in range(2)]
    reqs[1].sampling_params.output_kind = RequestOutputKind.DELTA
    for r in reqs:
        scheduler.add_request(r)
    plan = get_plan(scheduler.schedule())
    assert plan is not None and plan.max_steps == 4


def test_host_prefill_transitions_to_device_owned_decode(tmp_path):
    scheduler = make_scheduler(tmp_path, 1)
    r = request("0", [5, 6, 7], max_tokens=4)
    scheduler.add_request(r)
    prefill = scheduler.schedule()
    assert get_plan(prefill) is None and scheduler.last_rejection == "not-single-token-decode"
    host_step(scheduler, prefill, {"0": [101]})
    assert (r.num_computed_tokens, r.num_output_tokens) == (3, 1)
    first = scheduler.schedule()
    plan = get_plan(first)
    assert plan is not None and plan.max_steps == 2            # 3 tokens left -> K = 2
    q = plan.requests[0]
    assert (q.position, q.sequence_length, q.token_id, q.state_owner, q.kv_import_required) == (3, 4, 101, "host", True)
    commit_device_epoch(scheduler, first, {"0": [102, 103]})
    assert "0" in scheduler.resident.device_owned
    nxt = get_plan(scheduler.schedule())
    assert nxt.requests[0].state_owner == "device" and not nxt.requests[0].kv_import_required


def test_continuous_admission_isolates_host_prefill_and_reuses_rows(tmp_path):
    scheduler = make_scheduler(tmp_path, 2, ResidentEpochConfig(max_steps=2))
    a = request("A", [9707, 11], max_tokens=7)
    scheduler.add_request(a)
    prefill_a = scheduler.schedule()
    assert get_plan(prefill_a) is None
    host_step(scheduler, prefill_a, {"A": [101]})
    plan_a = commit_device_epoch(scheduler, scheduler.schedule(), {"A": [102, 103]})
    assert plan_a.max_steps == 2

    b = request("B", [9707, 11, 358], max_tokens=2)
    scheduler.add_request(b)
    prefill_b = scheduler.schedule()
    assert get_plan(prefill_b) is None and prefill_b.num_scheduled_tokens == {"B": 3}
    assert scheduler.last_rejection == "host-prefill-admission"
    assert [x.request_id for x in scheduler.running] == ["A", "B"]   # A paused, not dropped
    host_step(scheduler, prefill_b, {"B": [201]})
    import_b = scheduler.schedule()
    plan_b = get_plan(import_b)
    assert plan_b.max_steps == 1
    assert [(q.req_id, q.row, q.generation) for q in plan_b.requests] == [("A", 0, 1), ("B", 1, 2)]
    assert [(q.state_owner, q.kv_import_required) for q in plan_b.requests] == [("device", False), ("host", True)]
    commit_device_epoch(scheduler, import_b, {"A": [104], "B": [202]})
    assert b.status == RequestStatus.FINISHED_LENGTH_CAPPED

    c = request("C", [9707, 11, 358, 374], max_tokens=2)
    scheduler.add_request(c)
    prefill_c = scheduler.schedule()
    assert prefill_c.num_scheduled_tokens == {"C": 4} and scheduler.last_rejection == "host-prefill-admission"
    host_step(scheduler, prefill_c, {"C": [301]})
    plan_c = get_plan(import_c := scheduler.schedule())
    # C takes B's released row under a new generation
    assert [(q.req_id, q.row, q.generation) for q in plan_c.requests] == [("A", 0, 1), ("C", 1, 3)]
    commit_device_epoch(scheduler, import_c, {"A": [105], "C": [302]})
    finish = get_plan(finish_a := scheduler.schedule())
    assert finish.req_ids == ("A",) and finish.max_steps == 2
    commit_device_epoch(scheduler, finish_a, {"A": [106, 107]})
    assert a.status == RequestStatus.FINISHED_LENGTH_CAPPED


def test_unsupported_admission_runs_in_the_host_lane(tmp_path):
    scheduler = make_scheduler(tmp_path, 2, ResidentEpochConfig(max_steps=2))
    a = request("A", [9707, 11], max_tokens=7)
    scheduler.add_request(a)
    prefill_a = scheduler.schedule()
    host_step(scheduler, prefill_a, {"A": [101]})
    commit_device_epoch(scheduler, scheduler.schedule(), {"A": [102, 103]})
    u = request("u", [9707, 11], max_tokens=2, temperature=0.8)
    scheduler.add_request(u)
    out = scheduler.schedule()
    assert get_plan(out) is None and out.num_scheduled_tokens == {"u": 2}
    assert scheduler.last_rejection == "host-prefill-admission"
    host_step(scheduler, out, {"u": [201]})
    out = scheduler.schedule()
    assert get_plan(out) is None and out.num_scheduled_tokens == {"u": 1}
    assert scheduler.last_rejection == "unsupported-host-isolation"
    host_step(scheduler, out, {"u": [202]})
    assert u.status == RequestStatus.FINISHED_LENGTH_CAPPED
    resume = get_plan(scheduler.schedule())
    assert resume.req_ids == ("A",) and resume.requests[0].state_owner == "device"
    assert resume.requests[0].generation == 1


def test_two_prefills_beside_a_device_owned_request(tmp_path):
    scheduler = make_scheduler(tmp_path, 3, ResidentEpochConfig(max_steps=2))
    scheduler.add_request(request("A", [9707, 11], max_tokens=7))
    prefill_a = scheduler.schedule()
    host_step(scheduler, prefill_a, {"A": [101]})
    commit_device_epoch(scheduler, scheduler.schedule(), {"A": [102, 103]})
    scheduler.add_request(request("B", [9707, 11, 358], max_tokens=3))
    scheduler.add_request(request("C", [9707, 11, 358, 374], max_tokens=3))
    out = scheduler.schedule()
    assert get_plan(out) is None and out.num_scheduled_tokens == {"B": 3, "C": 4}
    host_step(scheduler, out, {"B": [201], "C": [301]})
    plan = get_plan(scheduler.schedule())
    assert plan.req_ids == ("A", "B", "C")
    assert [q.state_owner for q in plan.requests] == ["device", "host", "host"]
    assert [q.kv_import_required for q in plan.requests] == [False, True, True]


def test_scheduler_to_dedicated_worker_control_path(tmp_path, monkeypatch):
    from cruise_b200.worker import ResidentEpochWorker

    monkeypatch.setenv("VLLM_ASCEND_RESIDENT_EPOCH_BACKEND_FACTORY", "cruise_b200.testing:create_test_engine")
    scheduler = make_scheduler(tmp_path, 4)
    reqs = [request(str(i), [5 + i], max_tokens=4) for i in range(4)]
    for r in reqs:
        scheduler.add_request(r)
    output = scheduler.schedule()
    assert get_plan(output) is not None
    worker = ResidentEpochWorker(vllm_config=scheduler.vllm_config, local_rank=0, rank=0,
                                 distributed_init_method="tcp://127.0.0.1:1", is_driver_worker=True)
    worker.load_model()
    times = worker.compile_or_warm_up_model()
    assert times.language_model > 0 and worker.warmup_output.model_calls == 1
    assert len(worker.get_kv_cache_spec()) == QWEN25_7B.num_layers
    page = 2 * QWEN25_7B.block_size * QWEN25_7B.num_kv_heads * QWEN25_7B.head_dim * 2
    # the engine's 8 blocks plus vLLM's null block
    assert worker.determine_available_memory() == 9 * QWEN25_7B.num_layers * page
    scheduler.update_from_output(output, worker.execute_model(output))
    worker.shutdown()
    for r in reqs:
        assert (r.num_computed_tokens, r.num_output_tokens) == (4, 4)
        assert r.status == RequestStatus.FINISHED_LENGTH_CAPPED


def test_models_without_an_engine_preset_are_refused(tmp_path):
    from dataclasses import replace

    from cruise_b200.scheduler import native_model_rejection
    from types import SimpleNamespace

    good = SimpleNamespace(model_type="qwen2", num_hidden_layers=28, hidden_size=3584, num_attention_heads=28,
                           num_key_value_heads=4, intermediate_size=18944, vocab_size=152064)
    assert native_model_rejection(good) is None
    assert "vocab_size=151936" in native_model_rejection(replace_ns(good, vocab_size=151936))
    assert native_model_rejection(replace_ns(good, model_type="llama")).startswith("model_type")
    with pytest.raises(ValueError, match="native graph mismatch"):
        make_scheduler(tmp_path, 1, preset=replace(QWEN25_7B, vocab=151936, name="other"), adopt=False)
    make_scheduler(tmp_path, 1, adopt=False)   # the 7B preset itself is accepted


def replace_ns(ns, **changes):
    from types import SimpleNamespace

    return SimpleNamespace(**{**vars(ns), **changes})


def test_worker_names_the_rejection_of_a_host_step(tmp_path, monkeypatch):
    from cruise_b200.worker import ResidentEpochWorker

    monkeypatch.setenv("VLLM_ASCEND_RESIDENT_EPOCH_BACKEND_FACTORY", "cruise_b200.testing:create_test_engine")
    scheduler = make_scheduler(tmp_path, 1)
    scheduler.add_request(request("0", [5], max_tokens=8, temperature=0.8))
    output = scheduler.schedule()
    worker = ResidentEpochWorker(vllm_config=scheduler.vllm_config, local_rank=0, rank=0,
                                 distributed_init_method="tcp://127.0.0.1:1", is_driver_worker=True)
    worker.load_model()
    with pytest.raises(RuntimeError, match="scheduler: non-greedy-temperature"):
        worker.execute_model(output)
    assert worker.get_supported_tasks() == ("generate",)
    worker.shutdown()


def test_eos_from_a_single_stop_token_without_tokenizer(tmp_path):
    from cruise_b200.eligibility import effective_eos, request_rejection_reason

    scheduler = make_scheduler(tmp_path, 2)
    plain = request("p", [5], max_tokens=4)
    tokenizerless = Request(request_id="t", client_index=0, prompt_token_ids=[6], pooling_params=None,
                            sampling_params=SamplingParams(temperature=0.0, max_tokens=4))
    tokenizerless.sampling_params.update_from_generation_config({"eos_token_id": 77}, None)
    assert tokenizerless.sampling_params.eos_token_id is None and effective_eos(tokenizerless.sampling_params) == 77
    for r in (plain, tokenizerless):
        scheduler.add_request(r)
    plan = get_plan(scheduler.schedule())
    assert plan is not None and [q.eos_token_id for q in plan.requests] == [EOS, 77]
    both = request("b", [7], max_tokens=4)
    both.sampling_params.stop_token_ids = [9]
    assert request_rejection_reason(both) == "extra-stop-condition"
    two = Request(request_id="2", client_index=0, prompt_token_ids=[6], pooling_params=None,
                  sampling_params=SamplingParams(temperature=0.0, max_tokens=4, stop_token_ids=[3, 4]))
    assert request_rejection_reason(two) == "extra-stop-condition"
    none = Request(request_id="n", client_index=0, prompt_token_ids=[6], pooling_params=None,
                   sampling_params=SamplingParams(temperature=0.0, max_tokens=4))
    assert request_rejection_reason(none) == "missing-eos"


def test_resident_rows_reuse_freed_rows_with_fresh_generations():
    """Row bookkeeping (the reference's scheduler.py:62-86): a request keeps its
    row while it stays in the batch; a request that leaves frees its row and
    its device ownership; a new request takes the lowest free row and a
    generation never used before; more requests than rows, or an exhausted
    32-bit generation space, are errors rather than silent reuse."""
    from cruise_b200.scheduler import ResidentRows

    rows = ResidentRows()
    rows.assign(("a", "b", "c"), 4)
    assert rows.rows == {"a": 0, "b": 1, "c": 2} and rows.generations == {"a": 1, "b": 2, "c": 3}
    rows.device_owned.update({"a", "b"})
    rows.assign(("a", "c", "d", "e"), 4)               # b leaves; d takes its row, e the last one
    assert rows.rows == {"a": 0, "c": 2, "d": 1, "e": 3}
    assert rows.generations["d"] == 4 and rows.generations["e"] == 5 and rows.device_owned == {"a"}
    with pytest.raises(RuntimeError, match="exhausted"):
        rows.assign(("a", "c", "d", "e", "f"), 4)
    late = ResidentRows(next_generation=2**31 - 1)
    late.assign(("x",), 4)
    assert late.generations == {"x": 2**31 - 1}
    with pytest.raises(RuntimeError, match="generation space"):
        late.assign(("x", "y"), 4)


def device_prefill_config(**kw):
    return ResidentEpochConfig(logical_capacity=256, block_size=QWEN25_7B.block_size, device_prefill=True, **kw)


def test_device_prefill_puts_a_fresh_prompt_in_its_first_epoch(tmp_path):
    """device_prefill mode: a fresh prompt scheduled whole becomes a plan at
    once (no host step): the epoch prefills it on the device, imports its K/V
    and decodes from the last prompt token; vLLM's accounting then counts the
    prompt plus the K - 1 decoded positions as computed."""
    scheduler = make_scheduler(tmp_path, 1, device_prefill_config(max_steps=4))
    r = request("0", [5, 6, 7], max_tokens=6)
    scheduler.add_request(r)
    first = scheduler.schedule()
    plan = get_plan(first)
    assert plan is not None and first.num_scheduled_tokens == {"0": 3} and plan.max_steps == 4
    q = plan.requests[0]
    assert (q.position, q.sequence_length, q.token_id, q.state_owner, q.kv_import_required) == (2, 3, 7, "host", True)
    assert q.prompt_token_ids == (5, 6, 7)
    commit_device_epoch(scheduler, first, {"0": [101, 102, 103, 104]})
    assert (r.num_computed_tokens, r.num_tokens, r.num_output_tokens) == (6, 7, 4)
    assert "0" in scheduler.resident.device_owned
    nxt = scheduler.schedule()
    follow = get_plan(nxt)
    assert follow.max_steps == 2 and nxt.num_scheduled_tokens == {"0": 1}
    f = follow.requests[0]
    assert (f.position, f.token_id, f.state_owner, f.kv_import_required, f.prompt_token_ids) == (
        6, 104, "device", False, ())
    commit_device_epoch(scheduler, nxt, {"0": [105, 106]})
    assert r.status == RequestStatus.FINISHED_LENGTH_CAPPED


def test_device_prefill_joins_a_device_owned_request_without_a_host_lane(tmp_path):
    scheduler = make_scheduler(tmp_path, 2, device_prefill_config(max_steps=2))
    scheduler.add_request(request("A", [9707, 11], max_tokens=7))
    plan_a = commit_device_epoch(scheduler, scheduler.schedule(), {"A": [101, 102]})
    assert plan_a.requests[0].prompt_token_ids == (9707, 11)
    scheduler.add_request(request("B", [9707, 11, 358], max_tokens=3))
    out = scheduler.schedule()
    plan = get_plan(out)
    assert plan is not None and out.num_scheduled_tokens == {"A": 1, "B": 3}
    assert [(q.req_id, q.state_owner, q.prompt_token_ids) for q in plan.requests] == [
        ("A", "device", ()), ("B", "host", (9707, 11, 358))]
    commit_device_epoch(scheduler, out, {"A": [103, 104], "B": [201, 202]})
    assert scheduler.resident.device_owned == {"A", "B"}


def test_device_prefill_leaves_long_and_unsupported_prompts_to_the_host(tmp_path):
    # (prompts of a full block or more need the prefix cache's block hashes, which these bare requests lack)
    scheduler = make_scheduler(tmp_path, 1, device_prefill_config(), prefix_caching=False)
    scheduler.add_request(request("long", list(range(1, QWEN25_7B.block_size + 2)), max_tokens=2))
    out = scheduler.schedule()
    assert get_plan(out) is None and scheduler.last_rejection == "not-single-token-decode"
    sampled = make_scheduler(tmp_path, 1, device_prefill_config())
    sampled.add_request(request("t", [5, 6], max_tokens=2, temperature=0.8))
    assert get_plan(sampled.schedule()) is None and sampled.last_rejection == "not-single-token-decode"


def test_device_prefill_through_the_dedicated_worker(tmp_path, monkeypatch):
    from cruise_b200.worker import ResidentEpochWorker

    monkeypatch.setenv("VLLM_ASCEND_RESIDENT_EPOCH_BACKEND_FACTORY", "cruise_b200.testing:create_test_engine")
    scheduler = make_scheduler(tmp_path, 2, device_prefill_config(max_steps=4))
    reqs = [request("0", [5, 6, 7, 8], max_tokens=4), request("1", [9], max_tokens=4)]
    for r in reqs:
        scheduler.add_request(r)
    output = scheduler.schedule()
    plan = get_plan(output)
    assert [q.prompt_token_ids for q in plan.requests] == [(5, 6, 7, 8), ()]
    worker = ResidentEpochWorker(vllm_config=scheduler.vllm_config, local_rank=0, rank=0,
                                 distributed_init_method="tcp://127.0.0.1:1", is_driver_worker=True)
    worker.load_model()
    worker.compile_or_warm_up_model()
    runner = worker.execute_model(output)
    engine = worker._loaded_backend().engine
    assert engine.prefill_calls == 1
    scheduler.update_from_output(output, runner)
    assert scheduler.last_result.kv_transfer_mode == "device_prefill" and scheduler.last_result.kv_imported
    # the stand-in counts on from the last prompt token
    assert list(reqs[0].output_token_ids) == [9, 10, 11, 12] and list(reqs[1].output_token_ids) == [10, 11, 12, 13]
    worker.shutdown()


def test_four_rows_grow_to_two_blocks_without_preemption(tmp_path):
    """The dedicated worker offers vLLM the engine's 8 blocks plus one (vLLM
    keeps a null block), so four rows can all grow into their second block:
    every step stays a resident plan.  With only the 8 blocks vLLM would
    preempt a device-owned request."""
    from cruise_b200.model_config import QWEN25_7B as preset
    from cruise_b200.worker import ResidentKVLayout

    layout = ResidentKVLayout(preset, preset.block_size, preset.num_blocks)
    blocks = layout.capacity_bytes() // layout.bytes_per_block()
    assert blocks == preset.num_blocks + 1
    scheduler = make_scheduler(tmp_path, 4, device_prefill_config(max_steps=8), prefix_caching=False,
                               num_blocks=blocks)
    reqs = [request(str(i), [100 + i] * 120, max_tokens=24) for i in range(4)]
    for r in reqs:
        scheduler.add_request(r)
    steps = 0
    while not all(r.is_finished() for r in reqs):
        out = scheduler.schedule()
        plan = get_plan(out)
        assert plan is not None, scheduler.last_rejection
        commit_device_epoch(scheduler, out, {q.req_id: [7] * plan.max_steps for q in plan.requests})
        steps += 1
    assert steps == 3 and all(r.num_output_tokens == 24 for r in reqs)


def test_device_prefill_refuses_settings_that_split_prompts(tmp_path, monkeypatch):
    monkeypatch.setenv("VLLM_ASCEND_RESIDENT_EPOCH_DEVICE_PREFILL", "1")
    with pytest.raises(ValueError, match="enable_prefix_caching=False"):
        make_scheduler(tmp_path, 1, adopt=False)
    with pytest.raises(ValueError, match="max_num_batched_tokens >= 512"):
        make_scheduler(tmp_path, 1, adopt=False, prefix_caching=False, max_batched_tokens=256)
    make_scheduler(tmp_path, 1, adopt=False, prefix_caching=False)
