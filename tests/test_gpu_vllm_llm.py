"""vLLM's own front end (`LLM.generate`, V1 engine core in-process) with the
resident epoch scheduler and dedicated worker on the B200 engine (tiny
model): the engine core brings the worker up through vLLM's executor
(init_device, load_model, KV sizing, warm-up), schedules through the resident
scheduler and returns the engine's tokens.  Each request's greedy tokens must
equal the oracle's single-row greedy decode of the same prompt -- rows do not
interact in the engine's arithmetic, so batching does not change them."""

from __future__ import annotations

import pytest

pytest.importorskip("vllm")

from test_vllm_scheduler import hf_config_dir  # noqa: E402

pytestmark = pytest.mark.gpu


def _oracle_greedy(prompt_token: int, steps: int) -> list[int]:
    import numpy as np

    from cruise_b200.model_config import TINY
    from oracle.decoder import OracleDecoder
    from oracle.epoch import OracleEpochController
    from oracle.model import TINY as ORACLE_TINY, seeded_weights
    from scenario import compute_slot

    oracle = OracleEpochController(OracleDecoder(ORACLE_TINY, seeded_weights(ORACLE_TINY, 0)))
    block_table = np.arange(8, dtype=np.int32).reshape(4, 2)
    token = np.array([prompt_token, 0, 0, 0], dtype=np.int64)
    position = np.zeros(4, dtype=np.int64)
    slot = np.array([compute_slot(block_table, TINY.block_size, r, 0) for r in range(4)], dtype=np.int32)
    eos = TINY.configured_eos
    control = np.array([8, eos, eos, eos, eos, 0, 0, 1, 0, 0, 0], dtype=np.int32)
    history, _ = oracle.run(token=token, position=position, seq_len=np.array([1, 0, 0, 0], dtype=np.int32),
                            slot=slot, active=np.array([1, 0, 0, 0], dtype=np.int32),
                            block_table=block_table.reshape(-1), control=control)
    out = [int(t) for t in history[:, 0] if t >= 0]
    return out[:steps]


def test_llm_generate_through_the_resident_engine(cuda_ok, tmp_path, monkeypatch):
    from vllm import LLM, SamplingParams

    from cruise_b200.model_config import TINY

    monkeypatch.setenv("VLLM_ASCEND_RESIDENT_EPOCH_BACKEND_FACTORY", "cruise_b200.cuda_backend:create_cuda_engine")
    monkeypatch.setenv("VLLM_ASCEND_RESIDENT_EPOCH_MODEL", "tiny")
    monkeypatch.setenv("VLLM_ASCEND_RESIDENT_EPOCH_EXTERNAL_WEIGHTS", "synthetic:0")
    monkeypatch.setenv("VLLM_ENABLE_V1_MULTIPROCESSING", "0")
    llm = LLM(model=str(hf_config_dir(tmp_path, TINY)), skip_tokenizer_init=True, max_model_len=TINY.capacity,
              block_size=TINY.block_size, max_num_seqs=4, async_scheduling=False, enforce_eager=True,
              dtype="bfloat16", worker_cls="cruise_b200.worker.ResidentEpochWorker",
              scheduler_cls="cruise_b200.scheduler.ResidentEpochScheduler")
    try:
        prompts = [11, 108, 205]
        params = SamplingParams(temperature=0.0, max_tokens=7, detokenize=False)
        outputs = llm.generate([{"prompt_token_ids": [t]} for t in prompts], params)
    finally:
        # the executor's shutdown reaches the worker, which closes the engine
        # (one bridge engine per process: later tests create their own)
        llm.llm_engine.engine_core.shutdown()
    for prompt, output in zip(prompts, outputs):
        got = list(output.outputs[0].token_ids)
        want = _oracle_greedy(prompt, 7)
        assert got == want[: len(got)] and (len(got) == 7 or got[-1] == TINY.configured_eos), (prompt, got, want)


def _oracle_prompt_greedy(prompt: list[int], steps: int):
    """The oracle's token-by-token prefill of ``prompt`` in row 0 and its
    greedy decode: (tokens, top-2 margins per step)."""
    import numpy as np

    from cruise_b200.model_config import TINY
    from oracle.decoder import OracleDecoder
    from oracle.epoch import EpochTrace, OracleEpochController
    from oracle.model import TINY as ORACLE_TINY, seeded_weights
    from scenario import Scenario, decode_inputs, prefill_epochs

    oracle = OracleEpochController(OracleDecoder(ORACLE_TINY, seeded_weights(ORACLE_TINY, 0)))
    eos = TINY.configured_eos
    sc = Scenario(block_table=np.arange(8, dtype=np.int32).reshape(4, 2), prompts=[prompt, [], [], []],
                  budgets=[8, 0, 0, 0], generations=[1, 0, 0, 0], eos=[eos] * 4, k=8)
    for inputs in prefill_epochs(sc, TINY.block_size, TINY.vocab):
        oracle.run(**inputs)
    trace = EpochTrace()
    history, _ = oracle.run(**decode_inputs(sc, TINY.block_size), trace=trace)
    tokens = [int(t) for t in history[:, 0] if t >= 0]
    return tokens[:steps], [m[0] for m in trace.margins]


def test_llm_generate_prefills_prompts_on_the_device(cuda_ok, tmp_path, monkeypatch):
    """device_prefill mode (VLLM_ASCEND_RESIDENT_EPOCH_DEVICE_PREFILL=1): vLLM
    admits multi-token prompts straight into resident epochs; the engine
    prefills them on the device (batched tcgen05 prefill), imports their K/V
    and decodes.  No step runs on a host lane.  Each request's greedy tokens
    equal the oracle's token-by-token prefill and decode of its prompt, except
    after a step whose oracle top-2 margin is below 2e-2."""
    from vllm import LLM, SamplingParams

    from cruise_b200.model_config import TINY

    monkeypatch.setenv("VLLM_ASCEND_RESIDENT_EPOCH_BACKEND_FACTORY", "cruise_b200.cuda_backend:create_cuda_engine")
    monkeypatch.setenv("VLLM_ASCEND_RESIDENT_EPOCH_MODEL", "tiny")
    monkeypatch.setenv("VLLM_ASCEND_RESIDENT_EPOCH_EXTERNAL_WEIGHTS", "synthetic:0")
    monkeypatch.setenv("VLLM_ASCEND_RESIDENT_EPOCH_DEVICE_PREFILL", "1")
    monkeypatch.setenv("VLLM_ENABLE_V1_MULTIPROCESSING", "0")
    llm = LLM(model=str(hf_config_dir(tmp_path, TINY)), skip_tokenizer_init=True, max_model_len=TINY.capacity,
              block_size=TINY.block_size, max_num_seqs=4, async_scheduling=False, enforce_eager=True,
              dtype="bfloat16", enable_prefix_caching=False, worker_cls="cruise_b200.worker.ResidentEpochWorker",
              scheduler_cls="cruise_b200.scheduler.ResidentEpochScheduler")
    prompts = [[11, 12, 13], [108, 5], [205, 7, 9, 300, 41, 2, 77, 1000, 3, 9, 8, 7], [400]]
    try:
        params = SamplingParams(temperature=0.0, max_tokens=7, detokenize=False)
        # a step outside a resident plan would reach the dedicated worker and fail
        outputs = llm.generate([{"prompt_token_ids": p} for p in prompts], params)
    finally:
        llm.llm_engine.engine_core.shutdown()
    for prompt, output in zip(prompts, outputs):
        got = list(output.outputs[0].token_ids)
        want, margins = _oracle_prompt_greedy(prompt, 7)
        same = 0
        while same < min(len(got), len(want)) and got[same] == want[same]:
            same += 1
        if same < len(got):
            assert same < len(margins) and margins[same] < 2e-2, (prompt, got, want, same)
        assert len(got) == 7 or got[-1] == TINY.configured_eos, (prompt, got)
