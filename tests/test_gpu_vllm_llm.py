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
