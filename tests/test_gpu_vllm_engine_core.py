"""The reference's dynamic engine-core cohort (A -> [A, B] -> [A, C], row 1
reused with a new generation) through vLLM 0.22's V1 ``EngineCore``, the
resident epoch scheduler and the dedicated worker on the B200 engine (tiny
model).  Plans must match row for row, and every request's tokens must equal
the oracle's single-row greedy decode of the prompt token: rows do not
interact in the engine's arithmetic."""

from __future__ import annotations

import pytest

pytest.importorskip("vllm")

from test_vllm_engine_core import check_dynamic_cohort, make_engine_core, run_dynamic_cohort  # noqa: E402
from test_vllm_scheduler import hf_config_dir  # noqa: E402

pytestmark = pytest.mark.gpu


def test_engine_core_dynamic_cohort_on_the_b200_engine(cuda_ok, tmp_path, monkeypatch):
    import torch

    from cruise_b200.model_config import TINY
    from test_gpu_vllm_llm import _oracle_greedy

    token = 11
    want = _oracle_greedy(token, 6)
    assert len(want) == 6 and TINY.configured_eos not in want
    monkeypatch.setenv("VLLM_ASCEND_RESIDENT_EPOCH_BACKEND_FACTORY", "cruise_b200.cuda_backend:create_cuda_engine")
    monkeypatch.setenv("VLLM_ASCEND_RESIDENT_EPOCH_MODEL", "tiny")
    monkeypatch.setenv("VLLM_ASCEND_RESIDENT_EPOCH_EXTERNAL_WEIGHTS", "synthetic:0")
    monkeypatch.setenv("VLLM_ASCEND_RESIDENT_EPOCH_STEPS", "2")
    monkeypatch.setenv("VLLM_ENABLE_V1_MULTIPROCESSING", "0")
    core = make_engine_core(hf_config_dir(tmp_path, TINY), TINY, TINY.capacity)
    try:
        epochs, plans = run_dynamic_cohort(core, token, TINY.configured_eos)
        check_dynamic_cohort(epochs, plans, token, want)
    finally:
        # closes the worker's bridge engine (one per process)
        core.shutdown()
    assert not torch.distributed.is_initialized()
