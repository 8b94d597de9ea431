"""vLLM's V1 scheduler driving the B200 engine end to end: the resident epoch
scheduler plans greedy epochs, the dedicated worker runs them on the CUDA
engine through the reference-compatible bridge, and vLLM's accounting
advances by K tokens per epoch until every request is done.  Every epoch's
tokens equal the oracle's restatement of the bridge on the same plan."""

from __future__ import annotations

import pytest

pytest.importorskip("vllm")

from test_vllm_scheduler import make_scheduler, request  # noqa: E402

pytestmark = pytest.mark.gpu


def _oracle_tokens(oracle, plan, configured_eos):
    from oracle.epoch import bridge_execute

    toks, pos, lens, eos = [0] * 4, [0] * 4, [0] * 4, [configured_eos] * 4
    for r in plan.requests:
        toks[r.row], pos[r.row], lens[r.row], eos[r.row] = r.token_id, r.position, r.sequence_length, r.eos_token_id
    res = bridge_execute(oracle, len(plan.requests), plan.max_steps, toks, pos, lens, eos,
                         list(plan.row_generations), configured_eos=configured_eos)
    return {r.req_id: [int(t) for t in res.tokens[r.row * 8: r.row * 8 + res.executed[r.row]]] for r in plan.requests}


def test_vllm_scheduler_runs_cohorts_on_the_engine(cuda_ok, tmp_path, monkeypatch):
    from vllm.v1.request import RequestStatus

    from cruise_b200.config import ResidentEpochConfig
    from cruise_b200.contract import get_plan, get_result
    from cruise_b200.model_config import TINY
    from cruise_b200.worker import ResidentEpochWorker
    from oracle.decoder import OracleDecoder
    from oracle.epoch import OracleEpochController
    from oracle.model import TINY as ORACLE_TINY, seeded_weights

    monkeypatch.setenv("VLLM_ASCEND_RESIDENT_EPOCH_BACKEND_FACTORY", "cruise_b200.cuda_backend:create_cuda_engine")
    monkeypatch.setenv("VLLM_ASCEND_RESIDENT_EPOCH_MODEL", "tiny")
    monkeypatch.setenv("VLLM_ASCEND_RESIDENT_EPOCH_EXTERNAL_WEIGHTS", "synthetic:0")
    scheduler = make_scheduler(tmp_path, 4, ResidentEpochConfig.from_env(), preset=TINY, max_model_len=32)
    worker = ResidentEpochWorker(vllm_config=scheduler.vllm_config, local_rank=0, rank=0,
                                 distributed_init_method="tcp://127.0.0.1:1", is_driver_worker=True)
    worker.load_model()
    worker.compile_or_warm_up_model()
    oracle = OracleEpochController(OracleDecoder(ORACLE_TINY, seeded_weights(ORACLE_TINY, 0)))

    # three requests now, a fourth joins after the first epoch; budgets differ
    eos = TINY.configured_eos
    reqs = [request(f"q{i}", [11 + 97 * i], max_tokens=m, eos=eos) for i, m in enumerate((13, 6, 9))]
    for r in reqs:
        scheduler.add_request(r)
    late = request("q3", [777], max_tokens=5, eos=eos)
    epochs = 0
    while scheduler.has_unfinished_requests() or late is not None:
        output = scheduler.schedule()
        plan = get_plan(output)
        assert plan is not None, scheduler.last_rejection
        runner = worker.execute_model(output)
        result = get_result(runner)
        assert result.route == "device" and result.status == 0
        got = {rid: list(runner.sampled_token_ids[runner.req_id_to_index[rid]]) for rid in plan.req_ids}
        assert got == _oracle_tokens(oracle, plan, TINY.configured_eos), f"epoch {epochs}"
        scheduler.update_from_output(output, runner)
        epochs += 1
        if late is not None:
            scheduler.add_request(late)
            reqs.append(late)
            late = None
        assert epochs < 20
    worker.shutdown()
    for r in reqs:
        assert r.status in (RequestStatus.FINISHED_LENGTH_CAPPED, RequestStatus.FINISHED_STOPPED)
        assert 1 <= r.num_output_tokens <= r.max_tokens
    assert epochs >= 3
