"""The reference-compatible C ABI (resident_epoch_create/_execute/_destroy) on
the GPU against the oracle's restatement of the bridge, through the Python
NativeEpochEngine and backend exactly as a vLLM worker would drive it."""

import os

import numpy as np
import pytest
import torch

from oracle.decoder import OracleDecoder
from oracle.epoch import OracleEpochController, bridge_execute
from oracle.model import TINY, seeded_weights

pytestmark = pytest.mark.gpu


def plan_for(rows, steps, position=0, token=7, eos=4095, generation_base=1, import_required=False):
    from cruise_b200.contract import CONTRACT_VERSION, ResidentEpochPlan, ResidentEpochRequest

    reqs = tuple(
        ResidentEpochRequest(req_id=f"r{row}", row=row, generation=generation_base + row, token_id=token + row,
                             position=position, sequence_length=position + 1, eos_token_id=eos,
                             scheduler_block_ids=(row,), device_block_ids=(2 * row, 2 * row + 1),
                             kv_import_required=import_required)
        for row in rows)
    mask = tuple(1 if r in rows else 0 for r in range(4))
    return ResidentEpochPlan(version=CONTRACT_VERSION, graph_batch_size=4, max_steps=steps, logical_capacity=32,
                             requests=reqs, active_mask=mask)


@pytest.fixture()
def engines(cuda_ok):
    from cruise_b200.cuda_backend import CudaEpochEngine

    engine = CudaEpochEngine(model="tiny", weights="synthetic:0")
    oracle = OracleEpochController(OracleDecoder(TINY, seeded_weights(TINY, 0)))
    yield engine, oracle
    engine.close()


def oracle_tokens(oracle, plan):
    toks, pos, lens, eos, gens = [0] * 4, [0] * 4, [0] * 4, [4095] * 4, list(plan.row_generations)
    for r in plan.requests:
        toks[r.row], pos[r.row], lens[r.row], eos[r.row] = r.token_id, r.position, r.sequence_length, r.eos_token_id
    res = bridge_execute(oracle, len(plan.requests), plan.max_steps, toks, pos, lens, eos, gens, configured_eos=4095)
    return res, {r.req_id: [int(t) for t in res.tokens[r.row * 8: r.row * 8 + res.executed[r.row]]] for r in plan.requests}


def test_warmup_is_one_complete_step(engines):
    engine, _ = engines
    out = engine.warm_up()
    assert (out.status, out.model_calls, out.feed_calls, out.fetch_calls) == (0, 1, 1, 1)


def test_two_epochs_match_the_oracle_bridge(engines):
    engine, oracle = engines
    first = plan_for([0, 1, 2], steps=2)
    out = engine.execute(first)
    ref, tokens = oracle_tokens(oracle, first)
    assert out.status == ref.device_status == 0 and out.model_calls == ref.model_calls
    assert out.token_ids == tokens and out.row_generations == tuple(ref.row_generations)
    assert out.commit_state == 2 and out.feed_calls == out.fetch_calls == 1
    # continue the same generations from where they stopped
    from cruise_b200.contract import CONTRACT_VERSION, ResidentEpochPlan, ResidentEpochRequest
    reqs = tuple(ResidentEpochRequest(req_id=r.req_id, row=r.row, generation=r.generation,
                                      token_id=tokens[r.req_id][-1], position=2, sequence_length=3,
                                      eos_token_id=4095, scheduler_block_ids=(r.row,),
                                      device_block_ids=(2 * r.row, 2 * r.row + 1)) for r in first.requests)
    second = ResidentEpochPlan(version=CONTRACT_VERSION, graph_batch_size=4, max_steps=4, logical_capacity=32,
                               requests=reqs, active_mask=first.active_mask)
    out2 = engine.execute(second)
    ref2, tokens2 = oracle_tokens(oracle, second)
    assert out2.status == 0 and out2.token_ids == tokens2


def test_bridge_transport_statuses(engines):
    engine, _ = engines
    from cruise_b200.contract import ResidentEpochExecutionError

    bad_row = plan_for([0], steps=2, position=31)  # position + K beyond capacity is rejected on the host (11)
    object.__setattr__(bad_row, "logical_capacity", 64)
    with pytest.raises(ResidentEpochExecutionError) as caught:
        engine.execute(bad_row)
    assert caught.value.status == 11 and caught.value.input_preserving


def test_host_snapshot_import_through_backend(engines):
    engine, _ = engines
    from cruise_b200.backend import ResidentEpochBackend
    from cruise_b200.contract import get_result
    from cruise_b200.kv_transfer import KVGeometry, ResidentKVSnapshot, kv_payload_checksum

    g = KVGeometry.of(engine.config)
    plan = plan_for([1, 2], steps=2, position=3, import_required=True)
    rng = np.random.default_rng(0)
    payload = (rng.standard_normal(g.payload_bytes // 2).astype(np.float32) * 0.5)
    raw = torch.from_numpy(payload).to(torch.bfloat16).view(torch.int16).numpy()
    raw = raw.reshape(2, g.layers, 4, -1)
    raw[:, :, [0, 3]] = 0
    raw = raw.tobytes()
    mask = 0b0110
    snapshot = ResidentKVSnapshot(11, mask, (0, 2, 3, 0), raw, kv_payload_checksum(raw, mask, g), g)
    out = ResidentEpochBackend(engine).execute(plan, snapshot=snapshot)
    result = get_result(out)
    assert result.kv_imported and result.kv_import_checksum == snapshot.checksum
    assert result.kv_transfer_mode == "host_snapshot" and result.model_calls == 2
