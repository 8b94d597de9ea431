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


def _oracle_prefill_decode(oracle, prompts, generations, steps, eos=4095):
    """The oracle's token-by-token prefill of ``prompts`` (rows own blocks
    2r, 2r+1 as in the bridge) and the K-step epoch after it: (history, trace)."""
    from oracle.epoch import EpochTrace
    from scenario import Scenario, decode_inputs, prefill_epochs

    sc = Scenario(block_table=np.arange(8, dtype=np.int32).reshape(4, 2), prompts=prompts, budgets=[8] * 4,
                  generations=generations, eos=[eos] * 4, k=steps)
    for inputs in prefill_epochs(sc, TINY.block_size, TINY.vocab):
        oracle.run(**inputs)
    trace = EpochTrace()
    history, control = oracle.run(**decode_inputs(sc, TINY.block_size), trace=trace)
    return history, control, trace


def test_device_prefill_through_the_bridge(engines):
    """resident_epoch_prefill + the import epoch (no reference counterpart):
    two rows prefilled on the device, a third starting from a one-token
    prompt, one row empty; tokens equal the oracle's token-by-token prefill and
    decode (near-ties excepted), the import proof is nonzero, and a following
    epoch continues the device-owned rows."""
    engine, oracle = engines
    from cruise_b200.backend import ResidentEpochBackend
    from cruise_b200.contract import CONTRACT_VERSION, ResidentEpochPlan, ResidentEpochRequest, get_result
    from scenario import find_divergence

    prompts = [[11, 12, 13, 14, 15], [301], [], [7, 8, 9, 10, 11, 12, 13, 14, 15]]
    generations = [5, 6, 0, 7]
    reqs = tuple(
        ResidentEpochRequest(req_id=f"r{row}", row=row, generation=generations[row], token_id=p[-1],
                             position=len(p) - 1, sequence_length=len(p), eos_token_id=4095,
                             scheduler_block_ids=(row,), device_block_ids=(2 * row, 2 * row + 1),
                             kv_import_required=len(p) > 1, prompt_token_ids=tuple(p) if len(p) > 1 else ())
        for row, p in enumerate(prompts) if p)
    plan = ResidentEpochPlan(version=CONTRACT_VERSION, graph_batch_size=4, max_steps=4, logical_capacity=32,
                             requests=reqs, active_mask=(1, 1, 0, 1))
    out = ResidentEpochBackend(engine).execute(plan)
    result = get_result(out)
    assert result.kv_imported and result.kv_transfer_mode == "device_prefill" and result.kv_import_checksum != 0
    history, control, trace = _oracle_prefill_decode(oracle, prompts, generations, 4)
    got = np.full((8, 4), -1, dtype=np.int64)
    for q in plan.requests:
        tokens = out.sampled_token_ids[out.req_id_to_index[q.req_id]]
        got[:len(tokens), q.row] = tokens
    diverged = find_divergence(got, history, trace.margins)
    assert len(diverged) <= 1, diverged

    # the rows are device-owned now: the next epoch continues the rows that ran
    # all four steps without an import
    going = [q for q in plan.requests if got[3, q.row] >= 0 and 4095 not in got[:4, q.row]]
    if going:
        follow = ResidentEpochPlan(
            version=CONTRACT_VERSION, graph_batch_size=4, max_steps=2, logical_capacity=32,
            requests=tuple(ResidentEpochRequest(
                req_id=q.req_id, row=q.row, generation=q.generation, token_id=int(got[3, q.row]),
                position=q.position + 4, sequence_length=q.position + 5, eos_token_id=4095,
                scheduler_block_ids=q.scheduler_block_ids, device_block_ids=q.device_block_ids, state_owner="device")
                for q in going),
            active_mask=tuple(1 if r in {q.row for q in going} else 0 for r in range(4)))
        assert not get_result(ResidentEpochBackend(engine).execute(follow)).kv_imported


def test_prefill_import_needs_a_pending_prefill(engines):
    engine, _ = engines
    out = engine._call(request_count=1, max_steps=1, tokens=[5, 0, 0, 0], positions=[2, 0, 0, 0],
                       lengths=[3, 0, 0, 0], eos=[4095] * 4, generations=[9, 0, 0, 0], transfer_id=3)
    assert out["ret"] == 13
    tokens = (np.arange(4 * TINY.block_size, dtype=np.int64) % 100).copy()
    lens = np.array([3, 0, 4, 0], dtype=np.int32)
    lib = engine.library
    import ctypes
    assert lib.resident_epoch_prefill(engine.handle, tokens.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)),
                                      lens.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), TINY.block_size) == 0
    # row 2 was prefilled but does not run in this epoch
    out = engine._call(request_count=1, max_steps=1, tokens=[2, 0, 0, 0], positions=[2, 0, 0, 0],
                       lengths=[3, 0, 0, 0], eos=[4095] * 4, generations=[9, 0, 0, 0], transfer_id=4)
    assert out["ret"] == 13
    # both rows run, but row 2 does not start from its last prompt token (position 3)
    out = engine._call(request_count=2, max_steps=1, tokens=[2, 0, 5, 0], positions=[2, 0, 1, 0],
                       lengths=[3, 0, 2, 0], eos=[4095] * 4, generations=[9, 0, 10, 0], transfer_id=5)
    assert out["ret"] == 11
    too_long = np.array([TINY.block_size + 1, 0, 0, 0], dtype=np.int32)
    assert lib.resident_epoch_prefill(engine.handle, tokens.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)),
                                      too_long.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                      TINY.block_size) == 10
