"""The 9-in / 4-out decoder ABI on the device (cruise_decoder_step) and the
host-loop route over it.

* One decoder call against the oracle's decoder step (the reference's
  PagedQwenDecoderStep.forward, batched_decoder_step.py:277-417) on the same
  caches and inputs, with an inactive row: next positions exact, logits of the
  active rows and the KV caches within 2e-2 per row / head vector, blocks
  outside the block table and the inactive row untouched.
* Caller-held caches (device buffers passed in the ABI's K and V slots) give
  the same bits as the engine's resident caches, which stay untouched.
* K host-driven decoder calls (the reference's host runner) equal one
  resident K-step epoch bit for bit: tokens, accounting, KV.
"""

from __future__ import annotations

from dataclasses import replace

import numpy as np
import pytest
import torch

from cruise_b200.host_loop import host_loop_epoch
from oracle.decoder import OracleDecoder
from oracle.epoch import OracleEpochController
from oracle.model import TINY as ORACLE_TINY
from oracle.model import OracleConfig, seeded_weights, tensor_shapes
from scenario import assert_kv, decode_inputs, make_scenario, prefill_epochs, rel_err_rows
from test_oracle_epoch import CASE_MATRIX, case_matrix_inputs

pytestmark = pytest.mark.gpu

TOL = 2e-2


def _geometry(name):
    from cruise_b200.model_config import QWEN25_7B, TINY

    if name == "tiny":
        return TINY, ORACLE_TINY
    cfg = replace(QWEN25_7B, name="qwen2.5-7b-2l", num_layers=2)
    ocfg = OracleConfig(num_layers=2, hidden=cfg.hidden, num_heads=cfg.num_heads, num_kv_heads=cfg.num_kv_heads,
                        head_dim=cfg.head_dim, intermediate=cfg.intermediate, vocab=cfg.vocab,
                        block_size=cfg.block_size, blocks_per_row=cfg.blocks_per_row, num_blocks=cfg.num_blocks)
    return cfg, ocfg


def _engine(cfg):
    from cruise_b200.engine import EpochEngine

    engine = EpochEngine(cfg)
    engine.init_synthetic(0)
    return engine


def _weights(engine, ocfg):
    return {name: engine.get_weight(name, shape) for name, shape in tensor_shapes(ocfg).items()}


@pytest.mark.parametrize("geometry", ["tiny", "7b-2l"])
def test_decoder_step_matches_the_oracle_step(cuda_ok, geometry):
    cfg, ocfg = _geometry(geometry)
    engine = _engine(cfg)
    weights = _weights(engine, ocfg)
    oracle = OracleEpochController(OracleDecoder(ocfg, weights))
    sc = make_scenario(vocab=cfg.vocab, seed=8, active_rows=(1, 1, 1, 0), token_high=min(cfg.vocab, 151643))
    for inputs in prefill_epochs(sc, cfg.block_size, cfg.vocab):
        assert engine.run(**inputs).status == 0
        oracle.run(**inputs)
    inputs = decode_inputs(sc, cfg.block_size)
    inputs["token"][3] = 5   # the inactive row still needs an existing token
    logits, nxt = engine.decoder_step(inputs["token"], inputs["position"], inputs["seq_len"], inputs["slot"],
                                      inputs["active"], inputs["block_table"])
    bt = torch.from_numpy(np.asarray(inputs["block_table"], dtype=np.int32).reshape(4, -1).copy())
    want_logits, key, value, want_next = oracle.decoder.step(
        torch.from_numpy(inputs["token"]), torch.from_numpy(inputs["position"]),
        torch.from_numpy(inputs["seq_len"]), bt, torch.from_numpy(inputs["slot"]), oracle.key, oracle.value,
        torch.from_numpy(inputs["active"]))
    np.testing.assert_array_equal(nxt, want_next.numpy())
    rows = [r for r in range(4) if inputs["active"][r]]
    err = rel_err_rows(torch.from_numpy(logits[rows]), want_logits[rows])
    assert float(err.max()) <= TOL, f"logits rel err {float(err.max()):.3g}"
    gk, gv = engine.read_kv()
    assert_kv(gk, gv, key, value, inputs, cfg.block_size, tol=TOL)
    engine.close()


def test_caller_held_caches_equal_the_resident_ones(cuda_ok):
    cfg, _ = _geometry("tiny")
    resident, holder = _engine(cfg), _engine(cfg)
    sc = make_scenario(vocab=cfg.vocab, seed=9)
    for inputs in prefill_epochs(sc, cfg.block_size, cfg.vocab):
        for engine in (resident, holder):
            assert engine.run(**inputs).status == 0
    key0, value0 = holder.read_kv()
    key = key0.cuda(holder.device)
    value = value0.cuda(holder.device)
    inputs = decode_inputs(sc, cfg.block_size)
    args = (inputs["token"], inputs["position"], inputs["seq_len"], inputs["slot"], inputs["active"],
            inputs["block_table"])
    want_logits, want_next = resident.decoder_step(*args)
    logits, nxt = holder.decoder_step(*args, key=key, value=value)
    np.testing.assert_array_equal(nxt, want_next)
    rows = [r for r in range(4) if inputs["active"][r]]
    np.testing.assert_array_equal(logits[rows], want_logits[rows])
    rk, rv = resident.read_kv()
    assert torch.equal(key.cpu().view(torch.int16), rk.view(torch.int16))
    assert torch.equal(value.cpu().view(torch.int16), rv.view(torch.int16))
    hk, hv = holder.read_kv()   # the holder's own resident caches were not used
    assert torch.equal(hk.view(torch.int16), key0.view(torch.int16))
    assert torch.equal(hv.view(torch.int16), value0.view(torch.int16))
    resident.close()
    holder.close()


def _loop_vs_epoch(cfg, sc, inputs):
    epoch, loop = _engine(cfg), _engine(cfg)
    for prefill in prefill_epochs(sc, cfg.block_size, cfg.vocab):
        for engine in (epoch, loop):
            assert engine.run(**prefill).status == 0
    out = epoch.run(**inputs)
    assert out.status == 0
    history, control = host_loop_epoch(lambda *a: loop.decoder_step(*a), inputs, cfg.block_size, cfg.capacity)
    np.testing.assert_array_equal(history, out.history)
    same = [0, 3, 4, *range(6, 24)]
    np.testing.assert_array_equal(control[same], out.control_out[same])
    for a, b in zip(loop.read_kv(), epoch.read_kv()):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    epoch.close()
    loop.close()


@pytest.mark.parametrize("name, k, pattern", CASE_MATRIX, ids=[c[0] for c in CASE_MATRIX])
def test_host_loop_equals_the_device_epoch(cuda_ok, name, k, pattern):
    cfg, _ = _geometry("tiny")
    sc, inputs = case_matrix_inputs(seeded_weights(ORACLE_TINY, 0), name, k, pattern)
    _loop_vs_epoch(cfg, sc, inputs)


def test_host_loop_equals_the_device_epoch_7b_geometry(cuda_ok):
    cfg, _ = _geometry("7b-2l")
    sc = make_scenario(vocab=cfg.vocab, seed=12, active_rows=(1, 1, 1, 1), k=4, token_high=151643)
    _loop_vs_epoch(cfg, sc, decode_inputs(sc, cfg.block_size))


def test_decoder_step_rejects_what_it_cannot_index(cuda_ok):
    from cruise_b200.engine import EngineError

    cfg, _ = _geometry("tiny")
    engine = _engine(cfg)
    sc = make_scenario(vocab=cfg.vocab, seed=1)
    inputs = decode_inputs(sc, cfg.block_size)
    args = dict(token=inputs["token"].copy(), position=inputs["position"], seq_len=inputs["seq_len"],
                slot=inputs["slot"].copy(), active=inputs["active"], block_table=inputs["block_table"])
    bad = dict(args, token=np.array([cfg.vocab, 0, 0, 0]))
    with pytest.raises(EngineError, match="vocabulary"):
        engine.decoder_step(**bad)
    slot = args["slot"].copy()
    slot[0] += 1
    with pytest.raises(EngineError, match="block-table slot"):
        engine.decoder_step(**dict(args, slot=slot))
    logits, nxt = engine.decoder_step(**args)   # the engine still works
    assert logits.shape == (4, cfg.vocab)
    engine.close()
