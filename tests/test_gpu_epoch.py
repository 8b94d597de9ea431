"""GPU parity of the resident epoch against the CPU oracle (tiny geometry).

Every test drives the CUDA engine through its C ABI (``cruise_epoch_run``) and
the oracle controller through the same 8-in / 2-out inputs, then checks:
integer outputs (token history, 28-word control output, statuses, reasons,
executed counts, generations, import checksum) bit-exactly; logits and KV
within bf16 tolerance (max relative error 2e-2); untouched KV blocks exactly.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.decoder import OracleDecoder
from oracle.epoch import EpochTrace, OracleEpochController
from oracle.model import TINY as ORACLE_TINY
from oracle.model import seeded_weights, tensor_shapes
from scenario import check_epoch, decode_inputs, import_payload, make_scenario, prefill_epochs

pytestmark = pytest.mark.gpu

TOL = 2e-2


@pytest.fixture(scope="module")
def tiny_weights():
    return seeded_weights(ORACLE_TINY, seed=0)


def new_engine(weights=None, synthetic_seed=None):
    from cruise_b200.engine import EpochEngine

    engine = EpochEngine("tiny")
    if weights is not None:
        engine.load_weights(weights)
    else:
        engine.init_synthetic(synthetic_seed)
    return engine


def rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.float()
    b = b.float()
    scale = float(b.abs().max())
    return float((a - b).abs().max()) / max(scale, 1e-30)


def assert_kv_close(engine, oracle, rows_blocks, tol=TOL):
    key, value = engine.read_kv()
    for name, g, o in (("key", key, oracle.key), ("value", value, oracle.value)):
        owned = sorted(rows_blocks)
        for block in range(g.shape[1]):
            if block in owned:
                err = rel_err(g[:, block], o[:, block])
                assert err <= tol, f"{name} block {block}: rel err {err:.3g}"
            else:
                assert torch.equal(g[:, block].view(torch.int16), o[:, block].to(torch.bfloat16).view(torch.int16)), (
                    f"{name} block {block} not owned by an active row changed"
                )


def test_synthetic_weights_match_cpu_generator(cuda_ok, tiny_weights):
    engine = new_engine(synthetic_seed=0)
    for name, shape in tensor_shapes(ORACLE_TINY).items():
        got = engine.get_weight(name, shape)
        assert torch.equal(got.view(torch.int16), tiny_weights[name].view(torch.int16)), name
    engine.close()


def _prefill_both(engine, oracle, sc):
    for inputs in prefill_epochs(sc, ORACLE_TINY.block_size, ORACLE_TINY.vocab):
        out = engine.run(**inputs)
        history, control = oracle.run(**inputs)
        assert out.status == 0 and int(control[3]) == 0
        np.testing.assert_array_equal(out.history, history)
        np.testing.assert_array_equal(out.control_out, control)


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_prefill_then_decode_epoch(cuda_ok, tiny_weights, seed):
    sc = make_scenario(vocab=ORACLE_TINY.vocab, seed=seed)
    engine = new_engine(tiny_weights)
    oracle = OracleEpochController(OracleDecoder(ORACLE_TINY, tiny_weights))
    _prefill_both(engine, oracle, sc)
    owned = {int(b) for r in range(4) if sc.prompts[r] for b in sc.block_table[r]}
    assert_kv_close(engine, oracle, owned)

    inputs = decode_inputs(sc, ORACLE_TINY.block_size)
    trace = EpochTrace()
    out = engine.run(**inputs, want_logits=True)
    history, control = oracle.run(**inputs, trace=trace)
    assert out.status == int(control[3]) == 0
    key, value = engine.read_kv()
    check_epoch(out, history, control, trace, inputs, kv=(key, value, oracle.key, oracle.value),
                block_size=ORACLE_TINY.block_size, label=f"tiny decode seed {seed}")
    engine.close()


def test_configuration1_against_the_fp32_oracle(cuda_ok, tiny_weights):
    """configs[0] names torch fp32 for the tiny model.  The engine computes in
    bf16 (fp32 accumulation); against the fp32 oracle on the same seeded
    weights it stays within the parity rule: tokens, statuses and control
    words equal (near-ties excepted), logits and KV within 2e-2 per vector."""
    sc = make_scenario(vocab=ORACLE_TINY.vocab, seed=0)
    engine = new_engine(tiny_weights)
    oracle = OracleEpochController(OracleDecoder(ORACLE_TINY, tiny_weights, torch.float32))
    for inputs in prefill_epochs(sc, ORACLE_TINY.block_size, ORACLE_TINY.vocab):
        out = engine.run(**inputs)
        history, control = oracle.run(**inputs)
        assert out.status == int(control[3]) == 0
        np.testing.assert_array_equal(out.history, history)
    inputs = decode_inputs(sc, ORACLE_TINY.block_size)
    trace = EpochTrace()
    out = engine.run(**inputs, want_logits=True)
    history, control = oracle.run(**inputs, trace=trace)
    assert out.status == int(control[3]) == 0
    key, value = engine.read_kv()
    check_epoch(out, history, control, trace, inputs, kv=(key, value, oracle.key, oracle.value),
                block_size=ORACLE_TINY.block_size, label="tiny decode vs fp32 oracle")
    engine.close()


def test_import_then_decode_epoch(cuda_ok, tiny_weights):
    sc = make_scenario(vocab=ORACLE_TINY.vocab, seed=0)
    # prefill on the oracle only: it stands for the stock prefill whose KV is imported
    prefill = OracleEpochController(OracleDecoder(ORACLE_TINY, tiny_weights))
    for inputs in prefill_epochs(sc, ORACLE_TINY.block_size, ORACLE_TINY.vocab):
        prefill.run(**inputs)
    payload = import_payload(prefill.key, prefill.value, sc)

    engine = new_engine(tiny_weights)
    oracle = OracleEpochController(OracleDecoder(ORACLE_TINY, tiny_weights))
    inputs = decode_inputs(sc, ORACLE_TINY.block_size, importing=True)
    trace = EpochTrace()
    out = engine.run(**inputs, import_payload=payload)
    history, control = oracle.run(**inputs, import_payload=payload, trace=trace)
    assert out.status == int(control[3]) == 0
    assert int(out.control_out[5]) == int(control[5]) != 0   # Adler-32 of the imported blocks
    key, value = engine.read_kv()
    check_epoch(out, history, control, trace, inputs, kv=(key, value, oracle.key, oracle.value),
                block_size=ORACLE_TINY.block_size, label="tiny import")
    engine.close()


@pytest.mark.parametrize(
    "mutate, status",
    [
        (lambda i: i["control"].__setitem__(0, 9), 201),       # K = 9
        (lambda i: i["control"].__setitem__(5, 1), 205),       # sampling mode 1
        (lambda i: i["control"].__setitem__(6, 1), 206),       # graph variant 1
        (lambda i: i["block_table"].__setitem__(1, i["block_table"][0]), 203),  # duplicate block
        (lambda i: i["slot"].__setitem__(0, i["slot"][0] + 1), 204),            # slot mismatch
        (lambda i: i["position"].__setitem__(0, 31) or i["seq_len"].__setitem__(0, 32), 202),  # pos+K > C
    ],
)
def test_recovery_statuses_preserve_inputs(cuda_ok, tiny_weights, mutate, status):
    """Pre-execution fallbacks (reference recovery cases 201/202/205/206 and
    203/204) return with zero model calls, fallback reasons, and no KV change."""
    sc = make_scenario(vocab=ORACLE_TINY.vocab, seed=3)
    engine = new_engine(tiny_weights)
    oracle = OracleEpochController(OracleDecoder(ORACLE_TINY, tiny_weights))
    _prefill_both(engine, oracle, sc)
    key0, value0 = engine.read_kv()
    inputs = decode_inputs(sc, ORACLE_TINY.block_size)
    mutate(inputs)
    out = engine.run(**inputs)
    history, control = oracle.run(**inputs)
    assert int(control[3]) == status
    np.testing.assert_array_equal(out.control_out, control)
    np.testing.assert_array_equal(out.history, history)
    assert out.model_calls == 0
    key1, value1 = engine.read_kv()
    assert torch.equal(key0.view(torch.int16), key1.view(torch.int16))
    assert torch.equal(value0.view(torch.int16), value1.view(torch.int16))
    engine.close()


def test_non_finite_logits_mid_epoch_fall_back(cuda_ok, tiny_weights):
    """Status 209 on the device (controller :555-556): with a NaN embedding row
    for the token row 0 emits at the first step, the second step's logits of
    row 0 are non-finite.  The device must stop the epoch exactly where the
    oracle does: same history (first step kept), model calls 2, executed
    counts, FALLBACK reasons and status -- the whole control output."""
    from test_oracle_epoch import _poisoned_scenario

    _, bad, _ = _poisoned_scenario(tiny_weights)
    engine = new_engine(weights=bad)
    oracle = OracleEpochController(OracleDecoder(ORACLE_TINY, bad))
    sc = make_scenario(vocab=ORACLE_TINY.vocab, seed=6, active_rows=(1, 1, 1, 0), budget=(8, 8))
    for inputs in prefill_epochs(sc, ORACLE_TINY.block_size, ORACLE_TINY.vocab):
        assert engine.run(**inputs).status == 0
        oracle.run(**inputs)
    inputs = decode_inputs(sc, ORACLE_TINY.block_size)
    inputs["control"][0] = 4
    want_history, want_out = oracle.run(**inputs)
    got = engine.run(**inputs)
    engine.close()
    assert want_out[3] == 209
    np.testing.assert_array_equal(got.history, want_history)
    np.testing.assert_array_equal(got.control_out, want_out)


def test_replay_after_a_mid_epoch_fallback(cuda_ok, tiny_weights):
    """After the device's 209 the resident state has not moved: with the fault
    removed (the embedding row restored), the same inputs are accepted and the
    device emits what the oracle emits on the same replay."""
    from test_oracle_epoch import _poisoned_scenario

    _, bad, _ = _poisoned_scenario(tiny_weights)
    engine = new_engine(weights=bad)
    oracle = OracleEpochController(OracleDecoder(ORACLE_TINY, bad))
    sc = make_scenario(vocab=ORACLE_TINY.vocab, seed=6, active_rows=(1, 1, 1, 0), budget=(8, 8))
    for inputs in prefill_epochs(sc, ORACLE_TINY.block_size, ORACLE_TINY.vocab):
        assert engine.run(**inputs).status == 0
        oracle.run(**inputs)
    inputs = decode_inputs(sc, ORACLE_TINY.block_size)
    inputs["control"][0] = 4
    assert engine.run(**inputs).status == 209
    oracle.run(**inputs)
    engine.set_weight("model.embed_tokens.weight", tiny_weights["model.embed_tokens.weight"])
    oracle.decoder = OracleDecoder(ORACLE_TINY, tiny_weights)
    want_history, want_out = oracle.run(**inputs)
    got = engine.run(**inputs)
    engine.close()
    assert want_out[3] == 0
    np.testing.assert_array_equal(got.history, want_history)
    np.testing.assert_array_equal(got.control_out, want_out)


def _case_matrix():
    from test_oracle_epoch import CASE_MATRIX

    return CASE_MATRIX


@pytest.mark.parametrize("name, k, pattern", _case_matrix(), ids=[c[0] for c in _case_matrix()])
def test_epoch_case_matrix_on_device(cuda_ok, tiny_weights, name, k, pattern):
    """The reference's epoch case matrix (K 1/2/4/8; active, empty and finished
    rows; independent early EOS) on the device: token history and the whole
    control output equal the oracle's."""
    from test_oracle_epoch import case_matrix_inputs

    sc, inputs = case_matrix_inputs(tiny_weights, name, k, pattern)
    engine = new_engine(synthetic_seed=0)
    oracle = OracleEpochController(OracleDecoder(ORACLE_TINY, tiny_weights))
    for prefill in prefill_epochs(sc, ORACLE_TINY.block_size, ORACLE_TINY.vocab):
        assert engine.run(**prefill).status == 0
        oracle.run(**prefill)
    want_history, want_out = oracle.run(**inputs)
    got = engine.run(**inputs)
    engine.close()
    assert want_out[3] == 0
    np.testing.assert_array_equal(got.history, want_history)
    np.testing.assert_array_equal(got.control_out, want_out)
