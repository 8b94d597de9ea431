"""GPU parity of the benchmarked workload at full depth: the Qwen2.5-7B
architecture with all 28 layers, exactly the model bench.py times.

The oracle runs the whole model on the host (15 GB of bf16 weights, built by
the C restatement of the seeded generator on every host core; a decode step
takes a fraction of a second there).  Each case prefills a seeded B=4 cohort
of 2-5-token prompts on the oracle, imports the prefilled blocks through the
one-shot host-to-device import, and runs the greedy epoch on both sides.
Checked (scenario.check_epoch): tokens, termination reasons and every control
word, the Adler-32 import proof, logits per row and the whole 28-layer KV
cache per head vector within 2e-2, blocks outside the block table
bit-identical; a row may diverge only at a near-tie of the oracle's logits
(one row per K=2 epoch, two per K=8 epoch at most), and the slots and words
that do not depend on that row stay compared.

At 28 layers the logits carry about 1e-2 of relative error per row (bf16
rounding flips from a different fp32 summation order, compounded over the
residual stream), and a large share of the oracle's row-steps have a top-2
margin under 2e-2 among 152,064 candidates: measured on B200, the K=8 epoch
below had two rows flip at such near-ties (steps 0 and 3).
"""

from __future__ import annotations

import pytest
import torch

from oracle.decoder import OracleDecoder
from oracle.epoch import EpochTrace, OracleEpochController
from oracle.model import QWEN25_7B as ORACLE_7B
from oracle.model import seeded_weights, tensor_shapes
from scenario import check_epoch, decode_inputs, import_payload, make_scenario, prefill_epochs

pytestmark = pytest.mark.gpu

TOKEN_HIGH = 151643


@pytest.fixture(scope="module")
def full_model(cuda_ok):
    return seeded_weights(ORACLE_7B, seed=0, use_c=True)


def _engine():
    from cruise_b200.engine import EpochEngine
    from cruise_b200.model_config import QWEN25_7B

    engine = EpochEngine(QWEN25_7B)
    engine.init_synthetic(0)
    return engine


def test_device_weights_equal_the_host_generator_at_full_depth(full_model):
    """Spot check of the seeded weights at 28 layers: the deepest layer's
    tensors, the final norm, lm_head (the engine stores them tiled and padded)."""
    engine = _engine()
    shapes = tensor_shapes(ORACLE_7B)
    for name in ("model.layers.27.self_attn.q_proj.weight", "model.layers.27.self_attn.v_proj.bias",
                 "model.layers.27.mlp.up_proj.weight", "model.layers.27.mlp.down_proj.weight",
                 "model.norm.weight", "lm_head.weight"):
        got = engine.get_weight(name, shapes[name])
        assert torch.equal(got.view(torch.int16), full_model[name].view(torch.int16)), name
    engine.close()


def _import_epoch(full_model, seed: int, k: int, label: str, max_diverged: int = 1):
    sc = make_scenario(vocab=ORACLE_7B.vocab, seed=seed, active_rows=(1, 1, 1, 1), prompt_len=(2, 5),
                       budget=(2, 8), token_high=TOKEN_HIGH, k=k, eos=151645)
    prefill = OracleEpochController(OracleDecoder(ORACLE_7B, full_model))
    for inputs in prefill_epochs(sc, ORACLE_7B.block_size, ORACLE_7B.vocab):
        prefill.run(**inputs)
    payload = import_payload(prefill.key, prefill.value, sc)
    del prefill
    engine = _engine()
    oracle = OracleEpochController(OracleDecoder(ORACLE_7B, full_model))
    inputs = decode_inputs(sc, ORACLE_7B.block_size, importing=True)
    trace = EpochTrace()
    out = engine.run(**inputs, import_payload=payload, want_logits=True)
    history, control = oracle.run(**inputs, import_payload=payload, trace=trace)
    assert out.status == int(control[3]) == 0
    assert int(out.control_out[5]) == int(control[5]) != 0   # Adler-32 of the imported blocks
    key, value = engine.read_kv()
    check = check_epoch(out, history, control, trace, inputs, kv=(key, value, oracle.key, oracle.value),
                        block_size=ORACLE_7B.block_size, label=label, max_diverged=max_diverged)
    print(f"{label}: logits rel err {check.logits_err:.3g}, KV rel err {check.kv_err:.3g}, "
          f"diverged {check.diverged} of {check.near_ties} near-tie row-steps")
    engine.close()
    return check


@pytest.mark.parametrize("seed", [0, 1])
def test_config2_full_depth_import_then_k2_epoch(full_model, seed):
    """configs[1] at 28 layers: the one-shot import, then one K=2 greedy epoch."""
    _import_epoch(full_model, seed, 2, f"7b-28l config2 seed {seed}")


def test_full_depth_k8_epoch(full_model):
    """Eight decode steps at 28 layers after the import (the box-scale K)."""
    _import_epoch(full_model, 5, 8, "7b-28l k8 seed 5", max_diverged=2)
