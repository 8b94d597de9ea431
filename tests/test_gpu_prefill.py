"""Batched device prefill (cruise_epoch_prefill) against the oracle's
token-by-token prefill.

The oracle prefills each prompt with the single-token decoder step (forced
epochs), exports the rows' first blocks as the import payload and runs the
import epoch.  The engine runs all prompt tokens through the model at once on
the GPU, keeps the payload on the device and runs the same import epoch from
it.  Tokens and control words must match (up to permitted near-ties; the import
checksum word covers a payload that differs in fp32 summation order, so it is
checked against the engine's own imported blocks instead), logits and the KV
cache within 2e-2."""

from __future__ import annotations

from dataclasses import replace

import numpy as np
import pytest
import torch

from oracle.decoder import OracleDecoder
from oracle.epoch import EpochTrace, OracleEpochController
from oracle.model import TINY as ORACLE_TINY, OracleConfig, seeded_weights, tensor_shapes
from scenario import BATCH, check_epoch, decode_inputs, import_payload, make_scenario, prefill_epochs

pytestmark = pytest.mark.gpu



def _compare(cfg, ocfg, weights, sc):
    from cruise_b200.engine import EpochEngine
    from cruise_b200.kv_transfer import KVGeometry, kv_payload_checksum

    prefill = OracleEpochController(OracleDecoder(ocfg, weights))
    for inputs in prefill_epochs(sc, cfg.block_size, cfg.vocab):
        prefill.run(**inputs)
    payload = import_payload(prefill.key, prefill.value, sc)
    inputs = decode_inputs(sc, cfg.block_size, importing=True)
    oracle = OracleEpochController(OracleDecoder(ocfg, weights))
    trace = EpochTrace()
    history, control = oracle.run(**inputs, import_payload=payload, trace=trace)

    engine = EpochEngine(cfg)
    engine.init_synthetic(0)
    with pytest.raises(Exception, match="no prefilled cohort"):
        engine.run(**inputs)   # an import without a payload needs a prefill first
    engine.prefill(sc.prompts)
    out = engine.run(**inputs, want_logits=True)
    assert out.status == int(control[3]) == 0
    key, value = engine.read_kv()
    # control word 5 is the import checksum: the device prefill's K/V are
    # tolerance-equal to the oracle's, not bit-equal, so it is checked below
    check = check_epoch(out, history, control, trace, inputs, kv=(key, value, oracle.key, oracle.value),
                        block_size=cfg.block_size, skip_words=(5,), label=f"prefill {cfg.name}")
    diverged = set(check.diverged)
    # the device's import proof is the Adler-32 of exactly the blocks it imported
    # (the first block of each row, read back before any decoded position)
    mask = sum(1 << r for r in range(BATCH) if sc.prompts[r])
    g = KVGeometry.of(cfg)
    blocks = import_payload(key, value, sc)
    for r in range(BATCH):
        if sc.prompts[r]:
            blocks[:, :, r, len(sc.prompts[r]) - 1:] = 0   # positions the decode epoch wrote
    raw = blocks.contiguous().view(torch.int16).numpy().tobytes()
    assert (int(out.control_out[5]) & 0xFFFFFFFF) == kv_payload_checksum(raw, mask, g)
    engine.close()
    return diverged


@pytest.mark.parametrize("seed, rows", [(0, (1, 1, 1, 1)), (1, (1, 0, 1, 1)), (2, (0, 1, 0, 0))])
def test_tiny_prefill(cuda_ok, seed, rows):
    from cruise_b200.model_config import TINY

    weights = seeded_weights(ORACLE_TINY, seed=0)
    sc = make_scenario(vocab=TINY.vocab, seed=seed, active_rows=rows, prompt_len=(2, TINY.block_size), k=8,
                       budget=(8, 8))
    _compare(TINY, ORACLE_TINY, weights, sc)


@pytest.fixture(scope="module")
def qwen7b_2l():
    from cruise_b200.engine import EpochEngine
    from cruise_b200.model_config import QWEN25_7B

    cfg = replace(QWEN25_7B, name="qwen2.5-7b-2l", num_layers=2)
    ocfg = OracleConfig(num_layers=2, hidden=cfg.hidden, num_heads=cfg.num_heads, num_kv_heads=cfg.num_kv_heads,
                        head_dim=cfg.head_dim, intermediate=cfg.intermediate, vocab=cfg.vocab,
                        block_size=cfg.block_size, blocks_per_row=cfg.blocks_per_row, num_blocks=cfg.num_blocks)
    engine = EpochEngine(cfg)
    engine.init_synthetic(0)
    weights = {name: engine.get_weight(name, shape) for name, shape in tensor_shapes(ocfg).items()}
    engine.close()
    return cfg, ocfg, weights


# The cohort's prompt tokens (all rows, the last token of each excluded) set
# how the tensor-core GEMMs tile the tokens: up to 128 tokens one 128-token
# tile, up to 256 one 256-token tile, beyond that two 256-token sub-tiles
# (the last partly filled), 508 at most (4 rows x 127).
@pytest.mark.parametrize("seed, rows, prompt_len", [
    (3, (1, 1, 1, 0), (60, 120)),    # 177..357 tokens
    (4, (1, 1, 1, 1), (2, 33)),      # at most 128 tokens
    (5, (1, 0, 1, 1), (45, 86)),     # 132..255 tokens
    (6, (1, 1, 1, 1), (128, 128)),   # 508 tokens: every row's whole first block
])
def test_qwen7b_geometry_prefill(cuda_ok, qwen7b_2l, seed, rows, prompt_len):
    cfg, ocfg, weights = qwen7b_2l
    sc = make_scenario(vocab=cfg.vocab, seed=seed, active_rows=rows, prompt_len=prompt_len, k=4,
                       budget=(4, 4), token_high=151643)
    tokens = sum(len(p) - 1 for p in sc.prompts if p)
    assert prompt_len[0] * sum(rows) - sum(rows) <= tokens <= (prompt_len[1] - 1) * sum(rows)
    _compare(cfg, ocfg, weights, sc)
