"""bench.py's teacher-forced baseline (all rows of a cohort forced together)
prefills exactly what the row-by-row helper does: same KV cache, same
resident state, checked on the CPU oracle (tiny model)."""

from __future__ import annotations

import numpy as np
import torch

import bench
from oracle.decoder import OracleDecoder
from oracle.epoch import OracleEpochController
from oracle.model import TINY as ORACLE_TINY, seeded_weights
from scenario import decode_inputs, make_scenario, prefill_epochs


def test_all_rows_forcing_matches_row_by_row_prefill():
    from cruise_b200.model_config import TINY

    weights = seeded_weights(ORACLE_TINY, seed=0)
    sc = make_scenario(vocab=TINY.vocab, seed=4, active_rows=(1, 1, 1, 1), prompt_len=(3, 14), k=2)
    serial = OracleEpochController(OracleDecoder(ORACLE_TINY, weights))
    for inputs in prefill_epochs(sc, TINY.block_size, TINY.vocab):
        serial.run(**inputs)
    batched = OracleEpochController(OracleDecoder(ORACLE_TINY, weights))
    epochs = list(bench.forced_epochs_all_rows(sc, TINY, generation_offset=0))
    for inputs in epochs:
        _, control = batched.run(**inputs)
        assert int(control[3]) == 0
    assert torch.equal(serial.key, batched.key) and torch.equal(serial.value, batched.value)
    # both leave every row ready for the same decode epoch
    h1, c1 = serial.run(**decode_inputs(sc, TINY.block_size))
    h2, c2 = batched.run(**decode_inputs(sc, TINY.block_size))
    np.testing.assert_array_equal(h1, h2)
    np.testing.assert_array_equal(c1, c2)


def test_roofline_numerator_matches_the_checkpoint_tensor_sizes():
    """The bench's algorithmic bytes per decode step: every 7B tensor but the
    embedding table streams once (14,141,238,272 B, counted independently from
    the checkpoint map), 57,344 B of K/V per context position per active row,
    and one 7,168-byte embedding row per active row."""
    from cruise_b200.model_config import QWEN25_7B
    from oracle.model import QWEN25_7B as ORACLE_7B, tensor_shapes

    streamed = sum(int(np.prod(shape)) * 2 for name, shape in tensor_shapes(ORACLE_7B).items()
                   if name != "model.embed_tokens.weight")
    assert bench.weight_bytes_per_step(QWEN25_7B) == streamed == 14_141_238_272
    contexts = [3, 4, 5, 6]
    kv_token = 2 * 28 * 4 * 128 * 2
    assert kv_token == 57_344
    assert bench.step_bytes(QWEN25_7B, contexts) == streamed + kv_token * (sum(contexts) + 4) + 4 * 7_168


def test_tensor_parallel_shards_cover_the_step_once():
    """Summed over the ranks, the shards stream every weight once, except the
    norms, which each rank keeps whole, and the KV heads replicated when there
    are more ranks than KV heads (TP = 8 over 4 heads)."""
    from cruise_b200.model_config import QWEN25_7B, TpShard

    cfg = QWEN25_7B
    contexts = [10, 20, 30, 40]
    single = bench.step_bytes(cfg, contexts)
    assert bench.shard_step_bytes(cfg, TpShard.of(cfg, 0, 1), contexts) == single
    norms = 2 * (2 * cfg.num_layers * cfg.hidden + cfg.hidden)
    embed_rows = len(contexts) * cfg.hidden * 2
    for world in (2, 4, 8):
        total = sum(bench.shard_step_bytes(cfg, TpShard.of(cfg, r, world), contexts) for r in range(world))
        extra_kv_heads = max(world, cfg.num_kv_heads) - cfg.num_kv_heads
        kv_extra = 2 * cfg.num_layers * extra_kv_heads * cfg.head_dim * 2 * (sum(contexts) + len(contexts))
        qkv_extra = 2 * cfg.num_layers * extra_kv_heads * cfg.head_dim * (cfg.hidden + 1) * 2
        pad = sum(TpShard.of(cfg, r, world).ni for r in range(world)) - cfg.intermediate
        mlp_pad = 2 * cfg.num_layers * 3 * pad * cfg.hidden
        assert total == single + (world - 1) * (norms + embed_rows) + kv_extra + qkv_extra + mlp_pad, world


def test_second_cohort_takes_over_the_rows_under_new_generations():
    """The configs[4] figure (box_scale) prefills a fresh cohort on rows an
    earlier cohort still holds: with its generations moved, every epoch of the
    new cohort passes the controller's continuity check and decodes (CPU
    oracle, tiny model); the summary counts tokens per device second."""
    from cruise_b200.model_config import TINY

    engine = bench.OracleEngine(TINY, threads=1)
    sc, first = bench.setup_cohort(engine, TINY, seed=11, k=2, prompt_max=5)
    cohort = bench.Cohort(engine, TINY, sc, first)
    cohort.step()
    sc2, first2 = bench.setup_cohort(engine, TINY, seed=12, k=8, prompt_max=12, generation_offset=100)
    assert first2.status == 0 and sc2.generations == [g + 100 for g in sc.generations]
    second = bench.Cohort(engine, TINY, sc2, first2)
    out, _ = second.step()
    assert out.status == 0 and out.model_calls > 0
    summary = bench.box_scale_summary({"dev_s": 0.5, "tokens": 100, "wall": 0.6, "bytes": 10 ** 12,
                                       "model_calls": 25}, device=None, world=1, tp=False, peak=4000.0)
    assert summary["value"] == 200.0 and summary["us_per_decode_step"] == 20000.0
    assert summary["roofline_frac"] == 0.5 and summary["e2e_value"] == round(100 / 0.6, 2)
