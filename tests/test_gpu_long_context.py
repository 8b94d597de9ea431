"""GPU parity of paged decode attention at long context (head_dim 128, GQA).

The tiny geometry never leaves the first 32 positions.  These cases use a
512-position cache (4 blocks of 128 per row) with head_dim 128, so attention
runs more than one 256-position scores chunk and reads most V rows past the
ones staged in shared memory.  Each case imports rows at seeded positions up
to 498 (one K=1 epoch), overwrites the whole paged cache with the same seeded
values on both sides, then runs a K=8 greedy epoch that reads every cached
position of every row.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.decoder import OracleDecoder
from oracle.epoch import EpochTrace, OracleEpochController
from oracle.model import OracleConfig, seeded_weights
from scenario import check_epoch, compute_slot

pytestmark = pytest.mark.gpu

IMPORT_FLAG = 0x100


def _configs(hidden: int, heads: int, kv_heads: int):
    from cruise_b200.model_config import ModelConfig

    geometry = dict(num_layers=2, hidden=hidden, num_heads=heads, num_kv_heads=kv_heads, head_dim=128,
                    intermediate=1024, vocab=4096, block_size=128, blocks_per_row=4, num_blocks=16)
    return (ModelConfig(name=f"long{hidden}", configured_eos=4095, **geometry), OracleConfig(**geometry))


@pytest.mark.parametrize("hidden, heads, kv_heads, seed", [(512, 4, 1, 0), (1024, 8, 2, 1)])
def test_long_context_decode_epoch(cuda_ok, hidden, heads, kv_heads, seed):
    from cruise_b200.engine import EpochEngine

    cfg, ocfg = _configs(hidden, heads, kv_heads)
    weights = seeded_weights(ocfg, seed=seed)
    engine = EpochEngine(cfg)
    engine.init_synthetic(seed)
    oracle = OracleEpochController(OracleDecoder(ocfg, weights))

    gen = torch.Generator().manual_seed(100 + seed)
    bt = torch.randperm(ocfg.num_blocks, generator=gen).to(torch.int32).reshape(4, ocfg.blocks_per_row).numpy()
    positions = np.array([37, 200, 300, 498], dtype=np.int64)
    token = torch.randint(0, ocfg.vocab - 1, (4,), generator=gen).numpy().astype(np.int64)
    gens = [1, 2, 3, 4]
    eos = [ocfg.vocab - 1] * 4
    shape = (ocfg.num_layers, ocfg.num_blocks, ocfg.block_size, ocfg.num_kv_heads, ocfg.head_dim)

    # 1. import every row (first block from a seeded payload) and decode one step
    payload = torch.randn((2, ocfg.num_layers, 4, ocfg.block_size, ocfg.num_kv_heads, ocfg.head_dim),
                          generator=gen).to(torch.bfloat16)
    slot = np.array([compute_slot(bt, ocfg.block_size, r, int(positions[r])) for r in range(4)], dtype=np.int32)
    inputs = dict(token=token, position=positions, seq_len=(positions + 1).astype(np.int32), slot=slot,
                  active=np.ones(4, dtype=np.int32), block_table=bt.reshape(-1),
                  control=np.array([1, *eos, 0, IMPORT_FLAG | 0xF, *gens], dtype=np.int32))
    out = engine.run(**inputs, import_payload=payload)
    history, control = oracle.run(**inputs, import_payload=payload)
    assert out.status == int(control[3]) == 0
    np.testing.assert_array_equal(out.history, history)
    np.testing.assert_array_equal(out.control_out, control)

    # 2. the same seeded contents in every cache slot on both sides
    key = torch.randn(shape, generator=gen).to(torch.bfloat16)
    value = torch.randn(shape, generator=gen).to(torch.bfloat16)
    engine.write_kv(key, value)
    oracle.key.copy_(key.to(oracle.key.dtype))
    oracle.value.copy_(value.to(oracle.value.dtype))

    # 3. a K=8 epoch over contexts of 39 .. 507 positions
    pos2 = positions + 1
    slot2 = np.array([compute_slot(bt, ocfg.block_size, r, int(pos2[r])) for r in range(4)], dtype=np.int32)
    inputs = dict(token=history[0].copy(), position=pos2, seq_len=(pos2 + 1).astype(np.int32), slot=slot2,
                  active=np.ones(4, dtype=np.int32), block_table=bt.reshape(-1),
                  control=np.array([8, *eos, 0, 0, *gens], dtype=np.int32))
    trace = EpochTrace()
    out = engine.run(**inputs, want_logits=True)
    history, control = oracle.run(**inputs, trace=trace)
    assert out.status == int(control[3]) == 0
    gk, gv = engine.read_kv()
    check_epoch(out, history, control, trace, inputs, kv=(gk, gv, oracle.key, oracle.value),
                block_size=ocfg.block_size, label=f"long context {hidden}")
    engine.close()
