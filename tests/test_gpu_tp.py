"""Tensor-parallel epochs on 2, 4 or 8 GPUs (one spawned process per GPU),
against the CPU oracle of the whole model.

Each rank holds its shard (query/KV heads, intermediate and vocabulary rows)
and the kernel all-reduces the O / down partials and the vocabulary argmax
through peer memory.  The partial sums are added in a different order than
the single-GPU kernel's, so the bar is the tolerance one: tokens and integer
state bit-exact except where the oracle's top-2 margin is below 2e-2,
logits (reassembled from the ranks' vocabulary shards) and the KV shards
within max relative error 2e-2.  Every rank must report the same tokens and
control words (the epoch control is replicated).

* tiny model, TP=2: prefill epochs then a K=8 decode epoch;
* 7B geometry (2 layers), TP=2/4/8 as GPUs allow: the one-shot import with a
  K=2 epoch, and a masked K=8 epoch after device prefill.  TP=8 splits the
  7 query heads of each KV head 4/3 over two ranks.
"""

from __future__ import annotations

import hashlib
import os
import socket
import sys
from dataclasses import replace
from datetime import timedelta
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle.decoder import OracleDecoder
from oracle.epoch import EpochTrace, OracleEpochController
from oracle.model import TINY as ORACLE_TINY, OracleConfig, seeded_weights, tensor_shapes
from scenario import BATCH, compare_histories, decode_inputs, import_payload, make_scenario, prefill_epochs

pytestmark = pytest.mark.gpu

TOL = 2e-2
TOKEN_HIGH = 151643


def _gpus() -> int:
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _digest(t: torch.Tensor) -> str:
    return hashlib.sha1(t.contiguous().view(torch.int16).numpy().tobytes()).hexdigest()


def _worker(rank, world, port, cfg, runs, names, results):
    """One rank: a fresh TP engine per run, the run's epochs in lockstep, then
    this rank's KV shard; finally digests of its weight shards."""
    import torch.distributed as dist

    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=300))
    from cruise_b200.tp import create_tp_engine

    out_runs = []
    for epochs in runs:
        engine = create_tp_engine(cfg)
        engine.init_synthetic(0)
        outs = []
        for inputs, kw in epochs:
            dist.barrier()   # the ranks launch each epoch together
            o = engine.run(**inputs, **kw)
            s = engine.shard
            lg = o.logits[:, :, s.v0:s.v0 + s.nv].copy() if o.logits is not None else None
            outs.append((o.history.copy(), o.control_out.copy(), lg))
        key, value = engine.read_kv()
        out_runs.append((outs, key, value))
        dist.barrier()
        digests = {name: _digest(engine.get_weight(name, shape)) for name, shape in names.items()} \
            if epochs is runs[-1] else None
        engine.close()
    shard = engine.shard
    results[rank] = (out_runs, digests, (shard.v0, shard.nv, shard.kv0, shard.nkv))
    dist.barrier()
    dist.destroy_process_group()


def _shard_shapes(cfg, weights, world):
    """name -> this rank's shard shape, per rank."""
    from cruise_b200.model_config import TpShard

    out = []
    for r in range(world):
        s = TpShard.of(cfg, r, world)
        out.append({name: tuple(s.slice_tensor(cfg, name, w).shape) for name, w in weights.items()})
    return out


def _run_ranks(cfg, world, runs, weights):
    from cruise_b200.model_config import TpShard

    port = _free_port()
    manager = mp.get_context("spawn").Manager()   # no fork of a process that may hold a CUDA context
    results = manager.dict()
    shapes = _shard_shapes(cfg, weights, world)
    ctx = mp.start_processes(
        _rank_entry, args=(world, port, cfg, runs, shapes, results), nprocs=world, join=True,
        start_method="spawn",
    )
    del ctx
    res = [results[r] for r in range(world)]
    # every rank's weight shards are the slices of the whole seeded tensors
    for r in range(world):
        s = TpShard.of(cfg, r, world)
        for name, w in weights.items():
            assert res[r][1][name] == _digest(s.slice_tensor(cfg, name, w)), (r, name)
    return res


def _rank_entry(rank, world, port, cfg, runs, shapes, results):
    _worker(rank, world, port, cfg, runs, shapes[rank], results)


def _check(res, oracle_runs, world):
    """Compares every run's epochs and KV with the oracle's."""
    for run_index, (oracle, epochs) in enumerate(oracle_runs):
        traces, histories, controls = epochs
        for e in range(len(histories)):
            ranks = [res[r][0][run_index][0][e] for r in range(world)]
            for r in range(1, world):   # replicated control: identical on every rank
                np.testing.assert_array_equal(ranks[r][0], ranks[0][0])
                np.testing.assert_array_equal(ranks[r][1], ranks[0][1])
            history, control_out, _ = ranks[0]
            assert int(control_out[3]) == int(controls[e][3]) == 0
            trace = traces[e]
            if trace is None:   # teacher-forced prefill: tokens are the prompt
                np.testing.assert_array_equal(history, histories[e])
                continue
            diverged = compare_histories(history, histories[e], trace.margins)
            if not diverged:
                np.testing.assert_array_equal(control_out, controls[e])
            if ranks[0][2] is not None:
                for step, logits in enumerate(trace.logits):
                    merged = np.zeros(logits.shape[-1], dtype=np.float32)
                    for row in range(BATCH):
                        if not trace.active[step][row] or row in diverged:
                            continue
                        for r in range(world):
                            v0, nv = res[r][2][0], res[r][2][1]
                            merged[v0:v0 + nv] = ranks[r][2][step, row]
                        ref = logits[row].float()
                        err = float((torch.from_numpy(merged) - ref).abs().max()) / max(float(ref.abs().max()), 1e-30)
                        assert err <= TOL, f"run {run_index} step {step} row {row}: logits rel err {err:.3g}"
        if all(compare_histories(res[0][0][run_index][0][e][0], histories[e], traces[e].margins) == set()
               for e in range(len(histories)) if traces[e] is not None):
            for r in range(world):
                kv0, nkv = res[r][2][2], res[r][2][3]
                key, value = res[r][0][run_index][1], res[r][0][run_index][2]
                for name, g, o in (("key", key, oracle.key), ("value", value, oracle.value)):
                    ref = o[..., kv0:kv0 + nkv, :].float()
                    err = float((g.float() - ref).abs().max()) / max(float(ref.abs().max()), 1e-30)
                    assert err <= TOL, f"run {run_index} rank {r}: {name} cache rel err {err:.3g}"


def _oracle_epochs(ocfg, weights, epochs):
    """Runs the epochs on a fresh oracle; returns it and (traces, histories, controls)."""
    oracle = OracleEpochController(OracleDecoder(ocfg, weights))
    traces, histories, controls = [], [], []
    for inputs, kw in epochs:
        trace = EpochTrace() if kw.get("want_logits") else None
        okw = {k: v for k, v in kw.items() if k != "want_logits"}
        history, control = oracle.run(**inputs, trace=trace, **okw) if trace is not None else oracle.run(**inputs, **okw)
        traces.append(trace)
        histories.append(history)
        controls.append(control)
    return oracle, (traces, histories, controls)


def test_tiny_tp2(cuda_ok):
    if _gpus() < 2:
        pytest.skip("tensor parallelism needs 2 GPUs")
    from cruise_b200.model_config import TINY

    weights = seeded_weights(ORACLE_TINY, seed=0)
    sc = make_scenario(vocab=TINY.vocab, seed=0, active_rows=(1, 1, 1, 1), k=8, budget=(8, 8))
    epochs = [(inputs, {}) for inputs in prefill_epochs(sc, TINY.block_size, TINY.vocab)]
    epochs.append((decode_inputs(sc, TINY.block_size), {"want_logits": True}))
    oracle_runs = [_oracle_epochs(ORACLE_TINY, weights, epochs)]
    res = _run_ranks(TINY, 2, [epochs], weights)
    _check(res, oracle_runs, 2)


@pytest.fixture(scope="module")
def geometry(cuda_ok):
    """The 7B geometry cut to 2 layers and its seeded weights (read back from a
    single-GPU engine, whose generator the tiny tests pin against the CPU one)."""
    from cruise_b200.engine import EpochEngine
    from cruise_b200.model_config import QWEN25_7B

    if _gpus() < 2:
        pytest.skip("tensor parallelism needs 2 GPUs")
    cfg = replace(QWEN25_7B, name="qwen2.5-7b-2l", num_layers=2)
    ocfg = OracleConfig(num_layers=2, hidden=cfg.hidden, num_heads=cfg.num_heads,
                        num_kv_heads=cfg.num_kv_heads, head_dim=cfg.head_dim, intermediate=cfg.intermediate,
                        vocab=cfg.vocab, block_size=cfg.block_size, blocks_per_row=cfg.blocks_per_row,
                        num_blocks=cfg.num_blocks)
    engine = EpochEngine(cfg)
    engine.init_synthetic(0)
    weights = {name: engine.get_weight(name, shape) for name, shape in tensor_shapes(ocfg).items()}
    engine.close()
    return cfg, ocfg, weights


@pytest.mark.parametrize("world", [2, 4, 8])
def test_qwen7b_geometry_tp(geometry, world):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    cfg, ocfg, weights = geometry
    # run 1: prompts prefilled by the oracle, imported in one shot, K=2
    sc1 = make_scenario(vocab=cfg.vocab, seed=world, active_rows=(1, 1, 1, 1), prompt_len=(2, 5),
                        token_high=TOKEN_HIGH, k=2)
    prefill = OracleEpochController(OracleDecoder(ocfg, weights))
    for inputs in prefill_epochs(sc1, cfg.block_size, cfg.vocab):
        prefill.run(**inputs)
    payload = import_payload(prefill.key, prefill.value, sc1)
    run1 = [(decode_inputs(sc1, cfg.block_size, importing=True),
             {"import_payload": payload, "want_logits": True})]
    # run 2: device prefill, then a K=8 epoch with row 2 masked off
    sc2 = make_scenario(vocab=cfg.vocab, seed=20 + world, active_rows=(1, 1, 0, 1), prompt_len=(2, 5),
                        token_high=TOKEN_HIGH, k=8, budget=(8, 8))
    run2 = [(inputs, {}) for inputs in prefill_epochs(sc2, cfg.block_size, cfg.vocab)]
    run2.append((decode_inputs(sc2, cfg.block_size), {"want_logits": True}))
    oracle_runs = [_oracle_epochs(ocfg, weights, run1), _oracle_epochs(ocfg, weights, run2)]
    res = _run_ranks(cfg, world, [run1, run2], weights)
    _check(res, oracle_runs, world)
