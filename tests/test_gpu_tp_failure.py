"""Failure detection under tensor parallelism, without a GPU fault.

Two ranks (one GPU each) run the prefill epochs of a tiny-model cohort
together; then rank 1 leaves the group between epochs -- it does not launch the
next epoch, and keeps its exchange block mapped, no kernel in flight.  Rank
0's epoch must end on its own: its device waits for rank 1's partials give up
after the configured limit (CRUISE_TP_TIMEOUT_MS), the kernel winds down and
returns status 207 (the reference's model-error fallback) and names the wait
that gave up.  Rank 0's GPU stays usable: a fresh engine on it runs an
epoch normally.  Only then does rank 1 let go of its memory.  The ranks meet on
the host (gloo); no NCCL, no multicast."""

from __future__ import annotations

import os
import socket
import sys
import time
from datetime import timedelta
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

LIMIT_MS = 1500


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, port: int, results) -> None:
    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root))
    sys.path.insert(0, str(root / "tests"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), CRUISE_TP_TIMEOUT_MS=str(LIMIT_MS),
                      NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=timedelta(seconds=300))
    from cruise_b200.engine import EpochEngine, EngineError
    from cruise_b200.model_config import TINY
    from cruise_b200.tp import create_tp_engine
    from scenario import decode_inputs, make_scenario, prefill_epochs

    engine = create_tp_engine(TINY)
    engine.init_synthetic(0)
    sc = make_scenario(vocab=TINY.vocab, seed=0, active_rows=(1, 1, 1, 1), k=8, budget=(8, 8))
    for inputs in prefill_epochs(sc, TINY.block_size, TINY.vocab):
        dist.barrier()
        assert engine.run(**inputs).status == 0
    dist.barrier()
    if rank == 0:
        t0 = time.monotonic()
        out = engine.run(**decode_inputs(sc, TINY.block_size))   # rank 1 never joins this epoch
        elapsed = time.monotonic() - t0
        detail = engine.lib.cruise_epoch_last_error(engine.handle).decode()
        engine.close()
        # the device is fine: a fresh single-GPU engine decodes normally
        fresh = EpochEngine(TINY, device=0)
        fresh.init_synthetic(0)
        ok = all(fresh.run(**inputs).status == 0 for inputs in prefill_epochs(sc, TINY.block_size, TINY.vocab))
        fresh.close()
        results[0] = (out.status, elapsed, detail, ok, int(out.control_out[4]))
        dist.barrier()   # rank 1 may release its exchange block now
    else:
        dist.barrier()   # rank 0 finished and closed its mappings
        engine.close()
        results[1] = True
    dist.destroy_process_group()


def test_rank_leaving_ends_the_others_epoch_with_a_status(cuda_ok):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    mp.start_processes(_rank, args=(_free_port(), results), nprocs=2, join=True, start_method="spawn")
    status, elapsed, detail, fresh_ok, model_calls = results[0]
    assert status == 207, (status, detail)
    # the first wait to run out is the one on rank 1's partials (site 300) or,
    # as the exchange follows the phase's tile stream, the consumers' wait for
    # that epilogue (site 1004)
    assert "device-side wait that gave up" in detail, detail
    assert LIMIT_MS / 1000 * 0.9 < elapsed < 30, elapsed
    assert model_calls <= 1 and fresh_ok and results[1]
