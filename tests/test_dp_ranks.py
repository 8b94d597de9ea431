"""Data-parallel cohorts on two gloo ranks (CPU): each rank seeds its own
cohort, and the timing reduction is the max over ranks of the device time and
the sum of the tokens (bench.py's multi-GPU aggregation)."""

import os
import socket

import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root))
    sys.path.insert(0, str(root / "tests"))
    import bench
    from scenario import make_scenario

    sc = make_scenario(vocab=152064, seed=1000 + rank, active_rows=(1, 1, 1, 1), token_high=151643)
    dev_s, tokens, wall = 0.5 + rank, 8 * (rank + 1), 0.6 + rank
    t_max, tok_total, wall_max = bench.reduce_over_ranks(dev_s, tokens, wall, device=None)
    results[rank] = (t_max, tok_total, wall_max, tuple(map(tuple, sc.prompts)))
    dist.destroy_process_group()


def test_two_rank_reduction_and_independent_cohorts():
    world, port = 2, _free_port()
    manager = mp.Manager()
    results = manager.dict()
    mp.spawn(_worker, args=(world, port, results), nprocs=world, join=True)
    for rank in range(world):
        t_max, tok_total, wall_max, _ = results[rank]
        assert t_max == 1.5 and tok_total == 8 + 16 and wall_max == 1.6
    assert results[0][3] != results[1][3]    # each rank decodes its own prompts
