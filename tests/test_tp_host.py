"""Tensor-parallel host logic on CPU: the shard geometry (Python mirror against
the engine's own through the C ABI), weight slicing that reassembles the whole
tensors, and the IPC-handle exchange over two gloo ranks."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from cruise_b200.model_config import QWEN25_7B, TINY, TpShard
from cruise_b200.tp import HANDLE_BYTES, native_shard

MODELS = {"tiny": TINY, "qwen2.5-7b": QWEN25_7B}


@pytest.mark.parametrize("model", sorted(MODELS))
@pytest.mark.parametrize("size", range(1, 9))
def test_shard_geometry_matches_engine(model, size):
    cfg = MODELS[model]
    for rank in range(size):
        try:
            mine = TpShard.of(cfg, rank, size)
        except ValueError:
            with pytest.raises(ValueError):
                native_shard(cfg, rank, size)
            continue
        assert native_shard(cfg, rank, size) == mine


@pytest.mark.parametrize("size", [1, 2, 4, 7, 8])
def test_qwen7b_shards_cover_the_model(size):
    cfg = QWEN25_7B
    if size == 7:
        with pytest.raises(ValueError):
            TpShard.of(cfg, 0, size)      # 4 KV heads do not split over 7 ranks
        return
    shards = [TpShard.of(cfg, r, size) for r in range(size)]
    # query heads, intermediate rows and vocabulary rows are partitions
    for start, count, total in (("q0", "nq", cfg.num_heads), ("i0", "ni", cfg.intermediate),
                                ("v0", "nv", cfg.vocab)):
        pos = 0
        for s in shards:
            assert getattr(s, start) == pos and getattr(s, count) > 0
            pos += getattr(s, count)
        assert pos == total
    grp = cfg.num_heads // cfg.num_kv_heads
    for s in shards:
        # every query head of a shard reads a KV head the shard holds
        assert s.kv0 * grp <= s.q0 and s.q0 + s.nq <= (s.kv0 + s.nkv) * grp
    if size == 8:
        assert [s.nq for s in shards] == [4, 3] * 4 and all(s.nkv == 1 for s in shards)


def test_slices_reassemble_whole_tensors():
    cfg = TINY
    gen = torch.Generator().manual_seed(0)
    d = cfg.head_dim
    full = {
        "model.layers.0.self_attn.q_proj.weight": torch.randn(cfg.num_heads * d, cfg.hidden, generator=gen),
        "model.layers.0.self_attn.k_proj.bias": torch.randn(cfg.num_kv_heads * d, generator=gen),
        "model.layers.0.self_attn.o_proj.weight": torch.randn(cfg.hidden, cfg.num_heads * d, generator=gen),
        "model.layers.0.mlp.up_proj.weight": torch.randn(cfg.intermediate, cfg.hidden, generator=gen),
        "model.layers.0.mlp.down_proj.weight": torch.randn(cfg.hidden, cfg.intermediate, generator=gen),
        "lm_head.weight": torch.randn(cfg.vocab, cfg.hidden, generator=gen),
        "model.layers.0.input_layernorm.weight": torch.randn(cfg.hidden, generator=gen),
    }
    shards = [TpShard.of(cfg, r, 2) for r in range(2)]
    for name, tensor in full.items():
        parts = [s.slice_tensor(cfg, name, tensor) for s in shards]
        if name.endswith(("o_proj.weight", "down_proj.weight")):
            assert torch.equal(torch.cat(parts, dim=1), tensor)
        elif name.endswith("layernorm.weight"):
            assert all(torch.equal(p, tensor) for p in parts)    # replicated
        else:
            assert torch.equal(torch.cat(parts, dim=0), tensor)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class _FakeEngine:
    """Stands in for a rank's EpochEngine: a handle of its own, records connect."""

    def __init__(self, rank, size):
        self.shard = TpShard.of(TINY, rank, size)
        self.connected = None

    def tp_handle(self) -> bytes:
        return bytes([self.shard.rank + 1]) * HANDLE_BYTES

    def tp_connect(self, handles):
        self.connected = list(handles)


def _worker(rank, world, port, results):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from cruise_b200.tp import connect, exchange_handles

    engine = _FakeEngine(rank, world)
    connect(engine)
    results[rank] = engine.connected
    # a malformed handle is refused before anything is gathered
    try:
        exchange_handles(b"short")
        results[f"short{rank}"] = False
    except ValueError:
        results[f"short{rank}"] = True
    # an engine of another group size is refused
    try:
        connect(_FakeEngine(0, 1))
        results[f"size{rank}"] = False
    except ValueError:
        results[f"size{rank}"] = True
    dist.destroy_process_group()


def test_two_rank_handle_exchange():
    world, port = 2, _free_port()
    manager = mp.Manager()
    results = manager.dict()
    mp.spawn(_worker, args=(world, port, results), nprocs=world, join=True)
    expect = [bytes([r + 1]) * HANDLE_BYTES for r in range(world)]
    for rank in range(world):
        assert results[rank] == expect
        assert results[f"short{rank}"] and results[f"size{rank}"]


@pytest.mark.parametrize("size", [2, 4, 8])
def test_shard_step_bytes_partition_the_step(size):
    import bench

    cfg = QWEN25_7B
    ctx = [5, 17, 130, 2]
    shards = [TpShard.of(cfg, r, size) for r in range(size)]
    total = sum(bench.shard_step_bytes(cfg, s, ctx) for s in shards)
    # replicated on every rank: the norms and the embedding rows
    replicated = 2 * (cfg.num_layers * 2 * cfg.hidden + cfg.hidden) + len(ctx) * cfg.hidden * 2
    # ranks sharing a KV head (size > KV heads) each stream its K/V weights and cache
    dup = max(1, size // cfg.num_kv_heads)
    kv_w = cfg.num_layers * 2 * (cfg.kv_width * cfg.hidden + cfg.kv_width) * 2
    kv_c = 2 * cfg.num_layers * cfg.kv_width * 2 * (sum(ctx) + len(ctx))
    assert total == bench.step_bytes(cfg, ctx) + (size - 1) * replicated + (dup - 1) * (kv_w + kv_c)


def _gather_worker(rank, world, port, results):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import bench

    class _Engine:
        config = QWEN25_7B
        shard = TpShard.of(QWEN25_7B, rank, world)

    full = torch.arange(2 * 3 * 2 * 4 * 5, dtype=torch.float32).reshape(2, 3, 2, 4, 5)
    s = _Engine.shard
    key, value = bench.gather_kv_shards(_Engine(), full[:, :, :, s.kv0:s.kv0 + s.nkv].clone(),
                                        -full[:, :, :, s.kv0:s.kv0 + s.nkv].clone())
    results[rank] = bool(torch.equal(key, full) and torch.equal(value, -full))
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 8])
def test_kv_shards_gather_to_the_whole_cache(world):
    port = _free_port()
    manager = mp.Manager()
    results = manager.dict()
    mp.spawn(_gather_worker, args=(world, port, results), nprocs=world, join=True)
    assert all(results[r] for r in range(world))
