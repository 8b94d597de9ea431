"""Tensor-parallel epoch engines: one process per GPU, one engine per rank.

The ranks of a group shard one model (query/KV heads, intermediate rows and
vocabulary rows; ``TpShard``) and exchange the row-parallel O / down partials
and the argmax of their vocabulary shards inside the epoch kernel, through each
other's exchange blocks mapped by CUDA IPC.  The host side only has to hand the
64-byte IPC handles around once; this module does that over any
``torch.distributed`` process group (gloo is enough: the handles are bytes).

After ``connect`` every rank must run the same epochs with the same inputs
(the epoch control is replicated, so all ranks emit the same tokens); a rank
that stops calling leaves the others' next epoch to end with a device-side
timeout status instead of a hang.
"""

from __future__ import annotations

import ctypes

import torch.distributed as dist

from . import _lib
from .engine import EpochEngine
from .model_config import ModelConfig, PRESETS, TpShard

HANDLE_BYTES = 64


def native_shard(config: ModelConfig | str, rank: int, size: int) -> TpShard:
    """The engine's own sharding of rank ``rank`` of ``size`` (host-only query)."""
    config = PRESETS[config] if isinstance(config, str) else config
    out = (ctypes.c_int32 * 8)()
    c_config = config.to_c()
    if _lib.load().cruise_epoch_tp_shard(ctypes.byref(c_config), rank, size, out) != 0:
        raise ValueError(f"{config.name} does not split over {size} ranks")
    q0, nq, kv0, nkv, i0, ni, v0, nv = list(out)
    return TpShard(rank, size, q0, nq, kv0, nkv, i0, ni, v0, nv)


def exchange_handles(local: bytes, group=None) -> list[bytes]:
    """All ranks' handles in rank order (an all-gather over ``group``)."""
    if len(local) != HANDLE_BYTES:
        raise ValueError(f"an exchange handle is {HANDLE_BYTES} bytes, got {len(local)}")
    gathered: list = [None] * dist.get_world_size(group)
    dist.all_gather_object(gathered, local, group=group)
    if any(not isinstance(h, bytes) or len(h) != HANDLE_BYTES for h in gathered):
        raise RuntimeError("a rank contributed no valid exchange handle")
    return gathered


def connect(engine: EpochEngine, group=None) -> None:
    """Exports this rank's exchange block, gathers every rank's and maps them."""
    if dist.get_world_size(group) != engine.shard.size or dist.get_rank(group) != engine.shard.rank:
        raise ValueError(
            f"engine is rank {engine.shard.rank} of {engine.shard.size}, the group has "
            f"rank {dist.get_rank(group)} of {dist.get_world_size(group)}"
        )
    engine.tp_connect(exchange_handles(engine.tp_handle(), group))
    dist.barrier(group=group)


def create_tp_engine(config: ModelConfig | str, device: int | None = None, group=None) -> EpochEngine:
    """This process's rank of a tensor-parallel engine over ``group``, connected.

    ``device`` defaults to the rank, the one-process-per-GPU layout."""
    rank, size = dist.get_rank(group), dist.get_world_size(group)
    engine = EpochEngine(config, device=rank if device is None else device, tp_rank=rank, tp_size=size)
    if size > 1:
        connect(engine, group)
    return engine
