"""Model geometry of the engine (the ``CruiseModelConfig`` of include/cruise_epoch.h).

Replaces the 7B constants hard-coded across the reference controller
(``controller/g4c_b4_resident_epoch.cpp:13-38``) and decoder step
(``history/attempts/g4c-attempt69c-b4-air/batched_decoder_step.py:19-36``).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, replace

BATCH = 4
MAX_STEPS = 8


class CruiseModelConfigC(ctypes.Structure):
    _fields_ = [
        ("num_layers", ctypes.c_int32),
        ("hidden", ctypes.c_int32),
        ("num_heads", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("intermediate", ctypes.c_int32),
        ("vocab", ctypes.c_int32),
        ("rms_eps", ctypes.c_float),
        ("rope_theta", ctypes.c_float),
        ("block_size", ctypes.c_int32),
        ("blocks_per_row", ctypes.c_int32),
        ("num_blocks", ctypes.c_int32),
        ("configured_eos", ctypes.c_int32),
        ("reserved", ctypes.c_int32 * 7),
    ]


@dataclass(frozen=True)
class ModelConfig:
    name: str
    num_layers: int
    hidden: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    rms_eps: float = 1e-6
    rope_theta: float = 1_000_000.0
    block_size: int = 128
    blocks_per_row: int = 2
    num_blocks: int = 8
    configured_eos: int = 151645

    @property
    def capacity(self) -> int:
        return self.block_size * self.blocks_per_row

    @property
    def kv_width(self) -> int:
        return self.num_kv_heads * self.head_dim

    @property
    def import_payload_bytes(self) -> int:
        return 2 * self.num_layers * BATCH * self.block_size * self.kv_width * 2

    @property
    def kv_cache_shape(self) -> tuple[int, ...]:
        return (self.num_layers, self.num_blocks, self.block_size, self.num_kv_heads, self.head_dim)

    def to_c(self) -> CruiseModelConfigC:
        c = CruiseModelConfigC()
        for field in (
            "num_layers", "hidden", "num_heads", "num_kv_heads", "head_dim", "intermediate",
            "vocab", "block_size", "blocks_per_row", "num_blocks", "configured_eos",
        ):
            setattr(c, field, getattr(self, field))
        c.rms_eps = self.rms_eps
        c.rope_theta = self.rope_theta
        return c

    def with_(self, **changes) -> "ModelConfig":
        return replace(self, **changes)

    def weight_bytes(self) -> int:
        h, kv, i, v = self.hidden, self.kv_width, self.intermediate, self.vocab
        per_layer = 2 * h + (h + 2 * kv) * h + (h + 2 * kv) + h * h + 3 * i * h
        return 2 * (2 * v * h + h + self.num_layers * per_layer)


QWEN25_7B = ModelConfig(
    name="qwen2.5-7b", num_layers=28, hidden=3584, num_heads=28, num_kv_heads=4, head_dim=128,
    intermediate=18944, vocab=152064, block_size=128, configured_eos=151645,
)
TINY = ModelConfig(
    name="tiny", num_layers=2, hidden=256, num_heads=4, num_kv_heads=2, head_dim=64,
    intermediate=688, vocab=4096, block_size=16, configured_eos=4095,
)
PRESETS = {QWEN25_7B.name: QWEN25_7B, TINY.name: TINY}


def layer_tensor_names(num_layers: int) -> list[str]:
    keys = (
        "input_layernorm.weight", "post_attention_layernorm.weight",
        "self_attn.q_proj.weight", "self_attn.q_proj.bias",
        "self_attn.k_proj.weight", "self_attn.k_proj.bias",
        "self_attn.v_proj.weight", "self_attn.v_proj.bias",
        "self_attn.o_proj.weight", "mlp.gate_proj.weight",
        "mlp.up_proj.weight", "mlp.down_proj.weight",
    )
    names = ["model.embed_tokens.weight"]
    for layer in range(num_layers):
        names.extend(f"model.layers.{layer}.{key}" for key in keys)
    names.extend(["model.norm.weight", "lm_head.weight"])
    return names


@dataclass(frozen=True)
class TpShard:
    """Tensor-parallel shard of rank ``rank`` of ``size`` (the engine's
    ``tp_geometry``): query heads [q0, q0+nq), KV heads [kv0, kv0+nkv),
    intermediate rows [i0, i0+ni), vocabulary rows [v0, v0+nv)."""

    rank: int
    size: int
    q0: int
    nq: int
    kv0: int
    nkv: int
    i0: int
    ni: int
    v0: int
    nv: int

    @staticmethod
    def of(config: ModelConfig, rank: int, size: int) -> "TpShard":
        if size not in (1, 2, 4, 8) or not 0 <= rank < size:
            raise ValueError(f"rank {rank} of {size} (tensor parallelism over 1, 2, 4 or 8 ranks)")
        nq, nkv = config.num_heads, config.num_kv_heads
        grp = nq // nkv
        if size <= nkv:
            if nkv % size:
                raise ValueError(f"{nkv} KV heads do not split over {size} ranks")
            kvn = nkv // size
            kv0 = rank * kvn
            q0, qn = kv0 * grp, kvn * grp
        else:
            if size % nkv:
                raise ValueError(f"{size} ranks do not share {nkv} KV heads evenly")
            per = size // nkv
            if grp < per:
                raise ValueError("fewer query heads per KV head than ranks sharing it")
            part, base, extra = rank % per, grp // per, grp % per
            kv0, kvn = rank // per, 1
            q0 = kv0 * grp + part * base + min(part, extra)
            qn = base + (1 if part < extra else 0)
        if config.intermediate % size or (config.intermediate // size) % 8:
            raise ValueError(f"intermediate {config.intermediate} does not split over {size} ranks")
        ni = config.intermediate // size
        vs = -(-config.vocab // size)
        v0 = rank * vs
        nv = min(vs, config.vocab - v0)
        if nv <= 0:
            raise ValueError(f"vocabulary {config.vocab} leaves rank {rank} of {size} no rows")
        return TpShard(rank, size, q0, qn, kv0, kvn, rank * ni, ni, v0, nv)

    def kv_cache_shape(self, config: ModelConfig) -> tuple[int, ...]:
        return (config.num_layers, config.num_blocks, config.block_size, self.nkv, config.head_dim)

    def slice_tensor(self, config: ModelConfig, name: str, full):
        """This rank's part of a whole checkpoint tensor (a torch tensor)."""
        d = config.head_dim
        key = name.split(".", 3)[-1] if name.startswith("model.layers.") else name
        if key in ("self_attn.q_proj.weight", "self_attn.q_proj.bias"):
            return full[self.q0 * d:(self.q0 + self.nq) * d]
        if key in ("self_attn.k_proj.weight", "self_attn.k_proj.bias",
                   "self_attn.v_proj.weight", "self_attn.v_proj.bias"):
            return full[self.kv0 * d:(self.kv0 + self.nkv) * d]
        if key == "self_attn.o_proj.weight":
            return full[:, self.q0 * d:(self.q0 + self.nq) * d]
        if key in ("mlp.gate_proj.weight", "mlp.up_proj.weight"):
            return full[self.i0:self.i0 + self.ni]
        if key == "mlp.down_proj.weight":
            return full[:, self.i0:self.i0 + self.ni]
        if key == "lm_head.weight":
            return full[self.v0:self.v0 + self.nv]
        return full
