"""Model geometry and seeded weights for the oracle (test infrastructure only).

Tensor names and shapes follow the checkpoint map of the reference decoder
(``history/attempts/g4c-attempt69c-b4-air/batched_decoder_step.py:43-91``),
generalised from the hard-coded 7B constants to any Qwen2 geometry.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from .synth import synth_bf16_bits, synth_bf16_bits_c

LAYER_KEYS = (
    "input_layernorm.weight",
    "post_attention_layernorm.weight",
    "self_attn.q_proj.weight",
    "self_attn.q_proj.bias",
    "self_attn.k_proj.weight",
    "self_attn.k_proj.bias",
    "self_attn.v_proj.weight",
    "self_attn.v_proj.bias",
    "self_attn.o_proj.weight",
    "mlp.gate_proj.weight",
    "mlp.up_proj.weight",
    "mlp.down_proj.weight",
)


@dataclass(frozen=True)
class OracleConfig:
    num_layers: int
    hidden: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    rms_eps: float = 1e-6
    rope_theta: float = 1_000_000.0
    batch: int = 4
    block_size: int = 128
    blocks_per_row: int = 2
    num_blocks: int = 8
    max_steps: int = 8

    @property
    def capacity(self) -> int:
        return self.block_size * self.blocks_per_row

    @property
    def kv_width(self) -> int:
        return self.num_kv_heads * self.head_dim


TINY = OracleConfig(
    num_layers=2, hidden=256, num_heads=4, num_kv_heads=2, head_dim=64,
    intermediate=688, vocab=4096, block_size=16,
)
QWEN25_7B = OracleConfig(
    num_layers=28, hidden=3584, num_heads=28, num_kv_heads=4, head_dim=128,
    intermediate=18944, vocab=152064, block_size=128,
)
# the 7B model's attention shape -- 7 query heads per KV head, head size 128,
# rope theta 1e6 -- at a size the reference module runs in about a second on
# the CPU (golden fixture tests/golden/decoder_gqa7_d128.npz)
GQA7_D128 = OracleConfig(
    num_layers=1, hidden=1792, num_heads=14, num_kv_heads=2, head_dim=128,
    intermediate=1024, vocab=4096, block_size=16,
)


def tensor_shapes(cfg: OracleConfig) -> dict[str, tuple[int, ...]]:
    h, kv, inter = cfg.hidden, cfg.kv_width, cfg.intermediate
    per_layer = {
        "input_layernorm.weight": (h,),
        "post_attention_layernorm.weight": (h,),
        "self_attn.q_proj.weight": (h, h),
        "self_attn.q_proj.bias": (h,),
        "self_attn.k_proj.weight": (kv, h),
        "self_attn.k_proj.bias": (kv,),
        "self_attn.v_proj.weight": (kv, h),
        "self_attn.v_proj.bias": (kv,),
        "self_attn.o_proj.weight": (h, h),
        "mlp.gate_proj.weight": (inter, h),
        "mlp.up_proj.weight": (inter, h),
        "mlp.down_proj.weight": (h, inter),
    }
    shapes = {"model.embed_tokens.weight": (cfg.vocab, h)}
    for layer in range(cfg.num_layers):
        for key in LAYER_KEYS:
            shapes[f"model.layers.{layer}.{key}"] = per_layer[key]
    shapes["model.norm.weight"] = (h,)
    shapes["lm_head.weight"] = (cfg.vocab, h)
    return shapes


def tensor_id(cfg: OracleConfig, name: str) -> int:
    if name == "model.embed_tokens.weight":
        return 0
    if name == "model.norm.weight":
        return 1 + len(LAYER_KEYS) * cfg.num_layers
    if name == "lm_head.weight":
        return 2 + len(LAYER_KEYS) * cfg.num_layers
    parts = name.split(".")
    layer = int(parts[2])
    key = ".".join(parts[3:])
    return 1 + len(LAYER_KEYS) * layer + LAYER_KEYS.index(key)


def seeded_weights(
    cfg: OracleConfig, seed: int, std: float = 0.02, dtype: torch.dtype = torch.bfloat16,
    use_c: bool = False,
) -> dict[str, torch.Tensor]:
    """All weights of the model as CPU tensors with the generator's bf16 values.
    ``use_c`` computes them with oracle/csynth.c on every host core (the same
    bits; a full 7B model in seconds instead of minutes)."""
    weights = {}
    for name, shape in tensor_shapes(cfg).items():
        count = int(np.prod(shape))
        if use_c:
            bits = synth_bf16_bits_c(seed, tensor_id(cfg, name), count, std)
        else:
            bits = synth_bf16_bits(seed, tensor_id(cfg, name), count, std)
        value = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16)
        weights[name] = value.reshape(shape).to(dtype)
    return weights
