#!/usr/bin/env python3
"""Generate decoder-step golden vectors from the reference's own torch module.

Run in the container that holds the reference checkout (default path below):

    python tests/golden/make_golden.py --reference /path/to/Cruise [--geometry tiny|gqa7]

It imports ``PagedQwenDecoderStep`` from
``history/attempts/g4c-attempt69c-b4-air/batched_decoder_step.py`` unmodified,
overrides its module-level geometry constants with one of two configurations,
and registers for the CPU the bodies its custom ops are documented to
compute.  The configurations:

* ``tiny``: 2 layers, hidden 256, 4/2 heads of 64, intermediate 688, vocab
  4096, block 16, logical capacity 32 -> ``decoder_tiny.npz``;
* ``gqa7``: the 7B model's attention shape at a small size, 1 layer, hidden
  1792, 14/2 heads of 128 (7 query heads per KV head), intermediate 1024,
  vocab 4096, block 16 -> ``decoder_gqa7_d128.npz``.

The custom-op bodies:

* ``g4a_linear_t::mm_t``          = ``torch.mm(x, W.T)``   (``g4a_linear_t.py:17-18``)
* ``g4a_linear_t_bias::linear``   = ``F.linear(x, W, b)``  (``g4a_linear_t_bias.py:18-21``)
* ``g4a_qk::exact_qk``            = per-head ``a @ b`` with the input dtype as result
                                    (``qk-attempt50/export_qk_attempt50_air.py:47-56``)
* ``g4a_barrier::materialize`` and ``g4a_materialize::materialize`` = identity
                                    (``bf16-barrier/bf16_barrier.cpp:47-50``)

Weights come from the seeded generator (seed 0); caches and step inputs from a
seeded torch generator.
"""

from __future__ import annotations

import argparse
import importlib.util
import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO))

from oracle.model import GQA7_D128, TINY, seeded_weights  # noqa: E402

MODULE = "history/attempts/g4c-attempt69c-b4-air/batched_decoder_step.py"
GEOMETRIES = {"tiny": (TINY, "decoder_tiny.npz"), "gqa7": (GQA7_D128, "decoder_gqa7_d128.npz")}


def register_cpu_ops() -> None:
    lib_mm = torch.library.Library("g4a_linear_t", "DEF")
    lib_mm.define("mm_t(Tensor self, Tensor weight) -> Tensor")
    lib_mm.impl("mm_t", lambda x, w: torch.mm(x, w.transpose(0, 1)), "CPU")
    lib_lin = torch.library.Library("g4a_linear_t_bias", "DEF")
    lib_lin.define("linear(Tensor self, Tensor weight, Tensor bias) -> Tensor")
    lib_lin.impl("linear", lambda x, w, b: F.linear(x, w, b), "CPU")
    lib_qk = torch.library.Library("g4a_qk", "DEF")
    lib_qk.define("exact_qk(Tensor a, Tensor b, Tensor explicit_tiling) -> Tensor")
    lib_qk.impl(
        "exact_qk",
        lambda a, b, tiling: torch.bmm(a.transpose(0, 1), b).transpose(0, 1).contiguous(),
        "CPU",
    )
    libs = [lib_mm, lib_lin, lib_qk]
    for namespace in ("g4a_barrier", "g4a_materialize"):
        lib = torch.library.Library(namespace, "DEF")
        lib.define("materialize(Tensor x) -> Tensor")
        lib.impl("materialize", lambda x: x.clone(), "CPU")
        libs.append(lib)
    register_cpu_ops.libs = libs  # keep the registrations alive


def load_reference(reference: Path, cfg):
    spec = importlib.util.spec_from_file_location("ref_batched_decoder_step", reference / MODULE)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    module.NUM_LAYERS = cfg.num_layers
    module.HIDDEN_SIZE = cfg.hidden
    module.INTERMEDIATE_SIZE = cfg.intermediate
    module.NUM_HEADS = cfg.num_heads
    module.NUM_KV_HEADS = cfg.num_kv_heads
    module.NUM_KV_GROUPS = cfg.num_heads // cfg.num_kv_heads
    module.HEAD_DIM = cfg.head_dim
    module.VOCAB_SIZE = cfg.vocab
    module.RMS_EPS = cfg.rms_eps
    module.ROPE_THETA = cfg.rope_theta
    module.BATCH_SIZE = cfg.batch
    module.BLOCK_SIZE = cfg.block_size
    module.PHYSICAL_BLOCKS = cfg.num_blocks
    module.PHYSICAL_BLOCKS_PER_REQUEST = cfg.blocks_per_row
    module.LOGICAL_CAPACITY = cfg.capacity
    return module


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", type=Path, required=True, help="checkout of the reference project")
    parser.add_argument("--geometry", choices=sorted(GEOMETRIES), default="tiny")
    parser.add_argument("--output", type=Path, default=None)
    args = parser.parse_args()
    cfg, name = GEOMETRIES[args.geometry]
    output = args.output or REPO / "tests/golden" / name
    torch.set_num_threads(8)
    register_cpu_ops()
    ref = load_reference(args.reference, cfg)
    weights = seeded_weights(cfg, seed=0)
    model = ref.PagedQwenDecoderStep(dict(weights), batch_size=cfg.batch, physical_blocks=cfg.num_blocks)

    gen = torch.Generator().manual_seed(1234)
    cache_shape = (cfg.num_layers, cfg.num_blocks, cfg.block_size, cfg.num_kv_heads, cfg.head_dim)
    key_cache = (torch.randn(cache_shape, generator=gen) * 0.5).to(torch.bfloat16)
    value_cache = (torch.randn(cache_shape, generator=gen) * 0.5).to(torch.bfloat16)
    block_table = torch.randperm(cfg.num_blocks, generator=gen).to(torch.int32).reshape(cfg.batch, cfg.blocks_per_row)
    # rows: short context, second block context, full-window context, inactive
    position = torch.tensor([3, 20, cfg.capacity - 1, 5], dtype=torch.int64)
    active = torch.tensor([1, 1, 1, 0], dtype=torch.int32)
    seq_len = (position + 1).to(torch.int32)
    seq_len[3] = 0
    token = torch.randint(0, cfg.vocab, (cfg.batch, 1), generator=gen, dtype=torch.int64)
    slot = torch.tensor(
        [int(block_table[r, int(position[r]) // cfg.block_size]) * cfg.block_size + int(position[r]) % cfg.block_size
         for r in range(cfg.batch)],
        dtype=torch.int32,
    )
    tiling = torch.zeros(72, dtype=torch.uint8)
    with torch.no_grad():
        logits, new_key, new_value, next_position = model(
            token, position, seq_len, block_table, slot, key_cache, value_cache, tiling, active
        )
    np.savez_compressed(
        output,
        seed=np.int64(0),
        token=token.numpy(),
        position=position.numpy(),
        seq_len=seq_len.numpy(),
        block_table=block_table.numpy(),
        slot=slot.numpy(),
        active=active.numpy(),
        key_cache_in=bits(key_cache),
        value_cache_in=bits(value_cache),
        logits=logits.reshape(cfg.batch, cfg.vocab).numpy(),
        key_cache_out=bits(new_key),
        value_cache_out=bits(new_value),
        next_position=next_position.numpy(),
    )
    print(f"wrote {output}: argmax per row {logits.reshape(cfg.batch, -1).argmax(-1).tolist()}")


if __name__ == "__main__":
    main()
