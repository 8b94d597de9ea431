"""Seeded epoch scenarios shared by the GPU parity tests, ``smoke()`` and ``bench.py``.

A scenario is the tiny-configuration epoch workload generalised over the
model geometry: 4 rows, some inactive through the active mask, a seeded block
table, prompts of seeded length and ids, and a K-step greedy epoch.  Prompts
are prefilled row by row with teacher-forced epochs (the engine's device
prefill) and then handed to the decode epoch either directly (same resident
state) or through the one-shot import payload.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

BATCH = 4
MAX_STEPS = 8
IMPORT_FLAG = 0x100


@dataclass
class Scenario:
    block_table: np.ndarray              # i32 [4, blocks_per_row]
    prompts: list[list[int]]             # per row (empty for inactive rows)
    budgets: list[int]
    generations: list[int]               # 0 for inactive rows
    eos: list[int]
    k: int

    @property
    def active(self) -> np.ndarray:
        return np.array([1 if p else 0 for p in self.prompts], dtype=np.int32)


def make_scenario(
    *, vocab: int, seed: int, active_rows=(1, 1, 1, 0), prompt_len=(2, 5), budget=(2, 5),
    k: int = 2, num_blocks: int = 8, blocks_per_row: int = 2, eos: int | None = None,
    token_high: int | None = None,
) -> Scenario:
    gen = torch.Generator().manual_seed(seed)
    bt = torch.randperm(num_blocks, generator=gen)[: BATCH * blocks_per_row].to(torch.int32)
    prompts, budgets, gens = [], [], []
    high = token_high or vocab
    for row in range(BATCH):
        n = int(torch.randint(prompt_len[0], prompt_len[1] + 1, (1,), generator=gen))
        ids = torch.randint(0, high, (n,), generator=gen).tolist()
        b = int(torch.randint(budget[0], budget[1] + 1, (1,), generator=gen))
        if active_rows[row]:
            prompts.append(ids)
            budgets.append(b)
            gens.append(row + 1)
        else:
            prompts.append([])
            budgets.append(0)
            gens.append(0)
    eos_id = vocab - 1 if eos is None else eos
    return Scenario(bt.reshape(BATCH, blocks_per_row).numpy(), prompts, budgets, gens, [eos_id] * BATCH, k)


def compute_slot(block_table: np.ndarray, block_size: int, row: int, position: int) -> int:
    bpr = block_table.shape[1]
    if position < 0 or position >= block_size * bpr:
        return -1
    return int(block_table[row, position // block_size]) * block_size + position % block_size


def prefill_epochs(sc: Scenario, block_size: int, vocab: int):
    """Teacher-forced epochs that write the KV of every prompt token but the
    last, one row at a time, in chunks of at most 8 steps.  Yields the 8 epoch
    inputs plus the forced-token table."""
    for row in range(BATCH):
        prompt = sc.prompts[row]
        if not prompt:
            continue
        # an EOS id that the prompt does not contain, so forcing never stops early
        eos = next(t for t in range(vocab - 1, -1, -1) if t not in prompt)
        done = 0
        while done < len(prompt) - 1:
            steps = min(MAX_STEPS, len(prompt) - 1 - done)
            token = np.zeros(BATCH, dtype=np.int64)
            position = np.zeros(BATCH, dtype=np.int64)
            seq_len = np.zeros(BATCH, dtype=np.int32)
            active = np.zeros(BATCH, dtype=np.int32)
            gens = [0] * BATCH
            token[row] = prompt[done]
            position[row] = done
            seq_len[row] = done + 1
            active[row] = 1
            gens[row] = sc.generations[row]
            slot = np.array([compute_slot(sc.block_table, block_size, r, int(position[r])) for r in range(BATCH)],
                            dtype=np.int32)
            forced = np.full((MAX_STEPS, BATCH), -1, dtype=np.int64)
            for s in range(steps):
                forced[s, row] = prompt[done + s + 1]
            control = np.array([steps, eos, eos, eos, eos, 0, 0, *gens], dtype=np.int32)
            yield dict(token=token, position=position, seq_len=seq_len, slot=slot, active=active,
                       block_table=sc.block_table.reshape(-1), control=control, forced=forced)
            done += steps


def decode_inputs(sc: Scenario, block_size: int, importing: bool = False) -> dict:
    """The 8 inputs of the decode epoch that follows the prefill."""
    token = np.zeros(BATCH, dtype=np.int64)
    position = np.zeros(BATCH, dtype=np.int64)
    seq_len = np.zeros(BATCH, dtype=np.int32)
    for row in range(BATCH):
        prompt = sc.prompts[row]
        if prompt:
            token[row] = prompt[-1]
            position[row] = len(prompt) - 1
            seq_len[row] = len(prompt)
    slot = np.array([compute_slot(sc.block_table, block_size, r, int(position[r])) for r in range(BATCH)],
                    dtype=np.int32)
    mask = sum(1 << r for r in range(BATCH) if sc.prompts[r])
    variant = (IMPORT_FLAG | mask) if importing else 0
    control = np.array([sc.k, *sc.eos, 0, variant, *sc.generations], dtype=np.int32)
    return dict(token=token, position=position, seq_len=seq_len, slot=slot, active=sc.active,
                block_table=sc.block_table.reshape(-1), control=control)


def import_payload(key: torch.Tensor, value: torch.Tensor, sc: Scenario) -> torch.Tensor:
    """[K|V][layers][4 rows][block][kv_heads][head_dim] bf16 holding each active
    row's first logical block (the reference snapshot layout,
    kv_transfer.py:362-428), zeros for the other rows."""
    layers, _, bs, nkv, d = key.shape
    payload = torch.zeros((2, layers, BATCH, bs, nkv, d), dtype=torch.bfloat16)
    for row in range(BATCH):
        if sc.prompts[row]:
            block = int(sc.block_table[row, 0])
            payload[0, :, row] = key[:, block]
            payload[1, :, row] = value[:, block]
    return payload


@dataclass
class Divergence:
    rows: set = field(default_factory=set)


def compare_histories(gpu_history, oracle_history, margins, tol=2e-2) -> set:
    """Tokens must match exactly; a row may diverge only at a step where the
    oracle's relative top-2 logit margin is below ``tol`` (then later steps of
    that row are no longer comparable).  Returns the diverged rows."""
    diverged = set()
    steps = len(margins)
    for row in range(BATCH):
        for s in range(steps):
            o = int(oracle_history[s, row])
            g = int(gpu_history[s, row])
            if o == g:
                continue
            assert margins[s][row] < tol, (
                f"row {row} step {s}: gpu token {g} != oracle {o} with top-2 margin {margins[s][row]:.4g}"
            )
            diverged.add(row)
            break
    return diverged
