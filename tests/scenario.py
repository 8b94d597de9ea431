"""Seeded epoch scenarios shared by the GPU parity tests, ``smoke()`` and ``bench.py``.

A scenario is the tiny-configuration epoch workload generalised over the
model geometry: 4 rows, some inactive through the active mask, a seeded block
table, prompts of seeded length and ids, and a K-step greedy epoch.  Prompts
are prefilled row by row with teacher-forced epochs (the engine's device
prefill) and then handed to the decode epoch either directly (same resident
state) or through the one-shot import payload.
"""

from __future__ import annotations

from dataclasses import dataclass

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


# control_out word indexes (controller :296-324)
W_MODEL_CALLS, W_CHECKSUM = 4, 5
W_EXECUTED, W_REASON, W_FINAL_COUNT = 14, 18, 23
FINISH_EOS, FINISH_MAX_STEPS = 1, 2

# every epoch compared in this process: (label, rows compared, {row: step} of
# the permitted near-tie divergences, near-tie row-steps); summarised at the
# end of the session
EPOCH_LOG: list[tuple[str, int, dict, int]] = []


def find_divergence(gpu_history, oracle_history, margins, tol=2e-2) -> dict[int, int]:
    """Tokens must match exactly; a row may diverge only at a step where the
    oracle's relative top-2 logit margin is below ``tol``.  Returns {row: first
    diverged step}."""
    diverged = {}
    for row in range(BATCH):
        for s in range(len(margins)):
            o = int(oracle_history[s, row])
            g = int(gpu_history[s, row])
            if o == g:
                continue
            assert margins[s][row] < tol, (
                f"row {row} step {s}: gpu token {g} != oracle {o} with top-2 margin {margins[s][row]:.4g}"
            )
            diverged[row] = s
            break
    return diverged


def compare_histories(gpu_history, oracle_history, margins, tol=2e-2) -> set:
    """The rows of :func:`find_divergence` (history-only callers)."""
    return set(find_divergence(gpu_history, oracle_history, margins, tol))


def rel_err_rows(a, b) -> torch.Tensor:
    """max |a - b| / max |b| along the last dimension, per vector; a vector whose
    reference is exactly zero must be exactly zero (else inf)."""
    a, b = torch.as_tensor(a).float(), torch.as_tensor(b).float()
    diff = (a - b).abs().amax(dim=-1)
    scale = b.abs().amax(dim=-1)
    err = diff / scale.clamp_min(1e-30)
    return torch.where(scale > 0, err, torch.where(diff > 0, torch.full_like(err, float("inf")), err))


def _assert_control(g: np.ndarray, o: np.ndarray, diverged: dict, skip=()) -> None:
    """Every control word equal, except those a permitted divergence may change
    (the diverged rows' executed count and reason, model calls, final count);
    those are checked for consistency on the GPU side instead."""
    unchecked = set(skip)
    if diverged:
        unchecked |= {W_MODEL_CALLS, W_FINAL_COUNT}
        unchecked |= {W_EXECUTED + r for r in diverged} | {W_REASON + r for r in diverged}
    for i in range(len(o)):
        if i not in unchecked:
            assert int(g[i]) == int(o[i]), f"control word {i}: gpu {int(g[i])} != oracle {int(o[i])}"
    executed = [int(v) for v in g[W_EXECUTED:W_EXECUTED + BATCH]]
    reason = [int(v) for v in g[W_REASON:W_REASON + BATCH]]
    if int(g[3]) == 0:
        assert int(g[W_MODEL_CALLS]) == max(executed), "model calls != longest row"
        assert int(g[W_FINAL_COUNT]) == sum(r == FINISH_MAX_STEPS for r in reason), "final count != running rows"
    for row, step in diverged.items():
        assert executed[row] >= step + 1 and reason[row] in (FINISH_EOS, FINISH_MAX_STEPS), (row, executed, reason)


def _assert_history_shape(history: np.ndarray, control: np.ndarray, row: int) -> None:
    executed = int(control[W_EXECUTED + row])
    column = [int(t) for t in history[:, row]]
    assert all(t >= 0 for t in column[:executed]) and all(t == -1 for t in column[executed:]), (row, column)
    if int(control[W_REASON + row]) == FINISH_EOS:
        assert column[executed - 1] == int(control[6 + row]), f"row {row} ended by EOS on another token"


def assert_kv(key, value, oracle_key, oracle_value, inputs: dict, block_size: int, diverged=None,
              executed=None, tol=2e-2) -> float:
    """KV caches [L][NB][bs][kv_heads][d]: blocks in no row of the block table
    bit-identical; every other cache slot within ``tol`` per head vector, except
    the slots a diverged row wrote after its divergence step (computed from
    different tokens on the two sides).  Returns the largest error compared."""
    diverged = diverged or {}
    nb = key.shape[1]
    bt = np.asarray(inputs["block_table"], dtype=np.int64).reshape(BATCH, -1)
    compared = torch.zeros((nb, block_size), dtype=torch.bool)
    referenced = sorted({int(b) for b in bt.reshape(-1)})
    for b in referenced:
        compared[b] = True
    for row, step in diverged.items():
        p0 = int(inputs["position"][row])
        end = p0 + max(int(executed[0][row]), int(executed[1][row])) if executed is not None else bt.shape[1] * block_size
        for p in range(p0 + step + 1, min(end, bt.shape[1] * block_size)):
            compared[int(bt[row, p // block_size]), p % block_size] = False
    worst = 0.0
    for name, g, o in (("key", key, oracle_key), ("value", value, oracle_value)):
        o = o.to(torch.bfloat16)
        for b in range(nb):
            if b not in referenced:
                assert torch.equal(g[:, b].view(torch.int16), o[:, b].view(torch.int16)), (
                    f"{name} block {b}, in no row of the block table, changed")
        mask = compared.view(1, nb, block_size).expand(g.shape[0], nb, block_size)
        err = rel_err_rows(g[mask], o[mask])
        if err.numel():
            top = float(err.max())
            assert top <= tol, f"{name} cache: per-head-vector rel err {top:.3g} > {tol}"
            worst = max(worst, top)
    return worst


@dataclass
class EpochCheck:
    diverged: dict                  # {row: step} permitted near-tie divergences
    logits_err: float = 0.0         # largest per-row relative logits error compared
    kv_err: float = 0.0             # largest per-head-vector relative KV error compared
    near_ties: int = 0              # row-steps whose oracle top-2 margin is below the tolerance


def check_epoch(out, history, control, trace, inputs: dict, *, tol=2e-2, kv=None, block_size=None,
                skip_words=(), max_diverged=1, label="epoch", record=True) -> EpochCheck:
    """One epoch of the engine (``out``: history, control_out, optional logits)
    against the oracle's (``history``, ``control`` and its ``trace``).

    * tokens equal, or a row diverges at a step whose oracle top-2 margin is
      below ``tol`` (at most ``max_diverged`` rows per epoch);
    * every control word equal except the few a divergence may move, which
      are checked for consistency instead;
    * logits within ``tol`` per row at every step a row ran on equal inputs
      (a diverged row up to and including its divergence step);
    * with ``kv`` = (key, value, oracle key, oracle value): :func:`assert_kv`.
    """
    diverged = find_divergence(out.history, history, trace.margins, tol)
    # row-steps the oracle ran whose top-2 margin is below the tolerance: the
    # only places a divergence is allowed
    near = sum(1 for s, m in enumerate(trace.margins) for r in range(BATCH) if trace.active[s][r] and m[r] < tol)
    if record:   # (the checker's own CPU tests forge their divergences)
        EPOCH_LOG.append((label, int(np.count_nonzero(np.asarray(inputs["active"]))), dict(diverged), near))
    assert len(diverged) <= max_diverged, (
        f"{label}: {len(diverged)} rows diverged at near-ties ({near} near-tie row-steps): {diverged}")
    _assert_control(out.control_out, control, diverged, skip_words)
    for row in range(BATCH):
        _assert_history_shape(out.history, out.control_out, row)
    worst_logits = 0.0
    if getattr(out, "logits", None) is not None:
        for step, logits in enumerate(trace.logits):
            rows = [r for r in range(BATCH) if trace.active[step][r] and (r not in diverged or step <= diverged[r])]
            if not rows:
                continue
            err = rel_err_rows(torch.from_numpy(out.logits[step, rows]), logits[rows])
            top = float(err.max())
            assert top <= tol, f"{label} step {step}: logits rel err {top:.3g} (rows {rows})"
            worst_logits = max(worst_logits, top)
    worst_kv = 0.0
    if kv is not None:
        executed = (out.control_out[W_EXECUTED:W_EXECUTED + BATCH], control[W_EXECUTED:W_EXECUTED + BATCH])
        worst_kv = assert_kv(*kv, inputs, block_size, diverged, executed, tol)
    if diverged:
        print(f"{label}: permitted near-tie divergence {diverged} (row: step)")
    return EpochCheck(diverged, worst_logits, worst_kv, near)
