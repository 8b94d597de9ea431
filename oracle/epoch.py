"""Resident epoch controller on the CPU (test infrastructure only).

Restates the device UDF ``G4cB4ResidentEpoch`` of the reference
(``controller/g4c_b4_resident_epoch.cpp``) over :class:`OracleDecoder`:

* constants / control layout      ``:13-38``
* ``ComputeSlot``                 ``:84-97``
* ``ArgmaxFinite``                ``:99-119``
* ``ClearCacheRow``               ``:129-147``
* ``Adler32Update``               ``:149-163`` (== zlib.adler32 chaining)
* ``Proc``: decode control         ``:207-241``; validation ``:335-385``;
  import ``:387-446``; generation continuity ``:448-473``; K-loop ``:485-591``;
  reasons and resident state ``:593-614``; ``emit`` ``:296-324``.

Generalisations (the reference hard-codes the 7B geometry and B=4 rows of two
blocks with capacity 8): capacity = blocks_per_row * block_size, the row's
blocks come from the block table instead of ``row*2, row*2+1``, and the import
copies the payload block into the row's first logical block ``bt[row][0]``.
"""

from __future__ import annotations

import zlib
from dataclasses import dataclass, field

import numpy as np
import torch

from .decoder import OracleDecoder
from .model import OracleConfig

# statuses (controller :60-74)
OK = 0
INVALID_METADATA = 201
CAPACITY_EXCEEDED = 202
INVALID_BLOCK_TABLE = 203
SLOT_MISMATCH = 204
UNSUPPORTED_SAMPLING = 205
UNSUPPORTED_GRAPH = 206
MODEL_ERROR = 207
INVALID_MODEL_OUTPUT = 208
NON_FINITE_LOGITS = 209
POSITION_PROGRESS = 210
ALLOCATION_FAILURE = 211
RESIDENT_CONTINUITY = 212

# finish reasons (controller :51-58)
FINISH_NONE, FINISH_EOS, FINISH_MAX_STEPS, FINISH_FALLBACK, FINISH_EMPTY, FINISH_ALREADY_FINISHED = range(6)

IMPORT_FLAG = 0x100
CONTROL_IN = 11
CONTROL_OUT = 28


def compute_slot(cfg: OracleConfig, block_table: np.ndarray, row: int, position: int) -> int:
    if row < 0 or row >= cfg.batch or position < 0 or position >= cfg.capacity:
        return -1
    logical = position // cfg.block_size
    offset = position % cfg.block_size
    if logical >= cfg.blocks_per_row:
        return -1
    physical = int(block_table[row * cfg.blocks_per_row + logical])
    if physical < 0 or physical >= cfg.num_blocks:
        return -1
    return physical * cfg.block_size + offset


def argmax_finite(logits_row: torch.Tensor) -> int | None:
    """First index of the maximum (strict ``>``); None on any non-finite value."""
    if not bool(torch.isfinite(logits_row).all()):
        return None
    return int(torch.argmax(logits_row).item())  # torch returns the first maximum


def top2_margin(logits_row: torch.Tensor) -> float:
    """Relative gap between the two largest logits (the divergence allowance)."""
    top = torch.topk(logits_row.float(), 2).values
    scale = max(abs(float(top[0])), 1e-6)
    return float(top[0] - top[1]) / scale


@dataclass
class EpochTrace:
    logits: list = field(default_factory=list)      # per executed step: f32 [B, V]
    active: list = field(default_factory=list)      # active mask entering each step
    margins: list = field(default_factory=list)     # per step: [B] relative top-2 margin


class OracleEpochController:
    """Holds the resident K/V and per-row state across epochs, like the UDF."""

    def __init__(self, decoder: OracleDecoder) -> None:
        self.decoder = decoder
        cfg = decoder.cfg
        self.cfg = cfg
        shape = (cfg.num_layers, cfg.num_blocks, cfg.block_size, cfg.num_kv_heads, cfg.head_dim)
        self.key = torch.zeros(shape, dtype=decoder.dtype)
        self.value = torch.zeros(shape, dtype=decoder.dtype)
        b = cfg.batch
        self.res_generation = [0] * b
        self.res_token = [0] * b
        self.res_position = [0] * b
        self.res_length = [0] * b
        self.res_valid = [0] * b

    # -- helpers -------------------------------------------------------------
    def clear_row(self, block_table: np.ndarray, row: int) -> None:
        bpr = self.cfg.blocks_per_row
        for local in range(bpr):
            block = int(block_table[row * bpr + local])
            self.key[:, block].zero_()
            self.value[:, block].zero_()

    def _block_bytes(self, cache: torch.Tensor, layer: int, block: int) -> bytes:
        view = cache[layer, block].contiguous()
        if view.dtype == torch.bfloat16:
            return view.view(torch.int16).numpy().tobytes()
        return view.numpy().tobytes()

    # -- one epoch (8-in / 2-out ABI) ----------------------------------------
    def run(
        self,
        token: np.ndarray,
        position: np.ndarray,
        seq_len: np.ndarray,
        slot: np.ndarray,
        active: np.ndarray,
        block_table: np.ndarray,
        control: np.ndarray,
        import_payload: torch.Tensor | None = None,
        trace: EpochTrace | None = None,
        forced: np.ndarray | None = None,
    ) -> tuple[np.ndarray, np.ndarray]:
        """One epoch.  ``forced`` ([8][4], -1 = greedy) replaces the argmax of a
        row at a step: the teacher-forced prefill extension of the engine."""
        cfg = self.cfg
        b = cfg.batch
        history = np.full((cfg.max_steps, b), -1, dtype=np.int64)
        out = np.zeros(CONTROL_OUT, dtype=np.int32)
        token = np.asarray(token, dtype=np.int64).reshape(b).copy()
        position = np.asarray(position, dtype=np.int64).reshape(b).copy()
        seq_len = np.asarray(seq_len, dtype=np.int32).reshape(b).copy()
        active0 = np.asarray(active, dtype=np.int32).reshape(b).copy()
        block_table = np.asarray(block_table, dtype=np.int32).reshape(-1).copy()
        control = np.asarray(control, dtype=np.int32).reshape(CONTROL_IN)
        encoded_variant = int(control[2 + b])
        importing = (encoded_variant & IMPORT_FLAG) != 0
        import_mask = encoded_variant & (IMPORT_FLAG - 1) if importing else 0
        variant = encoded_variant & ~(IMPORT_FLAG | 0xF) if importing else encoded_variant
        if importing:
            slot = np.array([compute_slot(cfg, block_table, r, int(position[r])) for r in range(b)], dtype=np.int32)
        else:
            slot = np.asarray(slot, dtype=np.int32).reshape(b).copy()
        max_steps = int(control[0])
        eos = [int(control[1 + r]) for r in range(b)]
        sampling = int(control[1 + b])
        generation = [int(control[3 + b + r]) for r in range(b)]
        executed = [0] * b
        reason = [FINISH_NONE] * b
        state = {"model_calls": 0, "checksum": 0}

        def emit(status: int, final_active) -> tuple[np.ndarray, np.ndarray]:
            out[0] = max_steps
            out[1] = sampling
            out[2] = variant
            out[3] = status
            out[4] = state["model_calls"]
            out[5] = np.int32(np.uint32(state["checksum"]).view(np.int32)) if importing else (0 if status == OK else 1)
            for r in range(b):
                out[6 + r] = eos[r]
                out[6 + b + r] = active0[r]
                out[6 + 2 * b + r] = executed[r]
                out[6 + 3 * b + r] = reason[r]
                out[6 + 4 * b + 2 + r] = generation[r] if active0[r] == 1 else 0
            out[6 + 4 * b] = int(np.count_nonzero(active0))
            out[6 + 4 * b + 1] = int(np.count_nonzero(final_active))
            return history, out

        def fallback(status: int):
            for r in range(b):
                reason[r] = FINISH_FALLBACK
            return emit(status, active0)

        # validation (:335-385)
        if max_steps < 1 or max_steps > cfg.max_steps or sampling != 0 or variant != 0:
            if sampling != 0:
                return fallback(UNSUPPORTED_SAMPLING)
            if variant != 0:
                return fallback(UNSUPPORTED_GRAPH)
            return fallback(INVALID_METADATA)
        if any(e < 0 or e >= cfg.vocab for e in eos):
            return fallback(INVALID_METADATA)
        seen = set()
        for block in block_table[: b * cfg.blocks_per_row]:
            block = int(block)
            if block < 0 or block >= cfg.num_blocks or block in seen:
                return fallback(INVALID_BLOCK_TABLE)
            seen.add(block)
        for r in range(b):
            if (active0[r] not in (0, 1) or token[r] < 0 or token[r] >= cfg.vocab
                    or position[r] < 0 or position[r] >= cfg.capacity):
                return fallback(INVALID_METADATA)
            if active0[r] == 1:
                if generation[r] <= 0 or seq_len[r] != position[r] + 1:
                    return fallback(INVALID_METADATA)
                if position[r] + max_steps > cfg.capacity:
                    return fallback(CAPACITY_EXCEEDED)
            elif seq_len[r] == 0:
                if generation[r] != 0:
                    return fallback(INVALID_METADATA)
                reason[r] = FINISH_EMPTY
            elif seq_len[r] == position[r] + 1:
                reason[r] = FINISH_ALREADY_FINISHED
            else:
                return fallback(INVALID_METADATA)
            if compute_slot(cfg, block_table, r, int(position[r])) != int(slot[r]):
                return fallback(SLOT_MISMATCH)

        # import (:387-446)
        if importing:
            if import_mask <= 0 or import_mask >= (1 << b):
                return fallback(INVALID_METADATA)
            payload = import_payload.reshape(2, cfg.num_layers, b, cfg.block_size, cfg.num_kv_heads, cfg.head_dim)
            for r in range(b):
                if not import_mask & (1 << r):
                    continue
                if active0[r] != 1 or generation[r] <= 0:
                    return fallback(INVALID_METADATA)
                self.clear_row(block_table, r)
                first = int(block_table[r * cfg.blocks_per_row])
                self.key[:, first] = payload[0, :, r].to(self.key.dtype)
                self.value[:, first] = payload[1, :, r].to(self.value.dtype)
                self.res_generation[r] = generation[r]
                self.res_token[r] = int(token[r])
                self.res_position[r] = int(position[r])
                self.res_length[r] = int(seq_len[r])
                self.res_valid[r] = 1
            checksum = 1
            for cache in (self.key, self.value):
                for layer in range(cfg.num_layers):
                    for r in range(b):
                        if import_mask & (1 << r):
                            block = int(block_table[r * cfg.blocks_per_row])
                            checksum = zlib.adler32(self._block_bytes(cache, layer, block), checksum)
            state["checksum"] = checksum & 0xFFFFFFFF

        # generation continuity (:448-473)
        new_generation = [0] * b
        for r in range(b):
            if active0[r] == 0:
                continue
            if self.res_generation[r] == generation[r]:
                if (not self.res_valid[r] or self.res_token[r] != token[r]
                        or self.res_position[r] != position[r] or self.res_length[r] != seq_len[r]):
                    return fallback(RESIDENT_CONTINUITY)
            else:
                if position[r] != 0 or seq_len[r] != 1:
                    return fallback(RESIDENT_CONTINUITY)
                new_generation[r] = 1
        for r in range(b):
            if new_generation[r]:
                self.clear_row(block_table, r)

        # K-loop (:485-591)
        cur_active = active0.copy()
        cur_token = token.copy()
        cur_position = position.copy()
        cur_length = seq_len.copy()
        cur_slot = slot.copy()
        bt = torch.from_numpy(block_table[: b * cfg.blocks_per_row].reshape(b, cfg.blocks_per_row).copy())
        while state["model_calls"] < max_steps:
            if np.count_nonzero(cur_active) == 0:
                break
            logits, key, value, next_position = self.decoder.step(
                torch.from_numpy(cur_token), torch.from_numpy(cur_position),
                torch.from_numpy(cur_length), bt, torch.from_numpy(cur_slot),
                self.key, self.value, torch.from_numpy(cur_active),
            )
            state["model_calls"] += 1
            step = state["model_calls"] - 1
            if trace is not None:
                trace.logits.append(logits.clone())
                trace.active.append(cur_active.copy())
                trace.margins.append([top2_margin(logits[r]) for r in range(b)])
            next_position = next_position.numpy()
            next_token = cur_token.copy()
            next_length = cur_length.copy()
            next_slot = cur_slot.copy()
            next_active = cur_active.copy()
            for r in range(b):
                if cur_active[r] == 0:
                    if next_position[r] != cur_position[r]:
                        return fallback(POSITION_PROGRESS)
                    continue
                forced_token = int(forced[step, r]) if forced is not None else -1
                generated = forced_token if forced_token >= 0 else argmax_finite(logits[r])
                if generated is None:
                    return fallback(NON_FINITE_LOGITS)
                if next_position[r] != cur_position[r] + 1:
                    return fallback(POSITION_PROGRESS)
                history[step, r] = generated
                executed[r] += 1
                cur_position[r] = next_position[r]
                next_token[r] = generated
                next_length[r] = cur_position[r] + 1
                if cur_position[r] == cfg.capacity:
                    next_slot[r] = -1
                else:
                    s = compute_slot(cfg, block_table, r, int(cur_position[r]))
                    if s < 0:
                        return fallback(CAPACITY_EXCEEDED)
                    next_slot[r] = s
                if generated == eos[r]:
                    next_active[r] = 0
                    reason[r] = FINISH_EOS
            self.key, self.value = key, value
            cur_token, cur_length, cur_slot, cur_active = next_token, next_length, next_slot, next_active

        for r in range(b):
            if active0[r] == 1 and reason[r] == FINISH_NONE:
                reason[r] = FINISH_MAX_STEPS
        for r in range(b):
            if active0[r] == 0:
                continue
            self.res_generation[r] = generation[r]
            self.res_token[r] = int(cur_token[r])
            self.res_position[r] = int(cur_position[r])
            self.res_length[r] = int(cur_length[r])
            self.res_valid[r] = 1
        return emit(OK, cur_active)


# -- host bridge (native/resident_epoch_bridge.cpp:424-649) ---------------------
@dataclass
class BridgeResult:
    ret: int
    tokens: np.ndarray          # i64 [batch * max_steps], row-major [row][step]
    executed: np.ndarray        # i32 [batch]
    row_generations: np.ndarray  # i32 [batch]
    model_calls: int = 0
    device_status: int = -1
    feed_calls: int = 0
    fetch_calls: int = 0
    commit_state: int = 0
    kv_import_checksum: int = 0
    declared_input_bytes: int = 0
    declared_output_bytes: int = 0


DECLARED_INPUT_BYTES = 260
DECLARED_OUTPUT_BYTES = 368


def bridge_execute(
    controller: OracleEpochController,
    request_count: int,
    max_steps: int,
    token_ids, positions, seq_lens, eos_ids, row_generations,
    configured_eos: int,
    snapshot: tuple[int, torch.Tensor, int] | None = None,
) -> BridgeResult:
    """``resident_epoch_execute`` over the oracle controller.

    ``snapshot`` = (import_mask, payload tensor, expected checksum) stands for
    the /dev/shm transfer file (``ReadTransfer`` :108-154).  The block table
    is the reference's fixed ``[row*bpr + j]`` ownership (``:524-532``).
    """
    cfg = controller.cfg
    b, bpr = cfg.batch, cfg.blocks_per_row
    result = BridgeResult(
        ret=10,
        tokens=np.full(b * cfg.max_steps, -1, dtype=np.int64),
        executed=np.zeros(b, dtype=np.int32),
        row_generations=np.zeros(b, dtype=np.int32),
    )
    importing = snapshot is not None
    if request_count < 1 or request_count > b or max_steps < 1 or max_steps > cfg.max_steps:
        return result
    result.declared_input_bytes = (
        2 * cfg.num_layers * b * cfg.block_size * cfg.kv_width * 2 + 244
        if importing else DECLARED_INPUT_BYTES
    )
    result.declared_output_bytes = DECLARED_OUTPUT_BYTES
    tokens = np.zeros(b, dtype=np.int64)
    pos = np.zeros(b, dtype=np.int64)
    lengths = np.zeros(b, dtype=np.int32)
    active = np.zeros(b, dtype=np.int32)
    blocks = np.array([r * bpr + j for r in range(b) for j in range(bpr)], dtype=np.int32)
    slots = np.array([compute_slot(cfg, blocks, r, 0) for r in range(b)], dtype=np.int32)
    count = 0
    for r in range(b):
        if row_generations[r] == 0:
            continue
        count += 1
        if (row_generations[r] < 0 or token_ids[r] < 0 or token_ids[r] >= cfg.vocab
                or positions[r] < 0 or positions[r] + max_steps > cfg.capacity
                or seq_lens[r] != positions[r] + 1 or eos_ids[r] < 0 or eos_ids[r] >= cfg.vocab):
            result.ret = 11
            return result
        tokens[r] = token_ids[r]
        pos[r] = positions[r]
        lengths[r] = seq_lens[r]
        slots[r] = compute_slot(cfg, blocks, r, int(positions[r]))
        active[r] = 1
    if count != request_count:
        result.ret = 12
        return result
    control = np.zeros(CONTROL_IN, dtype=np.int32)
    control[0] = max_steps
    for r in range(b):
        control[1 + r] = eos_ids[r] if row_generations[r] != 0 else configured_eos
    control[2 + b] = (IMPORT_FLAG | snapshot[0]) if importing else 0
    for r in range(b):
        control[3 + b + r] = row_generations[r]
    result.commit_state = 1
    history, out = controller.run(
        tokens, pos, lengths, slots, active, blocks, control,
        import_payload=snapshot[1] if importing else None,
    )
    result.feed_calls = result.fetch_calls = 1
    result.device_status = int(out[3])
    result.model_calls = int(out[4])
    result.kv_import_checksum = int(out[5])
    if result.device_status == 0 and importing:
        if (result.kv_import_checksum & 0xFFFFFFFF) != snapshot[2]:
            result.ret = 34
            return result
    for r in range(b):
        executed = int(out[6 + 2 * b + r])
        if executed < 0 or executed > max_steps:
            result.ret = 33
            return result
        result.executed[r] = executed
        result.row_generations[r] = int(out[6 + 4 * b + 2 + r])
        for step in range(executed):
            result.tokens[r * cfg.max_steps + step] = history[step, r]
    result.commit_state = 2
    result.ret = 0
    return result
