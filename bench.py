#!/usr/bin/env python3
"""Benchmark: Qwen2.5-7B-arch B=4 resident decode epochs (decode tok/s, us/step,
% HBM roofline) on 1..N B200s of one node.

Workload (benchmark configuration 2 of the task): the 7B architecture with seeded random-init
bf16 weights (generated on the device), paged KV of 128-token blocks, 2 blocks
per row, B=4 rows all active with prompts of 2-5 tokens (ids in [0, 151643)).
Prompts are prefilled on the device with teacher-forced epochs, the prefilled
first blocks are read back and re-imported once through the one-shot
host-to-device KV import (the import epoch is the first K=2 epoch), and then
K=2 greedy epochs keep decoding.  A "step" of this benchmark is one epoch.

value    decode tokens/s over the timed epochs, device time (CUDA events around
         the epoch kernel on its own stream), max over ranks.
e2e      the same through the C-ABI call with host buffers: H2D of the epoch
         inputs and D2H of the token history + control output inside the timed
         wall-clock region.
cpu_baseline / --impl reference
         whole greedy epochs of the CPU oracle (a port of the reference's torch
         decode step and epoch controller; the reference path itself needs
         Ascend hardware), all 28 layers, on the host cores: the same seeded
         weights (the C restatement of the generator), the same cohort,
         prefilled and imported the same way, perf_counter around each epoch.

Multi-GPU (torchrun, N ranks): the headline is one tensor-parallel group over
the N GPUs decoding the same single B=4 cohort as N=1 (strong scaling): each GPU
streams its 1/N of the weights and the epoch kernel exchanges the O / down
partials and the vocabulary argmax over NVLink peer memory; value counts the
cohort's tokens once, and the roofline compares the group's shard bytes with N
x the per-GPU HBM peak.  tp_check compares the group's tokens with a single-GPU
engine's on the untimed epochs.  The line's "dp" key is the data-parallel
layout measured in the same run: every rank an independent B=4 cohort on its
own full-model engine (weak scaling, tokens summed).  --dp makes that layout
the headline instead.

Other options: --k (epoch length), --prompt-max (longest seeded prompt; the
box-scale variant uses 120), --trace (per-phase CTA-0 timeline of one extra
epoch on stderr), --prefill (a separate measurement: the batched device
prefill of a 4 x 120-token cohort against teacher-forced epochs).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from dataclasses import dataclass
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

METRIC = "Qwen2.5-7B-arch B=4 epoch: decode tok/s, µs/step, % HBM roofline"

# DRAM traffic of one resident_epoch_kernel launch of the default workload (K=2,
# 7B geometry), dram__bytes_read.sum + dram__bytes_write.sum from a one-pass ncu
# capture of this bench command; reported per decode step beside the
# algorithmic bytes.  It applies to the default K only.
PROFILED_TRAFFIC = {"k": 2, "bytes_per_launch": 28301151744 + 21519616, "steps_per_launch": 2}
KV_BYTES_PER_TOKEN = 28 * 4 * 128 * 2 * 2   # K and V over all layers, one position
FALLBACK_HBM_GBS = 6650.0
EPOCH_H2D_BYTES = 616   # EpochIO inputs (8-in ABI + forced-token table), one copy per epoch
EPOCH_D2H_BYTES = 368   # token history i64[8][4] + control output i32[28]


def hbm_peak() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def weight_bytes_per_step(cfg) -> int:
    """Bytes of weights one decode step streams (every projection, the norms,
    biases and lm_head; the embedding table contributes only 4 gathered rows)."""
    h, kv, i, v, L = cfg.hidden, cfg.kv_width, cfg.intermediate, cfg.vocab, cfg.num_layers
    per_layer = (h + 2 * kv) * h + (h + 2 * kv) + h * h + 2 * i * h + h * i + 2 * h
    return 2 * (L * per_layer + v * h + h)


def step_bytes(cfg, contexts: list[int]) -> int:
    """Algorithmic HBM bytes of one decode step: weights + KV read over each
    active row's context + KV write of the new position + embedding rows."""
    kv_token = 2 * cfg.num_layers * cfg.kv_width * 2
    return weight_bytes_per_step(cfg) + kv_token * (sum(contexts) + len(contexts)) + len(contexts) * cfg.hidden * 2


def shard_step_bytes(cfg, shard, contexts: list[int]) -> int:
    """step_bytes of one tensor-parallel rank: its query/KV heads, intermediate
    and vocabulary rows, the replicated norms and its KV heads' cache."""
    h, d, L = cfg.hidden, cfg.head_dim, cfg.num_layers
    qkv = (shard.nq + 2 * shard.nkv) * d
    per_layer = qkv * h + qkv + h * shard.nq * d + 3 * shard.ni * h + 2 * h
    weights = 2 * (L * per_layer + shard.nv * h + h)
    kv_token = 2 * L * shard.nkv * d * 2
    return weights + kv_token * (sum(contexts) + len(contexts)) + len(contexts) * h * 2


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons sampled during the timed
    region: NVML queries every 10 ms from a thread (read-only), else
    nvidia-smi at its 100 ms floor."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clock event reason bits
    REASONS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40}

    def __init__(self, device: int) -> None:
        self.device = device
        self.proc = None
        self.nvml = None
        self.lines: list[str] = []
        self.samples: list[tuple[float, float, int]] = []
        self.stop = threading.Event()

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nvml = pynvml
            self.handle = pynvml.nvmlDeviceGetHandleByIndex(self.device)
            self.thread = threading.Thread(target=self._poll, daemon=True)
            self.thread.start()
            deadline = time.time() + 2.0
            while not self.samples and time.time() < deadline:   # the first sample precedes the timed region
                time.sleep(0.002)
            return self
        except Exception:
            self.nvml = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
            )
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except FileNotFoundError:
            self.proc = None
        return self

    def _poll(self):
        nv = self.nvml
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self.stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM)
                mx = nv.nvmlDeviceGetMaxClockInfo(self.handle, nv.NVML_CLOCK_SM)
                reasons = get_reasons(self.handle)
                self.samples.append((float(sm), float(mx), int(reasons)))
            except Exception:
                break
            time.sleep(0.01)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        self.stop.set()
        if self.nvml is not None:
            self.thread.join(timeout=1)
            try:
                self.nvml.nvmlShutdown()
            except Exception:
                pass
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        return False

    def summary(self) -> dict:
        if self.samples:
            reasons = {name for name, bit in self.REASONS.items() if any(r & bit for _, _, r in self.samples)}
            return {"sm_mhz": statistics.median(sm for sm, _, _ in self.samples),
                    "sm_max_mhz": self.samples[-1][1], "reasons": sorted(reasons),
                    "samples": len(self.samples), "source": "nvml, 10 ms"}
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": mx,
            "reasons": sorted(reasons),
            "samples": len(sm),
        }


def gather_kv_shards(engine, key, value):
    """The whole KV cache from every tensor-parallel rank's head shard (an
    all-gather over the default process group; ranks sharing a KV head hold
    identical copies of it)."""
    import torch
    import torch.distributed as dist

    shard = engine.shard
    parts: list = [None] * dist.get_world_size()
    dist.all_gather_object(parts, (shard.kv0, shard.nkv, key, value))
    shape = list(key.shape)
    shape[3] = engine.config.num_kv_heads
    full_k = torch.empty(shape, dtype=key.dtype)
    full_v = torch.empty(shape, dtype=value.dtype)
    for kv0, nkv, k_part, v_part in parts:
        full_k[:, :, :, kv0:kv0 + nkv] = k_part
        full_v[:, :, :, kv0:kv0 + nkv] = v_part
    return full_k, full_v


def setup_cohort(engine, cfg, seed: int, k: int, prompt_max: int = 5, want_logits: bool = False,
                 generation_offset: int = 0):
    """Device prefill of a seeded B=4 cohort, then the one-shot import epoch.
    `generation_offset` moves the rows' generations, so a second cohort can
    take over rows that an earlier one left behind."""
    from scenario import decode_inputs, import_payload, make_scenario, prefill_epochs

    sc = make_scenario(vocab=cfg.vocab, seed=seed, active_rows=(1, 1, 1, 1), prompt_len=(2, prompt_max),
                       budget=(2, 8), k=k, eos=cfg.configured_eos, token_high=min(151643, cfg.vocab - 1))
    sc.generations = [g + generation_offset for g in sc.generations]
    for inputs in prefill_epochs(sc, cfg.block_size, cfg.vocab):
        out = engine.run(**inputs)
        assert out.status == 0, f"prefill epoch status {out.status}"
    key, value = engine.read_kv()
    if engine.shard.size > 1:
        key, value = gather_kv_shards(engine, key, value)
    payload = import_payload(key, value, sc)
    inputs = decode_inputs(sc, cfg.block_size, importing=True)
    out = engine.run(**inputs, import_payload=payload, want_logits=want_logits)
    assert out.status == 0, f"import epoch status {out.status}"
    return sc, out


class Cohort:
    """Keeps a cohort decoding epoch after epoch (continuing resident state)."""

    def __init__(self, engine, cfg, sc, last_out) -> None:
        self.engine, self.cfg, self.sc = engine, cfg, sc
        self.token = np.zeros(4, dtype=np.int64)
        self.position = np.zeros(4, dtype=np.int64)
        for r in range(4):
            self.position[r] = len(sc.prompts[r]) - 1
        self._advance(last_out)

    def _advance(self, out):
        for r in range(4):
            executed = int(out.control_out[6 + 8 + r])
            if executed:
                self.token[r] = out.history[executed - 1, r]
                self.position[r] += executed

    def inputs(self):
        from scenario import compute_slot

        cfg, sc = self.cfg, self.sc
        seq_len = (self.position + 1).astype(np.int32)
        slot = np.array([compute_slot(sc.block_table, cfg.block_size, r, int(self.position[r])) for r in range(4)],
                        dtype=np.int32)
        control = np.array([sc.k, *sc.eos, 0, 0, *sc.generations], dtype=np.int32)
        return dict(token=self.token.copy(), position=self.position.copy(), seq_len=seq_len, slot=slot,
                    active=np.ones(4, dtype=np.int32), block_table=sc.block_table.reshape(-1), control=control)

    def step(self, want_logits: bool = False):
        inputs = self.inputs()
        out = self.engine.run(**inputs, want_logits=want_logits) if want_logits else self.engine.run(**inputs)
        if out.status != 0:
            raise RuntimeError(f"epoch status {out.status}")
        self._advance(out)
        return out, inputs

    def room(self) -> int:
        return int(self.cfg.capacity - self.position.max() - 1)


def reduce_over_ranks(dev_s: float, tokens: int, wall: float, device,
                      sum_tokens: bool = True) -> tuple[float, float, float]:
    """(max device seconds, total tokens, max wall seconds) over the ranks of
    the default process group (identity without one).  A tensor-parallel group
    decodes one cohort: its tokens are counted once (sum_tokens=False)."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return dev_s, float(tokens), wall
    where = f"cuda:{device}" if device is not None else "cpu"
    times = torch.tensor([dev_s, wall], dtype=torch.float64, device=where)
    total = torch.tensor([float(tokens)], dtype=torch.float64, device=where)
    dist.all_reduce(times, op=dist.ReduceOp.MAX)
    dist.all_reduce(total, op=dist.ReduceOp.SUM if sum_tokens else dist.ReduceOp.MAX)
    return float(times[0]), float(total[0]), float(times[1])


def top2_margins(logits: np.ndarray) -> list[list[float]]:
    """[steps][rows] relative gap between the two largest logits of each row
    (the near-tie rule's measure), from f32 [steps, 4, V] logits."""
    top = np.sort(np.partition(logits, -2, axis=-1)[..., -2:], axis=-1)
    scale = np.maximum(np.abs(top[..., 1]), 1e-6)
    return ((top[..., 1] - top[..., 0]) / scale).tolist()


def tp_token_check(group_outs, single_outs, tol: float = 2e-2) -> dict:
    """The tensor-parallel group's token histories against a single-GPU
    engine's on the same cohort and epochs: a row may differ only at a step
    where the single-GPU logits' top-2 margin is below ``tol`` (the near-tie
    rule); a row that differed is not compared in later epochs."""
    from scenario import find_divergence

    done: dict[int, tuple[int, int]] = {}
    compared = 0
    for epoch, (g, o) in enumerate(zip(group_outs, single_outs)):
        calls = o.model_calls
        margins = top2_margins(o.logits[:calls])
        gh, oh = g.history.copy(), o.history.copy()
        for row in done:   # rows that differed earlier: excluded from here on
            gh[:, row] = oh[:, row]
        try:
            diverged = find_divergence(gh, oh, margins, tol)
        except AssertionError as exc:
            return {"ok": False, "epochs": epoch + 1, "error": str(exc)}
        for row, step in diverged.items():
            done[row] = (epoch, step)
        compared += sum(1 for r in range(4) if r not in done)
    return {"ok": True, "epochs": len(single_outs), "rows_compared": compared,
            "near_tie_divergences": {str(r): {"epoch": e, "step": s} for r, (e, s) in done.items()}}


def timed_epochs(cohort, cfg, steps: int, device: int, world: int, tp: bool, barrier) -> dict:
    """`steps` epochs of `cohort`, bracketed by barriers, with the SM clocks
    sampled during the timed region.  Device time is the CUDA-event time of
    each epoch kernel; wall time covers the whole C-ABI call with host buffers."""
    engine = cohort.engine
    barrier()
    tokens = 0
    device_us = []
    step_bytes_total = 0
    model_calls = 0
    with ClockSampler(device) as clocks:
        wall0 = time.perf_counter()
        for _ in range(steps):
            out, inputs = cohort.step()
            executed = out.control_out[6 + 8: 6 + 12]
            tokens += int(executed.sum())
            device_us.append(out.device_us)
            model_calls += out.model_calls
            contexts0 = [int(p) for p in inputs["position"]]
            for s in range(out.model_calls):
                ctx = [c + s for c, e in zip(contexts0, executed) if e > s]
                step_bytes_total += shard_step_bytes(cfg, engine.shard, ctx) * world if tp else step_bytes(cfg, ctx)
        wall = time.perf_counter() - wall0
    barrier()
    return {"tokens": tokens, "dev_s": sum(device_us) / 1e6, "wall": wall, "bytes": step_bytes_total,
            "model_calls": model_calls, "clocks": clocks.summary()}


BOX_SCALE_PROMPT_MAX = 120


def box_scale_epochs(engine, cfg, seed: int, device: int, world: int, tp: bool, barrier, epochs: int = 3) -> dict:
    """configs[4], the box-scale variant: a fresh B=4 cohort (prompts of 2-120
    tokens, new generations on the engine's rows) decoded in K=8 greedy epochs,
    one warm-up epoch then `epochs` timed ones; the same timing as the
    headline (device time of each epoch kernel, max over ranks)."""
    sc, first = setup_cohort(engine, cfg, seed=seed, k=8, prompt_max=BOX_SCALE_PROMPT_MAX, generation_offset=100)
    cohort = Cohort(engine, cfg, sc, first)
    if cohort.room() < 8 * (epochs + 1):
        raise RuntimeError("box-scale cohort: not enough KV capacity")
    cohort.step()
    return timed_epochs(cohort, cfg, epochs, device, world, tp, barrier)


def box_scale_summary(r: dict, device, world: int, tp: bool, peak: float) -> dict:
    """Whole-box decode tok/s, µs per decode step and HBM fraction of one
    box-scale run (tokens counted once for a tensor-parallel group, summed
    over independent cohorts)."""
    t_max, tok, wall = reduce_over_ranks(r["dev_s"], r["tokens"], r["wall"], device=device if world > 1 else None,
                                         sum_tokens=not tp)
    calls = max(r["model_calls"], 1)
    gbs = r["bytes"] / t_max / 1e9
    return {"value": round(tok / t_max, 2), "unit": "tok/s", "us_per_decode_step": round(t_max * 1e6 / calls, 2),
            "e2e_value": round(tok / wall, 2), "epochs": 3,
            "roofline_frac": round(gbs / (peak * (world if tp else 1)), 4)}


def host_loop_comparison(engine, cohort, cfg, ks=(2, 4, 8), reps: int = 3) -> dict | None:
    """The reference's central comparison on this engine: a K-step resident
    epoch (one C-ABI call, one kernel) against the host-loop route (K
    decoder-ABI calls, logits copied to pinned host memory and argmaxed there,
    cruise_b200.host_loop), wall clock around each, K = 2/4/8, median of
    `reps`.  The epochs run first and the host loops continue from where they
    ended (a host loop leaves the engine's resident row state behind)."""
    import torch

    from cruise_b200.host_loop import host_loop_epoch

    if cohort.room() < 2 * reps * sum(ks):
        return None
    epoch_s = {k: [] for k in ks}
    loop_s = {k: [] for k in ks}
    loop_dev = {k: [] for k in ks}
    for k in ks:
        for _ in range(reps):
            inputs = cohort.inputs()
            inputs["control"][0] = k
            t0 = time.perf_counter()
            out = engine.run(**inputs)
            epoch_s[k].append(time.perf_counter() - t0)
            assert out.status == 0, out.status
            cohort._advance(out)
    logits = torch.empty((4, cfg.vocab), dtype=torch.float32, pin_memory=True).numpy()
    device_us = []

    def step(*a):
        result = engine.decoder_step(*a, logits_out=logits)
        device_us.append(engine.last_timing()[0])
        return result

    for k in ks:
        for _ in range(reps):
            inputs = cohort.inputs()
            inputs["control"][0] = k
            device_us.clear()
            t0 = time.perf_counter()
            history, control = host_loop_epoch(step, inputs, cfg.block_size, cfg.capacity)
            loop_s[k].append(time.perf_counter() - t0)
            loop_dev[k].append(sum(device_us) / 1e6)
            cohort._advance(OracleOutput(history, control, None, 0.0))
    result = {}
    for k in ks:
        e, h = statistics.median(epoch_s[k]), statistics.median(loop_s[k])
        result[f"k{k}"] = {"epoch_ms": round(e * 1e3, 3), "host_loop_ms": round(h * 1e3, 3),
                           "host_loop_kernel_ms": round(statistics.median(loop_dev[k]) * 1e3, 3),
                           "speedup": round(h / e, 3)}
    result["note"] = ("wall clock per epoch through the C ABI with host buffers; the host loop keeps K/V on the "
                      "device and copies 4 x V f32 logits per step to pinned host memory (the reference's runner "
                      "also copies both caches out per step)")
    return result


def workload_config(args, world: int, tp: bool) -> dict:
    """The `config` object of both arms' lines (the reference arm times the
    same workload on the CPU)."""
    return {
        "workload": "configs[1]: Qwen2.5-7B arch, B=4 all active, K=%d greedy epochs after the "
                    "one-shot H2D KV import of the prefilled prompts (2-%d tokens)" % (args.k, args.prompt_max),
        "model": "Qwen2.5-7B architecture (28 layers, hidden 3584, 28/4 heads x 128, I 18944, V 152064)",
        "global_batch": 4 if (tp or world == 1) else 4 * world,
        "epoch_k": args.k,
        "kv": "paged, block 128, 2 blocks per row",
        "parallelism": (f"tp{world} (one cohort sharded over {world} GPUs)" if tp else
                        f"dp{world} (independent cohorts)" if world > 1 else "single GPU"),
        "l2": "no flush: every step streams 14.1 GB of weights, > 126 MB L2",
    }


def run_gpu(args) -> None:
    import torch
    import torch.distributed as dist

    from cruise_b200.engine import EpochEngine
    from cruise_b200.model_config import QWEN25_7B

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=300))
    device = local
    cfg = QWEN25_7B
    if args.layers or args.vocab:
        # reduced geometry for profiler captures only (never a bench line)
        cfg = cfg.with_(num_layers=args.layers or cfg.num_layers, vocab=args.vocab or cfg.vocab,
                        configured_eos=(args.vocab or cfg.vocab) - 1)
    tp = world > 1 and not args.dp

    def barrier():
        torch.cuda.synchronize(device)
        if world > 1:
            dist.barrier()

    t0 = time.perf_counter()
    group = None
    if tp:
        # one cohort sharded over all ranks (one GPU each); the kernel exchanges
        # the row-parallel partials and the vocabulary argmax over peer memory
        from cruise_b200.tp import create_tp_engine

        group = create_tp_engine(cfg, device=device)
        group.init_synthetic(seed=0)
    single = EpochEngine(cfg, device=device)
    single.init_synthetic(seed=0)
    synth_s = time.perf_counter() - t0
    need = (args.warmup + args.steps + (1 if args.trace else 0) + (1 if args.trace_cta else 0)) * args.k

    # the single-GPU cohort of this rank (seed 1000 + rank; rank 0's is the tensor-parallel cohort)
    check_logits = tp and rank == 0
    sc, first_single = setup_cohort(single, cfg, seed=1000 + rank, k=args.k, prompt_max=args.prompt_max,
                                    want_logits=check_logits)
    single_cohort = Cohort(single, cfg, sc, first_single)
    if single_cohort.room() < need:
        raise RuntimeError(f"capacity {cfg.capacity} too small for {need} more positions")
    single_warm = [single_cohort.step(want_logits=check_logits)[0] for _ in range(args.warmup)]
    if tp:
        sc_tp, first_tp = setup_cohort(group, cfg, seed=1000, k=args.k, prompt_max=args.prompt_max)
        tp_cohort = Cohort(group, cfg, sc_tp, first_tp)
        tp_warm = [tp_cohort.step()[0] for _ in range(args.warmup)]

    # ---- timed regions: device-resident epochs ----
    runs = {}
    if tp:
        runs["tp"] = timed_epochs(tp_cohort, cfg, args.steps, device, world, True, barrier)
    runs["single"] = timed_epochs(single_cohort, cfg, args.steps, device, world, False, barrier)
    head = runs["tp"] if tp else runs["single"]
    t_max, tok_total, e2e_wall = reduce_over_ranks(head["dev_s"], head["tokens"], head["wall"],
                                                   device=device if world > 1 else None, sum_tokens=not tp)
    if args.trace and (rank == 0 or tp):
        # a tensor-parallel group runs the traced epoch on every rank
        print_trace(group if tp else single, tp_cohort if tp else single_cohort, cfg, args.k, show=rank == 0)
    if args.trace_cta and (rank == 0 or tp):
        print_trace_cta(group if tp else single, tp_cohort if tp else single_cohort, cfg, show=rank == 0)
    dp = None
    if tp:
        d = runs["single"]
        dp_t, dp_tok, dp_wall = reduce_over_ranks(d["dev_s"], d["tokens"], d["wall"], device=device)
        dp = {"value": round(dp_tok / dp_t, 2), "unit": "tok/s", "scaling": "weak",
              "ms_per_step": round(dp_t * 1e3 / args.steps, 4), "global_batch": 4 * world,
              "e2e_value": round(dp_tok / dp_wall, 2),
              "note": "every rank an independent B=4 cohort on its own full-model engine, tokens summed"}
    peak, peak_kind = hbm_peak()
    per_epoch_us = t_max * 1e6 / args.steps
    achieved_gbs = head["bytes"] / (t_max if tp else head["dev_s"]) / 1e9
    if tp:
        peak = peak * world   # the group's aggregate HBM bandwidth
    value = tok_total / t_max
    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": "tok/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(per_epoch_us / 1e3, 4),
            "us_per_decode_step": round(per_epoch_us / args.k, 2),
            "higher_is_better": True,
            "scaling": "strong" if tp else "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded random-init weights generated on the device; seeded prompts)",
            "config": workload_config(args, world, tp),
            "roofline": {
                "bound": "hbm",
                "achieved": round(achieved_gbs, 1),
                "peak": peak,
                "peak_kind": f"{peak_kind}, x{world} GPUs (aggregate)" if tp else peak_kind,
                "unit": "GB/s",
                "frac": round(achieved_gbs / peak, 4),
                # the second denominator the north star asks for: nominal 8 TB/s per GPU
                "frac_of_nominal_8tbs": round(achieved_gbs / (8000.0 * (world if tp else 1)), 4),
                "logits": "not materialised (argmax fused into the lm_head phase): 0 of the 4 x V x 4 B = "
                          "2,433,024 B per step a materialising step would add",
                "traffic": (PROFILED_TRAFFIC["bytes_per_launch"] // PROFILED_TRAFFIC["steps_per_launch"]
                            if args.k == PROFILED_TRAFFIC["k"] and not args.layers and not args.vocab and not tp
                            else None),
                "traffic_unit": "bytes per decode step (ncu dram read + write)",
                "kernel": "resident_epoch_kernel",
                "bytes_per_decode_step": head["bytes"] // max(head["model_calls"], 1),
            },
            "e2e": {
                "value": round(tok_total / e2e_wall, 2),
                "unit": "tok/s",
                "h2d_bytes_per_step": EPOCH_H2D_BYTES,
                "d2h_bytes_per_step": EPOCH_D2H_BYTES,
                "host_control_ms_per_epoch": round(e2e_wall * 1e3 / args.steps, 4),
            },
            "gpu_launches": args.steps * world,   # one epoch kernel per step on every rank
            "clocks": head["clocks"],
            "setup": {"weight_synthesis_s": round(synth_s, 2)},
        }
        if tp:
            line["tp_check"] = tp_token_check([first_tp, *tp_warm], [first_single, *single_warm])
            line["dp"] = dp
    # configs[4] on the same GPUs: K=8, prompts of 2-120 tokens; a
    # tensor-parallel group decodes one cohort, the single-GPU engines one
    # cohort each (the data-parallel layout).  New cohorts take over the
    # engines' rows, so this runs after everything that continues the
    # headline cohorts.
    box_scale = not (args.layers or args.vocab or args.no_box_scale)
    box = {"workload": "configs[4]: B=4 per cohort, K=8 greedy epochs after prompts of 2-%d tokens"
                       % BOX_SCALE_PROMPT_MAX}
    if tp and box_scale:
        r = box_scale_epochs(group, cfg, 3000, device, world, True, barrier)
        box["tp"] = box_scale_summary(r, device, world, True, hbm_peak()[0])
    if tp:
        group.close()
    if rank == 0 and world == 1 and args.k != 8 and not (args.layers or args.vocab) and single_cohort.room() >= 40:
        # the same cohort in five K=8 epochs: the north star's epoch length
        k_default, single_cohort.sc.k = single_cohort.sc.k, 8
        r8 = timed_epochs(single_cohort, cfg, 5, device, 1, False, barrier)
        single_cohort.sc.k = k_default
        gbs8 = r8["bytes"] / r8["dev_s"] / 1e9
        line["k8"] = {"value": round(r8["tokens"] / r8["dev_s"], 2), "unit": "tok/s", "epochs": 5,
                      "us_per_decode_step": round(r8["dev_s"] * 1e6 / max(r8["model_calls"], 1), 2),
                      "roofline_frac": round(gbs8 / peak, 4), "e2e_value": round(r8["tokens"] / r8["wall"], 2)}
    if rank == 0 and world == 1 and not args.no_host_loop and not (args.layers or args.vocab):
        line["host_loop"] = host_loop_comparison(single, single_cohort, cfg)
    if box_scale:
        r = box_scale_epochs(single, cfg, 3000 + rank, device, world, False, barrier)
        box["dp" if world > 1 else "single"] = box_scale_summary(r, device, world, False, hbm_peak()[0])
        if rank == 0:
            line["box_scale"] = box
    if rank == 0 and not args.no_cpu_baseline and world == 1:
        line["cpu_baseline"] = cpu_baseline(cfg, args, first_single)
    if rank == 0:
        print(json.dumps(line), flush=True)
    single.close()
    if world > 1:
        dist.destroy_process_group()


# grid barriers per layer: QKV and attention share one (attention units wait
# for their KV head's QKV row groups), then O, gate/up, down
PHASE_NAMES = ("qkv+attention", "o_proj", "gate_up", "down")
PHASES_PER_LAYER = len(PHASE_NAMES)


def print_trace_cta(engine, cohort, cfg, show: bool = True) -> None:
    """One traced epoch with every CTA's phase marks: per phase kind, summed
    over layers and steps (us per decode step), the medians over CTAs of
    activation staging, tile stream and epilogue, the spread of the arrivals
    (last CTA minus median), the release (first and last CTA out minus last
    in), and the CTAs that arrived last most often."""
    engine.set_trace(2)
    out, _ = cohort.step()
    engine.set_trace(False)
    L = cfg.num_layers
    phases = PHASES_PER_LAYER * L + 2
    count = 2 + out.model_calls * phases + 1
    raw = engine.read_trace_cta(count).astype(np.int64)
    # unwrap the 32-bit stamps against barrier 1's exit of CTA 0
    base = raw[1, 0, 0]
    t = np.where(raw == 0, 0, (raw - base) % (1 << 32))
    first = 2
    acc, last_cta = {}, {}
    for step in range(out.model_calls):
        for ph in range(phases):
            j = first + step * phases + ph + 1
            name = ("lm_head" if ph == PHASES_PER_LAYER * L else "control" if ph > PHASES_PER_LAYER * L
                    else PHASE_NAMES[ph % PHASES_PER_LAYER])
            a = acc.setdefault(name, np.zeros(18))
            start, staged, tiles, arrive = t[j - 1, :, 0], t[j, :, 1], t[j, :, 2], t[j, :, 3]
            e_start, e_done, e_fenced = t[j, :, 4], t[j, :, 6], t[j, :, 7]
            if e_done.any():
                last_flush, warps_done = t[j, :, 8], t[j, :, 9]
                a[12] += np.median(warps_done - tiles)
                a[13] += np.median(last_flush - warps_done)
                a[14] += np.median(e_done - last_flush)
                a[8] += np.median(e_start - start)
                a[9] += np.median(raw[j, :, 5])
                a[10] += np.median(e_done - tiles)
                a[11] += np.median(e_fenced - e_done)
            exit_ = t[j, :, 0]
            a[0] += np.median(exit_) - np.median(start)
            if staged.any():
                loaded, shared = t[j, :, 10], t[j, :, 11]
                if loaded.any():
                    a[15] += np.median(loaded - start)
                    a[16] += np.median(shared - loaded)
                    a[17] += np.median(staged - shared)
                a[1] += np.median(staged - start)
                a[2] += np.median(tiles - staged)
                a[3] += np.median(arrive - tiles)
            else:
                a[3] += np.median(arrive - start)
            a[4] += arrive.max() - np.median(arrive)
            a[5] += exit_.min() - arrive.max()
            a[6] += exit_.max() - arrive.max()
            a[7] += start.max() - start.min()
            lc = last_cta.setdefault(name, {})
            c = int(arrive.argmax())
            lc[c] = lc.get(c, 0) + 1
    if not show:
        return
    calls = out.model_calls
    print(f"per-CTA trace: epoch {out.device_us:.1f} us, {calls} steps, {raw.shape[1]} CTAs; per step, us "
          f"[phase | med staging  med tiles  med epilogue | last-arrival lag | release first/last | start skew]"
          f"  last CTAs\n    epilogue warp, medians over CTAs: [start after phase start | partner wait | "
          f"last segment after last tile | fence]", file=sys.stderr)
    for name in (*PHASE_NAMES, "lm_head", "control"):
        a = acc.get(name, np.zeros(18)) / calls / 1e3
        top = sorted(last_cta.get(name, {}).items(), key=lambda kv: -kv[1])[:4]
        print(f"  {name:13s} {a[0]:8.1f} | {a[1]:7.1f} {a[2]:7.1f} {a[3]:7.1f} | {a[4]:7.1f} | {a[5]:6.1f} {a[6]:6.1f} "
              f"| {a[7]:6.1f}  {top}\n  {'':9s} {'':8s}   epilogue warp: {a[8]:7.1f} | {a[9]:7.1f} | {a[10]:7.1f} | "
              f"{a[11]:7.1f} || slowest consumer warp after warp 0: {a[12]:6.1f}, last flush taken after that: "
              f"{a[13]:6.1f}, last segment's epilogue: {a[14]:6.1f}"
              + (f"\n  {'':9s} {'':8s}   norm staging: loads {a[15]:6.1f}, sum of squares shared {a[16]:6.1f}, "
                 f"normalised {a[17]:6.1f}" if a[15] else ""), file=sys.stderr)


def print_trace(engine, cohort, cfg, k, show: bool = True) -> None:
    """One traced epoch: per phase kind, the time between grid barriers and its
    parts on CTA 0 (activation staging, tile stream, epilogue drain, wait for the
    last CTA, barrier release; under tensor parallelism also how much of the
    epilogue waited for the other ranks' partials), summed over layers and steps."""
    engine.set_trace(True)
    out, _ = cohort.step()
    engine.set_trace(False)
    L = cfg.num_layers
    phases = PHASES_PER_LAYER * L + 2
    count = 2 + out.model_calls * phases + 1
    tr = engine.read_trace(count).astype(np.int64)
    exit_ns, entry_ns, xready, tiles, last, tp_wait = tr
    end_ns = exit_ns   # a phase ends when CTA 0 leaves its grid barrier
    first = 2   # validation and continuity barriers precede the loop
    acc = {}
    for step in range(out.model_calls):
        for ph in range(phases):
            j = first + step * phases + ph + 1
            name = ("lm_head" if ph == PHASES_PER_LAYER * L else "control" if ph > PHASES_PER_LAYER * L
                    else PHASE_NAMES[ph % PHASES_PER_LAYER])
            a = acc.setdefault(name, np.zeros(7))
            start = end_ns[j - 1]
            a[0] += end_ns[j] - start
            if xready[j]:
                a[1] += xready[j] - start
                a[2] += tiles[j] - xready[j]
                a[3] += entry_ns[j] - tiles[j]
            else:
                a[3] += entry_ns[j] - start
            a[4] += max(last[j] - entry_ns[j], 0)
            a[5] += exit_ns[j] - max(last[j], entry_ns[j])
            a[6] += tp_wait[j]   # part of the epilogue: waiting for other ranks' partials
    if not show:
        return
    sh, h, d = engine.shard, cfg.hidden, cfg.head_dim   # this rank's shard (the whole model on one GPU)
    wbytes = {"qkv+attention": (sh.nq + 2 * sh.nkv) * d * h * 2 * L, "o_proj": h * sh.nq * d * 2 * L,
              "gate_up": 2 * sh.ni * h * 2 * L, "down": h * sh.ni * 2 * L, "lm_head": sh.nv * h * 2}
    calls = out.model_calls
    print(f"trace: epoch {out.device_us:.1f} us, {calls} steps; per step, us "
          f"[total | x-staging  tiles  epilogue | wait-last-CTA  release | epilogue tp-wait] and weight GB/s",
          file=sys.stderr)
    for name in (*PHASE_NAMES, "lm_head", "control"):
        a = acc.get(name, np.zeros(7)) / calls / 1e3
        bw = wbytes.get(name, 0) / (a[0] * 1e3) if name in wbytes and a[0] else 0.0
        print(f"  {name:13s} {a[0]:8.1f} | {a[1]:7.1f} {a[2]:7.1f} {a[3]:7.1f} | {a[4]:7.1f} {a[5]:7.1f} "
              f"{a[6]:7.1f}   {bw:6.0f}", file=sys.stderr)


@dataclass
class OracleOutput:
    history: np.ndarray
    control_out: np.ndarray
    logits: None
    device_us: float   # wall-clock time of the oracle epoch

    @property
    def status(self) -> int:
        return int(self.control_out[3])

    @property
    def model_calls(self) -> int:
        return int(self.control_out[4])


class OracleEngine:
    """The CPU oracle (the reference's decode step and epoch controller, ported
    to torch CPU) behind the engine's run / read_kv surface, with the engine's
    seeded weights at full depth.  Used by the CPU legs of this benchmark only."""

    def __init__(self, cfg, threads: int) -> None:
        import torch

        from cruise_b200.model_config import TpShard
        from oracle.decoder import OracleDecoder
        from oracle.epoch import OracleEpochController
        from oracle.model import OracleConfig, seeded_weights

        torch.set_num_threads(threads)
        self.config = cfg
        self.shard = TpShard.of(cfg, 0, 1)
        ocfg = OracleConfig(num_layers=cfg.num_layers, hidden=cfg.hidden, num_heads=cfg.num_heads,
                            num_kv_heads=cfg.num_kv_heads, head_dim=cfg.head_dim, intermediate=cfg.intermediate,
                            vocab=cfg.vocab, block_size=cfg.block_size, blocks_per_row=cfg.blocks_per_row,
                            num_blocks=cfg.num_blocks)
        t0 = time.perf_counter()
        weights = seeded_weights(ocfg, seed=0, use_c=True)
        self.synth_s = time.perf_counter() - t0
        self.controller = OracleEpochController(OracleDecoder(ocfg, weights))

    def run(self, import_payload=None, forced=None, want_logits=False, **inputs) -> OracleOutput:
        t0 = time.perf_counter()
        history, control = self.controller.run(**inputs, import_payload=import_payload, forced=forced)
        return OracleOutput(history, control, None, (time.perf_counter() - t0) * 1e6)

    def read_kv(self):
        return self.controller.key, self.controller.value


def oracle_epochs(cfg, k: int, prompt_max: int, warmup: int, steps: int, threads: int) -> dict:
    """Whole greedy epochs of the CPU oracle on the benchmark's cohort (seed
    1000): prefill and the import epoch untimed, `warmup` untimed epochs, then
    `steps` epochs each timed with perf_counter around the whole controller."""
    engine = OracleEngine(cfg, threads)
    sc, first = setup_cohort(engine, cfg, seed=1000, k=k, prompt_max=prompt_max)
    cohort = Cohort(engine, cfg, sc, first)
    for _ in range(warmup):
        cohort.step()
    tokens, seconds, calls = 0, 0.0, 0
    for _ in range(steps):
        out, _ = cohort.step()
        tokens += int(out.control_out[6 + 8: 6 + 12].sum())
        seconds += out.device_us / 1e6
        calls += out.model_calls
    return {"tokens": tokens, "seconds": seconds, "model_calls": calls, "import_history": first.history,
            "synth_s": engine.synth_s}


def cpu_baseline(cfg, args, gpu_first) -> dict:
    """The oracle on the GPU box's host cores, a bounded sample of the same
    workload: 1 warm-up epoch and 3 timed epochs after the import epoch."""
    threads = len(os.sched_getaffinity(0))
    r = oracle_epochs(cfg, args.k, args.prompt_max, warmup=1, steps=3, threads=threads)
    return {"value": round(r["tokens"] / r["seconds"], 3), "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"3 whole K={args.k} epochs of the 28-layer oracle (torch CPU, bf16) after the import "
                      f"epoch and 1 warm-up epoch, same seeded weights and cohort, {threads} threads",
            "ms_per_epoch": round(r["seconds"] * 1e3 / 3, 1),
            "us_per_decode_step": round(r["seconds"] * 1e6 / max(r["model_calls"], 1), 1),
            "import_epoch_tokens_equal_gpu": bool(np.array_equal(r["import_history"], gpu_first.history))}


def run_reference(args) -> None:
    """CPU arm: the oracle port of the reference path on the host cores, whole
    epochs of the same workload (rank 0 only under torchrun)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from cruise_b200.model_config import QWEN25_7B

    cfg = QWEN25_7B
    threads = len(os.sched_getaffinity(0))
    r = oracle_epochs(cfg, args.k, args.prompt_max, warmup=args.warmup, steps=args.steps, threads=threads)
    value = r["tokens"] / r["seconds"]
    sample = (f"{args.steps} whole K={args.k} epochs of the 28-layer oracle (torch CPU, bf16) after the import "
              f"epoch and {args.warmup} warm-up epochs, {threads} threads")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "tok/s", "n_gpus": 0,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(r["seconds"] * 1e3 / args.steps, 2),
        "us_per_decode_step": round(r["seconds"] * 1e6 / max(r["model_calls"], 1), 1), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded random-init weights, the GPU arm's; seeded prompts)",
        "config": workload_config(args, int(os.environ.get("WORLD_SIZE", "1")),
                                  int(os.environ.get("WORLD_SIZE", "1")) > 1 and not args.dp),
        "cpu_baseline": {"value": round(value, 3), "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "setup": {"weight_synthesis_s": round(r["synth_s"], 2)},
    }
    print(json.dumps(line), flush=True)


def forced_epochs_all_rows(sc, cfg, generation_offset: int):
    """Teacher-forced epochs writing the KV of every prompt token but the last,
    all rows of the cohort in the same epochs.  An epoch runs as many steps as
    the row with the fewest positions left (at most 8), so no row runs past its
    prompt; rows that are done drop out."""
    from scenario import BATCH, MAX_STEPS, compute_slot

    eos = next(t for t in range(cfg.vocab - 1, -1, -1) if all(t not in p for p in sc.prompts))
    gens = [g + generation_offset if g else 0 for g in sc.generations]
    done = [0] * BATCH
    while True:
        left = {r: len(p) - 1 - done[r] for r, p in enumerate(sc.prompts) if p and len(p) - 1 > done[r]}
        if not left:
            return
        steps = min(MAX_STEPS, min(left.values()))
        token = np.zeros(BATCH, dtype=np.int64)
        position = np.zeros(BATCH, dtype=np.int64)
        seq_len = np.zeros(BATCH, dtype=np.int32)
        active = np.zeros(BATCH, dtype=np.int32)
        forced = np.full((MAX_STEPS, BATCH), -1, dtype=np.int64)
        for row in left:
            prompt, d = sc.prompts[row], done[row]
            token[row], position[row], seq_len[row], active[row] = prompt[d], d, d + 1, 1
            forced[:steps, row] = prompt[d + 1: d + 1 + steps]
            done[row] += steps
        slot = np.array([compute_slot(sc.block_table, cfg.block_size, r, int(position[r])) for r in range(BATCH)],
                        dtype=np.int32)
        row_gens = [gens[r] if active[r] else 0 for r in range(BATCH)]
        control = np.array([steps, eos, eos, eos, eos, 0, 0, *row_gens], dtype=np.int32)
        yield dict(token=token, position=position, seq_len=seq_len, slot=slot, active=active,
                   block_table=sc.block_table.reshape(-1), control=control, forced=forced)


def run_prefill(args) -> None:
    """Prefill of a 4-row cohort of 120-token prompts on the 7B model: the
    batched device prefill (cruise_epoch_prefill + the import epoch) against the
    teacher-forced prefill epochs (one token per row per step).  Prints one
    JSON line; not part of the default decode benchmark."""
    import torch

    from cruise_b200.engine import EpochEngine
    from cruise_b200.model_config import QWEN25_7B
    from scenario import decode_inputs, make_scenario

    cfg = QWEN25_7B
    if args.layers or args.vocab:
        # reduced geometry for profiler captures only (never a bench line)
        cfg = cfg.with_(num_layers=args.layers or cfg.num_layers, vocab=args.vocab or cfg.vocab,
                        configured_eos=(args.vocab or cfg.vocab) - 1)
    engine = EpochEngine(cfg)
    engine.init_synthetic(seed=0)
    length = 120
    sc = make_scenario(vocab=cfg.vocab, seed=77, active_rows=(1, 1, 1, 1), prompt_len=(length, length), k=2,
                       budget=(2, 2), eos=cfg.configured_eos, token_high=min(151643, cfg.vocab - 1))
    tokens = sum(len(p) - 1 for p in sc.prompts)
    engine.prefill(sc.prompts)   # first call allocates the activation buffers
    batched = []
    with ClockSampler(0) as clocks:
        for _ in range(max(3, args.steps)):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            engine.prefill(sc.prompts)
            batched.append((time.perf_counter() - t0) * 1e3)
    out = engine.run(**decode_inputs(sc, cfg.block_size, importing=True))
    assert out.status == 0, out.status
    # the same prompts again as teacher-forced epochs (all four rows together,
    # 8 tokens per row per epoch), under new generations
    forced_dev, forced_wall = 0.0, time.perf_counter()
    epochs = 0
    for inputs in forced_epochs_all_rows(sc, cfg, generation_offset=10):
        o = engine.run(**inputs)
        assert o.status == 0, o.status
        forced_dev += o.device_us / 1e3
        epochs += 1
    forced_wall = (time.perf_counter() - forced_wall) * 1e3
    engine.close()
    ms = statistics.median(batched)
    print(json.dumps({
        "metric": "prefill of a B=4 cohort of 120-token prompts (7B arch), ms", "unit": "ms",
        "higher_is_better": False, "data": "synthetic (seeded weights and prompts)", "dtype": "bf16",
        "batched_device_prefill_ms": round(ms, 3), "prompt_tokens_prefilled": tokens,
        "batched_tok_per_s": round(tokens / ms * 1e3, 1),
        "teacher_forced_epochs": epochs, "teacher_forced_device_ms": round(forced_dev, 3),
        "teacher_forced_wall_ms": round(forced_wall, 3), "speedup_vs_teacher_forced": round(forced_wall / ms, 1),
        "batched_includes": "host token upload, all layers (tcgen05 GEMMs + prefill kernels), sync",
        "clocks": clocks.summary(),
    }), flush=True)


def run_serve(args) -> None:
    """Serving through vLLM's own front end (``LLM.generate``, engine core in
    this process) with the resident epoch scheduler, the dedicated worker and
    the 7B engine, device prefill on: B = 4 requests with seeded prompts of
    2-120 tokens, greedy, ``max_tokens`` each, all submitted together.  One
    warm-up generate, then ``--steps`` timed ones (at least 3).  Prints one
    JSON line: output tokens per second of wall time around ``generate``
    (prefill, every epoch and vLLM's own scheduling and output processing
    included) and the wall time per output step.  Not part of the default
    decode benchmark."""
    import tempfile

    for name, value in (("VLLM_ASCEND_RESIDENT_EPOCH_BACKEND_FACTORY", "cruise_b200.cuda_backend:create_cuda_engine"),
                        ("VLLM_ASCEND_RESIDENT_EPOCH_MODEL", "qwen2.5-7b"),
                        ("VLLM_ASCEND_RESIDENT_EPOCH_EXTERNAL_WEIGHTS", "synthetic:0"),
                        ("VLLM_ASCEND_RESIDENT_EPOCH_DEVICE_PREFILL", "1"),
                        ("VLLM_ENABLE_V1_MULTIPROCESSING", "0")):
        os.environ[name] = value
    from vllm import LLM, SamplingParams

    from cruise_b200.model_config import QWEN25_7B

    cfg = QWEN25_7B
    model_dir = Path(tempfile.mkdtemp(prefix="cruise-serve-"))
    (model_dir / "config.json").write_text(json.dumps({
        "architectures": ["Qwen2ForCausalLM"], "model_type": "qwen2", "hidden_size": cfg.hidden,
        "intermediate_size": cfg.intermediate, "num_hidden_layers": cfg.num_layers,
        "num_attention_heads": cfg.num_heads, "num_key_value_heads": cfg.num_kv_heads,
        "vocab_size": cfg.vocab, "max_position_embeddings": 32768, "rms_norm_eps": 1e-6,
        "rope_theta": 1000000.0, "torch_dtype": "bfloat16", "tie_word_embeddings": False,
        "hidden_act": "silu", "eos_token_id": cfg.configured_eos,
    }))
    (model_dir / "generation_config.json").write_text(json.dumps({"eos_token_id": cfg.configured_eos}))
    rng = np.random.default_rng(2026)
    prompts = [rng.integers(0, 151643, size=int(rng.integers(2, 121))).tolist() for _ in range(4)]
    max_tokens = 128
    t0 = time.perf_counter()
    llm = LLM(model=str(model_dir), skip_tokenizer_init=True, max_model_len=cfg.capacity,
              block_size=cfg.block_size, max_num_seqs=4, async_scheduling=False, enforce_eager=True,
              dtype="bfloat16", enable_prefix_caching=False, worker_cls="cruise_b200.worker.ResidentEpochWorker",
              scheduler_cls="cruise_b200.scheduler.ResidentEpochScheduler")
    setup_s = time.perf_counter() - t0
    try:
        params = SamplingParams(temperature=0.0, max_tokens=max_tokens, detokenize=False)
        llm.generate([{"prompt_token_ids": p[:8]} for p in prompts], SamplingParams(
            temperature=0.0, max_tokens=16, detokenize=False), use_tqdm=False)
        walls, tokens = [], []
        for _ in range(max(3, args.steps)):
            t0 = time.perf_counter()
            outs = llm.generate([{"prompt_token_ids": p} for p in prompts], params, use_tqdm=False)
            walls.append(time.perf_counter() - t0)
            tokens.append(sum(len(o.outputs[0].token_ids) for o in outs))
    finally:
        llm.llm_engine.engine_core.shutdown()
    wall = statistics.median(walls)
    produced = tokens[walls.index(wall)] if wall in walls else tokens[-1]
    print(json.dumps({
        "metric": "vLLM LLM.generate on the resident engine (7B arch, B=4, greedy), output tok/s", "unit": "tok/s",
        "higher_is_better": True, "data": "synthetic (seeded weights and prompts)", "dtype": "bf16",
        "value": round(produced / wall, 1), "wall_ms": round(wall * 1e3, 2), "output_tokens": produced,
        "ms_per_output_step": round(wall * 1e3 / max_tokens, 3), "requests": 4, "max_tokens": max_tokens,
        "prompt_tokens": [len(p) for p in prompts], "repeats": len(walls), "engine_setup_s": round(setup_s, 1),
        "path": "LLM.generate -> ResidentEpochScheduler (device prefill, K<=8 epochs) -> ResidentEpochWorker -> "
                "resident_epoch_prefill / resident_epoch_execute",
    }), flush=True)


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=20)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--k", type=int, default=2, choices=(1, 2, 4, 8))
    parser.add_argument("--impl", default="cruise", choices=("cruise", "reference"))
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-box-scale", action="store_true",
                        help="skip the configs[4] figure (K=8 epochs after prompts of 2-120 tokens)")
    parser.add_argument("--no-host-loop", action="store_true",
                        help="skip the resident-epoch vs host-loop comparison (N=1)")
    parser.add_argument("--trace", action="store_true", help="per-phase timing of one extra epoch (stderr)")
    parser.add_argument("--trace-cta", action="store_true",
                        help="every CTA's phase marks of one extra epoch, summarised (stderr)")
    parser.add_argument("--layers", type=int, default=0, help="profiling only: truncate the model to N layers")
    parser.add_argument("--vocab", type=int, default=0, help="profiling only: vocabulary size")
    parser.add_argument("--tp", action="store_true",
                        help="under torchrun: the ranks form one tensor-parallel group (the default)")
    parser.add_argument("--dp", action="store_true",
                        help="under torchrun: headline = independent data-parallel cohorts, no tensor parallelism")
    parser.add_argument("--prompt-max", type=int, default=5,
                        help="longest prompt of the seeded cohort (2..block_size; configs[4] uses 120)")
    parser.add_argument("--prefill", action="store_true",
                        help="measure the batched device prefill instead of the decode epochs")
    parser.add_argument("--serve", action="store_true",
                        help="measure serving through vLLM's LLM.generate (device prefill + resident epochs)")
    args = parser.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.serve:
        run_serve(args)
    elif args.prefill:
        run_prefill(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
