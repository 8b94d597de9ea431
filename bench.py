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
         the epoch kernel on its own stream), max over ranks, all ranks summed.
e2e      the same through the C-ABI call with host buffers: H2D of the epoch
         inputs and D2H of the token history + control output inside the timed
         wall-clock region.
--impl reference  times the CPU oracle (a port of the reference's torch decode
         step and controller, the reference path itself needs Ascend hardware)
         on the host cores on a bounded sample of the same workload.

Multi-GPU (torchrun): each rank runs an independent B=4 cohort on its own GPU
(data-parallel replicas, no collective on the data path); the process group is
only used for the start/stop barrier and the max-over-ranks timing.
With --tp the N ranks instead form one tensor-parallel group decoding a single
B=4 cohort (strong scaling): each GPU streams its 1/N of the weights and the
epoch kernel exchanges the O / down partials and the vocabulary argmax over
NVLink peer memory; value counts the cohort's tokens once, and the roofline
compares the group's shard bytes with N x the per-GPU HBM peak.

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


def setup_cohort(engine, cfg, seed: int, k: int, prompt_max: int = 5):
    """Device prefill of a seeded B=4 cohort, then the one-shot import epoch."""
    from scenario import decode_inputs, import_payload, make_scenario, prefill_epochs

    sc = make_scenario(vocab=cfg.vocab, seed=seed, active_rows=(1, 1, 1, 1), prompt_len=(2, prompt_max),
                       budget=(2, 8), k=k, eos=cfg.configured_eos, token_high=min(151643, cfg.vocab - 1))
    for inputs in prefill_epochs(sc, cfg.block_size, cfg.vocab):
        out = engine.run(**inputs)
        assert out.status == 0, f"prefill epoch status {out.status}"
    key, value = engine.read_kv()
    if engine.shard.size > 1:
        key, value = gather_kv_shards(engine, key, value)
    payload = import_payload(key, value, sc)
    inputs = decode_inputs(sc, cfg.block_size, importing=True)
    out = engine.run(**inputs, import_payload=payload)
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

    def step(self):
        inputs = self.inputs()
        out = self.engine.run(**inputs)
        if out.status != 0:
            raise RuntimeError(f"epoch status {out.status}")
        self._advance(out)
        return out, inputs

    def room(self) -> int:
        return int(self.cfg.capacity - self.position.max() - 1)


def reduce_over_ranks(dev_s: float, tokens: int, wall_s: float, device,
                      sum_tokens: bool = True) -> tuple[float, float, float]:
    """(max device seconds, total tokens, max wall seconds) over the ranks of
    the default process group (identity without one).  A tensor-parallel group
    decodes one cohort: its tokens are counted once (sum_tokens=False)."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return dev_s, float(tokens), wall_s
    where = f"cuda:{device}" if device is not None else "cpu"
    times = torch.tensor([dev_s, wall_s], dtype=torch.float64, device=where)
    total = torch.tensor([float(tokens)], dtype=torch.float64, device=where)
    dist.all_reduce(times, op=dist.ReduceOp.MAX)
    dist.all_reduce(total, op=dist.ReduceOp.SUM if sum_tokens else dist.ReduceOp.MAX)
    return float(times[0]), float(total[0]), float(times[1])


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
    tp = args.tp and world > 1
    if tp:
        # one cohort sharded over all ranks (one GPU each); the kernel exchanges
        # the row-parallel partials and the vocabulary argmax over peer memory
        from cruise_b200.tp import create_tp_engine

        engine = create_tp_engine(cfg, device=device)
    else:
        engine = EpochEngine(cfg, device=device)
    t0 = time.perf_counter()
    engine.init_synthetic(seed=0)
    synth_s = time.perf_counter() - t0
    sc, first = setup_cohort(engine, cfg, seed=1000 + (0 if tp else rank), k=args.k, prompt_max=args.prompt_max)
    cohort = Cohort(engine, cfg, sc, first)
    need = (args.warmup + args.steps + (1 if args.trace else 0)) * args.k
    if cohort.room() < need:
        raise RuntimeError(f"capacity {cfg.capacity} too small for {need} more positions")
    for _ in range(args.warmup):
        cohort.step()

    def barrier():
        torch.cuda.synchronize(device)
        if world > 1:
            dist.barrier()

    # ---- timed region: device-resident epochs (value) ----
    barrier()
    tokens = 0
    device_us = []
    step_bytes_total = 0
    with ClockSampler(device) as clocks:
        wall0 = time.perf_counter()
        for _ in range(args.steps):
            out, inputs = cohort.step()
            executed = out.control_out[6 + 8 : 6 + 12]
            tokens += int(executed.sum())
            device_us.append(out.device_us)
            contexts0 = [int(p) for p in inputs["position"]]
            for s in range(out.model_calls):
                ctx = [c + s for c, e in zip(contexts0, executed) if e > s]
                step_bytes_total += shard_step_bytes(cfg, engine.shard, ctx) * world if tp else step_bytes(cfg, ctx)
        wall = time.perf_counter() - wall0
    barrier()
    dev_s = sum(device_us) / 1e6
    model_calls = args.steps * args.k
    t_max, tok_total, e2e_wall = reduce_over_ranks(dev_s, tokens, wall, device=device if world > 1 else None,
                                                   sum_tokens=not tp)
    value = tok_total / t_max
    e2e_tokens = tok_total
    if args.trace and (rank == 0 or tp):
        # a tensor-parallel group runs the traced epoch on every rank
        print_trace(engine, cohort, cfg, args.k, show=rank == 0)
    peak, peak_kind = hbm_peak()
    per_epoch_us = t_max * 1e6 / args.steps
    achieved_gbs = step_bytes_total / (t_max if tp else dev_s) / 1e9
    if tp:
        peak = peak * world   # the group's aggregate HBM bandwidth
    clock = clocks.summary()
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
            "config": {
                "workload": "configs[1]: Qwen2.5-7B arch, B=4 all active, K=%d greedy epochs after the "
                            "one-shot H2D KV import of the device-prefilled prompts (2-%d tokens)"
                            % (args.k, args.prompt_max),
                "model": "Qwen2.5-7B architecture (28 layers, hidden 3584, 28/4 heads x 128, I 18944, V 152064)",
                "global_batch": 4 if tp else 4 * world,
                "epoch_k": args.k,
                "kv": "paged, block 128, 2 blocks per row",
                "parallelism": (f"tp{world} (one cohort sharded over {world} GPUs)" if tp else
                                f"dp{world} (independent cohorts)" if world > 1 else "single GPU"),
                "l2": "no flush: every step streams 14.1 GB of weights, > 126 MB L2",
            },
            "roofline": {
                "bound": "hbm",
                "achieved": round(achieved_gbs, 1),
                "peak": peak,
                "peak_kind": f"{peak_kind}, x{world} GPUs (aggregate)" if tp else peak_kind,
                "unit": "GB/s",
                "frac": round(achieved_gbs / peak, 4),
                "traffic": (PROFILED_TRAFFIC["bytes_per_launch"] // PROFILED_TRAFFIC["steps_per_launch"]
                            if args.k == PROFILED_TRAFFIC["k"] and not args.layers and not args.vocab and not tp
                            else None),
                "traffic_unit": "bytes per decode step (ncu dram read + write)",
                "kernel": "resident_epoch_kernel",
                "bytes_per_decode_step": step_bytes_total // model_calls,
            },
            "e2e": {
                "value": round(e2e_tokens / e2e_wall, 2),
                "unit": "tok/s",
                "h2d_bytes_per_step": EPOCH_H2D_BYTES,
                "d2h_bytes_per_step": EPOCH_D2H_BYTES,
                "host_control_ms_per_epoch": round(wall * 1e3 / args.steps, 4),
            },
            "gpu_launches": args.steps * world,   # one epoch kernel per step on every rank
            "clocks": clock,
            "setup": {"weight_synthesis_s": round(synth_s, 2)},
        }
        if not args.no_cpu_baseline and world == 1:
            line["cpu_baseline"] = cpu_baseline(engine, cfg)
        print(json.dumps(line), flush=True)
    engine.close()
    if world > 1:
        dist.destroy_process_group()


PHASE_NAMES = ("qkv", "attention", "o_proj", "gate_up", "down")


def print_trace(engine, cohort, cfg, k, show: bool = True) -> None:
    """One traced epoch: per phase kind, the time between grid barriers and its
    parts on CTA 0 (activation staging, tile stream, epilogue drain, wait for the
    last CTA, barrier release; under tensor parallelism also how much of the
    epilogue waited for the other ranks' partials), summed over layers and steps."""
    engine.set_trace(True)
    out, _ = cohort.step()
    engine.set_trace(False)
    L = cfg.num_layers
    phases = 5 * L + 2
    count = 2 + out.model_calls * phases + 1
    tr = engine.read_trace(count).astype(np.int64)
    exit_ns, entry_ns, xready, tiles, last, tp_wait = tr
    end_ns = exit_ns   # a phase ends when CTA 0 leaves its grid barrier
    first = 2   # validation and continuity barriers precede the loop
    acc = {}
    for step in range(out.model_calls):
        for ph in range(phases):
            j = first + step * phases + ph + 1
            name = "lm_head" if ph == 5 * L else "control" if ph > 5 * L else PHASE_NAMES[ph % 5]
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
    wbytes = {"qkv": (sh.nq + 2 * sh.nkv) * d * h * 2 * L, "o_proj": h * sh.nq * d * 2 * L,
              "gate_up": 2 * sh.ni * h * 2 * L, "down": h * sh.ni * 2 * L, "lm_head": sh.nv * h * 2}
    calls = out.model_calls
    print(f"trace: epoch {out.device_us:.1f} us, {calls} steps; per step, us "
          f"[total | x-staging  tiles  epilogue | wait-last-CTA  release | epilogue tp-wait] and weight GB/s",
          file=sys.stderr)
    for name in ("qkv", "attention", "o_proj", "gate_up", "down", "lm_head", "control"):
        a = acc.get(name, np.zeros(7)) / calls / 1e3
        bw = wbytes.get(name, 0) / (a[0] * 1e3) if name in wbytes and a[0] else 0.0
        print(f"  {name:9s} {a[0]:8.1f} | {a[1]:7.1f} {a[2]:7.1f} {a[3]:7.1f} | {a[4]:7.1f} {a[5]:7.1f} "
              f"{a[6]:7.1f}   {bw:6.0f}", file=sys.stderr)


SAMPLE_LAYERS = (1, 5)


def cpu_oracle_step_time(weights: dict, cfg, threads: int) -> tuple[float, str]:
    """Seconds of one 7B decode step of the CPU oracle (bf16 torch ops, the
    reference's own arithmetic), from a bounded sample: steps of the same
    geometry truncated to 1 and 5 layers give the per-layer and the fixed
    (embedding, final norm, lm_head) costs, extrapolated to all layers."""
    import torch

    from oracle.decoder import OracleDecoder
    from oracle.model import OracleConfig

    torch.set_num_threads(threads)
    times = {}
    for layers in SAMPLE_LAYERS:
        ocfg = OracleConfig(num_layers=layers, hidden=cfg.hidden, num_heads=cfg.num_heads,
                            num_kv_heads=cfg.num_kv_heads, head_dim=cfg.head_dim,
                            intermediate=cfg.intermediate, vocab=cfg.vocab, block_size=cfg.block_size)
        decoder = OracleDecoder(ocfg, weights)   # a truncation reads layers 0..layers-1 only
        shape = (layers, ocfg.num_blocks, ocfg.block_size, ocfg.num_kv_heads, ocfg.head_dim)
        key = torch.zeros(shape, dtype=torch.bfloat16)
        value = torch.zeros(shape, dtype=torch.bfloat16)
        token = torch.tensor([11, 12, 13, 14], dtype=torch.int64)
        position = torch.tensor([4, 4, 4, 4], dtype=torch.int64)
        seq_len = torch.tensor([5, 5, 5, 5], dtype=torch.int32)
        bt = torch.arange(8, dtype=torch.int32).reshape(4, 2)
        slot = torch.tensor([4, 260, 516, 772], dtype=torch.int32)
        active = torch.ones(4, dtype=torch.int32)
        decoder.step(token, position, seq_len, bt, slot, key, value, active)   # warm-up
        samples = []
        for _ in range(3):
            t = time.perf_counter()
            decoder.step(token, position, seq_len, bt, slot, key, value, active)
            samples.append(time.perf_counter() - t)
        times[layers] = min(samples)
    lo, hi = SAMPLE_LAYERS
    per_layer = max((times[hi] - times[lo]) / (hi - lo), 1e-9)
    fixed = max(times[lo] - lo * per_layer, 0.0)
    return fixed + cfg.num_layers * per_layer, (
        f"{lo}- and {hi}-layer truncations of the 7B decode step (B=4, ctx 5, {threads} threads), best of 3, "
        f"extrapolated to {cfg.num_layers} layers: {times[lo]*1e3:.0f} / {times[hi]*1e3:.0f} ms"
    )


def engine_weights_fn(engine):
    import torch

    from oracle.model import LAYER_KEYS

    cfg = engine.config

    def weights(layers: int):
        shapes = {"model.embed_tokens.weight": (cfg.vocab, cfg.hidden), "model.norm.weight": (cfg.hidden,),
                  "lm_head.weight": (cfg.vocab, cfg.hidden)}
        h, kv, i = cfg.hidden, cfg.kv_width, cfg.intermediate
        per = {"input_layernorm.weight": (h,), "post_attention_layernorm.weight": (h,),
               "self_attn.q_proj.weight": (h, h), "self_attn.q_proj.bias": (h,),
               "self_attn.k_proj.weight": (kv, h), "self_attn.k_proj.bias": (kv,),
               "self_attn.v_proj.weight": (kv, h), "self_attn.v_proj.bias": (kv,),
               "self_attn.o_proj.weight": (h, h), "mlp.gate_proj.weight": (i, h),
               "mlp.up_proj.weight": (i, h), "mlp.down_proj.weight": (h, i)}
        out = {name: engine.get_weight(name, shape) for name, shape in shapes.items()}
        for layer in range(layers):
            for key in LAYER_KEYS:
                out[f"model.layers.{layer}.{key}"] = engine.get_weight(f"model.layers.{layer}.{key}", per[key])
        return out

    return weights


def cpu_baseline(engine, cfg) -> dict:
    threads = len(os.sched_getaffinity(0))
    step_s, sample = cpu_oracle_step_time(engine_weights_fn(engine)(SAMPLE_LAYERS[-1]), cfg, threads)
    return {"value": round(4 / step_s, 3), "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": sample, "us_per_decode_step": round(step_s * 1e6, 1)}


def run_reference(args) -> None:
    """CPU arm: the oracle port of the reference path on the host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch

    from cruise_b200.model_config import QWEN25_7B

    cfg = QWEN25_7B
    threads = len(os.sched_getaffinity(0))

    weights = random_weights(cfg, layers=SAMPLE_LAYERS[-1], seed=0)
    samples = []
    sample_desc = ""
    for _ in range(args.warmup + args.steps):
        step_s, sample_desc = cpu_oracle_step_time(weights, cfg, threads)
        samples.append(step_s)
    timed = samples[args.warmup:]
    step_s = sum(timed) / len(timed)
    value = 4 / step_s
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "tok/s", "n_gpus": 0,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_s * args.k * 1e3, 2),
        "us_per_decode_step": round(step_s * 1e6, 1), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "configs[1] decode steps (B=4, 7B arch) on the host cores",
                   "epoch_k": args.k},
        "cpu_baseline": {"value": round(value, 3), "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": sample_desc},
        "e2e": {"value": round(value, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def random_weights(cfg, layers: int, seed: int) -> dict:
    """N(0, 0.02) bf16 weights of the 7B geometry truncated to `layers` layers
    (CPU timing does not depend on the values; torch's generator is fast)."""
    import torch

    from oracle.model import OracleConfig, tensor_shapes

    ocfg = OracleConfig(num_layers=layers, hidden=cfg.hidden, num_heads=cfg.num_heads,
                        num_kv_heads=cfg.num_kv_heads, head_dim=cfg.head_dim,
                        intermediate=cfg.intermediate, vocab=cfg.vocab, block_size=cfg.block_size)
    gen = torch.Generator().manual_seed(seed)
    return {name: torch.empty(shape, dtype=torch.bfloat16).normal_(0.0, 0.02, generator=gen)
            for name, shape in tensor_shapes(ocfg).items()}


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
    engine = EpochEngine(cfg)
    engine.init_synthetic(seed=0)
    length = 120
    sc = make_scenario(vocab=cfg.vocab, seed=77, active_rows=(1, 1, 1, 1), prompt_len=(length, length), k=2,
                       budget=(2, 2), eos=cfg.configured_eos, token_high=151643)
    tokens = sum(len(p) - 1 for p in sc.prompts)
    engine.prefill(sc.prompts)   # first call builds the untiled weights
    batched = []
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
        "batched_includes": "host token upload, all 28 layers (cuBLAS GEMMs + prefill kernels), sync",
    }), flush=True)


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=20)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--k", type=int, default=2, choices=(1, 2, 4, 8))
    parser.add_argument("--impl", default="cruise", choices=("cruise", "reference"))
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--trace", action="store_true", help="per-phase timing of one extra epoch (stderr)")
    parser.add_argument("--layers", type=int, default=0, help="profiling only: truncate the model to N layers")
    parser.add_argument("--vocab", type=int, default=0, help="profiling only: vocabulary size")
    parser.add_argument("--tp", action="store_true",
                        help="under torchrun: the ranks form one tensor-parallel group decoding one cohort")
    parser.add_argument("--prompt-max", type=int, default=5,
                        help="longest prompt of the seeded cohort (2..block_size; configs[4] uses 120)")
    parser.add_argument("--prefill", action="store_true",
                        help="measure the batched device prefill instead of the decode epochs")
    args = parser.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.prefill:
        run_prefill(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
