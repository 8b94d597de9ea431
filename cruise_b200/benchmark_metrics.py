"""Host-control counters of the resident epoch path, off unless asked for
(src/vllm_ascend_resident_epoch/benchmark_metrics.py:11-190).

Setting ``VLLM_ASCEND_RESIDENT_EPOCH_BENCHMARK_METRICS_PATH`` to a file under
/dev/shm turns them on for a scheduler.  Every schedule and every epoch
result then becomes one JSON line appended to ``<stem>.events.jsonl`` beside
that file, written through an O_APPEND descriptor, so a process that dies
keeps every line it wrote.  The counters derived from the events are
written to the file itself at exit (atomically, via a temporary file and a
rename).  ``replay_event_journal`` rebuilds the same counters from the
journal alone, for an engine core that exited without running its exit
hooks.

Live counting and replay apply events through one function
(:meth:`ResidentEpochBenchmarkMetrics.apply`), so the two cannot disagree.
The event schema, the counter names and the summary record match the
reference's, so its tooling reads these files.
"""

from __future__ import annotations

import atexit
import json
import os
from collections import Counter
from pathlib import Path
from typing import Any

METRICS_ENV = "VLLM_ASCEND_RESIDENT_EPOCH_BENCHMARK_METRICS_PATH"
SCHEMA_VERSION = 1
RECORD_KIND = "Cruise M4a benchmark-only resident epoch counters"   # the summary's format label
SHARED_MEMORY = Path("/dev/shm")

# result fields summed into counters of the same name (wall_us -> native_wall_us)
_RESULT_SUMS = (
    ("feed_calls", "feed_calls"),
    ("fetch_calls", "fetch_calls"),
    ("wall_us", "native_wall_us"),
    ("native_cpu_us", "native_cpu_us"),
    ("socket_send_calls", "socket_send_calls"),
    ("socket_receive_calls", "socket_receive_calls"),
)


def metrics_path(raw: str) -> Path:
    """The summary path the environment names: absolute and strictly inside
    /dev/shm (after resolving links), else ValueError."""
    path = Path(raw)
    if not path.is_absolute():
        raise ValueError(f"{METRICS_ENV} must be an absolute path")
    resolved = path.resolve(strict=False)
    shm = SHARED_MEMORY.resolve(strict=False)
    if shm not in resolved.parents:
        raise ValueError(f"{METRICS_ENV} must be under /dev/shm")
    return resolved


class ResidentEpochBenchmarkMetrics:
    """Counters of schedules and epoch results, with an append-only journal.
    Without a path every method is a no-op."""

    def __init__(self, path: Path | None = None) -> None:
        self.path = path
        self.counters: Counter[str] = Counter()
        self.rejections: Counter[str] = Counter()
        self.epoch_steps: Counter[int] = Counter()
        self._journal: int | None = None
        if path is not None:
            path.parent.mkdir(parents=True, exist_ok=True)
            journal = path.with_name(f"{path.stem}.events.jsonl")
            self._journal = os.open(journal, os.O_WRONLY | os.O_CREAT | os.O_APPEND, 0o600)

    @classmethod
    def from_env(cls) -> "ResidentEpochBenchmarkMetrics":
        raw = os.getenv(METRICS_ENV)
        metrics = cls(metrics_path(raw) if raw else None)
        if metrics.path is not None:
            atexit.register(metrics.flush)
        return metrics

    @property
    def journal_path(self) -> Path | None:
        return None if self.path is None else self.path.with_name(f"{self.path.stem}.events.jsonl")

    # -- events ---------------------------------------------------------------------------
    def apply(self, event: dict[str, Any]) -> None:
        """Adds one journal event to the counters."""
        c = self.counters
        if event.get("kind") == "schedule":
            c["schedule_calls"] += 1
            if event.get("device"):
                c["device_plan_calls"] += 1
                c["device_planned_requests"] += int(event["request_count"])
                c["device_planned_model_calls"] += int(event["max_steps"])
                self.epoch_steps[int(event["max_steps"])] += 1
            else:
                c["host_schedule_calls"] += 1
                self.rejections[event.get("rejection") or "unspecified"] += 1
        elif event.get("kind") == "result":
            if event.get("route") != "device":
                c["non_device_results"] += 1
                return
            c["device_epochs"] += 1
            c["device_model_calls"] += int(event["model_calls"])
            c["device_request_tokens"] += sum(int(v) for v in event["computed_steps"].values())
            for field, counter in _RESULT_SUMS:
                c[counter] += int(event[field])
            if event.get("kv_imported"):
                c["kv_imports"] += 1

    def _record(self, event: dict[str, Any]) -> None:
        self.apply(event)
        if self._journal is not None:
            os.write(self._journal, (json.dumps(event, sort_keys=True) + "\n").encode())

    def record_schedule(self, plan: Any | None, rejection: str | None) -> None:
        """One scheduler step: a device plan, or a host step and why."""
        if self.path is None:
            return
        if plan is None:
            self._record({"kind": "schedule", "device": False, "rejection": rejection})
        else:
            self._record({"kind": "schedule", "device": True, "request_count": len(plan.requests),
                          "max_steps": int(plan.max_steps)})

    def record_result(self, result: Any) -> None:
        """One epoch result (a ResidentEpochResult)."""
        if self.path is None:
            return
        if result.route != "device":
            self._record({"kind": "result", "route": result.route})
            return
        event = {"kind": "result", "route": "device", "model_calls": int(result.model_calls),
                 "computed_steps": {str(k): int(v) for k, v in result.computed_steps.items()},
                 "kv_imported": bool(result.kv_imported)}
        for field, _ in _RESULT_SUMS:
            event[field] = int(getattr(result, field))
        self._record(event)

    # -- summary ----------------------------------------------------------------------------
    def as_record(self) -> dict[str, Any]:
        return {
            "schema_version": SCHEMA_VERSION,
            "kind": RECORD_KIND,
            "counters": dict(sorted(self.counters.items())),
            "epoch_steps": {str(k): v for k, v in sorted(self.epoch_steps.items())},
            "rejections": dict(sorted(self.rejections.items())),
        }

    def flush(self) -> None:
        """Writes the summary (temporary file, then rename) and closes the journal."""
        if self.path is None:
            return
        self.path.parent.mkdir(parents=True, exist_ok=True)
        staging = self.path.with_name(f".{self.path.name}.{os.getpid()}.tmp")
        staging.write_text(json.dumps(self.as_record(), indent=2, sort_keys=True) + "\n", encoding="utf-8")
        os.replace(staging, self.path)
        if self._journal is not None:
            os.close(self._journal)
            self._journal = None


def replay_event_journal(path: Path) -> dict[str, Any]:
    """The summary record rebuilt from a journal alone."""
    metrics = ResidentEpochBenchmarkMetrics()
    with Path(path).open(encoding="utf-8") as stream:
        for line in stream:
            if line.strip():
                metrics.apply(json.loads(line))
    return metrics.as_record()
