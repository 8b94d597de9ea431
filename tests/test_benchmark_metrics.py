"""Host-control counters and their event journal (the reference's
tests/test_m4a_performance.py:224-259), the path rule for the environment
variable, and the counters a real vLLM scheduler records through a
host-prefill -> device-epoch sequence."""

from __future__ import annotations

import atexit
import json
import os
from pathlib import Path
from types import SimpleNamespace

import pytest

from cruise_b200.benchmark_metrics import METRICS_ENV, ResidentEpochBenchmarkMetrics, metrics_path, replay_event_journal


def _device_result(**kw):
    fields = dict(route="device", model_calls=2, computed_steps={"a": 2, "b": 2}, feed_calls=1, fetch_calls=1,
                  wall_us=100, native_cpu_us=20, socket_send_calls=1, socket_receive_calls=1, kv_imported=True)
    fields.update(kw)
    return SimpleNamespace(**fields)


def test_disabled_by_default_and_flush_once(tmp_path):
    disabled = ResidentEpochBenchmarkMetrics()
    disabled.record_schedule(SimpleNamespace(requests=(1,), max_steps=2), None)
    disabled.record_result(_device_result())
    disabled.flush()
    assert disabled.as_record()["counters"] == {} and list(tmp_path.iterdir()) == []

    output = tmp_path / "metrics.json"
    metrics = ResidentEpochBenchmarkMetrics(output)
    metrics.record_schedule(SimpleNamespace(requests=(1, 2), max_steps=2), None)
    metrics.record_schedule(None, "host-prefill-in-progress")
    metrics.record_schedule(None, None)
    metrics.record_result(_device_result())
    metrics.record_result(SimpleNamespace(route="host_fallback"))
    metrics.flush()
    payload = json.loads(output.read_text(encoding="utf-8"))
    counters = payload["counters"]
    assert payload["schema_version"] == 1
    assert counters["schedule_calls"] == 3 and counters["device_plan_calls"] == 1
    assert counters["device_planned_requests"] == 2 and counters["device_planned_model_calls"] == 2
    assert counters["host_schedule_calls"] == 2 and counters["non_device_results"] == 1
    assert counters["device_epochs"] == 1 and counters["device_request_tokens"] == 4
    assert counters["native_wall_us"] == 100 and counters["native_cpu_us"] == 20 and counters["kv_imports"] == 1
    assert payload["epoch_steps"] == {"2": 1}
    assert payload["rejections"] == {"host-prefill-in-progress": 1, "unspecified": 1}

    journal = output.with_name("metrics.events.jsonl")
    assert len(journal.read_text().splitlines()) == 5
    assert replay_event_journal(journal) == payload
    assert not any(p.name.endswith(".tmp") for p in tmp_path.iterdir())


def test_missing_directories_are_created(tmp_path):
    output = tmp_path / "new" / "dir" / "metrics.json"
    metrics = ResidentEpochBenchmarkMetrics(output)
    metrics.record_schedule(None, "x")
    metrics.flush()
    assert json.loads(output.read_text())["rejections"] == {"x": 1}


def test_journal_survives_a_process_that_never_flushes(tmp_path):
    """Events are on disk as they happen: a second writer appends, and the
    replay counts both even though neither wrote its summary."""
    output = tmp_path / "run.json"
    first = ResidentEpochBenchmarkMetrics(output)
    first.record_schedule(SimpleNamespace(requests=(1,), max_steps=4), None)
    second = ResidentEpochBenchmarkMetrics(output)
    second.record_result(_device_result(model_calls=4, computed_steps={"a": 4}, kv_imported=False))
    assert not output.exists()
    replayed = replay_event_journal(output.with_name("run.events.jsonl"))
    assert replayed["counters"]["device_plan_calls"] == 1 and replayed["counters"]["device_model_calls"] == 4
    assert replayed["epoch_steps"] == {"4": 1} and "kv_imports" not in replayed["counters"]


@pytest.mark.parametrize("raw", ["relative/metrics.json", "/tmp/metrics.json", "/dev/shm", "/dev/shm/../tmp/m.json"])
def test_metrics_path_must_lie_inside_shared_memory(raw):
    with pytest.raises(ValueError, match="absolute|/dev/shm"):
        metrics_path(raw)


def test_metrics_path_inside_shared_memory_is_accepted():
    assert metrics_path("/dev/shm/cruise/metrics.json") == Path("/dev/shm/cruise/metrics.json").resolve()


def test_scheduler_records_host_prefill_then_device_epochs(tmp_path, monkeypatch):
    pytest.importorskip("vllm")
    from test_vllm_scheduler import commit_device_epoch, host_step, make_scheduler, request

    shm = Path("/dev/shm") / f"cruise-metrics-{os.getpid()}"
    shm.mkdir(exist_ok=True)
    output = shm / "metrics.json"
    monkeypatch.setenv(METRICS_ENV, str(output))
    scheduler = None
    try:
        scheduler = make_scheduler(tmp_path, 2)
        scheduler.add_request(request("long", [5, 6, 7], max_tokens=4))
        out = scheduler.schedule()                     # host prefill of a 3-token prompt
        host_step(scheduler, out, {"long": [8]})
        out = scheduler.schedule()                     # then a K = 2 device epoch with the import
        plan = commit_device_epoch(scheduler, out, {"long": [9, 10]})
        assert plan.max_steps == 2
        scheduler.benchmark_metrics.flush()
        payload = json.loads(output.read_text())
        counters = payload["counters"]
        assert counters["schedule_calls"] == 2 and counters["host_schedule_calls"] == 1
        assert counters["device_plan_calls"] == 1 and counters["device_epochs"] == 1
        assert counters["device_request_tokens"] == 2 and counters["kv_imports"] == 1
        assert payload["epoch_steps"] == {"2": 1} and payload["rejections"] == {"not-single-token-decode": 1}
        assert replay_event_journal(output.with_name("metrics.events.jsonl")) == payload
    finally:
        if scheduler is not None:   # its exit-time flush would recreate the directory
            atexit.unregister(scheduler.benchmark_metrics.flush)
            scheduler.benchmark_metrics.flush()
        for path in shm.iterdir():
            path.unlink()
        shm.rmdir()
