"""The sidecar server and client without a GPU: wire layout, startup handshake,
exit codes and the client's checks.  Engine creation fails on a CPU host (no
CUDA device), which the server must report as startup status 100 + 3 and exit
with the same code -- that path exercises the real socket and message layout.
The client-side wire tests follow the reference's tests/test_sidecar_protocol.py
(round trip, reserved warm-up generation, device IPC reported as an import)."""

from __future__ import annotations

import os
import socket
import subprocess
import time
import uuid
from pathlib import Path

import pytest
import torch

from cruise_b200 import sidecar_backend as sc
from cruise_b200.build import SERVER, build


@pytest.fixture(scope="module")
def server() -> Path:
    build()
    assert SERVER.is_file()
    return SERVER


def _shm(name: str) -> Path:
    return Path("/dev/shm") / f"cruise-test-{name}-{uuid.uuid4().hex[:8]}"


def test_wire_sizes_match_the_protocol():
    assert sc.REQUEST.size == 136 and sc.RESPONSE.size == 352
    from cruise_b200.kv_transfer import IPC_METADATA_BYTES

    assert IPC_METADATA_BYTES == 4088


def test_usage_and_socket_path_errors(server):
    assert subprocess.run([str(server)], capture_output=True).returncode == 64
    # the control socket must live under /dev/shm
    assert subprocess.run([str(server), "/tmp/x.sock", "tiny", "", "", "synthetic:0", ""]).returncode == 65


@pytest.mark.skipif(torch.cuda.is_available(), reason="exercises the failed-create path of a GPU-less host")
def test_startup_response_layout_without_a_gpu(server):
    path = _shm("raw")
    proc = subprocess.Popen([str(server), str(path), "tiny", "", "", "synthetic:0", ""])
    try:
        deadline = time.monotonic() + 60
        while not path.exists():
            assert time.monotonic() < deadline and proc.poll() is None
            time.sleep(0.01)
        with socket.socket(socket.AF_UNIX, socket.SOCK_STREAM) as s:
            s.connect(str(path))
            data = b""
            while len(data) < sc.RESPONSE.size:
                chunk = s.recv(sc.RESPONSE.size - len(data))
                assert chunk
                data += chunk
        v = sc.RESPONSE.unpack(data)
        assert v[0] == sc.RESPONSE_MAGIC and v[1] == 103        # 100 + create status 3 (no device)
        assert v[2] == -1 and v[6] == 0                            # device status unset, commit PREPARED
        assert v[12:20] == (0,) * 8 and v[20:] == (-1,) * 32       # executed / generations / tokens
        assert proc.wait(timeout=60) == 103
    finally:
        if proc.poll() is None:
            proc.kill()
    assert not path.exists()   # the server removes its socket


@pytest.mark.skipif(torch.cuda.is_available(), reason="exercises the failed-create path of a GPU-less host")
def test_client_reports_failed_native_start(server, monkeypatch):
    path = _shm("client")
    monkeypatch.setenv("VLLM_ASCEND_RESIDENT_EPOCH_SOCKET", str(path))
    monkeypatch.setenv("VLLM_ASCEND_RESIDENT_EPOCH_MODEL", "tiny")
    with pytest.raises(RuntimeError, match=r"native initialization failed: 103|exited during startup with status 103"):
        sc.SidecarEpochEngine()
    assert not path.exists()


def test_client_refuses_a_socket_outside_shm(monkeypatch):
    monkeypatch.setenv("VLLM_ASCEND_RESIDENT_EPOCH_SOCKET", "/tmp/cruise.sock")
    with pytest.raises(RuntimeError, match="under /dev/shm"):
        sc.SidecarEpochEngine()


def test_transfer_checks_against_the_plan():
    from cruise_b200.contract import CONTRACT_VERSION, ResidentEpochPlan, ResidentEpochRequest

    reqs = tuple(ResidentEpochRequest(req_id=f"r{row}", row=row, generation=row + 1, token_id=5, position=3,
                                      sequence_length=4, eos_token_id=4095, scheduler_block_ids=(row,),
                                      device_block_ids=(2 * row, 2 * row + 1), kv_import_required=row == 1)
                 for row in (0, 1))
    plan = ResidentEpochPlan(version=CONTRACT_VERSION, graph_batch_size=4, max_steps=2, logical_capacity=32,
                             requests=reqs, active_mask=(1, 1, 0, 0))
    sc.SidecarEpochEngine._check_transfer(plan, 0b10, (0, 2, 0, 0), "x")
    with pytest.raises(ValueError, match="mask"):
        sc.SidecarEpochEngine._check_transfer(plan, 0b11, (1, 2, 0, 0), "x")
    with pytest.raises(ValueError, match="generations"):
        sc.SidecarEpochEngine._check_transfer(plan, 0b10, (0, 3, 0, 0), "x")
    assert sc._by_row(plan, "token_id", 0) == [5, 5, 0, 0]
    assert sc._by_row(plan, "eos_token_id", 7) == [4095, 4095, 7, 7]


def test_request_and_response_round_trip():
    from cruise_b200.contract import EpochCommitState

    request = sc.REQUEST.pack(sc.REQUEST_MAGIC, sc.SIDECAR_PROTOCOL_VERSION, sc.EXECUTE, 2, 4, 0, *range(4),
                              *range(4), *([1] * 4), *([151645] * 4), *([1, 2, 0, 0]))
    assert sc.REQUEST.unpack(request)[:5] == (sc.REQUEST_MAGIC, sc.SIDECAR_PROTOCOL_VERSION, sc.EXECUTE, 2, 4)
    response = sc.RESPONSE.pack(sc.RESPONSE_MAGIC, 0, 0, 4, 1, 1, EpochCommitState.COMMITTED, 0x12345678, 123, 45,
                                260, 368, *([4, 4, 0, 0]), *([1, 2, 0, 0]), *range(32))
    values = sc.RESPONSE.unpack(response)
    assert values[:12] == (sc.RESPONSE_MAGIC, 0, 0, 4, 1, 1, EpochCommitState.COMMITTED, 0x12345678, 123, 45, 260,
                           368)


class _RecordingSocket:
    def __init__(self):
        self.payloads = []

    def sendall(self, payload):
        self.payloads.append(payload)


def _wired_client(response: tuple) -> sc.SidecarEpochEngine:
    """A client whose socket records requests and whose reply is `response`."""
    from cruise_b200.model_config import QWEN25_7B

    engine = sc.SidecarEpochEngine.__new__(sc.SidecarEpochEngine)
    engine.socket = _RecordingSocket()
    engine.config = QWEN25_7B
    engine._receive = lambda: response
    return engine


def test_warmup_uses_the_reserved_generation():
    from cruise_b200.contract import EpochCommitState

    reply = sc.RESPONSE.unpack(sc.RESPONSE.pack(sc.RESPONSE_MAGIC, 0, 0, 1, 1, 1, EpochCommitState.COMMITTED, 0, 1, 1,
                                                260, 368, 1, 0, 0, 0, sc.WARMUP_GENERATION, 0, 0, 0,
                                                5, *([-1] * 31)))
    engine = _wired_client(reply)
    out = engine.warm_up()
    assert out.model_calls == 1 and out.commit_state == EpochCommitState.COMMITTED
    sent = sc.REQUEST.unpack(engine.socket.payloads[0])
    assert sent[:5] == (sc.REQUEST_MAGIC, sc.SIDECAR_PROTOCOL_VERSION, sc.WARM_UP, 1, 1)
    assert sent[-4:] == (sc.WARMUP_GENERATION, 0, 0, 0) and sent[6] == sc.WARMUP_TOKEN


def test_device_ipc_execute_is_reported_as_kv_import():
    from cruise_b200.contract import CONTRACT_VERSION, EpochCommitState, ResidentEpochPlan, ResidentEpochRequest
    from cruise_b200.kv_transfer import IPC_METADATA_BYTES

    reply = sc.RESPONSE.unpack(sc.RESPONSE.pack(sc.RESPONSE_MAGIC, 0, 0, 1, 1, 1, EpochCommitState.COMMITTED,
                                                0x12345678, 123, 45, 3776, 368, 1, 0, 0, 0, 7, 0, 0, 0,
                                                42, *([-1] * 31)))
    engine = _wired_client(reply)
    plan = ResidentEpochPlan(
        version=CONTRACT_VERSION, graph_batch_size=4, max_steps=1, logical_capacity=8,
        requests=(ResidentEpochRequest(req_id="request-0", row=0, generation=7, token_id=11, position=1,
                                       sequence_length=2, eos_token_id=151645, scheduler_block_ids=(0,),
                                       device_block_ids=(0, 1), kv_import_required=True),),
        active_mask=(1, 0, 0, 0))
    metadata = b"\0" * IPC_METADATA_BYTES
    out = engine._execute(plan, sc.DEVICE_IPC_EXECUTE, 9, metadata)
    assert out.kv_imported and out.kv_import_checksum == 0x12345678 and out.kv_transfer_mode == "device_ipc"
    assert out.token_ids == {"request-0": [42]} and out.row_generations == (7, 0, 0, 0)
    assert len(engine.socket.payloads) == 1 and engine.socket.payloads[0][sc.REQUEST.size:] == metadata
    sent = sc.REQUEST.unpack(engine.socket.payloads[0][: sc.REQUEST.size])
    assert sent[2] == sc.DEVICE_IPC_EXECUTE and sent[5] == 9


def test_transport_errors_keep_the_commit_state():
    from cruise_b200.contract import EpochCommitState, ResidentEpochExecutionError

    reply = sc.RESPONSE.unpack(sc.RESPONSE.pack(sc.RESPONSE_MAGIC, 12, -1, 0, 0, 0, EpochCommitState.PREPARED, 0,
                                                0, 0, 0, 0, *([0] * 8), *([-1] * 32)))
    engine = _wired_client(reply)
    from cruise_b200.contract import CONTRACT_VERSION, ResidentEpochPlan, ResidentEpochRequest

    plan = ResidentEpochPlan(
        version=CONTRACT_VERSION, graph_batch_size=4, max_steps=1, logical_capacity=8,
        requests=(ResidentEpochRequest(req_id="a", row=0, generation=1, token_id=1, position=0, sequence_length=1,
                                       eos_token_id=151645, scheduler_block_ids=(0,), device_block_ids=(0, 1)),),
        active_mask=(1, 0, 0, 0))
    with pytest.raises(ResidentEpochExecutionError) as caught:
        engine.execute(plan)
    assert caught.value.status == 12 and caught.value.commit_state == EpochCommitState.PREPARED


@pytest.fixture(scope="module")
def sanitized_server(server, tmp_path_factory) -> Path:
    """The sidecar server built with AddressSanitizer and UBSan (host code only;
    the engine library it links is the regular build)."""
    import shutil

    from cruise_b200.build import PACKAGE, SERVER_SOURCES

    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("no g++")
    out = tmp_path_factory.mktemp("asan") / "cruise_epoch_server_asan"
    cmd = [cxx, "-O1", "-g", "-std=c++17", "-fsanitize=address,undefined", "-fno-omit-frame-pointer",
           "-fno-sanitize-recover=undefined", "-o", str(out), *map(str, SERVER_SOURCES), f"-L{PACKAGE}",
           "-l:libcruise_epoch.so", f"-Wl,-rpath,{PACKAGE}"]
    if subprocess.run(cmd, capture_output=True).returncode != 0:
        pytest.skip("sanitizer runtime not available")
    return out


@pytest.mark.skipif(torch.cuda.is_available(), reason="exercises the failed-create path of a GPU-less host")
def test_server_host_code_is_sanitizer_clean(sanitized_server):
    env = dict(os.environ, ASAN_OPTIONS="detect_leaks=0:abort_on_error=0", UBSAN_OPTIONS="print_stacktrace=1")
    usage = subprocess.run([str(sanitized_server)], capture_output=True, env=env)
    assert usage.returncode == 64
    path = _shm("asan")
    proc = subprocess.Popen([str(sanitized_server), str(path), "tiny", "", "", "synthetic:0", ""],
                            stderr=subprocess.PIPE, env=env)
    try:
        deadline = time.monotonic() + 120
        while not path.exists():
            assert time.monotonic() < deadline and proc.poll() is None
            time.sleep(0.01)
        with socket.socket(socket.AF_UNIX, socket.SOCK_STREAM) as s:
            s.connect(str(path))
            data = b""
            while len(data) < sc.RESPONSE.size:
                chunk = s.recv(sc.RESPONSE.size - len(data))
                assert chunk
                data += chunk
        assert sc.RESPONSE.unpack(data)[1] == 103
        _, err = proc.communicate(timeout=120)
        assert proc.returncode == 103
        text = err.decode(errors="replace")
        assert "AddressSanitizer" not in text and "runtime error" not in text, text[-2000:]
    finally:
        if proc.poll() is None:
            proc.kill()
