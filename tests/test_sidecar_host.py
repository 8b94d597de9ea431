"""The sidecar server and client without a GPU: wire layout, startup handshake,
exit codes and the client's checks.  Engine creation fails on a CPU host (no
CUDA device), which the server must report as startup status 100 + 3 and exit
with the same code -- that path exercises the real socket and message layout."""

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
