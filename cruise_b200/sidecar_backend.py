"""``NativeEpochEngine`` over the out-of-process sidecar (``cruise_epoch_server``).

The replacement of the reference's ``SidecarDataFlowEngine``
(``src/vllm_ascend_resident_epoch/sidecar_backend.py:39-466``): it starts the
server, talks to it over a Unix stream socket under ``/dev/shm`` with the
reference's fixed-size messages (136-byte request, 352-byte response, the
4,088-byte device-IPC metadata appended to operation 5) and maps responses to
``NativeEpochOutput`` exactly like the in-process ctypes backend.  The engine
lives in the server process: a crash there cannot take the scheduler down.

Environment (the reference's names):

* ``VLLM_ASCEND_RESIDENT_EPOCH_SOCKET``   control socket, required, under /dev/shm
* ``VLLM_ASCEND_RESIDENT_EPOCH_SERVER``   server binary (default: in-tree build)
* ``VLLM_ASCEND_RESIDENT_EPOCH_MODEL``    model preset (default ``qwen2.5-7b``)
* ``VLLM_ASCEND_RESIDENT_EPOCH_EXTERNAL_WEIGHTS``  ``synthetic:<seed>`` or a
  directory of ``<tensor name>.bin`` files (default ``synthetic:0``)
* ``VLLM_ASCEND_RESIDENT_EPOCH_TILING``   optional 72-byte tiling blob
* ``VLLM_ASCEND_RESIDENT_EPOCH_STARTUP_TIMEOUT``  seconds (default 3600)
"""

from __future__ import annotations

import os
import socket
import struct
import subprocess
import time
from pathlib import Path

from .backend import NativeEpochOutput, NativeWarmupOutput
from .contract import EpochCommitState, ResidentEpochExecutionError, ResidentEpochPlan
from .kv_transfer import IPC_METADATA_BYTES, DeviceKVTransfer, ResidentKVSnapshot, write_kv_snapshot
from .model_config import PRESETS
from .version import SIDECAR_PROTOCOL_VERSION, SIDECAR_REQUEST_BYTES, SIDECAR_RESPONSE_BYTES

REQUEST_MAGIC = 0x71317131
RESPONSE_MAGIC = 0x71327132
EXECUTE, WARM_UP, SHUTDOWN, IMPORT_EXECUTE, DEVICE_IPC_EXECUTE = 1, 2, 3, 4, 5
GRAPH_BATCH_SIZE = 4
MAX_EPOCH_STEPS = 8
WARMUP_GENERATION = 2**31 - 1
WARMUP_TOKEN = 11690
# magic, version, operation, request count, max steps, transfer id,
# token[4], position[4], sequence length[4], eos[4], generation[4]
REQUEST = struct.Struct("<IHHiiQ4q4q4i4i4i")
# magic, transport status, device status, model calls, feed calls, fetch calls,
# commit state, import checksum, wall us, native cpu us, declared in / out
# bytes, executed[4], generation[4], tokens[4][8]
RESPONSE = struct.Struct("<Iiiiiiii4q4i4i32q")
assert REQUEST.size == SIDECAR_REQUEST_BYTES and RESPONSE.size == SIDECAR_RESPONSE_BYTES

DEFAULT_SERVER = Path(__file__).resolve().parent / "cruise_epoch_server"


def _commit_state(value: int) -> EpochCommitState:
    try:
        return EpochCommitState(value)
    except ValueError as exc:
        raise ResidentEpochExecutionError(
            f"sidecar returned invalid commit state {value}", commit_state=EpochCommitState.EXECUTING
        ) from exc


def _by_row(plan: ResidentEpochPlan, field: str, fill: int) -> list[int]:
    values = [fill] * GRAPH_BATCH_SIZE
    for request in plan.requests:
        values[request.row] = int(getattr(request, field))
    return values


def _shm_path(raw: str | None, what: str) -> Path:
    if not raw:
        raise RuntimeError(f"{what} is required by the resident epoch sidecar")
    path = Path(raw).resolve()
    if not str(path).startswith("/dev/shm/"):
        raise RuntimeError(f"{what} must be under /dev/shm: {path}")
    return path


class SidecarEpochEngine:
    def __init__(self) -> None:
        server = Path(os.getenv("VLLM_ASCEND_RESIDENT_EPOCH_SERVER") or DEFAULT_SERVER).resolve()
        if not server.is_file():
            raise RuntimeError(f"resident epoch sidecar server is missing: {server}")
        self.model = os.getenv("VLLM_ASCEND_RESIDENT_EPOCH_MODEL", "qwen2.5-7b")
        if self.model not in PRESETS:
            raise RuntimeError(f"unknown resident epoch model preset {self.model!r}")
        self.config = PRESETS[self.model]
        weights = os.getenv("VLLM_ASCEND_RESIDENT_EPOCH_EXTERNAL_WEIGHTS", "synthetic:0")
        tiling = os.getenv("VLLM_ASCEND_RESIDENT_EPOCH_TILING", "")
        self.socket_path = _shm_path(os.getenv("VLLM_ASCEND_RESIDENT_EPOCH_SOCKET"),
                                     "VLLM_ASCEND_RESIDENT_EPOCH_SOCKET")
        self.transfer_path = self.socket_path.with_name(f"{self.socket_path.name}.kv-transfer")
        self.socket_path.unlink(missing_ok=True)
        self.transfer_path.unlink(missing_ok=True)
        self.process = subprocess.Popen(
            [str(server), str(self.socket_path), self.model, "", "", weights, tiling], close_fds=True,
        )
        self.socket: socket.socket | None = None
        timeout = float(os.getenv("VLLM_ASCEND_RESIDENT_EPOCH_STARTUP_TIMEOUT", "3600"))
        deadline = time.monotonic() + timeout
        while time.monotonic() < deadline and self.socket is None:
            if self.process.poll() is not None:
                raise RuntimeError(
                    f"resident epoch sidecar exited during startup with status {self.process.returncode}")
            if self.socket_path.exists():
                candidate = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
                try:
                    candidate.connect(str(self.socket_path))
                    self.socket = candidate
                except OSError:
                    candidate.close()
            if self.socket is None:
                time.sleep(0.02)
        if self.socket is None:
            self._stop_process()
            raise TimeoutError("resident epoch sidecar socket startup timed out")
        self.socket.settimeout(timeout)
        startup = self._receive()
        if startup[1] != 0:
            self.close(force=True)
            raise RuntimeError(f"resident epoch sidecar native initialization failed: {startup[1]}")

    # -- wire ----------------------------------------------------------------------
    def _receive(self) -> tuple[int, ...]:
        assert self.socket is not None
        data = bytearray()
        while len(data) < RESPONSE.size:
            chunk = self.socket.recv(RESPONSE.size - len(data))
            if not chunk:
                raise RuntimeError(f"resident epoch sidecar closed the control socket (status={self.process.poll()})")
            data += chunk
        values = RESPONSE.unpack(bytes(data))
        if values[0] != RESPONSE_MAGIC:
            raise RuntimeError("resident epoch sidecar response magic mismatch")
        return values

    def _request(self, operation: int, count: int, max_steps: int, transfer_id: int, tokens, positions, lengths,
                 eos, generations, tail: bytes = b"") -> tuple[int, ...]:
        if self.socket is None:
            raise ResidentEpochExecutionError("resident epoch sidecar is closed",
                                              commit_state=EpochCommitState.PREPARED)
        payload = REQUEST.pack(REQUEST_MAGIC, SIDECAR_PROTOCOL_VERSION, operation, count, max_steps, transfer_id,
                               *tokens, *positions, *lengths, *eos, *generations) + tail
        try:
            self.socket.sendall(payload)
            return self._receive()
        except Exception as exc:
            raise ResidentEpochExecutionError(f"resident epoch response is ambiguous: {exc}",
                                              commit_state=EpochCommitState.EXECUTING) from exc

    # -- NativeEpochEngine -----------------------------------------------------------
    def warm_up(self) -> NativeWarmupOutput:
        eos = self.config.configured_eos
        v = self._request(WARM_UP, 1, 1, 0, [WARMUP_TOKEN % self.config.vocab, 0, 0, 0], [0] * 4, [1, 0, 0, 0],
                          [eos] * 4, [WARMUP_GENERATION, 0, 0, 0])
        commit_state = _commit_state(v[6])
        if v[1] != 0:
            raise ResidentEpochExecutionError(f"resident epoch warmup failed: {v[1]}", commit_state=commit_state,
                                              status=v[1])
        if v[12:16] != (1, 0, 0, 0) or v[16:20] != (WARMUP_GENERATION, 0, 0, 0):
            raise RuntimeError("resident epoch warmup did not run exactly one row")
        return NativeWarmupOutput(status=v[2], model_calls=v[3], feed_calls=v[4], fetch_calls=v[5],
                                  commit_state=commit_state, wall_us=v[8], native_cpu_us=v[9],
                                  declared_input_bytes=v[10], declared_output_bytes=v[11])

    def execute(self, plan: ResidentEpochPlan) -> NativeEpochOutput:
        return self._execute(plan, EXECUTE, 0)

    def execute_with_import(self, plan: ResidentEpochPlan, snapshot: ResidentKVSnapshot) -> NativeEpochOutput:
        snapshot.validate()
        self._check_transfer(plan, snapshot.import_mask, snapshot.row_generations, "KV snapshot")
        write_kv_snapshot(self.transfer_path, snapshot)
        try:
            return self._execute(plan, IMPORT_EXECUTE, snapshot.transfer_id)
        finally:
            self.transfer_path.unlink(missing_ok=True)

    def execute_with_device_transfer(self, plan: ResidentEpochPlan, transfer: DeviceKVTransfer) -> NativeEpochOutput:
        transfer.validate()
        self._check_transfer(plan, transfer.import_mask, transfer.row_generations, "device KV transfer")
        metadata = transfer.wire_bytes()
        if len(metadata) != IPC_METADATA_BYTES:
            raise ValueError("device KV transfer metadata has the wrong size")
        return self._execute(plan, DEVICE_IPC_EXECUTE, transfer.transfer_id, metadata)

    @staticmethod
    def _check_transfer(plan: ResidentEpochPlan, mask: int, generations, what: str) -> None:
        expected_mask = sum(1 << r.row for r in plan.requests if r.kv_import_required)
        if mask != expected_mask:
            raise ValueError(f"{what} mask does not match the resident plan")
        expected = [0] * GRAPH_BATCH_SIZE
        for r in plan.requests:
            if r.kv_import_required:
                expected[r.row] = r.generation
        if tuple(generations) != tuple(expected):
            raise ValueError(f"{what} generations do not match the resident plan")

    def _execute(self, plan: ResidentEpochPlan, operation: int, transfer_id: int, tail: bytes = b"") -> NativeEpochOutput:
        if plan.graph_batch_size != GRAPH_BATCH_SIZE:
            raise ValueError("the sidecar serves the static B=4 epoch")
        v = self._request(operation, len(plan.requests), plan.max_steps, transfer_id,
                          _by_row(plan, "token_id", 0), _by_row(plan, "position", 0),
                          _by_row(plan, "sequence_length", 0),
                          _by_row(plan, "eos_token_id", self.config.configured_eos), plan.row_generations, tail)
        commit_state = _commit_state(v[6])
        if v[1] != 0:
            raise ResidentEpochExecutionError(f"resident epoch sidecar execute failed: {v[1]}",
                                              commit_state=commit_state, status=v[1])
        executed, tokens = v[12:16], v[20:]
        token_ids: dict[str, list[int]] = {}
        for r in plan.requests:
            count = executed[r.row]
            if not 0 <= count <= plan.max_steps:
                raise ResidentEpochExecutionError("sidecar returned an invalid executed count",
                                                  commit_state=commit_state)
            base = r.row * MAX_EPOCH_STEPS
            token_ids[r.req_id] = list(tokens[base: base + count])
        imported = operation in (IMPORT_EXECUTE, DEVICE_IPC_EXECUTE)
        return NativeEpochOutput(
            status=v[2], model_calls=v[3], token_ids=token_ids, row_generations=tuple(v[16:20]),
            commit_state=commit_state, feed_calls=v[4], fetch_calls=v[5], wall_us=v[8], native_cpu_us=v[9],
            declared_input_bytes=v[10], declared_output_bytes=v[11], kv_imported=imported,
            kv_import_checksum=v[7] & 0xFFFFFFFF,
            kv_transfer_mode=("device_ipc" if operation == DEVICE_IPC_EXECUTE
                              else "host_snapshot" if operation == IMPORT_EXECUTE else "none"),
        )

    # -- lifecycle -----------------------------------------------------------------------
    def _stop_process(self) -> None:
        if self.process.poll() is None:
            self.process.terminate()
            try:
                self.process.wait(timeout=60)
            except subprocess.TimeoutExpired:
                self.process.kill()
                self.process.wait(timeout=60)

    def close(self, *, force: bool = False) -> None:
        if getattr(self, "socket", None) is not None:
            if not force and self.process.poll() is None:
                try:
                    self.socket.sendall(REQUEST.pack(REQUEST_MAGIC, SIDECAR_PROTOCOL_VERSION, SHUTDOWN, 0, 0, 0,
                                                     *([0] * 20)))
                    self._receive()
                except (OSError, RuntimeError):
                    force = True
            self.socket.close()
            self.socket = None
        if getattr(self, "process", None) is not None:
            if force:
                self._stop_process()
            else:
                try:
                    self.process.wait(timeout=300)
                except subprocess.TimeoutExpired:
                    self._stop_process()
        for path in (getattr(self, "socket_path", None), getattr(self, "transfer_path", None)):
            if path is not None:
                try:
                    path.unlink(missing_ok=True)
                except OSError:
                    pass

    def __del__(self) -> None:
        try:
            self.close(force=True)
        except Exception:
            pass


# the reference's class name, for callers that import it
SidecarDataFlowEngine = SidecarEpochEngine


def create_sidecar_engine() -> SidecarEpochEngine:
    return SidecarEpochEngine()
