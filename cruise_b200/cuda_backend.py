"""``NativeEpochEngine`` over the CUDA engine's reference-compatible C ABI.

The in-process replacement of ``CtypesDataFlowEngine``
(``src/vllm_ascend_resident_epoch/ctypes_backend.py:30-250``): it binds
``resident_epoch_create / _execute / _destroy`` of ``libcruise_epoch.so`` and
turns a plan into the bridge's host buffers, exactly as the reference's
ctypes backend does.  Environment (the reference's names where they exist):

* ``VLLM_ASCEND_RESIDENT_EPOCH_LIBRARY``   engine library (default: in-tree build)
* ``VLLM_ASCEND_RESIDENT_EPOCH_MODEL``     model preset (default ``qwen2.5-7b``)
* ``VLLM_ASCEND_RESIDENT_EPOCH_EXTERNAL_WEIGHTS``  ``synthetic:<seed>`` or a
  directory of ``<tensor name>.bin`` files (default ``synthetic:0``)
* ``VLLM_ASCEND_RESIDENT_EPOCH_TILING``    optional 72-byte tiling blob
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path
from typing import Any

from . import _lib
from .backend import NativeEpochOutput, NativeWarmupOutput
from .contract import EpochCommitState, ResidentEpochExecutionError, ResidentEpochPlan
from .kv_transfer import DeviceKVTransfer, ResidentKVSnapshot, write_kv_snapshot
from .model_config import PRESETS

MAX_EPOCH_STEPS = 8
WARMUP_GENERATION = 2**31 - 1   # sidecar_backend.py:218-272
WARMUP_TOKEN = 11690


class CudaEpochEngine:
    def __init__(self, model: str | None = None, weights: str | None = None, tiling: str | None = None) -> None:
        self.model = model or os.getenv("VLLM_ASCEND_RESIDENT_EPOCH_MODEL", "qwen2.5-7b")
        if self.model not in PRESETS:
            raise RuntimeError(f"unknown resident epoch model preset {self.model!r}")
        self.config = PRESETS[self.model]
        weights = weights or os.getenv("VLLM_ASCEND_RESIDENT_EPOCH_EXTERNAL_WEIGHTS", "synthetic:0")
        tiling = tiling or os.getenv("VLLM_ASCEND_RESIDENT_EPOCH_TILING")
        self.prefill_transfers = 0   # transfer ids of device-prefill imports
        self.library = _lib.load()
        status = ctypes.c_int32(-1)
        self.handle = self.library.resident_epoch_create(
            self.model.encode(), None, None, weights.encode(), tiling.encode() if tiling else None,
            ctypes.byref(status),
        )
        if not self.handle or status.value != 0:
            detail = self.library.cruise_epoch_last_error(None).decode()
            raise RuntimeError(f"failed to create the CUDA resident epoch, status={status.value}: {detail}")

    # -- NativeEpochEngine ---------------------------------------------------------
    def warm_up(self) -> NativeWarmupOutput:
        out = self._call(
            request_count=1, max_steps=1,
            tokens=[WARMUP_TOKEN % self.config.vocab, 0, 0, 0], positions=[0, 0, 0, 0], lengths=[1, 0, 0, 0],
            eos=[self.config.configured_eos] * 4, generations=[WARMUP_GENERATION, 0, 0, 0],
        )
        return NativeWarmupOutput(
            status=out["device_status"] if out["ret"] == 0 else out["ret"],
            model_calls=out["model_calls"], feed_calls=out["feed_calls"], fetch_calls=out["fetch_calls"],
            wall_us=out["wall_us"], commit_state=out["commit_state"], native_cpu_us=out["native_cpu_us"],
            declared_input_bytes=out["declared_input_bytes"], declared_output_bytes=out["declared_output_bytes"],
        )

    def execute(self, plan: ResidentEpochPlan) -> NativeEpochOutput:
        return self._execute(plan, transfer_path=None, transfer_id=0, ipc=None)

    def execute_with_import(self, plan: ResidentEpochPlan, snapshot: ResidentKVSnapshot) -> NativeEpochOutput:
        path = Path(f"/dev/shm/cruise-kv-transfer-{os.getpid()}-{snapshot.transfer_id}")
        write_kv_snapshot(path, snapshot)
        try:
            return self._execute(plan, transfer_path=path, transfer_id=snapshot.transfer_id, ipc=None)
        finally:
            path.unlink(missing_ok=True)

    def execute_with_device_transfer(self, plan: ResidentEpochPlan, transfer: DeviceKVTransfer) -> NativeEpochOutput:
        transfer.validate()
        metadata = ctypes.create_string_buffer(transfer.wire_bytes())
        return self._execute(plan, transfer_path=None, transfer_id=transfer.transfer_id, ipc=metadata)

    def execute_with_device_prefill(self, plan: ResidentEpochPlan) -> NativeEpochOutput:
        """The plan's prompts (its requests with ``prompt_token_ids``) run
        through the engine's batched device prefill, then the epoch imports
        their K/V from the device and decodes from each last prompt token
        (``resident_epoch_prefill``, then ``resident_epoch_execute`` with a
        transfer id and neither a file nor IPC metadata)."""
        stride = self.config.block_size
        tokens = (ctypes.c_int64 * (4 * stride))()
        lengths = (ctypes.c_int32 * 4)()
        for r in plan.requests:
            if not r.prompt_token_ids:
                continue
            if len(r.prompt_token_ids) > stride:
                raise ResidentEpochExecutionError(
                    f"a device prefill takes at most {stride} prompt tokens per row",
                    commit_state=EpochCommitState.PREPARED,
                )
            for i, token in enumerate(r.prompt_token_ids):
                tokens[r.row * stride + i] = int(token)
            lengths[r.row] = len(r.prompt_token_ids)
        ret = self.library.resident_epoch_prefill(self.handle, tokens, lengths, stride)
        if ret != 0:
            raise ResidentEpochExecutionError(
                f"resident_epoch_prefill failed with status {ret}", commit_state=EpochCommitState.PREPARED, status=ret
            )
        self.prefill_transfers += 1
        return self._execute(plan, transfer_path=None, transfer_id=self.prefill_transfers, ipc=None, prefill=True)

    def close(self) -> None:
        if getattr(self, "handle", None):
            self.library.resident_epoch_destroy(self.handle)
            self.handle = None

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass

    # -- the C call ------------------------------------------------------------------
    def _call(self, *, request_count, max_steps, tokens, positions, lengths, eos, generations,
              transfer_path=None, transfer_id=0, ipc=None) -> dict[str, Any]:
        i64, i32 = ctypes.c_int64, ctypes.c_int32
        out_tokens = (i64 * (4 * MAX_EPOCH_STEPS))()
        out_executed = (i32 * 4)()
        out_gens = (i32 * 4)()
        scalars = {name: i32(-1 if name == "device_status" else 0) for name in (
            "model_calls", "device_status", "feed_calls", "fetch_calls", "commit_state", "kv_import_checksum")}
        wide = {name: i64(0) for name in ("wall_us", "native_cpu_us", "declared_input_bytes", "declared_output_bytes")}
        scalars["commit_state"] = i32(-1)
        ret = self.library.resident_epoch_execute(
            self.handle, request_count, max_steps,
            (i64 * 4)(*tokens), (i64 * 4)(*positions), (i32 * 4)(*lengths), (i32 * 4)(*eos), (i32 * 4)(*generations),
            out_tokens, out_executed, out_gens,
            ctypes.byref(scalars["model_calls"]), ctypes.byref(scalars["device_status"]),
            ctypes.byref(scalars["feed_calls"]), ctypes.byref(scalars["fetch_calls"]),
            ctypes.byref(scalars["commit_state"]), ctypes.byref(scalars["kv_import_checksum"]),
            ctypes.byref(wide["wall_us"]), ctypes.byref(wide["native_cpu_us"]),
            ctypes.byref(wide["declared_input_bytes"]), ctypes.byref(wide["declared_output_bytes"]),
            str(transfer_path).encode() if transfer_path is not None else None, transfer_id,
            ctypes.cast(ipc, ctypes.c_void_p) if ipc is not None else None,
        )
        try:
            commit_state = EpochCommitState(scalars["commit_state"].value)
        except ValueError as exc:
            raise ResidentEpochExecutionError(
                "resident_epoch_execute returned no valid commit state",
                commit_state=EpochCommitState.EXECUTING, status=ret,
            ) from exc
        result = {name: v.value for name, v in scalars.items()}
        result.update({name: v.value for name, v in wide.items()})
        result.update(ret=ret, commit_state=commit_state, tokens=list(out_tokens), executed=list(out_executed),
                      row_generations=tuple(out_gens))
        return result

    def _execute(self, plan: ResidentEpochPlan, *, transfer_path, transfer_id, ipc, prefill=False) -> NativeEpochOutput:
        if plan.graph_batch_size != 4:
            raise ValueError("the CUDA engine serves the static B=4 epoch")
        tokens, positions, lengths = [0] * 4, [0] * 4, [0] * 4
        eos = [self.config.configured_eos] * 4
        for r in plan.requests:
            tokens[r.row], positions[r.row], lengths[r.row], eos[r.row] = (
                r.token_id, r.position, r.sequence_length, r.eos_token_id)
        out = self._call(
            request_count=len(plan.requests), max_steps=plan.max_steps, tokens=tokens, positions=positions,
            lengths=lengths, eos=eos, generations=list(plan.row_generations), transfer_path=transfer_path,
            transfer_id=transfer_id, ipc=ipc,
        )
        if out["ret"] != 0:
            raise ResidentEpochExecutionError(
                f"resident_epoch_execute failed with status {out['ret']}",
                commit_state=out["commit_state"], status=out["ret"],
            )
        token_ids: dict[str, list[int]] = {}
        for r in plan.requests:
            executed = out["executed"][r.row]
            if not 0 <= executed <= plan.max_steps:
                raise ResidentEpochExecutionError(
                    "native backend returned an invalid executed count", commit_state=out["commit_state"]
                )
            base = r.row * MAX_EPOCH_STEPS
            token_ids[r.req_id] = [int(t) for t in out["tokens"][base : base + executed]]
        return NativeEpochOutput(
            status=out["device_status"], model_calls=out["model_calls"], token_ids=token_ids,
            row_generations=out["row_generations"], commit_state=out["commit_state"],
            feed_calls=out["feed_calls"], fetch_calls=out["fetch_calls"], wall_us=out["wall_us"],
            native_cpu_us=out["native_cpu_us"], declared_input_bytes=out["declared_input_bytes"],
            declared_output_bytes=out["declared_output_bytes"],
            kv_imported=transfer_path is not None or ipc is not None or prefill,
            kv_import_checksum=out["kv_import_checksum"] & 0xFFFFFFFF,
            kv_transfer_mode=("device_ipc" if ipc is not None else "host_snapshot" if transfer_path
                              else "device_prefill" if prefill else "none"),
        )


def create_cuda_engine() -> CudaEpochEngine:
    return CudaEpochEngine()
