"""Python handle on the CUDA resident-epoch engine (over the C ABI).

``EpochEngine.run`` is the 8-input / 2-output epoch ABI of the reference's
device controller (``controller/g4c_b4_resident_epoch.cpp:40-49,296-324``):
one call submits the whole epoch to the GPU and returns the token history and
the 28-word control output.  PyTorch is used only for host tensors.
"""

from __future__ import annotations

import ctypes
import threading
import time
from dataclasses import dataclass
from typing import Callable

import numpy as np
import torch

from . import _lib
from .model_config import BATCH, MAX_STEPS, PRESETS, ModelConfig, TpShard, layer_tensor_names

CONTROL_IN = 11
CONTROL_OUT = 28
TILING_BYTES = 72


def _ptr(array: np.ndarray, ctype):
    return array.ctypes.data_as(ctypes.POINTER(ctype))


def rope_tables(config: ModelConfig) -> tuple[torch.Tensor, torch.Tensor]:
    """bf16 cos / sin tables [capacity, head_dim] computed exactly as the
    reference's ``rope`` (``batched_decoder_step.py:212-216,235-240``)."""
    d = config.head_dim
    inv_freq = 1.0 / (config.rope_theta ** (torch.arange(0, d, 2, dtype=torch.float32) / d))
    positions = torch.arange(config.capacity, dtype=torch.int64)
    frequencies = positions.float().reshape(-1, 1) * inv_freq.view(1, -1)
    embedding = torch.cat((frequencies, frequencies), dim=-1)
    return embedding.cos().to(torch.bfloat16), embedding.sin().to(torch.bfloat16)


@dataclass
class EpochOutput:
    history: np.ndarray        # i64 [8, 4] step-major, -1 filled
    control_out: np.ndarray    # i32 [28]
    logits: np.ndarray | None  # f32 [8, 4, V] when requested (a TP rank fills its vocabulary rows [v0, v0+nv))
    device_us: float           # CUDA-event time of the epoch kernel

    @property
    def status(self) -> int:
        return int(self.control_out[3])

    @property
    def model_calls(self) -> int:
        return int(self.control_out[4])


class EngineError(RuntimeError):
    pass


class EpochEngine:
    def __init__(self, config: ModelConfig | str, device: int = 0, tp_rank: int = 0, tp_size: int = 1) -> None:
        self.config = PRESETS[config] if isinstance(config, str) else config
        self.lib = _lib.load()
        self.shard = TpShard.of(self.config, tp_rank, tp_size)
        status = ctypes.c_int32(-1)
        c_config = self.config.to_c()
        if tp_size > 1:
            self.handle = self.lib.cruise_epoch_create_tp(ctypes.byref(c_config), device, tp_rank, tp_size,
                                                          ctypes.byref(status))
        else:
            self.handle = self.lib.cruise_epoch_create(ctypes.byref(c_config), device, ctypes.byref(status))
        if not self.handle or status.value != 0:
            detail = self.lib.cruise_epoch_last_error(None).decode()
            raise EngineError(f"cruise_epoch_create failed with status {status.value}: {detail}")
        self.device = device
        cos, sin = rope_tables(self.config)
        self._check(
            self.lib.cruise_epoch_set_rope_table(
                self.handle,
                cos.view(torch.int16).numpy().ctypes.data,
                sin.view(torch.int16).numpy().ctypes.data,
                cos.numel() * 2,
            ),
            "set_rope_table",
        )

    # -- lifecycle -------------------------------------------------------------
    def close(self) -> None:
        if getattr(self, "handle", None):
            self.lib.cruise_epoch_destroy(self.handle)
            self.handle = None

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc: int, what: str) -> None:
        if rc != 0:
            detail = self.lib.cruise_epoch_last_error(self.handle)
            raise EngineError(f"{what} failed ({rc}): {detail.decode() if detail else ''}")

    # -- weights -----------------------------------------------------------------
    def init_synthetic(self, seed: int, std: float = 0.02) -> None:
        self._check(self.lib.cruise_epoch_init_synthetic(self.handle, seed, std), "init_synthetic")

    def set_weight(self, name: str, tensor: torch.Tensor) -> None:
        value = tensor.detach().to(torch.bfloat16).contiguous().cpu()
        raw = value.view(torch.int16).numpy()
        self._check(
            self.lib.cruise_epoch_set_weight(self.handle, name.encode(), raw.ctypes.data, raw.nbytes),
            f"set_weight({name})",
        )

    def get_weight(self, name: str, shape: tuple[int, ...]) -> torch.Tensor:
        out = np.empty(shape, dtype=np.int16)
        self._check(
            self.lib.cruise_epoch_get_weight(self.handle, name.encode(), out.ctypes.data, out.nbytes),
            f"get_weight({name})",
        )
        return torch.from_numpy(out).view(torch.bfloat16)

    def load_weights(self, weights: dict[str, torch.Tensor]) -> None:
        """Loads whole checkpoint tensors (this rank's shards under tensor parallelism)."""
        for name in layer_tensor_names(self.config.num_layers):
            full = weights[name]
            self.set_weight(name, self.shard.slice_tensor(self.config, name, full) if self.shard.size > 1 else full)

    # -- tensor parallelism -------------------------------------------------------------
    def tp_handle(self) -> bytes:
        """The 64-byte IPC handle of this rank's exchange block."""
        buf = ctypes.create_string_buffer(64)
        self._check(self.lib.cruise_epoch_tp_handle(self.handle, buf), "tp_handle")
        return buf.raw

    def tp_connect(self, handles: list[bytes]) -> None:
        """Maps the other ranks' exchange blocks (handles in rank order)."""
        raw = b"".join(handles)
        self._check(self.lib.cruise_epoch_tp_connect(self.handle, raw), "tp_connect")

    # -- KV cache ------------------------------------------------------------------
    def read_kv(self) -> tuple[torch.Tensor, torch.Tensor]:
        """The resident K and V caches, bf16 [layers][blocks][block_size][kv
        heads][head_dim]; a tensor-parallel rank holds (and returns) its KV heads."""
        shape = self.shard.kv_cache_shape(self.config)
        key = np.empty(shape, dtype=np.int16)
        value = np.empty(shape, dtype=np.int16)
        self._check(
            self.lib.cruise_epoch_read_kv(self.handle, key.ctypes.data, value.ctypes.data, key.nbytes),
            "read_kv",
        )
        return torch.from_numpy(key).view(torch.bfloat16), torch.from_numpy(value).view(torch.bfloat16)

    def write_kv(self, key: torch.Tensor, value: torch.Tensor) -> None:
        k = key.to(torch.bfloat16).contiguous().view(torch.int16).numpy()
        v = value.to(torch.bfloat16).contiguous().view(torch.int16).numpy()
        self._check(
            self.lib.cruise_epoch_write_kv(self.handle, k.ctypes.data, v.ctypes.data, k.nbytes), "write_kv"
        )

    # -- one epoch (8-in / 2-out ABI) ------------------------------------------------
    def run(
        self,
        token,
        position,
        seq_len,
        slot,
        active,
        block_table,
        control,
        import_payload: torch.Tensor | bytes | None = None,
        want_logits: bool = False,
        tiling: np.ndarray | None = None,
        forced: np.ndarray | None = None,
    ) -> EpochOutput:
        cfg = self.config
        token = np.ascontiguousarray(np.asarray(token, dtype=np.int64).reshape(BATCH))
        position = np.ascontiguousarray(np.asarray(position, dtype=np.int64).reshape(BATCH))
        seq_len = np.ascontiguousarray(np.asarray(seq_len, dtype=np.int32).reshape(BATCH))
        slot = np.ascontiguousarray(np.asarray(slot, dtype=np.int32).reshape(BATCH))
        active = np.ascontiguousarray(np.asarray(active, dtype=np.int32).reshape(BATCH))
        block_table = np.ascontiguousarray(
            np.asarray(block_table, dtype=np.int32).reshape(BATCH * cfg.blocks_per_row)
        )
        control = np.ascontiguousarray(np.asarray(control, dtype=np.int32).reshape(CONTROL_IN))
        tiling_arr = np.zeros(TILING_BYTES, dtype=np.uint8) if tiling is None else np.ascontiguousarray(
            np.asarray(tiling, dtype=np.uint8).reshape(TILING_BYTES)
        )
        history = np.empty((MAX_STEPS, BATCH), dtype=np.int64)
        control_out = np.empty(CONTROL_OUT, dtype=np.int32)
        logits = np.empty((MAX_STEPS, BATCH, cfg.vocab), dtype=np.float32) if want_logits else None
        forced_arr = None
        if forced is not None:
            forced_arr = np.ascontiguousarray(np.asarray(forced, dtype=np.int64).reshape(MAX_STEPS, BATCH))
        payload_ptr, payload_bytes, keep = None, 0, None
        if import_payload is not None:
            if isinstance(import_payload, torch.Tensor):
                keep = import_payload.detach().contiguous().cpu().view(torch.uint8).numpy()
            else:
                keep = np.frombuffer(import_payload, dtype=np.uint8)
            payload_ptr, payload_bytes = keep.ctypes.data, keep.nbytes
        rc = self.lib.cruise_epoch_run(
            self.handle,
            _ptr(token, ctypes.c_int64), _ptr(position, ctypes.c_int64), _ptr(seq_len, ctypes.c_int32),
            _ptr(slot, ctypes.c_int32), _ptr(active, ctypes.c_int32), _ptr(block_table, ctypes.c_int32),
            _ptr(tiling_arr, ctypes.c_uint8), _ptr(control, ctypes.c_int32),
            payload_ptr, payload_bytes,
            _ptr(forced_arr, ctypes.c_int64) if forced_arr is not None else None,
            _ptr(history, ctypes.c_int64), _ptr(control_out, ctypes.c_int32),
            _ptr(logits, ctypes.c_float) if logits is not None else None,
        )
        self._check(rc, "cruise_epoch_run")
        device_us = ctypes.c_double(0.0)
        launches = ctypes.c_int32(0)
        self.lib.cruise_epoch_last_timing(self.handle, ctypes.byref(device_us), ctypes.byref(launches))
        return EpochOutput(history, control_out, logits, float(device_us.value))

    # -- one decoder step (9-in / 4-out decoder ABI) ---------------------------------
    def decoder_step(self, token, position, seq_len, slot, active, block_table, key: torch.Tensor | None = None,
                     value: torch.Tensor | None = None, logits_out: np.ndarray | None = None
                     ) -> tuple[np.ndarray, np.ndarray]:
        """One decoder call, no controller (``cruise_decoder_step``): returns the
        f32 logits [4, V] and the next positions [4].  ``key`` / ``value`` are
        caller-held bf16 CUDA caches in the engine's layout (updated in place),
        or None for the engine's resident caches.  ``logits_out`` may be a
        preallocated f32 [4, V] array (for example a view of pinned memory)."""
        cfg = self.config
        token = np.ascontiguousarray(np.asarray(token, dtype=np.int64).reshape(BATCH))
        position = np.ascontiguousarray(np.asarray(position, dtype=np.int64).reshape(BATCH))
        seq_len = np.ascontiguousarray(np.asarray(seq_len, dtype=np.int32).reshape(BATCH))
        slot = np.ascontiguousarray(np.asarray(slot, dtype=np.int32).reshape(BATCH))
        active = np.ascontiguousarray(np.asarray(active, dtype=np.int32).reshape(BATCH))
        block_table = np.ascontiguousarray(
            np.asarray(block_table, dtype=np.int32).reshape(BATCH * cfg.blocks_per_row))
        logits = np.empty((BATCH, cfg.vocab), dtype=np.float32) if logits_out is None else logits_out
        if logits.shape != (BATCH, cfg.vocab) or logits.dtype != np.float32 or not logits.flags.c_contiguous:
            raise ValueError(f"logits_out must be a contiguous float32 [{BATCH}, {cfg.vocab}] array")
        next_position = np.empty(BATCH, dtype=np.int64)
        caches = []
        for cache in (key, value):
            if cache is None:
                caches.append(None)
                continue
            if (not cache.is_cuda or cache.dtype != torch.bfloat16 or not cache.is_contiguous()
                    or tuple(cache.shape) != self.shard.kv_cache_shape(cfg)):
                raise ValueError(f"caches must be contiguous bf16 CUDA tensors of shape {self.shard.kv_cache_shape(cfg)}")
            caches.append(ctypes.c_void_p(cache.data_ptr()))
        rc = self.lib.cruise_decoder_step(
            self.handle, _ptr(token, ctypes.c_int64), _ptr(position, ctypes.c_int64), _ptr(seq_len, ctypes.c_int32),
            caches[0], _ptr(slot, ctypes.c_int32), _ptr(active, ctypes.c_int32), _ptr(block_table, ctypes.c_int32),
            caches[1], None, _ptr(logits, ctypes.c_float), _ptr(next_position, ctypes.c_int64),
        )
        self._check(rc, "cruise_decoder_step")
        return logits, next_position

    # -- batched device prefill -------------------------------------------------------
    def prefill(self, prompts) -> None:
        """Runs up to four prompts (row r <- prompts[r]; an empty prompt leaves the
        row alone) through the model on the GPU and keeps the K/V of all but
        each prompt's last token as the device-side import payload: the next
        :meth:`run` with the import flag and no ``import_payload`` imports it
        and decodes from the last prompt token (see tests/scenario.py:
        decode_inputs(importing=True))."""
        prompts = [list(map(int, p)) for p in prompts] + [[]] * (BATCH - len(prompts))
        if len(prompts) != BATCH:
            raise ValueError(f"at most {BATCH} prompts")
        stride = max(1, max(len(p) for p in prompts))
        tokens = np.zeros((BATCH, stride), dtype=np.int64)
        lens = np.zeros(BATCH, dtype=np.int32)
        for r, prompt in enumerate(prompts):
            tokens[r, : len(prompt)] = prompt
            lens[r] = len(prompt)
        self._check(self.lib.cruise_epoch_prefill(self.handle, tokens.ctypes.data, lens.ctypes.data, stride),
                    "prefill")

    # -- streaming egress ------------------------------------------------------------
    def run_streaming(self, on_step: Callable[[int, np.ndarray], None], poll_s: float = 5e-5,
                      **run_kwargs) -> EpochOutput:
        """One epoch exactly like :meth:`run`, while this thread hands every
        decode step's tokens (int64[4], -1 for rows that did not run) to
        ``on_step(step, tokens)`` in step order as soon as the device published
        them -- before the epoch ends.  The epoch itself runs on a helper
        thread (the C call releases the GIL)."""
        self._check(self.lib.cruise_epoch_stream_enable(self.handle, 1), "stream_enable")
        launch = self.lib.cruise_epoch_stream_next_id(self.handle)
        result: dict = {}

        def epoch() -> None:
            try:
                result["out"] = self.run(**run_kwargs)
            except BaseException as exc:   # re-raised on the caller's thread
                result["err"] = exc

        worker = threading.Thread(target=epoch, name="cruise-epoch", daemon=True)
        worker.start()
        tokens = np.empty((MAX_STEPS, BATCH), dtype=np.int64)
        seen = 0
        while True:
            running = worker.is_alive()
            n = self.lib.cruise_epoch_stream_poll(self.handle, launch, tokens.ctypes.data)
            while seen < n:
                on_step(seen, tokens[seen].copy())
                seen += 1
            if not running:
                break
            time.sleep(poll_s)
        worker.join()
        self._check(self.lib.cruise_epoch_stream_enable(self.handle, 0), "stream_enable")
        if "err" in result:
            raise result["err"]
        return result["out"]

    def set_trace(self, enable: bool | int) -> None:
        """True / 1: CTA 0's phase timeline; 2: also every CTA's (read_trace_cta)."""
        self._check(self.lib.cruise_epoch_set_trace(self.handle, int(enable)), "set_trace")

    def read_trace_cta(self, barriers: int) -> np.ndarray:
        """[barriers, ctas, 8] low 32 bits of globaltimer ns per CTA (0: not
        recorded): left barrier j, staged, last tile, arrived at barrier j;
        the epilogue warp's start, ns it waited for the stream-K partner,
        last segment done, outputs fenced, last consumer flush received; the
        last consumer warp's last tile (see cruise_epoch_read_trace_cta)."""
        ctas = ctypes.c_int32(0)
        self.lib.cruise_epoch_read_trace_cta(self.handle, None, 0, ctypes.byref(ctas))
        out = np.zeros((barriers, max(ctas.value, 1), 12), dtype=np.uint32)
        self._check(self.lib.cruise_epoch_read_trace_cta(self.handle, _ptr(out, ctypes.c_uint32), barriers,
                                                         ctypes.byref(ctas)), "read_trace_cta")
        return out

    def read_trace(self, count: int) -> np.ndarray:
        """[6, count] globaltimer ns per grid barrier of the last epoch: CTA 0
        exit, CTA 0 entry, activations staged, last tile consumed, last arrival,
        and (a duration) CTA 0's wait for other tensor-parallel ranks (or 0)."""
        out = np.zeros((6, count), dtype=np.uint64)
        for series in range(6):
            self._check(
                self.lib.cruise_epoch_read_trace(self.handle, series, _ptr(out[series], ctypes.c_uint64), count),
                "read_trace",
            )
        return out

    def last_timing(self) -> tuple[float, int]:
        device_us = ctypes.c_double(0.0)
        launches = ctypes.c_int32(0)
        self.lib.cruise_epoch_last_timing(self.handle, ctypes.byref(device_us), ctypes.byref(launches))
        return float(device_us.value), int(launches.value)
