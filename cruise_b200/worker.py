"""Dedicated vLLM V1 worker whose model and KV cache are the resident epoch
engine's (src/vllm_ascend_resident_epoch/worker.py:19-163).

vLLM's own model runner is never built: ``load_model`` binds the native
backend named by ``VLLM_ASCEND_RESIDENT_EPOCH_BACKEND_FACTORY`` (for this
engine ``cruise_b200.cuda_backend:create_cuda_engine`` in-process, or
``cruise_b200.sidecar_backend:create_sidecar_engine`` out of process), the KV
cache spec mirrors the engine's paged cache, and ``execute_model`` runs the
plan the ``ResidentEpochScheduler`` attached.  Anything outside the resident
envelope reaching this worker is an error: the scheduler isolates host work,
and a dedicated worker has no host model to run it on.

Select it with ``--worker-cls cruise_b200.worker.ResidentEpochWorker`` and
``--scheduler-cls cruise_b200.scheduler.ResidentEpochScheduler``.
"""

from __future__ import annotations

import os
from typing import Any

import torch
from vllm.v1.kv_cache_interface import FullAttentionSpec, KVCacheConfig, KVCacheSpec
from vllm.v1.outputs import ModelRunnerOutput
from vllm.v1.worker.worker_base import CompilationTimes, WorkerBase

from .backend import NativeWarmupOutput, ResidentEpochBackend, load_backend_from_env
from .config import ResidentEpochConfig
from .contract import get_plan
from .model_config import PRESETS

RESIDENT_WORKER_QUALNAME = "cruise_b200.worker.ResidentEpochWorker"


class ResidentEpochWorker(WorkerBase):
    def __init__(self, *args: Any, **kwargs: Any) -> None:
        super().__init__(*args, **kwargs)
        self.resident_config = ResidentEpochConfig.from_env()
        self.model_preset = PRESETS[os.getenv("VLLM_ASCEND_RESIDENT_EPOCH_MODEL", "qwen2.5-7b")]
        self.backend: ResidentEpochBackend | None = None
        self.warmup_output: NativeWarmupOutput | None = None
        self.kv_cache_config: KVCacheConfig | None = None
        self._owns_distributed_environment = False
        if self.parallel_config.tensor_parallel_size != 1 or self.parallel_config.pipeline_parallel_size != 1:
            raise ValueError("the resident epoch worker runs one engine (TP = PP = 1)")

    def init_device(self) -> None:
        # the engine owns its CUDA context and streams; vLLM only needs its
        # (single-rank, gloo) process groups for bookkeeping
        if self.parallel_config.worker_cls == RESIDENT_WORKER_QUALNAME:
            from vllm.distributed.parallel_state import (
                ensure_model_parallel_initialized,
                init_distributed_environment,
            )

            if not torch.distributed.is_initialized():
                init_distributed_environment(world_size=self.parallel_config.world_size, rank=self.rank,
                                             distributed_init_method=self.distributed_init_method,
                                             local_rank=self.local_rank, backend="gloo")
                self._owns_distributed_environment = True
            ensure_model_parallel_initialized(
                self.parallel_config.tensor_parallel_size, self.parallel_config.pipeline_parallel_size,
                self.parallel_config.prefill_context_parallel_size,
                self.parallel_config.decode_context_parallel_size, backend="gloo")
        self.device = torch.device(f"cuda:{self.local_rank}" if torch.cuda.is_available() else "cpu")

    def load_model(self, *, load_dummy_weights: bool = False) -> None:
        if load_dummy_weights:
            raise ValueError("the resident epoch worker loads its own weights (synthetic or a checkpoint)")
        self.backend = load_backend_from_env()

    def get_kv_cache_spec(self) -> dict[str, KVCacheSpec]:
        m = self.model_preset
        spec = FullAttentionSpec(block_size=self.resident_config.block_size, num_kv_heads=m.num_kv_heads,
                                 head_size=m.head_dim, dtype=torch.bfloat16)
        return {f"model.layers.{layer}.self_attn": spec for layer in range(m.num_layers)}

    def determine_available_memory(self) -> int:
        # exactly the engine's resident blocks: the scheduler must not hand out more
        page = next(iter(self.get_kv_cache_spec().values())).page_size_bytes
        return self.resident_config.physical_blocks * self.model_preset.num_layers * page

    def initialize_from_config(self, kv_cache_config: KVCacheConfig) -> None:
        if kv_cache_config.num_blocks < self.resident_config.physical_blocks:
            raise ValueError("scheduler KV capacity is smaller than the engine's resident cache")
        if len(kv_cache_config.kv_cache_groups) != 1:
            raise ValueError("the resident epoch worker requires one KV cache group")
        if kv_cache_config.kv_cache_groups[0].kv_cache_spec.block_size != self.resident_config.block_size:
            raise ValueError(f"the resident epoch worker requires {self.resident_config.block_size}-token KV blocks")
        self.kv_cache_config = kv_cache_config

    def compile_or_warm_up_model(self) -> CompilationTimes:
        if self.backend is None:
            raise RuntimeError("resident epoch backend is not loaded")
        self.warmup_output = self.backend.warm_up()
        return CompilationTimes(language_model=self.warmup_output.wall_us / 1_000_000, encoder=0.0)

    def execute_model(self, scheduler_output: Any):
        plan = get_plan(scheduler_output)
        if plan is None:
            if scheduler_output.total_num_scheduled_tokens == 0:
                return ModelRunnerOutput(req_ids=[], req_id_to_index={}, sampled_token_ids=[])
            reason = getattr(scheduler_output, "resident_epoch_rejection", None)
            raise RuntimeError("dedicated resident epoch worker received a request outside the native envelope"
                               f" (scheduler: {reason})")
        if self.backend is None:
            raise RuntimeError("resident epoch backend is not loaded")
        return self.backend.execute(plan)

    def get_supported_tasks(self) -> tuple[str, ...]:
        return ("generate",)

    def get_kv_connector_handshake_metadata(self) -> dict | None:
        return None   # the engine's KV cache is not shared through a vLLM connector

    def reset_mm_cache(self) -> None:
        return None

    def reset_encoder_cache(self) -> None:
        return None

    def execute_dummy_batch(self) -> None:
        return None   # nothing to keep in step with: the engine has no collective with other workers

    def take_draft_token_ids(self):
        return None

    def profile(self, is_start: bool = True, profile_prefix: str | None = None) -> None:
        return None   # the engine's own trace: cruise_epoch_set_trace / bench.py --trace

    def sample_tokens(self, grammar_output: Any):
        raise RuntimeError("the resident epoch worker returns sampled tokens with execute_model")

    def get_cache_block_size_bytes(self) -> int:
        return sum(spec.page_size_bytes for spec in self.get_kv_cache_spec().values())

    def get_model(self):
        raise RuntimeError("the resident epoch model is not a torch.nn.Module")

    def add_lora(self, lora_request: Any) -> bool:
        raise RuntimeError("LoRA is outside the resident epoch envelope")

    def remove_lora(self, lora_id: int) -> bool:
        return False

    def pin_lora(self, lora_id: int) -> bool:
        return False

    def list_loras(self) -> set[int]:
        return set()

    def update_max_model_len(self, max_model_len: int) -> None:
        if max_model_len != self.model_config.max_model_len:
            raise ValueError("the resident epoch worker does not resize its model length")

    def shutdown(self) -> None:
        if self.backend is not None:
            close = getattr(self.backend.engine, "close", None)
            if callable(close):
                close()
            self.backend = None
        if self._owns_distributed_environment:
            from vllm.distributed.parallel_state import destroy_distributed_environment, destroy_model_parallel

            destroy_model_parallel()
            destroy_distributed_environment()
            self._owns_distributed_environment = False
