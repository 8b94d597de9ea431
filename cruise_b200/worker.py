"""Dedicated vLLM V1 worker for the resident decode-epoch engine.

The worker the reference plugs into vLLM (src/vllm_ascend_resident_epoch/worker.py:19-163)
hands model and KV ownership to its native engine; this one does the same for
the B200 engine.  vLLM's own model runner is never built:

* the model is the engine behind the backend named by
  ``VLLM_ASCEND_RESIDENT_EPOCH_BACKEND_FACTORY`` (``cruise_b200.cuda_backend:
  create_cuda_engine`` in this process, ``cruise_b200.sidecar_backend:
  create_sidecar_engine`` in a sidecar);
* the KV cache the scheduler allocates from is exactly the engine's resident
  paged cache (:class:`ResidentKVLayout`), so block ids the scheduler hands out
  are rows of the engine's cache;
* ``execute_model`` runs the epoch plan the ``ResidentEpochScheduler`` attached
  to the scheduler output.  Work outside the resident envelope never reaches
  this worker (the scheduler keeps it on its host lane), so receiving some is
  an error, not a fallback.

Select it with ``--worker-cls cruise_b200.worker.ResidentEpochWorker`` and
``--scheduler-cls cruise_b200.scheduler.ResidentEpochScheduler``.
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Any

import torch
from vllm.v1.kv_cache_interface import FullAttentionSpec, KVCacheConfig, KVCacheSpec
from vllm.v1.outputs import ModelRunnerOutput
from vllm.v1.worker.worker_base import CompilationTimes, WorkerBase

from .backend import NativeWarmupOutput, ResidentEpochBackend, load_backend_from_env
from .config import ResidentEpochConfig
from .contract import get_plan
from .model_config import PRESETS, ModelConfig

RESIDENT_WORKER_QUALNAME = "cruise_b200.worker.ResidentEpochWorker"


@dataclass(frozen=True)
class ResidentKVLayout:
    """The engine's resident cache seen as vLLM KV-cache groups: one
    full-attention layer spec per decoder layer, as many physical blocks as
    the engine holds, bf16 K and V."""

    model: ModelConfig
    block_size: int
    physical_blocks: int

    def layer_spec(self) -> FullAttentionSpec:
        return FullAttentionSpec(block_size=self.block_size, num_kv_heads=self.model.num_kv_heads,
                                 head_size=self.model.head_dim, dtype=torch.bfloat16)

    def specs(self) -> dict[str, KVCacheSpec]:
        spec = self.layer_spec()
        return {f"model.layers.{i}.self_attn": spec for i in range(self.model.num_layers)}

    def bytes_per_block(self) -> int:
        """One block of every layer (K and V), the scheduler's unit of memory."""
        return self.layer_spec().page_size_bytes * self.model.num_layers

    def capacity_bytes(self) -> int:
        """What the scheduler may allocate: the engine's blocks plus one.
        vLLM's block pool keeps one block back as its null block, and every
        row must be able to hold its blocks_per_row blocks at once, else vLLM
        preempts a device-owned request once all rows have grown.  The
        scheduler's block ids never address device memory (a row's blocks are
        fixed by its row), so the extra block costs nothing."""
        return (self.physical_blocks + 1) * self.bytes_per_block()

    def check(self, config: KVCacheConfig) -> None:
        """Raises unless the scheduler's KV configuration maps onto the engine's cache."""
        problems = []
        if config.num_blocks < self.physical_blocks:
            problems.append(f"{config.num_blocks} scheduler blocks < {self.physical_blocks} engine blocks")
        if len(config.kv_cache_groups) != 1:
            problems.append(f"{len(config.kv_cache_groups)} KV cache groups (the engine has one)")
        elif config.kv_cache_groups[0].kv_cache_spec.block_size != self.block_size:
            problems.append(f"block size {config.kv_cache_groups[0].kv_cache_spec.block_size} "
                            f"(the engine's is {self.block_size})")
        if problems:
            raise ValueError("KV cache configuration does not fit the resident engine: " + "; ".join(problems))


class ResidentEpochWorker(WorkerBase):
    """vLLM worker whose model runner is the resident epoch engine."""

    def __init__(self, *args: Any, **kwargs: Any) -> None:
        super().__init__(*args, **kwargs)
        pc = self.parallel_config
        if (pc.tensor_parallel_size, pc.pipeline_parallel_size) != (1, 1):
            raise ValueError("the resident epoch worker drives one engine: tensor and pipeline parallel size 1 "
                             f"(got {pc.tensor_parallel_size} and {pc.pipeline_parallel_size})")
        settings = ResidentEpochConfig.from_env()
        model = PRESETS[os.getenv("VLLM_ASCEND_RESIDENT_EPOCH_MODEL", "qwen2.5-7b")]
        self.resident_config = settings
        self.model_preset = model
        self.layout = ResidentKVLayout(model, settings.block_size, settings.physical_blocks)
        self.backend: ResidentEpochBackend | None = None
        self.warmup_output: NativeWarmupOutput | None = None
        self.kv_cache_config: KVCacheConfig | None = None
        self._created_process_groups = False

    # -- bring-up ------------------------------------------------------------------
    def init_device(self) -> None:
        """The engine owns its CUDA context and stream.  vLLM still expects its
        world and model-parallel groups; a single-rank gloo world serves them
        when this class is the configured worker (no tensor traffic uses it)."""
        if self.parallel_config.worker_cls == RESIDENT_WORKER_QUALNAME:
            self._join_bookkeeping_groups()
        self.device = torch.device(f"cuda:{self.local_rank}" if torch.cuda.is_available() else "cpu")

    def _join_bookkeeping_groups(self) -> None:
        from vllm.distributed.parallel_state import ensure_model_parallel_initialized, init_distributed_environment

        pc = self.parallel_config
        if not torch.distributed.is_initialized():
            init_distributed_environment(world_size=pc.world_size, rank=self.rank,
                                         distributed_init_method=self.distributed_init_method,
                                         local_rank=self.local_rank, backend="gloo")
            self._created_process_groups = True
        ensure_model_parallel_initialized(pc.tensor_parallel_size, pc.pipeline_parallel_size,
                                          pc.prefill_context_parallel_size, pc.decode_context_parallel_size,
                                          backend="gloo")

    def load_model(self, *, load_dummy_weights: bool = False) -> None:
        if load_dummy_weights:
            raise ValueError("the resident epoch engine loads its own weights (seeded synthetic or a checkpoint)")
        self.backend = load_backend_from_env()

    def _loaded_backend(self) -> ResidentEpochBackend:
        if self.backend is None:
            raise RuntimeError("the resident epoch backend is not loaded (load_model first)")
        return self.backend

    # -- KV cache ------------------------------------------------------------------
    def get_kv_cache_spec(self) -> dict[str, KVCacheSpec]:
        return self.layout.specs()

    def determine_available_memory(self) -> int:
        return self.layout.capacity_bytes()

    def initialize_from_config(self, kv_cache_config: KVCacheConfig) -> None:
        self.layout.check(kv_cache_config)
        self.kv_cache_config = kv_cache_config

    def get_cache_block_size_bytes(self) -> int:
        return self.layout.bytes_per_block()

    def compile_or_warm_up_model(self) -> CompilationTimes:
        self.warmup_output = self._loaded_backend().warm_up()
        return CompilationTimes(language_model=self.warmup_output.wall_us / 1e6, encoder=0.0)

    # -- execution -----------------------------------------------------------------
    def execute_model(self, scheduler_output: Any):
        plan = get_plan(scheduler_output)
        if plan is not None:
            return self._loaded_backend().execute(plan)
        if scheduler_output.total_num_scheduled_tokens == 0:
            return ModelRunnerOutput(req_ids=[], req_id_to_index={}, sampled_token_ids=[])
        reason = getattr(scheduler_output, "resident_epoch_rejection", None)
        raise RuntimeError("the dedicated resident epoch worker received work outside the native envelope "
                           f"(scheduler: {reason})")

    def sample_tokens(self, grammar_output: Any):
        raise RuntimeError("the resident epoch worker returns its sampled tokens from execute_model")

    def get_supported_tasks(self) -> tuple[str, ...]:
        return ("generate",)

    # -- operations this worker has nothing to do for --------------------------------
    def get_kv_connector_handshake_metadata(self) -> dict | None:
        return None   # the engine's cache is not shared through a vLLM KV connector

    def reset_mm_cache(self) -> None:
        return None

    def reset_encoder_cache(self) -> None:
        return None

    def execute_dummy_batch(self) -> None:
        return None   # no collective with other workers to keep in step

    def take_draft_token_ids(self):
        return None

    def profile(self, is_start: bool = True, profile_prefix: str | None = None) -> None:
        return None   # the engine's own phase trace: cruise_epoch_set_trace / bench.py --trace

    def remove_lora(self, lora_id: int) -> bool:
        return False

    def pin_lora(self, lora_id: int) -> bool:
        return False

    def list_loras(self) -> set[int]:
        return set()

    # -- operations outside the envelope ---------------------------------------------
    def get_model(self):
        raise RuntimeError("the resident epoch model lives in the engine, not in a torch.nn.Module")

    def add_lora(self, lora_request: Any) -> bool:
        raise RuntimeError("LoRA adapters are outside the resident epoch envelope")

    def update_max_model_len(self, max_model_len: int) -> None:
        if max_model_len != self.model_config.max_model_len:
            raise ValueError("the resident epoch engine's capacity is fixed; the model length cannot change")

    # -- teardown --------------------------------------------------------------------
    def shutdown(self) -> None:
        backend, self.backend = self.backend, None
        close = getattr(getattr(backend, "engine", None), "close", None)
        if callable(close):
            close()
        if self._created_process_groups:
            from vllm.distributed.parallel_state import destroy_distributed_environment, destroy_model_parallel

            destroy_model_parallel()
            destroy_distributed_environment()
            self._created_process_groups = False
