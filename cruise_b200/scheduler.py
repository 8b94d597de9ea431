"""vLLM V1 scheduler that hands greedy single-token decode batches to the
resident epoch engine (src/vllm_ascend_resident_epoch/scheduler.py:18-366).

Each ``schedule()`` first lets vLLM schedule as usual.  When the result is an
all-decode batch of at most four supported requests, it turns the batch into
a ``ResidentEpochPlan``: fixed B=4 rows, K = the largest of 1/2/4/8 within
every request's remaining budget, paged KV by row.  The plan rides on the
``SchedulerOutput``; the worker runs it on the GPU and returns K tokens per
request with a ``ResidentEpochResult``.  ``update_from_output`` then advances
vLLM's token accounting by the K - 1 extra steps.

* Row and generation bookkeeping: a request keeps its row while it runs.  A
  new request gets a fresh generation, which the device uses to tell a
  continuing row from a new one.
* Ownership: a host-prefilled request is imported once (its first KV block
  rides along with the first epoch), then the device owns its state.  From
  then on the host must never run it.  A host-side need (a new prompt to
  prefill, or an unsupported request) is scheduled in an isolated host lane
  with the device-owned requests paused.
* Rejection reasons: every schedule without a plan records why in
  ``last_rejection`` (vocabulary of the reference).
* Device prefill (``VLLM_ASCEND_RESIDENT_EPOCH_DEVICE_PREFILL=1``; the
  reference has no such mode): a fresh greedy prompt of 2..block_size tokens
  that vLLM schedules whole goes into the plan at once with its prompt
  (``prompt_token_ids``).  The engine prefills it on the device, imports its
  K/V and decodes from its last prompt token in the same epoch, beside the
  device-owned rows, so such prompts need no host lane.  vLLM's accounting
  counts the prompt as scheduled and the epoch's K - 1 further positions as
  computed.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

from vllm.v1.core.sched.scheduler import Scheduler
from vllm.v1.outputs import ModelRunnerOutput

from .config import ResidentEpochConfig, epoch_steps
from .benchmark_metrics import ResidentEpochBenchmarkMetrics
from .contract import CONTRACT_VERSION, ResidentEpochPlan, ResidentEpochRequest, attach_plan, get_plan, get_result
from .eligibility import effective_eos, request_rejection_reason
from .model_config import PRESETS


@dataclass
class ResidentRows:
    """Which engine row and generation each resident request holds."""

    rows: dict[str, int] = field(default_factory=dict)
    generations: dict[str, int] = field(default_factory=dict)
    device_owned: set[str] = field(default_factory=set)
    next_generation: int = 1

    def assign(self, req_ids: tuple[str, ...], batch: int) -> None:
        """Releases rows of requests that left the batch, then gives every new
        request a free row and a fresh generation (scheduler.py:62-86)."""
        keep = set(req_ids)
        for req_id in [r for r in self.rows if r not in keep]:
            del self.rows[req_id]
            del self.generations[req_id]
            self.device_owned.discard(req_id)
        free = sorted(set(range(batch)) - set(self.rows.values()))
        for req_id in req_ids:
            if req_id in self.rows:
                continue
            if not free:
                raise RuntimeError("resident row allocator exhausted")
            if self.next_generation >= 2**31:
                raise RuntimeError("resident generation space exhausted")
            self.rows[req_id] = free.pop(0)
            self.generations[req_id] = self.next_generation
            self.next_generation += 1


def native_model_rejection(hf_config: Any) -> str | None:
    """None when the served model has the geometry of an engine preset."""
    if getattr(hf_config, "model_type", None) != "qwen2":
        return f"model_type={getattr(hf_config, 'model_type', None)!r}"
    for preset in PRESETS.values():
        fields = {
            "num_hidden_layers": preset.num_layers, "hidden_size": preset.hidden,
            "num_attention_heads": preset.num_heads, "num_key_value_heads": preset.num_kv_heads,
            "intermediate_size": preset.intermediate, "vocab_size": preset.vocab,
        }
        if all(getattr(hf_config, k, None) == v for k, v in fields.items()):
            return None
    return (f"no engine preset for num_hidden_layers={getattr(hf_config, 'num_hidden_layers', None)} "
            f"hidden_size={getattr(hf_config, 'hidden_size', None)} vocab_size={getattr(hf_config, 'vocab_size', None)}")


class ResidentEpochScheduler(Scheduler):
    def __init__(self, *args: Any, **kwargs: Any) -> None:
        super().__init__(*args, **kwargs)
        self.resident_config = ResidentEpochConfig.from_env()
        self.resident = ResidentRows()
        self.last_rejection: str | None = None
        self.last_plan: ResidentEpochPlan | None = None
        self.last_result: Any | None = None
        self.benchmark_metrics = ResidentEpochBenchmarkMetrics.from_env()
        if self.vllm_config.speculative_config is not None:
            raise ValueError("resident epoch scheduler cannot be combined with speculative decoding")
        if self.scheduler_config.async_scheduling:
            raise ValueError("resident epoch scheduler requires synchronous scheduling")
        parallel = self.vllm_config.parallel_config
        if parallel.tensor_parallel_size != 1 or parallel.pipeline_parallel_size != 1:
            raise ValueError("resident epoch scheduler runs one engine per vLLM instance (TP = PP = 1)")
        reason = native_model_rejection(self.vllm_config.model_config.hf_config)
        if reason is not None:
            raise ValueError(f"resident epoch native graph mismatch: {reason}")
        if self.resident_config.device_prefill:
            # vLLM must schedule every eligible prompt whole: a cached prefix, a
            # token budget smaller than a full cohort of block-size prompts or a
            # long-prefill threshold would leave part of a prompt for a host lane
            cfg, sched = self.resident_config, self.scheduler_config
            if self.cache_config.enable_prefix_caching:
                raise ValueError("resident epoch device prefill needs enable_prefix_caching=False")
            if sched.max_num_batched_tokens < cfg.max_batch_size * cfg.block_size:
                raise ValueError("resident epoch device prefill needs max_num_batched_tokens >= "
                                 f"{cfg.max_batch_size * cfg.block_size} (4 prompts of a block each)")
            threshold = getattr(sched, "long_prefill_token_threshold", 0) or 0
            if 0 < threshold < cfg.block_size:
                raise ValueError("resident epoch device prefill needs long_prefill_token_threshold 0 or >= "
                                 f"{cfg.block_size}")

    @classmethod
    def adopt(cls, scheduler: Scheduler, config: ResidentEpochConfig | None = None) -> "ResidentEpochScheduler":
        """Turns an already constructed vLLM scheduler into this class (tests and
        embedders that build the stock scheduler themselves)."""
        scheduler.__class__ = cls
        scheduler.resident_config = config or ResidentEpochConfig()
        scheduler.resident = ResidentRows()
        scheduler.last_rejection = None
        scheduler.last_plan = None
        scheduler.last_result = None
        scheduler.benchmark_metrics = ResidentEpochBenchmarkMetrics.from_env()
        return scheduler

    def _device_prefill_eligible(self, request: Any) -> bool:
        """A fresh request whose whole prompt the engine can prefill on the
        device inside its first epoch (device_prefill mode only): supported
        sampling, no output yet, 2..block_size prompt tokens."""
        cfg = self.resident_config
        return (cfg.device_prefill and request.num_output_tokens == 0
                and 2 <= request.num_prompt_tokens <= cfg.block_size
                and request_rejection_reason(request) is None)

    # -- host isolation (scheduler.py:102-162) ------------------------------------------
    def _host_lane_reason(self, device_running: tuple[Any, ...]) -> str | None:
        """Why the host must run something while device-owned requests wait."""
        if not device_running:
            return None
        host_running = [r for r in self.running if r not in device_running]
        if any(request_rejection_reason(r) is not None for r in host_running):
            return "unsupported-host-isolation"
        if any(r.num_computed_tokens < r.num_prompt_tokens for r in host_running):
            return "host-prefill-admission"
        waiting = list(self.waiting) + list(getattr(self, "skipped_waiting", ()))
        needs_host = any((r.num_prompt_tokens > 1 and not self._device_prefill_eligible(r))
                         or request_rejection_reason(r) is not None for r in waiting)
        if needs_host and len(self.running) < self.max_num_running_reqs:
            return "host-prefill-admission"
        return None

    def _schedule_lanes(self) -> tuple[Any, tuple[str, ...], str | None]:
        device_running = tuple(r for r in self.running if r.request_id in self.resident.device_owned)
        reason = self._host_lane_reason(device_running)
        if reason is None:
            return super().schedule(), (), None
        paused = device_running
        limit = self.max_num_running_reqs
        self.running[:] = [r for r in self.running if r not in paused]
        self.max_num_running_reqs = limit - len(paused)
        try:
            output = super().schedule()
        finally:
            self.running[:] = [*paused, *self.running]
            self.max_num_running_reqs = limit
        scheduled = set(output.num_scheduled_tokens)
        paused_ids = tuple(r.request_id for r in paused)
        if not scheduled:
            raise RuntimeError("isolated host lane did not schedule a request")
        if scheduled & set(paused_ids):
            raise RuntimeError("isolated host lane scheduled device-owned state")
        return output, paused_ids, reason

    # -- scheduling (scheduler.py:164-285) ------------------------------------------------
    def schedule(self):
        if self.num_lookahead_tokens != 0:
            raise RuntimeError("resident epoch lookahead conflicts with another feature")
        output, paused, lane_reason = self._schedule_lanes()
        plan, rejection = self._make_plan(output)
        if plan is None:
            stranded = set(output.num_scheduled_tokens) & self.resident.device_owned
            if stranded:
                raise RuntimeError("refusing host execution for device-owned requests: " + ",".join(sorted(stranded)))
        if paused:
            if plan is not None:
                raise RuntimeError("isolated host lane created a resident plan")
            rejection = lane_reason
        self.last_rejection, self.last_plan, self.last_result = rejection, plan, None
        self.benchmark_metrics.record_schedule(plan, rejection)
        if plan is not None:
            attach_plan(output, plan)
        else:
            output.resident_epoch_rejection = rejection   # why this step stays on the host
        return output

    def _make_plan(self, output: Any) -> tuple[ResidentEpochPlan | None, str | None]:
        cfg = self.resident_config
        req_ids = tuple(output.num_scheduled_tokens)
        # device_prefill mode: a fresh prompt scheduled whole in this step is
        # prefilled on the device inside the epoch (the engine's K/V import)
        prefill = {r for r in req_ids if self._device_prefill_eligible(self.requests[r])
                   and output.num_scheduled_tokens[r] == self.requests[r].num_prompt_tokens}
        gates = (
            (not req_ids, "empty-schedule"),
            (len(req_ids) > cfg.max_batch_size, "batch-too-large"),
            (any(output.num_scheduled_tokens[r] != 1 for r in req_ids if r not in prefill), "not-single-token-decode"),
            (bool(output.scheduled_spec_decode_tokens), "speculative-decode"),
            (bool(output.scheduled_encoder_inputs), "encoder-input"),
            (bool(output.preempted_req_ids), "preemption"),
            (self.connector is not None or getattr(self, "ec_connector", None) is not None, "cache-connector"),
            (self.block_size != cfg.block_size, "block-size"),
            (set(req_ids) != {r.request_id for r in self.running}, "partial-running-set"),
        )
        for failed, reason in gates:
            if failed:
                return None, reason
        self.resident.assign(req_ids, cfg.max_batch_size)
        requests = [self.requests[r] for r in req_ids]
        budgets = []
        for request in requests:
            reason = request_rejection_reason(request)
            if reason is not None:
                return None, reason
            owned = request.request_id in self.resident.device_owned
            if request.num_prompt_tokens > cfg.logical_capacity:
                return None, "prompt-exceeds-resident-capacity"
            if request.num_prompt_tokens > 1 and request.num_output_tokens == 0 and request.request_id not in prefill:
                return None, "host-prefill-in-progress"
            if request.num_prompt_tokens > 1 and not owned and len(self._block_ids(request)) != 1:
                return None, "multiple-kv-cache-groups"
            if request.num_computed_tokens != request.num_tokens:
                return None, "computed-token-accounting"
            remaining = request.max_tokens - request.num_output_tokens
            if remaining < 1:
                return None, "request-has-no-remaining-steps"
            budgets.append(remaining)
        steps = epoch_steps(min(cfg.max_steps, min(budgets)))
        planned = []
        mask = [0] * cfg.max_batch_size
        for request in requests:
            row = self.resident.rows[request.request_id]
            position = request.num_computed_tokens - 1   # the newest token is this epoch's input
            if position < 0 or position + steps > cfg.logical_capacity:
                return None, "logical-capacity"
            groups = self._block_ids(request)
            if len(groups) != 1:
                return None, "multiple-kv-cache-groups"
            blocks = tuple(groups[0])
            if not blocks:
                return None, "missing-kv-block"
            params = request.sampling_params
            owned = request.request_id in self.resident.device_owned
            planned.append(ResidentEpochRequest(
                req_id=request.request_id, row=row, generation=self.resident.generations[request.request_id],
                token_id=int(request.all_token_ids[position]), position=position, sequence_length=position + 1,
                eos_token_id=effective_eos(params), scheduler_block_ids=blocks,
                device_block_ids=(row * cfg.blocks_per_request, row * cfg.blocks_per_request + 1),
                state_owner="device" if owned else "host",
                kv_import_required=request.num_prompt_tokens > 1 and not owned,
                prompt_token_ids=(tuple(int(t) for t in request.prompt_token_ids)
                                  if request.request_id in prefill else ()),
            ))
            mask[row] = 1
        plan = ResidentEpochPlan(version=CONTRACT_VERSION, graph_batch_size=cfg.max_batch_size, max_steps=steps,
                                 logical_capacity=cfg.logical_capacity, requests=tuple(planned),
                                 active_mask=tuple(mask))
        plan.validate()
        return plan, None

    def _block_ids(self, request: Any):
        return self.kv_cache_manager.get_blocks(request.request_id).get_block_ids()

    # -- accounting (scheduler.py:287-366) ---------------------------------------------------
    def update_from_output(self, scheduler_output: Any, model_runner_output: ModelRunnerOutput):
        plan = get_plan(scheduler_output)
        result = get_result(model_runner_output)
        if plan is None:
            if result is not None:
                raise RuntimeError("resident epoch result has no scheduler plan")
            return super().update_from_output(scheduler_output, model_runner_output)
        if result is None:
            raise RuntimeError("resident epoch plan did not receive execution metadata")
        self.last_result = result
        self.benchmark_metrics.record_result(result)
        sampled = {r: list(model_runner_output.sampled_token_ids[model_runner_output.req_id_to_index[r]])
                   for r in plan.req_ids}
        result.validate_against(plan, sampled)
        # vLLM counts one computed token per scheduled token; an epoch computed
        # `steps` of them: credit the rest before vLLM appends the outputs
        extra = {}
        prefilled = {r.req_id for r in plan.requests if r.prompt_token_ids}
        for req_id, steps in result.computed_steps.items():
            request = self.requests[req_id]
            # a device prefill was scheduled as its whole prompt, computed with
            # the epoch's first step; a decode request as one token
            more = steps - (1 if req_id in prefilled else scheduler_output.num_scheduled_tokens[req_id])
            if more < 0:
                raise RuntimeError("resident epoch computed fewer than scheduled tokens")
            if request.num_computed_tokens + more > request.num_tokens + len(sampled[req_id]):
                raise RuntimeError("resident epoch would over-advance computed tokens")
            extra[req_id] = more
        for req_id, more in extra.items():
            self.requests[req_id].num_computed_tokens += more
        if result.route == "device":
            for request in plan.requests:
                if request.state_owner == "host":
                    self.resident.device_owned.add(request.req_id)
        return super().update_from_output(scheduler_output, model_runner_output)
