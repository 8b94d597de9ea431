"""Which requests the greedy resident epoch may serve
(src/vllm_ascend_resident_epoch/eligibility.py:4-47).

Returns the first reason a vLLM request falls outside the device epoch's
support envelope (greedy sampling with EOS only), or None.
"""

from __future__ import annotations

from typing import Any


def request_rejection_reason(request: Any) -> str | None:
    checks = (
        (request.pooling_params is not None, "pooling-request"),
        (bool(request.mm_features), "multimodal-input"),
        (request.lora_request is not None, "lora"),
        (request.prompt_embeds is not None, "prompt-embeds"),
        (bool(request.use_structured_output), "structured-output"),
    )
    for failed, reason in checks:
        if failed:
            return reason
    params = request.sampling_params
    if params is None:
        return "missing-sampling-params"
    sampling_checks = (
        (params.temperature != 0.0, "non-greedy-temperature"),
        (params.top_p != 1.0 or params.top_k != 0 or params.min_p != 0.0, "unsupported-sampling-filter"),
        (
            params.presence_penalty != 0.0
            or params.frequency_penalty != 0.0
            or params.repetition_penalty != 1.0,
            "sampling-penalty",
        ),
        (params.min_tokens != 0, "min-tokens"),
        (bool(params.ignore_eos), "ignore-eos"),
        (params.eos_token_id is None, "missing-eos"),
        (bool(params.stop) or bool(params.stop_token_ids), "extra-stop-condition"),
        (params.logprobs is not None or params.prompt_logprobs is not None, "logprobs"),
        (bool(params.logit_bias) or bool(params.allowed_token_ids), "logit-processor"),
        (bool(params.bad_words), "bad-words"),
        (getattr(params, "repetition_detection", None) is not None, "repetition-detection"),
        (bool(params.extra_args), "extra-sampling-args"),
    )
    for failed, reason in sampling_checks:
        if failed:
            return reason
    return None
