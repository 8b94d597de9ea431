"""Which requests the greedy resident epoch may serve
(src/vllm_ascend_resident_epoch/eligibility.py:4-47).

Returns the first reason a vLLM request falls outside the device epoch's
support envelope (greedy sampling with EOS only), or None.  One extension
over the reference: a request served without a tokenizer has no EOS id in
vLLM and carries the model's generation-config EOS as its single stop token
id; that token then acts as the request's EOS (``effective_eos``).
"""

from __future__ import annotations

from typing import Any


def effective_eos(params: Any) -> int | None:
    """The one token that ends a greedy request on the device: its EOS id; or,
    for a request served without a tokenizer (vLLM then has no EOS id and
    carries the model's generation-config EOS as the single stop token id),
    that stop token.  None when anything else could also stop it."""
    stop_ids = set(params.stop_token_ids or ())
    if params.eos_token_id is not None:
        return int(params.eos_token_id) if not stop_ids else None
    return int(next(iter(stop_ids))) if len(stop_ids) == 1 else None


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
        (params.eos_token_id is None and not params.stop_token_ids, "missing-eos"),
        (bool(params.stop) or effective_eos(params) is None, "extra-stop-condition"),
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
