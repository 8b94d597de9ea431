"""Paged Qwen2 decoder step on the CPU (test infrastructure only).

Restates ``PagedQwenDecoderStep`` of the reference
(``history/attempts/g4c-attempt69c-b4-air/batched_decoder_step.py:197-417``)
for any Qwen2 geometry, with the same torch operations in the same order so
that, in bf16 mode, it reproduces the reference module's CPU results bit for
bit:

* ``rms_norm``          ``:224-229``
* ``rotate_half``/rope  ``:231-240``
* cache update/gather   ``:242-275`` (logical window = the whole row capacity)
* QKV ``F.linear``      ``:305-313`` (``g4a_linear_t_bias.py:18-21``)
* ``exact_qk``          ``:356-366`` (``export_qk_attempt50_air.py:47-56``:
                        per-row batched q.K^T with a bf16 result)
* scale/mask/softmax    ``:367-377``; barrier/materialize are identities
* ``mm_t``              ``:380-386,391-403,406-408`` (``g4a_linear_t.py:17-18``)

``dtype=torch.float32`` runs the same graph with every bf16 rounding point
removed (the fp32 CPU case of the tiny configuration).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from .model import OracleConfig


class OracleDecoder:
    def __init__(
        self,
        cfg: OracleConfig,
        weights: dict[str, torch.Tensor],
        dtype: torch.dtype = torch.bfloat16,
    ) -> None:
        self.cfg = cfg
        self.dtype = dtype
        self.w = {name: value.to(dtype).contiguous() for name, value in weights.items()}
        d = cfg.head_dim
        self.inv_freq = 1.0 / (
            cfg.rope_theta ** (torch.arange(0, d, 2, dtype=torch.float32) / d)
        )
        self.physical_slots = torch.arange(cfg.num_blocks * cfg.block_size, dtype=torch.int32)
        self.logical_offsets = torch.arange(cfg.capacity, dtype=torch.int32)

    # -- reference helpers ---------------------------------------------------
    def rms_norm(self, hidden: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
        hidden_fp32 = hidden.float()
        variance = hidden_fp32.pow(2).mean(dim=-1, keepdim=True)
        normalized = (hidden_fp32 * torch.rsqrt(variance + self.cfg.rms_eps)).to(hidden.dtype)
        return normalized * weight

    def rotate_half(self, value: torch.Tensor) -> torch.Tensor:
        half = self.cfg.head_dim // 2
        return torch.cat((-value[..., half:], value[..., :half]), dim=-1)

    def rope(self, position: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        b = self.cfg.batch
        frequencies = position.float().reshape(b, 1) * self.inv_freq.view(1, -1)
        embedding = torch.cat((frequencies, frequencies), dim=-1)
        return embedding.cos().to(self.dtype), embedding.sin().to(self.dtype)

    def update_and_read_cache(self, layer_cache, new_value, block_table, slot_mapping, active_mask):
        cfg = self.cfg
        flat = layer_cache.reshape(cfg.num_blocks * cfg.block_size, cfg.num_kv_heads, cfg.head_dim)
        updated = flat
        for row in range(cfg.batch):
            slot_mask = (self.physical_slots == slot_mapping[row : row + 1]).view(-1, 1, 1)
            slot_mask = slot_mask & active_mask[row : row + 1].to(torch.bool).view(1, 1, 1)
            replacement = new_value[row].reshape(1, cfg.num_kv_heads, cfg.head_dim)
            updated = torch.where(slot_mask, replacement, updated)
        logical_blocks = self.logical_offsets // cfg.block_size
        offsets = self.logical_offsets - logical_blocks * cfg.block_size
        dense = []
        for row in range(cfg.batch):
            physical = torch.index_select(block_table[row], 0, logical_blocks.to(torch.int64))
            slots = (physical * cfg.block_size + offsets).to(torch.int64)
            dense.append(torch.index_select(updated, 0, slots))
        dense = torch.stack(dense)
        return updated.reshape_as(layer_cache), dense.permute(0, 2, 1, 3).contiguous()

    @staticmethod
    def exact_qk(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
        """``[1, H, D] x [H, D, C] -> [1, H, C]`` with the input dtype as result."""
        return torch.bmm(a.transpose(0, 1), b).transpose(0, 1)

    def _round_scores(self, scores: torch.Tensor) -> torch.Tensor:
        return scores.to(torch.bfloat16) if self.dtype == torch.bfloat16 else scores

    # -- one decoder step ----------------------------------------------------
    def step(self, token, position, seq_len, block_table, slot_mapping, key_cache, value_cache, active):
        """Returns ``(logits f32 [B,V], key_cache, value_cache, next_position)``.

        Argument shapes follow the 9-in decoder ABI (``config/graph_config.json``):
        token i64[B] (or [B,1]), position i64[B], seq_len i32[B], block_table
        i32[B, blocks_per_row], slot i32[B], caches [L, NB, bs, kv_heads, d],
        active i32[B].
        """
        cfg, w = self.cfg, self.w
        b, h, nq, nkv, d, cap = (
            cfg.batch, cfg.hidden, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, cfg.capacity,
        )
        groups = nq // nkv
        token = token.reshape(b).to(torch.int64)
        position = position.reshape(b).to(torch.int64)
        seq_len = seq_len.reshape(b)
        active = active.reshape(b)
        hidden = F.embedding(token, w["model.embed_tokens.weight"]).view(b, 1, h)
        cos, sin = self.rope(position)
        cos = cos.view(b, 1, 1, d)
        sin = sin.view(b, 1, 1, d)
        valid = self.logical_offsets.view(1, cap) < seq_len.reshape(b, 1)
        new_keys, new_values = [], []
        for layer in range(cfg.num_layers):
            p = f"model.layers.{layer}."
            residual = hidden
            normalized = self.rms_norm(hidden, w[p + "input_layernorm.weight"]).reshape(-1, h)
            query = F.linear(normalized, w[p + "self_attn.q_proj.weight"], w[p + "self_attn.q_proj.bias"])
            key = F.linear(normalized, w[p + "self_attn.k_proj.weight"], w[p + "self_attn.k_proj.bias"])
            value = F.linear(normalized, w[p + "self_attn.v_proj.weight"], w[p + "self_attn.v_proj.bias"])
            query = query.view(b, 1, nq, d).transpose(1, 2)
            key = key.view(b, 1, nkv, d).transpose(1, 2)
            value = value.view(b, 1, nkv, d).transpose(1, 2)
            query = query * cos + self.rotate_half(query) * sin
            key = key * cos + self.rotate_half(key) * sin
            updated_key, dense_key = self.update_and_read_cache(
                key_cache[layer], key, block_table, slot_mapping, active
            )
            updated_value, dense_value = self.update_and_read_cache(
                value_cache[layer], value, block_table, slot_mapping, active
            )
            new_keys.append(updated_key)
            new_values.append(updated_value)
            expanded_key = dense_key.unsqueeze(2).expand(b, nkv, groups, cap, d).reshape(b, nq, cap, d)
            expanded_value = dense_value.unsqueeze(2).expand(b, nkv, groups, cap, d).reshape(b, nq, cap, d)
            raw_qk = torch.cat(
                [
                    self.exact_qk(
                        query[row : row + 1].squeeze(2).contiguous(),
                        expanded_key[row].transpose(1, 2).contiguous(),
                    )
                    for row in range(b)
                ],
                dim=0,
            )
            scores = self._round_scores(raw_qk.float() / math.sqrt(d)).unsqueeze(2)
            scores = torch.where(
                valid.view(b, 1, 1, cap),
                scores,
                torch.full_like(scores, torch.finfo(torch.bfloat16).min),
            )
            probabilities = self._round_scores(torch.softmax(scores.float(), dim=-1))
            attention = torch.matmul(probabilities, expanded_value)
            attention = attention.transpose(1, 2).reshape(b, 1, h)
            projection = torch.mm(attention.reshape(-1, h), w[p + "self_attn.o_proj.weight"].t())
            hidden = residual + projection.reshape(b, 1, h)

            residual = hidden
            normalized = self.rms_norm(hidden, w[p + "post_attention_layernorm.weight"]).reshape(-1, h)
            gate = F.silu(torch.mm(normalized, w[p + "mlp.gate_proj.weight"].t()))
            up = torch.mm(normalized, w[p + "mlp.up_proj.weight"].t())
            projection = torch.mm(gate * up, w[p + "mlp.down_proj.weight"].t())
            hidden = residual + projection.reshape(b, 1, h)

        hidden = self.rms_norm(hidden, w["model.norm.weight"])
        logits = torch.mm(hidden.reshape(-1, h), w["lm_head.weight"].t()).float()
        next_position = torch.where(active.to(torch.bool), position + 1, position)
        return logits, torch.stack(new_keys), torch.stack(new_values), next_position
