"""Layer configuration (one dataclass; no import-time environment switches)."""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class Qwen3MoeConfig:
    """Shapes of Qwen3-30B-A3B (qwen.py:243-310 reads the same fields from the
    HF config): hidden 2048, 128 experts, top-8, moe_intermediate 768,
    32 query / 4 KV heads of 128, RMSNorm eps 1e-6, RoPE theta 1e6."""

    hidden_size: int = 2048
    num_experts: int = 128
    num_experts_per_tok: int = 8
    moe_intermediate_size: int = 768
    norm_topk_prob: bool = True
    num_attention_heads: int = 32
    num_key_value_heads: int = 4
    head_dim: int = 128
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1e6
    vocab_size: int = 151936
    num_hidden_layers: int = 48
    max_position_embeddings: int = 40960
