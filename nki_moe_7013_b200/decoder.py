"""Qwen3-MoE decoder layer with the reference's forward signature.

``Qwen3MoeDecoderLayer.forward(hidden_states, attention_mask=None,
position_ids=None, past_key_value=None, padding_mask=None, **kwargs)``
returns ``(hidden_states, present_key_value, cos_cache, sin_cache, None)``
like NeuronQwen3MoeDecoderLayer.forward (qwen.py:378-436):

    residual = x
    h = input_layernorm(x)                       (qwen.py:408-412)
    h, kv = self_attn(h, ...)                    (qwen.py:415-422)
    residual = residual + h                      (qwen.py:423)
    h = post_attention_layernorm(residual)       (qwen.py:428)
    out = residual + mlp(h, padding_mask)[0]     (qwen.py:429-430)

Here the residual add before the second norm, the norm, the MoE block and
the final residual add are one library call (``qmoe_moe_block_forward``).  With a
``padding_mask`` the masked MoE output needs the norm's outputs first, so
that path runs the add & norm, the MoE block and the masked residual add
(``ops.masked_residual_add``, one kernel) as three calls.  RoPE is applied
inside the attention kernels, so cos/sin caches are returned as None.
``attention_mask``: attention is causal over each sequence's cache; a 2D
left-padding key mask (batch, cached + new tokens) is honoured and every
other mask is refused (``attention.Qwen3MoeAttention``).

``mlp``: the MoE module to use instead of a single-GPU
``Qwen3MoeSparseMoeBlock`` -- e.g. an expert-parallel
``ep.PeerExpertParallelMoE`` (attention then stays data-parallel: each rank
runs its own sequences).  Such a block (``expert_parallel = True``) is called
as ``mlp(h, residual=s)`` after a separate add & norm kernel.
``timer`` (an ``attention.StageTimer`` keyword argument) records CUDA events
around the layer's stages.  ``capture_intermediates=True`` keeps the
post-attention residual stream and the MoE input of the last call in
``self.last`` (for layer-by-layer parity checks).
"""
from __future__ import annotations

from typing import Optional

import torch
from torch import nn

from . import ops
from .attention import AttnWeights, KVCache, Qwen3MoeAttention, stage
from .config import Qwen3MoeConfig
from .moe import MoEWeights, Qwen3MoeSparseMoeBlock


class Qwen3MoeDecoderLayer(nn.Module):
    def __init__(self, cfg: Qwen3MoeConfig, layer_idx: int = 0, attn_weights: Optional[AttnWeights] = None,
                 moe_weights: Optional[MoEWeights] = None, input_norm: Optional[torch.Tensor] = None,
                 post_norm: Optional[torch.Tensor] = None, device="cuda", seed: int = 0,
                 mlp: Optional[nn.Module] = None):
        super().__init__()
        self.cfg = cfg
        self.layer_idx = layer_idx
        self.self_attn = Qwen3MoeAttention(cfg, attn_weights, device=device, seed=seed)
        self.mlp = mlp if mlp is not None else Qwen3MoeSparseMoeBlock(cfg, moe_weights, device=device, seed=seed)
        g = torch.Generator(device=device)
        g.manual_seed(seed * 10 + 8)
        H = cfg.hidden_size
        self.input_layernorm = (input_norm if input_norm is not None
                                else 1.0 + 0.1 * torch.randn(H, generator=g, device=device)).float().contiguous()
        self.post_attention_layernorm = (post_norm if post_norm is not None
                                         else 1.0 + 0.1 * torch.randn(H, generator=g, device=device)).float().contiguous()

    def forward(self, hidden_states: torch.Tensor, attention_mask: Optional[torch.Tensor] = None,
                position_ids: Optional[torch.Tensor] = None, past_key_value: Optional[KVCache] = None,
                padding_mask: Optional[torch.Tensor] = None, **kwargs):
        B, S, H = hidden_states.shape
        eps = self.cfg.rms_norm_eps
        timer = kwargs.get("timer")
        x2d = hidden_states.reshape(B * S, H).to(torch.bfloat16).contiguous()
        with stage(timer, "input_norm"):
            h = ops.rmsnorm(x2d, self.input_layernorm, eps)
        a, present = self.self_attn(h.reshape(B, S, H), position_ids, past_key_value, timer=timer,
                                    attention_mask=attention_mask)
        a2d = a.reshape(B * S, H)
        if getattr(self.mlp, "expert_parallel", False):
            with stage(timer, "post_norm"):
                h2, residual = ops.rmsnorm(a2d, self.post_attention_layernorm, eps, residual=x2d)
            with stage(timer, "moe"):
                if padding_mask is None:
                    out = self.mlp(h2, residual=residual)
                else:
                    out = ops.masked_residual_add(self.mlp(h2), padding_mask, residual)
        elif padding_mask is None and timer is not None and not kwargs.get("capture_intermediates"):
            with stage(timer, "moe"):
                out = self.mlp._block(a2d, x2d, self.post_attention_layernorm, eps)
        elif padding_mask is None:
            capture = bool(kwargs.get("capture_intermediates"))
            h2 = torch.empty_like(x2d) if capture else None
            residual = torch.empty_like(x2d) if capture else None
            out = self.mlp._block(a2d, x2d, self.post_attention_layernorm, eps, moe_in_out=h2,
                                  residual_out=residual)
        else:
            h2, residual = ops.rmsnorm(a2d, self.post_attention_layernorm, eps, residual=x2d)
            moe, _, _ = self.mlp._moe(h2)
            out = ops.masked_residual_add(moe, padding_mask, residual)
        if kwargs.get("capture_intermediates"):
            self.last = dict(attn=a2d, residual=residual, moe_in=h2)
        return (out.reshape(B, S, H), present, None, None, None)
