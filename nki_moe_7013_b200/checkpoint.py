"""HF Qwen3-MoE checkpoints -> this library's device layouts.

Reads a transformers checkpoint directory (``config.json`` and one or more
``*.safetensors`` files, with or without ``model.safetensors.index.json``)
and builds a :class:`~nki_moe_7013_b200.model.Qwen3MoeModel` whose tensors
are in the layouts the kernels take.  It replaces the reference's
``convert_qwen3_moe_hf_to_neuron_state_dict`` (qwen.py:119-233):

* the per-expert ``gate_proj`` / ``up_proj`` (I, H) and ``down_proj`` (H, I)
  are stacked into gate_up (E, 2I, H), gate rows first, and down (E, H, I)
  -- the reference stacks the same matrices transposed, (E, H, 2I) and
  (E, I, H), for its kernels (qwen.py:164-226); checkpoints written with the
  fused ``experts.gate_up_proj`` / ``experts.down_proj`` tensors are taken as
  they are;
* q/k/v projections become one (nh*hd + 2*nkv*hd, H) matrix;
* fp8 weights stored with a ``<name>_scale_inv`` block scale are dequantised
  as the reference does (qwen.py:101-116): every element is multiplied by the
  scale of its block (``quantization_config.weight_block_size``, 128 x 128
  in the released checkpoints) in fp32, then rounded to bf16.

The reference pads the expert intermediate size for its tensor-parallel
split (qwen.py:195-226); nothing here splits I, so there is no padding.
Layers with a dense MLP (``mlp_only_layers`` / ``decoder_sparse_step`` > 1)
are not part of Qwen3-30B-A3B and are refused.
"""
from __future__ import annotations

import json
import os
from typing import Dict, Iterable, List, Optional, Tuple

import torch

from .attention import AttnWeights
from .config import Qwen3MoeConfig
from .moe import MoEWeights

INDEX_FILE = "model.safetensors.index.json"


def config_from_hf(hf: Dict) -> Qwen3MoeConfig:
    """The fields of an HF ``config.json`` (Qwen3MoeConfig) this library uses."""
    if hf.get("mlp_only_layers") or int(hf.get("decoder_sparse_step", 1)) != 1:
        raise NotImplementedError("dense-MLP layers (mlp_only_layers / decoder_sparse_step) are not supported")
    # the released checkpoints write rope_theta / num_experts; transformers 5
    # writes rope_parameters / num_local_experts
    rope = hf.get("rope_theta")
    if rope is None:
        rope = (hf.get("rope_parameters") or {}).get("rope_theta", Qwen3MoeConfig.rope_theta)
    n_exp = hf.get("num_experts", hf.get("num_local_experts"))
    if n_exp is None:
        raise KeyError("config.json has neither num_experts nor num_local_experts")
    nh = int(hf["num_attention_heads"])
    return Qwen3MoeConfig(
        hidden_size=int(hf["hidden_size"]), num_experts=int(n_exp),
        num_experts_per_tok=int(hf["num_experts_per_tok"]), moe_intermediate_size=int(hf["moe_intermediate_size"]),
        norm_topk_prob=bool(hf.get("norm_topk_prob", True)), num_attention_heads=nh,
        num_key_value_heads=int(hf.get("num_key_value_heads", nh)),
        head_dim=int(hf.get("head_dim") or int(hf["hidden_size"]) // nh),
        rms_norm_eps=float(hf.get("rms_norm_eps", 1e-6)), rope_theta=float(rope),
        vocab_size=int(hf["vocab_size"]), num_hidden_layers=int(hf["num_hidden_layers"]),
        max_position_embeddings=int(hf.get("max_position_embeddings", Qwen3MoeConfig.max_position_embeddings)))


class CheckpointReader:
    """Tensor access by name over the safetensors files of a checkpoint
    directory (one file open at a time per lookup; tensors load on demand)."""

    def __init__(self, path: str):
        from safetensors import safe_open

        self._safe_open = safe_open
        self.path = path
        self.where: Dict[str, str] = {}
        index = os.path.join(path, INDEX_FILE)
        if os.path.exists(index):
            with open(index) as f:
                for name, fname in json.load(f)["weight_map"].items():
                    self.where[name] = os.path.join(path, fname)
        else:
            files = sorted(f for f in os.listdir(path) if f.endswith(".safetensors"))
            if not files:
                raise FileNotFoundError(f"no .safetensors files in {path}")
            for fname in files:
                full = os.path.join(path, fname)
                with safe_open(full, framework="pt") as f:
                    for name in f.keys():
                        self.where[name] = full

    def __contains__(self, name: str) -> bool:
        return name in self.where

    def get(self, name: str) -> torch.Tensor:
        if name not in self.where:
            raise KeyError(f"tensor {name!r} not in the checkpoint at {self.path}")
        with self._safe_open(self.where[name], framework="pt") as f:
            return f.get_tensor(name)

    def names(self) -> Iterable[str]:
        return self.where.keys()


def dequantize_blocks(w: torch.Tensor, scale_inv: torch.Tensor, block: Tuple[int, int]) -> torch.Tensor:
    """w (R, C) quantised, scale_inv (ceil(R/b0), ceil(C/b1)): every element
    times the scale of its block, in fp32, rounded to bf16."""
    b0, b1 = block
    s = scale_inv.float().repeat_interleave(b0, dim=0).repeat_interleave(b1, dim=1)[: w.shape[0], : w.shape[1]]
    return (w.float() * s).to(torch.bfloat16)


class _Weights:
    """Named tensors of one checkpoint as bf16 (fp8 blocks dequantised)."""

    def __init__(self, reader: CheckpointReader, block: Optional[Tuple[int, int]]):
        self.r = reader
        self.block = block

    def has(self, name: str) -> bool:
        return name in self.r

    def bf16(self, name: str) -> torch.Tensor:
        w = self.r.get(name)
        scale = name + "_scale_inv"
        if scale in self.r:
            if self.block is None:
                raise ValueError(f"{name} has a block scale but the config has no weight_block_size")
            return dequantize_blocks(w, self.r.get(scale), self.block)
        return w.to(torch.bfloat16)


def _prefix(reader: CheckpointReader) -> str:
    return "model." if "model.embed_tokens.weight" in reader else ""


def load_layer_weights(w: _Weights, cfg: Qwen3MoeConfig, l: int, pre: str, device
                       ) -> Tuple[AttnWeights, MoEWeights, torch.Tensor, torch.Tensor]:
    """One decoder layer: attention weights, expert weights, input and
    post-attention RMSNorm weights, on `device`."""
    p = f"{pre}layers.{l}."
    bf = dict(device=device, dtype=torch.bfloat16)
    wqkv = torch.cat([w.bf16(p + f"self_attn.{n}_proj.weight") for n in ("q", "k", "v")], 0)
    attn = AttnWeights(wqkv.to(**bf).contiguous(), w.bf16(p + "self_attn.o_proj.weight").to(**bf).contiguous(),
                       w.bf16(p + "self_attn.q_norm.weight").float().to(device).contiguous(),
                       w.bf16(p + "self_attn.k_norm.weight").float().to(device).contiguous())
    E, H, I = cfg.num_experts, cfg.hidden_size, cfg.moe_intermediate_size
    router = w.bf16(p + "mlp.gate.weight").to(**bf).contiguous()
    if w.has(p + "mlp.experts.gate_up_proj"):
        gate_up = w.bf16(p + "mlp.experts.gate_up_proj").to(**bf).contiguous()
        down = w.bf16(p + "mlp.experts.down_proj").to(**bf).contiguous()
    else:
        gate_up = torch.empty((E, 2 * I, H), **bf)
        down = torch.empty((E, H, I), **bf)
        for e in range(E):
            q = p + f"mlp.experts.{e}."
            gate_up[e, :I].copy_(w.bf16(q + "gate_proj.weight"))
            gate_up[e, I:].copy_(w.bf16(q + "up_proj.weight"))
            down[e].copy_(w.bf16(q + "down_proj.weight"))
    if tuple(gate_up.shape) != (E, 2 * I, H) or tuple(down.shape) != (E, H, I) or tuple(router.shape) != (E, H):
        raise ValueError(f"layer {l}: expert weight shapes {tuple(router.shape)}, {tuple(gate_up.shape)}, "
                         f"{tuple(down.shape)} do not match the config")
    norm_in = w.bf16(p + "input_layernorm.weight").float().to(device).contiguous()
    norm_post = w.bf16(p + "post_attention_layernorm.weight").float().to(device).contiguous()
    return attn, MoEWeights(router, gate_up, down), norm_in, norm_post


def load_model(path: str, device="cuda", num_layers: Optional[int] = None):
    """A Qwen3MoeModel with the weights of the HF checkpoint at `path` (the
    first `num_layers` layers if given)."""
    from .decoder import Qwen3MoeDecoderLayer
    from .model import Qwen3MoeModel

    with open(os.path.join(path, "config.json")) as f:
        hf = json.load(f)
    cfg = config_from_hf(hf)
    qc = hf.get("quantization_config") or {}
    block = tuple(qc["weight_block_size"]) if qc.get("weight_block_size") else None
    reader = CheckpointReader(path)
    w = _Weights(reader, block)
    pre = _prefix(reader)
    dev = torch.device(device)
    L = cfg.num_hidden_layers if num_layers is None else min(num_layers, cfg.num_hidden_layers)
    layers: List = []
    for l in range(L):
        attn, moe_w, norm_in, norm_post = load_layer_weights(w, cfg, l, pre, dev)
        layers.append(Qwen3MoeDecoderLayer(cfg, layer_idx=l, attn_weights=attn, moe_weights=moe_w,
                                           input_norm=norm_in, post_norm=norm_post, device=dev))
    embed = w.bf16(pre + "embed_tokens.weight").to(dev).contiguous()
    if "lm_head.weight" in reader:
        lm_head = w.bf16("lm_head.weight").to(dev).contiguous()
    elif hf.get("tie_word_embeddings", False):
        lm_head = embed
    else:
        raise KeyError("checkpoint has no lm_head.weight and does not tie the embeddings")
    norm = w.bf16(pre + "norm.weight").float().to(dev).contiguous()
    return Qwen3MoeModel.from_parts(cfg, embed, layers, norm, lm_head)
