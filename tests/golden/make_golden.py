"""Generates the golden fixtures in this directory from the reference's own CPU
path: the HF transformers Qwen3-MoE modules that the reference instantiates in
CPU mode (qwen.py:35-37 imports Qwen3MoeForCausalLM / Qwen3MoeRMSNorm;
qwen.py:236-240 picks the HF RMSNorm on CPU).  The reference's NxDI device
path cannot run here (NxDI / neuronx are not installed), so these fixtures pin
the oracle to the reference's CPU semantics.

Inputs are regenerated from seeds with the counter-based generator
``nki_moe_7013_b200.synth.normal_bf16`` (stable across numpy/torch versions);
each fixture stores a checksum of its inputs to detect drift.

Run:  python tests/golden/make_golden.py   (writes *.npz next to this file)
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from nki_moe_7013_b200.synth import normal_bf16  # noqa: E402

MOE_CASES = {
    # name: (T, H, E, k, I, seed)
    "moe_small": (40, 512, 32, 4, 256, 11),
    "moe_cfg0_shapes_T16": (16, 2048, 128, 8, 768, 12),
}
ROUTER_CASES = {
    # cfg0 router: 128 tokens, hidden 2048, 128 experts, top-8
    "router_cfg0": (128, 2048, 128, 8, 0),
}


def checksum(*tensors) -> str:
    h = hashlib.sha256()
    for t in tensors:
        h.update(t.contiguous().view(torch.int16).numpy().tobytes())
    return h.hexdigest()[:16]


def moe_inputs(T, H, E, k, I, seed):
    x = normal_bf16(seed, "x", (T, H))
    wr = normal_bf16(seed, "w_router", (E, H), 0.02)
    wgu = normal_bf16(seed, "w_gate_up", (E, 2 * I, H), 0.02)
    wd = normal_bf16(seed, "w_down", (E, H, I), 0.02)
    return x, wr, wgu, wd


def hf_block(H, E, k, I, wr, wgu, wd, dtype):
    from transformers import Qwen3MoeConfig
    from transformers.models.qwen3_moe.modeling_qwen3_moe import Qwen3MoeSparseMoeBlock

    cfg = Qwen3MoeConfig(hidden_size=H, num_experts=E, num_experts_per_tok=k, moe_intermediate_size=I,
                         norm_topk_prob=True, hidden_act="silu")
    blk = Qwen3MoeSparseMoeBlock(cfg).to(dtype)
    with torch.no_grad():
        blk.gate.weight.copy_(wr.to(dtype))
        blk.experts.gate_up_proj.copy_(wgu.to(dtype))
        blk.experts.down_proj.copy_(wd.to(dtype))
    return blk.eval()


ATTN_CASES = {
    # name: (B, S, H, nh, nkv, E, k, I, seed) -- head_dim 128, 8 query heads per KV head
    "decoder_small": (2, 24, 512, 8, 1, 32, 4, 256, 21),
}


def hf_decoder_golden(B, S, H, nh, nkv, E, k, I, seed):
    """HF Qwen3MoeAttention and Qwen3MoeDecoderLayer in fp32 (eager attention)."""
    from transformers import Qwen3MoeConfig
    from transformers.models.qwen3_moe.modeling_qwen3_moe import (Qwen3MoeDecoderLayer,
                                                                  Qwen3MoeRotaryEmbedding)

    cfg = Qwen3MoeConfig(hidden_size=H, num_attention_heads=nh, num_key_value_heads=nkv, head_dim=128,
                         num_experts=E, num_experts_per_tok=k, moe_intermediate_size=I, norm_topk_prob=True,
                         rms_norm_eps=1e-6, rope_theta=1e6, hidden_act="silu", decoder_sparse_step=1,
                         mlp_only_layers=[], max_position_embeddings=4096)
    cfg._attn_implementation = "eager"
    layer = Qwen3MoeDecoderLayer(cfg, 0).float().eval()
    x = normal_bf16(seed, "x", (B, S, H))
    p = {
        "wq": normal_bf16(seed, "wq", (nh * 128, H), 0.02), "wk": normal_bf16(seed, "wk", (nkv * 128, H), 0.02),
        "wv": normal_bf16(seed, "wv", (nkv * 128, H), 0.02), "wo": normal_bf16(seed, "wo", (H, nh * 128), 0.02),
        "qn": normal_bf16(seed, "qn", (128,), 0.1, 1.0), "kn": normal_bf16(seed, "kn", (128,), 0.1, 1.0),
        "ln1": normal_bf16(seed, "ln1", (H,), 0.1, 1.0), "ln2": normal_bf16(seed, "ln2", (H,), 0.1, 1.0),
        "wr": normal_bf16(seed, "w_router", (E, H), 0.02), "wgu": normal_bf16(seed, "w_gate_up", (E, 2 * I, H), 0.02),
        "wd": normal_bf16(seed, "w_down", (E, H, I), 0.02)}
    with torch.no_grad():
        a = layer.self_attn
        a.q_proj.weight.copy_(p["wq"].float()); a.k_proj.weight.copy_(p["wk"].float())
        a.v_proj.weight.copy_(p["wv"].float()); a.o_proj.weight.copy_(p["wo"].float())
        a.q_norm.weight.copy_(p["qn"].float()); a.k_norm.weight.copy_(p["kn"].float())
        layer.input_layernorm.weight.copy_(p["ln1"].float())
        layer.post_attention_layernorm.weight.copy_(p["ln2"].float())
        layer.mlp.gate.weight.copy_(p["wr"].float())
        layer.mlp.experts.gate_up_proj.copy_(p["wgu"].float())
        layer.mlp.experts.down_proj.copy_(p["wd"].float())
        rot = Qwen3MoeRotaryEmbedding(cfg)
        pos = torch.arange(S).unsqueeze(0).expand(B, S)
        cos, sin = rot(x.float(), pos)
        mask = torch.full((S, S), float("-inf")).triu(1).expand(B, 1, S, S)
        xin = x.float()
        h = layer.input_layernorm(xin)
        attn_out, _ = a(h, (cos, sin), mask)
        out = layer(xin, attention_mask=mask, position_ids=pos, position_embeddings=(cos, sin))
        out = out[0] if isinstance(out, tuple) else out
    return x, p, attn_out.numpy(), out.numpy()


def main():
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    for name, (T, H, E, k, I, seed) in MOE_CASES.items():
        x, wr, wgu, wd = moe_inputs(T, H, E, k, I, seed)
        out = {}
        for tag, dt in (("fp32", torch.float32), ("bf16", torch.bfloat16)):
            blk = hf_block(H, E, k, I, wr, wgu, wd, dt)
            with torch.no_grad():
                probs, w, idx = blk.gate(x.to(dt))
                y = blk(x.to(dt).reshape(1, T, H)).reshape(T, H)
            out[f"{tag}_probs"] = probs.float().numpy()
            out[f"{tag}_topk_idx"] = idx.numpy().astype(np.int32)
            out[f"{tag}_topk_w"] = w.float().numpy()
            out[f"{tag}_out"] = y.float().numpy()
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), shape=np.array([T, H, E, k, I, seed]),
                            checksum=np.array(checksum(x, wr, wgu, wd)), **out)
        print("wrote", name)
    for name, (B, S, H, nh, nkv, E, k, I, seed) in ATTN_CASES.items():
        x, p, attn_out, out = hf_decoder_golden(B, S, H, nh, nkv, E, k, I, seed)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), shape=np.array([B, S, H, nh, nkv, E, k, I, seed]),
                            checksum=np.array(checksum(x, *p.values())), fp32_attn=attn_out, fp32_out=out)
        print("wrote", name)
    for name, (T, H, E, k, seed) in ROUTER_CASES.items():
        x = normal_bf16(seed, "x", (T, H))
        wr = normal_bf16(seed, "w_router", (E, H), 0.02)
        logits = torch.nn.functional.linear(x.float(), wr.float())
        probs = torch.softmax(logits, dim=-1)
        w, idx = torch.topk(probs, k, dim=-1)
        w = w / w.sum(-1, keepdim=True)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), shape=np.array([T, H, E, k, seed]),
                            checksum=np.array(checksum(x, wr)), fp32_logits=logits.numpy(),
                            fp32_topk_idx=idx.numpy().astype(np.int32), fp32_topk_w=w.numpy())
        print("wrote", name)


if __name__ == "__main__":
    main()
