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
