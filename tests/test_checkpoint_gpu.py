"""A checkpoint written by transformers (save_pretrained of a random
Qwen3MoeForCausalLM) loads into this library's model, and its prefill logits
follow the transformers model's."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_loaded_model_matches_transformers(tmp_path, cuda_dev):
    from transformers import Qwen3MoeConfig, Qwen3MoeForCausalLM

    from nki_moe_7013_b200 import _C
    from nki_moe_7013_b200.checkpoint import load_model

    torch.manual_seed(0)
    cfg = Qwen3MoeConfig(vocab_size=1024, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                         num_attention_heads=2, num_key_value_heads=1, head_dim=128, moe_intermediate_size=128,
                         num_experts=32, num_experts_per_tok=4, norm_topk_prob=True, rms_norm_eps=1e-6,
                         rope_theta=1e6, max_position_embeddings=512, decoder_sparse_step=1, mlp_only_layers=[],
                         tie_word_embeddings=False, hidden_act="silu")
    hf = Qwen3MoeForCausalLM(cfg).eval()
    with torch.no_grad():
        for p in hf.parameters():  # bf16-representable weights: only the arithmetic differs
            p.copy_(p.bfloat16().float())
        for name, p in hf.named_parameters():
            if name.endswith("norm.weight"):
                p.copy_((1.0 + 0.1 * torch.randn_like(p)).bfloat16().float())
    hf.save_pretrained(str(tmp_path / "ckpt"))
    model = load_model(str(tmp_path / "ckpt"), device=cuda_dev)
    assert model.cfg.num_experts == 32 and model.cfg.num_experts_per_tok == 4 and len(model.layers) == 2

    ids = torch.randint(0, 1024, (1, 16), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        ref = hf(ids).logits[0].float().numpy()
    logits, _ = model.forward(ids.to(cuda_dev))
    torch.cuda.synchronize()
    assert _C.device_error() == 0
    got = logits[0].float().cpu().numpy()
    err = float(np.abs(got - ref).max() / np.abs(ref).max())
    # bf16 activations against transformers' fp32 ones, two layers deep
    assert err <= 5e-2, f"logits max rel err {err:.3e}"
    assert int((got.argmax(-1) == ref.argmax(-1)).sum()) >= 14
