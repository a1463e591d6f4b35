"""HF checkpoint loading (CPU): per-expert and fused expert tensors, fp8 block
dequantisation, sharded checkpoints with an index, tied embeddings, and the
refusal of dense-MLP layers.  Tensors are compared bit for bit with the
layouts the kernels take."""
import json

import pytest
import torch

H, E, K, I, NH, NKV, HD, V, L = 256, 8, 2, 128, 2, 1, 128, 512, 2


def _hf_config(**extra):
    cfg = dict(hidden_size=H, num_experts=E, num_experts_per_tok=K, moe_intermediate_size=I, norm_topk_prob=True,
               num_attention_heads=NH, num_key_value_heads=NKV, head_dim=HD, rms_norm_eps=1e-6, rope_theta=1e6,
               vocab_size=V, num_hidden_layers=L, max_position_embeddings=4096, decoder_sparse_step=1,
               mlp_only_layers=[], tie_word_embeddings=False)
    cfg.update(extra)
    return cfg


def _tensors(seed=0):
    g = torch.Generator().manual_seed(seed)

    def rnd(*shape):
        return (0.02 * torch.randn(*shape, generator=g)).to(torch.bfloat16)

    sd = {"model.embed_tokens.weight": rnd(V, H), "model.norm.weight": (1 + rnd(H)), "lm_head.weight": rnd(V, H)}
    for l in range(L):
        p = f"model.layers.{l}."
        sd[p + "input_layernorm.weight"] = 1 + rnd(H)
        sd[p + "post_attention_layernorm.weight"] = 1 + rnd(H)
        sd[p + "self_attn.q_proj.weight"] = rnd(NH * HD, H)
        sd[p + "self_attn.k_proj.weight"] = rnd(NKV * HD, H)
        sd[p + "self_attn.v_proj.weight"] = rnd(NKV * HD, H)
        sd[p + "self_attn.o_proj.weight"] = rnd(H, NH * HD)
        sd[p + "self_attn.q_norm.weight"] = 1 + rnd(HD)
        sd[p + "self_attn.k_norm.weight"] = 1 + rnd(HD)
        sd[p + "mlp.gate.weight"] = rnd(E, H)
        for e in range(E):
            sd[p + f"mlp.experts.{e}.gate_proj.weight"] = rnd(I, H)
            sd[p + f"mlp.experts.{e}.up_proj.weight"] = rnd(I, H)
            sd[p + f"mlp.experts.{e}.down_proj.weight"] = rnd(H, I)
    return sd


def _write(path, sd, cfg, shards=1):
    from safetensors.torch import save_file

    path.mkdir(parents=True, exist_ok=True)
    (path / "config.json").write_text(json.dumps(cfg))
    names = sorted(sd)
    if shards == 1:
        save_file({n: sd[n].contiguous() for n in names}, str(path / "model.safetensors"))
        return
    weight_map = {}
    for s in range(shards):
        part = names[s::shards]
        fname = f"model-{s + 1:05d}-of-{shards:05d}.safetensors"
        save_file({n: sd[n].contiguous() for n in part}, str(path / fname))
        weight_map.update({n: fname for n in part})
    (path / "model.safetensors.index.json").write_text(json.dumps({"metadata": {}, "weight_map": weight_map}))


def _check_model(model, sd, dequant=None):
    dequant = dequant or {}

    def ref(name):
        return dequant.get(name, sd[name]).to(torch.bfloat16)

    assert torch.equal(model.embed, ref("model.embed_tokens.weight"))
    assert torch.equal(model.lm_head, ref("lm_head.weight"))
    assert torch.equal(model.norm, ref("model.norm.weight").float())
    assert len(model.layers) == L
    for l, layer in enumerate(model.layers):
        p = f"model.layers.{l}."
        w = layer.mlp.weights
        assert torch.equal(w.router, ref(p + "mlp.gate.weight"))
        for e in range(E):
            q = p + f"mlp.experts.{e}."
            assert torch.equal(w.gate_up[e, :I], ref(q + "gate_proj.weight"))
            assert torch.equal(w.gate_up[e, I:], ref(q + "up_proj.weight"))
            assert torch.equal(w.down[e], ref(q + "down_proj.weight"))
        a = layer.self_attn.w
        assert torch.equal(a.wqkv, torch.cat([ref(p + f"self_attn.{n}_proj.weight") for n in "qkv"], 0))
        assert torch.equal(a.wo, ref(p + "self_attn.o_proj.weight"))
        assert torch.equal(a.q_norm, ref(p + "self_attn.q_norm.weight").float())
        assert torch.equal(a.k_norm, ref(p + "self_attn.k_norm.weight").float())
        assert torch.equal(layer.input_layernorm, ref(p + "input_layernorm.weight").float())
        assert torch.equal(layer.post_attention_layernorm, ref(p + "post_attention_layernorm.weight").float())


@pytest.mark.parametrize("shards", [1, 3])
def test_load_per_expert_checkpoint(tmp_path, shards):
    from nki_moe_7013_b200.checkpoint import load_model

    sd = _tensors()
    _write(tmp_path / "ckpt", sd, _hf_config(), shards=shards)
    model = load_model(str(tmp_path / "ckpt"), device="cpu")
    assert model.cfg.hidden_size == H and model.cfg.num_experts == E and model.cfg.num_experts_per_tok == K
    assert model.cfg.moe_intermediate_size == I and model.cfg.head_dim == HD and model.vocab_size == V
    _check_model(model, sd)


def test_fp8_block_scales_are_dequantised(tmp_path):
    """An fp8 weight with a 128 x 128 block scale (the released checkpoints'
    quantization_config): every element times its block's scale in fp32,
    then bf16 -- checked against that product computed here."""
    from nki_moe_7013_b200.checkpoint import load_model

    sd = _tensors(1)
    g = torch.Generator().manual_seed(9)
    deq = {}
    for name, shape in [("model.layers.0.mlp.experts.3.gate_proj.weight", (I, H)),
                        ("model.layers.1.self_attn.o_proj.weight", (H, NH * HD))]:
        q = (torch.randn(*shape, generator=g) * 64).clamp(-440, 440).to(torch.float8_e4m3fn)
        scale = torch.rand((shape[0] + 127) // 128, (shape[1] + 127) // 128, generator=g) * 1e-3 + 1e-4
        sd[name] = q
        sd[name + "_scale_inv"] = scale
        expanded = scale.repeat_interleave(128, 0).repeat_interleave(128, 1)[: shape[0], : shape[1]]
        deq[name] = (q.float() * expanded).to(torch.bfloat16)
    cfg = _hf_config(quantization_config={"quant_method": "fp8", "weight_block_size": [128, 128]})
    _write(tmp_path / "ckpt", sd, cfg)
    model = load_model(str(tmp_path / "ckpt"), device="cpu")
    _check_model(model, {k: v for k, v in sd.items() if not k.endswith("_scale_inv")}, dequant=deq)


def test_fused_expert_tensors_and_tied_embeddings(tmp_path):
    """Checkpoints that store experts.gate_up_proj (E, 2I, H) / down_proj
    (E, H, I) take them as they are; tie_word_embeddings reuses the table."""
    from nki_moe_7013_b200.checkpoint import load_model

    sd = _tensors(2)
    fused = {k: v for k, v in sd.items() if ".experts." not in k and k != "lm_head.weight"}
    for l in range(L):
        p = f"model.layers.{l}.mlp.experts."
        fused[p + "gate_up_proj"] = torch.stack(
            [torch.cat([sd[p + f"{e}.gate_proj.weight"], sd[p + f"{e}.up_proj.weight"]], 0) for e in range(E)])
        fused[p + "down_proj"] = torch.stack([sd[p + f"{e}.down_proj.weight"] for e in range(E)])
    _write(tmp_path / "ckpt", fused, _hf_config(tie_word_embeddings=True))
    model = load_model(str(tmp_path / "ckpt"), device="cpu", num_layers=1)
    assert len(model.layers) == 1
    assert model.lm_head is model.embed
    w = model.layers[0].mlp.weights
    assert torch.equal(w.gate_up, fused["model.layers.0.mlp.experts.gate_up_proj"])
    assert torch.equal(w.down, fused["model.layers.0.mlp.experts.down_proj"])


def test_dense_mlp_layers_are_refused(tmp_path):
    from nki_moe_7013_b200.checkpoint import load_model

    _write(tmp_path / "ckpt", _tensors(3), _hf_config(mlp_only_layers=[0]))
    with pytest.raises(NotImplementedError):
        load_model(str(tmp_path / "ckpt"), device="cpu")
