"""The reference's operator seams on the GPU: ExpertMLPsV2
.torch_blockwise_matmul_inference (qwen_with_nki.py:5872-5881) and
.forward_selective_loading (qwen_with_nki.py:2377-2453), plus the module
drop-ins, against the CPU oracle."""
import numpy as np
import pytest
import torch

from helpers import MAX_REL, activations, assert_within_one_ulp, max_rel_err, moe_weights, to_f32_np

pytestmark = pytest.mark.gpu


def _blocks_from_routing(inter, E, B, dup_every=3):
    """NxDI-style blocks: per expert, its routed tokens in blocks of B with -1
    padding, and a duplicated token inside some blocks."""
    tpi, b2e = [], []
    for e in range(E):
        toks = list(inter["row_token"][inter["offsets"][e]:inter["offsets"][e + 1]])
        if not toks:
            continue
        for s in range(0, len(toks), B - 1):
            blk = toks[s:s + B - 1]
            if e % dup_every == 0:
                blk = blk + blk[:1]  # duplicate inside the same block
            blk = blk + [-1] * (B - len(blk))
            tpi += blk
            b2e.append(e)
    return np.array(tpi, np.int32), np.array(b2e, np.int32)


@pytest.mark.parametrize("T,H,E,k,I,B", [(128, 2048, 128, 8, 768, 512), (40, 512, 32, 4, 256, 64),
                                         (300, 512, 32, 8, 256, 100)])
def test_blockwise_seam_matches_oracle(cuda_dev, oracle, T, H, E, k, I, B):
    from nki_moe_7013_b200.moe import ExpertMLPs, MoEWeights

    wr, wgu, wd = moe_weights(7, E, H, I, cuda_dev)
    x = activations(7, T, H, cuda_dev)
    _, inter = oracle.moe_block(x.cpu(), wr.cpu(), wgu.cpu(), wd.cpu(), k, return_intermediates=True)
    aff = np.zeros((T + 1, E), np.float32)  # T+1 rows: the pad row of qwen_with_nki.py:5466-5470
    for t in range(T):
        aff[t, inter["topk_idx"][t]] = inter["topk_w"][t]
    tpi, b2e = _blocks_from_routing(inter, E, B)
    mlps = ExpertMLPs(MoEWeights(wr, wgu, wd))
    out = mlps.torch_blockwise_matmul_inference(
        B, len(b2e), x, torch.from_numpy(aff).to(cuda_dev), torch.from_numpy(tpi).to(cuda_dev),
        torch.from_numpy(b2e).to(cuda_dev))
    torch.cuda.synchronize()
    ref = oracle.blockwise_moe(x.cpu(), aff, tpi, b2e, B, wgu.cpu(), wd.cpu())
    err = max_rel_err(to_f32_np(out), oracle.round_to_bf16(ref))
    assert err <= MAX_REL, f"blockwise seam max rel err {err:.3e}"
    # the blockwise seam and the routed block compute the same layer
    routed = oracle.moe_block(x.cpu(), wr.cpu(), wgu.cpu(), wd.cpu(), k)
    assert max_rel_err(to_f32_np(out), routed) <= MAX_REL


@pytest.mark.parametrize("T", [1, 5, 64])
def test_selective_loading_seam_matches_oracle(cuda_dev, oracle, T):
    from nki_moe_7013_b200 import ops
    from nki_moe_7013_b200.moe import ExpertMLPs, MoEWeights

    H, E, k, I = 2048, 128, 8, 768
    wr, wgu, wd = moe_weights(8, E, H, I, cuda_dev)
    x = activations(8 + T, T, H, cuda_dev)
    idx, _, logits = ops.router_topk(x, wr, k, return_logits=True)
    affinities = torch.softmax(logits, dim=-1)  # (T, E) as RouterTopK returns them
    out = ExpertMLPs(MoEWeights(wr, wgu, wd)).forward_selective_loading(x, affinities, idx.long())
    torch.cuda.synchronize()
    ref = oracle.moe_block(x.cpu(), wr.cpu(), wgu.cpu(), wd.cpu(), k)
    err = max_rel_err(to_f32_np(out), oracle.round_to_bf16(ref))
    assert err <= MAX_REL


def test_module_dropins(cuda_dev, oracle):
    from nki_moe_7013_b200.config import Qwen3MoeConfig
    from nki_moe_7013_b200.moe import MoEWeights, Qwen3MoeSparseMoeBlock, Qwen3MoeSparseMoeBlockHF

    cfg = Qwen3MoeConfig()
    w = MoEWeights.random(cfg, seed=9, device=cuda_dev)
    x = activations(9, 2 * 48, cfg.hidden_size, cuda_dev).reshape(2, 48, cfg.hidden_size)
    mask = torch.ones(2, 48, device=cuda_dev)
    mask[1, 40:] = 0  # padded positions
    blk = Qwen3MoeSparseMoeBlock(cfg, weights=w, return_expert_index=True)
    out, eidx = blk(x, mask)
    hf = Qwen3MoeSparseMoeBlockHF(cfg, weights=w)(x)
    torch.cuda.synchronize()
    assert out.shape == x.shape and eidx.shape == (96, 8)
    ref = oracle.moe_block(x.reshape(96, -1).cpu(), w.router.cpu(), w.gate_up.cpu(), w.down.cpu(), 8)
    ref = oracle.round_to_bf16(ref).reshape(2, 48, -1)
    assert max_rel_err(to_f32_np(hf), ref) <= MAX_REL
    ref_masked = ref * mask.cpu().numpy()[..., None]
    assert max_rel_err(to_f32_np(out), ref_masked) <= MAX_REL
    assert torch.count_nonzero(out[1, 40:]).item() == 0
    # NxDI layout conversion round trip
    w2 = MoEWeights.from_neuron_layout(w.router, w.gate_up.transpose(1, 2), w.down.transpose(1, 2),
                                       device=cuda_dev)
    assert torch.equal(w2.gate_up, w.gate_up) and torch.equal(w2.down, w.down)


def test_masked_residual_add_bit_exact(cuda_dev):
    """ops.masked_residual_add equals the eager fp32 formula bit for bit, with
    0/1 and fractional masks, with and without a residual."""
    from nki_moe_7013_b200 import ops

    T, H = 300, 2048
    y = activations(60, T, H, cuda_dev)
    res = activations(61, T, H, cuda_dev)
    g = torch.Generator(device=cuda_dev)
    g.manual_seed(62)
    for mask in ((torch.rand(T, generator=g, device=cuda_dev) > 0.3).to(torch.int64),
                 torch.rand(T, generator=g, device=cuda_dev)):
        m = mask.reshape(-1, 1).float()
        assert torch.equal(ops.masked_residual_add(y, mask), (y.float() * m).to(torch.bfloat16))
        assert torch.equal(ops.masked_residual_add(y, mask, res), (res.float() + y.float() * m).to(torch.bfloat16))
    assert torch.equal(ops.masked_residual_add(y, None, res), (res.float() + y.float()).to(torch.bfloat16))


@pytest.mark.parametrize("normalize", [True, False])
def test_select_affinities_matches_torch(cuda_dev, normalize):
    """The chosen-affinity gather + F.normalize(p=1) kernel against torch."""
    from nki_moe_7013_b200 import ops

    T, E, k = 257, 128, 8
    g = torch.Generator(device=cuda_dev)
    g.manual_seed(63)
    aff = torch.softmax(torch.randn(T, E, generator=g, device=cuda_dev), -1)
    idx = torch.topk(aff, k, dim=-1).indices.to(torch.int32)
    w = ops.select_affinities(aff, idx, normalize)
    ref = torch.gather(aff, 1, idx.long())
    if normalize:
        ref = torch.nn.functional.normalize(ref, p=1.0, dim=1)
    # the kernel sums |w| in slot order, torch's reduction in its own order:
    # the L1 norms, and so the quotients, differ by a few fp32 ulps
    torch.testing.assert_close(w, ref, rtol=1e-6, atol=0)


def test_moe_block_padding_mask(cuda_dev):
    """Qwen3MoeSparseMoeBlock(x, padding_mask): masked tokens give zero rows,
    the others the unmasked output (two separate forwards: the combine adds a
    token's expert rows with fp32 atomics in a run-dependent order, so within
    one bf16 ulp)."""
    from nki_moe_7013_b200.config import Qwen3MoeConfig
    from nki_moe_7013_b200.moe import MoEWeights, Qwen3MoeSparseMoeBlock

    cfg = Qwen3MoeConfig()
    blk = Qwen3MoeSparseMoeBlock(cfg, MoEWeights.random(cfg, seed=12, device=cuda_dev), device=cuda_dev)
    B, S = 2, 40
    x = activations(64, B * S, cfg.hidden_size, cuda_dev).reshape(B, S, cfg.hidden_size)
    mask = torch.ones(B, S, dtype=torch.int64, device=cuda_dev)
    mask[0, :7] = 0  # left padding of the first sequence
    full = blk(x)[0]
    masked = blk(x, mask)[0]
    torch.cuda.synchronize()
    keep = mask.bool()
    assert_within_one_ulp(masked[keep], full[keep], "unmasked tokens")
    assert not masked[~keep].any()


def test_decoder_layer_padding_mask(cuda_dev):
    """Decoder layer with a padding_mask: a masked token's output is its
    post-attention residual exactly; the others match the unmasked layer to
    the rounding of the MoE output (the unmasked layer rounds residual + MoE
    once, the masked path rounds the MoE output to bf16 first: at most half
    an ulp of |MoE| <= |out| + |residual|, plus one ulp of the sum)."""
    from nki_moe_7013_b200.config import Qwen3MoeConfig
    from nki_moe_7013_b200.decoder import Qwen3MoeDecoderLayer

    cfg = Qwen3MoeConfig()
    layer = Qwen3MoeDecoderLayer(cfg, device=cuda_dev, seed=13)
    B, S, H = 2, 48, cfg.hidden_size
    x = activations(65, B * S, H, cuda_dev).reshape(B, S, H)
    pm = torch.ones(B * S, dtype=torch.float32, device=cuda_dev)
    pm[S:S + 5] = 0.0
    full = layer(x, capture_intermediates=True)[0].reshape(B * S, H)
    masked = layer(x, padding_mask=pm, capture_intermediates=True)[0].reshape(B * S, H)
    residual = layer.last["residual"]
    torch.cuda.synchronize()
    keep = pm.bool()
    assert torch.equal(masked[~keep], residual[~keep])
    m, f, r = masked[keep].float(), full[keep].float(), residual[keep].float()
    tol = 2.0 ** -7 * (f.abs() + r.abs()) + 1e-6
    assert bool(((m - f).abs() <= tol).all()), float(((m - f).abs() - tol).max())
