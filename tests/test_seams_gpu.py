"""The reference's operator seams on the GPU: ExpertMLPsV2
.torch_blockwise_matmul_inference (qwen_with_nki.py:5872-5881) and
.forward_selective_loading (qwen_with_nki.py:2377-2453), plus the module
drop-ins, against the CPU oracle."""
import numpy as np
import pytest
import torch

from helpers import MAX_REL, activations, max_rel_err, moe_weights, to_f32_np

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
