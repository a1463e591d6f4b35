"""The fused MoE block (post-attention add & norm + MoE + residual add, one
library call).  Its add & norm outputs equal the standalone RMSNorm kernel's
bit for bit and are checked against the oracle; its routing equals
moe_forward's on those rows bit for bit; its output is within the
activation tolerance of the oracle's block on the same rows and within one
bf16 ulp of the two-call path, at decode and prefill sizes."""
import numpy as np
import pytest
import torch

from helpers import MAX_REL, activations, assert_within_one_ulp, max_rel_err, moe_weights, to_f32_np

pytestmark = pytest.mark.gpu

EPS = 1e-6


def _norm_weight(seed, H, dev):
    g = torch.Generator().manual_seed(seed)
    return (1.0 + 0.1 * torch.randn(H, generator=g)).float().to(dev)


@pytest.mark.parametrize("T,H,E,k,I", [(1, 2048, 128, 8, 768), (2, 2048, 128, 8, 768), (5, 2048, 128, 8, 768),
                                       (16, 2048, 128, 8, 768), (17, 2048, 128, 8, 768), (100, 2048, 128, 8, 768),
                                       (1024, 2048, 128, 8, 768), (7, 4096, 64, 8, 128), (3, 256, 32, 4, 128),
                                       (12, 1024, 32, 32, 256)])
def test_block_forward_matches_norm_then_moe(cuda_dev, oracle, T, H, E, k, I):
    from nki_moe_7013_b200 import _C, ops

    wr, wgu, wd = moe_weights(70 + T, E, H, I, cuda_dev)
    a = activations(70 + T, T, H, cuda_dev)
    res = activations(71 + T, T, H, cuda_dev)
    w = _norm_weight(T, H, cuda_dev)
    h = torch.empty_like(a)
    s = torch.empty_like(a)
    out, idx, tw = ops.moe_block_forward(a, res, w, EPS, wr, wgu, wd, k, moe_in_out=h, residual_out=s,
                                         return_routing=True)
    out2 = ops.moe_block_forward(a, res, w, EPS, wr, wgu, wd, k)  # add & norm outputs in the workspace
    h_ref, s_ref = ops.rmsnorm(a, w, EPS, residual=res)
    out_ref, idx_ref, tw_ref = ops.moe_forward(h_ref, wr, wgu, wd, k, residual=s_ref, return_routing=True)
    torch.cuda.synchronize()
    assert _C.device_error() == 0
    # the add & norm: bit for bit the standalone kernel's, and the oracle's
    assert torch.equal(s, s_ref) and torch.equal(h, h_ref)
    s_np = oracle.round_to_bf16(to_f32_np(a) + to_f32_np(res))
    assert np.array_equal(to_f32_np(s), s_np)
    assert max_rel_err(to_f32_np(h), oracle.round_to_bf16(oracle.rmsnorm(s_np, w.cpu().numpy(), EPS))) < 1e-2
    # routing of the normalised rows: bit for bit
    assert torch.equal(idx, idx_ref) and torch.equal(tw, tw_ref)
    # the block output against the oracle's block on the same rows
    ref_out, inter = oracle.moe_block(h.cpu(), wr.cpu(), wgu.cpu(), wd.cpu(), k, return_intermediates=True)
    assert np.array_equal(idx.cpu().numpy(), inter["topk_idx"])
    assert max_rel_err(to_f32_np(out), oracle.round_to_bf16(ref_out + s_np)) <= MAX_REL
    # the same arithmetic as the two calls (the combine adds in arrival order,
    # so the fp32 sums may differ in their last bits)
    assert_within_one_ulp(out, out_ref, "block vs norm + moe_forward")
    assert_within_one_ulp(out2, out_ref, "block (outputs in the workspace) vs norm + moe_forward")


@pytest.mark.parametrize("T", [1, 5, 16, 24, 64, 65, 300])
def test_block_forward_stays_inside_its_workspace(cuda_dev, T):
    """Nothing is written past the reported workspace size."""
    from nki_moe_7013_b200 import _C, ops

    H, E, k, I = 2048, 128, 8, 768
    guard = 1 << 16
    wr, wgu, wd = moe_weights(97 + T, E, H, I, cuda_dev)
    a = activations(97 + T, T, H, cuda_dev)
    res = activations(98 + T, T, H, cuda_dev)
    w = _norm_weight(T, H, cuda_dev)
    nb = ops.moe_block_forward_workspace_size(T, H, E, k, I)
    ws = torch.full((nb + guard,), 0x5A, dtype=torch.uint8, device=cuda_dev)
    out = ops.moe_block_forward(a, res, w, EPS, wr, wgu, wd, k, workspace=ws)
    torch.cuda.synchronize()
    assert _C.device_error() == 0
    assert int((ws[nb:] != 0x5A).sum()) == 0
    assert torch.isfinite(out.float()).all()


def test_block_forward_plan_graph_replay(cuda_dev):
    """MoEPlan.run_block captured in a CUDA graph and replayed gives the eager
    call's result (the decode step's use)."""
    from nki_moe_7013_b200 import _C, ops
    from nki_moe_7013_b200.moe import MoEPlan, MoEWeights

    T, H, E, k, I = 8, 2048, 128, 8, 768
    wr, wgu, wd = moe_weights(81, E, H, I, cuda_dev)
    plan = MoEPlan(MoEWeights(wr, wgu, wd), T, k)
    a = activations(81, T, H, cuda_dev)
    res = activations(82, T, H, cuda_dev)
    w = _norm_weight(3, H, cuda_dev)
    eager = torch.empty_like(a)
    plan.run_block(a, res, w, EPS, eager)
    torch.cuda.synchronize()
    out = torch.zeros_like(a)
    s = torch.cuda.Stream(cuda_dev)
    s.wait_stream(torch.cuda.current_stream(cuda_dev))
    with torch.cuda.stream(s):
        plan.run_block(a, res, w, EPS, out)
    torch.cuda.current_stream(cuda_dev).wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        plan.run_block(a, res, w, EPS, out)
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert _C.device_error() == 0
    assert_within_one_ulp(out, eager, "graph replay vs eager")
    ref = ops.moe_block_forward(a, res, w, EPS, wr, wgu, wd, k)
    torch.cuda.synchronize()
    assert_within_one_ulp(out, ref, "graph replay vs ops.moe_block_forward")
    del g
