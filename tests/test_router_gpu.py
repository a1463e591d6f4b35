"""K1 router parity on the GPU: logits and expert indices bit-exact against the
C oracle (same fp32 reduction order), weights within fp32 rounding."""
import numpy as np
import pytest
import torch

from helpers import activations, moe_weights

pytestmark = pytest.mark.gpu


def _run(x, wr, k, bias=None, normalize=True):
    from nki_moe_7013_b200 import ops

    idx, w, logits, hist = ops.router_topk(x, wr, k, normalize=normalize, bias=bias,
                                           return_logits=True, return_hist=True)
    torch.cuda.synchronize()
    return idx.cpu().numpy(), w.cpu().numpy(), logits.cpu().numpy(), hist.cpu().numpy()


# 2000 and 1300 tokens: more chunks than SMs, the two-CTAs-per-SM configuration
@pytest.mark.parametrize("T,H,E,k", [(1, 2048, 128, 8), (7, 256, 32, 4), (128, 2048, 128, 8),
                                     (1000, 2048, 128, 8), (33, 512, 64, 8), (9, 4096, 256, 32),
                                     (2000, 2048, 128, 8), (1300, 512, 64, 8)])
def test_router_matches_oracle(cuda_dev, oracle, T, H, E, k):
    from nki_moe_7013_b200.synth import normal_bf16_device

    wr = normal_bf16_device(11 + T, (E, H), 0.02, cuda_dev)
    x = activations(T, T, H, cuda_dev)
    idx, w, logits, hist = _run(x, wr, k)
    ref_logits, ref_idx, ref_w = oracle.router(x.cpu(), wr.cpu(), k, True)
    assert np.array_equal(logits.view(np.uint32), ref_logits.view(np.uint32)), "logits not bit-exact"
    assert np.array_equal(idx, ref_idx), "expert indices differ"
    np.testing.assert_allclose(w, ref_w, rtol=2e-6, atol=1e-7)
    # chunk histogram = per-chunk expert counts
    chunk = 8
    for c in range(hist.shape[0]):
        sel = ref_idx[c * chunk:(c + 1) * chunk].reshape(-1)
        np.testing.assert_array_equal(hist[c], np.bincount(sel, minlength=E))


def test_router_ties_lower_index_wins(cuda_dev, oracle):
    from nki_moe_7013_b200.synth import normal_bf16_device

    T, H, E, k = 16, 2048, 128, 8
    wr = normal_bf16_device(5, (E, H), 0.02, cuda_dev)
    # duplicated expert rows give exactly equal logits
    for a, b in [(3, 77), (10, 11), (120, 5), (64, 65), (0, 127)]:
        wr[b] = wr[a]
    x = activations(3, T, H, cuda_dev)
    x[0].zero_()                      # all 128 logits equal -> experts 0..7
    x[1] = x[2]                       # identical tokens
    idx, w, logits, _ = _run(x, wr, k)
    ref_logits, ref_idx, ref_w = oracle.router(x.cpu(), wr.cpu(), k, True)
    assert np.array_equal(idx, ref_idx)
    assert list(idx[0]) == list(range(8))
    np.testing.assert_allclose(w[0], np.full(8, 0.125, np.float32), rtol=1e-6)
    assert np.array_equal(idx[1], idx[2])
    np.testing.assert_allclose(w, ref_w, rtol=2e-6, atol=1e-7)


def test_router_bias_and_unnormalized(cuda_dev, oracle):
    from nki_moe_7013_b200.synth import normal_bf16_device, zipf_expert_bias

    T, H, E, k = 64, 2048, 128, 8
    wr = normal_bf16_device(7, (E, H), 0.02, cuda_dev)
    x = activations(8, T, H, cuda_dev)
    bias = zipf_expert_bias(0, E).to(cuda_dev)
    idx, w, logits, _ = _run(x, wr, k, bias=bias, normalize=False)
    ref_logits, ref_idx, ref_w = oracle.router(x.cpu(), wr.cpu(), k, False, bias=bias.cpu().numpy())
    assert np.array_equal(logits.view(np.uint32), ref_logits.view(np.uint32))
    assert np.array_equal(idx, ref_idx)
    np.testing.assert_allclose(w, ref_w, rtol=2e-6, atol=1e-8)


@pytest.mark.parametrize("T,H,E,k", [(1, 2048, 128, 8), (2, 2048, 128, 8), (5, 256, 32, 4), (16, 2048, 128, 8),
                                     (7, 4096, 64, 8), (16, 512, 128, 1), (3, 1024, 32, 32)])
def test_route_small_matches_router_and_permute(cuda_dev, oracle, T, H, E, k):
    """The one-launch decode route (router + permutation in a cluster) gives
    the oracle's routing and rows bit for bit, and zero-fills the accumulator."""
    from nki_moe_7013_b200 import ops

    wr = moe_weights(50 + T, E, H, 128, cuda_dev)[0]
    x = activations(50 + T, T, H, cuda_dev)
    acc = torch.full((T, H), 3.0, dtype=torch.float32, device=cuda_dev)
    r = ops.route_small(x, wr, k, acc_zero=acc)
    torch.cuda.synchronize()
    ref_logits, ref_idx, ref_w = oracle.router(x.cpu(), wr.cpu(), k, True)
    assert np.array_equal(r["logits"].cpu().numpy().view(np.uint32), ref_logits.view(np.uint32))
    assert np.array_equal(r["topk_idx"].cpu().numpy(), ref_idx)
    np.testing.assert_allclose(r["topk_w"].cpu().numpy(), ref_w, rtol=2e-6, atol=1e-7)
    # identical to the separate kernels
    idx, w, hist = ops.router_topk(x, wr, k, return_hist=True)
    p = ops.moe_permute(idx, w, hist, E, x=x, gather=False)
    torch.cuda.synchronize()
    assert torch.equal(r["topk_w"], w)
    for key in ("counts", "offsets", "row_token", "row_w", "slot_row"):
        assert torch.equal(r[key], p[key]), key
    nt = int(p["tiles"][0])
    mt = p["max_tiles"]
    assert int(r["tiles"][0]) == nt
    for part in range(3):
        assert torch.equal(r["tiles"][1 + part * mt:1 + part * mt + nt], p["tiles"][1 + part * mt:1 + part * mt + nt])
    assert torch.count_nonzero(acc).item() == 0
    ref = oracle.permute(idx.cpu().numpy(), E)
    np.testing.assert_array_equal(r["row_token"].cpu().numpy(), ref["row_token"])


@pytest.mark.parametrize("T,H,E,k", [(1000, 2048, 128, 8), (65, 512, 64, 4), (1184, 256, 32, 8), (1300, 2048, 128, 8),
                                     (300, 4096, 256, 8)])
def test_route_permute_matches_router_and_permute(cuda_dev, oracle, T, H, E, k):
    """Router + permutation in one call (one launch up to one router chunk per
    SM, 1300 tokens: the two kernels) gives the separate kernels' outputs bit
    for bit, and zero-fills the accumulator and the counters."""
    from nki_moe_7013_b200 import _C, ops

    wr = moe_weights(60 + T, E, H, 128, cuda_dev)[0]
    x = activations(60 + T, T, H, cuda_dev)
    acc = torch.full((T, H), 3.0, dtype=torch.float32, device=cuda_dev)
    r = ops.route_permute(x, wr, k, acc_zero=acc)
    r2 = ops.route_permute(x, wr, k)  # a second call on fresh (uninitialised) outputs
    r3 = ops.route_permute(x, wr, k, gather=False)  # no permuted copy (the expert-parallel step)
    idx, w, hist = ops.router_topk(x, wr, k, return_hist=True)
    p = ops.moe_permute(idx, w, hist, E, x=x, gather=True)
    torch.cuda.synchronize()
    assert _C.device_error() == 0
    assert torch.equal(r["topk_idx"], idx) and torch.equal(r["topk_w"], w)
    for key in ("counts", "offsets", "row_token", "row_w", "slot_row", "x_perm"):
        assert torch.equal(r[key], p[key]), key
        assert torch.equal(r2[key], p[key]), key
        if key != "x_perm":
            assert torch.equal(r3[key], p[key]), key
    nt = int(p["tiles"][0])
    mt = p["max_tiles"]
    assert int(r["tiles"][0]) == nt
    for part in range(3):
        assert torch.equal(r["tiles"][1 + part * mt:1 + part * mt + nt], p["tiles"][1 + part * mt:1 + part * mt + nt])
    assert torch.count_nonzero(acc).item() == 0
    assert torch.count_nonzero(r2["done"]).item() == 0
    assert torch.count_nonzero(r["barrier"]).item() == 0  # left zero for the next call
    ref = oracle.permute(idx.cpu().numpy(), E)
    np.testing.assert_array_equal(r["row_token"].cpu().numpy(), ref["row_token"])
