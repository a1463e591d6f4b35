"""The CPU oracle on its own: canonical router order, tie rule, permutation
invariants, the reference's RMSNorm known-answer test, blockwise seam."""
import numpy as np
import torch

from nki_moe_7013_b200.synth import bf16_bits_to_f32, normal_bf16


def test_router_logits_follow_canonical_order(oracle):
    T, H, E = 3, 512, 32
    x = normal_bf16(1, "x", (T, H))
    w = normal_bf16(1, "w", (E, H), 0.02)
    got = oracle.router_logits(x, w)
    xf = bf16_bits_to_f32(x.view(torch.int16).numpy().view(np.uint16))
    wf = bf16_bits_to_f32(w.view(torch.int16).numpy().view(np.uint16))
    for t in range(T):
        for e in range(E):
            lanes = []
            for l in range(32):
                acc = np.float32(0)
                for g in range(H // 256):
                    for q in range(8):
                        i = 256 * g + 8 * l + q
                        acc = np.float32(acc + np.float32(xf[t, i] * wf[e, i]))
                lanes.append(acc)
            s = lanes
            for off in (16, 8, 4, 2, 1):
                s = [np.float32(s[l] + s[l ^ off]) for l in range(32)]
            assert got[t, e].view(np.uint32) == np.float32(s[0]).view(np.uint32)
    # and close to the plain dot product
    np.testing.assert_allclose(got, xf @ wf.T, rtol=1e-4, atol=1e-5)


def test_topk_ties_go_to_lower_index(oracle):
    logits = np.zeros((2, 16), np.float32)
    logits[1, [3, 9, 12]] = 1.0
    idx = oracle.topk(logits, 4)
    assert list(idx[0]) == [0, 1, 2, 3]
    assert list(idx[1]) == [3, 9, 12, 0]


def test_router_weights_normalised(oracle):
    x = normal_bf16(2, "x", (64, 2048))
    w = normal_bf16(2, "w", (128, 2048), 0.02)
    logits, idx, tw = oracle.router(x, w, 8, True)
    np.testing.assert_allclose(tw.sum(1), 1.0, rtol=1e-6)
    assert np.all(np.diff(np.take_along_axis(logits, idx.astype(np.int64), 1), axis=1) <= 0)
    assert all(len(set(r)) == 8 for r in idx)


def test_permute_invariants(oracle):
    rng = np.random.default_rng(0)
    T, E, k = 200, 32, 4
    idx = np.stack([rng.choice(E, k, replace=False) for _ in range(T)]).astype(np.int32)
    p = oracle.permute(idx, E)
    assert p["offsets"][-1] == T * k
    np.testing.assert_array_equal(p["counts"], np.bincount(idx.reshape(-1), minlength=E))
    for e in range(E):
        toks = p["row_token"][p["offsets"][e]:p["offsets"][e + 1]]
        assert np.all(np.diff(toks) > 0)  # ascending token id inside an expert
    for t in range(T):
        for j in range(k):
            r = p["slot_row"][t, j]
            assert p["row_token"][r] == t and p["row_slot"][r] == j


def test_rmsnorm_known_answer(oracle):
    """The reference's RMSNorm self-test (nki_custom_rmsnorm.py:182-214):
    seed 42, x ~ randn(256, 512), w ~ randn(512), eps 1e-6, pass if max diff < 1e-3."""
    np.random.seed(42)
    x = np.random.randn(256, 512).astype(np.float32)
    w = np.random.randn(512).astype(np.float32)
    expected = oracle.numpy_rmsnorm_known_answer(x, w, 1e-6)
    got = oracle.rmsnorm(x, w, 1e-6)
    assert np.max(np.abs(expected - got)) < 1e-3
    assert np.max(np.abs(expected - got)) < 1e-5


def test_blockwise_matches_routed_block(oracle):
    """The NxDI blockwise seam and the routed block agree when blocks carry the
    routed tokens (duplicates and padding slots included)."""
    T, H, E, k, I, B = 24, 256, 32, 4, 128, 16
    x = normal_bf16(3, "x", (T, H))
    wr = normal_bf16(3, "wr", (E, H), 0.02)
    wgu = normal_bf16(3, "wgu", (E, 2 * I, H), 0.02)
    wd = normal_bf16(3, "wd", (E, H, I), 0.02)
    out, inter = oracle.moe_block(x, wr, wgu, wd, k, return_intermediates=True)
    aff = np.zeros((T, E), np.float32)
    for t in range(T):
        aff[t, inter["topk_idx"][t]] = inter["topk_w"][t]
    tpi, b2e = [], []
    for e in range(E):
        toks = list(inter["row_token"][inter["offsets"][e]:inter["offsets"][e + 1]])
        if not toks:
            continue
        toks = toks + toks[:1]  # a duplicate inside the block
        for s in range(0, len(toks), B):
            blk = toks[s:s + B]
            blk = blk + [-1] * (B - len(blk))  # padding slots
            tpi += blk
            b2e.append(e)
    got = oracle.blockwise_moe(x, aff, np.array(tpi), np.array(b2e), B, wgu, wd)
    np.testing.assert_allclose(got, out, rtol=1e-5, atol=1e-6)
