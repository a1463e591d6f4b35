"""Attention sub-layer kernels (RMSNorm, dense projection, QK-norm + RoPE +
cache append, flash-prefill, split-KV flash-decode) and the decoder layer,
against the CPU oracle.  Activation tolerance: max relative error <= 2e-2."""
import numpy as np
import pytest
import torch

from helpers import MAX_REL, activations, max_rel_err, moe_weights, to_f32_np

pytestmark = pytest.mark.gpu


def test_rmsnorm_known_answer_on_gpu(cuda_dev, oracle):
    """The reference's RMSNorm self-test (nki_custom_rmsnorm.py:182-214): seed 42,
    x ~ randn(256, 512) fp32, w ~ randn(512), eps 1e-6, pass if max diff < 1e-3."""
    from nki_moe_7013_b200 import ops

    np.random.seed(42)
    x = np.random.randn(256, 512).astype(np.float32)
    w = np.random.randn(512).astype(np.float32)
    expected = oracle.numpy_rmsnorm_known_answer(x, w, 1e-6)
    got = ops.rmsnorm(torch.from_numpy(x).to(cuda_dev), torch.from_numpy(w).to(cuda_dev), 1e-6,
                      out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert np.max(np.abs(got.cpu().numpy() - expected)) < 1e-3


@pytest.mark.parametrize("rows,H", [(1, 2048), (1000, 2048), (33, 512), (4096, 2048), (2500, 4096)])
def test_rmsnorm_bf16_and_fused_residual(cuda_dev, oracle, rows, H):
    from nki_moe_7013_b200 import ops

    x = activations(rows, rows, H, cuda_dev)
    r = activations(rows + 1, rows, H, cuda_dev)
    w = (1.0 + 0.1 * torch.randn(H, device=cuda_dev)).float()
    y = ops.rmsnorm(x, w, 1e-6)
    y2, s = ops.rmsnorm(x, w, 1e-6, residual=r)
    torch.cuda.synchronize()
    ref = oracle.rmsnorm(to_f32_np(x), w.cpu().numpy(), 1e-6)
    assert max_rel_err(to_f32_np(y), ref) < 1e-2
    s_ref = oracle.round_to_bf16(to_f32_np(x) + to_f32_np(r))
    assert np.array_equal(to_f32_np(s), s_ref)  # the residual stream is bit-exact
    assert max_rel_err(to_f32_np(y2), oracle.rmsnorm(s_ref, w.cpu().numpy(), 1e-6)) < 1e-2


@pytest.mark.parametrize("H", [2048, 4096])
def test_rmsnorm_prefill_rows_match_decode_rows(cuda_dev, H):
    """bf16 RMSNorm over many rows (the low-register prefill kernel) equals,
    bit for bit, the same rows normalised 1024 at a time (the kernel that
    holds the norm weight in registers), with and without the residual add,
    for bf16 and fp32 outputs."""
    from nki_moe_7013_b200 import ops

    rows = 4096
    x = activations(80 + H, rows, H, cuda_dev)
    r = activations(81 + H, rows, H, cuda_dev)
    w = (1.0 + 0.1 * torch.randn(H, device=cuda_dev)).float()
    for dt in (torch.bfloat16, torch.float32):
        whole = ops.rmsnorm(x, w, 1e-6, out_dtype=dt)
        parts = torch.cat([ops.rmsnorm(x[i:i + 1024], w, 1e-6, out_dtype=dt) for i in range(0, rows, 1024)])
        assert torch.equal(whole, parts)
        y, s = ops.rmsnorm(x, w, 1e-6, residual=r, out_dtype=dt)
        pieces = [ops.rmsnorm(x[i:i + 1024], w, 1e-6, residual=r[i:i + 1024], out_dtype=dt)
                  for i in range(0, rows, 1024)]
        assert torch.equal(y, torch.cat([p[0] for p in pieces]))
        assert torch.equal(s, torch.cat([p[1] for p in pieces]))


@pytest.mark.parametrize("T,K,N", [(1, 2048, 5120), (1024, 2048, 5120), (77, 4096, 2048), (300, 256, 384),
                                   (700, 4096, 2048), (2048, 2048, 5120), (513, 2048, 384), (1100, 2048, 5120)])
def test_linear_tcgen05(cuda_dev, T, K, N):
    from nki_moe_7013_b200 import ops

    x = activations(T + K, T, K, cuda_dev)
    w = activations(N, N, K, cuda_dev) * 0.02
    w = w.to(torch.bfloat16).contiguous()
    y = ops.linear(x, w)
    torch.cuda.synchronize()
    ref = to_f32_np(x).astype(np.float64) @ to_f32_np(w).astype(np.float64).T
    assert max_rel_err(to_f32_np(y), ref) < 1e-2


@pytest.mark.parametrize("T,K,N", [(1, 2048, 5120), (3, 4096, 2048), (16, 2048, 512), (2, 2048, 151936)])
def test_linear_decode_split_k(cuda_dev, T, K, N):
    """Decode rows with a split-K scratch: same result as the unsplit call up
    to fp32 summation order, run-to-run identical, counters left at zero."""
    from nki_moe_7013_b200 import _C, ops

    x = activations(T + 7, T, K, cuda_dev)
    w = (activations(N + 1, N, K, cuda_dev) * 0.02).to(torch.bfloat16).contiguous()
    ws = ops.gateup_split_workspace(cuda_dev)
    plain = ops.linear(x, w)
    runs = [ops.linear(x, w, split_ws=ws) for _ in range(2)]
    torch.cuda.synchronize()
    assert _C.device_error() == 0
    assert torch.equal(runs[0], runs[1])
    n_slot_floats = 256 * 2 * 16 * 128
    assert torch.count_nonzero(ws.view(torch.int32)[n_slot_floats:n_slot_floats + 256]).item() == 0
    assert max_rel_err(to_f32_np(runs[0]), to_f32_np(plain)) < 1e-2
    ref = to_f32_np(x).astype(np.float64) @ to_f32_np(w).astype(np.float64).T
    assert max_rel_err(to_f32_np(runs[0]), ref) < 1e-2


@pytest.mark.parametrize("T,K,N", [(1, 2048, 5120), (2, 4096, 2048), (3, 1024, 384), (4, 2048, 1024),
                                   (4, 4096, 2048), (5, 2048, 5120)])
def test_linear_decode_rows(cuda_dev, T, K, N):
    """Decode rows (T <= 4) run the CUDA-core projection (5 rows: the
    tensor-core kernel): within the tolerance of an fp64 reference,
    run-to-run identical, and within the same tolerance of the tensor-core
    path (a 9-row call whose first T rows are these)."""
    from nki_moe_7013_b200 import _C, ops

    x9 = activations(T + K + 1, 9, K, cuda_dev)
    x = x9[:T].contiguous()
    w = (activations(N + 3, N, K, cuda_dev) * 0.02).to(torch.bfloat16).contiguous()
    runs = [ops.linear(x, w) for _ in range(2)]
    tc = ops.linear(x9, w)[:T]
    torch.cuda.synchronize()
    assert _C.device_error() == 0
    assert torch.equal(runs[0], runs[1])
    ref = to_f32_np(x).astype(np.float64) @ to_f32_np(w).astype(np.float64).T
    assert max_rel_err(to_f32_np(runs[0]), ref) < 1e-2
    assert max_rel_err(to_f32_np(runs[0]), to_f32_np(tc)) < 1e-2


def _attn_weights(cuda_dev, H, nh, nkv, seed):
    from nki_moe_7013_b200.synth import normal_bf16_device

    hd = 128
    wqkv = normal_bf16_device(seed * 10 + 5, ((nh + 2 * nkv) * hd, H), 0.02, cuda_dev)
    wo = normal_bf16_device(seed * 10 + 6, (H, nh * hd), 0.02, cuda_dev)
    g = torch.Generator(device=cuda_dev)
    g.manual_seed(seed)
    qn = (1.0 + 0.1 * torch.randn(hd, generator=g, device=cuda_dev)).float()
    kn = (1.0 + 0.1 * torch.randn(hd, generator=g, device=cuda_dev)).float()
    return wqkv, wo, qn, kn


# (2, 5, 4096) / (4, 5, 300): speculative-decoding verify shapes -- 5 new
# tokens per sequence on top of a filled cache
@pytest.mark.parametrize("B,S,L0", [(1, 1024, 0), (2, 200, 0), (2, 70, 37), (3, 1, 100), (2, 5, 4096), (4, 5, 300)])
def test_attention_layer_vs_oracle(cuda_dev, oracle, B, S, L0):
    """Projection -> QK-norm/RoPE/cache append -> prefill or decode -> o_proj,
    continuing a cache that already holds L0 tokens per sequence."""
    from nki_moe_7013_b200.attention import AttnWeights, KVCache, Qwen3MoeAttention
    from nki_moe_7013_b200.config import Qwen3MoeConfig

    cfg = Qwen3MoeConfig()
    H, nh, nkv = cfg.hidden_size, cfg.num_attention_heads, cfg.num_key_value_heads
    wqkv, wo, qn, kn = _attn_weights(cuda_dev, H, nh, nkv, 3 + S)
    attn = Qwen3MoeAttention(cfg, AttnWeights(wqkv, wo, qn, kn))
    cache = KVCache(B, nkv, L0 + S + 5, 128, cuda_dev)
    k_prev = v_prev = None
    if L0:
        cache.fill_random(L0, seed=5)
        k_prev = cache.k.float().cpu().numpy()
        v_prev = cache.v.float().cpu().numpy()
    x = activations(S, B * S, H, cuda_dev).reshape(B, S, H)
    out, cache = attn(x, past_key_value=cache)
    torch.cuda.synchronize()
    from nki_moe_7013_b200 import _C

    assert _C.device_error() == 0
    ref, new_k, new_v = oracle.attention_layer(
        x.reshape(B * S, H).cpu(), wqkv.cpu(), wo.cpu(), qn.cpu().numpy(), kn.cpu().numpy(), nh, nkv,
        cfg.rms_norm_eps, cfg.rope_theta, B, S, k_cache=k_prev, v_cache=v_prev, L0=[L0] * B)
    err = max_rel_err(to_f32_np(out).reshape(B * S, H), ref)
    assert err <= MAX_REL, f"attention layer max rel err {err:.3e}"
    assert cache.lengths == [L0 + S] * B
    # the appended K rows (normalised + rotated) and V rows
    got_k = cache.k[:, :, L0:L0 + S].float().cpu().numpy()
    assert max_rel_err(got_k, new_k[:, :, L0:L0 + S]) < 1e-2
    got_v = cache.v[:, :, L0:L0 + S].float().cpu().numpy()
    # V rows are the bf16 projection output: equal up to the last-bit rounding
    # of fp32 (GPU) vs fp64 (oracle) accumulation
    assert max_rel_err(got_v, new_v[:, :, L0:L0 + S]) < 1e-2


@pytest.mark.parametrize("B,L", [(1, 4096), (8, 4096), (4, 77), (2, 1)])
def test_flash_decode_long_cache(cuda_dev, oracle, B, L):
    """Config-2 decode shape: every sequence holds L cached tokens (~N(0,1))."""
    from nki_moe_7013_b200 import ops

    nh, nkv, hd = 32, 4, 128
    k = torch.randn(B, nkv, L + 8, hd, device=cuda_dev).to(torch.bfloat16)
    v = torch.randn(B, nkv, L + 8, hd, device=cuda_dev).to(torch.bfloat16)
    q = torch.randn(B, nh, hd, device=cuda_dev).to(torch.bfloat16)
    lens = torch.tensor([L - (b % 3) if L > 3 else L for b in range(B)], dtype=torch.int32, device=cuda_dev)
    out = ops.attention_decode(q, k, v, lens, int(lens.max().item()))
    torch.cuda.synchronize()
    qf, kf, vf = (t.double().cpu().numpy() for t in (q, k, v))
    ref = np.zeros((B, nh, hd))
    for b in range(B):
        n = int(lens[b])
        for h in range(nh):
            g = h // 8
            s = qf[b, h] @ kf[b, g, :n].T / np.sqrt(hd)
            p = np.exp(s - s.max())
            ref[b, h] = (p / p.sum()) @ vf[b, g, :n]
    assert max_rel_err(to_f32_np(out).reshape(B, nh, hd), ref) <= MAX_REL


def test_decoder_layer_cfg1_vs_oracle(cuda_dev, oracle):
    """Config 1: full decoder layer, prefill 1 x 1024 tokens."""
    from nki_moe_7013_b200.attention import AttnWeights
    from nki_moe_7013_b200.config import Qwen3MoeConfig
    from nki_moe_7013_b200.decoder import Qwen3MoeDecoderLayer
    from nki_moe_7013_b200.moe import MoEWeights

    cfg = Qwen3MoeConfig()
    B, S, H = 1, 1024, cfg.hidden_size
    wqkv, wo, qn, kn = _attn_weights(cuda_dev, H, cfg.num_attention_heads, cfg.num_key_value_heads, 11)
    wr, wgu, wd = moe_weights(11, cfg.num_experts, H, cfg.moe_intermediate_size, cuda_dev)
    layer = Qwen3MoeDecoderLayer(cfg, attn_weights=AttnWeights(wqkv, wo, qn, kn),
                                 moe_weights=MoEWeights(wr, wgu, wd), device=cuda_dev, seed=11)
    x = activations(12, B * S, H, cuda_dev).reshape(B, S, H)
    out, present, cos, sin, _ = layer(x, capture_intermediates=True)
    torch.cuda.synchronize()
    assert out.shape == (B, S, H) and present.lengths == [S] and cos is None
    mid = layer.last
    attn_args = dict(wqkv_bf16=wqkv.cpu(), wo_bf16=wo.cpu(), q_norm_w=qn.cpu().numpy(),
                     k_norm_w=kn.cpu().numpy(), nh=cfg.num_attention_heads, nkv=cfg.num_key_value_heads,
                     theta=cfg.rope_theta)
    moe_args = dict(w_router_bf16=wr.cpu(), w_gate_up_bf16=wgu.cpu(), w_down_bf16=wd.cpu(), k=8)
    eps = cfg.rms_norm_eps
    # (1) attention half: input norm -> attention -> residual add, vs the oracle
    x_np = to_f32_np(x).reshape(B * S, H)
    h = oracle.round_to_bf16(oracle.rmsnorm(x_np, layer.input_layernorm.cpu().numpy(), eps))
    a_ref, _, _ = oracle.attention_layer(torch.from_numpy(h).to(torch.bfloat16), B=B, S=S, eps=eps, **attn_args)
    assert max_rel_err(to_f32_np(mid["attn"]), a_ref) <= MAX_REL
    res_ref = oracle.round_to_bf16(x_np + oracle.round_to_bf16(a_ref))
    assert max_rel_err(to_f32_np(mid["residual"]), res_ref) <= MAX_REL
    # (2) MoE half on the GPU's own post-attention activations: routing is
    # bit-exact and the layer output matches residual + MoE
    moe_in = mid["moe_in"].cpu()
    moe_ref, inter = oracle.moe_block(moe_in, **moe_args, return_intermediates=True)
    out_ref = to_f32_np(mid["residual"]) + moe_ref
    err = max_rel_err(to_f32_np(out).reshape(B * S, H), out_ref)
    assert err <= MAX_REL, f"decoder layer max rel err {err:.3e}"
    # (3) end to end from x alone: tokens routed identically by the full oracle
    # chain agree within the bar (a few near-tie tokens may route differently
    # after last-bit differences upstream of the router)
    full = oracle.decoder_layer(x.reshape(B * S, H).cpu(), layer.input_layernorm.cpu().numpy(),
                                layer.post_attention_layernorm.cpu().numpy(), attn_args, moe_args, eps, B, S)
    h2_ref = oracle.round_to_bf16(oracle.rmsnorm(res_ref, layer.post_attention_layernorm.cpu().numpy(), eps))
    _, idx_ref, _ = oracle.router(torch.from_numpy(h2_ref).to(torch.bfloat16), wr.cpu(), 8)
    same = np.all(np.sort(idx_ref, 1) == np.sort(inter["topk_idx"], 1), axis=1)
    assert same.mean() > 0.97
    assert max_rel_err(to_f32_np(out).reshape(B * S, H)[same], full[same]) <= MAX_REL


def _attention_ref_fp32(q, k_cache, v_cache, q_start, slots, pads, B, S, nh, nkv, scale):
    """Plain torch fp32 causal GQA over the cache (the reference of the flash
    kernels): rows [pad, q_start + i] of each sequence's slot; padding
    queries (no visible key) give zeros."""
    out = torch.zeros(B * S, nh, 128, dtype=torch.float32, device=q.device)
    for b in range(B):
        L = q_start[b] + S
        kb = k_cache[slots[b], :, :L].float().repeat_interleave(nh // nkv, dim=0)  # (nh, L, 128)
        vb = v_cache[slots[b], :, :L].float().repeat_interleave(nh // nkv, dim=0)
        qb = q[b * S:(b + 1) * S].float().transpose(0, 1)                           # (nh, S, 128)
        sc = torch.matmul(qb, kb.transpose(1, 2)) * scale                          # (nh, S, L)
        keys = torch.arange(L, device=q.device)[None, :]
        pos = (q_start[b] + torch.arange(S, device=q.device))[:, None]
        masked = (keys > pos) | (keys < pads[b])
        sc = sc.masked_fill(masked[None], float("-inf"))
        live = ~masked.all(dim=1)
        p = torch.softmax(sc.masked_fill(~live[None, :, None], 0.0), dim=-1) * live[None, :, None]
        out[b * S:(b + 1) * S] = torch.matmul(p, vb).transpose(0, 1)
    return out.reshape(B * S, nh * 128)


# (B, S, L0, pads, slots): config-1 shape, partial query / key tiles, a
# continuing cache, left padding (inside a tile, exactly one tile, a whole
# sequence of padding), speculative-verify shape, slot remapping, config-3
# sequence length
@pytest.mark.parametrize("B,S,L0,pads,slots", [
    (1, 1024, 0, None, None),
    (2, 300, 37, [0, 50], None),
    (3, 129, 0, [0, 0, 128], None),
    (1, 5, 4096, None, None),
    (2, 64, 0, [0, 64], None),
    (4, 200, 100, [10, 0, 150, 299], [3, 1, 0, 2]),
    (1, 2048, 0, None, None),
])
def test_flash_prefill_kernel(cuda_dev, B, S, L0, pads, slots):
    """tcgen05 flash prefill against a plain torch fp32 reference.  Cache rows
    past each sequence's end hold NaN: no key past the last query may reach
    the output, not even through a zero probability."""
    from nki_moe_7013_b200 import _C, ops

    nh, nkv, hd = 32, 4, 128
    n_slots = B if slots is None else max(slots) + 1
    max_seq = L0 + S + 40
    g = torch.Generator(device=cuda_dev)
    g.manual_seed(B * 1000 + S)
    k = torch.randn(n_slots, nkv, max_seq, hd, generator=g, device=cuda_dev).to(torch.bfloat16)
    v = torch.randn(n_slots, nkv, max_seq, hd, generator=g, device=cuda_dev).to(torch.bfloat16)
    k[:, :, L0 + S:] = float("nan")
    v[:, :, L0 + S:] = float("nan")
    q = torch.randn(B * S, nh, hd, generator=g, device=cuda_dev).to(torch.bfloat16)
    q_start = torch.full((B,), L0, dtype=torch.int32, device=cuda_dev)
    slot_t = None if slots is None else torch.tensor(slots, dtype=torch.int32, device=cuda_dev)
    kv_start = None if pads is None else torch.tensor(pads, dtype=torch.int32, device=cuda_dev)
    out = ops.attention_prefill(q, k, v, q_start, B, S, cache_slot=slot_t, kv_start=kv_start)
    torch.cuda.synchronize()
    assert _C.device_error() == 0
    ref = _attention_ref_fp32(q, k, v, [L0] * B, slots or list(range(B)), pads or [0] * B, B, S, nh, nkv,
                              hd ** -0.5)
    o = out.float()
    assert torch.isfinite(o).all()
    err = float((o - ref).abs().max() / ref.abs().max())
    assert err <= MAX_REL, f"flash prefill max rel err {err:.3e}"
    if pads is not None:  # padding queries: exact zeros
        for b in range(B):
            n_pad_q = max(0, min(S, pads[b] - L0))
            if n_pad_q:
                assert torch.count_nonzero(out[b * S:b * S + n_pad_q]).item() == 0


def test_flash_prefill_run_to_run_identical(cuda_dev):
    from nki_moe_7013_b200 import ops

    nh, nkv, hd, B, S = 32, 4, 128, 2, 333
    k = torch.randn(B, nkv, S, hd, device=cuda_dev).to(torch.bfloat16)
    v = torch.randn(B, nkv, S, hd, device=cuda_dev).to(torch.bfloat16)
    q = torch.randn(B * S, nh, hd, device=cuda_dev).to(torch.bfloat16)
    qs = torch.zeros(B, dtype=torch.int32, device=cuda_dev)
    a = ops.attention_prefill(q, k, v, qs, B, S)
    b = ops.attention_prefill(q, k, v, qs, B, S)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


@pytest.mark.parametrize("B,L,pads", [(2, 300, [0, 120]), (3, 4096, [4000, 0, 1])])
def test_flash_decode_left_padding(cuda_dev, B, L, pads):
    from nki_moe_7013_b200 import _C, ops

    nh, nkv, hd = 32, 4, 128
    k = torch.randn(B, nkv, L + 8, hd, device=cuda_dev).to(torch.bfloat16)
    v = torch.randn(B, nkv, L + 8, hd, device=cuda_dev).to(torch.bfloat16)
    q = torch.randn(B, nh, hd, device=cuda_dev).to(torch.bfloat16)
    lens = torch.full((B,), L, dtype=torch.int32, device=cuda_dev)
    out = ops.attention_decode(q, k, v, lens, L, kv_start=torch.tensor(pads, dtype=torch.int32, device=cuda_dev))
    torch.cuda.synchronize()
    assert _C.device_error() == 0
    ref = _attention_ref_fp32(q, k, v, [L - 1] * B, list(range(B)), pads, B, 1, nh, nkv, hd ** -0.5)
    assert max_rel_err(to_f32_np(out), ref.cpu().numpy()) <= MAX_REL


def test_attention_left_padding_vs_oracle(cuda_dev, oracle):
    """A left-padded batch through the module (2D attention mask, HF
    convention), then one decode step on the same cache without a mask:
    real rows match the oracle's HF semantics (pad keys masked, RoPE at the
    pad-shifted positions), padding rows are zero."""
    from nki_moe_7013_b200 import _C
    from nki_moe_7013_b200.attention import AttnWeights, KVCache, Qwen3MoeAttention
    from nki_moe_7013_b200.config import Qwen3MoeConfig

    cfg = Qwen3MoeConfig()
    H, nh, nkv = cfg.hidden_size, cfg.num_attention_heads, cfg.num_key_value_heads
    B, S, pads = 2, 70, [0, 23]
    wqkv, wo, qn, kn = _attn_weights(cuda_dev, H, nh, nkv, 77)
    attn = Qwen3MoeAttention(cfg, AttnWeights(wqkv, wo, qn, kn))
    cache = KVCache(B, nkv, S + 4, 128, cuda_dev)
    mask = torch.ones(B, S, dtype=torch.int64)
    for b, p in enumerate(pads):
        mask[b, :p] = 0
    pos = (mask.cumsum(1) - 1).clamp_min(0)
    x = activations(91, B * S, H, cuda_dev).reshape(B, S, H)
    out, cache = attn(x, position_ids=pos, past_key_value=cache, attention_mask=mask)
    torch.cuda.synchronize()
    assert _C.device_error() == 0 and cache.pad == pads
    args = dict(nh=nh, nkv=nkv, eps=cfg.rms_norm_eps, theta=cfg.rope_theta)
    ref, rk, rv = oracle.attention_layer(x.reshape(B * S, H).cpu(), wqkv.cpu(), wo.cpu(), qn.cpu().numpy(),
                                         kn.cpu().numpy(), B=B, S=S, pad=pads, **args)
    o = to_f32_np(out).reshape(B, S, H)
    r = ref.reshape(B, S, H)
    for b, p in enumerate(pads):
        assert max_rel_err(o[b, p:], r[b, p:]) <= MAX_REL
        assert np.count_nonzero(o[b, :p]) == 0
    # one decode step: the cache keeps masking the padding
    x1 = activations(92, B, H, cuda_dev).reshape(B, 1, H)
    out1, cache = attn(x1, past_key_value=cache)
    torch.cuda.synchronize()
    ref1, _, _ = oracle.attention_layer(x1.reshape(B, H).cpu(), wqkv.cpu(), wo.cpu(), qn.cpu().numpy(),
                                        kn.cpu().numpy(), B=B, S=1, k_cache=rk, v_cache=rv, L0=[S] * B,
                                        pad=pads, **args)
    assert max_rel_err(to_f32_np(out1).reshape(B, H), ref1) <= MAX_REL
