"""The decoder stack (config-2 decode): embedding lookup bit for bit, the
static-shape decode step against the eager module path, the CUDA-graph replay
against eager steps, and the final norm + LM head against the oracle."""
import numpy as np
import pytest
import torch

from helpers import MAX_REL, max_rel_err, to_f32_np

pytestmark = pytest.mark.gpu


def test_embedding_gather_bit_exact(cuda_dev):
    from nki_moe_7013_b200 import _C, ops

    V, H = 1000, 2048
    table = torch.randn(V, H, device=cuda_dev).to(torch.bfloat16)
    ids = torch.tensor([0, 999, 17, 17, 500], dtype=torch.int32, device=cuda_dev)
    out = ops.embedding(ids, table)
    torch.cuda.synchronize()
    assert torch.equal(out, table[ids.long()])
    assert _C.device_error() == 0
    # ids outside [0, V): zero rows and device error 4, the other rows intact
    bad = torch.tensor([3, V, -1], dtype=torch.int32, device=cuda_dev)
    out = ops.embedding(bad, table)
    torch.cuda.synchronize()
    assert _C.device_error() == 4
    assert torch.equal(out[0], table[3]) and not out[1:].any()


def _small_model(cuda_dev, layers=2, vocab=2048, seed=3):
    from nki_moe_7013_b200.config import Qwen3MoeConfig
    from nki_moe_7013_b200.model import Qwen3MoeModel

    return Qwen3MoeModel(Qwen3MoeConfig(), num_layers=layers, vocab_size=vocab, device=cuda_dev, seed=seed)


@pytest.mark.parametrize("B", [1, 3])
def test_decode_step_matches_module_path(cuda_dev, oracle, B):
    from nki_moe_7013_b200 import _C
    from nki_moe_7013_b200.attention import KVCache
    from nki_moe_7013_b200.model import DecodeSession

    model = _small_model(cuda_dev)
    ctx = 64
    # projections without split K: the module path runs them unsplit, and a
    # different fp32 summation order could flip a near-tie in the routing
    sess = DecodeSession(model, B, context=ctx, max_new=8, seed=5, split_k=False)
    # the module path on copies of the same caches (host-side lengths = ctx)
    caches = []
    for c in sess.caches:
        k = KVCache(B, c.k.shape[1], c.max_seq, c.k.shape[3], device=cuda_dev)
        k.k.copy_(c.k)
        k.v.copy_(c.v)
        k.lengths = [ctx] * B
        caches.append(k)
    tokens = sess.tokens.clone()
    ref_logits, _ = model.forward(tokens.reshape(B, 1), past_key_values=caches)
    sess.step()
    torch.cuda.synchronize()
    assert _C.device_error() == 0
    err = max_rel_err(to_f32_np(sess.logits), to_f32_np(ref_logits.reshape(B, -1)))
    assert err <= 2e-2, f"decode step vs module path: {err:.3e}"
    # the new K/V rows landed at position ctx of every layer's cache
    for c, k in zip(sess.caches, caches):
        assert max_rel_err(to_f32_np(c.k[:, :, ctx]), to_f32_np(k.k[:, :, ctx])) <= 1e-2
    assert torch.equal(sess.positions, torch.full_like(sess.positions, ctx + 1))
    # final norm + LM head against the oracle on the step's last hidden state
    x_final = sess.x[len(model.layers) & 1]
    h = oracle.round_to_bf16(oracle.rmsnorm(to_f32_np(x_final), model.norm.cpu().numpy(), 1e-6))
    logits_ref = h.astype(np.float64) @ to_f32_np(model.lm_head).astype(np.float64).T
    assert max_rel_err(to_f32_np(sess.logits), logits_ref) <= MAX_REL
    assert torch.equal(sess.tokens.long(), torch.argmax(sess.logits, dim=-1))


def test_decode_graph_replay_matches_eager_steps(cuda_dev):
    from nki_moe_7013_b200 import _C
    from nki_moe_7013_b200.model import DecodeSession

    model = _small_model(cuda_dev, seed=4)
    eager = DecodeSession(model, 2, context=40, max_new=8, seed=6)
    graphed = DecodeSession(model, 2, context=40, max_new=8, seed=6)
    assert torch.equal(eager.tokens, graphed.tokens)
    for _ in range(3):
        eager.step()
    graphed.capture()          # one eager step, then the captured one
    graphed.step()
    graphed.step()
    torch.cuda.synchronize()
    assert _C.device_error() == 0
    assert graphed.steps_done == eager.steps_done == 3
    assert torch.equal(eager.positions, graphed.positions)
    assert max_rel_err(to_f32_np(graphed.logits), to_f32_np(eager.logits)) <= 1e-2
    graphed.release()


@pytest.mark.parametrize("B,V", [(1, 151936), (4, 4096), (3, 1001)])
def test_greedy_pick_matches_argmax(cuda_dev, B, V):
    """ops.greedy_pick equals torch.argmax (first maximal index, NaN largest)
    and advances positions and lengths by one; rows with ties and NaNs."""
    from nki_moe_7013_b200 import ops

    g = torch.Generator(device=cuda_dev)
    g.manual_seed(B * 7 + V)
    logits = torch.randn(B, V, generator=g, device=cuda_dev).to(torch.bfloat16)
    logits[0, V // 3] = 50.0
    logits[0, V // 2] = 50.0  # a tie: the lower index wins
    if B > 1:
        logits[1, V - 1] = float("nan")
        logits[1, 5] = float("inf")
    pos = torch.arange(B, dtype=torch.int32, device=cuda_dev)
    lens = pos + 10
    tok = ops.greedy_pick(logits, None, pos, lens)
    torch.cuda.synchronize()
    assert torch.equal(tok.long(), torch.argmax(logits, dim=-1))
    assert torch.equal(pos, torch.arange(B, dtype=torch.int32, device=cuda_dev) + 1)
    assert torch.equal(lens, pos + 10)
