"""Host-side API surface (no GPU): the module classes expose the reference's
entry points, and the routing comparison used by the expert-parallel parity
checks flags only what it should."""
import torch

from nki_moe_7013_b200 import decoder, ep, model, moe


def test_model_and_block_entry_points():
    for cls, names in [(model.Qwen3MoeModel, ["forward", "hidden_states", "routing_of", "new_caches",
                                              "expert_parallel", "from_parts", "close"]),
                       (model.DecodeSession, ["step", "capture", "release"]),
                       (decoder.Qwen3MoeDecoderLayer, ["forward"]),
                       (moe.Qwen3MoeSparseMoeBlock, ["forward"]),
                       (moe.ExpertMLPs, ["forward_selective_loading", "torch_blockwise_matmul_inference"]),
                       (ep.PeerExpertParallelMoE, ["forward", "capture", "replay", "static_input", "close"]),
                       (ep.ExpertParallelMoE, ["forward"])]:
        for n in names:
            assert callable(getattr(cls, n, None)), f"{cls.__name__}.{n}"
    assert ep.PeerExpertParallelMoE.expert_parallel is True


def test_routing_agreement_marks_near_ties():
    k = 2
    logits = torch.tensor([[3.0, 2.0, 1.0, 0.0],      # clear winners 0, 1
                           [3.0, 1.004, 1.0, 0.0],    # near tie between 1 and 2
                           [3.0, 2.0, 1.0, 0.0]])
    ids_b = torch.sort(torch.topk(logits, k, dim=1).indices.int(), dim=1).values
    ids_a = ids_b.clone()
    ids_a[1] = torch.tensor([0, 2], dtype=torch.int32)   # the near-tie token picked the other one
    r = model.routing_agreement(ids_a, ids_b, logits, k)
    assert r["agree"].tolist() == [True, False, True]
    assert abs(r["max_flip_gap"] - 0.004) < 1e-5
    ids_a[2] = torch.tensor([0, 2], dtype=torch.int32)   # a difference at a clear gap
    r = model.routing_agreement(ids_a, ids_b, logits, k)
    assert abs(r["max_flip_gap"] - 1.0) < 1e-6


def test_ops_refuse_cpu_tensors():
    """The torch wrappers check their tensors before any library call: a CPU
    tensor is refused (there is no CPU path to fall back to)."""
    import pytest

    from nki_moe_7013_b200 import ops

    y = torch.zeros(4, 256, dtype=torch.bfloat16)
    ids = torch.zeros(4, 8, dtype=torch.int32)
    calls = [
        lambda: ops.masked_residual_add(y, torch.ones(4)),
        lambda: ops.greedy_pick(y),
        lambda: ops.select_affinities(torch.zeros(4, 128), ids),
        lambda: ops.rmsnorm(y, torch.ones(256), 1e-6),
        lambda: ops.moe_forward(y, torch.zeros(128, 256, dtype=torch.bfloat16),
                                torch.zeros(128, 256, 256, dtype=torch.bfloat16),
                                torch.zeros(128, 256, 128, dtype=torch.bfloat16), 8),
    ]
    for call in calls:
        with pytest.raises(ValueError, match="no CPU path"):
            call()
