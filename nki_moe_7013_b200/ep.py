"""Expert-parallel sparse-MoE block over NCCL all-to-alls.

Rank r of P owns experts [r*E/P, (r+1)*E/P) (16 experts per GPU at P=8) and
its own tokens (data-parallel).  Per layer:

1. router on the local tokens (K1, all E experts);
2. ``ep_pack``: (token, slot) rows grouped by destination rank;
3. int32 all-to-all of the per-destination counts (one host sync per layer:
   NCCL's variable-size all-to-all needs the split sizes on the host);
4. dispatch all-to-all of the bf16 rows and of (local expert, weight);
5. local permutation + grouped GEMMs on the received rows, the routing weight
   applied in the down-projection epilogue;
6. combine all-to-all of the weighted rows back to their source rank;
7. ``ep_unpack``: per token, fp32 sum of its k returned rows (+ residual).

The reference's EP variant (qwen_with_nki.py:8148-8271) instead masks the
non-local experts on every rank and all-reduces the partial outputs
(qwen_with_nki.py:8173-8177).

The per-rank compute is injected through ``EPKernels`` so the exchange logic
can run under the gloo backend on the CPU in tests; the product path uses the
CUDA kernels (``CudaEPKernels``) and NCCL.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist
from torch import nn

from . import ops
from .config import Qwen3MoeConfig
from .moe import MoEWeights, _run_routed


class CudaEPKernels:
    """Per-rank compute of the EP block on the CUDA library."""

    def router(self, x, w_router, k, normalize, bias):
        return ops.router_topk(x, w_router, k, normalize=normalize, bias=bias)

    def pack(self, idx, tw, x, e_local, n_ranks):
        return ops.ep_pack(idx, tw, x, e_local, n_ranks)

    def local_moe(self, recv_x, recv_expert, recv_w, local: MoEWeights):
        if recv_x.shape[0] == 0:
            return torch.empty((0, recv_x.shape[1]), dtype=torch.bfloat16, device=recv_x.device)
        return _run_routed(recv_x, local, recv_expert.reshape(-1, 1), recv_w.reshape(-1, 1), 1)

    def unpack(self, y_back, pair_pos, residual):
        return ops.ep_unpack(y_back, pair_pos, residual)


class ExpertParallelMoE(nn.Module):
    """Sparse-MoE block with the experts sharded over the ranks of `group`.

    ``local`` holds this rank's experts (gate_up (E/P, 2I, H), down (E/P, H, I));
    ``router_weight`` is the full (E, H) router, identical on every rank."""

    def __init__(self, cfg: Qwen3MoeConfig, router_weight: torch.Tensor, local: MoEWeights,
                 group=None, kernels=None):
        super().__init__()
        self.cfg = cfg
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if cfg.num_experts % self.world:
            raise ValueError("num_experts must divide evenly over the ranks")
        self.e_local = cfg.num_experts // self.world
        if local.gate_up.shape[0] != self.e_local:
            raise ValueError("local expert weights do not match E / world")
        self.router_weight = router_weight
        self.local = local
        self.k = cfg.num_experts_per_tok
        self.normalize = cfg.norm_topk_prob
        self.router_bias: Optional[torch.Tensor] = None
        self.kernels = kernels if kernels is not None else CudaEPKernels()
        self.last_recv_rows = 0

    def forward(self, hidden_states: torch.Tensor, residual: Optional[torch.Tensor] = None,
                events=None) -> torch.Tensor:
        """``events``: optional dict name -> (start, end) CUDA events recorded
        around the stages "route", "dispatch", "experts", "combine"."""
        shape = hidden_states.shape
        H = shape[-1]
        x = hidden_states.reshape(-1, H).to(torch.bfloat16).contiguous()
        kn, g = self.kernels, self.group

        def mark(name, i):
            if events is not None:
                events[name][i].record()

        mark("route", 0)
        idx, tw = kn.router(x, self.router_weight, self.k, self.normalize, self.router_bias)
        pk = kn.pack(idx, tw, x, self.e_local, self.world)
        mark("route", 1)
        mark("dispatch", 0)
        send_counts = pk["send_counts"]
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=g)
        sc = [int(v) for v in send_counts.tolist()]
        rc = [int(v) for v in recv_counts.tolist()]
        n_send, n_recv = sum(sc), sum(rc)
        recv_x = torch.empty((n_recv, H), dtype=torch.bfloat16, device=x.device)
        dist.all_to_all_single(recv_x, pk["send_x"][:n_send], rc, sc, group=g)
        send_meta = torch.stack([pk["send_expert"][:n_send], pk["send_w"][:n_send].view(torch.int32)], 1)
        recv_meta = torch.empty((n_recv, 2), dtype=torch.int32, device=x.device)
        dist.all_to_all_single(recv_meta, send_meta, rc, sc, group=g)
        mark("dispatch", 1)
        mark("experts", 0)
        recv_e = recv_meta[:, 0].contiguous()
        recv_w = recv_meta[:, 1].contiguous().view(torch.float32)
        y = kn.local_moe(recv_x, recv_e, recv_w, self.local)
        self.last_recv_rows = n_recv
        mark("experts", 1)
        mark("combine", 0)
        y_back = torch.empty((n_send, H), dtype=torch.bfloat16, device=x.device)
        dist.all_to_all_single(y_back, y, sc, rc, group=g)
        res = None if residual is None else residual.reshape(-1, H).to(torch.bfloat16).contiguous()
        out = kn.unpack(y_back, pk["pair_pos"], res)
        mark("combine", 1)
        return out.reshape(shape)
