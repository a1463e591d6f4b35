"""Sparse-MoE block with the reference's module interfaces.

* ``Qwen3MoeSparseMoeBlock`` -- drop-in for the MoE module the decoder layer
  calls as ``self.mlp(hidden_states, padding_mask)[0]`` (qwen.py:429,
  ``initialize_moe_module`` at qwen.py:365-371).  Returns a tuple whose [0] is
  the (T, H) or (B, S, H) bf16 output.
* ``Qwen3MoeSparseMoeBlockHF`` -- same block with the HF signature
  ``forward(hidden_states) -> Tensor`` (transformers Qwen3MoeSparseMoeBlock).
* ``ExpertMLPs`` -- the two ExpertMLPsV2 operator seams the reference team
  patched: ``forward_selective_loading`` (qwen_with_nki.py:2377-2453) and
  ``torch_blockwise_matmul_inference`` (qwen_with_nki.py:5872-5881).
* ``MoEPlan`` -- buffers preallocated for a fixed token count; runs the five
  kernels through the C ABI with no per-call allocation (CUDA-graph friendly,
  and able to time every kernel with CUDA events).

All compute goes through the CUDA library; there is no CPU path.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
from torch import nn

from . import _C, ops
from .config import Qwen3MoeConfig


@dataclass
class MoEWeights:
    """Device layout: router (E,H), gate_up (E,2I,H) gate rows first, down (E,H,I)."""

    router: torch.Tensor
    gate_up: torch.Tensor
    down: torch.Tensor

    @property
    def num_experts(self) -> int:
        """Experts held here (all of them, or this rank's shard under EP)."""
        return self.gate_up.shape[0]

    @property
    def hidden_size(self) -> int:
        return self.router.shape[1]

    @property
    def intermediate_size(self) -> int:
        return self.down.shape[2]

    @staticmethod
    def random(cfg: Qwen3MoeConfig, seed: int = 0, device="cuda", std: float = 0.02) -> "MoEWeights":
        from .synth import normal_bf16_device

        E, H, I = cfg.num_experts, cfg.hidden_size, cfg.moe_intermediate_size
        return MoEWeights(normal_bf16_device(seed * 10 + 1, (E, H), std, device),
                          normal_bf16_device(seed * 10 + 2, (E, 2 * I, H), std, device),
                          normal_bf16_device(seed * 10 + 3, (E, H, I), std, device))

    @staticmethod
    def from_neuron_layout(router: torch.Tensor, gate_up_ehi: torch.Tensor, down_eih: torch.Tensor,
                           device="cuda") -> "MoEWeights":
        """From the NxDI layout of convert_qwen3_moe_hf_to_neuron_state_dict
        (qwen.py:164-226): gate_up (E, H, 2I) gate first, down (E, I, H)."""
        return MoEWeights(router.to(device=device, dtype=torch.bfloat16).contiguous(),
                          gate_up_ehi.to(device=device, dtype=torch.bfloat16).transpose(1, 2).contiguous(),
                          down_eih.to(device=device, dtype=torch.bfloat16).transpose(1, 2).contiguous())

    @staticmethod
    def from_hf_block(block, device="cuda") -> "MoEWeights":
        """From a transformers Qwen3MoeSparseMoeBlock (gate.weight (E,H),
        experts.gate_up_proj (E,2I,H), experts.down_proj (E,H,I))."""
        bf = dict(device=device, dtype=torch.bfloat16)
        return MoEWeights(block.gate.weight.detach().to(**bf).contiguous(),
                          block.experts.gate_up_proj.detach().to(**bf).contiguous(),
                          block.experts.down_proj.detach().to(**bf).contiguous())


class WorkspacePool:
    """One growing device byte buffer shared by MoE blocks that run one after
    another on one stream (the layers of a decoder stack): a 16,384-token
    prefill needs ~0.9 GB of workspace per call, which 48 blocks need not
    hold each.  Blocks that may run concurrently on different streams must
    not share a pool."""

    def __init__(self):
        self.buf: Optional[torch.Tensor] = None

    def get(self, nbytes: int, device) -> torch.Tensor:
        if self.buf is None or self.buf.numel() < nbytes or self.buf.device != torch.device(device):
            self.buf = None
            self.buf = torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)
        return self.buf


class Qwen3MoeSparseMoeBlock(nn.Module):
    """Routed-expert MoE of Qwen3 (no shared experts, qwen.py:253-255).

    ``workspace_pool`` (a ``WorkspacePool``, optional) supplies the forward's
    device workspace; without one the block keeps its own."""

    def __init__(self, cfg: Qwen3MoeConfig, weights: Optional[MoEWeights] = None, device="cuda",
                 seed: int = 0, return_router_logits: bool = False, return_expert_index: bool = False):
        super().__init__()
        self.cfg = cfg
        self.top_k = cfg.num_experts_per_tok
        self.normalize = cfg.norm_topk_prob
        self.return_router_logits = return_router_logits
        self.return_expert_index = return_expert_index
        w = weights if weights is not None else MoEWeights.random(cfg, seed, device)
        self.router_weight = nn.Parameter(w.router, requires_grad=False)
        self.gate_up = nn.Parameter(w.gate_up, requires_grad=False)
        self.down = nn.Parameter(w.down, requires_grad=False)
        self.router_bias: Optional[torch.Tensor] = None
        self._workspace: Optional[torch.Tensor] = None
        self.workspace_pool: Optional[WorkspacePool] = None

    @property
    def weights(self) -> MoEWeights:
        return MoEWeights(self.router_weight.data, self.gate_up.data, self.down.data)

    def _ws(self, nbytes: int, device) -> torch.Tensor:
        if self.workspace_pool is not None:
            return self.workspace_pool.get(nbytes, device)
        if self._workspace is None or self._workspace.numel() < nbytes or self._workspace.device != device:
            self._workspace = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=device)
        return self._workspace

    def _moe(self, x2d: torch.Tensor, residual: Optional[torch.Tensor] = None):
        T, H = x2d.shape
        ws = ops.moe_forward_workspace_size(T, H, self.cfg.num_experts, self.top_k,
                                            self.cfg.moe_intermediate_size)
        return ops.moe_forward(x2d, self.router_weight, self.gate_up, self.down, self.top_k,
                               normalize=self.normalize, residual=residual, bias=self.router_bias,
                               workspace=self._ws(ws, x2d.device), return_routing=True)

    def _block(self, x2d: torch.Tensor, residual: torch.Tensor, norm_weight: torch.Tensor, eps: float,
               moe_in_out: Optional[torch.Tensor] = None, residual_out: Optional[torch.Tensor] = None):
        """add & norm + this block + residual add (ops.moe_block_forward)."""
        T, H = x2d.shape
        ws = ops.moe_block_forward_workspace_size(T, H, self.cfg.num_experts, self.top_k,
                                                  self.cfg.moe_intermediate_size)
        return ops.moe_block_forward(x2d, residual, norm_weight, eps, self.router_weight, self.gate_up, self.down,
                                     self.top_k, normalize=self.normalize, bias=self.router_bias,
                                     workspace=self._ws(ws, x2d.device), moe_in_out=moe_in_out,
                                     residual_out=residual_out)

    def forward(self, hidden_states: torch.Tensor, padding_mask: Optional[torch.Tensor] = None):
        shape = hidden_states.shape
        x2d = hidden_states.reshape(-1, shape[-1]).to(torch.bfloat16).contiguous()
        out, idx, tw = self._moe(x2d)
        if padding_mask is not None:
            # padded positions (mask == 0) produce no MoE output
            out = ops.masked_residual_add(out, padding_mask)
        out = out.reshape(shape)
        result = (out,)
        if self.return_router_logits:
            logits = ops.router_topk(x2d, self.router_weight, self.top_k, bias=self.router_bias,
                                     return_logits=True)[2]
            result = result + (logits,)
        if self.return_expert_index:
            result = result + (idx.long(),)
        return result


class Qwen3MoeSparseMoeBlockHF(Qwen3MoeSparseMoeBlock):
    """HF-compatible variant: forward(hidden_states) -> Tensor."""

    def forward(self, hidden_states: torch.Tensor) -> torch.Tensor:  # type: ignore[override]
        return super().forward(hidden_states)[0]


class ExpertMLPs(nn.Module):
    """The ExpertMLPsV2 seams of the reference (weights in device layout)."""

    def __init__(self, weights: MoEWeights, normalize_top_k_affinities: bool = True):
        super().__init__()
        self.w = weights
        self.normalize_top_k_affinities = normalize_top_k_affinities

    def forward_selective_loading(self, hidden_states: torch.Tensor, expert_affinities: torch.Tensor,
                                  expert_index: torch.Tensor) -> torch.Tensor:
        """qwen_with_nki.py:2377-2453: affinities (T, E) over all experts,
        expert_index (T, k); the chosen affinities are L1-renormalised when
        normalize_top_k_affinities (qwen_with_nki.py:2402-2405)."""
        x = hidden_states.reshape(-1, hidden_states.shape[-1]).to(torch.bfloat16).contiguous()
        T, H = x.shape
        E = self.w.num_experts
        idx = expert_index.reshape(T, -1).to(torch.int32).contiguous()
        k = idx.shape[1]
        chosen = ops.select_affinities(expert_affinities.reshape(T, E), idx, self.normalize_top_k_affinities)
        return _run_routed(x, self.w, idx, chosen, k)

    def torch_blockwise_matmul_inference(self, block_size, num_blocks, hidden_states,
                                         expert_affinities_masked, token_position_to_id,
                                         block_to_expert, pad_inputs_for_matmul=False) -> torch.Tensor:
        """qwen_with_nki.py:5872-5881 / 5440-5502: blocks of ``block_size``
        token positions, one expert per block; positions outside [0, T) are
        padding; a token repeated inside a block contributes once."""
        return blockwise_forward(hidden_states, expert_affinities_masked, token_position_to_id,
                                 block_to_expert, int(block_size), int(num_blocks), self.w)


def _run_routed(x: torch.Tensor, w: MoEWeights, idx: torch.Tensor, tw: torch.Tensor, k: int,
                residual: Optional[torch.Tensor] = None, acc_rows: Optional[int] = None) -> torch.Tensor:
    """Permutation + grouped GEMMs + combine for caller-provided routing
    (idx (T, k) int32 expert ids, tw (T, k) fp32 weights)."""
    T, H = x.shape
    E = w.num_experts
    hist = ops.routing_histogram(idx, E)
    acc = torch.empty((T, H), dtype=torch.float32, device=x.device)
    if T > ops.FUSED_MIN_T:
        copy = T > ops.FUSED_GATHER_MAX_T
        p = ops.moe_permute(idx, tw, hist, E, x=x, gather=copy, acc_zero=acc)
        if copy:
            ops.moe_experts(p["x_perm"], w.gate_up, w.down, p["tiles"], p["max_tiles"], p["row_token"], p["row_w"],
                            acc, p["done"])
        else:
            ops.moe_experts(x, w.gate_up, w.down, p["tiles"], p["max_tiles"], p["row_token"], p["row_w"], acc,
                            p["done"], gather_rows=p["row_token"])
        return ops.combine_finalize(acc, residual)
    else:
        p = ops.moe_permute(idx, tw, hist, E, x=x, gather=False, acc_zero=acc)
        split = ops.gateup_split_workspace(x.device) if T * k <= ops.GATEUP_SPLIT_MAX_R else None
        act = ops.grouped_gemm_gateup_swiglu(x, w.gate_up, p["tiles"], p["max_tiles"], gather_rows=p["row_token"],
                                             split_ws=split)
    ops.grouped_gemm_down_combine(act, w.down, p["tiles"], p["max_tiles"], p["row_token"], p["row_w"], acc,
                                  tiles_ready=True)
    return ops.combine_finalize(acc, residual)


def blockwise_forward(hidden_states, expert_affinities_masked, token_position_to_id, block_to_expert,
                      block_size: int, num_blocks: int, w: MoEWeights) -> torch.Tensor:
    x = hidden_states.reshape(-1, hidden_states.shape[-1]).to(torch.bfloat16).contiguous()
    T, H = x.shape
    tpi = token_position_to_id.reshape(-1).to(torch.int32).contiguous()
    b2e = block_to_expert.reshape(-1).to(torch.int32).contiguous()
    aff = expert_affinities_masked.float().contiguous()
    acc = torch.zeros((T, H), dtype=torch.float32, device=x.device)
    prep = ops.blockwise_prepare(x, aff, tpi, b2e, block_size, num_blocks)
    act = ops.grouped_gemm_gateup_swiglu(prep["x_perm"], w.gate_up, prep["tiles"], prep["max_tiles"])
    ops.grouped_gemm_down_combine(act, w.down, prep["tiles"], prep["max_tiles"], prep["row_dst"],
                                  prep["row_w"], acc)
    return ops.combine_finalize(acc)


class MoEPlan:
    """Preallocated buffers + direct C-ABI launches for a fixed (T, H, E, k, I).

    ``run(x, out, residual=None)`` is one ``qmoe_moe_forward`` call (the
    library's fused forward on a preallocated workspace).  ``run(..., events)``
    runs the same kernels through the per-stage entry points instead and
    records the CUDA events (len(self.stages) + 1) before the first kernel and
    after each stage, on the current stream.  Stages: router, permute (scan +
    scatter), gate_up, down, finalize; batches of more than ops.FUSED_MIN_T
    tokens run gate/up and down as one kernel ("experts").  The fused forward
    folds the finalize into the last kernel."""

    STAGES = ("router", "permute", "gate_up", "down", "finalize")
    STAGES_FUSED = ("router", "permute", "experts", "finalize")
    STAGES_ROUTED = ("route", "experts", "finalize")  # router + permutation in one launch

    def __init__(self, weights: MoEWeights, T: int, k: int, normalize: bool = True,
                 bias: Optional[torch.Tensor] = None, prefill_gather: Optional[bool] = None,
                 fused: Optional[bool] = None):
        self.w = weights
        self.T, self.k = T, k
        self.E, self.H, self.I = weights.router.shape[0], weights.hidden_size, weights.intermediate_size
        self.normalize = normalize
        self.bias = bias
        dev = weights.router.device
        self.device = dev
        R = T * k
        E, H, I = self.E, self.H, self.I
        self.R = R
        self.max_tiles = ops.max_tiles(R, E)
        nchunks = (T + ops.ROUTER_CHUNK - 1) // ops.ROUTER_CHUNK
        i32 = dict(dtype=torch.int32, device=dev)
        f32 = dict(dtype=torch.float32, device=dev)
        self.topk_idx = torch.empty((T, k), **i32)
        self.topk_w = torch.empty((T, k), **f32)
        self.hist = torch.empty((max(nchunks, 1), E), **i32)
        self.counts = torch.empty(E, **i32)
        self.offsets = torch.empty(E + 1, **i32)
        self.row_token = torch.empty(max(R, 1), **i32)
        self.row_w = torch.empty(max(R, 1), **f32)
        self.slot_row = torch.empty((T, k), **i32)
        self.tiles = torch.empty(1 + 3 * self.max_tiles, **i32)
        self.act = torch.empty((max(R, 1), I), dtype=torch.bfloat16, device=dev)
        self.acc = torch.empty((max(T, 1), H), **f32)
        # prefill sizes read a permuted copy of the rows; decode sizes gather
        # prefill sizes: gate/up and down run as one persistent kernel, whose
        # per-tile counters the permutation zero-fills; its gate/up rows come
        # from a permuted copy or (prefill_gather) straight from the tokens
        self.fused = T > ops.FUSED_MIN_T if fused is None else (bool(fused) and T > ops.FUSED_MIN_T)
        if prefill_gather is None:
            prefill_gather = T <= ops.FUSED_GATHER_MAX_T
        self.x_perm = (torch.empty((max(R, 1), H), dtype=torch.bfloat16, device=dev)
                       if T > ops.GATHER_MAX_T and not (self.fused and prefill_gather) else None)
        self.done = torch.zeros(self.max_tiles + 1, **i32) if self.fused else None
        # prefill batches of at most one router chunk per SM route and permute
        # in one launch (the library forward does the same)
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        self.route_permute = (self.fused and self.x_perm is not None and T > ops.ROUTER_SMALL_MAX_T
                              and nchunks <= sms)
        self.route_barrier = torch.zeros(2, **i32) if self.route_permute else None
        self.stages = (self.STAGES_ROUTED if self.route_permute else
                       self.STAGES_FUSED if self.fused else self.STAGES)
        self.ws_bytes = int(_C.lib().qmoe_moe_forward_workspace_size(T, H, E, k, I))
        self.block_ws_bytes = int(_C.lib().qmoe_moe_block_forward_workspace_size(T, H, E, k, I))
        self.workspace = torch.empty(max(self.ws_bytes, self.block_ws_bytes, 256), dtype=torch.uint8, device=dev)
        # small batches route through the logits + selection kernels
        self.logits = torch.empty((T, E), **f32) if T <= ops.ROUTER_SMALL_MAX_T else None
        # a token's k experts are distinct: no tile holds more than T rows
        self.tile_rows = min(T, 128)
        # decode sizes: router + permutation in one launch
        self.route_small = T <= ops.ROUTE_SMALL_MAX_T and E <= ops.ROUTE_SMALL_MAX_E
        # decode sizes: the gate/up GEMM may split K (zero-filled scratch)
        self.split_ws = ops.gateup_split_workspace(dev) if R <= ops.GATEUP_SPLIT_MAX_R else None
        self._split_bytes = 0 if self.split_ws is None else self.split_ws.numel()
        self._lib = _C.lib()

    def run(self, x: torch.Tensor, out: torch.Tensor, residual: Optional[torch.Tensor] = None,
            events=None) -> torch.Tensor:
        lib, p = self._lib, ops._ptr
        s = torch.cuda.current_stream(self.device).cuda_stream
        T, H, E, k, I, R = self.T, self.H, self.E, self.k, self.I, self.R
        w = self.w
        if events is None:
            _C.check(lib.qmoe_moe_forward(p(x), p(w.router), p(self.bias), p(w.gate_up), p(w.down), p(residual),
                                          T, H, E, k, I, 1 if self.normalize else 0, p(out), p(self.topk_idx),
                                          p(self.topk_w), p(self.workspace), self.ws_bytes, s), "moe_forward")
            return out

        n_marked = [0]

        def mark():  # the event after the next stage
            if events is not None:
                events[n_marked[0]].record()
            n_marked[0] += 1

        mark()
        if self.route_small:
            _C.check(lib.qmoe_route_small(p(x), p(w.router), p(self.bias), T, H, E, k, 1 if self.normalize else 0,
                                          p(self.logits), p(self.topk_idx), p(self.topk_w), p(self.counts),
                                          p(self.offsets), p(self.row_token), p(self.row_w), p(self.slot_row),
                                          p(self.tiles), p(self.acc), s), "route_small")
            if self.fused:
                self.done.zero_()  # the library forward has the route kernel zero them
            mark()
            mark()
        elif self.route_permute:
            _C.check(lib.qmoe_route_permute(p(x), p(w.router), p(self.bias), T, H, E, k, 1 if self.normalize else 0,
                                            p(self.topk_idx), p(self.topk_w), p(self.hist), p(self.counts),
                                            p(self.offsets), p(self.row_token), p(self.row_w), p(self.slot_row),
                                            p(self.tiles), p(self.x_perm), p(self.acc), p(self.done),
                                            self.max_tiles + 1, p(self.route_barrier), s), "route")
            mark()
        else:
            _C.check(lib.qmoe_router_topk(p(x), p(w.router), p(self.bias), T, H, E, k,
                                          1 if self.normalize else 0, p(self.logits), p(self.topk_idx),
                                          p(self.topk_w), p(self.hist), s), "router")
            mark()
            _C.check(lib.qmoe_moe_permute(p(self.topk_idx), p(self.topk_w), p(self.hist), p(x), T, H, E, k,
                                          p(self.counts), p(self.offsets), p(self.row_token), p(self.row_w),
                                          p(self.slot_row), p(self.tiles), p(self.x_perm), p(self.acc),
                                          p(self.done), self.max_tiles + 1 if self.fused else 0, s),
                     "permute")
            mark()
        if self.fused:
            if self.x_perm is not None:
                src, src_rows, gather = self.x_perm, R, None
            else:
                src, src_rows, gather = x, T, self.row_token
            _C.check(lib.qmoe_moe_experts(p(src), src_rows, p(gather), p(w.gate_up), p(w.down), p(self.tiles),
                                          self.max_tiles, p(self.row_token), p(self.row_w), R, H, I, E, p(self.act),
                                          p(self.acc), T, p(self.done), s), "experts")
            mark()
            _C.check(lib.qmoe_combine_finalize(p(self.acc), p(residual), T, H, p(out), s), "finalize")
            mark()
            return out
        if self.x_perm is not None:
            _C.check(lib.qmoe_grouped_gemm_gateup_swiglu(p(self.x_perm), R, None, p(w.gate_up), p(self.tiles),
                                                         self.max_tiles, self.tile_rows, R, H, I, E, p(self.act),
                                                         p(self.split_ws), self._split_bytes, s), "gate_up")
        else:
            _C.check(lib.qmoe_grouped_gemm_gateup_swiglu(p(x), T, p(self.row_token), p(w.gate_up),
                                                         p(self.tiles), self.max_tiles, self.tile_rows, R, H, I, E,
                                                         p(self.act), p(self.split_ws), self._split_bytes, s),
                     "gate_up")
        mark()
        # tiles come from the routing kernels, before the gate/up GEMM
        _C.check(lib.qmoe_grouped_gemm_down_combine(p(self.act), p(w.down), p(self.tiles), self.max_tiles,
                                                    self.tile_rows, 1, p(self.row_token), p(self.row_w), R, H, I, E,
                                                    p(self.acc), T, s), "down")
        mark()
        _C.check(lib.qmoe_combine_finalize(p(self.acc), p(residual), T, H, p(out), s), "finalize")
        mark()
        return out

    def run_block(self, x: torch.Tensor, residual: torch.Tensor, norm_weight: torch.Tensor, eps: float,
                  out: torch.Tensor, moe_in_out: Optional[torch.Tensor] = None,
                  residual_out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """The decoder layer's post-attention add & norm, this block and the
        residual add (one ``qmoe_moe_block_forward`` call): out = s + MoE(h)
        with s = bf16(x + residual), h = rmsnorm(s) * norm_weight."""
        lib, p = self._lib, ops._ptr
        s = torch.cuda.current_stream(self.device).cuda_stream
        w = self.w
        _C.check(lib.qmoe_moe_block_forward(p(x), p(residual), p(norm_weight), float(eps), p(w.router), p(self.bias),
                                            p(w.gate_up), p(w.down), self.T, self.H, self.E, self.k, self.I,
                                            1 if self.normalize else 0, p(out), p(moe_in_out), p(residual_out),
                                            p(self.topk_idx), p(self.topk_w), p(self.workspace),
                                            self.workspace.numel(), s), "moe_block_forward")
        return out

    LAUNCHES_PER_RUN = 6  # router, scan, scatter, gate/up, down, finalize (T > 64)

    def experts_hit(self) -> int:
        """Distinct experts the last run routed to."""
        return int(torch.unique(self.topk_idx).numel())

    @property
    def launches_per_run(self) -> int:
        """Kernels one run launches: route_small (1) or router (2 when
        T <= 64: logits + selection) + scan + scatter, then gate/up, down,
        finalize."""
        if self.route_small:
            return 2 if self.fused else 3  # route, experts / gate/up + down (+ finalize folded in)
        if self.route_permute:
            return 2  # route + permutation, experts (+ finalize folded in)
        if self.fused:
            return 4  # router, scan, scatter, experts (+ finalize folded in)
        return (7 if self.T <= ops.ROUTER_SMALL_MAX_T else 6)
