"""Qwen3-MoE decoder stack and its decode step (config 2).

``Qwen3MoeModel`` is the reference model's forward (qwen.py:439-477):
token embedding -> ``num_hidden_layers`` decoder layers -> final RMSNorm ->
LM head, with the embedding lookup and the LM head on this library's kernels
(they replace the reference's NKI embedding and LM-head kernels,
qwen_with_nki.py:1541-1578 and 1766-1805).  ``forward`` is the eager module
path (host-side cache lengths, any number of new tokens); a prefill can ask
for the last position's logits only (``last_only``), as a serving prefill
does.  ``Qwen3MoeModel.expert_parallel`` builds the same random-init model
with every layer's MoE block expert-parallel over a process group (config 3:
attention data-parallel, each rank holding its own sequences and E/P
experts of every layer; the reference's EP option is qwen_with_nki.py:
9870-9876 with the EP-aware MoE at 8148-8271).

``DecodeSession`` runs B sequences one token per step with static shapes:
positions, cache lengths and the next tokens live on the device and advance
on the device, so a whole step -- 48 layers of RMSNorm, QKV projection, QK
norm + RoPE + cache append, split-KV decode attention, O projection, add &
norm and the MoE block (one library call), then the final norm, the LM head and a greedy pick --
captures into one CUDA graph and replays without the host.
"""
from __future__ import annotations

from typing import List, Optional

import torch

from . import ops
from .attention import KVCache
from .config import Qwen3MoeConfig
from .decoder import Qwen3MoeDecoderLayer
from .moe import MoEPlan, MoEWeights, WorkspacePool


class Qwen3MoeModel:
    def __init__(self, cfg: Qwen3MoeConfig, num_layers: Optional[int] = None, vocab_size: Optional[int] = None,
                 device="cuda", seed: int = 0, std: float = 0.02):
        from .synth import normal_bf16_device

        self.cfg = cfg
        self.device = torch.device(device)
        L = cfg.num_hidden_layers if num_layers is None else num_layers
        V = cfg.vocab_size if vocab_size is None else vocab_size
        H = cfg.hidden_size
        self.vocab_size = V
        self.embed = normal_bf16_device(seed * 1000 + 1, (V, H), std, self.device)
        self.layers: List[Qwen3MoeDecoderLayer] = [
            Qwen3MoeDecoderLayer(cfg, layer_idx=l, device=self.device, seed=seed * 1000 + 10 + l) for l in range(L)]
        g = torch.Generator(device=self.device)
        g.manual_seed(seed * 1000 + 3)
        self.norm = (1.0 + 0.1 * torch.randn(H, generator=g, device=self.device)).float().contiguous()
        self.lm_head = normal_bf16_device(seed * 1000 + 2, (V, H), std, self.device)
        self.exchange = None
        self._share_workspace()

    def _share_workspace(self) -> None:
        # the layers run one after another on one stream: one MoE workspace
        pool = WorkspacePool()
        for layer in self.layers:
            if hasattr(layer.mlp, "workspace_pool"):
                layer.mlp.workspace_pool = pool

    @classmethod
    def expert_parallel(cls, cfg: Qwen3MoeConfig, max_tokens: int, group=None, num_layers: Optional[int] = None,
                        vocab_size: Optional[int] = None, device="cuda", seed: int = 0,
                        std: float = 0.02) -> "Qwen3MoeModel":
        """The model ``Qwen3MoeModel(cfg, num_layers, vocab_size, device,
        seed, std)`` would build (identical weights), with each layer's MoE
        block expert-parallel over ``group``: this rank keeps every layer's
        router and its E/P experts [r*E/P, (r+1)*E/P); attention, norms,
        embedding and LM head are replicated.  All blocks share one
        ``PeerEPExchange`` sized for ``max_tokens`` local tokens per call.
        Collective over ``group``; every rank must then run the same layers
        in the same order.  ``close()`` unmaps the peers' buffers."""
        import torch.distributed as dist

        from .ep import PeerEPExchange, PeerExpertParallelMoE
        from .synth import normal_bf16_device

        m = cls.__new__(cls)
        m.cfg = cfg
        m.device = torch.device(device)
        L = cfg.num_hidden_layers if num_layers is None else num_layers
        V = cfg.vocab_size if vocab_size is None else vocab_size
        H, E = cfg.hidden_size, cfg.num_experts
        m.vocab_size = V
        m.embed = normal_bf16_device(seed * 1000 + 1, (V, H), std, m.device)
        world, rank = dist.get_world_size(group), dist.get_rank(group)
        el = E // world
        with torch.cuda.device(m.device):
            m.exchange = PeerEPExchange(cfg, max_tokens, group=group, device=m.device)
        m.layers = []
        for l in range(L):
            s = seed * 1000 + 10 + l
            full = MoEWeights.random(cfg, s, m.device)
            local = MoEWeights(full.router, full.gate_up[rank * el:(rank + 1) * el].clone(),
                               full.down[rank * el:(rank + 1) * el].clone())
            del full
            blk = PeerExpertParallelMoE(cfg, local.router, local, exchange=m.exchange)
            m.layers.append(Qwen3MoeDecoderLayer(cfg, layer_idx=l, device=m.device, seed=s, mlp=blk))
        g = torch.Generator(device=m.device)
        g.manual_seed(seed * 1000 + 3)
        m.norm = (1.0 + 0.1 * torch.randn(H, generator=g, device=m.device)).float().contiguous()
        m.lm_head = normal_bf16_device(seed * 1000 + 2, (V, H), std, m.device)
        return m

    def close(self) -> None:
        """Unmap the expert-parallel exchange's peer buffers (EP models)."""
        if self.exchange is not None:
            self.exchange.close()
            self.exchange = None

    @classmethod
    def from_parts(cls, cfg: Qwen3MoeConfig, embed: torch.Tensor, layers: List[Qwen3MoeDecoderLayer],
                   norm: torch.Tensor, lm_head: torch.Tensor) -> "Qwen3MoeModel":
        """A model from given weights (e.g. a checkpoint: checkpoint.load_model):
        embed (V, H) bf16, the decoder layers, final norm (H,) fp32, LM head
        (V, H) bf16 -- no random initialisation."""
        m = cls.__new__(cls)
        m.cfg = cfg
        m.device = embed.device
        m.vocab_size = embed.shape[0]
        m.embed = embed
        m.layers = list(layers)
        m.norm = norm
        m.lm_head = lm_head
        m.exchange = None
        m._share_workspace()
        return m

    def new_caches(self, n_slots: int, max_seq: int) -> List[KVCache]:
        return [layer.self_attn.new_cache(n_slots, max_seq) for layer in self.layers]

    def hidden_states(self, input_ids: torch.Tensor, past_key_values: Optional[List[KVCache]] = None,
                      num_layers: Optional[int] = None, timer=None, moe_inputs: Optional[list] = None):
        """input_ids (B, S) -> (hidden states (B, S, H) bf16 after the first
        ``num_layers`` layers (all by default), caches).  ``timer``: an
        ``attention.StageTimer`` given to every layer.  ``moe_inputs``: a
        list that receives each layer's MoE-block input (T, H) (layer-by-layer
        parity checks: the routing each layer saw)."""
        B, S = input_ids.shape
        H = self.cfg.hidden_size
        caches = past_key_values if past_key_values is not None else self.new_caches(B, S)
        x = ops.embedding(input_ids.reshape(-1).to(torch.int32).contiguous(), self.embed).reshape(B, S, H)
        n = len(self.layers) if num_layers is None else num_layers
        for layer, cache in zip(self.layers[:n], caches):
            x = layer(x, past_key_value=cache, timer=timer, capture_intermediates=moe_inputs is not None)[0]
            if moe_inputs is not None:
                moe_inputs.append(layer.last["moe_in"])
        return x, caches

    def routing_of(self, moe_inputs: list, with_logits: bool = False) -> list:
        """Top-k expert ids (T, k) int32, each row sorted, of each captured
        layer's MoE input (``hidden_states(..., moe_inputs=...)``); with
        ``with_logits`` a list of (ids, fp32 router logits (T, E))."""
        k = self.cfg.num_experts_per_tok
        out = []
        for layer, h in zip(self.layers, moe_inputs):
            idx, _, logits = ops.router_topk(h.contiguous(), layer.mlp.router_weight, k, return_logits=True)
            ids = torch.sort(idx, dim=1).values
            out.append((ids, logits) if with_logits else ids)
        return out


    def forward(self, input_ids: torch.Tensor, past_key_values: Optional[List[KVCache]] = None,
                last_only: bool = False):
        """input_ids (B, S) -> (logits (B, S, V) bf16, caches); the eager path
        through the decoder-layer modules.  ``last_only``: logits of each
        sequence's last position only, (B, 1, V)."""
        B, S = input_ids.shape
        H = self.cfg.hidden_size
        x, caches = self.hidden_states(input_ids, past_key_values)
        if last_only:
            x = x[:, -1:].contiguous()
            S = 1
        h = ops.rmsnorm(x.reshape(B * S, H), self.norm, self.cfg.rms_norm_eps)
        logits = ops.linear(h, self.lm_head)
        return logits.reshape(B, S, self.vocab_size), caches


def routing_agreement(ids_a: torch.Tensor, ids_b: torch.Tensor, logits_b: torch.Tensor, k: int) -> dict:
    """Compare two routings of the same tokens (sorted (T, k) expert ids) made
    from inputs that differ by rounding: ``agree`` (T,) bool marks tokens
    routed alike; for the others ``max_flip_gap`` is the largest gap, in
    routing ``b``'s fp32 logits, between its k-th and (k+1)-th expert -- small
    when every difference is a near tie at the selection boundary."""
    agree = (ids_a == ids_b).all(dim=1)
    top = torch.topk(logits_b.float(), k + 1, dim=1).values
    gap = top[:, k - 1] - top[:, k]
    flips = ~agree
    max_gap = float(gap[flips].max()) if bool(flips.any()) else 0.0
    return {"agree": agree, "frac": float(agree.float().mean()), "max_flip_gap": max_gap,
            "median_gap": float(gap.median())}


class DecodeSession:
    """B sequences, one new token each per ``step()``, static shapes.

    The caches hold ``context`` tokens per sequence on entry (config 2 fills
    them with ~N(0,1) values) and room for ``max_new`` more.  ``tokens`` (B,)
    int32 on the device is the input of the next step and is overwritten with
    its greedy output; ``logits`` (B, V) bf16 holds the last step's logits."""

    def __init__(self, model: Qwen3MoeModel, batch: int, context: int, max_new: int, seed: int = 0,
                 fill_random: bool = True, split_k: bool = True):
        cfg = model.cfg
        dev = model.device
        self.model = model
        self.B = batch
        self.max_seq = context + max_new
        self.caches = model.new_caches(batch, self.max_seq)
        if fill_random:
            for l, c in enumerate(self.caches):
                c.fill_random(context, seed=seed * 100 + l)
        i32 = dict(dtype=torch.int32, device=dev)
        self.positions = torch.full((batch,), context, **i32)   # position of the next token
        self.kv_len = self.positions + 1                        # cache length once it is appended
        self.slots = torch.arange(batch, **i32)
        g = torch.Generator(device=dev)
        g.manual_seed(seed * 100 + 99)
        self.tokens = torch.randint(0, model.vocab_size, (batch,), generator=g, device=dev, dtype=torch.int32)
        self.plans = [MoEPlan(layer.mlp.weights, batch, cfg.num_experts_per_tok) for layer in model.layers]
        lib_splits = ops._C.lib().qmoe_attention_decode_splits(batch, cfg.num_key_value_heads, self.max_seq)
        ws = ops._C.lib().qmoe_attention_decode_workspace_size(batch, cfg.num_attention_heads, int(lib_splits))
        self.attn_ws = torch.empty(max(int(ws), 1), dtype=torch.uint8, device=dev)
        # split-K scratch of the decode projections (one launch at a time uses it)
        self.split_ws = ops.gateup_split_workspace(dev) if (split_k and batch <= 16) else None
        H = cfg.hidden_size
        self.x = [torch.empty((batch, H), dtype=torch.bfloat16, device=dev) for _ in range(2)]
        self.logits = torch.empty((batch, model.vocab_size), dtype=torch.bfloat16, device=dev)
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.steps_done = 0

    def _layer(self, l: int, x: torch.Tensor, out: torch.Tensor) -> None:
        cfg = self.model.cfg
        layer = self.model.layers[l]
        attn = layer.self_attn
        cache = self.caches[l]
        eps = cfg.rms_norm_eps
        h = ops.rmsnorm(x, layer.input_layernorm, eps)
        qkv = ops.linear(h, attn.w.wqkv, split_ws=self.split_ws)
        q = ops.qk_norm_rope(qkv, self.positions, attn.w.q_norm, attn.w.k_norm, attn.inv_freq,
                             cfg.num_attention_heads, cfg.num_key_value_heads, eps, cache.k, cache.v,
                             cache_slot=self.slots)
        a = ops.attention_decode(q, cache.k, cache.v, self.kv_len, self.max_seq, workspace=self.attn_ws)
        o = ops.linear(a, attn.w.wo, split_ws=self.split_ws)
        # add & norm + MoE + residual add, one library call
        self.plans[l].run_block(o, x, layer.post_attention_layernorm, eps, out)

    def step(self) -> torch.Tensor:
        """One decode step on the current stream (or the captured graph)."""
        if self.graph is not None:
            self.graph.replay()
        else:
            self._step_kernels()
        self.steps_done += 1
        return self.tokens

    def _step_kernels(self) -> None:
        m = self.model
        x = ops.embedding(self.tokens, m.embed, out=self.x[0])
        for l in range(len(m.layers)):
            out = self.x[(l + 1) & 1]
            self._layer(l, x, out)
            x = out
        hf = ops.rmsnorm(x, m.norm, m.cfg.rms_norm_eps)
        ops.linear(hf, m.lm_head, out=self.logits, split_ws=self.split_ws)
        # greedy pick + the next step's position and cache length, one launch
        ops.greedy_pick(self.logits, self.tokens, self.positions, self.kv_len)

    def capture(self) -> None:
        """Capture one step into a CUDA graph (run one eager step first so
        every kernel's attributes are set outside the capture)."""
        dev = self.model.device
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            self._step_kernels()
            self.steps_done += 1
        torch.cuda.current_stream(dev).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._step_kernels()
        self.graph = g

    def release(self) -> None:
        self.graph = None
