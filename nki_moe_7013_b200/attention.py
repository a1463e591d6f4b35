"""Attention sub-layer of the Qwen3-MoE decoder layer (secondary target).

``Qwen3MoeAttention.forward(hidden_states, position_ids=None,
past_key_value=None, attention_mask=None) -> (out, present_kv)`` mirrors
NxDI's NeuronQwen3MoEAttention (qwen.py:313-341): fused QKV projection,
per-head q/k RMSNorm (qwen.py:333-335), RoPE theta 1e6 (qwen.py:315-319),
causal GQA over a KV cache, o_proj.  Positions follow the HF convention (the
position of a new token = the number of tokens already cached).

``attention_mask``: causal masking is built in; a 2D key-padding mask
(batch, cached + new tokens; 1 = token, 0 = padding) with LEFT padding only
(each row zeros then ones) is honoured -- the form NxDI / HF batch prefill
uses.  The cache remembers each slot's padding, so later decode steps keep
masking it.  RoPE is applied at the cache row; HF applies it at the
pad-shifted position (cumsum(mask) - 1), and since the rotary score depends
only on the difference of two positions the attention output is the same up
to fp32 rounding.  Padding query rows get a zero attention output.  Any
other mask (holes, right padding, 4D) is refused with a ValueError.

All kernels come from the CUDA library: tcgen05 projections (``ops.linear``),
the fused QK-norm + RoPE + cache append, flash-prefill / split-KV
flash-decode.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import torch
from torch import nn

from . import ops
from .config import Qwen3MoeConfig


def rope_inv_freq(head_dim: int, theta: float, device) -> torch.Tensor:
    """fp32 inverse frequencies, computed the way HF / NxDI RotaryEmbedding do."""
    return (1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))).to(device)


class KVCache:
    """K and V caches (slots, nkv, max_seq, head_dim) bf16 plus per-slot lengths.

    ``lengths`` is kept on the host (it drives shapes and launch sizes) and
    mirrored on the device for the kernels."""

    def __init__(self, n_slots: int, nkv: int, max_seq: int, head_dim: int, device="cuda"):
        self.k = torch.zeros((n_slots, nkv, max_seq, head_dim), dtype=torch.bfloat16, device=device)
        self.v = torch.zeros_like(self.k)
        self.lengths: List[int] = [0] * n_slots
        self.pad: List[int] = [0] * n_slots      # leading padding rows per slot
        self.max_seq = max_seq

    @property
    def n_slots(self) -> int:
        return self.k.shape[0]

    def fill_random(self, length: int, seed: int = 0) -> "KVCache":
        """Config-2 setup: every slot holds `length` tokens of ~N(0,1) bf16."""
        g = torch.Generator(device=self.k.device)
        g.manual_seed(seed)
        self.k[:, :, :length].normal_(generator=g)
        self.v[:, :, :length].normal_(generator=g)
        self.lengths = [length] * self.n_slots
        self.pad = [0] * self.n_slots
        return self

    def reset(self) -> "KVCache":
        """Empty every slot (the contents are overwritten by the next appends)."""
        self.lengths = [0] * self.n_slots
        self.pad = [0] * self.n_slots
        return self


def left_padding(attention_mask: Optional[torch.Tensor], B: int, S: int, L0: List[int]) -> Optional[List[int]]:
    """Leading padding count per sequence of a 2D key-padding mask (B, L0+S),
    1 = token, 0 = padding; None for no mask.  Refuses every other mask."""
    if attention_mask is None:
        return None
    if attention_mask.dim() != 2:
        raise ValueError("attention_mask: only a 2D (batch, cached + new tokens) key-padding mask is "
                         "supported; causal masking is built in")
    m = (attention_mask != 0).to(torch.int32).cpu()
    if m.shape[0] != B:
        raise ValueError(f"attention_mask has {m.shape[0]} rows for a batch of {B}")
    L = m.shape[1]
    if any(l0 + S != L for l0 in L0):
        raise ValueError(f"attention_mask must cover each sequence's cached and new tokens ({L0[0] + S}), "
                         f"got {L}")
    if L > 1 and not bool(torch.all(m[:, 1:] >= m[:, :-1])):
        raise ValueError("attention_mask: only left padding (zeros before ones in every row) is supported")
    return [int(v) for v in (L - m.sum(1)).tolist()]


@dataclass
class AttnWeights:
    wqkv: torch.Tensor     # (nh*hd + 2*nkv*hd, H) bf16: q rows, k rows, v rows
    wo: torch.Tensor       # (H, nh*hd) bf16
    q_norm: torch.Tensor   # (hd,) fp32
    k_norm: torch.Tensor   # (hd,) fp32

    @staticmethod
    def random(cfg: Qwen3MoeConfig, seed: int = 0, device="cuda", std: float = 0.02) -> "AttnWeights":
        from .synth import normal_bf16_device

        H, nh, nkv, hd = cfg.hidden_size, cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        g = torch.Generator(device=device)
        g.manual_seed(seed * 10 + 7)
        return AttnWeights(
            normal_bf16_device(seed * 10 + 5, ((nh + 2 * nkv) * hd, H), std, device),
            normal_bf16_device(seed * 10 + 6, (H, nh * hd), std, device),
            (1.0 + 0.1 * torch.randn(hd, generator=g, device=device)).float(),
            (1.0 + 0.1 * torch.randn(hd, generator=g, device=device)).float())

    @staticmethod
    def from_hf(attn, device="cuda") -> "AttnWeights":
        """From a transformers Qwen3MoeAttention (q/k/v/o_proj, q_norm, k_norm)."""
        bf = dict(device=device, dtype=torch.bfloat16)
        wqkv = torch.cat([attn.q_proj.weight, attn.k_proj.weight, attn.v_proj.weight], 0)
        return AttnWeights(wqkv.detach().to(**bf).contiguous(), attn.o_proj.weight.detach().to(**bf).contiguous(),
                           attn.q_norm.weight.detach().float().to(device).contiguous(),
                           attn.k_norm.weight.detach().float().to(device).contiguous())


class StageTimer:
    """Optional per-stage CUDA events: ``with timer("name"):`` records an
    event pair around the kernels issued inside on the current stream and
    appends (name, start, end) to ``timer.marks``.  A ``None`` timer costs
    nothing (``stage(None, name)``)."""

    def __init__(self):
        self.marks = []

    def __call__(self, name: str):
        return _Stage(self, name)

    def totals_ms(self) -> dict:
        """Summed elapsed time per stage name (synchronise first)."""
        out: dict = {}
        for name, a, b in self.marks:
            out[name] = out.get(name, 0.0) + a.elapsed_time(b)
        return out


class _Stage:
    def __init__(self, timer, name):
        self.timer, self.name = timer, name

    def __enter__(self):
        if self.timer is not None:
            self.a = torch.cuda.Event(enable_timing=True)
            self.b = torch.cuda.Event(enable_timing=True)
            self.a.record()
        return self

    def __exit__(self, *exc):
        if self.timer is not None:
            self.b.record()
            self.timer.marks.append((self.name, self.a, self.b))
        return False


def stage(timer: Optional[StageTimer], name: str) -> _Stage:
    return _Stage(timer, name)


class Qwen3MoeAttention(nn.Module):
    def __init__(self, cfg: Qwen3MoeConfig, weights: Optional[AttnWeights] = None, device="cuda",
                 seed: int = 0):
        super().__init__()
        if cfg.head_dim != 128:
            raise ValueError("the attention kernels are built for head_dim 128")
        self.cfg = cfg
        self.w = weights if weights is not None else AttnWeights.random(cfg, seed, device)
        self.inv_freq = rope_inv_freq(cfg.head_dim, cfg.rope_theta, self.w.wqkv.device)
        self._decode_ws: Optional[torch.Tensor] = None

    def new_cache(self, n_slots: int, max_seq: int) -> KVCache:
        return KVCache(n_slots, self.cfg.num_key_value_heads, max_seq, self.cfg.head_dim, self.w.wqkv.device)

    def forward(self, hidden_states: torch.Tensor, position_ids: Optional[torch.Tensor] = None,
                past_key_value: Optional[KVCache] = None, timer: Optional[StageTimer] = None,
                attention_mask: Optional[torch.Tensor] = None):
        cfg = self.cfg
        B, S, H = hidden_states.shape
        dev = hidden_states.device
        cache = past_key_value if past_key_value is not None else self.new_cache(B, S)
        if cache.n_slots < B:
            raise ValueError("KV cache has fewer slots than the batch")
        L0 = cache.lengths[:B]
        if max(L0) + S > cache.max_seq:
            raise ValueError("KV cache is full")
        x2d = hidden_states.reshape(B * S, H).to(torch.bfloat16).contiguous()
        pads = left_padding(attention_mask, B, S, L0)
        if pads is not None:
            for b in range(B):
                cache.pad[b] = pads[b]
        pad_now = cache.pad[:B]
        pos = (torch.tensor(L0, dtype=torch.int32).unsqueeze(1) + torch.arange(S, dtype=torch.int32))
        if position_ids is not None:
            given = position_ids.reshape(B, S).to(torch.int32).cpu()
            shifted = pos - torch.tensor(pad_now, dtype=torch.int32).unsqueeze(1)
            real = shifted >= 0  # padding tokens may carry any position
            if not (torch.equal(given, pos) or bool(torch.all((given == shifted) | ~real))):
                raise ValueError("position_ids must continue each sequence's cache contiguously (or, with left "
                                 "padding, count from the first real token)")
        positions = pos.reshape(-1).to(dev, non_blocking=True)
        kv_start = (torch.tensor(pad_now, dtype=torch.int32).to(dev, non_blocking=True)
                    if any(pad_now) else None)
        slots = torch.arange(B, dtype=torch.int32).repeat_interleave(S).to(dev, non_blocking=True)
        with stage(timer, "qkv_proj"):
            qkv = ops.linear(x2d, self.w.wqkv)
        with stage(timer, "qk_norm_rope"):
            q = ops.qk_norm_rope(qkv, positions, self.w.q_norm, self.w.k_norm, self.inv_freq,
                                 cfg.num_attention_heads, cfg.num_key_value_heads, cfg.rms_norm_eps,
                                 cache.k, cache.v, cache_slot=slots)
        if S == 1:
            kv_len = torch.tensor([l + 1 for l in L0], dtype=torch.int32).to(dev, non_blocking=True)
            with stage(timer, "attention"):
                attn = ops.attention_decode(q, cache.k, cache.v, kv_len, max(L0) + 1,
                                            workspace=self._decode_ws, kv_start=kv_start)
        else:
            q_start = torch.tensor(L0, dtype=torch.int32).to(dev, non_blocking=True)
            with stage(timer, "attention"):
                attn = ops.attention_prefill(q, cache.k, cache.v, q_start, B, S, kv_start=kv_start)
        for b in range(B):
            cache.lengths[b] += S
        with stage(timer, "o_proj"):
            out = ops.linear(attn, self.w.wo)
        return out.reshape(B, S, H), cache
