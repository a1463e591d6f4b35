"""Seeded synthetic inputs for the Qwen3-MoE layer.

The reference measures on a real Qwen3-30B-A3B checkpoint and text prompts;
none are available here, so every config uses random-init weights and
activations of the same shapes and value distributions
(weights ~N(0, 0.02), activations ~N(0, 1), rounded to bf16).

Two generators:

* ``normal_bf16`` -- counter-based (splitmix64 + Box-Muller in numpy).  The
  stream depends only on (seed, name, index), never on the numpy or torch
  version, so committed golden fixtures can be regenerated bit-for-bit on any
  machine.  Used for the small golden / parity shapes.
* ``normal_bf16_device`` -- ``torch.randn`` with a seeded generator on the
  target device.  Fast enough for the 1.2 GB of expert weights of a full
  layer; deterministic for a given torch build and device.
"""
from __future__ import annotations

import hashlib

import numpy as np
import torch

_MASK64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def _stream_key(seed: int, name: str) -> np.uint64:
    h = hashlib.sha256(f"{seed}:{name}".encode()).digest()
    return np.uint64(int.from_bytes(h[:8], "little"))


def _splitmix64(z: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = (z + np.uint64(0x9E3779B97F4A7C15)) & _MASK64
        z = ((z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)) & _MASK64
        z = ((z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)) & _MASK64
        return z ^ (z >> np.uint64(31))


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16, returned as uint16 bit patterns."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    rounding = ((u >> np.uint32(16)) & np.uint32(1)) + np.uint32(0x7FFF)
    return ((u + rounding) >> np.uint32(16)).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def normal_bf16(seed: int, name: str, shape, std: float = 1.0, mean: float = 0.0) -> torch.Tensor:
    """Counter-based N(mean, std^2) sample rounded to bf16 (CPU tensor)."""
    n = int(np.prod(shape)) if len(shape) else 1
    key = _stream_key(seed, name)
    out = np.empty(n, dtype=np.uint16)
    block = 1 << 18  # cache-sized blocks
    for s0 in range(0, n, block):
        ctr = np.arange(s0, min(n, s0 + block), dtype=np.uint64)
        with np.errstate(over="ignore"):
            base = (ctr * np.uint64(2)) ^ key
        a = _splitmix64(base)
        b = _splitmix64(base ^ np.uint64(0xD1B54A32D192ED03))
        # 53-bit uniforms in (0, 1]
        u1 = ((a >> np.uint64(11)).astype(np.float64) + 1.0) / 9007199254740992.0
        u2 = (b >> np.uint64(11)).astype(np.float64) / 9007199254740992.0
        z = np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)
        out[s0:s0 + len(ctr)] = f32_to_bf16_bits((z * std + mean).astype(np.float32))
    return torch.from_numpy(out.view(np.int16)).view(torch.bfloat16).reshape(shape)


def normal_bf16_device(seed: int, shape, std: float = 1.0, device="cuda") -> torch.Tensor:
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    t = torch.randn(*shape, generator=g, device=device, dtype=torch.float32)
    if std != 1.0:
        t.mul_(std)
    return t.to(torch.bfloat16)


def zipf_expert_bias(seed: int, num_experts: int, s: float = 1.2) -> torch.Tensor:
    """Per-expert router-logit bias b_e = log p_e with p_e proportional to
    rank(e)^-s under a seeded permutation of ranks (config 4's skew)."""
    rng = np.random.default_rng(seed)
    ranks = rng.permutation(num_experts) + 1
    p = ranks.astype(np.float64) ** (-s)
    p /= p.sum()
    return torch.from_numpy(np.log(p).astype(np.float32))
