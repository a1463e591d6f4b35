"""Shared test utilities: seeded inputs and the tolerance metric."""
from __future__ import annotations

import numpy as np
import torch

from nki_moe_7013_b200.synth import normal_bf16, normal_bf16_device

# Activation tolerance of the north star: max relative error <= 2e-2, measured
# normwise as max|actual - expected| / max|expected|.
MAX_REL = 2e-2


def max_rel_err(actual, expected) -> float:
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    denom = max(float(np.abs(e).max()), 1e-30)
    return float(np.abs(a - e).max()) / denom


def to_f32_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def moe_weights(seed: int, E: int, H: int, I: int, device, std: float = 0.02):
    """Router (E,H), gate_up (E,2I,H), down (E,H,I) bf16 ~N(0, std^2) on `device`."""
    if str(device).startswith("cuda"):
        wr = normal_bf16_device(seed * 10 + 1, (E, H), std, device)
        wgu = normal_bf16_device(seed * 10 + 2, (E, 2 * I, H), std, device)
        wd = normal_bf16_device(seed * 10 + 3, (E, H, I), std, device)
    else:
        wr = normal_bf16(seed, "w_router", (E, H), std)
        wgu = normal_bf16(seed, "w_gate_up", (E, 2 * I, H), std)
        wd = normal_bf16(seed, "w_down", (E, H, I), std)
    return wr, wgu, wd


def activations(seed: int, T: int, H: int, device):
    if str(device).startswith("cuda"):
        return normal_bf16_device(seed * 10 + 4, (T, H), 1.0, device)
    return normal_bf16(seed, "x", (T, H), 1.0)


def assert_within_one_ulp(actual: torch.Tensor, expected: torch.Tensor, what: str = "") -> None:
    """bf16 results of the same arithmetic whose fp32 sums were added in a
    different order: every element within one bf16 ulp of the other (2^-7 of
    its magnitude), nothing more.  A missed, doubled or overwritten
    contribution is far larger."""
    a = actual.float()
    e = expected.float()
    tol = e.abs() * 2.0 ** -7 + 1e-6
    bad = (a - e).abs() > tol
    n = int(bad.sum())
    if n:
        i = torch.nonzero(bad)[0].tolist()
        raise AssertionError(f"{what}: {n} elements differ by more than one bf16 ulp, first at {i}: "
                             f"{float(a[tuple(i)])} vs {float(e[tuple(i)])}")
