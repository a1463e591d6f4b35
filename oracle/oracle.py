"""CPU oracle for the Qwen3-MoE decoder-layer hot path.

TEST INFRASTRUCTURE ONLY.  Only tests/, ``__graft_entry__.smoke()`` and
bench.py's CPU-baseline leg import this module, and only to check or to time
the reference behaviour.  The product path (``nki_moe_7013_b200``) never
imports it and has no CPU fallback.

Integer / ordering work (router logits in the canonical fp32 order, top-k,
permutation) is done by ``moe_oracle.c`` (exact); floating-point work that is
compared within a tolerance is done here in numpy (fp64 accumulation).

Reference semantics restated (charleshong3/nki-moe-7013):

* router: fp32 logits (qwen.py:260-261), softmax (qwen.py:263), top-8, L1
  renormalisation of the chosen affinities (qwen.py:269,
  qwen_with_nki.py:2402-2405, ``F.normalize(p=1)``: x / max(|x|_1, 1e-12)).
  Ties at equal logits go to the lower expert index.
* experts: ``[g|u] = x @ W_gu[e]`` with the gate half first
  (qwen.py:164-190), ``a = silu(g) * u`` in fp32 and one bf16 cast
  (qwen_with_nki.py:5203-5210), ``y = a @ W_d[e]`` (qwen.py:204-226).
* combine: ``out[t] = sum_j w[t,j] * y[t,j]`` accumulated in fp32 and cast
  to bf16 once (the fp32-internal schedules at qwen_with_nki.py:2360-2373 and
  qwen_with_nki.py:4695-4700, up to final rounding).
* blockwise seam (qwen_with_nki.py:5440-5502, 5656-5667): blocks of
  ``block_size`` token positions, one expert per block, padding positions
  (-1 or T) contribute nothing, a token repeated inside one block counts once.
* RMSNorm: ``x * rsqrt(mean(x^2) + eps) * w`` in fp32 with one output cast
  (qwen_with_nki.py:1286-1342; known-answer test nki_custom_rmsnorm.py:174-214).

Weight layout used here is the device layout of the product: HF order
``w_gate_up (E, 2I, H)`` (gate rows first) and ``w_down (E, H, I)``; the
NxDI layout ``(E, H, 2I)`` / ``(E, I, H)`` (qwen.py:164-226) is its transpose.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None


def build_oracle_lib() -> str:
    src = os.path.join(_HERE, "moe_oracle.c")
    if (not os.path.exists(_LIB_PATH)) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is None:
        build_oracle_lib()
        lib = ctypes.CDLL(_LIB_PATH)
        P = ctypes.c_void_p
        I64 = ctypes.c_int64
        lib.oracle_router_logits.argtypes = [P, P, I64, I64, I64, P]
        lib.oracle_topk.argtypes = [P, I64, I64, I64, P]
        lib.oracle_permute.argtypes = [P, I64, I64, I64, P, P, P, P, P]
        for f in (lib.oracle_router_logits, lib.oracle_topk, lib.oracle_permute):
            f.restype = ctypes.c_int
        _lib = lib
    return _lib


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def as_bf16_bits(t) -> np.ndarray:
    """Accept a torch bf16 tensor or a uint16 array; return uint16 bits."""
    try:
        import torch

        if isinstance(t, torch.Tensor):
            assert t.dtype == torch.bfloat16
            return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)
    except ImportError:  # pragma: no cover
        pass
    a = np.asarray(t)
    assert a.dtype == np.uint16
    return np.ascontiguousarray(a)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def round_to_bf16(a: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 (round to nearest even) -> fp32."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    rounding = ((u >> np.uint32(16)) & np.uint32(1)) + np.uint32(0x7FFF)
    return (((u + rounding) >> np.uint32(16)) << np.uint32(16)).astype(np.uint32).view(np.float32)


# ----------------------------------------------------------------------------
# router
# ----------------------------------------------------------------------------

def router_logits(x_bf16, w_router_bf16, bias=None) -> np.ndarray:
    """Canonical-order fp32 logits (T, E); ``bias`` (E,) fp32 is added after
    the dot product with one fp32 rounding."""
    xb = as_bf16_bits(x_bf16)
    wb = as_bf16_bits(w_router_bf16)
    T, H = xb.shape
    E = wb.shape[0]
    out = np.empty((T, E), dtype=np.float32)
    rc = _load().oracle_router_logits(_ptr(xb), _ptr(wb), T, H, E, _ptr(out))
    if rc != 0:
        raise ValueError(f"oracle_router_logits failed ({rc}); H must be a multiple of 256")
    if bias is not None:
        out = (out + np.asarray(bias, dtype=np.float32)[None, :]).astype(np.float32)
    return out


def topk(logits: np.ndarray, k: int) -> np.ndarray:
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    T, E = logits.shape
    idx = np.empty((T, k), dtype=np.int32)
    rc = _load().oracle_topk(_ptr(logits), T, E, k, _ptr(idx))
    if rc != 0:
        raise ValueError("oracle_topk failed")
    return idx


def softmax(logits: np.ndarray) -> np.ndarray:
    l64 = logits.astype(np.float64)
    m = l64.max(axis=1, keepdims=True)
    p = np.exp(l64 - m)
    return p / p.sum(axis=1, keepdims=True)


def router(x_bf16, w_router_bf16, k: int, normalize: bool = True, bias=None):
    """Returns (logits fp32 (T,E), topk_idx int32 (T,k), topk_w fp32 (T,k))."""
    logits = router_logits(x_bf16, w_router_bf16, bias)
    idx = topk(logits, k)
    p = softmax(logits)
    chosen = np.take_along_axis(p, idx.astype(np.int64), axis=1)
    if normalize:
        chosen = chosen / np.maximum(chosen.sum(axis=1, keepdims=True), 1e-12)
    return logits, idx, chosen.astype(np.float32)


# ----------------------------------------------------------------------------
# permutation
# ----------------------------------------------------------------------------

def permute(topk_idx: np.ndarray, num_experts: int):
    idx = np.ascontiguousarray(topk_idx, dtype=np.int32)
    T, k = idx.shape
    E = num_experts
    counts = np.empty(E, dtype=np.int32)
    offsets = np.empty(E + 1, dtype=np.int32)
    row_token = np.empty(T * k, dtype=np.int32)
    row_slot = np.empty(T * k, dtype=np.int32)
    slot_row = np.empty(T * k, dtype=np.int32)
    rc = _load().oracle_permute(_ptr(idx), T, E, k, _ptr(counts), _ptr(offsets),
                                _ptr(row_token), _ptr(row_slot), _ptr(slot_row))
    if rc != 0:
        raise ValueError("oracle_permute failed (expert id out of range)")
    return dict(counts=counts, offsets=offsets, row_token=row_token,
                row_slot=row_slot, slot_row=slot_row.reshape(T, k))


# ----------------------------------------------------------------------------
# experts + combine
# ----------------------------------------------------------------------------

def silu(x):
    return x / (1.0 + np.exp(-x))


def expert_gate_up_swiglu(x_rows_f32: np.ndarray, w_gate_up_e_f32: np.ndarray) -> np.ndarray:
    """x (n, H) @ W_gu[e]^T (2I, H) -> silu(g)*u, fp64 math, bf16-rounded (n, I)."""
    I2 = w_gate_up_e_f32.shape[0]
    I = I2 // 2
    gu = x_rows_f32.astype(np.float64) @ w_gate_up_e_f32.astype(np.float64).T
    a = silu(gu[:, :I]) * gu[:, I:]
    return round_to_bf16(a.astype(np.float32))


def moe_block(x_bf16, w_router_bf16, w_gate_up_bf16, w_down_bf16, k: int,
              normalize: bool = True, bias=None, return_intermediates: bool = False):
    """Full sparse-MoE block. Returns out fp32 (T, H) before the final bf16
    cast (callers round with ``round_to_bf16``) and optionally intermediates."""
    x = bf16_bits_to_f32(as_bf16_bits(x_bf16))
    wgu = bf16_bits_to_f32(as_bf16_bits(w_gate_up_bf16))
    wd = bf16_bits_to_f32(as_bf16_bits(w_down_bf16))
    E = wgu.shape[0]
    T, H = x.shape
    I = wd.shape[2]
    logits, idx, w = router(x_bf16, w_router_bf16, k, normalize, bias)
    perm = permute(idx, E)
    R = T * k
    act = np.zeros((R, I), dtype=np.float32)
    y = np.zeros((R, H), dtype=np.float64)
    offs = perm["offsets"]
    for e in range(E):
        r0, r1 = int(offs[e]), int(offs[e + 1])
        if r1 == r0:
            continue
        rows = x[perm["row_token"][r0:r1]]
        a = expert_gate_up_swiglu(rows, wgu[e])
        act[r0:r1] = a
        y[r0:r1] = a.astype(np.float64) @ wd[e].astype(np.float64).T
    out = np.zeros((T, H), dtype=np.float64)
    for j in range(k):
        out += w[:, j:j + 1].astype(np.float64) * y[perm["slot_row"][:, j]]
    out = out.astype(np.float32)
    if return_intermediates:
        return out, dict(logits=logits, topk_idx=idx, topk_w=w, act=act, **perm)
    return out


def blockwise_moe(hidden_bf16, affinities_masked, token_position_to_id, block_to_expert,
                  block_size: int, w_gate_up_bf16, w_down_bf16) -> np.ndarray:
    """NxDI blockwise seam (qwen_with_nki.py:5872-5881, 5440-5502).

    ``affinities_masked`` (T or T+1, E) fp32/bf16 values, ``token_position_to_id``
    (N*B,), ``block_to_expert`` (N,).  Weight layout is the product's
    (E, 2I, H) / (E, H, I).  Returns fp32 (T, H) before the output cast."""
    x = bf16_bits_to_f32(as_bf16_bits(hidden_bf16))
    wgu = bf16_bits_to_f32(as_bf16_bits(w_gate_up_bf16))
    wd = bf16_bits_to_f32(as_bf16_bits(w_down_bf16))
    aff = np.asarray(affinities_masked, dtype=np.float32)
    T, H = x.shape
    tpi = np.asarray(token_position_to_id).reshape(-1, block_size)
    b2e = np.asarray(block_to_expert).reshape(-1)
    out = np.zeros((T, H), dtype=np.float64)
    for b in range(tpi.shape[0]):
        e = int(b2e[b])
        toks = tpi[b]
        seen = set()
        chosen = []
        # last occurrence of a token in the block wins (earlier ones redirected)
        for p in range(block_size - 1, -1, -1):
            t = int(toks[p])
            if t < 0 or t >= T or t in seen:
                continue
            seen.add(t)
            chosen.append(t)
        if not chosen:
            continue
        chosen = np.array(sorted(chosen), dtype=np.int64)
        a = expert_gate_up_swiglu(x[chosen], wgu[e])
        y = a.astype(np.float64) @ wd[e].astype(np.float64).T
        out[chosen] += aff[chosen, e].astype(np.float64)[:, None] * y
    return out.astype(np.float32)


# ----------------------------------------------------------------------------
# norms
# ----------------------------------------------------------------------------

def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """fp32 RMSNorm (NxDI / NKI schedule: weight multiply in fp32, one cast by caller)."""
    x64 = np.asarray(x, dtype=np.float64)
    var = np.mean(x64 * x64, axis=-1, keepdims=True)
    return (x64 / np.sqrt(var + eps) * np.asarray(w, dtype=np.float64)).astype(np.float32)


def numpy_rmsnorm_known_answer(x, weight, eps):
    """The reference's own numpy golden (nki_custom_rmsnorm.py:174-179), restated."""
    variance = np.mean(x ** 2, axis=-1, keepdims=True)
    x_norm = x / np.sqrt(variance + eps)
    return x_norm * weight


# ----------------------------------------------------------------------------
# attention sub-layer and decoder layer (HF Qwen3MoeAttention semantics,
# qwen.py:313-341; decoder layer qwen.py:378-436)
# ----------------------------------------------------------------------------

def rope_inv_freq(head_dim: int, theta: float) -> np.ndarray:
    """fp32 inverse frequencies as HF / NxDI RotaryEmbedding compute them."""
    import torch

    return (1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))).numpy()


def rope_apply(x: np.ndarray, pos: np.ndarray, inv_freq: np.ndarray) -> np.ndarray:
    """rotate-half RoPE on (..., T, hd) with per-token positions (T,)."""
    hd = x.shape[-1]
    ang = pos.astype(np.float32)[:, None] * inv_freq[None, :].astype(np.float32)  # fp32 angle (as HF)
    cos = np.cos(ang.astype(np.float64))
    sin = np.sin(ang.astype(np.float64))
    x1, x2 = x[..., : hd // 2], x[..., hd // 2:]
    return np.concatenate([x1 * cos - x2 * sin, x2 * cos + x1 * sin], axis=-1)


def attention_layer(x_bf16, wqkv_bf16, wo_bf16, q_norm_w, k_norm_w, nh: int, nkv: int, eps: float,
                    theta: float, B: int, S: int, k_cache=None, v_cache=None, L0=None, pad=None):
    """Attention sub-layer on B sequences of S new tokens each.

    ``k_cache``/``v_cache`` (B, nkv, Lmax, hd) fp32 hold bf16 values of earlier
    tokens (rows [0, L0[b])).  Intermediates are rounded to bf16 where the GPU
    path stores bf16 (qkv, normalised+rotated q/k, attention output).
    ``pad`` (per sequence, HF left padding as given by a 2D attention mask):
    cache rows [0, pad[b]) are padding -- never attended to -- and, as in HF
    transformers (position_ids = cumsum(mask) - 1), RoPE rotates the token in
    cache row c by position c - pad[b]; padding query rows get a zero output.
    Returns (out fp32 (B*S, H) before its bf16 cast, new_k, new_v)."""
    x = bf16_bits_to_f32(as_bf16_bits(x_bf16)).astype(np.float64)
    wqkv = bf16_bits_to_f32(as_bf16_bits(wqkv_bf16)).astype(np.float64)
    wo = bf16_bits_to_f32(as_bf16_bits(wo_bf16)).astype(np.float64)
    hd = 128
    L0 = np.zeros(B, np.int64) if L0 is None else np.asarray(L0, np.int64)
    pad = np.zeros(B, np.int64) if pad is None else np.asarray(pad, np.int64)
    qkv = round_to_bf16((x @ wqkv.T).astype(np.float32)).astype(np.float64)
    qkv = qkv.reshape(B, S, nh + 2 * nkv, hd)
    inv_freq = rope_inv_freq(hd, theta)
    out_heads = np.zeros((B, S, nh, hd))
    Lmax = int((L0 + S).max())
    new_k = np.zeros((B, nkv, Lmax, hd))
    new_v = np.zeros((B, nkv, Lmax, hd))
    for b in range(B):
        pos = L0[b] + np.arange(S)           # cache rows of the new tokens
        rpos = np.maximum(pos - pad[b], 0)   # their RoPE positions
        q = qkv[b, :, :nh]
        k = qkv[b, :, nh:nh + nkv]
        v = qkv[b, :, nh + nkv:]

        def head_norm(t, w):
            var = np.mean(t * t, axis=-1, keepdims=True)
            return t / np.sqrt(var + eps) * np.asarray(w, np.float64)

        q = rope_apply(head_norm(q, q_norm_w).transpose(1, 0, 2), rpos, inv_freq)  # (nh, S, hd)
        k = rope_apply(head_norm(k, k_norm_w).transpose(1, 0, 2), rpos, inv_freq)  # (nkv, S, hd)
        q = round_to_bf16(q.astype(np.float32)).astype(np.float64)
        k = round_to_bf16(k.astype(np.float32)).astype(np.float64)
        v = v.transpose(1, 0, 2)
        if L0[b] > 0:
            new_k[b, :, :L0[b]] = k_cache[b, :, :L0[b]]
            new_v[b, :, :L0[b]] = v_cache[b, :, :L0[b]]
        new_k[b, :, L0[b]:L0[b] + S] = k
        new_v[b, :, L0[b]:L0[b] + S] = v
        L = L0[b] + S
        for h in range(nh):
            g = h // (nh // nkv)
            sc = q[h] @ new_k[b, g, :L].T / np.sqrt(hd)  # (S, L)
            keys = np.arange(L)[None, :]
            mask = (keys > pos[:, None]) | (keys < pad[b])
            sc = np.where(mask, -np.inf, sc)
            live = ~np.all(mask, axis=1)          # padding queries see no key
            sc = np.where(live[:, None], sc - np.where(live, sc.max(axis=1), 0.0)[:, None], -np.inf)
            p = np.exp(sc)
            p /= np.where(live, p.sum(axis=1), 1.0)[:, None]
            out_heads[b, :, h] = p @ new_v[b, g, :L]
    attn = round_to_bf16(out_heads.reshape(B * S, nh * hd).astype(np.float32)).astype(np.float64)
    return (attn @ wo.T).astype(np.float32), new_k, new_v


def decoder_layer(x_bf16, w_in, w_post, attn_args: dict, moe_args: dict, eps: float, B: int, S: int):
    """Full decoder layer (prefill from an empty cache).  Returns fp32 (B*S, H)
    before the final bf16 cast."""
    import torch

    x = bf16_bits_to_f32(as_bf16_bits(x_bf16))
    h = round_to_bf16(rmsnorm(x, w_in, eps))
    hb = torch.from_numpy(h).to(torch.bfloat16)
    a, _, _ = attention_layer(hb, B=B, S=S, eps=eps, **attn_args)
    a = round_to_bf16(a)
    res2 = round_to_bf16(x + a)
    h2 = round_to_bf16(rmsnorm(res2, w_post, eps))
    moe = moe_block(torch.from_numpy(h2).to(torch.bfloat16), **moe_args)
    return (res2.astype(np.float64) + moe.astype(np.float64)).astype(np.float32)
