"""torch-facing wrappers of the C ABI (one function per qmoe_* entry point).

Every wrapper checks dtype / device / contiguity, allocates outputs with the
torch caching allocator, passes raw pointers plus the current CUDA stream to
the library, and raises ``QmoeError`` on a non-zero status.  Nothing here
computes on the CPU.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _C

ROUTER_CHUNK = 8  # QMOE_ROUTER_CHUNK
ROUTER_SMALL_MAX_T = 64  # batches up to this size take the two-kernel small-batch router
GATHER_MAX_T = 64  # batches up to this size gather token rows inside the gate/up GEMM
FUSED_GATHER_MAX_T = GATHER_MAX_T  # the fused experts kernel reads the permuted copy (faster from 256 tokens)
FUSED_MIN_T = 2  # above this many tokens the forward runs the experts as the fused persistent kernel
GATEUP_SPLIT_MAX_R = 128  # routed rows up to which the gate/up GEMM may split K
ROUTE_SMALL_MAX_T = 16  # batches up to this size (E <= 128) route + permute in one launch
ROUTE_SMALL_MAX_E = 128


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def _stream(dev: torch.device):
    return torch.cuda.current_stream(dev).cuda_stream


def _need(t: torch.Tensor, name: str, dtype=None, dim=None):
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a tensor")
    if t.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor (got {t.device}); there is no CPU path")
    if dtype is not None and t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype} (got {t.dtype})")
    if dim is not None and t.dim() != dim:
        raise ValueError(f"{name} must have {dim} dims (got shape {tuple(t.shape)})")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return t


def max_tiles(rows: int, num_experts: int) -> int:
    return int(_C.lib().qmoe_max_tiles(rows, num_experts))


def router_topk(x: torch.Tensor, w_router: torch.Tensor, k: int, normalize: bool = True,
                bias: Optional[torch.Tensor] = None, return_logits: bool = False,
                return_hist: bool = False):
    """K1.  Returns (topk_idx int32 (T,k), topk_w fp32 (T,k)[, logits fp32 (T,E)][, chunk_hist])."""
    _need(x, "x", torch.bfloat16, 2)
    _need(w_router, "w_router", torch.bfloat16, 2)
    T, H = x.shape
    E = w_router.shape[0]
    if bias is not None:
        _need(bias, "bias", torch.float32, 1)
    dev = x.device
    idx = torch.empty((T, k), dtype=torch.int32, device=dev)
    w = torch.empty((T, k), dtype=torch.float32, device=dev)
    # a logits buffer also enables the small-batch router path
    logits = (torch.empty((T, E), dtype=torch.float32, device=dev)
              if (return_logits or T <= ROUTER_SMALL_MAX_T) else None)
    hist = (torch.empty(((T + ROUTER_CHUNK - 1) // ROUTER_CHUNK, E), dtype=torch.int32, device=dev)
            if return_hist else None)
    with torch.cuda.device(dev):
        _C.check(_C.lib().qmoe_router_topk(
            _ptr(x), _ptr(w_router), _ptr(bias), T, H, E, k, 1 if normalize else 0,
            _ptr(logits), _ptr(idx), _ptr(w), _ptr(hist), _stream(dev)), "qmoe_router_topk")
    out = [idx, w]
    if return_logits:
        out.append(logits)
    if return_hist:
        out.append(hist)
    return tuple(out)


def route_small(x: torch.Tensor, w_router: torch.Tensor, k: int, normalize: bool = True,
                bias: Optional[torch.Tensor] = None, acc_zero: Optional[torch.Tensor] = None):
    """K1 + K2 in one launch for T <= ROUTE_SMALL_MAX_T tokens (E <= 128).
    Returns a dict with the router outputs (topk_idx, topk_w, logits) and the
    permutation outputs (counts, offsets, row_token, row_w, slot_row, tiles,
    max_tiles); ``acc_zero`` (T, H) fp32 is zero-filled."""
    _need(x, "x", torch.bfloat16, 2)
    _need(w_router, "w_router", torch.bfloat16, 2)
    T, H = x.shape
    E = w_router.shape[0]
    if bias is not None:
        _need(bias, "bias", torch.float32, 1)
    dev = x.device
    R = T * k
    mt = max_tiles(R, E)
    i32 = dict(dtype=torch.int32, device=dev)
    f32 = dict(dtype=torch.float32, device=dev)
    out = dict(topk_idx=torch.empty((T, k), **i32), topk_w=torch.empty((T, k), **f32),
               logits=torch.empty((T, E), **f32), counts=torch.empty(E, **i32),
               offsets=torch.empty(E + 1, **i32), row_token=torch.empty(max(R, 1), **i32),
               row_w=torch.empty(max(R, 1), **f32), slot_row=torch.empty((T, k), **i32),
               tiles=torch.zeros(1 + 3 * mt, **i32), max_tiles=mt)
    with torch.cuda.device(dev):
        _C.check(_C.lib().qmoe_route_small(
            _ptr(x), _ptr(w_router), _ptr(bias), T, H, E, k, 1 if normalize else 0, _ptr(out["logits"]),
            _ptr(out["topk_idx"]), _ptr(out["topk_w"]), _ptr(out["counts"]), _ptr(out["offsets"]),
            _ptr(out["row_token"]), _ptr(out["row_w"]), _ptr(out["slot_row"]), _ptr(out["tiles"]),
            _ptr(acc_zero), _stream(dev)), "qmoe_route_small")
    return out


def moe_permute(topk_idx: torch.Tensor, topk_w: torch.Tensor, chunk_hist: torch.Tensor,
                num_experts: int, x: Optional[torch.Tensor] = None, gather: bool = True,
                acc_zero: Optional[torch.Tensor] = None):
    """K2.  ``chunk_hist`` is overwritten.  Returns a dict of device tensors,
    among them ``done``: the zero-filled counters moe_experts needs."""
    _need(topk_idx, "topk_idx", torch.int32, 2)
    _need(topk_w, "topk_w", torch.float32, 2)
    _need(chunk_hist, "chunk_hist", torch.int32, 2)
    T, k = topk_idx.shape
    E = num_experts
    R = T * k
    dev = topk_idx.device
    H = 0
    x_perm = None
    if x is not None:
        _need(x, "x", torch.bfloat16, 2)
        H = x.shape[1]
        if gather:
            x_perm = torch.empty((R, H), dtype=torch.bfloat16, device=dev)
    if acc_zero is not None:
        _need(acc_zero, "acc_zero", torch.float32, 2)
        H = acc_zero.shape[1]
    mt = max_tiles(R, E)
    counts = torch.empty(E, dtype=torch.int32, device=dev)
    offsets = torch.empty(E + 1, dtype=torch.int32, device=dev)
    row_token = torch.empty(R, dtype=torch.int32, device=dev)
    row_w = torch.empty(R, dtype=torch.float32, device=dev)
    slot_row = torch.empty((T, k), dtype=torch.int32, device=dev)
    tiles = torch.empty(1 + 3 * mt, dtype=torch.int32, device=dev)
    done = torch.empty(mt + 1, dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        _C.check(_C.lib().qmoe_moe_permute(
            _ptr(topk_idx), _ptr(topk_w), _ptr(chunk_hist), _ptr(x), T, H, E, k,
            _ptr(counts), _ptr(offsets), _ptr(row_token), _ptr(row_w), _ptr(slot_row),
            _ptr(tiles), _ptr(x_perm), _ptr(acc_zero), _ptr(done), mt + 1,
            _stream(dev)), "qmoe_moe_permute")
    return dict(counts=counts, offsets=offsets, row_token=row_token, row_w=row_w,
                slot_row=slot_row, tiles=tiles, max_tiles=mt, x_perm=x_perm, done=done)


def route_permute(x: torch.Tensor, w_router: torch.Tensor, k: int, normalize: bool = True,
                  bias: Optional[torch.Tensor] = None, gather: bool = True,
                  acc_zero: Optional[torch.Tensor] = None):
    """K1 + K2 in one call (one launch for prefill batches of at most one
    router chunk per SM): the outputs of router_topk followed by moe_permute,
    as moe_permute's dict plus topk_idx / topk_w."""
    _need(x, "x", torch.bfloat16, 2)
    _need(w_router, "w_router", torch.bfloat16, 2)
    T, H = x.shape
    E = w_router.shape[0]
    R = T * k
    dev = x.device
    i32 = dict(dtype=torch.int32, device=dev)
    mt = max_tiles(R, E)
    out = dict(topk_idx=torch.empty((T, k), **i32), topk_w=torch.empty((T, k), dtype=torch.float32, device=dev),
               chunk_hist=torch.empty((max((T + ROUTER_CHUNK - 1) // ROUTER_CHUNK, 1), E), **i32),
               counts=torch.empty(E, **i32), offsets=torch.empty(E + 1, **i32), row_token=torch.empty(R, **i32),
               row_w=torch.empty(R, dtype=torch.float32, device=dev), slot_row=torch.empty((T, k), **i32),
               tiles=torch.empty(1 + 3 * mt, **i32), max_tiles=mt, done=torch.empty(mt + 1, **i32),
               x_perm=torch.empty((R, H), dtype=torch.bfloat16, device=dev) if gather else None)
    barrier = torch.zeros(2, **i32)
    if acc_zero is not None:
        _need(acc_zero, "acc_zero", torch.float32, 2)
    if bias is not None:
        _need(bias, "bias", torch.float32, 1)
    with torch.cuda.device(dev):
        _C.check(_C.lib().qmoe_route_permute(
            _ptr(x), _ptr(w_router), _ptr(bias), T, H, E, k, 1 if normalize else 0, _ptr(out["topk_idx"]),
            _ptr(out["topk_w"]), _ptr(out["chunk_hist"]), _ptr(out["counts"]), _ptr(out["offsets"]),
            _ptr(out["row_token"]), _ptr(out["row_w"]), _ptr(out["slot_row"]), _ptr(out["tiles"]),
            _ptr(out["x_perm"]), _ptr(acc_zero), _ptr(out["done"]), mt + 1, _ptr(barrier), _stream(dev)),
            "qmoe_route_permute")
    out["barrier"] = barrier
    return out


def moe_experts(x: torch.Tensor, w_gate_up: torch.Tensor, w_down: torch.Tensor, tiles: torch.Tensor,
                max_tiles_: int, row_dst: torch.Tensor, row_w: torch.Tensor, acc: torch.Tensor,
                done: torch.Tensor, act: Optional[torch.Tensor] = None,
                gather_rows: Optional[torch.Tensor] = None) -> torch.Tensor:
    """K3a + K3b in one persistent kernel (prefill): acc[row_dst[r]] +=
    row_w[r] * SwiGLU(x_r) @ W_down[e]^T, x_r = x_perm[r] (``x`` = the
    permuted rows) or x[gather_rows[r]] (``x`` = the token rows).  ``done``
    (max_tiles + 1,) int32 must be zero-filled (moe_permute's ``done``).
    Returns acc."""
    _need(x, "x", torch.bfloat16, 2)
    _need(w_gate_up, "w_gate_up", torch.bfloat16, 3)
    _need(w_down, "w_down", torch.bfloat16, 3)
    _need(tiles, "tiles", torch.int32, 1)
    _need(acc, "acc", torch.float32, 2)
    _need(done, "done", torch.int32, 1)
    rows, H = x.shape
    R = rows
    if gather_rows is not None:
        _need(gather_rows, "gather_rows", torch.int32, 1)
        R = gather_rows.shape[0]
    E, I2, H2 = w_gate_up.shape
    I = I2 // 2
    if H2 != H or tuple(w_down.shape) != (E, H, I) or acc.shape[1] != H:
        raise ValueError("moe_experts: weight / activation shapes do not match")
    dev = x.device
    if act is None:
        act = torch.empty((max(R, 1), I), dtype=torch.bfloat16, device=dev)
    with torch.cuda.device(dev):
        _C.check(_C.lib().qmoe_moe_experts(
            _ptr(x), rows, _ptr(gather_rows), _ptr(w_gate_up), _ptr(w_down), _ptr(tiles), max_tiles_,
            _ptr(row_dst), _ptr(row_w), R, H, I, E, _ptr(act), _ptr(acc), acc.shape[0], _ptr(done), _stream(dev)),
            "qmoe_moe_experts")
    return acc


def gateup_split_workspace(device) -> torch.Tensor:
    """Zero-filled scratch that lets decode-sized gate/up calls split K over
    several CTAs (``split_ws`` of grouped_gemm_gateup_swiglu); every launch
    leaves it zero-filled.  Calls that share one must not overlap on the GPU."""
    n = int(_C.lib().qmoe_grouped_gemm_gateup_split_workspace_size())
    return torch.zeros(n, dtype=torch.uint8, device=device)


def grouped_gemm_gateup_swiglu(x: torch.Tensor, w_gate_up: torch.Tensor, tiles: torch.Tensor,
                               max_tiles_: int, out: Optional[torch.Tensor] = None,
                               gather_rows: Optional[torch.Tensor] = None,
                               split_ws: Optional[torch.Tensor] = None, max_tile_rows: int = 128) -> torch.Tensor:
    """K3a.  act (R, I) bf16 = SiLU(x W_gate^T) * (x W_up^T) in grouped order.
    ``x`` is x_perm (R, H), or with ``gather_rows`` (R,) int32 the source
    activations whose row gather_rows[r] is grouped row r.  ``split_ws``
    (from gateup_split_workspace) lets R <= 128 calls split K.
    ``max_tile_rows``: a bound on the rows of any tile (min(T, 128) for
    router-built tiles); <= 16 selects the decode configuration."""
    _need(x, "x", torch.bfloat16, 2)
    _need(w_gate_up, "w_gate_up", torch.bfloat16, 3)
    _need(tiles, "tiles", torch.int32, 1)
    rows, H = x.shape
    R = rows
    if gather_rows is not None:
        _need(gather_rows, "gather_rows", torch.int32, 1)
        R = gather_rows.shape[0]
    E, I2, H2 = w_gate_up.shape
    if H2 != H or I2 % 2:
        raise ValueError("w_gate_up must be (E, 2I, H) matching x")
    I = I2 // 2
    dev = x.device
    act = out if out is not None else torch.empty((R, I), dtype=torch.bfloat16, device=dev)
    with torch.cuda.device(dev):
        _C.check(_C.lib().qmoe_grouped_gemm_gateup_swiglu(
            _ptr(x), rows, _ptr(gather_rows), _ptr(w_gate_up), _ptr(tiles), max_tiles_, max_tile_rows, R, H, I, E,
            _ptr(act), _ptr(split_ws), 0 if split_ws is None else split_ws.numel() * split_ws.element_size(),
            _stream(dev)), "qmoe_grouped_gemm_gateup_swiglu")
    return act


def grouped_gemm_down_combine(act: torch.Tensor, w_down: torch.Tensor, tiles: torch.Tensor,
                              max_tiles_: int, row_dst: torch.Tensor, row_w: torch.Tensor,
                              acc: torch.Tensor, max_tile_rows: int = 128,
                              tiles_ready: bool = False) -> torch.Tensor:
    """K3b.  acc[row_dst[r]] += row_w[r] * act[r] @ W_down[e]^T (fp32, in place).
    ``max_tile_rows`` as for grouped_gemm_gateup_swiglu.  ``tiles_ready``:
    the tile list was complete before the previous kernel on the stream began
    (QMOE_GEMM_TILES_READY), e.g. right after the gate/up GEMM on the same tiles."""
    _need(act, "act", torch.bfloat16, 2)
    _need(w_down, "w_down", torch.bfloat16, 3)
    _need(tiles, "tiles", torch.int32, 1)
    _need(row_dst, "row_dst", torch.int32, 1)
    _need(row_w, "row_w", torch.float32, 1)
    _need(acc, "acc", torch.float32, 2)
    R, I = act.shape
    E, H, I2 = w_down.shape
    if I2 != I or acc.shape[1] != H:
        raise ValueError("w_down must be (E, H, I) matching act and acc")
    dev = act.device
    with torch.cuda.device(dev):
        _C.check(_C.lib().qmoe_grouped_gemm_down_combine(
            _ptr(act), _ptr(w_down), _ptr(tiles), max_tiles_, max_tile_rows, 1 if tiles_ready else 0,
            _ptr(row_dst), _ptr(row_w),
            R, H, I, E, _ptr(acc), acc.shape[0], _stream(dev)), "qmoe_grouped_gemm_down_combine")
    return acc


def blockwise_prepare(x: torch.Tensor, affinities: torch.Tensor, token_position_to_id: torch.Tensor,
                      block_to_expert: torch.Tensor, block_size: int, num_blocks: int):
    """NxDI blockwise seam -> rows + tiles for the grouped GEMMs."""
    _need(x, "x", torch.bfloat16, 2)
    _need(affinities, "affinities", torch.float32, 2)
    _need(token_position_to_id, "token_position_to_id", torch.int32, 1)
    _need(block_to_expert, "block_to_expert", torch.int32, 1)
    T, H = x.shape
    E = affinities.shape[1]
    n = block_size * num_blocks
    if token_position_to_id.numel() != n or block_to_expert.numel() != num_blocks:
        raise ValueError("token_position_to_id must hold num_blocks*block_size ids")
    dev = x.device
    mt = int(_C.lib().qmoe_blockwise_max_tiles(block_size, num_blocks))
    x_perm = torch.empty((max(n, 1), H), dtype=torch.bfloat16, device=dev)
    row_dst = torch.empty(max(n, 1), dtype=torch.int32, device=dev)
    row_w = torch.empty(max(n, 1), dtype=torch.float32, device=dev)
    tiles = torch.zeros(1 + 3 * mt, dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        _C.check(_C.lib().qmoe_blockwise_prepare(
            _ptr(x), _ptr(affinities), affinities.shape[0], _ptr(token_position_to_id),
            _ptr(block_to_expert), T, H, E, block_size, num_blocks, _ptr(x_perm), _ptr(row_dst),
            _ptr(row_w), _ptr(tiles), _stream(dev)), "qmoe_blockwise_prepare")
    return dict(x_perm=x_perm, row_dst=row_dst, row_w=row_w, tiles=tiles, max_tiles=mt)


def combine_finalize(acc: torch.Tensor, residual: Optional[torch.Tensor] = None,
                     out: Optional[torch.Tensor] = None) -> torch.Tensor:
    _need(acc, "acc", torch.float32, 2)
    T, H = acc.shape
    if residual is not None:
        _need(residual, "residual", torch.bfloat16, 2)
    dev = acc.device
    out = out if out is not None else torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    with torch.cuda.device(dev):
        _C.check(_C.lib().qmoe_combine_finalize(_ptr(acc), _ptr(residual), T, H, _ptr(out),
                                                _stream(dev)), "qmoe_combine_finalize")
    return out


def embedding(ids: torch.Tensor, table: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out[i] = table[ids[i]] (bf16 rows); ids outside [0, V) give zero rows
    and device error 4."""
    _need(ids, "ids", torch.int32, 1)
    _need(table, "table", torch.bfloat16, 2)
    V, H = table.shape
    n = ids.shape[0]
    dev = table.device
    out = out if out is not None else torch.empty((n, H), dtype=torch.bfloat16, device=dev)
    with torch.cuda.device(dev):
        _C.check(_C.lib().qmoe_embedding_gather(_ptr(table), V, H, _ptr(ids), n, _ptr(out), _stream(dev)),
                 "qmoe_embedding_gather")
    return out


def masked_residual_add(y: torch.Tensor, mask: Optional[torch.Tensor] = None,
                        residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out = bf16(residual + mask[:, None] * y), fp32 arithmetic and one
    rounding (mask None = 1, residual None = 0): the MoE output under the
    block's padding_mask plus the decoder layer's residual, in one launch."""
    _need(y, "y", torch.bfloat16, 2)
    T, H = y.shape
    dev = y.device
    m = None
    if mask is not None:
        m = mask.reshape(-1).to(device=dev, dtype=torch.float32).contiguous()
        if m.numel() != T:
            raise ValueError(f"mask has {m.numel()} entries for {T} rows")
    if residual is not None:
        _need(residual, "residual", torch.bfloat16, 2)
        if tuple(residual.shape) != (T, H):
            raise ValueError("residual must have the shape of y")
        residual = residual.contiguous()
    y = y.contiguous()
    out = torch.empty_like(y)
    with torch.cuda.device(dev):
        _C.check(_C.lib().qmoe_masked_residual_add(_ptr(y), _ptr(m), _ptr(residual), T, H, _ptr(out),
                                                   _stream(dev)), "qmoe_masked_residual_add")
    return out


def greedy_pick(logits: torch.Tensor, tokens: Optional[torch.Tensor] = None,
                positions: Optional[torch.Tensor] = None, lengths: Optional[torch.Tensor] = None) -> torch.Tensor:
    """tokens[b] = argmax of logits[b] (int32; first maximal index, NaN
    largest), and positions / lengths (int32, B) advanced by one, in one
    launch."""
    _need(logits, "logits", torch.bfloat16, 2)
    B, V = logits.shape
    dev = logits.device
    logits = logits.contiguous()
    tokens = torch.empty(B, dtype=torch.int32, device=dev) if tokens is None else tokens
    for name, t in (("tokens", tokens), ("positions", positions), ("lengths", lengths)):
        if t is not None:
            _need(t, name, torch.int32, 1)
            if t.shape[0] != B or not t.is_contiguous():
                raise ValueError(f"{name} must be a contiguous ({B},) int32 tensor")
    with torch.cuda.device(dev):
        _C.check(_C.lib().qmoe_greedy_pick(_ptr(logits), B, V, _ptr(tokens), _ptr(positions), _ptr(lengths),
                                           _stream(dev)), "qmoe_greedy_pick")
    return tokens


def select_affinities(affinities: torch.Tensor, idx: torch.Tensor, normalize: bool = True) -> torch.Tensor:
    """w (T, k) fp32 = affinities[t, idx[t, j]], L1-normalised per token when
    ``normalize`` (F.normalize(p=1): divided by max(sum |w|, 1e-12))."""
    _need(idx, "idx", torch.int32, 2)
    T, k = idx.shape
    dev = idx.device
    a = affinities.reshape(T, -1).to(device=dev, dtype=torch.float32).contiguous()
    w = torch.empty((T, k), dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        _C.check(_C.lib().qmoe_select_affinities(_ptr(a), _ptr(idx.contiguous()), T, a.shape[1], k,
                                                 1 if normalize else 0, _ptr(w), _stream(dev)),
                 "qmoe_select_affinities")
    return w


def moe_forward_workspace_size(T: int, H: int, E: int, k: int, I: int) -> int:
    return int(_C.lib().qmoe_moe_forward_workspace_size(T, H, E, k, I))


def moe_forward(x: torch.Tensor, w_router: torch.Tensor, w_gate_up: torch.Tensor,
                w_down: torch.Tensor, k: int, normalize: bool = True,
                residual: Optional[torch.Tensor] = None, bias: Optional[torch.Tensor] = None,
                workspace: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
                return_routing: bool = False):
    """Fused sparse-MoE block (K1..finalize).  Returns out (T,H) bf16
    [, topk_idx (T,k) int32, topk_w (T,k) fp32]."""
    _need(x, "x", torch.bfloat16, 2)
    _need(w_router, "w_router", torch.bfloat16, 2)
    _need(w_gate_up, "w_gate_up", torch.bfloat16, 3)
    _need(w_down, "w_down", torch.bfloat16, 3)
    if residual is not None:
        _need(residual, "residual", torch.bfloat16, 2)
    if bias is not None:
        _need(bias, "bias", torch.float32, 1)
    T, H = x.shape
    E = w_router.shape[0]
    I = w_down.shape[2]
    dev = x.device
    ws_bytes = moe_forward_workspace_size(T, H, E, k, I)
    if workspace is None or workspace.numel() < ws_bytes:
        workspace = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    out = out if out is not None else torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    idx = torch.empty((T, k), dtype=torch.int32, device=dev) if return_routing else None
    tw = torch.empty((T, k), dtype=torch.float32, device=dev) if return_routing else None
    with torch.cuda.device(dev):
        _C.check(_C.lib().qmoe_moe_forward(
            _ptr(x), _ptr(w_router), _ptr(bias), _ptr(w_gate_up), _ptr(w_down), _ptr(residual),
            T, H, E, k, I, 1 if normalize else 0, _ptr(out), _ptr(idx), _ptr(tw),
            _ptr(workspace), workspace.numel(), _stream(dev)), "qmoe_moe_forward")
    if return_routing:
        return out, idx, tw
    return out


def moe_block_forward_workspace_size(T: int, H: int, E: int, k: int, I: int) -> int:
    return int(_C.lib().qmoe_moe_block_forward_workspace_size(T, H, E, k, I))


def moe_block_forward(x: torch.Tensor, residual: torch.Tensor, norm_weight: torch.Tensor, eps: float,
                      w_router: torch.Tensor, w_gate_up: torch.Tensor, w_down: torch.Tensor, k: int,
                      normalize: bool = True, bias: Optional[torch.Tensor] = None,
                      workspace: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
                      moe_in_out: Optional[torch.Tensor] = None, residual_out: Optional[torch.Tensor] = None,
                      return_routing: bool = False):
    """The decoder layer's post-attention add & norm + MoE block + residual
    add in one library call (qwen.py:423-430): s = bf16(x + residual),
    h = rmsnorm(s) * norm_weight, out = bf16(s + MoE(h)).  ``moe_in_out`` /
    ``residual_out`` receive h and s when given.  Returns out (T, H) bf16
    [, topk_idx (T, k) int32, topk_w (T, k) fp32]."""
    _need(x, "x", torch.bfloat16, 2)
    _need(residual, "residual", torch.bfloat16, 2)
    _need(norm_weight, "norm_weight", torch.float32, 1)
    _need(w_router, "w_router", torch.bfloat16, 2)
    _need(w_gate_up, "w_gate_up", torch.bfloat16, 3)
    _need(w_down, "w_down", torch.bfloat16, 3)
    for name, t in (("moe_in_out", moe_in_out), ("residual_out", residual_out)):
        if t is not None:
            _need(t, name, torch.bfloat16, 2)
    if bias is not None:
        _need(bias, "bias", torch.float32, 1)
    T, H = x.shape
    if tuple(residual.shape) != (T, H) or norm_weight.numel() != H:
        raise ValueError("residual must match x and norm_weight must have H elements")
    E = w_router.shape[0]
    I = w_down.shape[2]
    dev = x.device
    ws_bytes = moe_block_forward_workspace_size(T, H, E, k, I)
    if workspace is None or workspace.numel() < ws_bytes:
        workspace = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    out = out if out is not None else torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    idx = torch.empty((T, k), dtype=torch.int32, device=dev) if return_routing else None
    tw = torch.empty((T, k), dtype=torch.float32, device=dev) if return_routing else None
    with torch.cuda.device(dev):
        _C.check(_C.lib().qmoe_moe_block_forward(
            _ptr(x), _ptr(residual), _ptr(norm_weight), float(eps), _ptr(w_router), _ptr(bias), _ptr(w_gate_up),
            _ptr(w_down), T, H, E, k, I, 1 if normalize else 0, _ptr(out), _ptr(moe_in_out), _ptr(residual_out),
            _ptr(idx), _ptr(tw), _ptr(workspace), workspace.numel(), _stream(dev)), "qmoe_moe_block_forward")
    if return_routing:
        return out, idx, tw
    return out


# ----------------------------------------------------------------------------
# attention sub-layer
# ----------------------------------------------------------------------------

def linear(x: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None,
           split_ws: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out (T, N) bf16 = x (T, K) @ w (N, K)^T on the tcgen05 GEMM.  With
    ``split_ws`` (gateup_split_workspace) decode-sized calls may split K."""
    _need(x, "x", torch.bfloat16, 2)
    _need(w, "w", torch.bfloat16, 2)
    T, K = x.shape
    N = w.shape[0]
    if w.shape[1] != K:
        raise ValueError("w must be (N, K)")
    dev = x.device
    out = out if out is not None else torch.empty((T, N), dtype=torch.bfloat16, device=dev)
    with torch.cuda.device(dev):
        _C.check(_C.lib().qmoe_linear(_ptr(x), _ptr(w), T, K, N, _ptr(out), _ptr(split_ws),
                                      0 if split_ws is None else split_ws.numel() * split_ws.element_size(),
                                      _stream(dev)), "qmoe_linear")
    return out


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, residual: Optional[torch.Tensor] = None,
            out_dtype=torch.bfloat16):
    """RMSNorm over the last dim.  With ``residual`` returns (norm(x + residual),
    x + residual) -- the decoder layer's add & norm."""
    if x.dtype not in (torch.bfloat16, torch.float32):
        raise TypeError("x must be bf16 or fp32")
    _need(x, "x", None, 2)
    _need(weight, "weight", torch.float32, 1)
    rows, H = x.shape
    dev = x.device
    out = torch.empty((rows, H), dtype=out_dtype, device=dev)
    res_out = None
    if residual is not None:
        _need(residual, "residual", torch.bfloat16, 2)
        res_out = torch.empty((rows, H), dtype=torch.bfloat16, device=dev)
    with torch.cuda.device(dev):
        _C.check(_C.lib().qmoe_rmsnorm(_ptr(x), 1 if x.dtype == torch.float32 else 0, _ptr(residual),
                                       _ptr(weight), rows, H, float(eps), _ptr(out),
                                       1 if out_dtype == torch.float32 else 0, _ptr(res_out),
                                       _stream(dev)), "qmoe_rmsnorm")
    return out if residual is None else (out, res_out)


def qk_norm_rope(qkv: torch.Tensor, positions: torch.Tensor, q_norm_w: torch.Tensor,
                 k_norm_w: torch.Tensor, inv_freq: torch.Tensor, nh: int, nkv: int, eps: float,
                 k_cache: torch.Tensor, v_cache: torch.Tensor,
                 cache_slot: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Fused per-head QK-RMSNorm + RoPE; appends K/V into the caches.
    Returns q (T, nh, 128) bf16."""
    _need(qkv, "qkv", torch.bfloat16, 2)
    _need(positions, "positions", torch.int32, 1)
    _need(k_cache, "k_cache", torch.bfloat16, 4)
    _need(v_cache, "v_cache", torch.bfloat16, 4)
    if cache_slot is not None:
        _need(cache_slot, "cache_slot", torch.int32, 1)
    T = qkv.shape[0]
    hd = k_cache.shape[3]
    dev = qkv.device
    q = torch.empty((T, nh, hd), dtype=torch.bfloat16, device=dev)
    with torch.cuda.device(dev):
        _C.check(_C.lib().qmoe_qk_norm_rope(
            _ptr(qkv), _ptr(positions), _ptr(cache_slot), _ptr(q_norm_w), _ptr(k_norm_w), _ptr(inv_freq),
            T, nh, nkv, hd, float(eps), _ptr(q), _ptr(k_cache), _ptr(v_cache), k_cache.shape[0],
            k_cache.shape[2], _stream(dev)), "qmoe_qk_norm_rope")
    return q


def attention_prefill(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                      q_start: torch.Tensor, B: int, S: int, scale: Optional[float] = None,
                      cache_slot: Optional[torch.Tensor] = None,
                      kv_start: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Causal GQA over the cache; q (B*S, nh, 128) -> (B*S, nh*128) bf16.
    ``kv_start`` (B,) int32: left padding, cache rows before it are masked."""
    _need(q, "q", torch.bfloat16, 3)
    _need(q_start, "q_start", torch.int32, 1)
    if kv_start is not None:
        _need(kv_start, "kv_start", torch.int32, 1)
    nh, hd = q.shape[1], q.shape[2]
    nkv, max_seq = k_cache.shape[1], k_cache.shape[2]
    scale = hd ** -0.5 if scale is None else scale
    dev = q.device
    out = torch.empty((B * S, nh * hd), dtype=torch.bfloat16, device=dev)
    with torch.cuda.device(dev):
        _C.check(_C.lib().qmoe_attention_prefill(
            _ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(q_start), _ptr(cache_slot), _ptr(kv_start), B, S, nh,
            nkv, hd,
            k_cache.shape[0], max_seq, float(scale), _ptr(out), _stream(dev)), "qmoe_attention_prefill")
    return out


def attention_decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                     kv_len: torch.Tensor, max_len: int, scale: Optional[float] = None,
                     cache_slot: Optional[torch.Tensor] = None,
                     workspace: Optional[torch.Tensor] = None,
                     kv_start: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Split-KV flash-decode; q (B, nh, 128) -> (B, nh*128) bf16.
    ``kv_start`` (B,) int32: left padding, cache rows before it are masked."""
    _need(q, "q", torch.bfloat16, 3)
    _need(kv_len, "kv_len", torch.int32, 1)
    if kv_start is not None:
        _need(kv_start, "kv_start", torch.int32, 1)
    B, nh, hd = q.shape
    nkv, max_seq = k_cache.shape[1], k_cache.shape[2]
    scale = hd ** -0.5 if scale is None else scale
    dev = q.device
    lib = _C.lib()
    nsplit = int(lib.qmoe_attention_decode_splits(B, nkv, max_len))
    ws_bytes = int(lib.qmoe_attention_decode_workspace_size(B, nh, nsplit))
    if workspace is None or workspace.numel() < ws_bytes:
        workspace = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    out = torch.empty((B, nh * hd), dtype=torch.bfloat16, device=dev)
    with torch.cuda.device(dev):
        _C.check(lib.qmoe_attention_decode(
            _ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(kv_len), _ptr(cache_slot), _ptr(kv_start), B, nh, nkv, hd,
            k_cache.shape[0], max_seq, max_len, nsplit, float(scale), _ptr(out), _ptr(workspace),
            workspace.numel(), _stream(dev)),
            "qmoe_attention_decode")
    return out


# ----------------------------------------------------------------------------
# expert parallelism helpers
# ----------------------------------------------------------------------------

def routing_histogram(topk_idx: torch.Tensor, num_experts: int) -> torch.Tensor:
    """Per-chunk (8 tokens) expert histogram of caller-given routing."""
    _need(topk_idx, "topk_idx", torch.int32, 2)
    T, k = topk_idx.shape
    dev = topk_idx.device
    hist = torch.empty(((T + ROUTER_CHUNK - 1) // ROUTER_CHUNK, num_experts), dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        _C.check(_C.lib().qmoe_routing_histogram(_ptr(topk_idx), T, k, num_experts, _ptr(hist), _stream(dev)),
                 "qmoe_routing_histogram")
    return hist


def ep_pack(topk_idx: torch.Tensor, topk_w: torch.Tensor, x: torch.Tensor, e_local: int, n_ranks: int):
    """Rows grouped by destination rank.  Returns dict(send_counts (n_ranks,),
    send_x (T*k, H), send_expert (T*k,), send_w (T*k,), pair_pos (T, k))."""
    _need(topk_idx, "topk_idx", torch.int32, 2)
    _need(topk_w, "topk_w", torch.float32, 2)
    _need(x, "x", torch.bfloat16, 2)
    T, k = topk_idx.shape
    H = x.shape[1]
    dev = x.device
    R = T * k
    nchunks = (T + ROUTER_CHUNK - 1) // ROUTER_CHUNK
    hist = torch.empty((max(nchunks, 1), n_ranks), dtype=torch.int32, device=dev)
    out = dict(send_counts=torch.empty(n_ranks, dtype=torch.int32, device=dev),
               send_x=torch.empty((max(R, 1), H), dtype=torch.bfloat16, device=dev),
               send_expert=torch.empty(max(R, 1), dtype=torch.int32, device=dev),
               send_w=torch.empty(max(R, 1), dtype=torch.float32, device=dev),
               pair_pos=torch.empty((T, k), dtype=torch.int32, device=dev))
    with torch.cuda.device(dev):
        _C.check(_C.lib().qmoe_ep_pack(
            _ptr(topk_idx), _ptr(topk_w), _ptr(x), T, H, k, e_local, n_ranks, _ptr(hist),
            _ptr(out["send_counts"]), _ptr(out["send_x"]), _ptr(out["send_expert"]), _ptr(out["send_w"]),
            _ptr(out["pair_pos"]), _stream(dev)), "qmoe_ep_pack")
    return out


def ep_unpack(y_back: torch.Tensor, pair_pos: Optional[torch.Tensor], residual: Optional[torch.Tensor] = None,
              n_back: Optional[int] = None, T: Optional[int] = None, k: Optional[int] = None) -> torch.Tensor:
    """out[t] = residual[t] + sum_j y_back[pair_pos[t, j]] (fp32 sum).  With
    pair_pos None the rows are t*k + j (pass T and k)."""
    _need(y_back, "y_back", torch.bfloat16, 2)
    if pair_pos is not None:
        _need(pair_pos, "pair_pos", torch.int32, 2)
        T, k = pair_pos.shape
    elif T is None or k is None:
        raise ValueError("T and k are needed without pair_pos")
    H = y_back.shape[1]
    if residual is not None:
        _need(residual, "residual", torch.bfloat16, 2)
    dev = y_back.device
    out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    n_back = y_back.shape[0] if n_back is None else n_back
    with torch.cuda.device(dev):
        _C.check(_C.lib().qmoe_ep_unpack(_ptr(y_back), _ptr(pair_pos), _ptr(residual), T, H, k, n_back,
                                         _ptr(out), _stream(dev)), "qmoe_ep_unpack")
    return out
