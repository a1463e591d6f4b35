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

import ctypes
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


class PeerEPExchange:
    """Device buffers and peer mappings of the peer-memory expert-parallel
    exchange, shared by every EP block of a model (the blocks of a decoder
    stack run one after another on one stream, so one set of buffers serves
    all of them).

    Buffers (identical shapes on every rank, two parity halves each):
    token rows (P*max_tokens, H: one region per source rank, each token row
    sent once per destination), the expert-grouped receive list (meta) and
    receive rows (P*max_tokens*k, H), return rows (max_tokens*k, H), and the
    control block (counts + flags + the rank's step counter); plus the
    routing buffers of the local tokens.  The token, meta, return and control
    buffers are exported with CUDA IPC and every peer's copy is mapped here
    (``peer``: name -> int64 tensor of the P device pointers).  Creating one
    is collective over ``group``."""

    def __init__(self, cfg: Qwen3MoeConfig, max_tokens: int, group=None, device=None):
        from . import _C

        self._lib = _C.lib()
        self.cfg = cfg
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        E, H, I, k = cfg.num_experts, cfg.hidden_size, cfg.moe_intermediate_size, cfg.num_experts_per_tok
        if E % self.world:
            raise ValueError("num_experts must divide evenly over the ranks")
        self.E, self.H, self.I, self.k = E, H, I, k
        self.e_local = E // self.world
        self.max_tokens = max_tokens
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.device = dev
        self.cap = self.world * max_tokens * k          # receive rows per parity
        self.ret_rows = max_tokens * k                  # return rows per parity
        i32 = dict(dtype=torch.int32, device=dev)
        f32 = dict(dtype=torch.float32, device=dev)
        self.tok_rows = 2 * self.world * max_tokens     # token rows, both parities
        self.tok = torch.empty((self.tok_rows, H), dtype=torch.bfloat16, device=dev)
        self.recv_x = torch.empty((2 * self.cap, H), dtype=torch.bfloat16, device=dev)
        self.recv_meta = torch.zeros((2 * self.cap, 4), **i32)
        self.ret = torch.empty((2 * self.ret_rows, H), dtype=torch.bfloat16, device=dev)
        self.ctrl = torch.zeros(int(self._lib.qmoe_ep_ctrl_words(self.world, E)), **i32)
        self.dest_base = torch.empty(E, **i32)
        self.max_tiles = self.e_local + self.cap // 128 + 1
        self.tiles = torch.zeros(1 + 3 * self.max_tiles, **i32)
        self.recv_rows = torch.zeros(1, **i32)
        self.act = torch.empty((self.cap, I), dtype=torch.bfloat16, device=dev)
        # counters of the fused expert kernel (zeroed each step by the exchange)
        self.done = torch.zeros(self.max_tiles + 2, **i32)
        # routing / permutation buffers of the local tokens (max_tokens)
        R = max_tokens * k
        nchunks = (max_tokens + ops.ROUTER_CHUNK - 1) // ops.ROUTER_CHUNK
        self.topk_idx = torch.empty((max_tokens, k), **i32)
        self.topk_w = torch.empty((max_tokens, k), **f32)
        self.hist = torch.empty((max(nchunks, 1), E), **i32)
        self.counts = torch.empty(E, **i32)
        self.offsets = torch.empty(E + 1, **i32)
        self.row_token = torch.empty(max(R, 1), **i32)
        self.row_w = torch.empty(max(R, 1), **f32)
        self.slot_row = torch.empty((max_tokens, k), **i32)
        self.perm_tiles = torch.empty(1 + 3 * ops.max_tiles(R, E), **i32)
        self.route_barrier = torch.zeros(2, **i32)  # left zero by every completed route
        self.sms = torch.cuda.get_device_properties(dev).multi_processor_count
        torch.cuda.synchronize(dev)
        self._imported = []
        names = ("tok", "recv_meta", "ret", "ctrl")
        mine = {}
        for n in names:
            h = ctypes.create_string_buffer(64)
            off = ctypes.c_int64(0)
            _C.check(self._lib.qmoe_ipc_export(getattr(self, n).data_ptr(), h, ctypes.byref(off)),
                     "qmoe_ipc_export")
            mine[n] = (h.raw, off.value)
        gathered = [None] * self.world
        dist.all_gather_object(gathered, mine, group=group)
        ptrs = {n: [] for n in names}
        for r in range(self.world):
            for n in names:
                if r == self.rank:
                    ptrs[n].append(getattr(self, n).data_ptr())
                    continue
                handle, off = gathered[r][n]
                p = ctypes.c_void_p()
                base = ctypes.c_void_p()
                _C.check(self._lib.qmoe_ipc_import(handle, off, ctypes.byref(p), ctypes.byref(base)),
                         "qmoe_ipc_import")
                self._imported.append(base.value)
                ptrs[n].append(p.value)
        self.peer = {n: torch.tensor(ptrs[n], dtype=torch.int64, device=dev) for n in names}
        torch.cuda.synchronize(dev)
        dist.barrier(group=group)
        self.steps = 0        # steps issued (the device counter follows in stream order)

    def close(self):
        """Unmap the peers' buffers (all ranks should be done with the exchange)."""
        from . import _C

        torch.cuda.synchronize(self.device)
        for base in self._imported:
            _C.check(self._lib.qmoe_ipc_close(base), "qmoe_ipc_close")
        self._imported = []

    def launches_per_step(self, T: int) -> int:
        """Kernels one step launches: route (router + permutation: one launch
        up to one router chunk per SM and T > 64, else router + scan +
        scatter), count exchange, dispatch, signal + wait + expand, experts,
        signal + wait + unpack."""
        nchunks = (T + ops.ROUTER_CHUNK - 1) // ops.ROUTER_CHUNK
        one = T > ops.ROUTER_SMALL_MAX_T and nchunks <= self.sms
        return (1 if one else 3) + 5


class PeerExpertParallelMoE(nn.Module):
    """Expert-parallel block whose exchange runs through peer memory inside
    one node (CUDA IPC mappings over NVLink / NVSwitch) with no host sync, so
    a step is a fixed sequence of stream-ordered kernels.

    Kernels per step: router, permutation (counts / offsets / slot rows),
    count exchange, dispatch (each token row once to every rank owning one
    of its experts, plus a receive-list entry per (token, slot), grouped by
    expert), signal/wait and the local expansion of the receive list into
    expert-grouped rows, gate/up + down in one persistent kernel on those
    rows whose down epilogue stores the weighted rows into the source ranks'
    return buffers, signal/wait and the unpack of the returned rows.

    The buffers live in a ``PeerEPExchange`` (``exchange``): pass one shared
    exchange to every block of a decoder stack, or let the block create its
    own (``max_tokens`` sizes it).  The kernels take the step's epoch from the
    device-side step counter, so each parity's step has fixed arguments:
    ``capture`` records one CUDA graph per parity and ``replay`` runs the next
    step with no host work beyond the graph launch.  Every rank must run the
    same steps in the same order (each step's exchange waits for every peer's
    step of the same number); a rank that runs an extra step waits out the
    bounded wait limit and records device error 5."""

    expert_parallel = True

    def __init__(self, cfg: Qwen3MoeConfig, router_weight: torch.Tensor, local: MoEWeights,
                 max_tokens: Optional[int] = None, group=None, exchange: Optional[PeerEPExchange] = None):
        super().__init__()
        from . import _C

        self._lib = _C.lib()
        if exchange is None:
            if max_tokens is None:
                raise ValueError("give max_tokens or a shared exchange")
            exchange = PeerEPExchange(cfg, max_tokens, group=group, device=router_weight.device)
            self._owns_exchange = True
        else:
            self._owns_exchange = False
        self.x = exchange
        self.cfg = cfg
        self.group = exchange.group
        self.world, self.rank = exchange.world, exchange.rank
        self.E, self.H, self.I, self.k = exchange.E, exchange.H, exchange.I, exchange.k
        self.e_local = exchange.e_local
        if local.gate_up.shape[0] != self.e_local:
            raise ValueError("local expert weights do not match E / world")
        self.router_weight = router_weight
        self.local = local
        self.router_bias: Optional[torch.Tensor] = None
        self.max_tokens = exchange.max_tokens
        self.device = exchange.device
        self._graphs = None   # (graph of parity 0, graph of parity 1)
        self._static = None   # per parity: (x, residual, out)

    # views of the shared exchange (read by callers and tests)
    @property
    def recv_rows(self) -> torch.Tensor:
        return self.x.recv_rows

    @property
    def topk_idx(self) -> torch.Tensor:
        return self.x.topk_idx

    @property
    def steps(self) -> int:
        return self.x.steps

    def close(self):
        """Drop the graphs; unmap the peers' buffers if this block owns its
        exchange (all ranks should be done with the exchange)."""
        torch.cuda.synchronize(self.device)
        self._graphs = None
        if self._owns_exchange:
            self.x.close()

    STAGES = ("route", "exchange", "dispatch", "wait_expand", "experts", "return")

    def launches_per_step(self, T: int) -> int:
        return self.x.launches_per_step(T)

    def _issue(self, x: torch.Tensor, residual: Optional[torch.Tensor], out: torch.Tensor, par: int,
               events=None) -> None:
        """The step's kernels for parity `par` on the current stream (epochs
        from the device step counter).  ``events``: len(STAGES) + 1 CUDA
        events recorded before the first kernel and after each stage."""
        from . import _C

        def mark(i):
            if events is not None:
                events[i].record()

        mark(0)
        X = self.x
        T = x.shape[0]
        H, E, k, I = self.H, self.E, self.k, self.I
        lib, pt = self._lib, ops._ptr
        s = torch.cuda.current_stream(self.device).cuda_stream
        # router + permutation of the local tokens (one launch at prefill sizes)
        _C.check(lib.qmoe_route_permute(pt(x), pt(self.router_weight), pt(self.router_bias), T, H, E, k, 1,
                                        pt(X.topk_idx), pt(X.topk_w), pt(X.hist), pt(X.counts),
                                        pt(X.offsets), pt(X.row_token), pt(X.row_w), pt(X.slot_row),
                                        pt(X.perm_tiles), None, None, None, 0, pt(X.route_barrier), s),
                 "qmoe_route_permute")
        mark(1)
        _C.check(lib.qmoe_ep_exchange_counts(
            pt(X.counts), pt(X.peer["ctrl"]), pt(X.ctrl), self.rank, self.world, E, self.e_local,
            par, 0, pt(X.dest_base), pt(X.tiles), X.max_tiles, pt(X.recv_rows), X.cap,
            pt(X.done), X.max_tiles + 2, s), "qmoe_ep_exchange_counts")
        mark(2)
        _C.check(lib.qmoe_ep_dispatch(
            pt(x), pt(X.topk_idx), pt(X.topk_w), pt(X.slot_row), pt(X.offsets), pt(X.dest_base),
            pt(X.peer["tok"]), pt(X.peer["recv_meta"]), T, k, H, self.e_local, self.rank, self.world, par,
            X.cap, X.max_tokens, s), "qmoe_ep_dispatch")
        mark(3)
        recv_x = X.recv_x[par * X.cap:(par + 1) * X.cap]
        _C.check(lib.qmoe_ep_wait_expand(
            pt(X.peer["ctrl"]), pt(X.ctrl), self.world, E, self.rank, par, 0, pt(X.tok), X.tok_rows,
            pt(X.recv_meta[par * X.cap:]), pt(recv_x), pt(X.recv_rows), X.cap, H, s), "qmoe_ep_wait_expand")
        mark(4)
        # gate/up + down in one persistent kernel; its down epilogue stores
        # each weighted row into the source rank's return buffer
        _C.check(lib.qmoe_moe_experts_return(
            pt(recv_x), pt(self.local.gate_up), pt(self.local.down), pt(X.tiles), X.max_tiles,
            pt(X.recv_meta[par * X.cap:]), pt(X.peer["ret"]), par * X.ret_rows, X.ret_rows,
            self.world, X.cap, H, I, self.e_local, pt(X.act), pt(X.done), s), "qmoe_moe_experts_return")
        mark(5)
        # "your rows are back" flags, the wait for every peer's, and the
        # fp32 sum of each token's k returned rows (+ residual), one launch
        y_back = X.ret[par * X.ret_rows:]
        _C.check(lib.qmoe_ep_wait_unpack(pt(X.peer["ctrl"]), pt(X.ctrl), self.world, E, self.rank, par, 0,
                                         pt(y_back), pt(residual), T, H, k, pt(out), s), "qmoe_ep_wait_unpack")
        mark(6)

    def forward(self, hidden_states: torch.Tensor, residual: Optional[torch.Tensor] = None,
                events=None) -> torch.Tensor:
        """out = MoE(hidden_states) [+ residual], in the input's shape (bf16)."""
        shape = hidden_states.shape
        x = hidden_states.reshape(-1, self.H).to(torch.bfloat16).contiguous()
        T = x.shape[0]
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed max_tokens={self.max_tokens} of the EP buffers")
        res = None if residual is None else residual.reshape(-1, self.H).to(torch.bfloat16).contiguous()
        out = torch.empty((T, self.H), dtype=torch.bfloat16, device=self.device)
        self.x.steps += 1
        self._issue(x, res, out, self.x.steps & 1, events)
        return out.reshape(shape)

    def capture(self, hidden_states: torch.Tensor, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Record one CUDA graph per parity, each over its own static copies
        of the inputs and its own output, so a caller can upload the next
        step's input (``static_input()``) and download the last step's output
        while a step runs.  Returns the output of the next replay.  Every rank
        captures with the same shapes (no kernel runs during capture)."""
        x = hidden_states.reshape(-1, self.H).to(torch.bfloat16).contiguous()
        T = x.shape[0]
        res = None if residual is None else residual.reshape(-1, self.H).to(torch.bfloat16).contiguous()
        graphs, static = [], []
        for par in (0, 1):
            xs = x.clone()
            rs = None if res is None else res.clone()
            out = torch.empty((T, self.H), dtype=torch.bfloat16, device=self.device)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._issue(xs, rs, out, par)
            graphs.append(g)
            static.append((xs, rs, out))
        self._graphs = tuple(graphs)
        self._static = tuple(static)
        return self._static[(self.x.steps + 1) & 1][2]

    def replay(self) -> torch.Tensor:
        """Run the next step from the captured graphs; returns that step's
        output buffer (overwritten again two steps later)."""
        if self._graphs is None:
            raise RuntimeError("capture() first")
        self.x.steps += 1
        par = self.x.steps & 1
        self._graphs[par].replay()
        return self._static[par][2]

    def static_input(self, ahead: int = 1) -> torch.Tensor:
        """The static input buffer the ``ahead``-th next ``replay`` reads
        (1: the next one)."""
        return self._static[(self.x.steps + ahead) & 1][0]

    def static_output(self, ahead: int = 1) -> torch.Tensor:
        return self._static[(self.x.steps + ahead) & 1][2]
