"""K2 permutation (bit-exact), K3a / K3b grouped GEMMs and the fused MoE block
against the CPU oracle.  Activation tolerance: max relative error <= 2e-2
(normwise: max|gpu - oracle| / max|oracle|), the north-star bar."""
import numpy as np
import pytest
import torch

from helpers import MAX_REL, activations, max_rel_err, moe_weights, to_f32_np

pytestmark = pytest.mark.gpu


def _routing(cuda_dev, x, wr, k):
    from nki_moe_7013_b200 import ops

    idx, w, hist = ops.router_topk(x, wr, k, return_hist=True)
    return idx, w, hist


@pytest.mark.parametrize("T,H,E,k", [(1, 2048, 128, 8), (5, 256, 32, 4), (128, 2048, 128, 8),
                                     (1024, 2048, 128, 8), (37, 512, 64, 8)])
def test_permute_bit_exact(cuda_dev, oracle, T, H, E, k):
    from nki_moe_7013_b200 import ops

    wr = moe_weights(2, E, H, 128, cuda_dev)[0]
    x = activations(2, T, H, cuda_dev)
    idx, w, hist = _routing(cuda_dev, x, wr, k)
    acc = torch.full((T, H), 7.0, dtype=torch.float32, device=cuda_dev)
    p = ops.moe_permute(idx, w, hist, E, x=x, gather=True, acc_zero=acc)
    torch.cuda.synchronize()
    ref = oracle.permute(idx.cpu().numpy(), E)
    np.testing.assert_array_equal(p["counts"].cpu().numpy(), ref["counts"])
    np.testing.assert_array_equal(p["offsets"].cpu().numpy(), ref["offsets"])
    np.testing.assert_array_equal(p["row_token"].cpu().numpy(), ref["row_token"])
    np.testing.assert_array_equal(p["slot_row"].cpu().numpy(), ref["slot_row"])
    wn = w.cpu().numpy()
    np.testing.assert_array_equal(p["row_w"].cpu().numpy(),
                                  wn.reshape(-1)[np.argsort(ref["slot_row"].reshape(-1))])
    # x_perm rows are the gathered token rows
    xp = p["x_perm"].cpu()
    assert torch.equal(xp, x.cpu()[torch.from_numpy(ref["row_token"]).long()])
    assert torch.count_nonzero(acc).item() == 0
    # tile list: every expert's rows cut into 128-row tiles in expert order
    tiles = p["tiles"].cpu().numpy()
    mt = p["max_tiles"]
    nt = tiles[0]
    exp_tiles = []
    for e in range(E):
        n = int(ref["counts"][e])
        for i in range(0, n, 128):
            exp_tiles.append((e, int(ref["offsets"][e]) + i, min(128, n - i)))
    got = list(zip(tiles[1:1 + nt], tiles[1 + mt:1 + mt + nt], tiles[1 + 2 * mt:1 + 2 * mt + nt]))
    assert [tuple(map(int, g)) for g in got] == exp_tiles


@pytest.mark.parametrize("T,H,E,k,I", [(1, 2048, 128, 8, 768), (128, 2048, 128, 8, 768),
                                       (16, 256, 32, 4, 128), (300, 512, 32, 8, 256)])
def test_grouped_gemms_vs_oracle(cuda_dev, oracle, T, H, E, k, I):
    from nki_moe_7013_b200 import ops

    wr, wgu, wd = moe_weights(3, E, H, I, cuda_dev)
    x = activations(3, T, H, cuda_dev)
    idx, w, hist = _routing(cuda_dev, x, wr, k)
    acc = torch.empty((T, H), dtype=torch.float32, device=cuda_dev)
    p = ops.moe_permute(idx, w, hist, E, x=x, gather=True, acc_zero=acc)
    act = ops.grouped_gemm_gateup_swiglu(p["x_perm"], wgu, p["tiles"], p["max_tiles"])
    # the gathered form (TMA gather4 straight from x) gives the same activations
    act_g = ops.grouped_gemm_gateup_swiglu(x, wgu, p["tiles"], p["max_tiles"], gather_rows=p["row_token"])
    ops.grouped_gemm_down_combine(act, wd, p["tiles"], p["max_tiles"], p["row_token"], p["row_w"], acc)
    torch.cuda.synchronize()
    assert torch.equal(act, act_g)
    from nki_moe_7013_b200 import _C

    assert _C.device_error() == 0
    ref_out, inter = oracle.moe_block(x.cpu(), wr.cpu(), wgu.cpu(), wd.cpu(), k,
                                      return_intermediates=True)
    assert np.array_equal(idx.cpu().numpy(), inter["topk_idx"])
    err_act = max_rel_err(to_f32_np(act), inter["act"])
    assert err_act <= MAX_REL, f"act max rel err {err_act:.3e}"
    err_out = max_rel_err(acc.cpu().numpy(), ref_out)
    assert err_out <= MAX_REL, f"combine max rel err {err_out:.3e}"


@pytest.mark.parametrize("T,H,E,k,I", [(1, 2048, 128, 8, 768), (2, 2048, 128, 8, 768), (1, 256, 32, 4, 128),
                                       (3, 512, 32, 8, 256), (16, 2048, 128, 8, 768)])
def test_gateup_split_k(cuda_dev, oracle, T, H, E, k, I):
    """Decode-sized gate/up with a split-K scratch: same activations as the
    unsplit kernel up to fp32 summation order, run-to-run identical, and the
    scratch's arrival counters back at zero after every launch."""
    from nki_moe_7013_b200 import _C, ops

    wr, wgu, wd = moe_weights(4, E, H, I, cuda_dev)
    x = activations(4 + T, T, H, cuda_dev)
    idx, w, hist = _routing(cuda_dev, x, wr, k)
    p = ops.moe_permute(idx, w, hist, E, x=x, gather=False)
    ws = ops.gateup_split_workspace(cuda_dev)
    plain = ops.grouped_gemm_gateup_swiglu(x, wgu, p["tiles"], p["max_tiles"], gather_rows=p["row_token"])
    runs = [ops.grouped_gemm_gateup_swiglu(x, wgu, p["tiles"], p["max_tiles"], gather_rows=p["row_token"],
                                           split_ws=ws) for _ in range(3)]
    torch.cuda.synchronize()
    assert _C.device_error() == 0
    assert torch.equal(runs[0], runs[1]) and torch.equal(runs[0], runs[2])
    n_slots_floats = 256 * 2 * 16 * 128
    counters = ws.view(torch.int32)[n_slots_floats:n_slots_floats + 256]
    assert torch.count_nonzero(counters).item() == 0
    assert max_rel_err(to_f32_np(runs[0]), to_f32_np(plain)) <= 1e-2
    _, inter = oracle.moe_block(x.cpu(), wr.cpu(), wgu.cpu(), wd.cpu(), k, return_intermediates=True)
    err = max_rel_err(to_f32_np(runs[0]), inter["act"])
    assert err <= MAX_REL, f"split-K act max rel err {err:.3e}"


@pytest.mark.parametrize("T,gather", [(1, True), (4, True), (16, True), (9, False)])
def test_small_tile_configuration(cuda_dev, oracle, T, gather):
    """Tiles of <= 16 rows (max_tile_rows <= 16) run the deeper-pipeline
    configuration of both GEMMs; results equal the normal configuration's
    (same k order, same epilogue), and a tile larger than the promised bound
    is refused on the device with error 4 instead of being computed."""
    from nki_moe_7013_b200 import _C, ops

    H, E, k, I = 2048, 128, 8, 768
    wr, wgu, wd = moe_weights(5, E, H, I, cuda_dev)
    x = activations(60 + T, T, H, cuda_dev)
    idx, w, hist = _routing(cuda_dev, x, wr, k)
    p = ops.moe_permute(idx, w, hist, E, x=x, gather=not gather)
    src = dict(x=x, gather_rows=p["row_token"]) if gather else dict(x=p["x_perm"])
    outs = []
    for rows in (128, T):
        act = ops.grouped_gemm_gateup_swiglu(src["x"], wgu, p["tiles"], p["max_tiles"],
                                             gather_rows=src.get("gather_rows"), max_tile_rows=rows)
        acc = torch.zeros((T, H), dtype=torch.float32, device=cuda_dev)
        # the small configuration also streams weights before its dependency
        # wait (the tile list predates the gate/up launch)
        ops.grouped_gemm_down_combine(act, wd, p["tiles"], p["max_tiles"], p["row_token"], p["row_w"], acc,
                                      max_tile_rows=rows, tiles_ready=rows < 128)
        outs.append((act, acc))
    torch.cuda.synchronize()
    assert _C.device_error() == 0
    assert torch.equal(outs[0][0], outs[1][0])
    assert max_rel_err(outs[1][1].cpu().numpy(), outs[0][1].cpu().numpy()) <= 1e-5
    ref_out, _ = oracle.moe_block(x.cpu(), wr.cpu(), wgu.cpu(), wd.cpu(), k, return_intermediates=True)
    assert max_rel_err(outs[1][1].cpu().numpy(), ref_out) <= MAX_REL


def test_small_tile_configuration_refuses_larger_tiles(cuda_dev):
    """A caller that promises tiles of <= 16 rows but passes a 32-row tile
    gets device error 4 and untouched outputs, never an overrun stage."""
    from nki_moe_7013_b200 import _C, ops

    H, E, k, I, T = 2048, 128, 8, 768, 32
    wr, wgu, wd = moe_weights(6, E, H, I, cuda_dev)
    x = activations(6, 1, H, cuda_dev).repeat(T, 1).contiguous()  # identical tokens: 32 rows per expert
    idx, w, hist = _routing(cuda_dev, x, wr, k)
    p = ops.moe_permute(idx, w, hist, E, x=x, gather=False)
    assert int(p["counts"].max()) == T
    act = torch.full((T * k, I), 7.0, dtype=torch.bfloat16, device=cuda_dev)
    ops.grouped_gemm_gateup_swiglu(x, wgu, p["tiles"], p["max_tiles"], gather_rows=p["row_token"],
                                   max_tile_rows=16, out=act)
    torch.cuda.synchronize()
    assert _C.device_error() == 4
    assert bool((act == 7.0).all())
    acc = torch.full((T, H), 5.0, dtype=torch.float32, device=cuda_dev)
    ops.grouped_gemm_down_combine(act, wd, p["tiles"], p["max_tiles"], p["row_token"], p["row_w"], acc,
                                  max_tile_rows=16, tiles_ready=True)
    torch.cuda.synchronize()
    assert _C.device_error() == 4
    assert bool((acc == 5.0).all())


def test_oversized_tiles_refused(cuda_dev):
    """A tile list with a tile of more than 128 rows: the grouped GEMMs refuse
    the launch (device error 4, outputs untouched); the fused kernel skips
    that tile's units (device error 4) and completes every other tile -- no
    stage is ever overrun."""
    from nki_moe_7013_b200 import _C, ops

    H, E, k, I, T = 2048, 128, 8, 768, 1024
    wr, wgu, wd = moe_weights(4, E, H, I, cuda_dev)
    x = activations(4, T, H, cuda_dev)
    idx, w, hist = _routing(cuda_dev, x, wr, k)
    p = ops.moe_permute(idx, w, hist, E, x=x, gather=True)
    mt = p["max_tiles"]
    nt = int(p["tiles"][0])
    bad = p["tiles"].clone()
    bad[1 + 2 * mt] = 200  # tile 0 (rows from 0) claims 200 rows
    act = torch.full((T * k, I), 7.0, dtype=torch.bfloat16, device=cuda_dev)
    ops.grouped_gemm_gateup_swiglu(p["x_perm"], wgu, bad, mt, out=act)
    torch.cuda.synchronize()
    assert _C.device_error() == 4
    assert bool((act == 7.0).all())
    acc = torch.zeros((T, H), dtype=torch.float32, device=cuda_dev)
    ops.moe_experts(p["x_perm"], wgu, wd, bad, mt, p["row_token"], p["row_w"], acc, p["done"], act=act)
    torch.cuda.synchronize()
    assert _C.device_error() == 4
    assert int(p["done"][0]) == 0
    assert bool((p["done"][1:nt] == I // 128).all())


@pytest.mark.parametrize("T,H,E,k,I", [(65, 2048, 128, 8, 768), (1024, 2048, 128, 8, 768), (300, 512, 32, 8, 256),
                                       (2048, 256, 64, 4, 128), (777, 1024, 256, 8, 384)])
def test_moe_experts_fused_matches_separate_gemms(cuda_dev, oracle, T, H, E, k, I):
    """The persistent gate/up -> down kernel gives the separate kernels'
    activations bit for bit and the same combine (fp32 atomics: order only)."""
    from nki_moe_7013_b200 import _C, ops

    wr, wgu, wd = moe_weights(7, E, H, I, cuda_dev)
    x = activations(70 + T, T, H, cuda_dev)
    idx, w, hist = _routing(cuda_dev, x, wr, k)
    acc_f = torch.empty((T, H), dtype=torch.float32, device=cuda_dev)
    p = ops.moe_permute(idx, w, hist, E, x=x, gather=True, acc_zero=acc_f)
    act_f = torch.empty((T * k, I), dtype=torch.bfloat16, device=cuda_dev)
    ops.moe_experts(p["x_perm"], wgu, wd, p["tiles"], p["max_tiles"], p["row_token"], p["row_w"], acc_f,
                    p["done"], act=act_f)
    act = ops.grouped_gemm_gateup_swiglu(p["x_perm"], wgu, p["tiles"], p["max_tiles"])
    acc = torch.zeros((T, H), dtype=torch.float32, device=cuda_dev)
    ops.grouped_gemm_down_combine(act, wd, p["tiles"], p["max_tiles"], p["row_token"], p["row_w"], acc)
    # the same kernel gathering token rows itself (no permuted copy)
    done_g = torch.zeros_like(p["done"])
    acc_g = torch.zeros((T, H), dtype=torch.float32, device=cuda_dev)
    act_g = torch.empty_like(act_f)
    ops.moe_experts(x, wgu, wd, p["tiles"], p["max_tiles"], p["row_token"], p["row_w"], acc_g, done_g, act=act_g,
                    gather_rows=p["row_token"])
    torch.cuda.synchronize()
    assert _C.device_error() == 0
    assert torch.equal(act_f, act)
    assert torch.equal(act_g, act)
    assert max_rel_err(acc_f.cpu().numpy(), acc.cpu().numpy()) <= 1e-5
    assert max_rel_err(acc_g.cpu().numpy(), acc.cpu().numpy()) <= 1e-5
    # every tile's counter reached the number of gate/up feature blocks
    nt = int(p["tiles"][0])
    assert bool((p["done"][:nt] == I // 128).all())
    ref_out, _ = oracle.moe_block(x.cpu(), wr.cpu(), wgu.cpu(), wd.cpu(), k, return_intermediates=True)
    assert max_rel_err(acc_f.cpu().numpy(), ref_out) <= MAX_REL


@pytest.mark.parametrize("T", [1, 2, 5, 8, 10, 40, 64, 128, 1024])  # 5 / 10 / 40: spec-verify batches
def test_moe_forward_cfg0_shapes(cuda_dev, oracle, T):
    from nki_moe_7013_b200 import ops

    H, E, k, I = 2048, 128, 8, 768
    wr, wgu, wd = moe_weights(0, E, H, I, cuda_dev)
    x = activations(0, T, H, cuda_dev)
    out, idx, tw = ops.moe_forward(x, wr, wgu, wd, k, return_routing=True)
    torch.cuda.synchronize()
    ref_out, inter = oracle.moe_block(x.cpu(), wr.cpu(), wgu.cpu(), wd.cpu(), k,
                                      return_intermediates=True)
    assert np.array_equal(idx.cpu().numpy(), inter["topk_idx"])
    np.testing.assert_allclose(tw.cpu().numpy(), inter["topk_w"], rtol=2e-6, atol=1e-7)
    err = max_rel_err(to_f32_np(out), oracle.round_to_bf16(ref_out))
    assert err <= MAX_REL, f"moe_forward max rel err {err:.3e}"


@pytest.mark.parametrize("T,H,E,k,I", [(1184, 256, 32, 4, 128), (300, 1024, 256, 8, 256), (65, 512, 64, 2, 128),
                                       (700, 4096, 128, 8, 128), (1185, 512, 32, 8, 128)])
def test_moe_forward_route_permute_shapes(cuda_dev, oracle, T, H, E, k, I):
    """Prefill batches of at most one router chunk per SM route and permute in
    one launch (grid-wide barrier); 1185 tokens (149 chunks) take the separate
    kernels.  Routing bit-exact, output within the activation tolerance."""
    from nki_moe_7013_b200 import _C, ops

    wr, wgu, wd = moe_weights(12, E, H, I, cuda_dev)
    x = activations(12 + T, T, H, cuda_dev)
    out, idx, tw = ops.moe_forward(x, wr, wgu, wd, k, return_routing=True)
    torch.cuda.synchronize()
    assert _C.device_error() == 0
    ref_out, inter = oracle.moe_block(x.cpu(), wr.cpu(), wgu.cpu(), wd.cpu(), k, return_intermediates=True)
    assert np.array_equal(idx.cpu().numpy(), inter["topk_idx"])
    np.testing.assert_allclose(tw.cpu().numpy(), inter["topk_w"], rtol=2e-6, atol=1e-7)
    assert max_rel_err(to_f32_np(out), oracle.round_to_bf16(ref_out)) <= MAX_REL


def test_moe_forward_residual_and_determinism(cuda_dev, oracle):
    from nki_moe_7013_b200 import ops

    T, H, E, k, I = 96, 2048, 128, 8, 768
    wr, wgu, wd = moe_weights(4, E, H, I, cuda_dev)
    x = activations(4, T, H, cuda_dev)
    res = activations(5, T, H, cuda_dev)
    out1, idx1, _ = ops.moe_forward(x, wr, wgu, wd, k, residual=res, return_routing=True)
    out2, idx2, _ = ops.moe_forward(x, wr, wgu, wd, k, residual=res, return_routing=True)
    torch.cuda.synchronize()
    assert torch.equal(idx1, idx2)  # routing is bit-reproducible
    ref = oracle.moe_block(x.cpu(), wr.cpu(), wgu.cpu(), wd.cpu(), k) + to_f32_np(res)
    err = max_rel_err(to_f32_np(out1), ref)
    assert err <= MAX_REL


def test_moe_forward_zipf_skew(cuda_dev, oracle):
    """Config-4-style skew: Zipf(1.2) expert popularity through a router bias."""
    from nki_moe_7013_b200 import ops
    from nki_moe_7013_b200.synth import zipf_expert_bias

    T, H, E, k, I = 2048, 2048, 128, 8, 768
    wr, wgu, wd = moe_weights(6, E, H, I, cuda_dev)
    x = activations(6, T, H, cuda_dev)
    bias = zipf_expert_bias(0, E).to(cuda_dev)
    out, idx, _ = ops.moe_forward(x, wr, wgu, wd, k, bias=bias, return_routing=True)
    torch.cuda.synchronize()
    ref_out, inter = oracle.moe_block(x.cpu(), wr.cpu(), wgu.cpu(), wd.cpu(), k,
                                      bias=bias.cpu().numpy(), return_intermediates=True)
    assert np.array_equal(idx.cpu().numpy(), inter["topk_idx"])
    counts = np.bincount(inter["topk_idx"].reshape(-1), minlength=E)
    assert counts.max() > 4 * counts.mean()  # the skew is real: several 128-row tiles per hot expert
    err = max_rel_err(to_f32_np(out), oracle.round_to_bf16(ref_out))
    assert err <= MAX_REL


@pytest.mark.parametrize("T,H,E,k,I", [(1, 2048, 128, 8, 768), (2, 2048, 128, 8, 768), (3, 2048, 128, 8, 768),
                                       (16, 2048, 128, 8, 768), (17, 2048, 128, 8, 768), (24, 2048, 128, 8, 768),
                                       (64, 2048, 128, 8, 768), (65, 2048, 128, 8, 768), (300, 2048, 128, 8, 768),
                                       (1200, 2048, 128, 8, 768), (5, 1024, 256, 8, 256), (40, 1024, 256, 8, 256)])
def test_forward_stays_inside_its_workspace(cuda_dev, T, H, E, k, I):
    """qmoe_moe_forward writes nothing past the workspace size it reports, on
    every routing path (decode route kernel, one-launch route + permutation,
    separate router and permutation kernels): a guard of pattern bytes after
    the workspace stays untouched.  (The one-launch route's two barrier words
    once sat outside the layout for 17-64 tokens and zeroed the 8 bytes after
    the workspace.)"""
    from nki_moe_7013_b200 import _C, ops

    guard = 1 << 16
    wr, wgu, wd = moe_weights(95 + T, E, H, I, cuda_dev)
    x = activations(95 + T, T, H, cuda_dev)
    res = activations(96 + T, T, H, cuda_dev)
    nb = ops.moe_forward_workspace_size(T, H, E, k, I)
    ws = torch.full((nb + guard,), 0x5A, dtype=torch.uint8, device=cuda_dev)
    out = ops.moe_forward(x, wr, wgu, wd, k, residual=res, workspace=ws)
    torch.cuda.synchronize()
    assert _C.device_error() == 0
    assert int((ws[nb:] != 0x5A).sum()) == 0, "moe_forward wrote past its workspace"
    assert torch.isfinite(out.float()).all()


@pytest.mark.parametrize("T", [1, 2, 3, 17, 24, 40, 100, 300])
def test_moe_forward_repeatable_on_dirty_workspace(cuda_dev, T):
    """Repeated forwards on workspaces pre-filled with NaN, huge and zero
    bytes, routing kept in the workspace: every output within one bf16 ulp of
    the first (the combine adds in arrival order) and of a call that returns
    its routing.  Catches reads of unwritten scratch and cross-CTA ordering
    faults."""
    from helpers import assert_within_one_ulp
    from nki_moe_7013_b200 import _C, ops

    H, E, k, I = 2048, 128, 8, 768
    wr, wgu, wd = moe_weights(90 + T, E, H, I, cuda_dev)
    x = activations(90 + T, T, H, cuda_dev)
    res = activations(91 + T, T, H, cuda_dev)
    ref, _, _ = ops.moe_forward(x, wr, wgu, wd, k, residual=res, return_routing=True)
    nb = ops.moe_forward_workspace_size(T, H, E, k, I)
    for i, fill in enumerate([0xFF, 0x7F, 0x00, 0x3F] * 3):
        ws = torch.full((nb,), fill, dtype=torch.uint8, device=cuda_dev)
        out = ops.moe_forward(x, wr, wgu, wd, k, residual=res, workspace=ws)
        torch.cuda.synchronize()
        assert not torch.isnan(out).any()
        assert_within_one_ulp(out, ref, f"T={T} run {i}")
    assert _C.device_error() == 0


@pytest.mark.parametrize("T,H,E,k,I", [(1, 2048, 128, 8, 768), (2, 2048, 128, 8, 768), (1, 4096, 64, 8, 256),
                                       (2, 1024, 32, 32, 512), (2, 2048, 256, 8, 768)])
def test_decode_expert_rows_match_tensor_core_path(cuda_dev, oracle, T, H, E, k, I):
    """1-2 token forwards run the expert GEMMs on the CUDA cores (the down
    kernel also adds the residual and writes the output): routing identical,
    output within the activation tolerance of the oracle and of the
    tensor-core kernels on the same routing (MoEPlan's per-stage path), and
    run-to-run identical (no atomics)."""
    from nki_moe_7013_b200 import _C, ops
    from nki_moe_7013_b200.moe import MoEPlan, MoEWeights

    wr, wgu, wd = moe_weights(110 + T, E, H, I, cuda_dev)
    x = activations(110 + T, T, H, cuda_dev)
    res = activations(111 + T, T, H, cuda_dev)
    outs = [ops.moe_forward(x, wr, wgu, wd, k, residual=res, return_routing=True) for _ in range(2)]
    plan = MoEPlan(MoEWeights(wr, wgu, wd), T, k)
    staged = torch.empty((T, H), dtype=torch.bfloat16, device=cuda_dev)
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(len(plan.stages) + 1)]
    plan.run(x, staged, residual=res, events=evs)
    torch.cuda.synchronize()
    assert _C.device_error() == 0
    out, idx, tw = outs[0]
    assert torch.equal(out, outs[1][0])
    assert torch.equal(idx, plan.topk_idx) and torch.equal(tw, plan.topk_w)
    assert max_rel_err(to_f32_np(out), to_f32_np(staged)) <= 1e-2
    ref = oracle.moe_block(x.cpu(), wr.cpu(), wgu.cpu(), wd.cpu(), k) + to_f32_np(res)
    assert max_rel_err(to_f32_np(out), ref) <= MAX_REL


@pytest.mark.parametrize("H,E,k,I", [(2048, 128, 8, 768), (1024, 64, 8, 512), (2048, 32, 4, 768)])
def test_one_token_forward_matches_row_of_two_token_forward(cuda_dev, H, E, k, I):
    """The decode expert kernels sum each token's expert outputs in ascending
    expert order with no atomics, so a token's result does not depend on the
    batch around it: a one-token forward equals row 0 of a two-token forward
    bit for bit -- with and without a residual, call after call."""
    from nki_moe_7013_b200 import _C, ops

    wr, wgu, wd = moe_weights(130 + E, E, H, I, cuda_dev)
    x2 = activations(131, 2, H, cuda_dev)
    res2 = activations(132, 2, H, cuda_dev)
    two, idx2, _ = ops.moe_forward(x2, wr, wgu, wd, k, residual=res2, return_routing=True)
    two_nr = ops.moe_forward(x2, wr, wgu, wd, k)
    for _ in range(2):
        one, idx1, _ = ops.moe_forward(x2[:1].contiguous(), wr, wgu, wd, k, residual=res2[:1].contiguous(),
                                       return_routing=True)
        one_nr = ops.moe_forward(x2[:1].contiguous(), wr, wgu, wd, k)
        torch.cuda.synchronize()
        assert _C.device_error() == 0
        assert torch.equal(idx1[0], idx2[0])
        assert torch.equal(one[0], two[0])
        assert torch.equal(one_nr[0], two_nr[0])
