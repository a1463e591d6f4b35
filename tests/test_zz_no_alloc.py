"""qmoe_moe_forward_noalloc: the allocation-free fused forward, for callers that
cannot allocate device memory where they run the layer (plugin enqueue hooks of
inference runtimes, embedders that hand the library no workspace).  It must
give the same result as the workspace entry point qmoe_moe_forward, call after
call, while taking its scratch from the library's built-in device array.

This file is collected last so that, if it fails, a run stopping at the first
failure has already run every other test."""
import ctypes

import pytest
import torch

from helpers import activations, assert_within_one_ulp, moe_weights

pytestmark = pytest.mark.gpu

H, E, K, I = 2048, 128, 8, 768


def _forward_with_workspace(lib, x, wr, wgu, wd, res, stream):
    T = x.shape[0]
    out = torch.empty((T, H), dtype=torch.bfloat16, device=x.device)
    idx = torch.empty((T, K), dtype=torch.int32, device=x.device)
    tw = torch.empty((T, K), dtype=torch.float32, device=x.device)
    ws_bytes = lib.qmoe_moe_forward_workspace_size(T, H, E, K, I)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)
    st = lib.qmoe_moe_forward(x.data_ptr(), wr.data_ptr(), None, wgu.data_ptr(), wd.data_ptr(),
                              res.data_ptr(), T, H, E, K, I, 1, out.data_ptr(), idx.data_ptr(),
                              tw.data_ptr(), ws.data_ptr(), ws_bytes, stream)
    assert st == 0, lib.qmoe_last_error()
    return out, idx, tw


def _forward_noalloc(lib, x, wr, wgu, wd, res, stream):
    T = x.shape[0]
    out = torch.empty((T, H), dtype=torch.bfloat16, device=x.device)
    idx = torch.empty((T, K), dtype=torch.int32, device=x.device)
    tw = torch.empty((T, K), dtype=torch.float32, device=x.device)
    st = lib.qmoe_moe_forward_noalloc(x.data_ptr(), wr.data_ptr(), None, wgu.data_ptr(),
                                      wd.data_ptr(), res.data_ptr(), T, H, E, K, I, 1,
                                      out.data_ptr(), idx.data_ptr(), tw.data_ptr(), stream)
    assert st == 0, lib.qmoe_last_error()
    return out, idx, tw


@pytest.mark.parametrize("T", [1, 24, 64, 156])
def test_noalloc_matches_workspace_forward_twice(cuda_dev, T):
    from nki_moe_7013_b200 import _C

    lib = _C.lib()
    stream = torch.cuda.current_stream(cuda_dev).cuda_stream
    wr, wgu, wd = moe_weights(21, E, H, I, cuda_dev)
    x = activations(21 + T, T, H, cuda_dev)
    res = activations(40 + T, T, H, cuda_dev)
    ref_out, ref_idx, ref_w = _forward_with_workspace(lib, x, wr, wgu, wd, res, stream)
    # two calls in a row on the shared built-in scratch: the same kernels as
    # the workspace forward, so routing and weights are identical and the
    # outputs differ at most by the order of the fp32 combine sums (one bf16
    # ulp)
    for _ in range(2):
        out, idx, tw = _forward_noalloc(lib, x, wr, wgu, wd, res, stream)
        torch.cuda.synchronize()
        assert torch.equal(idx, ref_idx)
        assert torch.equal(tw, ref_w)
        assert_within_one_ulp(out, ref_out, "noalloc vs workspace forward")
    assert _C.device_error() == 0


# 156 tokens are the most the 8 MiB scratch holds at these shapes
LIMIT_T = 156


def test_noalloc_limit_is_where_the_scratch_runs_out(cuda_dev):
    from nki_moe_7013_b200 import _C

    lib = _C.lib()
    cap = 8 << 20
    assert lib.qmoe_moe_forward_workspace_size(LIMIT_T, H, E, K, I) <= cap
    assert lib.qmoe_moe_forward_workspace_size(LIMIT_T + 1, H, E, K, I) > cap


@pytest.mark.parametrize("T", [LIMIT_T + 1, 4096])
def test_noalloc_rejects_more_than_its_scratch(cuda_dev, T):
    from nki_moe_7013_b200 import _C

    lib = _C.lib()
    x = torch.zeros((T, H), dtype=torch.bfloat16, device=cuda_dev)
    w = torch.zeros(16, dtype=torch.bfloat16, device=cuda_dev)
    out = torch.full((T, H), 7.0, dtype=torch.bfloat16, device=cuda_dev)
    st = lib.qmoe_moe_forward_noalloc(x.data_ptr(), w.data_ptr(), None, w.data_ptr(), w.data_ptr(),
                                      None, T, H, E, K, I, 1, out.data_ptr(), None, None,
                                      ctypes.c_void_p(0))
    assert st == -4  # QMOE_ERR_WORKSPACE_TOO_SMALL, nothing launched
    assert b"scratch" in lib.qmoe_last_error()
    torch.cuda.synchronize()
    assert bool((out == 7.0).all())  # output untouched
