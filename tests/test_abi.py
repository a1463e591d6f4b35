"""The C-ABI library: it loads without a GPU, exports every function the public
header declares, and rejects bad arguments on the host before any launch."""
import ctypes

import pytest

from nki_moe_7013_b200 import _C
from nki_moe_7013_b200.build import LIB_PATH, build


@pytest.fixture(scope="module")
def lib():
    build()
    return _C.lib()


def test_exports_every_header_symbol(lib):
    names = _C.header_symbols()
    assert len(names) >= 10
    handle = ctypes.CDLL(LIB_PATH)
    missing = [n for n in names if not hasattr(handle, n)]
    assert not missing, f"declared but not exported: {missing}"
    # and the binding table covers every declared symbol
    assert sorted(_C._SIGNATURES) == names


def test_status_strings(lib):
    assert lib.qmoe_version() >= 100
    assert lib.qmoe_status_string(0) == b"ok"
    assert lib.qmoe_status_string(-4) == b"workspace too small"


def test_host_side_validation_needs_no_gpu(lib):
    # null pointers are refused before the device is touched
    st = lib.qmoe_router_topk(None, None, None, 4, 2048, 128, 8, 1, None, None, None, None, None)
    assert st == -1 and b"null" in lib.qmoe_last_error()
    buf = ctypes.create_string_buffer(64)
    p = ctypes.addressof(buf)
    # unsupported hidden size
    st = lib.qmoe_router_topk(p, p, None, 4, 300, 128, 8, 1, None, p, p, None, None)
    assert st == -2
    # k > E
    st = lib.qmoe_router_topk(p, p, None, 4, 2048, 32, 33, 1, None, p, p, None, None)
    assert st == -1
    # I not a multiple of 128
    st = lib.qmoe_grouped_gemm_gateup_swiglu(p, 0, None, p, p, 10, 128, 8, 2048, 100, 128, p, None, 0, None)
    assert st == -2
    # split-K scratch smaller than the query says
    st = lib.qmoe_grouped_gemm_gateup_swiglu(p, 0, None, p, p, 10, 128, 8, 2048, 768, 128, p, p, 64, None)
    assert st == -4 and lib.qmoe_grouped_gemm_gateup_split_workspace_size() > 64
    # misaligned pointer
    st = lib.qmoe_combine_finalize(p + 4, None, 2, 64, p, None)
    assert st == -3


def test_workspace_size_query(lib):
    small = lib.qmoe_moe_forward_workspace_size(1, 2048, 128, 8, 768)
    big = lib.qmoe_moe_forward_workspace_size(1024, 2048, 128, 8, 768)
    assert 0 < small < big
    # prefill sizes: permuted rows (T*k*H bf16) + act (T*k*I bf16) + fp32
    # accumulator (T*H); decode sizes gather token rows inside the GEMM
    assert big >= 1024 * 8 * 2048 * 2 + 1024 * 8 * 768 * 2 + 1024 * 2048 * 4
    assert lib.qmoe_moe_forward_workspace_size(64, 2048, 128, 8, 768) < 64 * 8 * 2048 * 2
    assert lib.qmoe_max_tiles(8192, 128) == 128 + 64 + 1
    # the fused block adds room for the add & norm outputs (2 x T*H bf16)
    for T in (1, 16, 1024):
        plain = lib.qmoe_moe_forward_workspace_size(T, 2048, 128, 8, 768)
        block = lib.qmoe_moe_block_forward_workspace_size(T, 2048, 128, 8, 768)
        assert block >= plain + 2 * 2 * T * 2048


def test_block_forward_validation_needs_no_gpu(lib):
    buf = ctypes.create_string_buffer(64)
    p = ctypes.addressof(buf)
    f = ctypes.c_float(1e-6)

    def call(x, res, w, H, I, ws_bytes, h_out=None):
        return lib.qmoe_moe_block_forward(x, res, w, f, p, None, p, p, 4, H, 128, 8, I, 1, p, h_out, None, None,
                                          None, p, ws_bytes, None)
    # no residual / no norm weight
    assert call(p, None, p, 2048, 768, 1 << 30) == -1 and b"null" in lib.qmoe_last_error()
    assert call(p, p, None, 2048, 768, 1 << 30) == -1
    # unsupported hidden size; I not a multiple of 128
    assert call(p, p, p, 300, 768, 1 << 30) == -2
    assert call(p, p, p, 2048, 100, 1 << 30) == -2
    # a workspace smaller than the query says
    assert call(p, p, p, 2048, 768, 64) == -4
    # misaligned optional output
    assert call(p, p, p, 2048, 768, 1 << 30, h_out=p + 4) == -3
