"""CPU checks of the C-ABI library: it loads and exports every declared symbol."""

from __future__ import annotations

import os
import re

import pytest

from llada_quant_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "llada_quant.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(llq_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_abi():
    names = declared_symbols()
    assert "llq_fused_moe_packed" in names and "llq_quantize_pack" in names
    assert set(names) == set(_lib.SIGNATURES), "ctypes table and header must agree"


def test_library_loads_and_exports_every_symbol():
    if not os.path.exists(_lib.LIB_PATH):
        pytest.fail("libllada_quant_cuda.so is not built (run __graft_entry__.build())")
    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert lib.llq_version() >= 100
    assert isinstance(lib.llq_last_error(), bytes)


def test_workspace_queries_need_no_gpu():
    lib = _lib.load()
    assert lib.llq_moe_workspace_size(256, 8, 64, 2048, 1024) > 256 * 8 * (2048 * 2 * 2 + 1024 * 2)
    assert lib.llq_align_workspace_size(256, 8, 64) >= 64 * 4


def test_argument_validation_needs_no_gpu():
    """Bad arguments are rejected before any launch, with the reference's messages."""
    lib = _lib.load()
    rc = lib.llq_quantize_pack(None, 2, 4, 6, 5, 128, 0, 24, 0.5, 0, 1, None, None, None)
    assert rc == _lib.LLQ_EINVAL
    assert b"bits must be 8 or 4" in lib.llq_last_error()
    rc = lib.llq_quantize_pack(1, 2, 4, 7, 4, 128, 0, 24, 0.5, 0, 1, 1, 1, None)
    assert rc == _lib.LLQ_EINVAL and b"even last dimension" in lib.llq_last_error()
    rc = lib.llq_quantize_pack(1, 2, 4, 8, 4, 33, 0, 24, 0.5, 0, 1, 1, 1, None)
    assert rc == _lib.LLQ_EINVAL and b"even group_size" in lib.llq_last_error()
    rc = lib.llq_quantize_pack(1, 2, 4, 8, 4, 8, 1, 0, 0.5, 0, 1, 1, 1, None)
    assert rc == _lib.LLQ_EINVAL and b"grid must be >= 1" in lib.llq_last_error()
    rc = lib.llq_quantize_pack(1, 2, 4, 8, 4, 8, 1, 4, 1.0, 0, 1, 1, 1, None)
    assert rc == _lib.LLQ_EINVAL and b"max_shrink" in lib.llq_last_error()
    rc = lib.llq_fused_moe_packed(*([None] * 7), 4, 8, 64, 32, 2, 4, 128, None, None, 0, 0, None)
    assert rc == _lib.LLQ_ENOSPACE
    # the block call: bad shape, missing routing outputs, no workspace -- all before any launch
    blk = lambda T, E, k, tw, ids: lib.llq_moe_block_packed(None, None, None, 0, T, E, 64, 32, k, None, None, None,
                                                             None, 4, 128, None, tw, ids, None, None, 0, 0, None)
    assert blk(4, 8, 9, 1, 1) == _lib.LLQ_EINVAL and b"bad shape" in lib.llq_last_error()
    assert blk(4, 8, 2, None, 1) == _lib.LLQ_EINVAL and b"topk_w" in lib.llq_last_error()
    assert blk(4, 8, 2, 1, 1) == _lib.LLQ_ENOSPACE
    assert blk(0, 8, 2, None, None) == _lib.LLQ_OK


def _a256(v):
    return (v + 255) // 256 * 256


def test_ep_window_layout_and_validation_need_no_gpu():
    """The exchange window holds the signal words, the received (id, weight) pairs and the
    received / returned rows of every rank, each 256-byte aligned."""
    lib = _lib.load()
    R, cap, H = 8, 2048, 2048
    expect = _a256(4 * (5 * R + 8)) + 2 * _a256(4 * R * cap) + 2 * _a256(R * cap * H * 2)
    assert lib.llq_ep_window_bytes(R, cap, H) == expect
    assert lib.llq_ep_window_bytes(0, cap, H) == 0
    assert lib.llq_ipc_handle_bytes() == 64
    # T*k beyond the window capacity, bad world/rank: rejected before any launch
    rc = lib.llq_ep_dispatch(1, 1, 1, 300, 8, H, 8, 1, 1, 0, 8, 2048, 1, 1, None)
    assert rc == _lib.LLQ_EINVAL and b"exceeds the window capacity" in lib.llq_last_error()
    rc = lib.llq_ep_dispatch(1, 1, 1, 1, 8, H, 8, 1, 1, 3, 2, 2048, 1, 1, None)
    assert rc == _lib.LLQ_EINVAL and b"rank 3" in lib.llq_last_error()
    rc = lib.llq_ep_experts(1, 1, 0, 2, 2048, 1, 1, 1, 1, 1, 32, H, 1024, 4, 128, 2048, 1, 1 << 30,
                            _lib.LLQ_GEMM_SIMT, None)
    assert rc == _lib.LLQ_EUNSUPPORTED
    assert lib.llq_ep_set_timeout_ms(0) == _lib.LLQ_EINVAL


def test_quant_linear_validation_needs_no_gpu():
    lib = _lib.load()
    rc = lib.llq_quant_linear(1, 4, 1024, 256, 1, 1, 3, 128, 1, None, 0, 0, None)
    assert rc == _lib.LLQ_EUNSUPPORTED and b"bits must be 8 or 4" in lib.llq_last_error()
    rc = lib.llq_quant_linear(1, 4, 1023, 256, 1, 1, 4, 128, 1, None, 0, 0, None)
    assert rc == _lib.LLQ_EINVAL and b"even last dimension" in lib.llq_last_error()
    rc = lib.llq_quant_linear(1, 4, 1024, 256, 1, 1, 4, 128, 1, None, 0, _lib.LLQ_GEMM_TCGEN05_FAST, None)
    assert rc == _lib.LLQ_EUNSUPPORTED
    assert lib.llq_quant_linear(None, 0, 1024, 256, None, None, 4, 128, None, None, 0, 0, None) == _lib.LLQ_OK
    # one 1-token row of a 2048 x 2048 layer is 8 output tiles: split K so that the SMs are covered
    assert lib.llq_quant_linear_workspace_size(1, 2048, 2048) % (2048 * 4) == 0
    assert lib.llq_quant_linear_workspace_size(1, 2048, 2048) >= 2 * 2048 * 4
