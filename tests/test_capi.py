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
