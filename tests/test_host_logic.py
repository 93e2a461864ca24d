"""Host-side logic that needs no GPU: the product path refuses CPU tensors."""

from __future__ import annotations

import pytest
import torch

from llada_quant_b200 import ops, symmetric


def test_ops_refuse_cpu_tensors():
    w = torch.randn(4, 128, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        symmetric.quantize_tensor(w, bits=4, group_size=128)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        ops.route(torch.zeros(2, 8, dtype=torch.bfloat16), torch.zeros(4, 8, dtype=torch.bfloat16), 2, None, False)


def test_reference_error_messages_before_any_launch():
    with pytest.raises(ValueError, match="bits must be 8 or 4"):
        symmetric.quantize_tensor(torch.zeros(2, 8), bits=3)
    with pytest.raises(ValueError, match="cannot quantize an empty tensor"):
        symmetric.quantize_tensor(torch.zeros(0, 8))
    with pytest.raises(ValueError, match="even last dimension"):
        symmetric.quantize_tensor(torch.zeros(2, 7), bits=4)
    with pytest.raises(ValueError, match="scale_search must be"):
        symmetric.quantize_tensor(torch.zeros(2, 8), bits=8, scale_search="magic")
    with pytest.raises(ValueError, match="grid must be >= 1"):
        symmetric.search_group_scale(torch.zeros(2, 1, 8), bits=4, grid=0)


def test_block_k_alignment_helpers():
    assert symmetric.block_k_is_scale_aligned(64, 128)
    assert symmetric.block_k_is_scale_aligned(256, 128)
    assert not symmetric.block_k_is_scale_aligned(96, 128)
    with pytest.raises(ValueError, match="BLOCK_SIZE_K=96"):
        symmetric.validate_block_k_alignment(96, 128)
    assert symmetric.storage_bytes(1024, 4, 128) == 512 + 8 * 4


def test_effective_groups_mirror_the_fallback():
    assert ops.effective_groups(2048, 128) == (128, 16)
    assert ops.effective_groups(100, 64) == (-1, 1)
    assert ops.effective_groups(100, -1) == (-1, 1)
