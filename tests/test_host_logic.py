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


# ---- routing statistics (analysis/moe_regime.py:150-213; reference tests test_moe_regime.py:89-108)
def test_expert_token_stats_counts_real_routing():
    from llada_quant_b200.routing_stats import expert_token_stats
    stats = expert_token_stats(torch.tensor([[0, 1], [0, 2], [0, 1]]), num_experts=4)
    assert stats.counts == [3, 2, 1, 0]
    assert stats.active_experts == 3
    assert stats.mean == pytest.approx(1.5)
    assert stats.imbalance == pytest.approx(2.0)
    assert stats.to_dict()["max"] == 3


def test_expert_token_stats_rejects_wrong_rank():
    from llada_quant_b200.routing_stats import expert_token_stats
    with pytest.raises(ValueError, match=r"\[tokens, top_k\]"):
        expert_token_stats(torch.zeros(4), num_experts=4)


def test_expert_token_stats_balanced():
    from llada_quant_b200.routing_stats import expert_token_stats
    stats = expert_token_stats(torch.tensor([[0, 1], [2, 3], [0, 1], [2, 3]]), 4)
    assert stats.imbalance == 1.0 and stats.mean == 2.0
    d = stats.to_dict()
    assert d["p50"] == 2.0 and d["min"] == 2 and d["imbalance_max_over_mean"] == 1.0


# ---- QuantLinear (runtime/linear.py:29-131) host-side contract
def test_quant_linear_buffers_and_storage():
    from llada_quant_b200.linear import QuantLinear, kernel_supports
    m = QuantLinear(1024, 512, bits=4, group_size=128, bias=True)
    assert tuple(m.qweight.shape) == (512, 512) and m.qweight.dtype == torch.int8
    assert tuple(m.scale.shape) == (512, 8) and m.scale.dtype == torch.float32
    assert m.storage_bytes() == 512 * 512 + 512 * 8 * 4 + 512 * 2
    assert "int4x2 codes" in m.extra_repr()
    m8 = QuantLinear(100, 256, bits=8, group_size=128)
    assert tuple(m8.scale.shape) == (256, 1)  # per-row fallback when the group does not divide K
    assert kernel_supports(1024, 512, 128) and kernel_supports(2048, 256, -1)
    assert not kernel_supports(100, 256, 128) and not kernel_supports(4096, 256, 128)
    assert not kernel_supports(1024, 384, 128) and not kernel_supports(1024, 512, 64)
    with pytest.raises(ValueError, match="bits must be 8 or 4"):
        QuantLinear(64, 64, bits=3)
    with pytest.raises(RuntimeError, match="CUDA"):
        m(torch.zeros(2, 1024))


def test_router_capture_accessors_on_host_tensors():
    import torch
    from llada_quant_b200.router_capture import RouterCapture
    cap = RouterCapture()
    cap.record("b", torch.tensor([[1, 0]], dtype=torch.int32), torch.zeros(1, 4, dtype=torch.bfloat16))
    cap.record("a", torch.tensor([[2, 3]], dtype=torch.int32), torch.ones(1, 4, dtype=torch.bfloat16))
    assert cap.layer_names == ["a", "b"]
    assert cap.topk_ids["a"].dtype == torch.int64 and cap.topk_ids["a"].tolist() == [[2, 3]]
    assert cap.gates["a"].dtype == torch.float32
    with cap:
        pass
    cap.record("c", torch.zeros(1, 2, dtype=torch.int32), torch.zeros(1, 4))
    assert "c" not in cap.layer_names
    cap.remove()
    cap.clear()
    assert cap.layer_names == []
