"""GPU parity of the routed W4A16/W8A16 expert FFN.

Oracle: oracle/moe.py (bf16 weights exactly as the PACKED property returns
them, fp32 accumulation, the external kernel's rounding order), pinned to the
reference in tests/test_oracle_golden.py.

Tolerance (stated): the kernels accumulate in fp32 in another order than the
oracle, so a bf16 rounding of gate/up/h/y can land one ulp apart and carry
forward.  Layer outputs: rel-L2 <= 3e-3 against the oracle (the bar of the
reference's own kernel test, tests/unit/test_w8a16_kernel.py:59-66), and
max-abs <= 2 bf16 ulps of the output's largest magnitude.  Per-GEMM outputs:
rel-L2 <= 2e-3.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import moe as M
from oracle import symmetric as S
from tests._util import random_routing, synthetic_layer, synthetic_tokens, to_np

pytestmark = pytest.mark.gpu

IMPLS = ["simt", "tcgen05", "tcgen05_fast"]


@pytest.fixture(autouse=True)
def _no_device_timeouts():
    """Every bounded wait inside the tcgen05 kernels must have completed normally."""
    from llada_quant_b200 import ops
    ops.clear_device_error()
    yield
    torch.cuda.synchronize()
    assert ops.device_error() == 0, f"device error word {ops.device_error():#x}"


def _impl_or_skip(impl, bits=4):
    from llada_quant_b200 import _lib
    if impl == "tcgen05_fast":
        if bits != 4:
            pytest.skip("the fast (scale-after-MMA) mode is INT4 only")
        return _lib.LLQ_GEMM_TCGEN05_FAST
    if impl == "tcgen05":
        return _lib.LLQ_GEMM_TCGEN05
    return _lib.LLQ_GEMM_SIMT


def _quantize(E, H, I, bits, search="amax", seed=0):
    from llada_quant_b200 import symmetric as G
    w1, w2 = synthetic_layer(E, H, I, seed=seed)
    r1 = G.quantize_tensor(w1.cuda(), bits=bits, group_size=128, scale_search=search)
    r2 = G.quantize_tensor(w2.cuda(), bits=bits, group_size=128, scale_search=search)
    return r1, r2


def _assert_layer_close(out, ref, fast=False, truth=None):
    """Exact-weight modes: rel-L2 <= 3e-3 and max-abs <= 2 bf16 ulps of the largest output.
    Fast mode (W = q*s without bf16 weight rounding): rel-L2 <= 1e-2 against the oracle,
    and -- when the fp64 evaluation of the quantized layer is given -- no further from it
    than the oracle (the reference path) itself is, with 10% slack."""
    rel = M.rel_l2(out, ref)
    mx = M.max_abs(out, ref)
    if fast:
        assert rel <= 1e-2, rel
        if truth is not None:
            assert M.rel_l2(out, truth) <= 1.1 * M.rel_l2(ref, truth) + 1e-6, (
                M.rel_l2(out, truth), M.rel_l2(ref, truth))
        return rel, mx
    bound = 2 * 2.0 ** -7 * max(np.abs(ref).max(), 1e-6)
    assert rel <= 3e-3, rel
    assert mx <= bound, (mx, bound)
    return rel, mx


def _run_layer(T, E, H, I, k, bits, impl, skew=None, search="amax", seed=0):
    from llada_quant_b200 import ops
    code = _impl_or_skip(impl, bits)
    r1, r2 = _quantize(E, H, I, bits, search, seed)
    x = synthetic_tokens(T, H)
    tw, ids = random_routing(T, E, k, seed=seed + T, skew=skew)
    out = ops.fused_moe_packed(x.cuda(), r1.q, r1.scale, r2.q, r2.scale,
                               torch.from_numpy(tw).cuda(), torch.from_numpy(ids).cuda(), bits, code)
    args = (to_np(x), to_np(r1.q), to_np(r1.scale), to_np(r2.q), to_np(r2.scale), tw, ids, bits)
    ref = M.fused_moe_packed(*args)
    truth = M.fused_moe_f64(*args) if impl == "tcgen05_fast" else None
    return to_np(out), ref, truth


@pytest.mark.parametrize("impl", IMPLS)
@pytest.mark.parametrize("T,E,H,I,k,bits", [
    (256, 16, 1024, 512, 2, 4),     # C1 layer
    (1024, 16, 1024, 512, 2, 8),    # C2, W8A16
    (256, 64, 2048, 1024, 8, 4),    # C3 layer
    (33, 64, 2048, 1024, 8, 4),     # ragged, many empty experts
    (1, 16, 1024, 512, 2, 4),       # single token
    (7, 16, 1024, 512, 2, 8),
    (2048, 16, 1024, 512, 2, 4),    # > 96 rows per expert: the 128-token prefill tiles
    (2048, 16, 1024, 512, 2, 8),
])
def test_fused_layer_matches_oracle(impl, T, E, H, I, k, bits):
    out, ref, truth = _run_layer(T, E, H, I, k, bits, impl)
    _assert_layer_close(out, ref, impl == "tcgen05_fast", truth)


@pytest.mark.parametrize("impl", IMPLS)
def test_skewed_routing_one_hot_expert(impl):
    """Zipf-skewed routing: one expert gets most tokens (> one token tile)."""
    out, ref, truth = _run_layer(600, 16, 1024, 512, 2, 4, impl, skew=3.0)
    _assert_layer_close(out, ref, impl == "tcgen05_fast", truth)


@pytest.mark.parametrize("impl", IMPLS)
def test_mse_weights(impl):
    out, ref, truth = _run_layer(128, 16, 1024, 512, 2, 4, impl, search="mse")
    _assert_layer_close(out, ref, impl == "tcgen05_fast", truth)


@pytest.mark.parametrize("impl", IMPLS)
@pytest.mark.parametrize("name", ["moe_i4_amax", "moe_i8_amax", "moe_i4_mse"])
def test_layer_vs_reference_golden(golden, impl, name):
    """Golden layer outputs built from the reference's own dequantize_tensor."""
    from llada_quant_b200 import ops
    E, H, I, T, K = (int(v) for v in golden["moe/shape"])
    bits = int(golden[f"{name}/bits"])
    x = torch.from_numpy(S.from_bf16_bits(golden["moe/x"])).to(torch.bfloat16).cuda()
    t = lambda a: torch.from_numpy(golden[a]).cuda()
    code = _impl_or_skip(impl, bits)
    out = ops.fused_moe_packed(x, t(f"{name}/qw1"), t(f"{name}/sw1"), t(f"{name}/qw2"),
                               t(f"{name}/sw2"), t("moe/topk_w"), t("moe/topk_ids"), bits, code)
    truth = None
    if impl == "tcgen05_fast":
        truth = M.fused_moe_f64(S.from_bf16_bits(golden["moe/x"]), golden[f"{name}/qw1"],
                                golden[f"{name}/sw1"], golden[f"{name}/qw2"], golden[f"{name}/sw2"],
                                golden["moe/topk_w"], golden["moe/topk_ids"], bits)
    _assert_layer_close(to_np(out), S.from_bf16_bits(golden[f"{name}/out"]), impl == "tcgen05_fast", truth)


@pytest.mark.parametrize("impl", ["simt", "tcgen05"])
def test_gemm_stages_match_oracle(impl):
    """GEMM1 (SiLU epilogue) and GEMM2 (routed weight, scatter) separately."""
    from llada_quant_b200 import ops
    T, E, H, I, k, bits = 256, 64, 2048, 1024, 8, 4
    r1, r2 = _quantize(E, H, I, bits)
    x = synthetic_tokens(T, H)
    tw, ids = random_routing(T, E, k, seed=5)
    offsets, slots = ops.moe_align(torch.from_numpy(ids).cuda(), E)
    xs = ops.moe_permute(x.cuda(), slots, k)
    h = ops.moe_gemm1(xs, offsets, r1.q, r1.scale, bits, _impl_or_skip(impl))
    _, inter = M.fused_moe_packed(to_np(x), to_np(r1.q), to_np(r1.scale), to_np(r2.q),
                                  to_np(r2.scale), tw, ids, bits, return_intermediates=True)
    assert M.rel_l2(to_np(h), inter["h_sorted"]) <= 2e-3
    # GEMM2 from the oracle's h so the two stages are judged independently
    h_ref = torch.from_numpy(inter["h_sorted"]).to(torch.bfloat16).cuda()
    y = ops.moe_gemm2(h_ref, offsets, slots, torch.from_numpy(tw).cuda(), r2.q, r2.scale, bits,
                      _impl_or_skip(impl))
    assert M.rel_l2(to_np(y), inter["y_slots"]) <= 2e-3


def test_block_packed_mode_end_to_end():
    """A fused expert block quantized in PACKED mode: w1 per access == reference dequant,
    and the block's forward through fused_moe matches the oracle."""
    import torch.nn as nn
    from llada_quant_b200 import moe as RM
    from llada_quant_b200.fused_moe import fused_moe, moe_layer

    class Block(nn.Module):
        def __init__(self):
            super().__init__()
            w1, w2 = synthetic_layer(16, 1024, 512)
            self.w1 = nn.Parameter(w1.cuda())
            self.w2 = nn.Parameter(w2.cuda())
            self.gate_w = (torch.randn(16, 1024) * 0.02).to(torch.bfloat16).cuda()

    b = Block()
    weights = RM.QuantExpertWeights.quantize(b.w1.detach(), b.w2.detach(), bits=4, group_size=128)
    RM.attach_packed_buffers(b, weights, torch.bfloat16)
    RM.install_packed_expert_access(b)
    assert RM.is_packed_expert_block(b)
    a, c = b.w1, b.w1
    assert torch.equal(a, c) and a.data_ptr() != c.data_ptr()
    ref_w1 = S.dequantize_tensor(to_np(b._qw1), to_np(b._sw1), 4, 128, packed=True, to_bf16=True)
    assert np.array_equal(to_np(a), ref_w1)
    x = synthetic_tokens(64, 1024).cuda()
    out = moe_layer(x, b.gate_w, b.packed_experts(), top_k=2)
    out_ref, *_ = M.moe_layer(to_np(x), to_np(b.gate_w), to_np(b._qw1), to_np(b._sw1),
                              to_np(b._qw2), to_np(b._sw2), 2, 4)
    # routing may legitimately differ on near-tied logits; compare the layer via the
    # same ids through fused_moe as well
    logits = (x.float() @ b.gate_w.float().t()).to(torch.bfloat16)
    tw, ids = torch.topk(torch.softmax(logits.float(), -1), 2)
    out2 = fused_moe(x, b.packed_experts(), None, logits, ids.int())
    ref2 = M.fused_moe_packed(to_np(x), to_np(b._qw1), to_np(b._sw1), to_np(b._qw2), to_np(b._sw2),
                              to_np(tw), to_np(ids).astype(np.int32), 4)
    _assert_layer_close(to_np(out2), ref2)
    assert M.rel_l2(to_np(out), out_ref) < 0.05


def _kperm_pos(n: np.ndarray) -> np.ndarray:
    j = n & 7
    return (n & ~7) | np.where(j < 4, 2 * j, 2 * (j - 4) + 1)


@pytest.mark.parametrize("impl", IMPLS)
@pytest.mark.parametrize("bits", [4, 8])
def test_gemm2_one_hot_rows_read_back_the_dequantized_weights(impl, bits):
    """With one-hot activation rows and routed weight 1, GEMM2 returns single weights:
    y[e*I + k, n] = bf16(q[e,n,k] * s) -- the in-register dequantization must equal
    dequantize_tensor bit for bit, for every nibble position and over group
    magnitudes from 1e-30 to 1."""
    from llada_quant_b200 import ops
    from llada_quant_b200 import symmetric as G
    code = _impl_or_skip(impl, bits)
    E, H, I = 2, 256, 1024
    rng = np.random.default_rng(11)
    mag = 10.0 ** rng.uniform(-30, 0, size=(E, H, I // 128, 1))
    w = (rng.standard_normal((E, H, I // 128, 128)) * mag).reshape(E, H, I).astype(np.float32)
    w2 = torch.from_numpy(w).to(torch.bfloat16)
    r2 = G.quantize_tensor(w2.cuda(), bits=bits, group_size=128)
    n = E * I
    cols = np.tile(np.arange(I), E)
    if impl == "tcgen05_fast":
        cols = _kperm_pos(cols)
    h = torch.zeros(n, I, dtype=torch.bfloat16)
    h[torch.arange(n), torch.from_numpy(cols)] = 1.0
    offsets = torch.tensor([0, I, 2 * I], dtype=torch.int32).cuda()
    slots = torch.arange(n, dtype=torch.int32).cuda()
    y = ops.moe_gemm2(h.cuda(), offsets, slots, torch.ones(n).cuda(), r2.q, r2.scale, bits, code)
    ref = S.dequantize_tensor(to_np(r2.q), to_np(r2.scale), bits, 128, packed=bits == 4, to_bf16=True)
    ref = np.ascontiguousarray(ref.transpose(0, 2, 1)).reshape(n, H)
    got = to_np(y)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), np.argwhere(got != ref)[:5]


@pytest.mark.parametrize("T,bits", [(256, 4), (2048, 4), (300, 8)])
def test_fused_gemm12_equals_the_two_launches(T, bits):
    """GEMM1 and GEMM2 in one launch (GEMM2 work waits per token tile for its h rows) equal
    the two separate launches bit for bit; the counters come back zeroed, so a second call
    on the same buffer is right too."""
    from llada_quant_b200 import ops
    E, H, I, k = 16, 1024, 512, 2
    r1, r2 = _quantize(E, H, I, bits)
    x = synthetic_tokens(T, H).cuda()
    tw, ids = random_routing(T, E, k, seed=T)
    tw, ids = torch.from_numpy(tw).cuda(), torch.from_numpy(ids).cuda()
    offsets, slots = ops.moe_align(ids, E)
    xs = ops.moe_permute(x, slots, k)
    code = _impl_or_skip("tcgen05", bits)
    h = ops.moe_gemm1(xs, offsets, r1.q, r1.scale, bits, code)
    y_ref = ops.moe_gemm2(h, offsets, slots, tw, r2.q, r2.scale, bits, code)
    counters = ops.gemm12_counters(T * k, E, "cuda")
    for _ in range(2):
        y = ops._moe_gemm12_impl(xs, offsets, slots, tw, r1.q, r1.scale, r2.q, r2.scale, bits, counters)
        torch.cuda.synchronize()
        assert torch.equal(y, y_ref)
        assert int(counters.abs().sum()) == 0


@pytest.mark.parametrize("bits", [4, 8])
def test_prefill_layer_on_dequantized_weights(bits):
    """Prefill-sized calls (>= 512 routed rows per expert) dequantize the layer's weights once
    (bit-identical to dequantize_tensor) and run both expert GEMMs with the bf16 weights
    staged in shared memory by TMA.  Same oracle and tolerance as the packed path, and the
    packed two-launch path as a second reference."""
    from llada_quant_b200 import _lib, ops
    T, E, H, I, k = 4096, 16, 1024, 512, 2
    r1, r2 = _quantize(E, H, I, bits, seed=11)
    x = synthetic_tokens(T, H, seed=12).cuda()
    tw, ids = random_routing(T, E, k, seed=13, skew=0.5)
    tw_d, ids_d = torch.from_numpy(tw).cuda(), torch.from_numpy(ids).cuda()
    out = ops.fused_moe_packed(x, r1.q, r1.scale, r2.q, r2.scale, tw_d, ids_d, bits, _lib.LLQ_GEMM_AUTO)
    ref = M.fused_moe_packed(to_np(x), to_np(r1.q), to_np(r1.scale), to_np(r2.q), to_np(r2.scale), tw, ids, bits)
    _assert_layer_close(to_np(out), ref)
    off, slots = ops.moe_align(ids_d, E)
    h = ops.moe_gemm1(ops.moe_permute(x, slots, k), off, r1.q, r1.scale, bits, _lib.LLQ_GEMM_TCGEN05)
    y = ops.moe_gemm2(h, off, slots, tw_d, r2.q, r2.scale, bits, _lib.LLQ_GEMM_TCGEN05)
    packed = ops.moe_combine(y, k)
    _assert_layer_close(to_np(out), to_np(packed))
