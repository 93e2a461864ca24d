"""Pin the numpy oracle to golden vectors produced by the reference package.

Bit-exact for every integer/byte result and for the amax scales; the MSE scale
search is bit-exact whenever the reference's float32 group sums do not make a
near-tie decision (the only order-dependent step, symmetric.py:198), and every
disagreement is checked to be such a near-tie.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import moe as M
from oracle import symmetric as S


def test_unpack_every_byte(golden):
    every_byte = np.arange(-128, 128, dtype=np.int8).reshape(1, 256)
    assert np.array_equal(S.unpack_int4(every_byte), golden["unpack_every_byte"])


def test_pack_every_pair(golden):
    pairs = golden["pack_every_pair_in"]
    packed = S.pack_int4(pairs)
    assert np.array_equal(packed, golden["pack_every_pair_out"])
    assert np.array_equal(S.unpack_int4(packed), pairs)


def test_pack_rejects_out_of_range_and_odd_shapes():
    with pytest.raises(ValueError, match=r"\[-8, 7\]"):
        S.pack_int4(np.array([[8, 0]], dtype=np.int8))
    with pytest.raises(ValueError, match="even"):
        S.pack_int4(np.zeros((1, 3), dtype=np.int8))


def _case(golden, name):
    bits, gs, mse, eff_gs, packed = (int(v) for v in golden[f"{name}/meta"])
    return golden[f"{name}/w"], bits, gs, mse, eff_gs, packed


@pytest.mark.parametrize("name", [
    "amax_i4_g128_bf16", "amax_i8_g128_bf16", "amax_i4_g64_fp16", "amax_i8_g32_fp32",
    "amax_i4_rowfallback", "amax_i8_rowfallback", "amax_i4_zero_groups",
])
def test_amax_quantize_is_bit_exact(golden, name):
    w, bits, gs, _, eff_gs, packed = _case(golden, name)
    q, scale, g_eff, was_packed, shape = S.quantize_tensor(w, bits=bits, group_size=gs)
    assert g_eff == eff_gs and int(was_packed) == packed
    assert np.array_equal(q, golden[f"{name}/q"])
    assert np.array_equal(scale.view(np.uint32), golden[f"{name}/scale"].view(np.uint32))
    deq = S.dequantize_tensor(q, scale, bits, g_eff, packed=was_packed, to_bf16=True)
    assert np.array_equal(S.bf16_bits(deq), golden[f"{name}/deq_bf16"])


@pytest.mark.parametrize("name", [
    "mse_i4_g128_heavy", "mse_i8_g128_heavy", "mse_i4_g128_bf16", "mse_i4_zero_groups",
])
def test_mse_quantize_matches_up_to_near_ties(golden, name):
    w, bits, gs, _, eff_gs, packed = _case(golden, name)
    q, scale, g_eff, was_packed, _ = S.quantize_tensor(w, bits=bits, group_size=gs, scale_search="mse")
    ref_scale = golden[f"{name}/scale"]
    flips = scale.view(np.uint32) != ref_scale.view(np.uint32)
    if flips.any():
        # every flip must be a near tie between the two candidates' exact SSEs
        w_g, _ = S.as_groups(w.astype(np.float32), gs)
        for idx in zip(*np.nonzero(flips)):
            wg = w_g[idx[:-1] + (idx[-1],)]
            e_ours = S.group_sse_terms(wg, np.float32(scale[idx]), bits).astype(np.float64).sum()
            e_ref = S.group_sse_terms(wg, np.float32(ref_scale[idx]), bits).astype(np.float64).sum()
            assert e_ours <= e_ref
            assert (e_ref - e_ours) <= 1e-5 * e_ref, (idx, e_ours, e_ref)
    assert flips.mean() < 0.01
    # where the scales agree the codes agree
    same = ~flips
    if bits == 4:
        q_u = S.unpack_int4(q)
        rq_u = S.unpack_int4(golden[f"{name}/q"])
    else:
        q_u, rq_u = q, golden[f"{name}/q"]
    qs = q_u.reshape(*same.shape, -1)
    rqs = rq_u.reshape(*same.shape, -1)
    assert np.array_equal(qs[same], rqs[same])


def test_search_grid8(golden):
    heavy = golden["mse_i4_g128_heavy/w"]
    w_g, _ = S.as_groups(heavy, 128)
    ours = S.search_group_scale(w_g, 4, grid=8)
    assert np.array_equal(ours.view(np.uint32), golden["search_grid8/scale"].view(np.uint32))


def test_search_hyperparameters_are_validated():
    w = np.zeros((4, 1, 64), np.float32)
    with pytest.raises(ValueError, match="grid must be >= 1"):
        S.search_group_scale(w, 4, grid=0)
    with pytest.raises(ValueError, match="max_shrink must lie in"):
        S.search_group_scale(w, 4, max_shrink=1.0)


def test_routing_matches_router_capture_up_to_ties(golden):
    logits = S.from_bf16_bits(golden["route/logits"])
    x = S.from_bf16_bits(golden["route/x"])
    gate_w = S.from_bf16_bits(golden["route/gate_w"])
    # the bf16 logits: fp32-accumulated dot products rounded once; torch's CPU
    # bf16 Linear sums in its own blocked order, so a few logits sit one bf16
    # ulp away (a rounding-boundary effect, never more than one ulp)
    ours_logits = M.router_logits(x, gate_w)
    ulps = np.abs(S.bf16_bits(ours_logits).astype(np.int32) - golden["route/logits"].astype(np.int32))
    assert ulps.max() <= 1 and (ulps > 0).mean() < 0.02
    k = golden["route/topk_ids"].shape[1]
    w, ids = M.route_topk(logits, k)
    ref_w = golden["route/topk_w"]
    # the selected values are the same sequence (ties may permute ids)
    np.testing.assert_allclose(w, ref_w, rtol=1e-6, atol=0)
    p = M.softmax_fp32(logits)
    np.testing.assert_allclose(p, golden["route/probs"], rtol=1e-6, atol=1e-9)
    ref_ids = golden["route/topk_ids"]
    for t in range(ids.shape[0]):
        for j in range(k):
            if ids[t, j] != ref_ids[t, j]:
                assert p[t, ids[t, j]] == p[t, ref_ids[t, j]], "ids may differ only among equal values"


@pytest.mark.parametrize("name", ["moe_i4_amax", "moe_i8_amax", "moe_i4_mse"])
def test_moe_layer_matches_reference_restatement(golden, name):
    E, H, I, T, K = (int(v) for v in golden["moe/shape"])
    x = S.from_bf16_bits(golden["moe/x"])
    bits = int(golden[f"{name}/bits"])
    out = M.fused_moe_packed(x, golden[f"{name}/qw1"], golden[f"{name}/sw1"], golden[f"{name}/qw2"],
                             golden[f"{name}/sw2"], golden["moe/topk_w"], golden["moe/topk_ids"], bits)
    ref = S.from_bf16_bits(golden[f"{name}/out"])
    # both sides: bf16 weights, fp32 accumulation in different orders, bf16 rounding
    # of gate/up/h/y/out; differences are a few bf16 ulps on a few elements
    assert M.rel_l2(out, ref) < 2e-3
    assert np.mean(out != ref) < 0.05
