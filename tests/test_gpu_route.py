"""GPU parity of the router, alignment, permute and combine kernels.

Bars: logits within one bf16 ulp of the oracle (fp32 sums in a different
order); top-k ids identical given identical logits except among values equal to
fp32 precision; alignment, permute and combine bit-exact.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import moe as M
from oracle import symmetric as S
from tests._util import random_routing, to_np

pytestmark = pytest.mark.gpu


def _check_topk(w, ids, ref_w, ref_ids, p):
    np.testing.assert_allclose(w, ref_w, rtol=2e-6, atol=1e-9)
    for t in range(ids.shape[0]):
        for j in range(ids.shape[1]):
            if ids[t, j] != ref_ids[t, j]:
                a, b = p[t, ids[t, j]], p[t, ref_ids[t, j]]
                assert abs(a - b) <= 2e-6 * max(a, b), (t, j)


@pytest.mark.parametrize("T,H,E,k", [(96, 256, 16, 4), (256, 2048, 64, 8), (7, 1024, 16, 2), (1, 2048, 64, 8)])
def test_route_matches_oracle(T, H, E, k):
    from llada_quant_b200 import ops
    g = torch.Generator().manual_seed(T + E)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    gw = (torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16)
    w, ids, logits = ops.route(x.cuda(), gw.cuda(), k, None, False)
    ref_logits = M.router_logits(to_np(x), to_np(gw))
    ulps = np.abs(S.bf16_bits(to_np(logits)).astype(np.int32) - S.bf16_bits(ref_logits).astype(np.int32))
    assert ulps.max() <= 1 and (ulps > 0).mean() < 0.02
    # top-k from OUR logits must match the oracle's top-k of the same logits
    ref_w, ref_ids = M.route_topk(to_np(logits), k)
    _check_topk(to_np(w), to_np(ids), ref_w, ref_ids, M.softmax_fp32(to_np(logits)))


def test_route_golden_router_capture(golden):
    """Against the reference's RouterCapture recomputation (golden logits fed in)."""
    from llada_quant_b200 import ops
    logits = torch.from_numpy(S.from_bf16_bits(golden["route/logits"])).to(torch.bfloat16).cuda()
    k = golden["route/topk_ids"].shape[1]
    w, ids = ops.route_topk(logits, k, None, False)
    _check_topk(to_np(w), to_np(ids), golden["route/topk_w"], golden["route/topk_ids"],
                golden["route/probs"])


def test_route_bias_and_renormalize():
    from llada_quant_b200 import ops
    g = torch.Generator().manual_seed(9)
    logits = torch.randn(64, 64, generator=g)
    rng = np.random.default_rng(0)
    bias = (-1.1 * np.log(rng.permutation(64) + 1.0)).astype(np.float32)
    w, ids = ops.route_topk(logits.cuda(), 8, torch.from_numpy(bias).cuda(), True)
    ref_w, ref_ids = M.route_topk(logits.numpy(), 8, bias=bias, renormalize=True)
    p = M.softmax_fp32((logits.numpy() + bias[None]).astype(np.float32))
    _check_topk(to_np(w), to_np(ids), ref_w, ref_ids, p)


@pytest.mark.parametrize("T,E,k,skew", [(256, 64, 8, None), (3000, 64, 8, 1.1), (1, 16, 2, None),
                                         (37, 16, 2, 3.0), (5000, 256, 8, None)])
def test_align_is_stable_and_exact(T, E, k, skew):
    from llada_quant_b200 import ops
    _, ids = random_routing(T, E, k, seed=T, skew=skew)
    offsets, slots = ops.moe_align(torch.from_numpy(ids).cuda(), E)
    ref_off, ref_slots = M.moe_align(ids, E)
    assert np.array_equal(to_np(offsets), ref_off)
    assert np.array_equal(to_np(slots), ref_slots)


def test_align_all_tokens_to_one_expert():
    from llada_quant_b200 import ops
    ids = np.zeros((300, 1), dtype=np.int32) + 5
    offsets, slots = ops.moe_align(torch.from_numpy(ids).cuda(), 16)
    ref_off, ref_slots = M.moe_align(ids, 16)
    assert np.array_equal(to_np(offsets), ref_off) and np.array_equal(to_np(slots), ref_slots)


def test_permute_and_combine_exact():
    from llada_quant_b200 import ops
    T, H, E, k = 50, 512, 16, 4
    _, ids = random_routing(T, E, k, seed=1)
    x = torch.randn(T, H).to(torch.bfloat16)
    offsets, slots = ops.moe_align(torch.from_numpy(ids).cuda(), E)
    xs = ops.moe_permute(x.cuda(), slots, k)
    assert torch.equal(xs.cpu(), x[torch.from_numpy(to_np(slots)).long() // k])
    y = torch.randn(T * k, H).to(torch.bfloat16)
    out = ops.moe_combine(y.cuda(), k)
    ref = np.zeros((T, H), np.float32)
    yn = to_np(y).reshape(T, k, H)
    for j in range(k):
        ref = (ref + yn[:, j]).astype(np.float32)
    assert np.array_equal(to_np(out), S.round_to_bf16(ref))


def test_permute_kperm_reorders_each_8_block():
    from llada_quant_b200 import ops
    T, H, E, k = 9, 64, 4, 2
    _, ids = random_routing(T, E, k, seed=2)
    x = torch.randn(T, H).to(torch.bfloat16)
    offsets, slots = ops.moe_align(torch.from_numpy(ids).cuda(), E)
    plain = ops.moe_permute(x.cuda(), slots, k).cpu()
    perm = ops.moe_permute(x.cuda(), slots, k, True).cpu()
    order = torch.tensor([0, 4, 1, 5, 2, 6, 3, 7])
    idx = (torch.arange(H) // 8) * 8 + order.repeat(H // 8)
    assert torch.equal(perm, plain[:, idx])


def test_ep_pack_and_combine_exact():
    """Expert-parallel pack (rows, local ids, weights, inverse positions) and combine."""
    from llada_quant_b200 import ops
    T, H, E, k, world = 40, 256, 16, 4, 4
    epr = E // world
    tw, ids = random_routing(T, E, k, seed=7)
    x = torch.randn(T, H).to(torch.bfloat16)
    dest = torch.from_numpy(ids // epr).cuda()
    offsets, order = ops.moe_align(dest, world)
    rows, lid, wts, inv = ops.ep_pack(x.cuda(), torch.from_numpy(ids).cuda(), torch.from_numpy(tw).cuda(),
                                      order, epr)
    o = to_np(order).astype(np.int64)
    assert np.array_equal(to_np(offsets), np.concatenate([[0], np.cumsum(np.bincount(ids.reshape(-1) // epr, minlength=world))]))
    assert torch.equal(rows.cpu(), x[torch.from_numpy(o // k)])
    assert np.array_equal(to_np(lid), ids.reshape(-1)[o] % epr)
    assert np.array_equal(to_np(wts), tw.reshape(-1)[o])
    assert np.array_equal(to_np(inv)[o], np.arange(T * k))
    back = torch.randn(T * k, H).to(torch.bfloat16)
    out = ops.ep_combine(back.cuda(), inv, k)
    b = to_np(back)
    ref = np.zeros((T, H), np.float32)
    for j in range(k):
        ref = (ref + b[to_np(inv).reshape(T, k)[:, j]]).astype(np.float32)
    assert np.array_equal(to_np(out), S.round_to_bf16(ref))


def test_router_capture_records_the_kernels_routing():
    """RouterCapture (trajectory/llada.py:157-268 accessors) fed by moe_layer's own router:
    the recorded ids are those the layer's GEMMs used, the logits those of the oracle."""
    from llada_quant_b200 import symmetric as G
    from llada_quant_b200.fused_moe import moe_layer
    from llada_quant_b200.moe import PackedExperts
    from llada_quant_b200.router_capture import RouterCapture
    from tests._util import synthetic_layer, synthetic_tokens
    T, E, H, I, k = 64, 16, 1024, 512, 2
    w1, w2 = synthetic_layer(E, H, I, seed=4)
    r1 = G.quantize_tensor(w1.cuda(), bits=4, group_size=128)
    r2 = G.quantize_tensor(w2.cuda(), bits=4, group_size=128)
    packed = PackedExperts(r1.q, r1.scale, r2.q, r2.scale, 4, 128)
    gw = (torch.randn(E, H, generator=torch.Generator().manual_seed(5)) * 0.02).to(torch.bfloat16)
    with RouterCapture() as cap:
        for layer in range(2):
            x = synthetic_tokens(T, H, seed=20 + layer).cuda()
            moe_layer(x, gw.cuda(), packed, k, capture=cap, name=f"layers.{layer}.mlp")
            ref_logits = M.router_logits(to_np(x), to_np(gw))
            got = cap.gates[f"layers.{layer}.mlp"].numpy()
            ulps = np.abs(S.bf16_bits(got).astype(np.int32) - S.bf16_bits(ref_logits).astype(np.int32))
            assert ulps.max() <= 1
            ids = cap.topk_ids[f"layers.{layer}.mlp"]
            assert ids.dtype == torch.int64 and tuple(ids.shape) == (T, k)
            ref_w, ref_ids = M.route_topk(got, k)
            _check_topk(ref_w, ids.numpy(), ref_w, ref_ids, M.softmax_fp32(got))
    assert cap.layer_names == ["layers.0.mlp", "layers.1.mlp"]
    moe_layer(x, gw.cuda(), packed, k, capture=cap, name="after")  # removed: nothing recorded
    assert "after" not in cap.layer_names
    cap.clear()
    assert cap.layer_names == []


@pytest.mark.parametrize("T,H,E,k,bias,renorm", [
    (256, 2048, 64, 8, False, False),
    (1, 2048, 64, 8, False, False),
    (37, 512, 16, 2, True, True),      # ragged token tile, bias, renormalized weights
    (40, 384, 24, 4, False, False),    # outside the tcgen05 shapes: the CUDA-core GEMMs
])
def test_block_call_matches_router_then_layer(T, H, E, k, bias, renorm):
    """llq_moe_block_packed (router inside the call) against llq_route followed by
    llq_fused_moe_packed on the same inputs: identical logits, routing and output
    over repeated calls."""
    from llada_quant_b200 import ops
    from llada_quant_b200 import symmetric as G
    from llada_quant_b200.moe import PackedExperts
    dev = torch.device("cuda")
    I = 256
    g = torch.Generator().manual_seed(T + H + E)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16).to(dev)
    gw = (torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16).to(dev)
    b = (torch.randn(E, generator=g) * 0.1).to(dev) if bias else None
    r1 = G.quantize_tensor((torch.randn(E, 2 * I, H, generator=g) * 0.02).to(torch.bfloat16).to(dev), bits=4,
                           group_size=128)
    r2 = G.quantize_tensor((torch.randn(E, H, I, generator=g) * 0.02).to(torch.bfloat16).to(dev), bits=4,
                           group_size=128)
    p = PackedExperts(r1.q, r1.scale, r2.q, r2.scale, 4, 128)
    tw, ids, logits = ops.route(x, gw, k, b, renorm)
    ref = ops.fused_moe_packed(x, p.qw1, p.sw1, p.qw2, p.sw2, tw, ids, 4, 0)
    for _ in range(3):
        out, tw2, ids2, lg2 = ops._moe_block_packed_impl(x, gw, b, renorm, p.qw1, p.sw1, p.qw2, p.sw2, k, 4, 0,
                                                         want_logits=True)
        torch.cuda.synchronize()
        assert torch.equal(lg2, logits)
        assert torch.equal(ids2, ids)
        assert torch.equal(tw2, tw)
        assert torch.equal(out, ref)
    assert ops.device_error() == 0
