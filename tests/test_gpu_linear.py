"""GPU parity of the dense QuantLinear forward and of the on-device routing statistics.

QuantLinear: the reference computes ``F.linear(x, dequantize_weight())``
(runtime/linear.py:127-131), i.e. ``bf16(x . W^T)`` with W = bf16(q * s).
Oracle: the same product in float64 over the exact bf16 weights, rounded to
bf16.  The kernel accumulates in fp32 in its own order, so an output can land
one bf16 ulp from the oracle; bar: rel-L2 <= 2e-3 (the per-GEMM bar of the
expert tests) and max-abs <= 2 bf16 ulps of the largest output.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import moe as M
from oracle import symmetric as S
from tests._util import to_np

pytestmark = pytest.mark.gpu


def _oracle_linear(x, q, s, bits, group):
    w = S.dequantize_tensor(to_np(q), to_np(s), bits, group, packed=bits == 4, to_bf16=True)
    return S.round_to_bf16((to_np(x).astype(np.float64) @ w.astype(np.float64).T).astype(np.float32))


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("M_,K,N", [(1, 1024, 256), (7, 2048, 512), (33, 1024, 2048), (256, 2048, 1024),
                                     (1000, 1024, 256)])
def test_quant_linear_matches_oracle(bits, M_, K, N):
    from llada_quant_b200.linear import QuantLinear
    g = torch.Generator().manual_seed(M_ + K + N + bits)
    lin = torch.nn.Linear(K, N, bias=False)
    with torch.no_grad():
        lin.weight.copy_(torch.randn(N, K, generator=g) * 0.02)
    m = QuantLinear.from_linear(lin.cuda(), bits=bits, group_size=128)
    assert m.uses_kernel()
    x = torch.randn(M_, K, generator=g).to(torch.bfloat16).cuda()
    out = m(x)
    torch.cuda.synchronize()
    ref = _oracle_linear(x, m.qweight, m.scale, bits, 128)
    got = to_np(out)
    assert M.rel_l2(got, ref) <= 2e-3
    assert M.max_abs(got, ref) <= 2 * 2.0 ** -7 * np.abs(ref).max()
    # the reference algorithm on the same GPU (dequantize + cuBLAS) agrees to the same bar
    ref_gpu = to_np(torch.nn.functional.linear(x, m.dequantize_weight()))
    assert M.rel_l2(got, ref_gpu) <= 2e-3


def test_quant_linear_bias_3d_and_fallback_shapes():
    from llada_quant_b200.linear import QuantLinear
    g = torch.Generator().manual_seed(5)
    lin = torch.nn.Linear(1024, 512, bias=True)
    with torch.no_grad():
        lin.weight.copy_(torch.randn(512, 1024, generator=g) * 0.02)
        lin.bias.copy_(torch.randn(512, generator=g) * 0.1)
    m = QuantLinear.from_linear(lin.cuda(), bits=4, group_size=128)
    x = torch.randn(2, 5, 1024, generator=g).to(torch.bfloat16).cuda()
    out = m(x)
    assert out.shape == (2, 5, 512) and out.dtype == torch.bfloat16
    ref = torch.nn.functional.linear(x, m.dequantize_weight()) + m.bias
    assert M.rel_l2(to_np(out), to_np(ref)) <= 2e-3
    # a shape outside the kernel's rules runs the reference algorithm on the GPU
    odd = QuantLinear.from_linear(torch.nn.Linear(200, 96, bias=False).cuda(), bits=8, group_size=128)
    assert not odd.uses_kernel()
    y = odd(torch.randn(3, 200).cuda())
    assert y.shape == (3, 96)


def test_quant_linear_dequantized_weights_read_back_exactly():
    """One-hot rows read back single weights: y[k, n] = bf16(q[n, k] * s)."""
    from llada_quant_b200 import ops
    from llada_quant_b200 import symmetric as G
    K, N = 1024, 256
    w = (torch.randn(N, K) * 0.05).to(torch.bfloat16).cuda()
    r = G.quantize_tensor(w, bits=4, group_size=128)
    eye = torch.eye(K, dtype=torch.bfloat16).cuda()
    y = ops._quant_linear_impl(eye, r.q, r.scale, 4)
    ref = S.dequantize_tensor(to_np(r.q), to_np(r.scale), 4, 128, packed=True, to_bf16=True).T
    assert np.array_equal(to_np(y).view(np.uint32), np.ascontiguousarray(ref).view(np.uint32))


def test_expert_counts_and_recorder():
    from llada_quant_b200 import symmetric as G
    from llada_quant_b200.fused_moe import moe_layer
    from llada_quant_b200.moe import PackedExperts
    from llada_quant_b200.routing_stats import RoutingRecorder, expert_counts, expert_token_stats
    E, H, I, K = 16, 1024, 512, 2
    g = torch.Generator(device="cuda").manual_seed(0)
    r1 = G.quantize_tensor((torch.randn(E, 2 * I, H, generator=g, device="cuda") * 0.02).to(torch.bfloat16), 4, 128)
    r2 = G.quantize_tensor((torch.randn(E, H, I, generator=g, device="cuda") * 0.02).to(torch.bfloat16), 4, 128)
    packed = PackedExperts(r1.q, r1.scale, r2.q, r2.scale, 4, 128)
    gate = (torch.randn(E, H, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    rec = RoutingRecorder(E, "cuda")
    total = torch.zeros(E, dtype=torch.int64)
    from llada_quant_b200 import ops
    for t in (5, 64, 300):
        x = torch.randn(t, H, generator=g, device="cuda").to(torch.bfloat16)
        moe_layer(x, gate, packed, K, recorder=rec)
        _, ids, _ = ops._route_impl(x, gate, K, None, False)
        total += torch.bincount(ids.reshape(-1).cpu().long(), minlength=E)
        assert torch.equal(expert_counts(ids, E).cpu().long(), torch.bincount(ids.reshape(-1).cpu().long(), minlength=E))
        assert expert_token_stats(ids, E).counts == torch.bincount(ids.reshape(-1).cpu().long(), minlength=E).tolist()
    st = rec.stats()
    assert st.counts == total.tolist() and st.tokens == 369 and rec.calls == 3
