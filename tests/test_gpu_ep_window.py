"""Peer-memory expert parallelism (EPWindow) on one GPU.

With a group of one the window is this GPU's own memory, so every phase of the
protocol runs -- dispatch stores and flags, the masked receive alignment, the
GEMM2 scatter into the back region with its last-CTA flag, the waiting
combine -- and every wait is satisfied by a kernel that already completed on
the same stream.  The result must equal the single-GPU layer bit for bit.
The bounded wait is checked by asking the combine for an epoch that no kernel
ever publishes: it must give up after the limit, record its code in the
device error word and leave the context usable.
"""

from __future__ import annotations

import pytest
import torch

from llada_quant_b200 import ops
from llada_quant_b200 import symmetric as G
from llada_quant_b200.ep import EPWindow, set_wait_timeout_ms
from llada_quant_b200.fused_moe import IMPL
from llada_quant_b200.moe import PackedExperts

pytestmark = pytest.mark.gpu


def _layer(E, H, I, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    w1 = (torch.randn(E, 2 * I, H, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(E, H, I, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    gate = (torch.randn(E, H, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    r1 = G.quantize_tensor(w1, bits=4, group_size=128)
    r2 = G.quantize_tensor(w2, bits=4, group_size=128)
    return PackedExperts(r1.q, r1.scale, r2.q, r2.scale, 4, 128), gate


@pytest.mark.parametrize("gemm", ["tcgen05", "tcgen05_fast"])
@pytest.mark.parametrize("T", [1, 77, 256])
def test_window_equals_single_gpu_layer(gemm, T):
    E, H, I, K = 16, 1024, 512, 4
    packed, gate = _layer(E, H, I)
    win = EPWindow(256, K, H, 0, 1, torch.device("cuda", 0))
    try:
        for step in range(3):  # the window is reused across calls (epochs 1..3)
            x = torch.randn(T, H, device="cuda", generator=torch.Generator(device="cuda").manual_seed(step))
            x = x.to(torch.bfloat16)
            tw, ids, _ = ops._route_impl(x, gate, K, None, False)
            got = win.layer(x, tw, ids, packed, IMPL[gemm])
            ref = ops._fused_moe_packed_impl(x, packed.qw1, packed.sw1, packed.qw2, packed.sw2, tw, ids, 4,
                                             IMPL[gemm])
            torch.cuda.synchronize()
            assert ops.device_error() == 0
            assert torch.equal(got, ref), (step, (got.float() - ref.float()).abs().max().item())
    finally:
        win.close()


def test_window_rejects_overflow():
    E, H, I, K = 16, 1024, 512, 4
    packed, gate = _layer(E, H, I)
    win = EPWindow(8, K, H, 0, 1, torch.device("cuda", 0))
    try:
        x = torch.randn(9, H, device="cuda").to(torch.bfloat16)
        tw, ids, _ = ops._route_impl(x, gate, K, None, False)
        with pytest.raises(ValueError):
            win.layer(x, tw, ids, packed, IMPL["tcgen05"])
    finally:
        win.close()


def test_combine_wait_gives_up_on_a_missing_flag():
    from llada_quant_b200._lib import check, load
    H, K, T = 1024, 4, 16
    win = EPWindow(T, K, H, 0, 1, torch.device("cuda", 0))
    set_wait_timeout_ms(200)
    try:
        ops.clear_device_error()
        inv = torch.full((T * K,), -1, dtype=torch.int32, device="cuda")
        out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
        # epoch 7 is never published on this window: the wait must run out
        check(load().llq_ep_combine_wait(win.base, 0, 1, win.cap, 7, inv.data_ptr(), T, K, H, out.data_ptr(),
                                         torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
        assert ops.device_error() == 0x503
        assert torch.count_nonzero(out.float()) == 0  # entries never sent add nothing
        ops.clear_device_error()
        # the context is still usable
        y = torch.ones(4, device="cuda") * 2
        assert y.sum().item() == 8
    finally:
        set_wait_timeout_ms(5000)
        ops.clear_device_error()
        win.close()
