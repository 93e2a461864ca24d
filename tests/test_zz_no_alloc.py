"""GPU test of llq_fused_moe_packed_noalloc, the layer entry point that allocates nothing.

It exists for callers that cannot allocate device memory -- a plugin living in
a framework that owns the allocator, a runtime that reserved all memory up
front.  The test calls it through the C ABI (ctypes), twice in a row, and
checks each output against the workspace-taking llq_fused_moe_packed on the
same inputs, within the layer tolerance the other MoE tests use (rel-L2 <= 3e-3,
max-abs <= 2 bf16 ulps of the largest output).  This file sorts last so that a
failure here never hides the other tests' results.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import moe as M
from tests._util import random_routing, synthetic_layer, synthetic_tokens, to_np

pytestmark = pytest.mark.gpu


def _close(out, ref):
    rel = M.rel_l2(out, ref)
    assert rel <= 3e-3, rel
    assert M.max_abs(out, ref) <= 2 * 2.0 ** -7 * max(np.abs(ref).max(), 1e-6)


@pytest.mark.parametrize("T,E,H,I,k,bits,fast", [(256, 64, 2048, 1024, 8, 4, False),
                                                  (256, 64, 2048, 1024, 8, 4, True),
                                                  (200, 16, 1024, 512, 2, 8, False)])
def test_noalloc_matches_workspace_entry_point_twice(T, E, H, I, k, bits, fast):
    from llada_quant_b200 import _lib, ops
    from llada_quant_b200 import symmetric as G

    lib = _lib.load()
    w1, w2 = synthetic_layer(E, H, I, seed=7)
    r1 = G.quantize_tensor(w1.cuda(), bits=bits, group_size=128)
    r2 = G.quantize_tensor(w2.cuda(), bits=bits, group_size=128)
    impl = _lib.LLQ_GEMM_TCGEN05_FAST if fast else _lib.LLQ_GEMM_AUTO
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        x = synthetic_tokens(T, H, seed=11 + call).cuda()
        tw, ids = random_routing(T, E, k, seed=13 + call)
        tw_d, ids_d = torch.from_numpy(tw).cuda(), torch.from_numpy(ids).cuda()
        ref = ops.fused_moe_packed(x, r1.q, r1.scale, r2.q, r2.scale, tw_d, ids_d, bits, impl)
        out = torch.full((T, H), float("nan"), dtype=torch.bfloat16, device="cuda")
        rc = lib.llq_fused_moe_packed_noalloc(
            x.data_ptr(), r1.q.data_ptr(), r1.scale.data_ptr(), r2.q.data_ptr(), r2.scale.data_ptr(),
            tw_d.data_ptr(), ids_d.data_ptr(), T, E, H, I, k, bits, 128, out.data_ptr(),
            impl, stream)
        assert rc == 0, lib.llq_last_error()
        torch.cuda.synchronize()
        _close(to_np(out), to_np(ref))


def test_noalloc_rejects_sizes_beyond_its_scratch():
    from llada_quant_b200 import _lib
    lib = _lib.load()
    rc = lib.llq_fused_moe_packed_noalloc(None, None, None, None, None, None, None, 4096, 64, 2048,
                                          1024, 8, 4, 128, None, 0, None)
    assert rc == _lib.LLQ_EINVAL
    assert b"exceeds its fixed scratch" in lib.llq_last_error()


def test_noalloc_rejects_fast_mode_outside_its_shapes():
    """The scale-after-MMA mode is INT4 only; an INT8 request is refused before any launch."""
    from llada_quant_b200 import _lib
    lib = _lib.load()
    rc = lib.llq_fused_moe_packed_noalloc(None, None, None, None, None, None, None, 16, 16, 1024,
                                          512, 2, 8, 128, None, _lib.LLQ_GEMM_TCGEN05_FAST, None)
    assert rc == _lib.LLQ_EUNSUPPORTED
    assert b"LLQ_GEMM_TCGEN05_FAST" in lib.llq_last_error()
