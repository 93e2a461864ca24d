"""``fused_moe`` with the external signature, running on PACKED weights.

The external inference repository calls
``fused_moe(hidden_states, w1, w2, gating_output, topk_ids, fuse_silu=None)``
(INFERENCE_REPO_CHANGES.md:109-111) with ``w1``/``w2`` read from the block's
PACKED-mode properties, which dequantize to BF16 on every access
(src/LLaDA_Quant/runtime/moe.py:199-216).  Here ``w1`` may instead be the
block's :class:`~llada_quant_b200.moe.PackedExperts` handle
(``block.packed_experts()``; pass ``w2=None``): the layer then runs
align -> permute -> W4A16/W8A16 GEMM1 with the SiLU epilogue -> GEMM2 with the
routed weight -> combine, reading the packed bytes directly.

``gating_output`` is the router logits ``[T, E]``.  The routed weights are
``softmax(gating_output, fp32)`` at ``topk_ids`` (no renormalisation unless
asked): the external kernel's exact weighting is not visible in the reference
tree, so this is a stated choice.  ``fuse_silu`` must be None or True: the
SiLU epilogue is always fused.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _lib, ops
from .moe import PackedExperts

IMPL = {"auto": _lib.LLQ_GEMM_AUTO, "tcgen05": _lib.LLQ_GEMM_TCGEN05, "simt": _lib.LLQ_GEMM_SIMT,
        "tcgen05_fast": _lib.LLQ_GEMM_TCGEN05_FAST}


def routing_weights(gating_output: torch.Tensor, topk_ids: torch.Tensor,
                    renormalize: bool = False) -> torch.Tensor:
    """fp32 softmax of the logits gathered at ``topk_ids`` (one fused kernel would be
    ``ops.route_topk``; this form keeps caller-chosen ids)."""
    p = torch.softmax(gating_output.float(), dim=-1)
    w = torch.gather(p, 1, topk_ids.long())
    if renormalize:
        w = w / w.sum(dim=-1, keepdim=True)
    return w


def fused_moe(hidden_states: torch.Tensor, w1, w2, gating_output: Optional[torch.Tensor],
              topk_ids: Optional[torch.Tensor], fuse_silu: Optional[bool] = None, *,
              top_k: Optional[int] = None, topk_weights: Optional[torch.Tensor] = None,
              renormalize: bool = False, impl: str = "auto") -> torch.Tensor:
    """Routed expert FFN over packed experts; returns bf16 ``[T, H]``."""
    if fuse_silu is False:
        raise ValueError("the packed kernels always fuse SiLU into GEMM1 (fuse_silu=False is not offered)")
    if not isinstance(w1, PackedExperts):
        raise TypeError(
            "fused_moe here consumes packed experts: pass block.packed_experts() as w1 (and "
            "w2=None); dense BF16 weights are the REFERENCE-mode path this replaces"
        )
    packed = w1
    shape = hidden_states.shape
    x = hidden_states.reshape(-1, shape[-1]).to(torch.bfloat16)
    if topk_ids is None:
        if gating_output is None or top_k is None:
            raise ValueError("pass topk_ids, or gating_output and top_k")
        topk_weights, topk_ids = ops.route_topk(gating_output.reshape(-1, gating_output.shape[-1]),
                                                top_k, None, renormalize)
    elif topk_weights is None:
        if gating_output is None:
            raise ValueError("pass gating_output or topk_weights with topk_ids")
        topk_weights = routing_weights(gating_output.reshape(-1, gating_output.shape[-1]),
                                       topk_ids, renormalize)
    out = ops.fused_moe_packed(x, packed.qw1, packed.sw1, packed.qw2, packed.sw2,
                               topk_weights.reshape(x.shape[0], -1),
                               topk_ids.reshape(x.shape[0], -1), packed.bits, IMPL[impl])
    return out.reshape(shape)


def moe_layer(x: torch.Tensor, gate_w: torch.Tensor, packed: PackedExperts, top_k: int,
              bias: Optional[torch.Tensor] = None, renormalize: bool = False,
              impl: str = "auto", recorder=None, capture=None, name: str = "") -> torch.Tensor:
    """Router + routed experts, the forward of a PACKED LLaDA MoE block: one router
    kernel (bf16 logits, fp32 softmax, top-k) then :func:`fused_moe`.  With a
    ``routing_stats.RoutingRecorder`` the call's per-expert loads are added to it on
    the device, from the expert offsets the GEMMs used; with a
    ``router_capture.RouterCapture`` the router kernel's own ids and logits are
    recorded under ``name``."""
    # eager hot path: one library call (router through combine), no per-call dispatcher cost
    out, topk_w, topk_ids, logits = ops._moe_block_packed_impl(
        x, gate_w, bias, renormalize, packed.qw1, packed.sw1, packed.qw2, packed.sw2, top_k, packed.bits,
        IMPL[impl], want_logits=capture is not None)
    if capture is not None:
        capture.record(name, topk_ids, logits)
    if recorder is not None:
        E = packed.num_experts
        T = x.shape[0]
        ws = ops.moe_workspace(T, top_k, E, packed.hidden, packed.intermediate, x.device)
        recorder.record_offsets(ws[:4 * (E + 1)].view(torch.int32), T, top_k)  # offsets lead the workspace
    return out
