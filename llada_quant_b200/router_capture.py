"""Per-layer routing captured from the router kernel itself.

The trajectory tools of LLaDA_Quant read each MoE block's top-k expert ids
through ``RouterCapture`` (src/LLaDA_Quant/trajectory/llada.py:157-268).  The
external fused block never exposes its ``topk_ids``, so that class stashes the
block input in a forward pre-hook and runs the router a second time
(``gate`` -> fp32 softmax -> top-k) for every captured layer.

Here the routing comes from the router kernel of the layer call itself:
:func:`llada_quant_b200.fused_moe.moe_layer` hands its ``topk_ids`` and bf16
logits to a :class:`RouterCapture` passed as ``capture=`` (with the layer's
name), so the expert choice that is recorded is, by construction, the one the
expert GEMMs consumed -- no recomputation, no second router pass.  The
accessors match the reference class: ``topk_ids`` (global expert ids, int64
``[tokens, top_k]`` on the host), ``gates`` (raw router logits, fp32
``[tokens, num_experts]`` on the host), ``layer_names``, ``clear``, ``remove``
and use as a context manager.  Captured tensors stay on the device until an
accessor is read.

Equal softmax values: the kernel orders them by the smaller expert id; torch's
``topk`` leaves their order unspecified.
"""

from __future__ import annotations

from typing import Dict, List, Tuple

import torch


class RouterCapture:
    """Collects each layer's routing from the kernel's own outputs (see module docstring)."""

    def __init__(self) -> None:
        self._captured: Dict[str, Tuple[torch.Tensor, torch.Tensor]] = {}
        self._open = True

    def record(self, name: str, topk_ids: torch.Tensor, logits: torch.Tensor) -> None:
        """Keep one layer call's ``topk_ids`` ``[T, k]`` and router ``logits`` ``[T, E]`` (the
        most recent call per name wins, as with a forward of the reference's hooked model)."""
        if not self._open:
            return
        self._captured[name] = (topk_ids.detach(), logits.detach())

    @property
    def topk_ids(self) -> Dict[str, torch.Tensor]:
        """Per-layer ``[tokens, top_k]`` expert ids (int64, host) from the most recent call."""
        return {n: ids.to(torch.int64).cpu() for n, (ids, _) in self._captured.items()}

    @property
    def gates(self) -> Dict[str, torch.Tensor]:
        """Per-layer raw router logits ``[tokens, num_experts]`` (fp32, host)."""
        return {n: lg.float().cpu() for n, (_, lg) in self._captured.items()}

    @property
    def layer_names(self) -> List[str]:
        return sorted(self._captured)

    def clear(self) -> None:
        self._captured.clear()

    def remove(self) -> None:
        """Stop recording (the reference detaches its hooks here).  Safe to call twice."""
        self._open = False

    def __enter__(self) -> "RouterCapture":
        return self

    def __exit__(self, *exc: object) -> None:
        self.remove()
