"""Routing statistics from the kernels' own routing (mirrors analysis/moe_regime.py:150-213).

``ExpertTokenStats`` and ``expert_token_stats`` keep the reference's fields,
properties and error message.  On CUDA the per-expert counts come from the
package's alignment kernel (the same expert offsets the expert GEMMs consume),
so no pre-hook has to recompute the router; ``RoutingRecorder`` accumulates
them across layer calls on the device and is read once at the end
(``fused_moe.moe_layer(..., recorder=...)``).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import List

import torch

from . import ops


@dataclass
class ExpertTokenStats:
    """Per-expert row counts of real routing, with the summary fields and ``to_dict`` keys
    of the reference report (analysis/moe_regime.py:150-194)."""

    tokens: int
    top_k: int
    num_experts: int
    counts: List[int] = field(default_factory=list)

    @property
    def active_experts(self) -> int:
        """Experts that received at least one row."""
        return sum(c > 0 for c in self.counts)

    @property
    def mean(self) -> float:
        return float(sum(self.counts)) / len(self.counts) if self.counts else 0.0

    @property
    def imbalance(self) -> float:
        """Busiest expert's rows divided by the mean; the busiest expert bounds a layer's
        time, so 1.0 means no expert waits on another."""
        m = self.mean
        return max(self.counts) / m if self.counts and m else 1.0

    def percentile(self, p: float) -> float:
        """Nearest-rank percentile of the counts (index rounded on the sorted list)."""
        if not self.counts:
            return 0.0
        s = sorted(self.counts)
        i = int(round(p / 100.0 * (len(s) - 1)))
        return float(s[min(max(i, 0), len(s) - 1)])

    def to_dict(self) -> dict:
        c = self.counts
        return {"tokens": self.tokens, "top_k": self.top_k, "num_experts": self.num_experts,
                "active_experts": self.active_experts, "min": min(c) if c else 0,
                "p50": self.percentile(50), "mean": round(self.mean, 2), "p90": self.percentile(90),
                "p99": self.percentile(99), "max": max(c) if c else 0,
                "imbalance_max_over_mean": round(self.imbalance, 3)}


def expert_counts(topk_ids: torch.Tensor, num_experts: int) -> torch.Tensor:
    """Per-expert row counts on the device (int32 ``[E]``), from one alignment kernel."""
    if topk_ids.dim() != 2:
        raise ValueError(f"topk_ids must be [tokens, top_k], got {tuple(topk_ids.shape)}")
    offsets, _ = ops._moe_align_impl(topk_ids.to(torch.int32), num_experts)
    return offsets[1:] - offsets[:-1]


def expert_token_stats(topk_ids: torch.Tensor, num_experts: int) -> ExpertTokenStats:
    """moe_regime.py:197-213.  CUDA ids are counted by the alignment kernel; host ids (the
    analysis tools' captured routing) by ``bincount`` as in the reference."""
    if topk_ids.dim() != 2:
        raise ValueError(f"topk_ids must be [tokens, top_k], got {tuple(topk_ids.shape)}")
    if topk_ids.is_cuda:
        counts = expert_counts(topk_ids, num_experts).tolist()
    else:
        counts = torch.bincount(topk_ids.reshape(-1), minlength=num_experts).tolist()
    return ExpertTokenStats(tokens=topk_ids.shape[0], top_k=topk_ids.shape[1], num_experts=num_experts,
                            counts=counts)


class RoutingRecorder:
    """Per-expert loads summed over layer calls, kept on the device until read."""

    def __init__(self, num_experts: int, device) -> None:
        self.num_experts = num_experts
        self.counts = torch.zeros(num_experts, dtype=torch.int64, device=device)
        self.tokens = 0
        self.calls = 0
        self.top_k = 0

    def record_offsets(self, offsets: torch.Tensor, tokens: int, top_k: int) -> None:
        """Add one call's expert offsets ``[E + 1]`` (stream-ordered, no host read)."""
        self.counts += (offsets[1:self.num_experts + 1] - offsets[:self.num_experts]).to(torch.int64)
        self.tokens += tokens
        self.top_k = top_k
        self.calls += 1

    def stats(self) -> ExpertTokenStats:
        return ExpertTokenStats(tokens=self.tokens, top_k=self.top_k, num_experts=self.num_experts,
                                counts=self.counts.tolist())

    def reset(self) -> None:
        self.counts.zero_()
        self.tokens = self.calls = 0
