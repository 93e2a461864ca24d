"""Test helpers: bf16 <-> numpy, seeded synthetic MoE weights."""

from __future__ import annotations

import numpy as np
import torch


def to_np(t: torch.Tensor) -> np.ndarray:
    """float view of a (bf16/fp16/fp32) tensor as float32 numpy; ints unchanged."""
    t = t.detach().cpu()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.float().numpy()
    return t.numpy()


def bf16_from_np(a: np.ndarray, device="cuda") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16).to(device)


def synthetic_layer(E, H, I, seed=0, device="cpu"):
    """w1 [E,2I,H], w2 [E,H,I] ~ N(0, 0.02) in bf16, seeded like the reference's fixtures."""
    g = torch.Generator().manual_seed(seed)
    w1 = (torch.randn(E, 2 * I, H, generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(E, H, I, generator=g) * 0.02).to(torch.bfloat16)
    return w1.to(device), w2.to(device)


def synthetic_tokens(T, H, seed=2, device="cpu"):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(T, H, generator=g).to(torch.bfloat16).to(device)


def random_routing(T, E, k, seed=3, skew=None):
    """Distinct expert ids per token; ``skew`` concentrates tokens on few experts."""
    rng = np.random.default_rng(seed)
    ids = np.empty((T, k), dtype=np.int32)
    p = None
    if skew is not None:
        p = np.arange(1, E + 1, dtype=np.float64) ** (-skew)
        p /= p.sum()
    for t in range(T):
        ids[t] = rng.choice(E, size=k, replace=False, p=p)
    w = rng.random((T, k)).astype(np.float32) / k
    return w, ids
