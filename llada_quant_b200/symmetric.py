"""Drop-in mirror of ``LLaDA_Quant.algorithms.symmetric`` on the B200 kernels.

Same names, argument meaning, results and error messages as
``src/LLaDA_Quant/algorithms/symmetric.py``; the arithmetic runs in
``libllada_quant_cuda.so`` (bit-exact codes and scales for amax search; MSE
search equal up to the reference's own near-tie reduction-order effects).
Inputs must be CUDA tensors: there is no CPU path.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence, Tuple

import torch

from . import _lib
from . import ops

SCALE_SEARCH_AMAX = "amax"
SCALE_SEARCH_MSE = "mse"
KNOWN_SCALE_SEARCH = (SCALE_SEARCH_AMAX, SCALE_SEARCH_MSE)
_SCALE_ROUND = {torch.float32: _lib.LLQ_F32, torch.bfloat16: _lib.LLQ_BF16, torch.float16: _lib.LLQ_F16}


def qmax_for_bits(bits: int) -> int:
    """symmetric.py:29-31."""
    return 2 ** (bits - 1) - 1


def qmin_for_bits(bits: int) -> int:
    """symmetric.py:34-36."""
    return -(2 ** (bits - 1))


@dataclass
class QuantResult:
    """Integer weights plus per-group scales (symmetric.py:39-82)."""

    q: torch.Tensor
    scale: torch.Tensor
    bits: int
    group_size: int
    packed: bool = False
    logical_shape: Tuple[int, ...] = ()

    def __post_init__(self) -> None:
        if not self.logical_shape:
            shape = list(self.q.shape)
            if self.packed:
                shape[-1] *= 2
            self.logical_shape = tuple(shape)

    def dequantize(self, dtype: torch.dtype = torch.float32) -> torch.Tensor:
        return dequantize_tensor(self.q, self.scale, self.bits, self.group_size, dtype=dtype,
                                 packed=self.packed)

    def storage_bytes(self) -> int:
        return self.q.numel() * self.q.element_size() + self.scale.numel() * self.scale.element_size()


def validate_int4_layout(shape: Sequence[int], group_size: int) -> None:
    """symmetric.py:93-108."""
    if shape[-1] % 2 != 0:
        raise ValueError(
            f"int4 packing needs an even last dimension, got {tuple(shape)}; "
            "the last axis is the K axis and two values share one byte"
        )
    if group_size != -1 and group_size % 2 != 0:
        raise ValueError(
            f"int4 packing needs an even group_size so groups stay byte-aligned, got {group_size}"
        )


def search_group_scale(w_g: torch.Tensor, bits: int, grid: int = 24, max_shrink: float = 0.5,
                       chunk_elements: int = 64_000_000) -> torch.Tensor:
    """symmetric.py:122-204: per-group MSE-optimal scale, shape ``[..., groups, 1]``.

    ``chunk_elements`` is accepted for signature compatibility; the kernel keeps
    no full-size temporaries, so there is nothing to chunk.
    """
    if grid < 1:
        raise ValueError(f"grid must be >= 1, got {grid}")
    if not 0.0 <= max_shrink < 1.0:
        raise ValueError(f"max_shrink must lie in [0, 1), got {max_shrink}")
    g = w_g.shape[-1]
    flat = w_g.reshape(-1, g)
    _, scale = ops.quantize_pack(flat, bits, g, _lib.LLQ_SEARCH_MSE, grid, float(max_shrink),
                                 _lib.LLQ_F32, False)
    return scale.reshape(*w_g.shape[:-1], 1)


def quantize_tensor(w: torch.Tensor, bits: int = 8, group_size: int = 128,
                    scale_dtype: torch.dtype = torch.float32, pack: bool = True,
                    scale_search: str = SCALE_SEARCH_AMAX, search_grid: int = 24) -> QuantResult:
    """symmetric.py:207-269 on the GPU (one kernel: scale search, rounding, packing)."""
    if bits not in (8, 4):
        raise ValueError(f"bits must be 8 or 4, got {bits}")
    if w.numel() == 0:
        raise ValueError("cannot quantize an empty tensor")
    if bits == 4 and pack:
        validate_int4_layout(w.shape, group_size)
    if w.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        w = w.to(torch.float32)
    if scale_search not in KNOWN_SCALE_SEARCH:
        raise ValueError(
            f"scale_search must be one of {list(KNOWN_SCALE_SEARCH)}, got {scale_search!r}"
        )
    if scale_dtype not in _SCALE_ROUND:
        raise ValueError(f"scale_dtype must be float32, bfloat16 or float16, got {scale_dtype}")
    logical_shape = tuple(w.shape)
    search = _lib.LLQ_SEARCH_MSE if scale_search == SCALE_SEARCH_MSE else _lib.LLQ_SEARCH_AMAX
    q, scale = ops.quantize_pack(w, bits, group_size, search, search_grid, 0.5,
                                 _SCALE_ROUND[scale_dtype], pack)
    eff_group, _ = ops.effective_groups(w.shape[-1], group_size)
    if scale_dtype != torch.float32:
        scale = scale.to(scale_dtype)  # exact: the kernel already rounded it
    return QuantResult(q=q, scale=scale, bits=bits, group_size=eff_group,
                       packed=bits == 4 and pack, logical_shape=logical_shape)


def dequantize_tensor(q: torch.Tensor, scale: torch.Tensor, bits: int, group_size: int,
                      dtype: torch.dtype = torch.float32, packed: bool = False) -> torch.Tensor:
    """symmetric.py:272-293: fp32 ``q * s`` then one cast to ``dtype``."""
    K = q.shape[-1] * (2 if packed else 1)
    if packed and q.dtype != torch.int8:
        raise ValueError(f"packed int4 storage must be int8, got {q.dtype}")
    grouped = not (group_size == -1 or K % group_size != 0)
    expect = K // group_size if grouped else 1
    if scale.shape[-1] != expect or tuple(scale.shape[:-1]) != tuple(q.shape[:-1]):
        # the reference fails in its reshape here; never return a plausible tensor
        raise RuntimeError(
            f"scale shape {tuple(scale.shape)} does not match {expect} group(s) of q "
            f"{tuple(q.shape)} (packed={packed}, group_size={group_size})"
        )
    if dtype not in (torch.float32, torch.float16, torch.bfloat16):
        return ops.dequantize(q, scale, bits, group_size, packed, torch.float32).to(dtype)
    return ops.dequantize(q, scale, bits, group_size, packed, dtype)


def pack_int4(q8: torch.Tensor) -> torch.Tensor:
    """symmetric.py:296-313 (raises on values outside [-8, 7], like the reference)."""
    if q8.shape[-1] % 2 != 0:
        raise ValueError("last dim must be even for int4 packing")
    packed, flag = ops.pack_int4(q8.to(torch.int8))
    if q8.numel() and int(flag.item()) != 0:
        raise ValueError(
            f"int4 packing needs values in [-8, 7], got [{int(q8.min())}, {int(q8.max())}]"
        )
    return packed


def unpack_int4(packed: torch.Tensor) -> torch.Tensor:
    """symmetric.py:316-346."""
    if packed.dtype != torch.int8:
        raise ValueError(f"packed int4 storage must be int8, got {packed.dtype}")
    return ops.unpack_int4(packed)


def storage_bytes(numel: int, bits: int, group_size: int, scale_bytes: int = 4) -> int:
    """symmetric.py:349-362."""
    if bits == 8:
        value_bytes = numel
    elif bits == 4:
        value_bytes = numel // 2
    else:
        raise ValueError(f"bits must be 8 or 4, got {bits}")
    groups = 1 if group_size == -1 else max(1, numel // group_size)
    return value_bytes + groups * scale_bytes


def block_k_is_scale_aligned(block_k: int, group_size: int) -> bool:
    """symmetric.py:365-378."""
    if group_size == -1:
        return True
    if block_k <= 0 or group_size <= 0:
        return False
    return block_k % group_size == 0 or group_size % block_k == 0


def validate_block_k_alignment(block_k: int, group_size: int) -> None:
    """symmetric.py:381-394."""
    if not block_k_is_scale_aligned(block_k, group_size):
        raise ValueError(
            f"BLOCK_SIZE_K={block_k} cannot address group_size={group_size} scales "
            "exactly: one must divide the other, or a K-tile straddles a group "
            "boundary and half of it is dequantized with the wrong scale"
        )
