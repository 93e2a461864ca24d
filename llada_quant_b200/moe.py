"""Mirror of ``LLaDA_Quant.runtime.moe``: PACKED residency served by the B200 kernels.

Same buffers (``_qw1``/``_sw1``/``_qw2``/``_sw2``), metadata attribute and
generated ``PackedQuant<Cls>`` subclass as ``src/LLaDA_Quant/runtime/moe.py``
(:41-45, :147-169, :246-286), so checkpoints and callers see no change:

* ``block.w1`` / ``block.w2`` still return a freshly dequantized bf16 tensor on
  every access (runtime/moe.py:199-216) -- now one CUDA kernel
  (``llada_quant::dequantize``) instead of the eager unpack/upcast/scale/cast
  chain;
* new: ``block.packed_experts()`` hands the packed buffers to
  :func:`llada_quant_b200.fused_moe.fused_moe`, which runs the routed expert
  FFN straight from them, so the forward never materialises BF16 weights.
"""

from __future__ import annotations

import functools

from dataclasses import dataclass
from typing import Dict, Tuple

import torch
import torch.nn as nn

from .symmetric import QuantResult, dequantize_tensor, quantize_tensor

W1 = "w1"
W2 = "w2"
EXPERT_PARAM_NAMES = (W1, W2)
PACKED_BUFFERS = ("_qw1", "_sw1", "_qw2", "_sw2")
QUANT_META_ATTR = "_llada_quant_meta"


@dataclass
class QuantExpertWeights:
    """Packed values + scales for one MoE layer's ``w1`` and ``w2`` (runtime/moe.py:48-79)."""

    w1: QuantResult
    w2: QuantResult

    @classmethod
    def quantize(cls, w1: torch.Tensor, w2: torch.Tensor, bits: int = 8, group_size: int = 128,
                 scale_dtype: torch.dtype = torch.float32, scale_search: str = "amax",
                 search_grid: int = 24) -> "QuantExpertWeights":
        kw = dict(bits=bits, group_size=group_size, scale_dtype=scale_dtype,
                  scale_search=scale_search, search_grid=search_grid)
        return cls(w1=quantize_tensor(w1, **kw), w2=quantize_tensor(w2, **kw))

    def dequantize(self, dtype: torch.dtype = torch.bfloat16) -> Tuple[torch.Tensor, torch.Tensor]:
        return self.w1.dequantize(dtype=dtype), self.w2.dequantize(dtype=dtype)

    def storage_bytes(self) -> int:
        return self.w1.storage_bytes() + self.w2.storage_bytes()


def quant_result_from_buffers(q: torch.Tensor, scale: torch.Tensor, bits: int) -> QuantResult:
    """runtime/moe.py:82-102: the group size is derived from the scale shape."""
    packed = bits == 4
    k_logical = q.shape[-1] * (2 if packed else 1)
    num_groups = scale.shape[-1] if scale.dim() else 1
    group_size = -1 if num_groups <= 1 else k_logical // num_groups
    return QuantResult(q=q, scale=scale, bits=bits, group_size=group_size, packed=packed,
                       logical_shape=tuple(list(q.shape[:-1]) + [k_logical]))


@dataclass(frozen=True)
class PackedExperts:
    """The packed buffers of one fused expert block, as the kernels consume them."""

    qw1: torch.Tensor
    sw1: torch.Tensor
    qw2: torch.Tensor
    sw2: torch.Tensor
    bits: int
    group_size: int

    @property
    def num_experts(self) -> int:
        return self.qw1.shape[0]

    @property
    def hidden(self) -> int:
        return self.qw2.shape[1]

    @property
    def intermediate(self) -> int:
        return self.qw1.shape[1] // 2


def attach_packed_buffers(block: nn.Module, weights: QuantExpertWeights,
                          compute_dtype: torch.dtype, compile_dequant: bool = False) -> None:
    """runtime/moe.py:147-169."""
    block.register_buffer("_qw1", weights.w1.q, persistent=True)
    block.register_buffer("_sw1", weights.w1.scale, persistent=True)
    block.register_buffer("_qw2", weights.w2.q, persistent=True)
    block.register_buffer("_sw2", weights.w2.scale, persistent=True)
    setattr(block, QUANT_META_ATTR, {
        "bits": weights.w1.bits,
        "group_size": weights.w1.group_size,
        "packed": weights.w1.packed,
        "compute_dtype": compute_dtype,
        "compile_dequant": compile_dequant,
        "logical_shape": {W1: weights.w1.logical_shape, W2: weights.w2.logical_shape},
    })


def _meta(self: nn.Module) -> dict:
    meta = getattr(self, QUANT_META_ATTR, None)
    if meta is None:
        raise RuntimeError(
            f"{type(self).__name__} is served from packed buffers but "
            f"{QUANT_META_ATTR} is missing. Reload through "
            "load_quantized_weights() so the quantization config is applied."
        )
    return meta


def _packed_expert_weight(self: nn.Module, which: str) -> torch.Tensor:
    """Dense ``compute_dtype`` w1 or w2, made by one dequantize kernel launch on every access
    (so each access returns a new tensor, as the PACKED property of runtime/moe.py:199-216)."""
    meta = _meta(self)
    suffix = which[-1]
    return dequantize_tensor(getattr(self, f"_qw{suffix}"), getattr(self, f"_sw{suffix}"),
                             meta["bits"], meta["group_size"], dtype=meta["compute_dtype"],
                             packed=meta["packed"])


def _packed_experts(self: nn.Module) -> PackedExperts:
    meta = _meta(self)
    return PackedExperts(self._qw1, self._sw1, self._qw2, self._sw2, meta["bits"], meta["group_size"])


WEIGHT_MUTATING_METHODS = ("load_state_dict_from_unfused",)


def _blocked_method(name: str):
    def blocked(self, *args, **kwargs):
        raise RuntimeError(
            f"{type(self).__mro__[1].__name__}.{name}() writes into w1/w2 in place, "
            "but this block is quantized in PACKED mode where those are derived "
            "from packed buffers -- the write would be silently discarded.\n"
            "Load the weights first, then quantize:\n"
            f"    block.{name}(...)\n"
            "    quantize_model(model, config)"
        )

    blocked.__name__ = name
    return blocked


@functools.lru_cache(maxsize=None)
def _packed_subclass(cls: type) -> type:
    """Build (once per block class) the ``PackedQuant<Cls>`` subclass whose ``w1``/``w2``
    are read-only properties over the packed buffers (the reference's generated class,
    runtime/moe.py:246-269 -- name and behaviour are part of its checkpoint contract),
    with the in-place loaders refused and a ``packed_experts()`` handle added."""
    attrs = {
        "_llada_quant_packed": True,
        "_packed_expert_weight": _packed_expert_weight,
        "packed_experts": _packed_experts,
        "__doc__": f"{cls.__name__} with w1/w2 served from packed integer buffers.",
    }
    attrs.update({w: property(functools.partial(_packed_expert_weight, which=w)) for w in (W1, W2)})
    attrs.update({m: _blocked_method(m) for m in WEIGHT_MUTATING_METHODS if hasattr(cls, m)})
    return type(f"PackedQuant{cls.__name__}", (cls,), attrs)


def _packed_class(cls: type) -> type:
    """The packed subclass of ``cls`` (``cls`` itself when it already is one)."""
    return cls if getattr(cls, "_llada_quant_packed", False) else _packed_subclass(cls)


def install_packed_expert_access(block: nn.Module) -> None:
    """Switch ``block`` to packed serving in place: drop its dense expert parameters and
    re-class it (runtime/moe.py:272-286); the packed buffers must already be attached."""
    absent = [n for n in PACKED_BUFFERS if not hasattr(block, n)]
    if absent:
        raise RuntimeError(f"cannot install packed access, missing buffers: {absent}")
    for n in EXPERT_PARAM_NAMES:
        block._parameters.pop(n, None)
    block.__class__ = _packed_class(type(block))


def is_packed_expert_block(module: nn.Module) -> bool:
    """True for blocks re-classed by :func:`install_packed_expert_access` (runtime/moe.py:289-291)."""
    return bool(getattr(type(module), "_llada_quant_packed", False))


def expert_storage_bytes(block: nn.Module) -> int:
    """Device bytes of the block's packed expert buffers, codes and scales (runtime/moe.py:294-301)."""
    bufs = (getattr(block, n, None) for n in PACKED_BUFFERS)
    return sum(b.numel() * b.element_size() for b in bufs if b is not None)
