"""Drop-in quantized linear module on the B200 kernels (mirrors runtime/linear.py).

Same buffers, constructor, ``from_linear``, ``dequantize_weight``,
``storage_bytes`` and call semantics as the reference ``QuantLinear``
(runtime/linear.py:29-131); its checkpoints load unchanged.  The forward reads
the packed ``qweight`` directly: ``bf16(x . bf16(q * s)^T)`` with fp32
accumulation on the tcgen05 expert kernel run as a single dense expert
(``llq_quant_linear``), instead of materialising the BF16 weight every call
(runtime/linear.py:127-131).  Shapes outside that kernel's rules (K % 128,
K <= 2048, out_features % 256, group % 128) and non-bf16 compute dtypes take
the reference algorithm on the GPU (dequantize kernel + ``F.linear``).  There is
no CPU path: CPU tensors raise.
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops
from .symmetric import QuantResult, dequantize_tensor, quantize_tensor, validate_int4_layout


def kernel_supports(in_features: int, out_features: int, group_size: int) -> bool:
    """Whether ``llq_quant_linear`` covers this layer (see include/llada_quant.h)."""
    grouped = group_size != -1 and in_features % group_size == 0
    if grouped and group_size % 128 != 0:
        return False
    return in_features % 128 == 0 and in_features <= 2048 and out_features % 256 == 0


class QuantLinear(nn.Module):
    """Quantized replacement for ``nn.Linear`` (runtime/linear.py:29-131).

    ``qweight`` is ``[out_features, in_features]`` int8 at 8 bits, or
    ``[out_features, in_features // 2]`` at 4 bits; ``scale`` is
    ``[out_features, num_groups]`` fp32 (groups along K).
    """

    def __init__(self, in_features: int, out_features: int, bits: int = 8, group_size: int = 128,
                 compute_dtype: torch.dtype = torch.bfloat16, bias: bool = False,
                 scale_dtype: torch.dtype = torch.float32) -> None:
        super().__init__()
        if bits not in (8, 4):
            raise ValueError(f"bits must be 8 or 4, got {bits}")
        if bits == 4:
            validate_int4_layout((out_features, in_features), group_size)
        self.in_features = in_features
        self.out_features = out_features
        self.bits = bits
        self.group_size = group_size
        self.compute_dtype = compute_dtype
        self.packed = bits == 4
        stored_cols = in_features // 2 if self.packed else in_features
        self.register_buffer("qweight", torch.empty(out_features, stored_cols, dtype=torch.int8))
        self.register_buffer("scale", torch.empty(out_features, self._num_groups(), dtype=scale_dtype))
        if bias:
            self.register_buffer("bias", torch.zeros(out_features, dtype=compute_dtype))
        else:
            self.register_buffer("bias", None)

    def _num_groups(self) -> int:
        if self.group_size == -1 or self.in_features % self.group_size != 0:
            return 1
        return self.in_features // self.group_size

    @classmethod
    def from_linear(cls, linear: nn.Linear, bits: int = 8, group_size: int = 128,
                    compute_dtype: torch.dtype = torch.bfloat16, scale_search: str = "amax",
                    search_grid: int = 24) -> "QuantLinear":
        """runtime/linear.py:76-102: quantize the (fp32) weight on its GPU."""
        w = linear.weight.detach().to(torch.float32)
        q: QuantResult = quantize_tensor(w, bits=bits, group_size=group_size, scale_search=scale_search,
                                         search_grid=search_grid)
        out = cls(in_features=linear.in_features, out_features=linear.out_features, bits=bits,
                  group_size=group_size, compute_dtype=compute_dtype, bias=linear.bias is not None)
        out = out.to(w.device)
        out.qweight.copy_(q.q)
        out.scale.copy_(q.scale)
        if linear.bias is not None:
            out.bias.copy_(linear.bias.detach())
        return out

    def dequantize_weight(self) -> torch.Tensor:
        """The weight as a dense ``compute_dtype`` matrix (one dequantize kernel launch)."""
        return dequantize_tensor(self.qweight, self.scale, self.bits, self.group_size,
                                 dtype=self.compute_dtype, packed=self.packed)

    def storage_bytes(self) -> int:
        """Bytes held on the device by qweight, scale and (if any) bias."""
        tensors = [self.qweight, self.scale] + ([self.bias] if self.bias is not None else [])
        return sum(t.numel() * t.element_size() for t in tensors)

    def extra_repr(self) -> str:
        layout = "int4x2" if self.packed else f"int{self.bits}"
        return (f"{self.in_features} -> {self.out_features}, {layout} codes, "
                f"group {self.group_size}, B200 kernel {'on' if self.uses_kernel() else 'off'}")

    def uses_kernel(self) -> bool:
        return (self.compute_dtype == torch.bfloat16 and self.scale.dtype == torch.float32
                and kernel_supports(self.in_features, self.out_features, self.group_size))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not x.is_cuda:
            raise RuntimeError("llada_quant_b200.QuantLinear runs on CUDA tensors only (no CPU path)")
        xs = x.to(self.compute_dtype)
        if self.uses_kernel():
            lead = xs.shape[:-1]
            out = ops._quant_linear_impl(xs.reshape(-1, self.in_features), self.qweight, self.scale,
                                         self.bits).reshape(*lead, self.out_features)
        else:
            out = F.linear(xs, self.dequantize_weight())
        if self.bias is not None:
            out = out + self.bias
        return out
