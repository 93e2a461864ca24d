"""llada_quant_b200 -- B200-native (sm_100a) kernels for LLaDA_Quant's quantized MoE path.

Three parts, each behind a PyTorch custom op over the C ABI in
``include/llada_quant.h``:

* quantize-and-pack (amax and MSE scale search), bit-exact with
  ``LLaDA_Quant.algorithms.symmetric``;
* the routed W4A16/W8A16 expert FFN over the frozen packed buffers
  (GEMM1 with the SiLU epilogue, GEMM2 with the routed weight);
* router top-k, expert alignment, permute and combine.

``symmetric`` and ``moe`` mirror the reference modules of the same names;
``fused_moe`` keeps the external ``fused_moe`` signature.  CUDA only: no CPU
fallback exists.
"""

from __future__ import annotations

from . import _lib  # noqa: F401

__all__ = ["ops", "symmetric", "moe", "fused_moe"]
__version__ = "0.1.0"


def __getattr__(name):
    if name in __all__:
        import importlib
        return importlib.import_module(f"{__name__}.{name}")
    raise AttributeError(name)
