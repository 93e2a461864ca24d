"""ctypes binding of ``libllada_quant_cuda.so`` (the C ABI in ``include/llada_quant.h``).

The library is built in-tree by ``llada_quant_b200.build``.  There is no CPU
fallback anywhere in the package: if the library is missing, or a tensor is
not on a CUDA device, the call raises.
"""

from __future__ import annotations

import ctypes
import os
from ctypes import c_double, c_int, c_int64, c_size_t, c_void_p

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libllada_quant_cuda.so")

LLQ_OK, LLQ_EINVAL, LLQ_EUNSUPPORTED, LLQ_ECUDA, LLQ_ETIMEOUT, LLQ_ENOSPACE = range(6)
LLQ_F32, LLQ_F16, LLQ_BF16 = 0, 1, 2
LLQ_SEARCH_AMAX, LLQ_SEARCH_MSE = 0, 1
LLQ_GEMM_AUTO, LLQ_GEMM_TCGEN05, LLQ_GEMM_SIMT, LLQ_GEMM_TCGEN05_FAST = 0, 1, 2, 3

P = c_void_p
I = c_int
L = c_int64

#: every entry point of include/llada_quant.h with its ctypes signature
SIGNATURES = {
    "llq_version": (I, []),
    "llq_last_error": (ctypes.c_char_p, []),
    "llq_quantize_pack": (I, [P, I, L, L, I, I, I, I, c_double, I, I, P, P, P]),
    "llq_search_errors": (I, [P, I, L, L, I, I, I, c_double, P, P]),
    "llq_dequantize": (I, [P, P, L, L, I, I, I, P, I, P]),
    "llq_pack_int4": (I, [P, L, P, P, P]),
    "llq_unpack_int4": (I, [P, L, P, P]),
    "llq_route": (I, [P, P, L, I, I, I, P, I, P, P, P, P]),
    "llq_route_topk": (I, [P, I, L, I, I, P, I, P, P, P]),
    "llq_align_workspace_size": (c_size_t, [L, I, I]),
    "llq_moe_align": (I, [P, L, I, I, P, P, P, c_size_t, P]),
    "llq_moe_permute": (I, [P, L, I, I, P, I, P, P]),
    "llq_moe_combine": (I, [P, L, I, I, P, P]),
    "llq_ep_pack": (I, [P, P, P, L, I, I, I, P, P, P, P, P, P]),
    "llq_ep_combine": (I, [P, P, L, I, I, P, P]),
    "llq_moe_gemm1": (I, [P, P, L, I, I, I, P, P, I, I, P, I, P]),
    "llq_moe_gemm2": (I, [P, P, P, P, L, I, I, I, P, P, I, I, P, I, P]),
    "llq_quant_linear_workspace_size": (c_size_t, [L, I, I]),
    "llq_quant_linear": (I, [P, L, I, I, P, P, I, I, P, P, c_size_t, I, P]),
    "llq_moe_gemm12_counters": (c_size_t, [L, I]),
    "llq_moe_gemm12": (I, [P, P, P, P, L, I, I, I, P, P, P, P, I, I, P, P, P, P]),
    "llq_moe_workspace_size": (c_size_t, [L, I, I, I, I]),
    "llq_fused_moe_packed": (I, [P, P, P, P, P, P, P, L, I, I, I, I, I, I, P, P, c_size_t, I, P]),
    "llq_fused_moe_packed_noalloc": (I, [P, P, P, P, P, P, P, L, I, I, I, I, I, I, P, I, P]),
    "llq_moe_block_packed": (I, [P, P, P, I, L, I, I, I, I, P, P, P, P, I, I, P, P, P, P, P, c_size_t, I, P]),
    "llq_ep_window_bytes": (c_size_t, [I, I, I]),
    "llq_ep_set_timeout_ms": (I, [I]),
    "llq_ipc_handle_bytes": (I, []),
    "llq_ipc_alloc": (I, [c_size_t, P, P]),
    "llq_ipc_open": (I, [P, P]),
    "llq_ipc_close": (I, [P]),
    "llq_ipc_free": (I, [P]),
    "llq_ep_dispatch": (I, [P, P, P, L, I, I, I, P, P, I, I, I, ctypes.c_uint32, P, P]),
    "llq_ep_experts_workspace_size": (c_size_t, [I, I, I, I, I]),
    "llq_ep_experts": (I, [P, P, I, I, I, ctypes.c_uint32, P, P, P, P, I, I, I, I, I, L, P, c_size_t, I, P]),
    "llq_ep_combine_wait": (I, [P, I, I, I, ctypes.c_uint32, P, L, I, I, P, P]),
    "llq_device_error": (I, [P]),
    "llq_clear_device_error": (I, []),
}

_lib = None


class LLQError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load (once) and return the library; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise RuntimeError(
            f"libllada_quant_cuda.so not found at {path}; build it with "
            "`python -m llada_quant_b200.build` (there is no CPU fallback)"
        )
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(rc: int, what: str = "") -> None:
    if rc == LLQ_OK:
        return
    msg = load().llq_last_error().decode(errors="replace")
    if rc == LLQ_EINVAL:
        raise ValueError(msg)
    raise LLQError(rc, f"{what}: {msg}" if what else msg)
