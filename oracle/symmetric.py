"""numpy restatement of LLaDA_Quant's symmetric groupwise quantizer (TEST ORACLE).

Test infrastructure only (see ``oracle/__init__.py``).  Every function cites
the reference function it restates, by path within the LLaDA_Quant project.

Floating point: numpy float32 division and multiplication are IEEE
correctly rounded, ``np.rint`` rounds half to even, exactly like
``torch.round`` and ``/`` on float32 tensors.  BF16/FP16 inputs are carried
as float32 arrays holding the exactly representable values (``amax`` of such
values is exact in either dtype, so nothing changes).
"""

from __future__ import annotations

import numpy as np

SCALE_SEARCH_AMAX = "amax"
SCALE_SEARCH_MSE = "mse"


def qmax_for_bits(bits: int) -> int:
    """``src/LLaDA_Quant/algorithms/symmetric.py:29-31``."""
    return 2 ** (bits - 1) - 1


def qmin_for_bits(bits: int) -> int:
    """``src/LLaDA_Quant/algorithms/symmetric.py:34-36``."""
    return -(2 ** (bits - 1))


# ---------------------------------------------------------------------------
# bf16 helpers (round to nearest even, as torch's float32 -> bfloat16 cast)
# ---------------------------------------------------------------------------


def round_to_bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest-even bfloat16, returned as float32 (NaN-free inputs)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """The uint16 storage of ``round_to_bf16(x)``."""
    return (round_to_bf16(x).view(np.uint32) >> 16).astype(np.uint16)


def from_bf16_bits(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------------------
# groups
# ---------------------------------------------------------------------------


def as_groups(w: np.ndarray, group_size: int):
    """``_as_groups`` (symmetric.py:85-90): per-ROW fallback when g does not divide K."""
    if group_size == -1 or w.shape[-1] % group_size != 0:
        return w, 1
    k = w.shape[-1]
    return w.reshape(*w.shape[:-1], k // group_size, group_size), k // group_size


def validate_int4_layout(shape, group_size: int) -> None:
    """``validate_int4_layout`` (symmetric.py:93-108)."""
    if shape[-1] % 2 != 0:
        raise ValueError(
            f"int4 packing needs an even last dimension, got {tuple(shape)}; "
            "the last axis is the K axis and two values share one byte"
        )
    if group_size != -1 and group_size % 2 != 0:
        raise ValueError(
            f"int4 packing needs an even group_size so groups stay byte-aligned, got {group_size}"
        )


def amax_scale(w_g: np.ndarray, bits: int, reciprocal: bool = False) -> np.ndarray:
    """``_amax_scale`` (symmetric.py:117-119): fp32 amax divided (not multiplied) by Qmax.

    ``reciprocal=True`` gives what the same line computes when the reference runs
    in CUDA torch: ATen's CUDA kernel divides a tensor by a Python scalar as a
    multiplication by the float32 reciprocal, amax * float32(1/Qmax), which is
    one ulp off the division for part of the groups.  The kernels follow the
    division (CPU torch, the golden vectors); tests use this form only to explain
    the differences from a CUDA-torch run of the reference.
    """
    amax = np.abs(w_g).max(axis=-1, keepdims=True).astype(np.float32)
    if reciprocal:
        return (amax * np.float32(1.0 / qmax_for_bits(bits))).astype(np.float32)
    return (amax / np.float32(qmax_for_bits(bits))).astype(np.float32)


def group_sse_terms(wf: np.ndarray, safe: np.ndarray, bits: int) -> np.ndarray:
    """The squared-error terms of one candidate, rounded exactly as the reference's
    in-place chain ``(round(w/s).clamp * s - w) ** 2`` (symmetric.py:195-198): four
    separately rounded float32 operations, no fused multiply-add."""
    work = np.rint(wf / safe).astype(np.float32)
    work = np.clip(work, qmin_for_bits(bits), qmax_for_bits(bits)).astype(np.float32)
    work = (work * safe).astype(np.float32)
    work = (work - wf).astype(np.float32)
    return (work * work).astype(np.float32)


def search_group_scale(w_g: np.ndarray, bits: int, grid: int = 24, max_shrink: float = 0.5,
                       sum_dtype=np.float64, return_errors: bool = False, reciprocal: bool = False):
    """``search_group_scale`` (symmetric.py:122-204).

    ``ratio`` is a Python double, then rounded to float32 when it multiplies the
    float32 ``base`` (ATen's scalar handling for float tensors; checked against
    torch in ``tests/test_oracle_golden.py``).  Ties keep the earliest (largest)
    ratio because only a strictly smaller error replaces the incumbent.

    The per-group sum is the one place where the reference's result depends on
    its reduction order (ATen's vectorised CPU sum).  The oracle sums the exactly
    rounded float32 terms in float64 by default, i.e. it picks the truly best
    candidate; the callers report how often that differs from the reference
    (only ever at near-ties).  Chunking (symmetric.py:164-180) does not change
    the result and is not restated.  ``reciprocal`` selects the CUDA-torch form of
    the base scale (see ``amax_scale``).
    """
    if grid < 1:
        raise ValueError(f"grid must be >= 1, got {grid}")
    if not 0.0 <= max_shrink < 1.0:
        raise ValueError(f"max_shrink must lie in [0, 1), got {max_shrink}")
    wf = w_g.astype(np.float32)
    base = amax_scale(w_g, bits, reciprocal)
    best_scale = base.copy()
    best_err = np.full(base.shape, np.inf, dtype=sum_dtype)
    errors = []
    for step in range(grid):
        ratio = 1.0 - max_shrink * step / grid
        candidate = (base * np.float32(ratio)).astype(np.float32)
        safe = np.where(candidate > 0, candidate, np.float32(1.0)).astype(np.float32)
        err = group_sse_terms(wf, safe, bits).astype(sum_dtype).sum(axis=-1, keepdims=True)
        if return_errors:
            errors.append(err)
        better = err < best_err
        best_err = np.where(better, err, best_err)
        best_scale = np.where(better, candidate, best_scale)
    out = np.where(base > 0, best_scale, np.float32(0.0)).astype(np.float32)
    if return_errors:
        return out, np.concatenate(errors, axis=-1)
    return out


def pack_int4(q8: np.ndarray) -> np.ndarray:
    """``pack_int4`` (symmetric.py:296-313): low nibble = even index, two's complement."""
    if q8.shape[-1] % 2 != 0:
        raise ValueError("last dim must be even for int4 packing")
    if q8.size and (int(q8.max()) > 7 or int(q8.min()) < -8):
        raise ValueError(
            f"int4 packing needs values in [-8, 7], got [{int(q8.min())}, {int(q8.max())}]"
        )
    q = q8.astype(np.int16)
    lo = q[..., 0::2] & 0x0F
    hi = q[..., 1::2] & 0x0F
    return (lo | (hi << 4)).astype(np.uint8).view(np.int8)


def unpack_int4(packed: np.ndarray) -> np.ndarray:
    """``unpack_int4`` (symmetric.py:316-346): arithmetic-shift sign extension."""
    if packed.dtype != np.int8:
        raise ValueError(f"packed int4 storage must be int8, got {packed.dtype}")
    p = packed.astype(np.int16)
    low = ((p << 12) >> 12).astype(np.int8)  # (b << 4) >> 4 on an int8
    high = (p >> 4).astype(np.int8)
    out = np.empty((*packed.shape[:-1], packed.shape[-1] * 2), dtype=np.int8)
    out[..., 0::2] = low
    out[..., 1::2] = high
    return out


def quantize_tensor(w: np.ndarray, bits: int = 8, group_size: int = 128, pack: bool = True,
                    scale_search: str = SCALE_SEARCH_AMAX, search_grid: int = 24):
    """``quantize_tensor`` (symmetric.py:207-269) with ``scale_dtype=float32``.

    Returns ``(q, scale, effective_group_size, packed, logical_shape)``.
    """
    if bits not in (8, 4):
        raise ValueError(f"bits must be 8 or 4, got {bits}")
    if w.size == 0:
        raise ValueError("cannot quantize an empty tensor")
    if bits == 4 and pack:
        validate_int4_layout(w.shape, group_size)
    if scale_search not in (SCALE_SEARCH_AMAX, SCALE_SEARCH_MSE):
        raise ValueError(
            f"scale_search must be one of ['amax', 'mse'], got {scale_search!r}"
        )
    w = np.asarray(w, dtype=np.float32)
    logical_shape = tuple(w.shape)
    w_g, num_groups = as_groups(w, group_size)
    if scale_search == SCALE_SEARCH_MSE:
        scale = search_group_scale(w_g, bits, grid=search_grid)
    else:
        scale = amax_scale(w_g, bits)
    safe = np.where(scale > 0, scale, np.float32(1.0)).astype(np.float32)
    q = np.clip(np.rint(w_g / safe), qmin_for_bits(bits), qmax_for_bits(bits)).astype(np.int8)
    scale = scale.reshape(*logical_shape[:-1], num_groups)
    q = q.reshape(logical_shape)
    packed = False
    if bits == 4 and pack:
        q = pack_int4(q)
        packed = True
    return q, scale, (group_size if num_groups > 1 else -1), packed, logical_shape


def dequantize_tensor(q: np.ndarray, scale: np.ndarray, bits: int, group_size: int,
                      packed: bool = False, to_bf16: bool = False) -> np.ndarray:
    """``dequantize_tensor`` (symmetric.py:272-293): fp32 ``q * s``, then the cast.

    With ``to_bf16`` the result is rounded to bfloat16 (carried as float32), the
    value the PACKED-mode ``w1``/``w2`` property returns (runtime/moe.py:199-216).
    """
    if packed:
        q = unpack_int4(q)
    qf = q.astype(np.float32)
    if group_size == -1 or q.shape[-1] % group_size != 0:
        out = (qf * scale.astype(np.float32)).astype(np.float32)
    else:
        k = q.shape[-1]
        g = k // group_size
        out = (qf.reshape(*q.shape[:-1], g, group_size)
               * scale.astype(np.float32).reshape(*q.shape[:-1], g, 1)).reshape(q.shape)
        out = out.astype(np.float32)
    return round_to_bf16(out) if to_bf16 else out


def storage_bytes(numel: int, bits: int, group_size: int, scale_bytes: int = 4) -> int:
    """``storage_bytes`` (symmetric.py:349-362)."""
    if bits == 8:
        value_bytes = numel
    elif bits == 4:
        value_bytes = numel // 2
    else:
        raise ValueError(f"bits must be 8 or 4, got {bits}")
    groups = 1 if group_size == -1 else max(1, numel // group_size)
    return value_bytes + groups * scale_bytes
