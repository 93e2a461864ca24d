"""numpy restatement of the routed, PACKED-mode MoE expert layer (TEST ORACLE).

Test infrastructure only (see ``oracle/__init__.py``).

What is restated, and from where (paths within the LLaDA_Quant project):

* routing -- ``logits = gate(x)`` (bf16 Linear, no bias), ``softmax(logits,
  fp32)``, ``topk`` (``src/LLaDA_Quant/trajectory/llada.py:225-234``).  torch's
  CPU ``topk`` orders equal values arbitrarily, so the oracle fixes a rule:
  larger value first, then the smaller expert id.  Tests compare routing modulo
  ties and feed the same ``topk_ids`` to both sides of every layer comparison.
* weights -- ``dequantize_tensor(..., dtype=bf16, packed=...)`` exactly as the
  PACKED-mode ``w1``/``w2`` property does (``src/LLaDA_Quant/runtime/moe.py:199-216``).
* expert FFN -- gate rows ``[0, I)``, up rows ``[I, 2I)`` of ``w1``
  (``tests/unit/conftest.py:37-43``); GEMM1 epilogue rounds gate and up to
  bf16, evaluates ``g / (1 + exp(-g))`` in fp32, rounds to bf16, multiplies by
  ``up`` in fp32 and stores bf16 (``INFERENCE_REPO_CHANGES.md:296-309``);
  GEMM2 multiplies the fp32 accumulator by the routed weight and stores bf16
  per (token, slot) (``MUL_ROUTED_WEIGHT``, ``INFERENCE_REPO_CHANGES.md:259-265``);
  the top-k slots are summed in fp32 in slot order and rounded once to bf16.
* alignment -- tokens grouped by expert, stable in (token, slot) order, the
  contract of the external ``moe_align_block_size``
  (``INFERENCE_REPO_CHANGES.md:274-278``).

GEMM accumulations run in float32 (BLAS order); the kernels under test
accumulate in float32 in their own order, so layer outputs are compared with a
stated tolerance, never bit for bit.
"""

from __future__ import annotations

import numpy as np

from .symmetric import dequantize_tensor, round_to_bf16


def router_logits(x: np.ndarray, gate_w: np.ndarray) -> np.ndarray:
    """bf16 ``gate(x)``: fp32-accumulated dot products rounded to bf16."""
    acc = x.astype(np.float64) @ gate_w.astype(np.float64).T
    return round_to_bf16(acc.astype(np.float32))


def softmax_fp32(logits: np.ndarray) -> np.ndarray:
    """``softmax(logits, dim=-1, dtype=float32)``: max-shift, exp, multiply by 1/sum."""
    l = logits.astype(np.float32)
    m = l.max(axis=-1, keepdims=True)
    e = np.exp((l - m).astype(np.float32)).astype(np.float32)
    s = e.astype(np.float32).sum(axis=-1, keepdims=True, dtype=np.float32)
    return (e * (np.float32(1.0) / s)).astype(np.float32)


def route_topk(logits: np.ndarray, k: int, bias: np.ndarray | None = None, renormalize: bool = False):
    """Top-k over ``softmax(logits + bias)``; ties -> smaller expert id first.

    Returns ``(topk_w float32 [T,k], topk_ids int32 [T,k])``.  ``bias`` is the
    optional per-expert logit offset the expert-parallel benchmark uses to
    skew routing; it is added in fp32 before the softmax.
    """
    l = logits.astype(np.float32)
    if bias is not None:
        l = (l + bias.astype(np.float32)[None, :]).astype(np.float32)
    p = softmax_fp32(l)
    T, E = p.shape
    # lexsort: last key is primary -> sort by -p, then by id
    ids = np.empty((T, k), dtype=np.int32)
    for t in range(T):
        order = np.lexsort((np.arange(E), -p[t]))
        ids[t] = order[:k]
    w = np.take_along_axis(p, ids.astype(np.int64), axis=1).astype(np.float32)
    if renormalize:
        w = (w / w.sum(axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)
    return w, ids


def moe_align(topk_ids: np.ndarray, num_experts: int):
    """Stable grouping of the ``T*k`` (token, slot) entries by expert.

    Returns ``(expert_offsets int32 [E+1], sorted_slots int32 [T*k])`` where the
    rows of expert ``e`` are ``sorted_slots[offsets[e]:offsets[e+1]]`` and each
    entry is ``token * k + slot``.
    """
    flat = topk_ids.reshape(-1).astype(np.int64)
    order = np.argsort(flat, kind="stable").astype(np.int32)
    counts = np.bincount(flat, minlength=num_experts)
    offsets = np.zeros(num_experts + 1, dtype=np.int32)
    offsets[1:] = np.cumsum(counts)
    return offsets, order


def silu_bf16(gate_bf16: np.ndarray) -> np.ndarray:
    g = gate_bf16.astype(np.float32)
    return round_to_bf16((g / (np.float32(1.0) + np.exp(-g).astype(np.float32))).astype(np.float32))


def dequantize_experts(qw1, sw1, qw2, sw2, bits: int):
    """bf16 ``w1`` [E,2I,H] and ``w2`` [E,H,I] exactly as the PACKED property returns them."""
    packed = bits == 4
    g1 = -1 if sw1.shape[-1] <= 1 else (qw1.shape[-1] * (2 if packed else 1)) // sw1.shape[-1]
    g2 = -1 if sw2.shape[-1] <= 1 else (qw2.shape[-1] * (2 if packed else 1)) // sw2.shape[-1]
    w1 = dequantize_tensor(qw1, sw1, bits, g1, packed=packed, to_bf16=True)
    w2 = dequantize_tensor(qw2, sw2, bits, g2, packed=packed, to_bf16=True)
    return w1, w2


def expert_ffn_rows(x_rows: np.ndarray, w1_e: np.ndarray, w2_e: np.ndarray, routed_w: np.ndarray):
    """One expert over its rows: returns the bf16 per-(token,slot) outputs ``[m, H]``
    and the bf16 GEMM1 activations ``[m, I]``."""
    inter = w2_e.shape[-1]
    acc = x_rows.astype(np.float32) @ w1_e.astype(np.float32).T          # [m, 2I] fp32
    gate = round_to_bf16(acc[:, :inter])
    up = round_to_bf16(acc[:, inter:])
    h = round_to_bf16((silu_bf16(gate) * up).astype(np.float32))
    y = (h @ w2_e.astype(np.float32).T).astype(np.float32)             # [m, H] fp32
    y = round_to_bf16((y * routed_w.astype(np.float32)[:, None]).astype(np.float32))
    return y, h


def fused_moe_packed(x: np.ndarray, qw1, sw1, qw2, sw2, topk_w: np.ndarray, topk_ids: np.ndarray,
                     bits: int, weights=None, return_intermediates: bool = False):
    """Routed PACKED-mode MoE layer: ``x`` bf16 values [T,H] -> bf16 values [T,H].

    ``weights`` may pass pre-dequantized ``(w1, w2)`` to skip the dequantize.
    """
    T, H = x.shape
    k = topk_ids.shape[1]
    E = qw1.shape[0]
    w1, w2 = weights if weights is not None else dequantize_experts(qw1, sw1, qw2, sw2, bits)
    offsets, sorted_slots = moe_align(topk_ids, E)
    inter = w2.shape[-1]
    y_slots = np.zeros((T * k, H), dtype=np.float32)
    h_sorted = np.zeros((T * k, inter), dtype=np.float32)
    flat_w = topk_w.reshape(-1)
    for e in range(E):
        lo, hi = int(offsets[e]), int(offsets[e + 1])
        if lo == hi:
            continue
        slots = sorted_slots[lo:hi].astype(np.int64)
        y, h = expert_ffn_rows(x[slots // k], w1[e], w2[e], flat_w[slots])
        y_slots[slots] = y
        h_sorted[lo:hi] = h
    out = np.zeros((T, H), dtype=np.float32)
    ys = y_slots.reshape(T, k, H)
    for j in range(k):
        out = (out + ys[:, j]).astype(np.float32)
    out = round_to_bf16(out)
    if return_intermediates:
        return out, dict(offsets=offsets, sorted_slots=sorted_slots, h_sorted=h_sorted,
                         y_slots=y_slots, w1=w1, w2=w2)
    return out


def fused_moe_f64(x: np.ndarray, qw1, sw1, qw2, sw2, topk_w: np.ndarray, topk_ids: np.ndarray,
                  bits: int) -> np.ndarray:
    """The quantized layer's exact mathematics: W = q * s in float64, no intermediate
    rounding at all.  Neither the reference path nor any kernel computes this; it is
    the yardstick both are measured against."""
    from .symmetric import unpack_int4
    packed = bits == 4

    def deq64(q, s):
        qq = unpack_int4(q) if packed else q
        K = qq.shape[-1]
        G = s.shape[-1]
        if G <= 1:
            return qq.astype(np.float64) * s.astype(np.float64)
        g = K // G
        return (qq.astype(np.float64).reshape(*qq.shape[:-1], G, g)
                * s.astype(np.float64)[..., None]).reshape(qq.shape)

    w1 = deq64(qw1, sw1)
    w2 = deq64(qw2, sw2)
    inter = w2.shape[-1]
    T, H = x.shape
    out = np.zeros((T, H), dtype=np.float64)
    offsets, slots = moe_align(topk_ids, qw1.shape[0])
    k = topk_ids.shape[1]
    flat_w = topk_w.reshape(-1).astype(np.float64)
    for e in range(qw1.shape[0]):
        lo, hi = int(offsets[e]), int(offsets[e + 1])
        if lo == hi:
            continue
        sl = slots[lo:hi].astype(np.int64)
        a = x[sl // k].astype(np.float64) @ w1[e].T
        g, u = a[:, :inter], a[:, inter:]
        h = g / (1.0 + np.exp(-g)) * u
        y = (h @ w2[e].T) * flat_w[sl][:, None]
        np.add.at(out, sl // k, y)
    return out


def moe_layer(x: np.ndarray, gate_w: np.ndarray, qw1, sw1, qw2, sw2, k: int, bits: int,
              bias=None, renormalize: bool = False, weights=None):
    """Full layer: router + routed experts.  Returns ``(out, topk_w, topk_ids, logits)``."""
    logits = router_logits(x, gate_w)
    topk_w, topk_ids = route_topk(logits, k, bias=bias, renormalize=renormalize)
    out = fused_moe_packed(x, qw1, sw1, qw2, sw2, topk_w, topk_ids, bits, weights=weights)
    return out, topk_w, topk_ids, logits


def rel_l2(a: np.ndarray, b: np.ndarray) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / den) if den > 0 else float(np.linalg.norm(a - b))


def max_abs(a: np.ndarray, b: np.ndarray) -> float:
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64)))) if np.size(a) else 0.0
