"""PyTorch custom ops (namespace ``llada_quant``) over the C ABI.

Each op takes CUDA tensors, launches on the current stream and never
synchronizes the host.  Fake (meta) implementations give output shapes for
tracing.  There is no CPU implementation: a CPU tensor raises.

Every op ``name`` is a ``torch.library`` custom op wrapping the plain function
``_name_impl``; latency-critical eager callers (the expert-parallel layer,
the whole-layer helpers) call ``_name_impl`` directly and skip the
dispatcher's per-call host cost (tens of microseconds).
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import _lib
from ._lib import check, load

_DT = {torch.float32: _lib.LLQ_F32, torch.float16: _lib.LLQ_F16, torch.bfloat16: _lib.LLQ_BF16}


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def _stream(t: torch.Tensor):
    return torch.cuda.current_stream(t.device).cuda_stream


def _need_cuda(*ts: Optional[torch.Tensor]) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError(
                "llada_quant_b200 ops run only on CUDA tensors (B200); there is no CPU fallback"
            )


def effective_groups(K: int, group_size: int) -> Tuple[int, int]:
    """(effective group size, groups per row) -- -1/one group when g does not divide K."""
    if group_size == -1 or group_size <= 0 or K % group_size != 0:
        return -1, 1
    return group_size, K // group_size


# ---------------------------------------------------------------------------
# quantize / dequantize / pack
# ---------------------------------------------------------------------------


def _quantize_pack_impl(w: torch.Tensor, bits: int, group_size: int, scale_search: int, grid: int,
                  max_shrink: float, scale_round: int, pack: bool) -> Tuple[torch.Tensor, torch.Tensor]:
    _need_cuda(w)
    w = w.contiguous()
    if w.dtype not in _DT:
        w = w.to(torch.float32)
    K = w.shape[-1]
    rows = w.numel() // K if K else 0
    _, groups = effective_groups(K, group_size)
    packed = bits == 4 and pack
    q = torch.empty(*w.shape[:-1], K // 2 if packed else K, dtype=torch.int8, device=w.device)
    scale = torch.empty(*w.shape[:-1], groups, dtype=torch.float32, device=w.device)
    check(load().llq_quantize_pack(w.data_ptr(), _DT[w.dtype], rows, K, bits, group_size,
                                   scale_search, grid, max_shrink, scale_round, int(pack),
                                   q.data_ptr(), scale.data_ptr(), _stream(w)), "quantize_pack")
    return q, scale


quantize_pack = torch.library.custom_op("llada_quant::quantize_pack", mutates_args=())(_quantize_pack_impl)


@quantize_pack.register_fake
def _(w, bits, group_size, scale_search, grid, max_shrink, scale_round, pack):
    K = w.shape[-1]
    _, groups = effective_groups(K, group_size)
    packed = bits == 4 and pack
    return (w.new_empty(*w.shape[:-1], K // 2 if packed else K, dtype=torch.int8),
            w.new_empty(*w.shape[:-1], groups, dtype=torch.float32))


def _search_errors_impl(w: torch.Tensor, bits: int, group_size: int, grid: int,
                  max_shrink: float) -> torch.Tensor:
    _need_cuda(w)
    w = w.contiguous()
    if w.dtype not in _DT:
        w = w.to(torch.float32)
    K = w.shape[-1]
    rows = w.numel() // K
    _, groups = effective_groups(K, group_size)
    errs = torch.empty(*w.shape[:-1], groups, grid, dtype=torch.float32, device=w.device)
    check(load().llq_search_errors(w.data_ptr(), _DT[w.dtype], rows, K, bits, group_size, grid,
                                   max_shrink, errs.data_ptr(), _stream(w)), "search_errors")
    return errs


search_errors = torch.library.custom_op("llada_quant::search_errors", mutates_args=())(_search_errors_impl)


@search_errors.register_fake
def _(w, bits, group_size, grid, max_shrink):
    _, groups = effective_groups(w.shape[-1], group_size)
    return w.new_empty(*w.shape[:-1], groups, grid, dtype=torch.float32)


def _dequantize_impl(q: torch.Tensor, scale: torch.Tensor, bits: int, group_size: int, packed: bool,
               dtype: torch.dtype) -> torch.Tensor:
    _need_cuda(q, scale)
    q = q.contiguous()
    scale = scale.contiguous().to(torch.float32)
    K = q.shape[-1] * (2 if packed else 1)
    rows = q.numel() // q.shape[-1] if q.shape[-1] else 0
    out = torch.empty(*q.shape[:-1], K, dtype=dtype, device=q.device)
    check(load().llq_dequantize(q.data_ptr(), scale.data_ptr(), rows, K, bits, group_size,
                                int(packed), out.data_ptr(), _DT[dtype], _stream(q)), "dequantize")
    return out


dequantize = torch.library.custom_op("llada_quant::dequantize", mutates_args=())(_dequantize_impl)


@dequantize.register_fake
def _(q, scale, bits, group_size, packed, dtype):
    K = q.shape[-1] * (2 if packed else 1)
    return q.new_empty(*q.shape[:-1], K, dtype=dtype)


def _pack_int4_impl(values: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Returns (packed, range_error) -- range_error is a device int32 flag (1 = out of [-8, 7])."""
    _need_cuda(values)
    values = values.contiguous()
    out = torch.empty(*values.shape[:-1], values.shape[-1] // 2, dtype=torch.int8, device=values.device)
    flag = torch.zeros(1, dtype=torch.int32, device=values.device)
    check(load().llq_pack_int4(values.data_ptr(), values.numel(), out.data_ptr(), flag.data_ptr(),
                               _stream(values)), "pack_int4")
    return out, flag


pack_int4 = torch.library.custom_op("llada_quant::pack_int4", mutates_args=())(_pack_int4_impl)


@pack_int4.register_fake
def _(values):
    return (values.new_empty(*values.shape[:-1], values.shape[-1] // 2, dtype=torch.int8),
            values.new_empty(1, dtype=torch.int32))


def _unpack_int4_impl(packed: torch.Tensor) -> torch.Tensor:
    _need_cuda(packed)
    packed = packed.contiguous()
    out = torch.empty(*packed.shape[:-1], packed.shape[-1] * 2, dtype=torch.int8, device=packed.device)
    check(load().llq_unpack_int4(packed.data_ptr(), packed.numel() * 2, out.data_ptr(),
                                 _stream(packed)), "unpack_int4")
    return out


unpack_int4 = torch.library.custom_op("llada_quant::unpack_int4", mutates_args=())(_unpack_int4_impl)


@unpack_int4.register_fake
def _(packed):
    return packed.new_empty(*packed.shape[:-1], packed.shape[-1] * 2, dtype=torch.int8)


# ---------------------------------------------------------------------------
# routing
# ---------------------------------------------------------------------------


def _route_impl(x: torch.Tensor, gate_w: torch.Tensor, k: int, bias: Optional[torch.Tensor],
          renormalize: bool) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """bf16 router logits, fp32 softmax, top-k -> (topk_w f32 [T,k], topk_ids i32 [T,k], logits bf16 [T,E])."""
    _need_cuda(x, gate_w, bias)
    x = x.contiguous()
    gate_w = gate_w.contiguous()
    T, H = x.shape
    E = gate_w.shape[0]
    w = torch.empty(T, k, dtype=torch.float32, device=x.device)
    ids = torch.empty(T, k, dtype=torch.int32, device=x.device)
    logits = torch.empty(T, E, dtype=torch.bfloat16, device=x.device)
    b = None if bias is None else bias.contiguous().to(torch.float32)
    check(load().llq_route(x.data_ptr(), gate_w.data_ptr(), T, H, E, k, _ptr(b), int(renormalize),
                           logits.data_ptr(), w.data_ptr(), ids.data_ptr(), _stream(x)), "route")
    return w, ids, logits


route = torch.library.custom_op("llada_quant::route", mutates_args=())(_route_impl)


@route.register_fake
def _(x, gate_w, k, bias, renormalize):
    T, E = x.shape[0], gate_w.shape[0]
    return (x.new_empty(T, k, dtype=torch.float32), x.new_empty(T, k, dtype=torch.int32),
            x.new_empty(T, E, dtype=torch.bfloat16))


def _route_topk_impl(logits: torch.Tensor, k: int, bias: Optional[torch.Tensor],
               renormalize: bool) -> Tuple[torch.Tensor, torch.Tensor]:
    _need_cuda(logits, bias)
    logits = logits.contiguous()
    if logits.dtype not in (torch.bfloat16, torch.float32):
        logits = logits.to(torch.float32)
    T, E = logits.shape
    w = torch.empty(T, k, dtype=torch.float32, device=logits.device)
    ids = torch.empty(T, k, dtype=torch.int32, device=logits.device)
    b = None if bias is None else bias.contiguous().to(torch.float32)
    check(load().llq_route_topk(logits.data_ptr(), _DT[logits.dtype], T, E, k, _ptr(b),
                                int(renormalize), w.data_ptr(), ids.data_ptr(), _stream(logits)),
          "route_topk")
    return w, ids


route_topk = torch.library.custom_op("llada_quant::route_topk", mutates_args=())(_route_topk_impl)


@route_topk.register_fake
def _(logits, k, bias, renormalize):
    T = logits.shape[0]
    return logits.new_empty(T, k, dtype=torch.float32), logits.new_empty(T, k, dtype=torch.int32)


def _moe_align_impl(topk_ids: torch.Tensor, num_experts: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """-> (expert_offsets i32 [E+1], sorted_slots i32 [T*k])."""
    _need_cuda(topk_ids)
    ids = topk_ids.contiguous().to(torch.int32)
    T, k = ids.shape
    offsets = torch.empty(num_experts + 1, dtype=torch.int32, device=ids.device)
    slots = torch.empty(T * k, dtype=torch.int32, device=ids.device)
    lib = load()
    nbytes = lib.llq_align_workspace_size(T, k, num_experts)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=ids.device)
    check(lib.llq_moe_align(ids.data_ptr(), T, k, num_experts, offsets.data_ptr(), slots.data_ptr(),
                            ws.data_ptr(), nbytes, _stream(ids)), "moe_align")
    return offsets, slots


moe_align = torch.library.custom_op("llada_quant::moe_align", mutates_args=())(_moe_align_impl)


@moe_align.register_fake
def _(topk_ids, num_experts):
    T, k = topk_ids.shape
    return (topk_ids.new_empty(num_experts + 1, dtype=torch.int32),
            topk_ids.new_empty(T * k, dtype=torch.int32))


def _moe_permute_impl(x: torch.Tensor, sorted_slots: torch.Tensor, k: int, kperm: bool = False) -> torch.Tensor:
    """Rows of ``x`` in expert order; ``kperm`` also applies the fast-mode K order."""
    _need_cuda(x, sorted_slots)
    x = x.contiguous()
    T, H = x.shape
    out = torch.empty(sorted_slots.numel(), H, dtype=x.dtype, device=x.device)
    check(load().llq_moe_permute(x.data_ptr(), T, H, k, sorted_slots.data_ptr(), int(kperm),
                                 out.data_ptr(), _stream(x)), "moe_permute")
    return out


moe_permute = torch.library.custom_op("llada_quant::moe_permute", mutates_args=())(_moe_permute_impl)


@moe_permute.register_fake
def _(x, sorted_slots, k, kperm=False):
    return x.new_empty(sorted_slots.shape[0], x.shape[1])


def _moe_combine_impl(y_slots: torch.Tensor, k: int) -> torch.Tensor:
    _need_cuda(y_slots)
    y_slots = y_slots.contiguous()
    n, H = y_slots.shape
    T = n // k
    out = torch.empty(T, H, dtype=torch.bfloat16, device=y_slots.device)
    check(load().llq_moe_combine(y_slots.data_ptr(), T, k, H, out.data_ptr(), _stream(y_slots)),
          "moe_combine")
    return out


moe_combine = torch.library.custom_op("llada_quant::moe_combine", mutates_args=())(_moe_combine_impl)


@moe_combine.register_fake
def _(y_slots, k):
    return y_slots.new_empty(y_slots.shape[0] // k, y_slots.shape[1], dtype=torch.bfloat16)


def _ep_pack_impl(x: torch.Tensor, topk_ids: torch.Tensor, topk_w: torch.Tensor, sorted_slots: torch.Tensor,
            experts_per_rank: int) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Expert-parallel send buffers: (rows [T*k, H], local expert ids, routed weights, inverse positions)."""
    _need_cuda(x, topk_ids, topk_w, sorted_slots)
    x = x.contiguous()
    T, H = x.shape
    k = topk_ids.shape[1]
    ids = topk_ids.contiguous().to(torch.int32)
    w = topk_w.contiguous().to(torch.float32)
    n = T * k
    rows = torch.empty(n, H, dtype=x.dtype, device=x.device)
    lid = torch.empty(n, dtype=torch.int32, device=x.device)
    wts = torch.empty(n, dtype=torch.float32, device=x.device)
    inv = torch.empty(n, dtype=torch.int32, device=x.device)
    check(load().llq_ep_pack(x.data_ptr(), ids.data_ptr(), w.data_ptr(), T, k, H, experts_per_rank,
                             sorted_slots.data_ptr(), rows.data_ptr(), lid.data_ptr(), wts.data_ptr(),
                             inv.data_ptr(), _stream(x)), "ep_pack")
    return rows, lid, wts, inv


ep_pack = torch.library.custom_op("llada_quant::ep_pack", mutates_args=())(_ep_pack_impl)


@ep_pack.register_fake
def _(x, topk_ids, topk_w, sorted_slots, experts_per_rank):
    n = topk_ids.numel()
    return (x.new_empty(n, x.shape[1]), x.new_empty(n, dtype=torch.int32), x.new_empty(n, dtype=torch.float32),
            x.new_empty(n, dtype=torch.int32))


def _ep_combine_impl(back: torch.Tensor, inv_pos: torch.Tensor, k: int) -> torch.Tensor:
    _need_cuda(back, inv_pos)
    back = back.contiguous()
    n, H = back.shape
    T = inv_pos.numel() // k
    out = torch.empty(T, H, dtype=torch.bfloat16, device=back.device)
    check(load().llq_ep_combine(back.data_ptr(), inv_pos.data_ptr(), T, k, H, out.data_ptr(), _stream(back)),
          "ep_combine")
    return out


ep_combine = torch.library.custom_op("llada_quant::ep_combine", mutates_args=())(_ep_combine_impl)


@ep_combine.register_fake
def _(back, inv_pos, k):
    return back.new_empty(inv_pos.numel() // k, back.shape[1], dtype=torch.bfloat16)


# ---------------------------------------------------------------------------
# grouped expert GEMMs and the whole layer
# ---------------------------------------------------------------------------


def _group_of(q: torch.Tensor, scale: torch.Tensor, bits: int) -> int:
    K = q.shape[-1] * (2 if bits == 4 else 1)
    g = scale.shape[-1]
    return -1 if g <= 1 else K // g


def _moe_gemm1_impl(x_sorted: torch.Tensor, expert_offsets: torch.Tensor, qw1: torch.Tensor,
              sw1: torch.Tensor, bits: int, impl: int) -> torch.Tensor:
    _need_cuda(x_sorted, expert_offsets, qw1, sw1)
    E, two_i = qw1.shape[0], qw1.shape[1]
    H = x_sorted.shape[1]
    inter = two_i // 2
    n = x_sorted.shape[0]
    h = torch.empty(n, inter, dtype=torch.bfloat16, device=x_sorted.device)
    check(load().llq_moe_gemm1(x_sorted.data_ptr(), expert_offsets.data_ptr(), n, E, H, inter,
                               qw1.data_ptr(), sw1.data_ptr(), bits, _group_of(qw1, sw1, bits),
                               h.data_ptr(), impl, _stream(x_sorted)), "moe_gemm1")
    return h


moe_gemm1 = torch.library.custom_op("llada_quant::moe_gemm1", mutates_args=())(_moe_gemm1_impl)


@moe_gemm1.register_fake
def _(x_sorted, expert_offsets, qw1, sw1, bits, impl):
    return x_sorted.new_empty(x_sorted.shape[0], qw1.shape[1] // 2, dtype=torch.bfloat16)


def _moe_gemm2_impl(h_sorted: torch.Tensor, expert_offsets: torch.Tensor, sorted_slots: torch.Tensor,
              topk_w: torch.Tensor, qw2: torch.Tensor, sw2: torch.Tensor, bits: int,
              impl: int) -> torch.Tensor:
    _need_cuda(h_sorted, expert_offsets, sorted_slots, topk_w, qw2, sw2)
    E, H = qw2.shape[0], qw2.shape[1]
    inter = h_sorted.shape[1]
    n = h_sorted.shape[0]
    y = torch.empty(n, H, dtype=torch.bfloat16, device=h_sorted.device)
    tw = topk_w.contiguous().to(torch.float32)
    check(load().llq_moe_gemm2(h_sorted.data_ptr(), expert_offsets.data_ptr(), sorted_slots.data_ptr(),
                               tw.data_ptr(), n, E, H, inter, qw2.data_ptr(), sw2.data_ptr(), bits,
                               _group_of(qw2, sw2, bits), y.data_ptr(), impl, _stream(h_sorted)),
          "moe_gemm2")
    return y


moe_gemm2 = torch.library.custom_op("llada_quant::moe_gemm2", mutates_args=())(_moe_gemm2_impl)


@moe_gemm2.register_fake
def _(h_sorted, expert_offsets, sorted_slots, topk_w, qw2, sw2, bits, impl):
    return h_sorted.new_empty(h_sorted.shape[0], qw2.shape[1], dtype=torch.bfloat16)


_WS_CACHE: dict = {}


def _moe_gemm12_impl(x_sorted: torch.Tensor, expert_offsets: torch.Tensor, sorted_slots: torch.Tensor,
                     topk_w: torch.Tensor, qw1: torch.Tensor, sw1: torch.Tensor, qw2: torch.Tensor,
                     sw2: torch.Tensor, bits: int, counters: torch.Tensor) -> torch.Tensor:
    """GEMM1 (+SiLU) and GEMM2 (+routed weight) in one launch; returns y in (token, slot) order.
    ``counters``: int32 zeros of ``llq_moe_gemm12_counters(n, E)`` (left zeroed by every call)."""
    _need_cuda(x_sorted, expert_offsets, sorted_slots, topk_w, qw1, sw1, qw2, sw2, counters)
    n, H = x_sorted.shape
    E, two_i = qw1.shape[0], qw1.shape[1]
    inter = two_i // 2
    h = torch.empty(n, inter, dtype=torch.bfloat16, device=x_sorted.device)
    y = torch.empty(n, H, dtype=torch.bfloat16, device=x_sorted.device)
    tw = topk_w.contiguous().to(torch.float32)
    check(load().llq_moe_gemm12(x_sorted.data_ptr(), expert_offsets.data_ptr(), sorted_slots.data_ptr(),
                                tw.data_ptr(), n, E, H, inter, qw1.data_ptr(), sw1.data_ptr(), qw2.data_ptr(),
                                sw2.data_ptr(), bits, _group_of(qw1, sw1, bits), h.data_ptr(), y.data_ptr(),
                                counters.data_ptr(), _stream(x_sorted)), "moe_gemm12")
    return y


def gemm12_counters(n_rows: int, num_experts: int, device) -> torch.Tensor:
    return torch.zeros(load().llq_moe_gemm12_counters(n_rows, num_experts), dtype=torch.int32, device=device)


def moe_workspace(T: int, k: int, E: int, H: int, I: int, device) -> torch.Tensor:
    """A cached per-device workspace large enough for ``fused_moe_packed``."""
    need = load().llq_moe_workspace_size(T, k, E, H, I)
    key = (str(device),)
    ws = _WS_CACHE.get(key)
    if ws is None or ws.numel() < need:
        ws = torch.empty(need, dtype=torch.uint8, device=device)
        _WS_CACHE[key] = ws
    return ws


def _quant_linear_impl(x: torch.Tensor, qweight: torch.Tensor, scale: torch.Tensor, bits: int) -> torch.Tensor:
    """``F.linear(x, dequantize(qweight, scale))`` on the tcgen05 kernel: x bf16 [M, K] -> bf16 [M, N]."""
    _need_cuda(x, qweight, scale)
    x = x.contiguous()
    M, K = x.shape
    N = qweight.shape[0]
    out = torch.empty(M, N, dtype=torch.bfloat16, device=x.device)
    lib = load()
    need = lib.llq_quant_linear_workspace_size(M, K, N)
    ws = _linear_workspace(need, x.device) if need else None
    check(lib.llq_quant_linear(x.data_ptr(), M, K, N, qweight.data_ptr(), scale.data_ptr(), bits,
                               _group_of(qweight, scale, bits), out.data_ptr(),
                               ws.data_ptr() if ws is not None else None, need, 0, _stream(x)),
          "quant_linear")
    return out


_LIN_WS: dict = {}


def _linear_workspace(nbytes: int, device) -> torch.Tensor:
    key = str(device)
    ws = _LIN_WS.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(nbytes, dtype=torch.uint8, device=device)
        _LIN_WS[key] = ws
    return ws


quant_linear = torch.library.custom_op("llada_quant::quant_linear", mutates_args=())(_quant_linear_impl)


@quant_linear.register_fake
def _(x, qweight, scale, bits):
    return x.new_empty(x.shape[0], qweight.shape[0], dtype=torch.bfloat16)


def _fused_moe_packed_impl(x: torch.Tensor, qw1: torch.Tensor, sw1: torch.Tensor, qw2: torch.Tensor,
                     sw2: torch.Tensor, topk_w: torch.Tensor, topk_ids: torch.Tensor, bits: int,
                     impl: int) -> torch.Tensor:
    """Routed MoE layer on PACKED weights: align, permute, GEMM1(+SiLU), GEMM2(+weight), combine."""
    _need_cuda(x, qw1, sw1, qw2, sw2, topk_w, topk_ids)
    x = x.contiguous()
    T, H = x.shape
    E, two_i = qw1.shape[0], qw1.shape[1]
    inter = two_i // 2
    k = topk_ids.shape[1]
    ids = topk_ids.contiguous().to(torch.int32)
    tw = topk_w.contiguous().to(torch.float32)
    out = torch.empty(T, H, dtype=torch.bfloat16, device=x.device)
    ws = moe_workspace(T, k, E, H, inter, x.device)
    # one config group size; the library applies the per-row fallback to the
    # tensor whose K it does not divide, as quantize_tensor did
    g = _group_pair(qw1, sw1, qw2, sw2, bits)
    check(load().llq_fused_moe_packed(x.data_ptr(), qw1.data_ptr(), sw1.data_ptr(), qw2.data_ptr(),
                                      sw2.data_ptr(), tw.data_ptr(), ids.data_ptr(), T, E, H, inter,
                                      k, bits, g, out.data_ptr(), ws.data_ptr(), ws.numel(), impl,
                                      _stream(x)), "fused_moe_packed")
    return out


fused_moe_packed = torch.library.custom_op("llada_quant::fused_moe_packed", mutates_args=())(_fused_moe_packed_impl)


@fused_moe_packed.register_fake
def _(x, qw1, sw1, qw2, sw2, topk_w, topk_ids, bits, impl):
    return torch.empty_like(x, dtype=torch.bfloat16)


def _group_pair(qw1: torch.Tensor, sw1: torch.Tensor, qw2: torch.Tensor, sw2: torch.Tensor, bits: int) -> int:
    g1, g2 = _group_of(qw1, sw1, bits), _group_of(qw2, sw2, bits)
    if g1 != -1 and g2 != -1 and g1 != g2:
        raise ValueError("w1 and w2 must share the group size")
    return g1 if g1 != -1 else g2


def _moe_block_packed_impl(x: torch.Tensor, gate_w: torch.Tensor, bias: Optional[torch.Tensor], renormalize: bool,
                           qw1: torch.Tensor, sw1: torch.Tensor, qw2: torch.Tensor, sw2: torch.Tensor, k: int,
                           bits: int, impl: int, want_logits: bool = False):
    """Router + routed experts on PACKED weights in one library call ->
    (out bf16 [T,H], topk_w f32 [T,k], topk_ids i32 [T,k], logits bf16 [T,E] or None)."""
    _need_cuda(x, gate_w, bias, qw1, sw1, qw2, sw2)
    x = x.contiguous()
    gate_w = gate_w.contiguous()
    T, H = x.shape
    E, two_i = qw1.shape[0], qw1.shape[1]
    inter = two_i // 2
    tw = torch.empty(T, k, dtype=torch.float32, device=x.device)
    ids = torch.empty(T, k, dtype=torch.int32, device=x.device)
    logits = torch.empty(T, E, dtype=torch.bfloat16, device=x.device) if want_logits else None
    b = None if bias is None else bias.contiguous().to(torch.float32)
    out = torch.empty(T, H, dtype=torch.bfloat16, device=x.device)
    ws = moe_workspace(T, k, E, H, inter, x.device)
    check(load().llq_moe_block_packed(x.data_ptr(), gate_w.data_ptr(), _ptr(b), int(renormalize), T, E, H, inter, k,
                                      qw1.data_ptr(), sw1.data_ptr(), qw2.data_ptr(), sw2.data_ptr(), bits,
                                      _group_pair(qw1, sw1, qw2, sw2, bits), _ptr(logits), tw.data_ptr(),
                                      ids.data_ptr(), out.data_ptr(), ws.data_ptr(), ws.numel(), impl, _stream(x)),
          "moe_block_packed")
    return out, tw, ids, logits


def device_error() -> int:
    import ctypes
    code = ctypes.c_int32(0)
    check(load().llq_device_error(ctypes.addressof(code)), "device_error")
    return int(code.value)


def clear_device_error() -> None:
    check(load().llq_clear_device_error(), "clear_device_error")
