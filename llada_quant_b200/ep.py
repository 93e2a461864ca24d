"""Expert parallelism: the routed MoE layer with experts sharded across ranks.

Rank ``r`` of ``R`` owns the contiguous experts ``[r*E/R, (r+1)*E/R)`` (their
packed ``_qw*``/``_sw*`` slices); the router is replicated and tokens are
data-parallel.  One layer call on each rank:

1. route its own tokens (global expert ids, fp32 routed weights);
2. group its ``T*k`` (token, slot) entries by destination rank (stable);
3. exchange per-destination counts, then the token rows and their
   (local expert id, routed weight) -- NCCL ``all_to_all_single`` over
   NVLink/NVSwitch, one flat stage;
4. run the local experts on the received rows as a top-1 layer (the routed
   weight is applied inside GEMM2, exactly as on one GPU);
5. send the per-(token, slot) results back with the inverse all-to-all and
   combine each token's ``k`` slots in slot order.

Because every (token, slot) result is computed by the same kernels on the
same row, and the slots are summed in the same order, the output equals the
single-GPU layer bit for bit.

Two transports carry steps 3 and 5:

* ``EPWindow`` (the GPU default): each rank owns an exchange window mapped
  into every peer through CUDA IPC; the dispatch kernel stores rows straight
  into the owners' windows, the expert GEMM2 stores its results straight back
  into the source ranks' windows, and device flags with epochs replace the
  host synchronisation (three library calls per layer, no collective on the
  data path);
* ``ep_dispatch_combine``: ``torch.distributed`` all-to-alls (nccl on GPUs,
  gloo in the CPU tests, where a caller-supplied ``local_fn`` stands in for
  the kernels), with one host read of the split sizes.
"""

from __future__ import annotations

from typing import Callable, Optional

import ctypes

import torch
import torch.distributed as dist

LocalFn = Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor]


def _mark(marks: Optional[list], name: str) -> None:
    """Record a CUDA event named ``name`` on the current stream into ``marks`` (phase timing)."""
    if marks is not None:
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        marks.append((name, ev))


def _exchange(t: torch.Tensor, out_splits, in_splits, group) -> torch.Tensor:
    out = t.new_empty((sum(out_splits),) + tuple(t.shape[1:]))
    dist.all_to_all_single(out, t.contiguous(), output_split_sizes=list(out_splits),
                           input_split_sizes=list(in_splits), group=group)
    return out


def ep_dispatch_combine(x: torch.Tensor, topk_w: torch.Tensor, topk_ids: torch.Tensor,
                        experts_per_rank: int, local_fn: LocalFn, group=None,
                        marks: Optional[list] = None) -> torch.Tensor:
    """Steps 2-5 above.  ``local_fn(rows, local_expert_ids, routed_w) -> rows`` computes
    ``routed_w * expert(row)`` (bf16) for each received row."""
    world = dist.get_world_size(group)
    T, H = x.shape
    k = topk_ids.shape[1]
    if x.is_cuda:
        return _ep_cuda(x, topk_w, topk_ids, experts_per_rank, local_fn, group, world, marks)
    ids = topk_ids.reshape(-1).to(torch.int64)
    dest = torch.div(ids, experts_per_rank, rounding_mode="floor")
    order = torch.argsort(dest, stable=True)                     # sorted (token, slot) entries
    send_counts = torch.bincount(dest, minlength=world)
    rows = x.index_select(0, torch.div(order, k, rounding_mode="floor"))
    recv_counts = torch.empty_like(send_counts)
    dist.all_to_all_single(recv_counts, send_counts, group=group)
    counts = torch.stack([send_counts, recv_counts]).tolist()
    sc, rc = counts[0], counts[1]
    meta = torch.stack([(ids[order] - dest[order] * experts_per_rank).to(torch.int32),
                        topk_w.reshape(-1)[order].to(torch.float32).view(torch.int32)], dim=1)
    recv_rows = _exchange(rows, rc, sc, group)
    recv_meta = _exchange(meta, rc, sc, group)
    if recv_rows.shape[0]:
        y = local_fn(recv_rows, recv_meta[:, 0].contiguous(), recv_meta[:, 1].contiguous().view(torch.float32))
    else:
        y = recv_rows.new_empty((0, H))
    back = _exchange(y.to(x.dtype), sc, rc, group)
    y_slots = x.new_empty((T * k, H))
    y_slots.index_copy_(0, order, back)
    # combine in slot order, fp32 sum, one rounding (as the single-GPU combine)
    acc = torch.zeros((T, H), dtype=torch.float32, device=x.device)
    ys = y_slots.view(T, k, H)
    for j in range(k):
        acc += ys[:, j].float()
    return acc.to(x.dtype)


def _ep_cuda(x, topk_w, topk_ids, experts_per_rank, local_fn, group, world, marks=None):
    """The same steps on the package's kernels (called below the dispatcher): grouping over
    ranks (moe_align), one pack kernel for rows + metadata, two NCCL all-to-alls out and one
    back, the local layer, one combine kernel.  The single host synchronisation reads the
    split sizes NCCL needs."""
    from . import ops
    T, H = x.shape
    k = topk_ids.shape[1]
    ids32 = topk_ids.to(torch.int32)
    dest = torch.div(ids32, experts_per_rank, rounding_mode="floor")
    offsets, order = ops._moe_align_impl(dest, world)
    rows, lid, wts, inv = ops._ep_pack_impl(x, ids32, topk_w, order, experts_per_rank)
    meta = torch.stack([lid, wts.view(torch.int32)], dim=1)
    send_counts = (offsets[1:] - offsets[:-1]).to(torch.int64)
    _mark(marks, "pack")
    recv_counts = torch.empty_like(send_counts)
    dist.all_to_all_single(recv_counts, send_counts, group=group)
    counts = torch.stack([send_counts, recv_counts]).tolist()
    sc, rc = counts[0], counts[1]
    _mark(marks, "counts")
    recv_rows = _exchange(rows, rc, sc, group)
    recv_meta = _exchange(meta, rc, sc, group)
    _mark(marks, "dispatch")
    if recv_rows.shape[0]:
        y = local_fn(recv_rows, recv_meta[:, 0:1], recv_meta[:, 1:2].view(torch.float32))
    else:
        y = recv_rows.new_empty((0, H))
    _mark(marks, "experts")
    back = _exchange(y, sc, rc, group)
    _mark(marks, "return")
    out = ops._ep_combine_impl(back, inv, k)
    _mark(marks, "combine")
    return out


def local_packed_fn(packed, impl: int) -> LocalFn:
    """The local experts through the B200 kernels, as a top-1 layer."""
    from . import ops

    def fn(rows: torch.Tensor, local_ids: torch.Tensor, routed_w: torch.Tensor) -> torch.Tensor:
        return ops._fused_moe_packed_impl(rows, packed.qw1, packed.sw1, packed.qw2, packed.sw2,
                                          routed_w.reshape(-1, 1), local_ids.reshape(-1, 1), packed.bits, impl)
    return fn


def ep_moe_layer(x: torch.Tensor, gate_w: torch.Tensor, packed, top_k: int, rank: int, world: int,
                 bias: Optional[torch.Tensor] = None, renormalize: bool = False, impl: int = 0,
                 group=None, window: Optional["EPWindow"] = None,
                 marks: Optional[list] = None) -> torch.Tensor:
    """One expert-parallel MoE layer on this rank's tokens ``x`` [T_r, H]: over the
    peer-memory ``window`` when one is given, else over torch.distributed all-to-alls.
    ``marks``, when given, collects (phase name, CUDA event) pairs recorded at the end of
    each phase on the current stream."""
    from . import ops
    _mark(marks, "start")
    topk_w, topk_ids, _ = ops._route_impl(x, gate_w, top_k, bias, renormalize)
    _mark(marks, "route")
    if window is not None:
        return window.layer(x, topk_w, topk_ids, packed, impl, marks=marks)
    return ep_dispatch_combine(x, topk_w, topk_ids, packed.num_experts, local_packed_fn(packed, impl),
                               group=group, marks=marks)


class EPWindow:
    """This rank's peer-memory exchange window for expert-parallel layers.

    ``max_tokens``: the most tokens this rank passes to one layer call (the
    window holds ``max_tokens * top_k`` entries from every rank).  Creating and
    closing a window are collective over ``group``; the calls in between are
    not -- ranks only meet through device flags.  One window serves every layer
    of a model (the calls are ordered on one stream)."""

    def __init__(self, max_tokens: int, top_k: int, hidden: int, rank: int, world: int,
                 device: torch.device, group=None):
        from ._lib import check, load
        lib = load()
        self.rank, self.world, self.k, self.hidden = rank, world, top_k, hidden
        self.cap = max(1, max_tokens * top_k)
        self.device = torch.device(device)
        self.group = group
        self.nbytes = lib.llq_ep_window_bytes(world, self.cap, hidden)
        handle = ctypes.create_string_buffer(lib.llq_ipc_handle_bytes())
        base = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            check(lib.llq_ipc_alloc(self.nbytes, ctypes.byref(base), handle), "ep window")
        self.base = base.value
        self._opened = []
        bases = [0] * world
        bases[rank] = self.base
        if world > 1:
            handles = [None] * world
            dist.all_gather_object(handles, handle.raw, group=group)
            with torch.cuda.device(self.device):
                for r in range(world):
                    if r == rank:
                        continue
                    p = ctypes.c_void_p()
                    check(lib.llq_ipc_open(ctypes.create_string_buffer(handles[r], len(handles[r])),
                                           ctypes.byref(p)), "ep window open")
                    bases[r] = p.value
                    self._opened.append(p.value)
            dist.barrier(group=group)
        self.peers = torch.tensor(bases, dtype=torch.int64, device=self.device)
        self.epoch = 0
        self._ws = None

    def _workspace(self, E: int, I: int) -> torch.Tensor:
        from ._lib import load
        n = load().llq_ep_experts_workspace_size(self.world, self.cap, E, self.hidden, I)
        if self._ws is None or self._ws.numel() < n:
            self._ws = torch.empty(n, dtype=torch.uint8, device=self.device)
        return self._ws

    def layer(self, x: torch.Tensor, topk_w: torch.Tensor, topk_ids: torch.Tensor, packed, impl: int,
              marks: Optional[list] = None) -> torch.Tensor:
        """Steps 2-5 for routed tokens ``x`` [T, H] against this rank's expert shard ``packed``."""
        from ._lib import check, load
        from .ops import _group_of, _stream
        lib = load()
        T, H = x.shape
        k = topk_ids.shape[1]
        if H != self.hidden or T * k > self.cap:
            raise ValueError(f"window holds {self.cap} entries of hidden size {self.hidden}; "
                             f"got T*k = {T * k}, H = {H}")
        x = x.contiguous()
        ids = topk_ids.contiguous().to(torch.int32)
        w = topk_w.contiguous().to(torch.float32)
        E_local, I = packed.num_experts, packed.intermediate
        self.epoch = (self.epoch + 1) & 0xFFFFFFFF
        st = _stream(x)
        inv = torch.empty(T * k, dtype=torch.int32, device=x.device)
        check(lib.llq_ep_dispatch(x.data_ptr(), ids.data_ptr(), w.data_ptr(), T, k, H, E_local, self.base,
                                  self.peers.data_ptr(), self.rank, self.world, self.cap, self.epoch,
                                  inv.data_ptr(), st), "ep_dispatch")
        _mark(marks, "dispatch")
        ws = self._workspace(E_local, I)
        check(lib.llq_ep_experts(self.base, self.peers.data_ptr(), self.rank, self.world, self.cap, self.epoch,
                                 packed.qw1.data_ptr(), packed.sw1.data_ptr(), packed.qw2.data_ptr(),
                                 packed.sw2.data_ptr(), E_local, H, I, packed.bits,
                                 _group_of(packed.qw1, packed.sw1, packed.bits), T * k, ws.data_ptr(),
                                 ws.numel(), impl, st), "ep_experts")
        _mark(marks, "experts")
        out = torch.empty(T, H, dtype=torch.bfloat16, device=x.device)
        check(lib.llq_ep_combine_wait(self.base, self.rank, self.world, self.cap, self.epoch, inv.data_ptr(),
                                      T, k, H, out.data_ptr(), st), "ep_combine")
        _mark(marks, "combine")
        return out

    def close(self) -> None:
        """Collective: unmap the peers' windows and free this one."""
        from ._lib import check, load
        if self.base is None:
            return
        lib = load()
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for p in self._opened:
                check(lib.llq_ipc_close(p), "ep window close")
            self._opened = []
        if self.world > 1:
            dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            check(lib.llq_ipc_free(self.base), "ep window free")
        self.base = None


def set_wait_timeout_ms(ms: int) -> None:
    """Bound of every cross-GPU wait of the peer-memory path (default 5000 ms)."""
    from ._lib import check, load
    check(load().llq_ep_set_timeout_ms(int(ms)), "ep timeout")
