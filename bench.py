"""Benchmark: W4A16 MoE-layer tokens/s at the LLaDA-MoE-7B-A1B shape on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one MoE layer forward (router + align + permute + W4A16 GEMM1 with
SiLU + GEMM2 with routed weight + combine) over T=256 tokens (32 masked
positions x batch 8, ~32 tokens/expert), E=64, H=2048, I=1024, top-8,
INT4 group 128 (the C3 layer).  Synthetic seeded data: weights N(0,0.02)
bf16 quantized by this package's pack kernel, x ~ N(0,1) bf16, router N(0,0.02).
Steps rotate over 4 distinct layer weight sets (855 MB > the 126 MB L2), so no
step reads weights left in L2 by the previous one.

At N > 1 the layer runs expert-parallel (experts sharded contiguously), T=256
tokens per rank (weak scaling); rows travel by peer-memory stores through each
rank's exchange window (``--ep-transport window``, the default) or by NCCL
all-to-alls (``--ep-transport nccl``).

Timing: the K-step region (barrier + synchronize on both sides, CUDA events,
max over ranks) is repeated until at least one second of steps has been timed;
``ms_per_step`` is the total over all repeats divided by their steps.  After
every timed region the device error word (bounded waits that gave up) is read,
and a non-zero word fails the run.

At N = 1 the line also carries ``gpu_reference``: the reference's own PACKED
algorithm on the same B200 -- dequantize every expert to BF16 (the property's
fresh tensor per access) and a routed BF16 grouped matmul -- in torch ops; and
``c4``: the 16-layer stack over batch 32 x seq 1024 tokens (tensor-bound).
At N > 1 it carries ``c5`` (the Zipf-skewed token sweep), ``phases`` (per-rank
CUDA-event time of each exchange step, min and max over ranks) and
``nccl_transport`` (the same layer over NCCL all-to-alls).

``--impl reference`` times the reference's CPU path (the numpy port of
dequantize_tensor + the routed dequant-then-matmul, oracle/moe.py) on the host
cores, rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

E, H, I, TOPK, BITS, GROUP = 64, 2048, 1024, 8, 4, 128
T_PER_RANK = 256
N_LAYERS = 4
METRIC = "W4A16 MoE-layer tokens/s (LLaDA-MoE-7B-A1B layer, T=256, top-8)"
UNIT = "tokens/s"


def layer_bytes(T: int, k: int, experts_hit: int) -> int:
    """Algorithmic HBM bytes of one layer call: packed w1/w2 + fp32 scales of every expert
    hit, x in, out written, router weights, routing ids + weights."""
    per_expert = (2 * I * H // 2) + (2 * I * H // GROUP) * 4 + (H * I // 2) + (H * I // GROUP) * 4
    return experts_hit * per_expert + 2 * T * H * 2 + E * H * 2 + T * k * 8


def gemm1_bytes(n_rows: int, experts_hit: int) -> int:
    """Bytes one GEMM1 launch must move: packed w1 + scales of the experts hit, the permuted
    activation rows in, the bf16 SiLU(gate)*up rows out."""
    return experts_hit * ((2 * I * H // 2) + (2 * I * H // GROUP) * 4) + n_rows * H * 2 + n_rows * I * 2


def fused_bytes(n_rows: int, experts_hit: int) -> int:
    """Bytes the fused GEMM1+GEMM2 launch must move: packed w1, w2 and their scales for the
    experts hit, the permuted activation rows in, the (token, slot) output rows out (h stays
    inside the launch's L2 working set and is not counted)."""
    per_expert = (2 * I * H // 2) + (2 * I * H // GROUP) * 4 + (H * I // 2) + (H * I // GROUP) * 4
    return experts_hit * per_expert + n_rows * H * 2 + n_rows * H * 2


def bench_config(world: int, gemm: str, ep_transport: str, router_bias: str) -> dict:
    """The workload description both arms print (identical dicts for the same command)."""
    return {"workload": "C3 LLaDA-MoE-7B-A1B layer: E=64 H=2048 I=1024 top-8 W4A16 g128",
            "tokens_per_rank": T_PER_RANK, "gemm": gemm,
            "parallelism": "ep%d" % world if world > 1 else "single",
            "ep_transport": (ep_transport if world > 1 else None),
            "router_bias": router_bias,
            "l2": "inputs larger than L2: 4 rotated layer weight sets (4 x 214 MB)"}


MIN_TIMED_S = 1.0


def timed_steps(step, steps: int, world: int, device, barrier, min_seconds: float = MIN_TIMED_S):
    """Repeat the K-step region (barrier + synchronize on both sides, CUDA events) until at
    least ``min_seconds`` of steps are timed.  Returns (ms per step, max over ranks; repeats;
    seconds timed)."""
    import torch
    import torch.distributed as dist
    total_ms, repeats = 0.0, 0
    while True:
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for i in range(steps):
            step(i)
        b.record()
        torch.cuda.synchronize()
        barrier()
        ms = a.elapsed_time(b)
        if world > 1:
            t = torch.tensor([ms], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        total_ms += ms
        repeats += 1
        # ms is the max over ranks, so every rank takes the same decision
        if total_ms >= min_seconds * 1e3 or repeats >= 100000:
            break
    return total_ms / (repeats * steps), repeats, total_ms / 1e3


def check_device_error(where: str) -> int:
    """Read the library's device error word after a timed region; a non-zero word (a bounded
    wait that gave up) fails the run."""
    from llada_quant_b200 import ops
    code = ops.device_error()
    if code != 0:
        raise SystemExit(f"bench: device error word 0x{code:x} after {where}")
    return code


def read_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def read_traffic(name):
    """Per-launch DRAM bytes of the dominant kernel from its committed ncu summary."""
    if name is None:
        return None
    path = os.path.join(ROOT, "profiles", name)
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return int(line.split(":", 1)[1].strip())
    except OSError:
        pass
    return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.rows = []
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True,
                                     timeout=5).stdout.strip()
                if out:
                    self.rows.append([c.strip() for c in out.split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            for name, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(self.rows)}


_CPU_CASE = {}


def _cpu_case():
    """Seeded C3 layer for the CPU path, quantized once by the oracle (not timed)."""
    if not _CPU_CASE:
        import torch
        from oracle import symmetric as S
        g = torch.Generator().manual_seed(0)
        w1 = (torch.randn(E, 2 * I, H, generator=g) * 0.02).to(torch.bfloat16).float().numpy()
        q1, s1, *_ = S.quantize_tensor(w1, bits=BITS, group_size=GROUP)
        del w1
        w2 = (torch.randn(E, H, I, generator=g) * 0.02).to(torch.bfloat16).float().numpy()
        q2, s2, *_ = S.quantize_tensor(w2, bits=BITS, group_size=GROUP)
        del w2
        gate_w = (torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16).float().numpy()
        x = torch.randn(T_PER_RANK, H, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16).float().numpy()
        _CPU_CASE.update(q1=q1, s1=s1, q2=q2, s2=s2, gate_w=gate_w, x=x)
    return _CPU_CASE


def cpu_reference(sample_layers: int = 1, threads=None):
    """Time the reference CPU path on a bounded sample: ``sample_layers`` C3 layer calls of
    256 tokens, each dequantizing every expert (what the PACKED property does) and running
    the routed dequant-then-matmul.  With the unmodified reference installed in
    baseline/_ref this is its own ``dequantize_tensor`` in torch on the host cores plus the
    routed restatement (kind "reference"); otherwise the numpy port (kind "port").
    Returns (tokens/s, cores, seconds, kind)."""
    from threadpoolctl import threadpool_limits
    c = _cpu_case()
    cores = threads or os.cpu_count()
    pkg = _reference_package()
    if pkg is not None:
        import torch
        RS = pkg[0]
        torch.set_num_threads(cores)
        if "torch" not in c:
            from llada_quant_b200.moe import PackedExperts
            c["torch"] = (torch.from_numpy(c["x"]).to(torch.bfloat16), torch.from_numpy(c["gate_w"]).to(torch.bfloat16),
                          PackedExperts(torch.from_numpy(c["q1"]), torch.from_numpy(c["s1"]),
                                        torch.from_numpy(c["q2"]), torch.from_numpy(c["s2"]), BITS, GROUP))
        x, gate_w, layer = c["torch"]
        deq = lambda q, sc: RS.dequantize_tensor(q, sc, BITS, GROUP, dtype=torch.bfloat16, packed=True)
        t0 = time.perf_counter()
        for _ in range(sample_layers):
            _ref_layer(x, gate_w, layer, False, deq)
        dt = time.perf_counter() - t0
        return sample_layers * T_PER_RANK / dt, cores, dt, "reference"
    from oracle import moe as M
    with threadpool_limits(limits=cores):
        t0 = time.perf_counter()
        for _ in range(sample_layers):
            M.moe_layer(c["x"], c["gate_w"], c["q1"], c["s1"], c["q2"], c["s2"], TOPK, BITS)
        dt = time.perf_counter() - t0
    return sample_layers * T_PER_RANK / dt, cores, dt, "port"


def run_reference(args, rank: int):
    """The reference arm: rank 0 times the CPU path; warm-up is capped at one call (it only
    faults pages in) so that the whole run stays within a few minutes."""
    if rank != 0:
        return
    vals = []
    for _ in range(min(args.warmup, 1)):
        cpu_reference(1)
    cores = os.cpu_count()
    kind = "port"
    for _ in range(args.steps):
        v, cores, dt, kind = cpu_reference(1)
        vals.append(v)
    value = statistics.median(vals)
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": T_PER_RANK / value * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int4 weights, bf16 activations, fp32 accumulate",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) tokens)", "impl": "reference",
        "config": bench_config(args.gpus, args.gemm, args.ep_transport, args.router_bias),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": kind,
                         "sample": "one C3 layer call (256 tokens) per step: "
                                   + ("the reference's own dequantize_tensor (baseline/_ref) in torch on the host"
                                      " cores + the routed dequant-then-matmul" if kind == "reference" else
                                      "numpy port of the reference's PACKED dequantize + routed dequant-then-matmul")},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def make_layers(device, n_layers: int, E_local: int, e0: int):
    """Quantize ``n_layers`` seeded layer weight sets on the GPU with this package's pack kernel."""
    import torch
    from llada_quant_b200 import symmetric as G
    from llada_quant_b200.moe import PackedExperts

    layers = []
    for l in range(n_layers):
        g = torch.Generator(device=device).manual_seed(1000 + l)
        packs = []
        for shape in ((E, 2 * I, H), (E, H, I)):
            w = (torch.randn(*shape, generator=g, device=device) * 0.02).to(torch.bfloat16)[e0:e0 + E_local]
            r = G.quantize_tensor(w.contiguous(), bits=BITS, group_size=GROUP)
            packs.append(r)
            del w
        layers.append(PackedExperts(packs[0].q, packs[0].scale, packs[1].q, packs[1].scale, BITS, GROUP))
    g = torch.Generator(device=device).manual_seed(1)
    gate_w = (torch.randn(E, H, generator=g, device=device) * 0.02).to(torch.bfloat16)
    return layers, gate_w


def _ref_dequantize(q, s, bits: int):
    """The reference's dequantize_tensor on PACKED buffers (symmetric.py:272-293, unpack_int4
    :316-346) in torch ops: sign-extend both nibbles, fp32 q * scale per group, cast to bf16."""
    import torch
    if bits == 4:
        lo = torch.bitwise_right_shift(torch.bitwise_left_shift(q, 4), 4)
        hi = torch.bitwise_right_shift(q, 4)
        v = torch.stack([lo, hi], dim=-1).reshape(*q.shape[:-1], q.shape[-1] * 2)
    else:
        v = q
    g = s.shape[-1]
    K = v.shape[-1]
    w = v.float().reshape(*v.shape[:-1], g, K // g) * s.float().unsqueeze(-1)
    return w.reshape(v.shape).to(torch.bfloat16)


def _reference_package():
    """The unmodified reference installed in baseline/_ref (pip --target), when present."""
    path = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(path):
        return None
    if path not in sys.path:
        sys.path.insert(0, path)
    try:
        from LLaDA_Quant.algorithms import symmetric as RS
        from LLaDA_Quant.runtime import moe as RM
        from LLaDA_Quant.runtime.kernels import w8a16_gemm as RK
        return RS, RM, RK
    except Exception:
        return None


def _ref_layer(x, gate_w, layer, grouped: bool, deq):
    """The reference PACKED forward on the GPU: block.w1/w2 dequantized afresh by ``deq``
    (the PACKED property, runtime/moe.py:199-216), router softmax(fp32).topk
    (trajectory/llada.py:225-234), and the routed FFN in the fused_moe rounding order
    (INFERENCE_REPO_CHANGES.md:259-265, 296-309) as BF16 matmuls (torch._grouped_mm, or
    one matmul per expert)."""
    import torch
    import torch.nn.functional as F
    W1 = deq(layer.qw1, layer.sw1)
    W2 = deq(layer.qw2, layer.sw2)
    probs = F.softmax(F.linear(x, gate_w), dim=-1, dtype=torch.float32)
    tw, ti = probs.topk(TOPK, dim=-1)
    flat = ti.reshape(-1)
    order = torch.argsort(flat, stable=True)
    counts = torch.bincount(flat, minlength=E)
    xs = x.index_select(0, order // TOPK)
    if grouped:
        offs = torch.cumsum(counts, 0).to(torch.int32)
        a = torch._grouped_mm(xs, W1.transpose(1, 2), offs=offs)
    else:
        a = torch.empty(xs.shape[0], 2 * I, dtype=torch.bfloat16, device=x.device)
        c = counts.tolist()
        o = 0
        for e in range(E):
            if c[e]:
                a[o:o + c[e]] = xs[o:o + c[e]] @ W1[e].t()
            o += c[e]
    gt, up = a[:, :I].float(), a[:, I:].float()
    h = ((gt / (1.0 + torch.exp(-gt))).to(torch.bfloat16).float() * up).to(torch.bfloat16)
    if grouped:
        # the grouped GEMM only returns its input dtype: the bf16 result is widened before the
        # routed-weight multiply (one extra bf16 rounding of the expert output)
        y = torch._grouped_mm(h, W2.transpose(1, 2), offs=offs).float()
    else:
        y = torch.empty(h.shape[0], H, dtype=torch.float32, device=x.device)
        o = 0
        for e in range(E):
            if c[e]:
                y[o:o + c[e]] = (h[o:o + c[e]] @ W2[e].t()).float()
            o += c[e]
    y = (y * tw.reshape(-1)[order].unsqueeze(1)).to(torch.bfloat16)
    slots = torch.empty_like(y)
    slots[order] = y
    return slots.view(-1, TOPK, H).float().sum(dim=1).to(torch.bfloat16)


def _time_ref(fn, steps):
    import torch
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(steps):
        fn(i)
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / steps


def time_gpu_reference(xs, gate_w, layers, args, device):
    """The reference algorithm on the same B200, timed like our device value: the
    reference's own dequantize_tensor (eager, and its torch.compile'd variant) from
    baseline/_ref when installed, else its restatement in torch ops."""
    import torch
    pkg = _reference_package()
    if pkg is not None:
        RS, RM, _ = pkg
        eager = lambda q, sc: RS.dequantize_tensor(q, sc, BITS, GROUP, dtype=torch.bfloat16, packed=True)
        source = "baseline/_ref (unmodified LLaDA_Quant package): dequantize_tensor"
    else:
        eager = lambda q, sc: _ref_dequantize(q, sc, BITS)
        source = "restatement of dequantize_tensor in torch ops (baseline/_ref not installed)"
    grouped, grouped_error = True, None
    try:
        _ref_layer(xs[0], gate_w, layers[0], True, eager)
        torch.cuda.synchronize()
    except Exception as exc:  # recorded in the line, never hidden
        grouped, grouped_error = False, f"{type(exc).__name__}: {exc}"[:300]
    steps = max(3, min(args.steps, 10))
    out = {}
    variants = [("eager", eager)]
    if pkg is not None:
        comp = RM.compiled_dequantize()
        variants.append(("compiled", lambda q, sc: comp(q, sc, BITS, GROUP, dtype=torch.bfloat16, packed=True)))
    for name, deq in variants:
        try:
            for i in range(max(2, min(args.warmup, 3))):
                _ref_layer(xs[i % N_LAYERS], gate_w, layers[i % N_LAYERS], grouped, deq)
            torch.cuda.synchronize()
            ms = _time_ref(lambda i: _ref_layer(xs[i % N_LAYERS], gate_w, layers[i % N_LAYERS], grouped, deq), steps)
            out[name] = {"value": T_PER_RANK / (ms / 1e3), "unit": UNIT, "ms_per_step": ms, "steps": steps}
        except Exception as exc:  # a failing baseline leg is reported, never hidden
            out[name] = {"error": f"{type(exc).__name__}: {exc}"[:200]}
    from llada_quant_b200 import ops
    ref = _ref_layer(xs[0], gate_w, layers[0], grouped, eager).float()
    tw, ids, _ = ops._route_impl(xs[0], gate_w, TOPK, None, False)
    ours = ops._fused_moe_packed_impl(xs[0], layers[0].qw1, layers[0].sw1, layers[0].qw2, layers[0].sw2, tw, ids,
                                      BITS, 0).float()
    best = min((v for v in out.values() if "value" in v), key=lambda v: v["ms_per_step"], default=None)
    line = {"source": source,
            "method": "PACKED dequantize of w1/w2 to bf16 per call + "
                      + ("torch._grouped_mm" if grouped else "per-expert torch matmul") + " (bf16)",
            "rel_l2_vs_ours": float((ours - ref).norm() / ref.norm()), "variants": out,
            "grouped_mm_error": grouped_error}
    if best is not None:
        line.update(value=best["value"], unit=UNIT, ms_per_step=best["ms_per_step"])
    return line


def time_w8a16_comparator(device):
    """The reference's Triton w8a16_gemm (runtime/kernels/w8a16_gemm.py:74-85) against this
    package's dense W8A16 kernel on the same plain GEMM (K=2048, N=8192, 16 MiB of int8
    weights, 12 rotated copies so that no call reads weights left in L2)."""
    import torch
    pkg = _reference_package()
    if pkg is None or not pkg[2].HAS_TRITON:
        return {"unavailable": "baseline/_ref with Triton is not installed"}
    RK = pkg[2]
    from llada_quant_b200 import ops
    K, N, copies = 2048, 8192, 12
    g = torch.Generator(device=device).manual_seed(7)
    ws = [torch.randint(-127, 128, (N, K), generator=g, device=device, dtype=torch.int8) for _ in range(copies)]
    ss = [torch.rand(N, K // 128, generator=g, device=device) * 0.01 for _ in range(copies)]
    rows = []
    for M in (16, 64, 128, 256):
        a = torch.randn(M, K, generator=g, device=device).to(torch.bfloat16)
        for i in range(3):
            RK.w8a16_gemm(a, ws[i], ss[i])
            ops._quant_linear_impl(a, ws[i], ss[i], 8)
        torch.cuda.synchronize()
        t_ref = _time_ref(lambda i: RK.w8a16_gemm(a, ws[i % copies], ss[i % copies]), 24)
        t_ours = _time_ref(lambda i: ops._quant_linear_impl(a, ws[i % copies], ss[i % copies], 8), 24)
        y_ref = RK.w8a16_gemm(a, ws[0], ss[0]).float()
        y_ours = ops._quant_linear_impl(a, ws[0], ss[0], 8).float()
        rows.append({"M": M, "reference_triton_us": round(t_ref * 1e3, 2), "ours_us": round(t_ours * 1e3, 2),
                     "rel_l2": float((y_ours - y_ref).norm() / y_ref.norm())})
    return {"shape": {"K": K, "N": N, "bits": 8, "group": 128}, "rows": rows,
            "note": "per call, host-launched (both sides pay their launch overhead)"}


def phase_breakdown(call, n: int, world: int, device) -> dict:
    """Per-phase CUDA-event time of ``n`` layer calls (``call(i, marks)`` appends (name, event)
    pairs), averaged per call on each rank, then the min and max over ranks of each phase."""
    import torch
    import torch.distributed as dist
    runs = []
    for i in range(n):
        marks = []
        call(i, marks)
        runs.append(marks)
    torch.cuda.synchronize()
    names = [m[0] for m in runs[0][1:]]
    per = torch.zeros(len(names), dtype=torch.float64)
    for marks in runs:
        for j in range(1, len(marks)):
            per[j - 1] += marks[j - 1][1].elapsed_time(marks[j][1])
    per /= n
    per = per.to(device)
    if world > 1:
        lo, hi = per.clone(), per.clone()
        dist.all_reduce(lo, op=dist.ReduceOp.MIN)
        dist.all_reduce(hi, op=dist.ReduceOp.MAX)
    else:
        lo = hi = per
    lo, hi = lo.tolist(), hi.tolist()
    return {name: {"ms_min": round(lo[j], 4), "ms_max": round(hi[j], 4)} for j, name in enumerate(names)}


def c5_sweep(args, world: int, rank: int, device, layers, gate_w, barrier) -> list:
    """The C5 workload at this world size: the C3 layer expert-parallel with the Zipf(1.1)
    router bias b_e = -1.1 ln(rank_e), T tokens per rank for T in 256..65536 (a point is
    skipped, with its reason, when its exchange window would not fit in free memory).
    Tokens/s of the whole job, ms per layer (max over ranks), the HBM fraction of the layer
    bytes each rank reads (its expert shard) and the tensor fraction of the layer FLOPs."""
    import torch
    import torch.distributed as dist
    from llada_quant_b200 import ep, ops
    from llada_quant_b200.fused_moe import IMPL
    impl = IMPL[args.gemm]
    rank_e = torch.randperm(E, generator=torch.Generator().manual_seed(3)).to(torch.float32) + 1.0
    bias = (-1.1 * torch.log(rank_e)).to(device)
    hbm, _ = read_peaks()
    tflops_peak, _ = read_tensor_peak()
    E_local = E // world
    shard_bytes = E_local * ((2 * I * H // 2) + (2 * I * H // GROUP) * 4 + (H * I // 2) + (H * I // GROUP) * 4)
    out = []
    for T in (256, 1024, 4096, 16384, 65536):
        need = 2 * world * T * TOPK * H * 2 + 6 * T * TOPK * max(H, I) * 2
        free = torch.tensor([float(torch.cuda.mem_get_info(device)[0])], device=device)
        if world > 1:
            dist.all_reduce(free, op=dist.ReduceOp.MIN)
        if need > 0.8 * float(free.item()):
            out.append({"T_per_rank": T, "skipped": f"needs ~{need / 2**30:.1f} GiB of exchange buffers"})
            continue
        g = torch.Generator(device=device).manual_seed(50 + rank)
        xs = [torch.randn(T, H, generator=g, device=device).to(torch.bfloat16) for _ in range(2)]
        window = ep.EPWindow(T, TOPK, H, rank, world, device) if args.ep_transport == "window" else None

        def step(i):
            return ep.ep_moe_layer(xs[i & 1], gate_w, layers[i % N_LAYERS], TOPK, rank, world, bias=bias,
                                   impl=impl, window=window)
        ops.clear_device_error()
        for i in range(2):
            step(i)
        steps = 10 if T <= 4096 else 4
        ms, repeats, timed_s = timed_steps(step, steps, world, device, barrier, min_seconds=0.3)
        dev_err = check_device_error(f"the C5 region at T={T}")
        flops = 2.0 * T * world * TOPK * (2 * I * H + H * I) / world  # per rank, balanced share
        out.append({"T_per_rank": T, "tokens_per_s": T * world / (ms / 1e3), "ms_per_step": round(ms, 4),
                    "hbm_frac": round(shard_bytes / (ms / 1e3) / 1e9 / hbm, 4),
                    "tensor_frac": round(flops / (ms / 1e3) / 1e12 / tflops_peak, 4),
                    "timed_region_s": round(timed_s, 3), "device_error": dev_err})
        if window is not None:
            window.close()
        del xs
        torch.cuda.empty_cache()
    return out


def run_ours(args, rank: int, world: int, local_rank: int):
    import torch
    import torch.distributed as dist

    from llada_quant_b200 import ops
    from llada_quant_b200.fused_moe import IMPL

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    impl = IMPL[args.gemm]
    if world > 1:
        from llada_quant_b200 import ep
        E_local = E // world
        layers, gate_w = make_layers(device, N_LAYERS, E_local, rank * E_local)
    else:
        E_local = E
        layers, gate_w = make_layers(device, N_LAYERS, E, 0)
    g = torch.Generator(device=device).manual_seed(2 + rank)
    xs = [torch.randn(T_PER_RANK, H, generator=g, device=device).to(torch.bfloat16) for _ in range(N_LAYERS)]
    bias = None
    if args.router_bias == "zipf":
        # C5 skew: b_e = -1.1 ln(rank_e), rank_e a seeded permutation of 1..E
        rank_e = torch.randperm(E, generator=torch.Generator().manual_seed(3)).to(torch.float32) + 1.0
        bias = (-1.1 * torch.log(rank_e)).to(device)
    window = None
    if world > 1 and args.ep_transport == "window":
        window = ep.EPWindow(T_PER_RANK, TOPK, H, rank, world, device)

    def step(i):
        layer = layers[i % N_LAYERS]
        x = xs[i % N_LAYERS]
        if world > 1:
            return ep.ep_moe_layer(x, gate_w, layer, TOPK, rank, world, bias=bias, impl=impl, window=window)
        return ops._moe_block_packed_impl(x, gate_w, bias, False, layer.qw1, layer.sw1, layer.qw2, layer.sw2, TOPK,
                                          BITS, impl)[0]

    def barrier():
        if world > 1:
            dist.barrier()

    # ---- warm-up + timed device region -------------------------------------------
    ops.clear_device_error()
    for i in range(args.warmup):
        step(i)
    with ClockSampler(local_rank) as clocks:
        ms_per_step, repeats, timed_s = timed_steps(step, args.steps, world, device, barrier)
    dev_err = check_device_error("the timed device region")
    tokens_per_step = T_PER_RANK * world
    value = tokens_per_step / (ms_per_step / 1e3)

    # ---- end to end through the public API with pinned host buffers ---------------
    # Every step copies its tokens in from pinned host memory and its result back out.
    # The copies run on their own streams, so step i+1's input lands while step i
    # computes and step i's result leaves while step i+1 computes; the timed region
    # starts before the first input copy and ends after the last result copy.
    from llada_quant_b200.fused_moe import moe_layer
    x_host = [x.cpu().pin_memory() for x in xs]
    out_host = [torch.empty(T_PER_RANK, H, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    x_dev = [torch.empty(T_PER_RANK, H, dtype=torch.bfloat16, device=device) for _ in range(2)]
    comp = torch.cuda.current_stream(device)
    h2d, d2h = torch.cuda.Stream(device), torch.cuda.Stream(device)
    in_ready = [torch.cuda.Event() for _ in range(2)]
    computed = [torch.cuda.Event() for _ in range(2)]
    out_done = [torch.cuda.Event() for _ in range(2)]
    used = [False, False]

    def layer_call(x, i):
        if world > 1:
            from llada_quant_b200 import ep
            return ep.ep_moe_layer(x, gate_w, layers[i % N_LAYERS], TOPK, rank, world, bias=bias, impl=impl,
                                   window=window)
        return moe_layer(x, gate_w, layers[i % N_LAYERS], TOPK, bias=bias, impl=args.gemm)

    def issue_input(i):
        b = i & 1
        with torch.cuda.stream(h2d):
            if used[b]:
                h2d.wait_event(computed[b])  # the layer that read this buffer has finished
            x_dev[b].copy_(x_host[i % N_LAYERS], non_blocking=True)
            in_ready[b].record(h2d)

    outs = [None, None]  # each result stays referenced until its copy-back is known done

    def e2e_run(n, start=None):
        used[0] = used[1] = False
        if start is not None:
            h2d.wait_event(start)
        issue_input(0)
        for i in range(n):
            b = i & 1
            comp.wait_event(in_ready[b])
            if outs[b] is not None:
                comp.wait_event(out_done[b])  # later allocations on this stream may reuse its memory
                outs[b] = None
            out = layer_call(x_dev[b], i)
            computed[b].record(comp)
            used[b] = True
            if i + 1 < n:
                issue_input(i + 1)
            with torch.cuda.stream(d2h):
                d2h.wait_event(computed[b])
                out_host[b].copy_(out, non_blocking=True)
                out_done[b].record(d2h)
            outs[b] = out
        comp.wait_stream(d2h)

    e2e_run(args.warmup)
    torch.cuda.synchronize()
    ms_e2e_total, e2e_repeats = 0.0, 0
    while ms_e2e_total < MIN_TIMED_S * 1e3:
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record(comp)
        e2e_run(args.steps, start=s2)
        e2.record(comp)
        torch.cuda.synchronize()
        barrier()
        ms_e2e = s2.elapsed_time(e2)
        if world > 1:
            t = torch.tensor([ms_e2e], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms_e2e = float(t.item())
        ms_e2e_total += ms_e2e
        e2e_repeats += 1
    check_device_error("the end-to-end region")
    e2e_value = tokens_per_step / (ms_e2e_total / (e2e_repeats * args.steps) / 1e3)

    # ---- dominant kernel (the fused expert GEMMs) timed alone with CUDA events ---------
    kernel = None
    if world == 1:
        preps = []
        for l in range(N_LAYERS):
            tw, ids, _ = ops.route(xs[l], gate_w, TOPK, bias, False)
            offsets, slots = ops.moe_align(ids, E)
            xsrt = ops.moe_permute(xs[l], slots, TOPK, args.gemm == "tcgen05_fast")
            hit = int((offsets[1:] - offsets[:-1] > 0).sum().item())
            preps.append((xsrt, offsets, slots, tw, hit))
        n_rows = T_PER_RANK * TOPK
        fused = args.gemm in ("auto", "tcgen05")
        if fused:
            counters = ops.gemm12_counters(n_rows, E, device)
            run = lambda l: ops._moe_gemm12_impl(preps[l][0], preps[l][1], preps[l][2], preps[l][3], layers[l].qw1,
                                                 layers[l].sw1, layers[l].qw2, layers[l].sw2, BITS, counters)
        else:
            run = lambda l: ops.moe_gemm1(preps[l][0], preps[l][1], layers[l].qw1, layers[l].sw1, BITS, impl)
        for l in range(N_LAYERS):
            run(l)
        torch.cuda.synchronize()
        k_ms, _, _ = timed_steps(lambda i: run(i % N_LAYERS), max(args.steps, 8), 1, device, barrier)
        check_device_error("the dominant-kernel region")
        hit = int(round(statistics.mean(p[4] for p in preps)))
        algo = fused_bytes(n_rows, hit) if fused else gemm1_bytes(n_rows, hit)
        peak, peak_kind = read_peaks()
        achieved = algo / (k_ms / 1e3) / 1e9
        prof = "fused_gemms_c3.txt" if fused else None  # ncu summaries cover the default kernel
        kernel = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                  "frac": round(achieved / peak, 4), "peak_source": peak_kind, "traffic": read_traffic(prof),
                  "kernel": ("moe GEMM1 + GEMM2 in one launch (W4A16, SiLU and routed-weight epilogues)" if fused
                             else "moe GEMM1 (W4A16, SiLU epilogue)"),
                  "algorithmic_bytes": algo, "launch_ms": round(k_ms, 5)}
        layer_algo = layer_bytes(T_PER_RANK, TOPK, hit)
        layer_gbs = layer_algo / (ms_per_step / 1e3) / 1e9
        kernel["layer"] = {"algorithmic_bytes": layer_algo, "achieved": round(layer_gbs, 1),
                           "frac": round(layer_gbs / peak, 4)}

    gpu_ref = w8a16 = None
    if world == 1 and not args.no_gpu_ref:
        gpu_ref = time_gpu_reference(xs, gate_w, layers, args, device)
        w8a16 = time_w8a16_comparator(device)

    # ---- the other BASELINE workloads at this world size ------------------------------
    extras = {}
    if world == 1 and not args.no_c4:
        extras["c4"] = measure_c4(args, steps=3, warmup=1)
        extras["pack"] = measure_pack(device)
    if world > 1:
        from llada_quant_b200 import ep as _ep
        extras["phases"] = {
            "transport": args.ep_transport,
            "per_layer": phase_breakdown(
                lambda i, m: _ep.ep_moe_layer(xs[i % N_LAYERS], gate_w, layers[i % N_LAYERS], TOPK, rank, world,
                                              bias=bias, impl=impl, window=window, marks=m), 20, world, device)}
        if args.ep_transport == "window":
            # the same layer over NCCL all-to-alls, on the same box, for comparison
            nccl_step = lambda i: _ep.ep_moe_layer(xs[i % N_LAYERS], gate_w, layers[i % N_LAYERS], TOPK, rank,
                                                   world, bias=bias, impl=impl, window=None)
            for i in range(3):
                nccl_step(i)
            ms_n, rep_n, ts_n = timed_steps(nccl_step, args.steps, world, device, barrier, min_seconds=0.5)
            check_device_error("the NCCL-transport region")
            extras["nccl_transport"] = {
                "value": tokens_per_step / (ms_n / 1e3), "unit": UNIT, "ms_per_step": ms_n,
                "timed_region_s": round(ts_n, 3),
                "phases": phase_breakdown(
                    lambda i, m: _ep.ep_moe_layer(xs[i % N_LAYERS], gate_w, layers[i % N_LAYERS], TOPK, rank,
                                                  world, bias=bias, impl=impl, window=None, marks=m),
                    10, world, device)}
        if not args.no_c5:
            extras["c5"] = c5_sweep(args, world, rank, device, layers, gate_w, barrier)

    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu:
            cpu_reference(1)  # warm-up: page in, thread pools
            v, cores, dt, kind = cpu_reference(1)
            cpu = {"value": v, "unit": UNIT, "cores": cores, "kind": kind,
                   "sample": f"one C3 layer call (256 tokens), {dt:.2f} s: "
                             + ("the reference's own dequantize_tensor (baseline/_ref) in torch + routed matmul"
                                if kind == "reference" else "numpy port of the reference CPU path")}
        # ours per step: router, align, permute, GEMM1+GEMM2 (one launch in exact mode), combine; at N > 1 over the
        # window: router, dispatch, align, permute, GEMM1, GEMM2, combine; over NCCL: router,
        # rank grouping, pack, align, permute, GEMM1, GEMM2, combine, slot combine
        fused_path = args.gemm in ("auto", "tcgen05")
        launches_per_step = (5 if fused_path else 6) if world == 1 else (7 if window is not None else 9)
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int4 weights, bf16 activations, fp32 accumulate",
            "data": "synthetic (seeded N(0,0.02) weights quantized on device, N(0,1) tokens)",
            "config": bench_config(world, args.gemm, args.ep_transport, args.router_bias),
            "timing": {"repeats": repeats, "timed_region_s": round(timed_s, 3), "device_error": dev_err},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": T_PER_RANK * H * 2,
                    "d2h_bytes_per_step": T_PER_RANK * H * 2,
                    "copies": "pinned host <-> device every step, on their own streams, overlapped with the "
                              "neighbouring steps' layers"},
            "gpu_launches": launches_per_step * args.steps * repeats,
            "roofline": kernel,
            "cpu_baseline": cpu,
            "clocks": clocks.summary(),
        }
        if gpu_ref is not None:
            line["gpu_reference"] = gpu_ref
        if w8a16 is not None:
            line["gpu_reference_w8a16_gemm"] = w8a16
        line.update(extras)
        print(json.dumps(line), flush=True)
    if window is not None:
        window.close()


C4_TOKENS, C4_LAYERS = 32 * 1024, 16


def c4_flops() -> float:
    """Algorithmic FLOPs of one C4 step: 16 layers x (router + GEMM1 + GEMM2) over 32768 tokens."""
    per_layer = 2.0 * C4_TOKENS * TOPK * (2 * I * H + H * I) + 2.0 * C4_TOKENS * H * E
    return per_layer * C4_LAYERS


def measure_pack(device) -> dict:
    """The quantize-and-pack kernel on the C3 w1 tensor (bf16 [64, 2048, 2048], amax, INT4
    group 128): HBM bytes it must move (bf16 read, packed codes + fp32 scales written) over its
    CUDA-event time, two rotated copies so that no call reads its input from L2."""
    import torch
    from llada_quant_b200 import ops
    g = torch.Generator(device=device).manual_seed(0)
    ws = [(torch.randn(E, 2 * I, H, generator=g, device=device) * 0.02).to(torch.bfloat16) for _ in range(2)]
    q = torch.empty(E, 2 * I, H // 2, dtype=torch.int8, device=device)
    sc = torch.empty(E, 2 * I, H // GROUP, dtype=torch.float32, device=device)
    from llada_quant_b200._lib import check, load, LLQ_BF16, LLQ_F32, LLQ_SEARCH_AMAX
    lib = load()
    st = torch.cuda.current_stream(device).cuda_stream

    def call(i):
        w = ws[i & 1]
        check(lib.llq_quantize_pack(w.data_ptr(), LLQ_BF16, E * 2 * I, H, BITS, GROUP, LLQ_SEARCH_AMAX, 24, 0.5,
                                    LLQ_F32, 1, q.data_ptr(), sc.data_ptr(), st), "quantize_pack")
    for i in range(3):
        call(i)
    ms, repeats, timed_s = timed_steps(call, 10, 1, device, lambda: None, min_seconds=0.5)
    algo = ws[0].numel() * 2 + q.numel() + sc.numel() * 4
    hbm, kind = read_peaks()
    gbs = algo / (ms / 1e3) / 1e9
    del ws
    torch.cuda.empty_cache()
    return {"kernel": "quantize_g128_bf16_kernel (amax, INT4 g128) on C3 w1", "algorithmic_bytes": algo,
            "launch_ms": round(ms, 5), "achieved": round(gbs, 1), "unit": "GB/s", "peak": hbm,
            "frac": round(gbs / hbm, 4), "peak_source": kind, "timed_region_s": round(timed_s, 3)}


def read_tensor_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops_sustained"]), "measured (sustained)"
    except Exception:
        return 1400.0, "fallback (sustained)"


def measure_c4(args, steps: int, warmup: int) -> dict:
    """The C4 workload: 16 chained C3-shaped layers (x <- x + moe_l(x)) over 32768 tokens on one
    GPU; attention/norms are outside the hot path and not modelled.  Tokens/s of the stack, with
    TFLOP/s against the measured sustained dense bf16 peak (a seconds-long step)."""
    import torch
    from llada_quant_b200 import ops
    from llada_quant_b200.fused_moe import IMPL
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    layers, gate_w = make_layers(device, C4_LAYERS, E, 0)
    x0 = torch.randn(C4_TOKENS, H, generator=torch.Generator(device=device).manual_seed(2),
                     device=device).to(torch.bfloat16)
    impl = IMPL[args.gemm]

    def step(_i=0):
        x = x0
        for lay in layers:
            y = ops._moe_block_packed_impl(x, gate_w, None, False, lay.qw1, lay.sw1, lay.qw2, lay.sw2, TOPK, BITS,
                                           impl)[0]
            x = x + y
        return x

    ops.clear_device_error()
    for _ in range(warmup):
        step()
    with ClockSampler(0) as clocks:
        ms, repeats, timed_s = timed_steps(step, steps, 1, device, lambda: None)
    dev_err = check_device_error("the C4 region")
    tflops = c4_flops() / (ms / 1e3) / 1e12
    peak, kind = read_tensor_peak()
    out = {"workload": "C4 16-layer MoE stack, T=32768 (batch 32 x seq 1024), E=64 H=2048 I=1024 top-8 W4A16 g128",
           "value": C4_TOKENS / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms, "steps": steps,
           "repeats": repeats, "timed_region_s": round(timed_s, 3), "device_error": dev_err,
           "roofline": {"bound": "tensor", "achieved": round(tflops, 1), "peak": peak, "unit": "TFLOP/s",
                        "frac": round(tflops / peak, 4), "peak_source": kind, "algorithmic_flops": c4_flops()},
           "clocks": clocks.summary()}
    del layers
    torch.cuda.empty_cache()
    return out


def run_c4(args):
    """--workload c4: the C4 stack as its own bench line."""
    c4 = measure_c4(args, args.steps, args.warmup)
    line = {
        "metric": "W4A16 MoE stack tokens/s (LLaDA-MoE-7B-A1B, 16 layers, batch 32 x seq 1024)",
        "value": c4["value"], "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": c4["ms_per_step"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int4 weights, bf16 activations, fp32 accumulate",
        "data": "synthetic (seeded N(0,0.02) weights quantized on device, N(0,1) tokens)",
        "config": {"workload": c4["workload"], "gemm": args.gemm,
                   "l2": "inputs larger than L2 (16 layer weight sets, 3.4 GB)"},
        "roofline": dict(c4["roofline"], traffic=None),
        "gpu_launches": 7 * C4_LAYERS * args.steps * c4["repeats"],
        "timing": {"repeats": c4["repeats"], "timed_region_s": c4["timed_region_s"],
                   "device_error": c4["device_error"]},
        "clocks": c4["clocks"],
    }
    print(json.dumps(line), flush=True)


def kernel_case_pack():
    """The pack kernel on the C3 w1 tensor: one bf16 [64, 2048, 2048] weight (537 MB)
    quantized to packed INT4 + fp32 scales (amax, group 128), twice."""
    import torch
    from llada_quant_b200 import symmetric as G
    device = torch.device("cuda", 0)
    w = (torch.randn(E, 2 * I, H, generator=torch.Generator(device=device).manual_seed(0), device=device)
         * 0.02).to(torch.bfloat16)
    for _ in range(2):
        r = G.quantize_tensor(w, bits=BITS, group_size=GROUP)
    torch.cuda.synchronize()
    print(json.dumps({"kernel_case": "pack", "bytes_in": w.numel() * 2,
                      "bytes_out": r.q.numel() + r.scale.numel() * 4}))


def kernel_case_c4():
    """One C4-sized layer call (T = 32768 tokens, top-8): the weights dequantized once, then the
    bf16 expert GEMMs from shared memory; twice."""
    import torch
    from llada_quant_b200 import ops
    device = torch.device("cuda", 0)
    layers, gate_w = make_layers(device, 1, E, 0)
    lay = layers[0]
    x = torch.randn(C4_TOKENS, H, generator=torch.Generator(device=device).manual_seed(2),
                    device=device).to(torch.bfloat16)
    for _ in range(2):
        tw, ids, _ = ops._route_impl(x, gate_w, TOPK, None, False)
        y = ops._fused_moe_packed_impl(x, lay.qw1, lay.sw1, lay.qw2, lay.sw2, tw, ids, BITS, 0)
    torch.cuda.synchronize()
    print(json.dumps({"kernel_case": "C4 layer", "out_abs_mean": float(y.float().abs().mean())}))


def kernel_case(args):
    """One C3 layer weight set, route -> align -> permute -> fused GEMM1+GEMM2 (exact; two
    launches in fast mode) -> combine, twice."""
    if args.case == "pack":
        return kernel_case_pack()
    if args.case == "c4":
        return kernel_case_c4()
    import torch
    from llada_quant_b200 import ops
    from llada_quant_b200.fused_moe import IMPL
    device = torch.device("cuda", 0)
    layers, gate_w = make_layers(device, 1, E, 0)
    lay = layers[0]
    x = torch.randn(T_PER_RANK, H, generator=torch.Generator(device=device).manual_seed(2),
                    device=device).to(torch.bfloat16)
    impl = IMPL[args.gemm]
    for _ in range(2):
        tw, ids, _ = ops.route(x, gate_w, TOPK, None, False)
        off, slots = ops.moe_align(ids, E)
        xs = ops.moe_permute(x, slots, TOPK, args.gemm == "tcgen05_fast")
        if args.gemm in ("auto", "tcgen05"):
            counters = ops.gemm12_counters(T_PER_RANK * TOPK, E, device)
            y = ops._moe_gemm12_impl(xs, off, slots, tw, lay.qw1, lay.sw1, lay.qw2, lay.sw2, BITS, counters)
        else:
            h = ops.moe_gemm1(xs, off, lay.qw1, lay.sw1, BITS, impl)
            y = ops.moe_gemm2(h, off, slots, tw, lay.qw2, lay.sw2, BITS, impl)
        out = ops.moe_combine(y, TOPK)
    torch.cuda.synchronize()
    print(json.dumps({"kernel_case": "C3", "gemm": args.gemm, "out_abs_mean": float(out.float().abs().mean())}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--gemm", choices=["auto", "tcgen05", "tcgen05_fast", "simt"], default="auto")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-c4", action="store_true", help="N=1: skip the C4 stack measurement")
    ap.add_argument("--no-c5", action="store_true", help="N>1: skip the C5 token sweep")
    ap.add_argument("--no-gpu-ref", action="store_true",
                    help="skip the reference-algorithm-on-B200 leg (dequantize + BF16 matmul)")
    ap.add_argument("--ep-transport", choices=["window", "nccl"], default="window",
                    help="expert-parallel row exchange at N > 1")
    ap.add_argument("--router-bias", choices=["none", "zipf"], default="none",
                    help="zipf: the C5 per-expert router bias -1.1 ln(rank_e) (skewed expert load)")
    ap.add_argument("--workload", choices=["c3", "c4"], default="c3",
                    help="c3: one LLaDA-MoE layer at 256 tokens (default, HBM-bound); c4: the 16-layer "
                         "stack over batch 32 x seq 1024 tokens (tensor-bound)")
    ap.add_argument("--case", choices=["c3", "pack", "c4"], default="c3",
                    help="with --kernel-case: which kernels to run (the C3 layer, the pack kernel on C3 w1, "
                         "one C4-sized layer)")
    ap.add_argument("--kernel-case", action="store_true",
                    help="run the C3 layer's kernels twice on one small input set and exit "
                         "(the command the ncu captures under profiles/ were taken on)")
    args = ap.parse_args()
    if args.kernel_case:
        kernel_case(args)
        return
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if args.workload == "c4":
        run_c4(args)
        return
    if world > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
