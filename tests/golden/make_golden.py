"""Generate the golden vectors that pin the CPU oracle to the reference.

Run in a container that has the LLaDA_Quant reference source tree::

    python tests/golden/make_golden.py --reference-src <path to LLaDA_Quant>/src

It imports the reference package and records, for seeded inputs, exactly what
its public functions return: ``quantize_tensor`` (amax and MSE search, INT4
and INT8, grouped and per-row fallback), ``search_group_scale``,
``dequantize_tensor``, ``pack_int4``/``unpack_int4``, the router recomputation
``softmax(gate(x), fp32).topk`` of ``RouterCapture``, and a routed MoE layer
built from the reference's own ``dequantize_tensor`` plus torch ops in the
external ``fused_moe``'s rounding order.  The output, ``golden.npz``, is small
and committed; the GPU box never needs the reference tree.
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))


def bf16_to_u16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().to(torch.float32).numpy().copy()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-src", default=os.environ.get("LLQ_REFERENCE_SRC", ""))
    ap.add_argument("--out", default=os.path.join(HERE, "golden.npz"))
    args = ap.parse_args()
    if not args.reference_src:
        raise SystemExit("pass --reference-src <LLaDA_Quant>/src")
    sys.path.insert(0, args.reference_src)
    from LLaDA_Quant.algorithms import symmetric as S  # noqa: E402

    torch.set_num_threads(1)
    out: dict[str, np.ndarray] = {}

    # -- pack / unpack: every byte, every nibble pair (test_int4.py:181-204)
    every_byte = torch.arange(-128, 128, dtype=torch.int8).reshape(1, 256)
    out["unpack_every_byte"] = S.unpack_int4(every_byte).numpy()
    vals = torch.arange(-8, 8, dtype=torch.int8)
    pairs = torch.stack(torch.meshgrid(vals, vals, indexing="ij"), -1).reshape(1, -1)
    out["pack_every_pair_in"] = pairs.numpy()
    out["pack_every_pair_out"] = S.pack_int4(pairs).numpy()

    # -- quantize_tensor cases
    cases = []
    g = torch.Generator().manual_seed(0)
    w_bf16 = (torch.randn(2, 64, 256, generator=g) * 0.02).to(torch.bfloat16)
    g = torch.Generator().manual_seed(1)
    torch.manual_seed(0)  # the heavy_tailed fixture of test_scale_search.py:46-49
    heavy = torch.distributions.StudentT(3.0).sample((32, 512)) * 0.01
    w_fp16 = (torch.randn(4, 32, 128, generator=g) * 0.05).to(torch.float16)
    w_fallback = (torch.randn(3, 7, 100, generator=g) * 0.02).to(torch.bfloat16)
    w_zero = (torch.randn(4, 8, 256, generator=g) * 0.02).to(torch.bfloat16)
    w_zero[0] = 0
    w_zero[1, :, :128] = 0
    w_zero[2, 3, 64:192] = 0
    cases += [
        ("amax_i4_g128_bf16", w_bf16, 4, 128, "amax"),
        ("amax_i8_g128_bf16", w_bf16, 8, 128, "amax"),
        ("amax_i4_g64_fp16", w_fp16, 4, 64, "amax"),
        ("amax_i8_g32_fp32", heavy, 8, 32, "amax"),
        ("amax_i4_rowfallback", w_fallback, 4, 64, "amax"),
        ("amax_i8_rowfallback", w_fallback, 8, 33, "amax"),
        ("amax_i4_zero_groups", w_zero, 4, 128, "amax"),
        ("mse_i4_g128_heavy", heavy, 4, 128, "mse"),
        ("mse_i8_g128_heavy", heavy, 8, 128, "mse"),
        ("mse_i4_g128_bf16", w_bf16, 4, 128, "mse"),
        ("mse_i4_zero_groups", w_zero, 4, 128, "mse"),
    ]
    names = []
    for name, w, bits, gs, search in cases:
        r = S.quantize_tensor(w, bits=bits, group_size=gs, scale_search=search)
        names.append(name)
        out[f"{name}/w"] = f32(w)
        out[f"{name}/dtype"] = np.array(str(w.dtype).replace("torch.", ""))
        out[f"{name}/meta"] = np.array([bits, gs, 1 if search == "mse" else 0, r.group_size, int(r.packed)])
        out[f"{name}/q"] = r.q.numpy().copy()
        out[f"{name}/scale"] = f32(r.scale)
        out[f"{name}/deq_bf16"] = bf16_to_u16(r.dequantize(torch.bfloat16))
    out["quant_cases"] = np.array(names)

    # -- search_group_scale with a short grid and chunking (test_scale_search.py:203-215)
    w_g, _ = S._as_groups(heavy, 128)
    out["search_grid8/scale"] = f32(S.search_group_scale(w_g, bits=4, grid=8, chunk_elements=0))

    # -- routing as RouterCapture recomputes it (trajectory/llada.py:225-234)
    g = torch.Generator().manual_seed(5)
    T, H, E, K = 96, 256, 16, 4
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    gate = torch.nn.Linear(H, E, bias=False)
    with torch.no_grad():
        gate.weight.copy_(torch.randn(E, H, generator=g) * 0.02)
    gate = gate.to(torch.bfloat16)
    with torch.no_grad():
        logits = gate(x)
        probs = F.softmax(logits, dim=-1, dtype=torch.float32)
        tw, ti = probs.topk(K, dim=-1)
    out["route/x"] = bf16_to_u16(x)
    out["route/gate_w"] = bf16_to_u16(gate.weight.detach())
    out["route/logits"] = bf16_to_u16(logits)
    out["route/probs"] = f32(probs)
    out["route/topk_w"] = f32(tw)
    out["route/topk_ids"] = ti.numpy().astype(np.int32)

    # -- routed MoE layer from the reference's dequantize_tensor + torch ops
    moe_cases = [("moe_i4_amax", 4, "amax"), ("moe_i8_amax", 8, "amax"), ("moe_i4_mse", 4, "mse")]
    E, H, I, T, K = 4, 256, 128, 40, 2
    g = torch.Generator().manual_seed(0)
    w1 = (torch.randn(E, 2 * I, H, generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(E, H, I, generator=g) * 0.02).to(torch.bfloat16)
    gate_w = (torch.randn(E, H, generator=torch.Generator().manual_seed(1)) * 0.02).to(torch.bfloat16)
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16)
    logits = (x.float() @ gate_w.float().t()).to(torch.bfloat16)
    probs = F.softmax(logits, dim=-1, dtype=torch.float32)
    tw, ti = probs.topk(K, dim=-1)
    out["moe/x"] = bf16_to_u16(x)
    out["moe/topk_w"] = f32(tw)
    out["moe/topk_ids"] = ti.numpy().astype(np.int32)
    out["moe/shape"] = np.array([E, H, I, T, K])
    for name, bits, search in moe_cases:
        r1 = S.quantize_tensor(w1, bits=bits, group_size=128, scale_search=search)
        r2 = S.quantize_tensor(w2, bits=bits, group_size=128, scale_search=search)
        W1 = r1.dequantize(torch.bfloat16)   # what the PACKED property returns
        W2 = r2.dequantize(torch.bfloat16)
        y = torch.zeros(T, K, H, dtype=torch.bfloat16)
        for t in range(T):
            for j in range(K):
                e = int(ti[t, j])
                acc = x[t].float() @ W1[e].float().t()
                gt = acc[:I].to(torch.bfloat16).float()
                up = acc[I:].to(torch.bfloat16).float()
                silu = (gt / (1.0 + torch.exp(-gt))).to(torch.bfloat16).float()
                h = (silu * up).to(torch.bfloat16)
                acc2 = h.float() @ W2[e].float().t()
                y[t, j] = (acc2 * tw[t, j]).to(torch.bfloat16)
        o = y.sum(dim=1)
        out[f"{name}/qw1"] = r1.q.numpy().copy()
        out[f"{name}/sw1"] = f32(r1.scale)
        out[f"{name}/qw2"] = r2.q.numpy().copy()
        out[f"{name}/sw2"] = f32(r2.scale)
        out[f"{name}/bits"] = np.array(bits)
        out[f"{name}/out"] = bf16_to_u16(o)
    out["moe_cases"] = np.array([c[0] for c in moe_cases])

    np.savez_compressed(args.out, **out)
    print(f"wrote {args.out}: {os.path.getsize(args.out)} bytes, {len(out)} arrays")


if __name__ == "__main__":
    main()
