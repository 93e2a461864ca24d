"""Expert-parallel dispatch/combine host logic on CPU ranks (gloo, world_size 2).

The local experts are the numpy oracle; the layer assembled across two ranks
must equal the oracle's single-process layer on the same tokens and routing,
bit for bit (every (token, slot) row goes through the same arithmetic and the
slots are summed in the same order).
"""

from __future__ import annotations

import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import moe as M
from oracle import symmetric as S

E, H, I, K, T = 8, 64, 32, 2, 24


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _case():
    rng = np.random.default_rng(0)
    w1 = (rng.standard_normal((E, 2 * I, H)) * 0.05).astype(np.float32)
    w2 = (rng.standard_normal((E, H, I)) * 0.05).astype(np.float32)
    q1, s1, *_ = S.quantize_tensor(S.round_to_bf16(w1), 4, 32)
    q2, s2, *_ = S.quantize_tensor(S.round_to_bf16(w2), 4, 32)
    x = S.round_to_bf16(rng.standard_normal((2 * T, H)).astype(np.float32))
    ids = np.stack([rng.choice(E, K, replace=False) for _ in range(2 * T)]).astype(np.int32)
    ids[:5] = [0, 1]   # tokens routed only to rank 0's experts
    ids[5:9] = [6, 7]  # and only to rank 1's
    w = (rng.random((2 * T, K)) / K).astype(np.float32)
    return q1, s1, q2, s2, x, ids, w


def _row_fn(w1d, w2d):
    def one(xrow, e, wt):
        y, _ = M.expert_ffn_rows(xrow[None, :], w1d[e], w2d[e], np.array([wt], np.float32))
        return y[0]
    return one


def _worker(rank, world, port, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from llada_quant_b200.ep import ep_dispatch_combine
    q1, s1, q2, s2, x, ids, w = _case()
    epr = E // world
    one = _row_fn(*M.dequantize_experts(q1, s1, q2, s2, 4))

    def local_fn(rows, local_ids, routed_w):
        r = rows.float().numpy()
        out = np.stack([one(r[i], rank * epr + int(local_ids[i]), float(routed_w[i]))
                        for i in range(rows.shape[0])]) if rows.shape[0] else np.zeros((0, H), np.float32)
        return torch.from_numpy(out).to(torch.bfloat16)

    sl = slice(rank * T, (rank + 1) * T)
    out = ep_dispatch_combine(torch.from_numpy(x[sl]).to(torch.bfloat16), torch.from_numpy(w[sl]),
                              torch.from_numpy(ids[sl]), epr, local_fn)
    np.save(f"{out_path}.{rank}.npy", out.float().numpy())
    dist.barrier()
    dist.destroy_process_group()


def test_ep_two_ranks_equals_single_process(tmp_path):
    path = str(tmp_path / "ep")
    mp.start_processes(_worker, args=(2, _free_port(), path), nprocs=2, join=True, start_method="spawn")
    got = np.concatenate([np.load(f"{path}.{r}.npy") for r in range(2)])
    q1, s1, q2, s2, x, ids, w = _case()
    one = _row_fn(*M.dequantize_experts(q1, s1, q2, s2, 4))
    ref = np.zeros((2 * T, H), np.float32)
    for j in range(K):
        ys = np.stack([one(x[t], ids[t, j], w[t, j]) for t in range(2 * T)])
        ref = (ref + ys).astype(np.float32)
    assert np.array_equal(got, S.round_to_bf16(ref))
