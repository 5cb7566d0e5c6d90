"""Expert-parallel exchange protocol on the CPU: world_size-2 gloo ranks run
the message flow of the expert-parallel forward (qauntrunner_b200/csrc/ep.cuh,
qrmoe.cu) with the oracle's arithmetic and must reproduce the single-process
oracle forward bit for bit: each rank routes its own tokens, all-gathers
(xn, top-k) records, computes its block of experts for every rank's tokens,
returns output block q row t*k+j to token owner q, and the owner combines in
slot order (residual, w_j y_j in slot order, shared expert)."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tests import oracle_api as O
from tests.moe_case import make_case, make_input

WORLD = 2
T = 3          # tokens per rank


def _case():
    return make_case("c5", seed=21, d_model=256, expert_ffn=256, n_experts=8, n_active=4, norm_random=True)


def _expert(case, e, xn, shared=False):
    cfg = case.cfg
    d, f = cfg["d_model"], cfg["expert_ffn"]
    limit = cfg["swiglu_limit"] if cfg["moe_sigmoid"] else 0.0
    if shared:
        gate, up, down = case.shared
        fg, fu, fd = case.fmt_sh
    else:
        gate, up, down = case.gate[e], case.up[e], case.down[e]
        fg, fu, fd = case.fmt_gate, case.fmt_up, case.fmt_down
    g = O.matvec(fg, gate, f, d, xn)
    u = O.matvec(fu, up, f, d, xn)
    return O.matvec(fd, down, d, f, O.swiglu(g, u, limit))


def _rank(rank, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        case = _case()
        cfg = case.cfg
        d, E, k = cfg["d_model"], cfg["n_experts"], min(cfg["n_active"], 8)
        epr = E // WORLD
        first = rank * epr
        flags = O.APPLY_NORM | O.ADD_RESIDUAL
        x_all = make_input(case, WORLD * T, seed=5)
        x = x_all[rank * T:(rank + 1) * T]
        # 1. route this rank's tokens
        r = O.moe_forward(case, x, flags)
        rec = np.concatenate([r["xn"], r["topk_idx"].view(np.float32), r["topk_w"]], axis=1)
        # 2. all-gather the records
        got = [torch.empty((T, d + 2 * k)) for _ in range(WORLD)]
        dist.all_gather(got, torch.from_numpy(np.ascontiguousarray(rec)))
        rec_all = torch.cat(got).numpy()
        xn_all = rec_all[:, :d]
        idx_all = np.ascontiguousarray(rec_all[:, d:d + k]).view(np.int32)
        # 3. this rank's experts for every rank's tokens; block q, row t*k+j
        send = np.zeros((WORLD, T * k, d), np.float32)
        for a in range(WORLD * T * k):
            t, j = divmod(a, k)
            e = int(idx_all[t, j])
            if first <= e < first + epr:
                qq, tl = divmod(t, T)
                send[qq, tl * k + j] = _expert(case, e, xn_all[t])
        # shared expert for all gathered tokens (the same weights stream either way)
        ys_all = np.stack([_expert(case, 0, xn_all[t], shared=True) for t in range(WORLD * T)]) if case.shared else None
        # 4. blocks back to the owners (gathered; each rank keeps the blocks meant for it)
        blocks = [torch.empty((WORLD, T * k, d)) for _ in range(WORLD)]
        dist.all_gather(blocks, torch.from_numpy(send))
        recv = np.stack([blocks[h].numpy()[rank] for h in range(WORLD)])   # [holder][T*k][d]
        # 5. combine on the owner in slot order
        out = np.zeros((T, d), np.float32)
        for t in range(T):
            acc = x[t].astype(np.float32).copy()
            for j in range(k):
                e = int(r["topk_idx"][t, j])
                y = recv[e // epr, t * k + j]
                acc = (acc + (np.float32(r["topk_w"][t, j]) * y).astype(np.float32)).astype(np.float32)
            if ys_all is not None:
                acc = (acc + (np.float32(1.0) * ys_all[rank * T + t]).astype(np.float32)).astype(np.float32)
            out[t] = acc
        ref = O.moe_forward(case, x_all, flags)
        q.put((rank, bool(np.array_equal(out, ref["out"][rank * T:(rank + 1) * T])),
               bool(np.array_equal(r["topk_idx"], ref["topk_idx"][rank * T:(rank + 1) * T])),
               float(np.max(np.abs(out - ref["out"][rank * T:(rank + 1) * T])))))
    finally:
        dist.destroy_process_group()


def test_ep_protocol_matches_single_process():
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    import queue
    import time
    res, t0 = [], time.time()
    while len(res) < WORLD:
        try:
            res.append(q.get(timeout=2))
        except queue.Empty:
            dead = [p for p in procs if p.exitcode not in (None, 0)]
            assert not dead, "a rank failed"
            assert time.time() - t0 < 240, "ranks did not finish"
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, out_equal, idx_equal, maxdiff in sorted(res):
        assert idx_equal, f"rank {rank}: routing differs"
        assert out_equal, f"rank {rank}: output differs by {maxdiff}"
