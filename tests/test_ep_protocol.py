"""Expert-parallel exchange protocol on the CPU: world_size-2 gloo ranks run
the message flow of the peer-memory expert-parallel forward
(qauntrunner_b200/csrc/ep.cuh, qrmoe.cu) with the oracle's arithmetic and must
reproduce the single-process oracle forward bit for bit: each rank routes its
own tokens, sends every rank the top-k rows of all its tokens and the token
rows only of tokens with an expert there, computes its experts for the
assignments it holds, stores each output row at row t*k+j of the owner's one
receive block, runs the shared expert for its own tokens, and the owner
combines in slot order (residual, w_j y_j in slot order, shared expert)."""
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
        idx_own = np.ascontiguousarray(r["topk_idx"].astype(np.int32))
        # 2. records to every rank q: the top-k rows of all T tokens; the token
        #    rows only of tokens with an expert on q (all of them to itself).
        #    Point-to-point messages stand in for the stores into q's mailbox.
        owners = idx_own // epr                                   # [T][k] holder rank of each slot
        xn_all = np.full((WORLD * T, d), np.nan, np.float32)      # rows never sent stay unread
        idx_all = np.zeros((WORLD * T, k), np.int32)
        reqs = []
        for qq in range(WORLD):
            rows = [t for t in range(T) if qq == rank or (owners[t] == qq).any()]
            payload = np.zeros((T, d + k + 1), np.float32)
            payload[:, d:d + k] = idx_own.view(np.float32)
            for t in rows:
                payload[t, :d] = r["xn"][t]
                payload[t, d + k] = 1.0                           # "row sent" marker (for the check below)
            if qq == rank:
                mine = payload
            else:
                reqs.append(dist.isend(torch.from_numpy(payload), qq))
        got = {rank: mine}
        for qq in range(WORLD):
            if qq != rank:
                buf = torch.empty((T, d + k + 1))
                dist.recv(buf, qq)
                got[qq] = buf.numpy()
        for rq in reqs:
            rq.wait()
        for p_ in range(WORLD):
            pl = got[p_]
            idx_all[p_ * T:(p_ + 1) * T] = np.ascontiguousarray(pl[:, d:d + k]).view(np.int32)
            sent = pl[:, d + k] == 1.0
            xn_all[p_ * T:(p_ + 1) * T][sent] = pl[sent, :d]
        # 3. this rank's experts for the assignments it holds (gathered token
        #    u = owner*T + t, slot j) -> owner's block row t*k + j
        out_rows = {qq: {} for qq in range(WORLD)}
        for u in range(WORLD * T):
            qq, tl = divmod(u, T)
            for j in range(k):
                e = int(idx_all[u, j])
                if first <= e < first + epr:
                    assert not np.isnan(xn_all[u]).any(), "a needed token row was not sent"
                    out_rows[qq][tl * k + j] = _expert(case, e, xn_all[u])
        # the shared expert for this rank's own tokens only
        ys = np.stack([_expert(case, 0, r["xn"][t], shared=True) for t in range(T)]) if case.shared else None
        # 4. output rows to their owners: one [T*k][d] block per owner, each
        #    row written by the one rank that holds the slot's expert
        recv = np.full((T * k, d), np.nan, np.float32)
        for rr, y in out_rows[rank].items():
            recv[rr] = y
        for step in range(1, WORLD):
            dst, src = (rank + step) % WORLD, (rank - step) % WORLD
            rows = sorted(out_rows[dst])
            msg = np.zeros((T * k, d + 1), np.float32)
            for rr in rows:
                msg[rr, :d] = out_rows[dst][rr]
                msg[rr, d] = 1.0
            buf = torch.empty((T * k, d + 1))
            sreq = dist.isend(torch.from_numpy(msg), dst)
            dist.recv(buf, src)
            sreq.wait()
            b = buf.numpy()
            for rr in np.nonzero(b[:, d] == 1.0)[0]:
                recv[rr] = b[rr, :d]
        # 5. combine on the owner in slot order
        out = np.zeros((T, d), np.float32)
        for t in range(T):
            acc = x[t].astype(np.float32).copy()
            for j in range(k):
                y = recv[t * k + j]
                acc = (acc + (np.float32(r["topk_w"][t, j]) * y).astype(np.float32)).astype(np.float32)
            if ys is not None:
                acc = (acc + (np.float32(1.0) * ys[t]).astype(np.float32)).astype(np.float32)
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
