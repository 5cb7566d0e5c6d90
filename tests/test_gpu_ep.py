"""Expert parallelism on 2 GPUs: each rank holds half of the routed experts;
its forward (own tokens; the exchanges inside the library, as NVLink stores
into the peer's memory or as NCCL all-gather and send/recv) must equal a
single-GPU layer holding every expert on the same tokens, bit for bit, and the
routing must be identical, over several consecutive forwards (the peer-memory
flags advance per forward).  Skipped with fewer than 2 GPUs."""
import numpy as np
import pytest

import qauntrunner_b200 as Q

pytestmark = pytest.mark.gpu

WORLD = 2


def _gpus():
    import torch
    return torch.cuda.device_count()


def _rank(rank, nccl_id, cfgname, over, T, transport, q):
    import os
    import torch
    os.environ["QRM_EP_P2P"] = "1" if transport == "peer" else "0"
    from tests.gpu_helpers import make_layer
    from tests.moe_case import make_case, make_input
    try:
        torch.cuda.set_device(rank)
        case = make_case(cfgname, seed=31, **over)
        x_all = make_input(case, WORLD * T, seed=9)
        x = np.ascontiguousarray(x_all[rank * T:(rank + 1) * T])
        ep = make_layer(case, max_tokens=T, device=rank, rank=rank, world=WORLD, nccl_id=nccl_id)
        single = make_layer(case, max_tokens=WORLD * T, device=rank)
        assert ep.ep_transport() == transport, ep.ep_transport()
        res = []
        for flags in (Q.APPLY_NORM, Q.APPLY_NORM | Q.ADD_RESIDUAL, Q.APPLY_NORM, Q.APPLY_NORM):
            out, idx, w = ep.forward(x, apply_norm=True, add_residual=bool(flags & Q.ADD_RESIDUAL))
            ro, ri, rw = single.forward(x_all, apply_norm=True, add_residual=bool(flags & Q.ADD_RESIDUAL))
            sl = slice(rank * T, (rank + 1) * T)
            res.append((bool(np.array_equal(idx, ri[sl])), bool(np.array_equal(w, rw[sl])),
                        bool(np.array_equal(out, ro[sl])), float(np.max(np.abs(out - ro[sl])))))
        ep.sync()
        ep.close()
        single.close()
        q.put((rank, res, None))
    except Exception as ex:  # report instead of hanging the parent
        q.put((rank, None, repr(ex)))


@pytest.mark.parametrize("transport", ["peer", "nccl"])
@pytest.mark.parametrize("cfgname,over,T", [
    ("c5", dict(d_model=1024, expert_ffn=512, n_experts=16, n_active=4), 1),
    ("c5", dict(d_model=1024, expert_ffn=512, n_experts=16, n_active=4), 3),
    ("c1", dict(n_experts=8), 2),
])
def test_ep_equals_single_gpu(cfgname, over, T, transport):
    if _gpus() < WORLD:
        pytest.skip("needs 2 GPUs")
    import queue
    import time
    import torch.multiprocessing as mp
    nid = Q.nccl_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, nid, cfgname, over, T, transport, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res, t0 = [], time.time()
    while len(res) < WORLD:
        try:
            res.append(q.get(timeout=2))
        except queue.Empty:
            assert not [p for p in procs if p.exitcode not in (None, 0)], "a rank failed"
            assert time.time() - t0 < 300, "ranks did not finish"
    for p in procs:
        p.join(timeout=60)
    for rank, r, err in sorted(res, key=lambda v: v[0]):
        assert err is None, f"rank {rank}: {err}"
        for idx_eq, w_eq, out_eq, md in r:
            assert idx_eq and w_eq, f"rank {rank}: routing differs"
            assert out_eq, f"rank {rank}: output differs by {md}"
