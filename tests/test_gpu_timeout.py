"""Failure paths of the bounded device waits, without faulting a GPU: the
waits give up on things nothing completes (an mbarrier nothing arrives at, a
peer flag nothing raises) and report QRM_E_TIMEOUT while the device stays
usable; an expert-parallel rank whose peer skips a forward gets
QRM_E_TIMEOUT from qrm_sync and both layers are destroyed in bounded time.
Also sweeps the routing kernels' binary32 exp over every float against the C
runtime's expf (what the reference's MathF.Exp calls)."""
import ctypes as C
import os
import subprocess
import tempfile
import time

import numpy as np
import pytest

import qauntrunner_b200 as Q
from tests.gpu_helpers import assert_parity
from tests.moe_case import make_case, make_input
from tests import oracle_api as O

pytestmark = pytest.mark.gpu


def test_bounded_waits_give_up_and_device_stays_usable():
    gave = (C.c_int * 2)()
    t0 = time.time()
    rc = Q.lib().qrm_selftest_waits(0, 20000, gave)     # 20 ms
    dt = time.time() - t0
    assert rc == Q.E_TIMEOUT, Q.lib().qrm_last_error().decode()
    assert list(gave) == [1, 1]
    assert dt < 5.0
    # the context is still good: a forward runs and matches the oracle
    case = make_case("c5", seed=3, d_model=512, expert_ffn=256, n_experts=16, n_active=4)
    assert_parity(case, make_input(case, 2, seed=4), O.APPLY_NORM)


HOST_EXPF = r"""
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <thread>
#include <vector>
extern "C" void host_expf(uint32_t first, uint32_t count, uint32_t* out, int nt) {
    std::vector<std::thread> th;
    for (int t = 0; t < nt; t++)
        th.emplace_back([=]() {
            for (uint64_t i = t; i < count; i += nt) {
                uint32_t b = first + (uint32_t)i;
                float x; memcpy(&x, &b, 4);
                float y = expf(x);
                memcpy(out + i, &y, 4);
            }
        });
    for (auto& x : th) x.join();
}
"""


def test_device_expf_matches_c_runtime_on_all_floats():
    import torch
    with tempfile.TemporaryDirectory() as td:
        src, so = os.path.join(td, "h.cpp"), os.path.join(td, "libh.so")
        with open(src, "w") as fh:
            fh.write(HOST_EXPF)
        subprocess.run(["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-pthread", src, "-o", so, "-lm"], check=True)
        h = C.CDLL(so)
        h.host_expf.argtypes = [C.c_uint32, C.c_uint32, C.c_void_p, C.c_int]
        n = 1 << 27
        dev = torch.empty(n, dtype=torch.int32, device="cuda")
        got = torch.empty(n, dtype=torch.int32).pin_memory()
        want = np.empty(n, np.uint32)
        nt = max(1, (os.cpu_count() or 2) - 1)
        bad = 0
        for first in range(0, 1 << 32, n):
            Q._check(Q.lib().qrm_selftest_expf(first, n, dev.data_ptr(), None))
            got.copy_(dev)
            h.host_expf(first, n, want.ctypes.data, nt)
            g = got.numpy().view(np.uint32)
            diff = g != want
            if diff.any():
                gn = (g & 0x7F800000) == 0x7F800000
                wn = (want & 0x7F800000) == 0x7F800000
                both_nan = gn & wn & ((g & 0x7FFFFF) != 0) & ((want & 0x7FFFFF) != 0)
                bad += int((diff & ~both_nan).sum())
        assert bad == 0, f"{bad} floats whose device exp differs from the C runtime's expf"


def _ep_rank(rank, nccl_id, skip, q):
    os.environ["QRM_EP_P2P"] = "1"
    os.environ["QRM_WAIT_LIMIT_US"] = "300000"
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch
    from tests.gpu_helpers import make_layer
    try:
        torch.cuda.set_device(rank)
        case = make_case("c5", seed=31, d_model=1024, expert_ffn=512, n_experts=16, n_active=4)
        x = make_input(case, 1, seed=9 + rank)
        ep = make_layer(case, max_tokens=1, device=rank, rank=rank, world=2, nccl_id=nccl_id)
        code = 0
        if rank != skip:
            try:
                ep.forward(x, apply_norm=True)
                ep.sync()
            except Q.QrmError as ex:
                code = ex.code
        t0 = time.time()
        ep.close()   # collective: both ranks meet here
        q.put((rank, code, time.time() - t0, None))
    except Exception as ex:
        q.put((rank, None, None, repr(ex)))


def test_ep_rank_that_skips_a_forward():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import queue
    import torch.multiprocessing as mp
    nid = Q.nccl_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_ep_rank, args=(r, nid, 1, q)) for r in range(2)]
    for p in procs:
        p.start()
    res, t0 = [], time.time()
    while len(res) < 2:
        try:
            res.append(q.get(timeout=2))
        except queue.Empty:
            assert not [p for p in procs if p.exitcode not in (None, 0)], "a rank failed"
            assert time.time() - t0 < 240, "ranks did not finish"
    for p in procs:
        p.join(timeout=60)
    res = {r[0]: r for r in res}
    for r in (0, 1):
        assert res[r][3] is None, f"rank {r}: {res[r][3]}"
    assert res[0][1] == Q.E_TIMEOUT, f"rank 0 got {res[0][1]}"
    assert res[1][1] == 0
    assert res[0][2] < 30 and res[1][2] < 30
