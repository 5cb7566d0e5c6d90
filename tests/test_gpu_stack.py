"""MoE layer stacks (qrm_stack_*): the residual stream through n layers on the
device equals the chain of the same layers run one by one (bit for bit),
whether the layers' weights are resident in HBM or streamed from pinned host
memory through the two device slots (several forwards, so the slots are
refilled across forwards), and each layer of that chain matches the oracle
on its own input (routing bit-exact, output within 1e-3)."""
import numpy as np
import pytest

import qauntrunner_b200 as Q
from tests import oracle_api as O
from tests.gpu_helpers import OUT_TOL, make_layer, row_rel_err
from tests.moe_case import make_case, make_input

pytestmark = pytest.mark.gpu

N_LAYERS = 5
SHAPE = dict(d_model=512, expert_ffn=1024, n_experts=8, n_active=2)


def _cases(name):
    return [make_case(name, seed=100 + l, **SHAPE) for l in range(N_LAYERS)]


def _stack(cases, T, budget):
    c = cases[0]
    cfg = c.cfg
    S = Q.MoeStack(N_LAYERS, cfg["d_model"], cfg["n_experts"], cfg["n_active"], cfg["expert_ffn"], hbm_budget=budget,
                   moe_sigmoid=bool(cfg["moe_sigmoid"]), routed_scale=cfg["routed_scale"], n_shared=cfg["n_shared"],
                   swiglu_limit=cfg["swiglu_limit"], rms_eps=cfg["rms_eps"],
                   fmt=(c.fmt_gate, c.fmt_up, c.fmt_down), shared_fmt=c.fmt_sh if c.shared else None, max_tokens=T)
    for L, case in zip(S.layers, cases):
        L.upload_norm(case.norm_w)
        L.upload_router(case.router, case.router_bias)
        for e in range(cfg["n_experts"]):
            L.upload_expert(e, Q.GATE, case.fmt_gate, case.gate[e])
            L.upload_expert(e, Q.UP, case.fmt_up, case.up[e])
            L.upload_expert(e, Q.DOWN, case.fmt_down, case.down[e])
        if case.shared:
            for w in range(3):
                L.upload_expert(Q.SHARED_EXPERT, w, case.fmt_sh[w], case.shared[w])
    return S


@pytest.mark.parametrize("name", ["c2", "c3"])
def test_stack_resident_and_streamed(name):
    import torch
    cases = _cases(name)
    T = 3
    flags = O.APPLY_NORM | O.ADD_RESIDUAL
    xs = [make_input(cases[0], T, seed=200 + i) for i in range(3)]
    # the chain of single layers, and the oracle on each layer's GPU input
    singles = [make_layer(c, max_tokens=T) for c in cases]
    chains = []
    try:
        for x in xs:
            cur, steps = x, []
            for L, case in zip(singles, cases):
                out, idx, _ = L.forward(cur, apply_norm=True, add_residual=True)
                steps.append((cur, out, idx))
                cur = out
            chains.append(cur)
        for (cur, out, idx), case in zip(steps, cases):   # the last input's chain, layer by layer
            ref = O.moe_forward(case, cur, flags)
            assert np.array_equal(idx, ref["topk_idx"]), "routing differs from the oracle"
            assert row_rel_err(out, ref["out"]) <= OUT_TOL
    finally:
        for L in singles:
            L.close()
    lb = None
    for budget_layers in (0, 1, 4):
        S = _stack(cases, T, 0)
        if lb is None:
            lb = S.info()[1]
        S.close()
        S = _stack(cases, T, budget_layers * lb)
        try:
            n_res, _ = S.info()
            assert n_res == (N_LAYERS if budget_layers == 0 else max(1, budget_layers - 2))
            if budget_layers:
                assert n_res < N_LAYERS
                # a streamed layer's bytes come back from its host image
                nb = O.tensor_bytes(SHAPE["d_model"] * SHAPE["expert_ffn"], cases[-1].fmt_down)
                got = S.layers[-1].download_expert(5, Q.DOWN, nb)
                assert np.array_equal(got, np.frombuffer(cases[-1].down[5], np.uint8))
            d = SHAPE["d_model"]
            xd = torch.empty((T, d), device="cuda")
            od = torch.empty((T, d), device="cuda")
            for x, want in zip(xs, chains):
                xd.copy_(torch.from_numpy(x))
                S.forward_device(xd.data_ptr(), T, od.data_ptr(), flags)
                torch.cuda.synchronize()
                S.sync()
                assert np.array_equal(od.cpu().numpy(), want), f"stack (budget {budget_layers} layers) != layer chain"
        finally:
            S.close()
