"""The formats kept exactly as stored (Q2_K, Q3_K, Q5_K, I8_BLK, B1, B1X, T1E,
T1E_LO) on the GPU: the matrix operator against the oracle's DotKernels
restatement for several token counts, a MoE layer with such experts against
the oracle's MoE forward (routing bit-exact, outputs within 1e-3), and the
bytes read back unchanged."""
import numpy as np
import pytest

import qauntrunner_b200 as Q
from tests import oracle_api as O
from tests.gpu_helpers import OUT_TOL, assert_parity, row_rel_err
from tests.moe_case import MoeCase, make_case, make_input
from tests.raw_blocks import make_matrix

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("fmt", O.RAW_FORMATS)
def test_matrix_gemv_raw(fmt):
    import torch
    rng = np.random.default_rng(100 + int(fmt))
    rows, cols = 96, 2048
    w = make_matrix(fmt, rows, cols, rng)
    M = Q.Matrix(fmt, rows, cols, w)
    try:
        for T in (1, 3, 9):
            x = rng.standard_normal((T, cols), dtype=np.float32)
            ref = np.stack([O.matvec(fmt, w, rows, cols, x[t]) for t in range(T)])
            xd = torch.from_numpy(x).cuda()
            yd = torch.empty((T, rows), device="cuda")
            M.gemv(xd.data_ptr(), T, yd.data_ptr())
            torch.cuda.synchronize()
            err = row_rel_err(yd.cpu().numpy(), ref)
            assert err <= OUT_TOL, f"format {fmt}, T {T}: relative error {err:.3e}"
    finally:
        M.close()


def _raw_case(name, fmts, shared_fmts=None, seed=7, **over):
    """make_case's routing (router, bias, offsets, norm) with expert matrices
    of the given raw formats."""
    base = make_case(name, seed=seed, **over)
    cfg = base.cfg
    d, f, E = cfg["d_model"], cfg["expert_ffn"], cfg["n_experts"]
    rng = np.random.default_rng(seed + 1)
    mats = [[make_matrix(fmts[w], *((d, f) if w == 2 else (f, d)), rng) for _ in range(E)] for w in range(3)]
    shared, fmt_sh = None, (0, 0, 0)
    if base.shared is not None:
        sf = shared_fmts or fmts
        shared = tuple(make_matrix(sf[w], *((d, f) if w == 2 else (f, d)), rng) for w in range(3))
        fmt_sh = tuple(sf)
    return MoeCase(cfg=cfg, norm_w=base.norm_w, router=base.router, router_bias=base.router_bias,
                   logit_offset=base.logit_offset, gate=mats[0], up=mats[1], down=mats[2], fmt_gate=fmts[0],
                   fmt_up=fmts[1], fmt_down=fmts[2], shared=shared, fmt_sh=fmt_sh)


@pytest.mark.parametrize("name,fmts,shared_fmts,over,T", [
    ("c1", (O.Q5_K, O.Q5_K, O.Q3_K), None, dict(d_model=1024, expert_ffn=1024, n_experts=8), 3),
    ("c3", (O.Q2_K, O.Q2_K, O.I8_BLK), (O.B1X, O.B1X, O.B1), dict(d_model=512, expert_ffn=512, n_experts=16), 4),
    ("c5", (O.T1E, O.T1E, O.T1E_LO), (O.I8_BLK, O.I8_BLK, O.Q5_K),
     dict(d_model=768, expert_ffn=512, n_experts=16, n_active=4), 2),
])
def test_moe_layer_raw_formats(name, fmts, shared_fmts, over, T):
    case = _raw_case(name, fmts, shared_fmts, **over)
    x = make_input(case, T, seed=11)
    flags = O.APPLY_NORM | (0 if case.cfg["moe_sigmoid"] else O.ADD_RESIDUAL)
    r = assert_parity(case, x, flags)
    assert r["err"] <= OUT_TOL


def test_raw_bytes_round_trip():
    from tests.gpu_helpers import make_layer
    case = _raw_case("c1", (O.Q2_K, O.Q2_K, O.B1X), None, d_model=512, expert_ffn=512, n_experts=4)
    L = make_layer(case, max_tokens=1)
    try:
        for e in range(4):
            nb = O.tensor_bytes(512 * 512, O.B1X)
            assert np.array_equal(L.download_expert(e, Q.DOWN, nb), case.down[e])
    finally:
        L.close()
