"""GPU parity: the CUDA path (through the C ABI) against the CPU oracle on
the same seeded inputs.  Routing (xn, logits, top-k indices and weights, the
dispatch permutation) must be bit-exact; layer outputs within max relative
error 1e-3 (tests/gpu_helpers.OUT_TOL)."""
import numpy as np
import pytest

import qauntrunner_b200 as Q
from tests import oracle_api as O
from tests.gpu_helpers import OUT_TOL, assert_parity, make_layer, row_rel_err
from tests.moe_case import make_case, make_input

pytestmark = pytest.mark.gpu

NORM = O.APPLY_NORM
RESID = O.ADD_RESIDUAL


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    assert torch.cuda.is_available()
    return torch


# ----------------------------------------------------------- operator (MatVec)

@pytest.mark.parametrize("fmt", [O.Q4_0, O.Q8_0, O.Q4_K, O.Q6_K, O.TRI])
@pytest.mark.parametrize("T", [1, 3, 9])
def test_matrix_gemv_matches_oracle(torch_cuda, fmt, T):
    torch = torch_cuda
    rng = np.random.default_rng(11 + fmt)
    bs, _ = O.BLOCK_SPEC[fmt]
    cols = 1024 if bs < 256 else 1536
    rows = 200
    w = (rng.standard_normal(rows * cols) * 0.4).astype(np.float32)
    wq = O.quantize(fmt, w)
    x = (rng.standard_normal((T, cols)) * 0.5).astype(np.float32)
    ref = np.stack([O.matvec(fmt, wq, rows, cols, x[t]) for t in range(T)])
    m = Q.Matrix(fmt, rows, cols, wq)
    xd = torch.from_numpy(x).cuda()
    yd = torch.zeros((T, rows), dtype=torch.float32, device="cuda")
    m.gemv(xd.data_ptr(), T, yd.data_ptr())
    torch.cuda.synchronize()
    got = yd.cpu().numpy()
    m.close()
    # DotMatches bound of the reference (2e-4), scaled by the row magnitude
    assert row_rel_err(got, ref) <= 2e-4


# ------------------------------------------------------------------ layouts

@pytest.mark.parametrize("fmt", [O.Q4_0, O.Q8_0, O.Q4_K, O.Q6_K, O.TRI])
def test_upload_download_is_byte_exact(fmt):
    bs, _ = O.BLOCK_SPEC[fmt]
    d = 512 if bs < 256 else 1024
    f = 256 if bs < 256 else 512
    case = make_case("c1", seed=3, d_model=d, expert_ffn=f, n_experts=2, n_active=1, fmt=(fmt, fmt, fmt))
    rng = np.random.default_rng(4)
    L = make_layer(case, max_tokens=1)
    try:
        for e in range(2):
            for which, src in ((Q.GATE, case.gate[e]), (Q.UP, case.up[e]), (Q.DOWN, case.down[e])):
                got = L.download_expert(e, which, src.nbytes)
                assert np.array_equal(got, src)
        # arbitrary bytes (including the Q4_0 pad bytes) survive too
        raw = rng.integers(0, 256, case.gate[0].nbytes, dtype=np.uint8)
        L.upload_expert(0, Q.GATE, fmt, raw)
        assert np.array_equal(L.download_expert(0, Q.GATE, raw.nbytes), raw)
    finally:
        L.close()


# ------------------------------------------------------------ MoE layer parity

SMALL = {
    # name: (config, overrides)
    "c1_full": ("c1", {}),
    "c2_small": ("c2", dict(d_model=1024, expert_ffn=2048)),
    "c3_small": ("c3", dict(d_model=1536, expert_ffn=512, n_experts=32)),
    "c3_small_limit10": ("c3", dict(d_model=1536, expert_ffn=512, n_experts=32, swiglu_limit=10.0)),
    "c4_small": ("c4", dict(d_model=1024, expert_ffn=1024, n_experts=16)),
    "c5_small": ("c5", dict(d_model=1024, expert_ffn=512, n_experts=64)),
}


@pytest.mark.parametrize("name", list(SMALL))
@pytest.mark.parametrize("T", [1, 5, 33])
def test_layer_parity(name, T):
    cfg, over = SMALL[name]
    case = make_case(cfg, seed=7, **over)
    x = make_input(case, T, seed=8 + T)
    flags = NORM | (RESID if not case.cfg["moe_sigmoid"] else 0)
    r = assert_parity(case, x, flags)
    assert r["err"] <= OUT_TOL


@pytest.mark.parametrize("flags", [0, NORM, RESID, NORM | RESID])
def test_layer_flags(flags):
    case = make_case("c1", seed=21, d_model=512, expert_ffn=512, n_experts=8, norm_random=True)
    x = make_input(case, 4, seed=22)
    assert_parity(case, x, flags)


def test_legacy_into_and_glm_without_bias():
    case = make_case("c3", seed=31, d_model=512, expert_ffn=256, n_experts=16, bias_sigma=0)
    assert case.router_bias is None
    x = make_input(case, 6, seed=32)
    assert_parity(case, x, NORM)
    case2 = make_case("c1", seed=33, d_model=512, expert_ffn=512, n_experts=8)
    assert_parity(case2, make_input(case2, 3, seed=34), NORM)   # LegacyMoeInto semantics


def test_reference_synthetic_router_all_ones():
    # The reference's synthetic models set the router to ones (Program.cs:358-360):
    # every logit ties, so the order is the sort's; for 8 experts Array.Sort is an
    # insertion sort (stable), so experts 0..k-1 are selected in index order.
    case = make_case("c1", seed=41, d_model=512, expert_ffn=512, n_experts=8)
    case.router[:] = 1.0
    x = make_input(case, 3, seed=42)
    r = assert_parity(case, x, NORM | RESID)
    L = make_layer(case, 3)
    _, idx, w = L.forward(x, apply_norm=True, add_residual=True)
    L.close()
    assert (idx == np.array([0, 1])).all()
    assert (w == np.float32(0.5)).all()


def test_large_batch_routing_and_skew():
    # 256 tokens: tiled router path, uneven expert loads from the logit offsets
    case = make_case("c5", seed=51, d_model=1024, expert_ffn=256, n_experts=64)
    x = make_input(case, 256, seed=52)
    assert_parity(case, x, NORM)


@pytest.mark.parametrize("T", [2, 31, 32])
def test_fused_topk_dispatch_bounds(T):
    # batches at the edges of the single-CTA top-k + dispatch (T <= 32)
    case = make_case("c5", seed=71, d_model=1024, expert_ffn=256, n_experts=64)
    assert_parity(case, make_input(case, T, seed=72 + T), NORM)


def test_forward_is_deterministic():
    case = make_case("c3", seed=61, d_model=1024, expert_ffn=512, n_experts=32)
    x = make_input(case, 17, seed=62)
    L = make_layer(case, 17)
    try:
        a = L.forward(x)[0]
        b = L.forward(x)[0]
    finally:
        L.close()
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


# ---------------------------------------------------------------- errors

def test_error_codes():
    case = make_case("c1", seed=71, d_model=512, expert_ffn=512, n_experts=4)
    L = Q.MoeLayer(512, 4, 2, 512, fmt=(O.Q4_0,) * 3, max_tokens=2)
    try:
        x = make_input(case, 1, seed=1)
        with pytest.raises(Q.QrmError) as ei:
            L.forward(x)
        assert ei.value.code == -4          # router never uploaded
        L.upload_router(case.router)
        L.upload_norm(case.norm_w)
        with pytest.raises(Q.QrmError) as ei:
            L.forward(x)
        assert ei.value.code == -4 and "e0" in str(ei.value)   # experts missing
        with pytest.raises(Q.QrmError) as ei:
            L.upload_expert(0, Q.GATE, O.Q4_0, case.gate[0][:-1])
        assert ei.value.code == -3
        with pytest.raises(Q.QrmError) as ei:
            L.upload_expert(0, Q.GATE, O.Q8_0, case.gate[0])
        assert ei.value.code == -2
        with pytest.raises(Q.QrmError) as ei:
            L.upload_expert(4, Q.GATE, O.Q4_0, case.gate[0])
        assert ei.value.code == -1
        with pytest.raises(Q.QrmError) as ei:
            L.upload_expert(Q.SHARED_EXPERT, Q.GATE, O.Q4_0, case.gate[0])
        assert ei.value.code == -1          # no shared expert on a softmax layer
        for e in range(4):
            L.upload_expert(e, Q.GATE, O.Q4_0, case.gate[e])
            L.upload_expert(e, Q.UP, O.Q4_0, case.up[e])
            L.upload_expert(e, Q.DOWN, O.Q4_0, case.down[e])
        L.forward(x)
        with pytest.raises(Q.QrmError) as ei:
            L.forward(make_input(case, 3, seed=2))
        assert ei.value.code == -9          # more tokens than max_tokens
    finally:
        L.close()
