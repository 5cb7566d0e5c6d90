"""GPU parity of the tcgen05 grouped expert path (csrc/umma.cuh) against the
oracle.  The library takes that path for large per-expert groups; these tests
force it for every batch (QRM_UMMA=1, read when a layer is created) so that
small shapes, one-token groups, multi-block groups (more than 256 tokens of
one expert) and the shared expert in another format all run through it.
Routing stays bit-exact; outputs within OUT_TOL (f16 operands, f32 sums)."""
import numpy as np
import pytest

from tests import oracle_api as O
from tests.gpu_helpers import OUT_TOL, assert_parity, check_synth_batch
from tests.moe_case import make_case, make_input
from tests.synth_layer import SynthLayer

pytestmark = pytest.mark.gpu

NORM, RESID = O.APPLY_NORM, O.ADD_RESIDUAL

CASES = {
    "c1_full_q4_0": ("c1", {}),
    "c2_small_q4k": ("c2", dict(d_model=1024, expert_ffn=1024)),
    "c5_small_q4k_shared_q8_0": ("c5", dict(d_model=1024, expert_ffn=512, n_experts=64)),
    "c5_small_q8_0": ("c5", dict(d_model=1024, expert_ffn=512, n_experts=32, fmt=(O.Q8_0,) * 3)),
    "c5_small_limit": ("c5", dict(d_model=1024, expert_ffn=512, n_experts=32, swiglu_limit=7.0)),
    "c4_small_tri": ("c4", dict(d_model=1024, expert_ffn=1024, n_experts=16)),
    "c3_small_q6k_down": ("c3", dict(d_model=1536, expert_ffn=512, n_experts=32)),
}


@pytest.fixture
def umma_on(monkeypatch):
    monkeypatch.setenv("QRM_UMMA", "1")
    yield


@pytest.mark.parametrize("name", list(CASES))
@pytest.mark.parametrize("T", [1, 7, 64, 300])
def test_grouped_path_parity(umma_on, name, T):
    cfg, over = CASES[name]
    case = make_case(cfg, seed=9, **over)
    x = make_input(case, T, seed=10 + T)
    flags = NORM | (RESID if not case.cfg["moe_sigmoid"] else 0)
    r = assert_parity(case, x, flags)
    assert r["err"] <= OUT_TOL


def test_grouped_path_matches_decode_path(monkeypatch):
    """The same layer and tokens through both expert paths agree within the
    output tolerance (each is also checked against the oracle above)."""
    from tests.gpu_helpers import make_layer, row_rel_err
    case = make_case("c5", seed=13, d_model=1024, expert_ffn=512, n_experts=64)
    x = make_input(case, 96, seed=14)
    monkeypatch.setenv("QRM_UMMA", "0")
    L0 = make_layer(case, 96)
    monkeypatch.setenv("QRM_UMMA", "1")
    L1 = make_layer(case, 96)
    try:
        a = L0.forward(x)[0]
        b = L1.forward(x)[0]
        b2 = L1.forward(x)[0]
    finally:
        L0.close()
        L1.close()
    assert row_rel_err(b, a) <= OUT_TOL
    assert np.array_equal(b.view(np.uint32), b2.view(np.uint32))   # deterministic run to run


@pytest.mark.parametrize("T", [1024, 4096])
def test_grouped_path_c5_full_shape(umma_on, T):
    import torch
    import qauntrunner_b200 as Q
    spec = SynthLayer("c5", pool=8)
    L = spec.build(torch, Q, 0, T)
    try:
        x = np.random.default_rng(500 + T).standard_normal((T, 7168), dtype=np.float32)
        r = check_synth_batch(spec, L, x, NORM)
        assert r["err"] <= OUT_TOL, r
        if T == 4096:
            assert r["max_group"] > 256   # the skewed batch has groups of several token blocks
    finally:
        L.close()
