"""MoE layers loaded from .qw files (qrm_qw_layer_desc + qrm_load_qw, the
counterpart of ModelStore.Open and the engine's Store.Get by canonical name,
ModelStore.cs:85-126, StreamingEngine.cs:186-201,633-790) match the oracle on
the tensors the file holds: routing bit-exact (routers stored as F32, F16 and
BF16 are widened exactly, which is what the reference's DotF16 / DotBf16 do
lane by lane, DotKernels.cs:57-120), outputs within 1e-3, and the expert
bytes read back unchanged."""
import numpy as np
import pytest

import qauntrunner_b200 as Q
from tests import oracle_api as O
from tests.gpu_helpers import assert_parity
from tests.moe_case import make_case, make_input
from tests.qw_writer import BF16, F16, F32, case_to_qw

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cfgname,over,router_fmt,layer", [
    ("c3", dict(d_model=512, expert_ffn=256, n_experts=16, n_active=8), F16, 3),
    ("c5", dict(d_model=1024, expert_ffn=512, n_experts=32, n_active=8), BF16, 0),
    ("c1", dict(n_experts=8), F32, 1),
])
def test_layer_from_qw(tmp_path, cfgname, over, router_fmt, layer):
    case = make_case(cfgname, seed=41, **over)
    path = str(tmp_path / f"{cfgname}.qw")
    router, bias = case_to_qw(path, case, layer=layer, router_fmt=router_fmt, n_layers=layer + 1,
                              header_reserve=(1 << 16) if layer else 0)
    case.router = router                  # the values the file holds
    if bias is not None:
        case.router_bias = bias
    T = 5
    x = make_input(case, T, seed=43)
    L = Q.MoeLayer.from_qw(path, layer, device=0, max_tokens=T)
    try:
        if case.logit_offset is not None:
            L.upload_logit_offset(case.logit_offset)     # harness-only skew, not part of the file
        flags = O.APPLY_NORM | (0 if case.cfg["moe_sigmoid"] else O.ADD_RESIDUAL)
        r = assert_parity(case, x, flags, L=L)
        assert r["err"] <= 1e-3
        nb = O.tensor_bytes(case.cfg["expert_ffn"] * case.cfg["d_model"], case.fmt_gate)
        got = L.download_expert(3, Q.UP, nb)
        assert np.array_equal(got, np.frombuffer(case.up[3], np.uint8)), "expert bytes changed on the way in"
    finally:
        L.close()


def test_missing_expert_tensor(tmp_path):
    case = make_case("c1", seed=42, n_experts=4, d_model=256, expert_ffn=256)
    path = str(tmp_path / "gap.qw")
    case_to_qw(path, case)
    raw = bytearray(open(path, "rb").read())
    i = raw.find(b'"l0.e2.w_down"')
    raw[i:i + 14] = b'"l0.e2.w_dowX"'         # same length: offsets stay valid
    open(path, "wb").write(bytes(raw))
    with pytest.raises(Q.QrmError) as ei:
        Q.MoeLayer.from_qw(path, 0, device=0, max_tokens=1)
    assert ei.value.code == Q.E_STATE and "l0.e2.w_down" in str(ei.value)
