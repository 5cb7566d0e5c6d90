"""The .qw header reader of libqrmoe (qrm_qw_layer_desc) on files written the
way the reference's ModelStoreBuilder writes them (ModelStore.cs:142-225):
layer descriptions from the header config and tensor formats, and the errors
of ModelStore.Open (ModelStore.cs:85-126) for malformed files.  No GPU."""
import json
import struct

import numpy as np
import pytest

import qauntrunner_b200 as Q
from tests import oracle_api as O
from tests.moe_case import make_case
from tests.qw_writer import BF16, F16, F32, case_to_qw, write_qw


def _glm_case():
    return make_case("c3", seed=5, d_model=256, expert_ffn=256, n_experts=8, n_active=4)


def test_desc_from_header(tmp_path):
    case = _glm_case()
    p = tmp_path / "glm.qw"
    case_to_qw(str(p), case, layer=2, n_layers=3, header_reserve=1 << 16)
    d = Q.qw_layer_desc(str(p), 2, device=1, max_tokens=7)
    c = case.cfg
    assert (d.d_model, d.n_experts, d.n_active, d.expert_ffn) == (c["d_model"], c["n_experts"], c["n_active"],
                                                                  c["expert_ffn"])
    assert d.moe_sigmoid == 1 and d.n_shared == 1
    assert np.float32(d.routed_scale) == np.float32(c["routed_scale"])
    assert np.float32(d.rms_eps) == np.float32(c["rms_eps"])
    assert (d.fmt_gate, d.fmt_up, d.fmt_down) == (case.fmt_gate, case.fmt_up, case.fmt_down)
    assert (d.fmt_sh_gate, d.fmt_sh_up, d.fmt_sh_down) == tuple(case.fmt_sh)
    assert (d.device, d.max_tokens) == (1, 7)
    # a layer index with no router is a dense layer: no MoE description
    with pytest.raises(Q.QrmError) as ei:
        Q.qw_layer_desc(str(p), 0)
    assert ei.value.code == Q.E_STATE


def test_shared_expert_needs_its_tensors(tmp_path):
    case = _glm_case()
    case.shared = None                      # config says n_shared 1, file has no sw_* tensors
    p = tmp_path / "noshared.qw"
    case_to_qw(str(p), case)
    d = Q.qw_layer_desc(str(p), 0)
    assert d.n_shared == 0                  # the engine skips the shared expert then (StreamingEngine.cs:779)


def test_expert_ffn_falls_back_to_ffn(tmp_path):
    case = make_case("c1", seed=6, d_model=256, expert_ffn=512, n_experts=4)
    p = tmp_path / "mix.qw"
    case_to_qw(str(p), case, extra_config={"expert_ffn": -1, "ffn": 512})   # ModelConfig.EffectiveExpertFfn
    d = Q.qw_layer_desc(str(p), 0)
    assert d.expert_ffn == 512 and d.moe_sigmoid == 0 and d.fmt_gate == O.Q4_0


def _raw(p, hb, body=b""):
    with open(p, "wb") as fh:
        fh.write(b"QWR1" + struct.pack("<i", len(hb)) + hb)
        fh.write(b"\0" * ((-(8 + len(hb))) % 64) + body)


def test_malformed_files(tmp_path):
    with pytest.raises(Q.QrmError) as ei:
        Q.qw_layer_desc(str(tmp_path / "missing.qw"), 0)
    assert ei.value.code == Q.E_INVALID
    bad = tmp_path / "bad.qw"
    bad.write_bytes(b"GGUF" + b"\0" * 64)
    with pytest.raises(Q.QrmError) as ei:
        Q.qw_layer_desc(str(bad), 0)
    assert ei.value.code == Q.E_INVALID and "not a QuantRunner" in str(ei.value)
    # header length past the end of the file
    trunc = tmp_path / "trunc.qw"
    trunc.write_bytes(b"QWR1" + struct.pack("<i", 4096) + b"{}")
    with pytest.raises(Q.QrmError) as ei:
        Q.qw_layer_desc(str(trunc), 0)
    assert ei.value.code == Q.E_INVALID
    # a tensor that extends past the end of the file
    hb = json.dumps({"config": {"dim": 32}, "tensors": [{"name": "l0.router", "dims": [4, 32], "format": 0,
                                                         "offset": 0, "size": 512}]}).encode()
    short = tmp_path / "short.qw"
    _raw(short, hb, b"\0" * 100)
    with pytest.raises(Q.QrmError) as ei:
        Q.qw_layer_desc(str(short), 0)
    assert ei.value.code == Q.E_INVALID and "outside the file" in str(ei.value)
    # not JSON
    junk = tmp_path / "junk.qw"
    _raw(junk, b"{\"config\": [1, 2,")
    with pytest.raises(Q.QrmError) as ei:
        Q.qw_layer_desc(str(junk), 0)
    assert ei.value.code == Q.E_INVALID and "JSON" in str(ei.value)


def test_json_forms(tmp_path):
    """Escapes, exponent-form numbers and key order as System.Text.Json may
    write them."""
    d, f, E = 64, 64, 4
    cfg = {"n_active": 2, "dim": 6.4E1, "n_experts": E, "expert_ffn": 64, "rms_eps": 1E-05, "moe_sigmoid": False,
           "source": "café \"quoted\" \\ path", "extra": {"nested": [1, {"a": None}, True]}}
    nb = O.tensor_bytes(f * d, O.Q8_0)
    ts = [("l0.router", [E, d], F32, np.zeros(E * d, np.float32).tobytes())]
    for e in range(E):
        for w, nm in enumerate(("w_gate", "w_up", "w_down")):
            ts.append((f"l0.e{e}.{nm}", [f, d], O.Q8_0, np.zeros(nb, np.uint8).tobytes()))
    p = tmp_path / "forms.qw"
    write_qw(str(p), cfg, ts)
    raw = p.read_bytes()
    # re-encode the header with \u escapes and a tensor name spelled with one
    hlen = struct.unpack("<i", raw[4:8])[0]
    head = json.loads(raw[8:8 + hlen])
    hb = json.dumps(head, ensure_ascii=True).replace("l0.router", "l0\\u002erouter").encode()
    body = raw[(8 + hlen + 63) & ~63:]
    q = tmp_path / "forms2.qw"
    _raw(q, hb, body)
    dd = Q.qw_layer_desc(str(q), 0)
    assert (dd.d_model, dd.n_experts, dd.n_active, dd.expert_ffn, dd.fmt_gate) == (64, E, 2, 64, O.Q8_0)
    assert np.float32(dd.rms_eps) == np.float32(1e-5)
