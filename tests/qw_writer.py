"""Writes QuantRunner .qw weight files for the loader tests, laid out as the
reference's ModelStoreBuilder writes them (src/QuantRunner.Core/Memory/
ModelStore.cs:142-225): "QWR1", int32 header length, the JSON header
{"config": ..., "tensors": [{"name", "dims", "format", "offset", "size"}]}
(plus "data_offset" when a header region is reserved), zero padding to a
64-byte data start, then the tensor bodies in plan order."""
import json
import struct

import numpy as np

F32, F16, BF16 = 0, 1, 2


def write_qw(path, config, tensors, header_reserve=0):
    """tensors: list of (name, dims, format id, bytes-like body)."""
    entries, off = [], 0
    for name, dims, fmt, body in tensors:
        n = len(memoryview(body).cast("B"))
        entries.append({"name": name, "dims": [int(x) for x in dims], "format": int(fmt), "offset": off, "size": n})
        off += n
    head = {"config": config, "tensors": entries}
    hb = json.dumps(head).encode()
    if header_reserve > 0:
        data_start = (8 + header_reserve + 63) & ~63
        head["data_offset"] = data_start
        hb = json.dumps(head).encode()
        assert 8 + len(hb) <= data_start, "reserved header region too small"
    else:
        data_start = (8 + len(hb) + 63) & ~63
    with open(path, "wb") as fh:
        fh.write(b"QWR1")
        fh.write(struct.pack("<i", len(hb)))
        fh.write(hb)
        fh.write(b"\0" * (data_start - 8 - len(hb)))
        for _, _, _, body in tensors:
            fh.write(bytes(memoryview(body).cast("B")))


def as_float_tensor(a, fmt):
    """(bytes, values the reference reads back) of an f32 array stored as
    F32, F16 or BF16 (BF16 by truncation of the f32 bits)."""
    a = np.ascontiguousarray(a, np.float32)
    if fmt == F32:
        return a.tobytes(), a
    if fmt == F16:
        h = a.astype(np.float16)
        return h.tobytes(), h.astype(np.float32)
    b = (a.view(np.uint32) >> 16).astype(np.uint16)
    return b.tobytes(), (b.astype(np.uint32) << 16).view(np.float32)


def case_to_qw(path, case, layer=0, router_fmt=F32, n_layers=None, header_reserve=0, extra_config=None):
    """The MoE layer of a tests.moe_case.MoeCase as layer `layer` of a .qw
    file (canonical names, NameMapper.cs:7-12).  Returns the router and bias
    values the file holds (after any narrowing), for the oracle."""
    cfg = case.cfg
    d, f, E = cfg["d_model"], cfg["expert_ffn"], cfg["n_experts"]
    config = {"arch": "moe", "dim": d, "layers": n_layers or layer + 1, "heads": 8, "ffn": f, "vocab": 32,
              "rms_eps": cfg["rms_eps"], "n_experts": E, "n_active": cfg["n_active"], "expert_ffn": f,
              "moe_sigmoid": bool(cfg["moe_sigmoid"]), "routed_scale": cfg["routed_scale"],
              "n_shared": cfg["n_shared"], "swiglu_limit": cfg["swiglu_limit"]}
    config.update(extra_config or {})
    L = f"l{layer}."
    rb, rv = as_float_tensor(case.router, router_fmt)
    ts = [(L + "router", [E, d], router_fmt, rb)]
    if case.norm_w is not None:
        ts.insert(0, (L + "ffn_norm", [d], F32, np.ascontiguousarray(case.norm_w, np.float32).tobytes()))
    bv = None
    if case.router_bias is not None:
        bb, bv = as_float_tensor(case.router_bias, router_fmt)
        ts.append((L + "router_bias", [E], router_fmt, bb))
    for e in range(E):
        ts.append((L + f"e{e}.w_gate", [f, d], case.fmt_gate, case.gate[e]))
        ts.append((L + f"e{e}.w_up", [f, d], case.fmt_up, case.up[e]))
        ts.append((L + f"e{e}.w_down", [d, f], case.fmt_down, case.down[e]))
    if case.shared:
        for w, nm in enumerate(("sw_gate", "sw_up", "sw_down")):
            ts.append((L + nm, [d, f] if w == 2 else [f, d], case.fmt_sh[w], case.shared[w]))
    write_qw(path, config, ts, header_reserve=header_reserve)
    return rv.reshape(E, d), bv
