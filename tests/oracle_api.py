"""ctypes binding of the CPU oracle (oracle/liboracle.so) for the tests.

The oracle is test infrastructure: it restates the reference's CPU algorithm
and is only ever used as the checker (see oracle/oracle.h).
"""
import ctypes as C
import os
import subprocess

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORACLE_DIR = os.path.join(ROOT, "oracle")
ORACLE_SO = os.path.join(ORACLE_DIR, "liboracle.so")

F32, F16, BF16, Q4_0, Q8_0, Q4_K, Q6_K, TRI = 0, 1, 2, 3, 4, 6, 7, 8
Q2_K, I8_BLK, Q3_K, Q5_K, B1, B1X, T1E, T1E_LO = 5, 9, 10, 11, 12, 13, 14, 15
RAW_FORMATS = (Q2_K, Q3_K, Q5_K, I8_BLK, B1, B1X, T1E, T1E_LO)
TRI_LEGACY = 108
BLOCK_SPEC = {F32: (1, 4), F16: (1, 2), BF16: (1, 2), Q4_0: (32, 20), Q8_0: (32, 34),
              Q4_K: (256, 144), Q6_K: (256, 210), TRI: (64, 18), Q2_K: (256, 84), Q3_K: (256, 110),
              Q5_K: (256, 176), I8_BLK: (256, 258), B1: (256, 34), B1X: (256, 47), T1E: (256, 40),
              T1E_LO: (256, 32)}
APPLY_NORM, ADD_RESIDUAL = 1, 2

_lib = None


def build():
    """Build liboracle.so when missing or older than its sources."""
    srcs = [os.path.join(ORACLE_DIR, n) for n in ("oracle.cpp", "oracle.h", "Makefile")]
    if os.path.exists(ORACLE_SO) and all(os.path.getmtime(ORACLE_SO) >= os.path.getmtime(s) for s in srcs):
        return ORACLE_SO
    subprocess.run(["make", "-s", "-C", ORACLE_DIR], check=True)
    return ORACLE_SO


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = C.CDLL(ORACLE_SO)
        _setup(_lib)
    return _lib


P = C.c_void_p


def _setup(L):
    L.orc_f16_to_f32.restype = C.c_float
    L.orc_f16_to_f32.argtypes = [C.c_uint16]
    L.orc_f32_to_f16.restype = C.c_uint16
    L.orc_f32_to_f16.argtypes = [C.c_float]
    L.orc_f32_to_f16_batch.argtypes = [P, P, C.c_int64]
    L.orc_quantize.argtypes = [C.c_int, P, C.c_int64, P]
    L.orc_dequantize.argtypes = [C.c_int, P, C.c_int64, P]
    L.orc_dot_row.restype = C.c_float
    L.orc_dot_row.argtypes = [C.c_int, P, P, C.c_int]
    L.orc_matvec.argtypes = [C.c_int, P, C.c_int64, C.c_int64, P, P]
    L.orc_matvec_parallel.argtypes = [C.c_int, P, C.c_int64, C.c_int64, P, P, C.c_int]
    L.orc_rmsnorm.argtypes = [P, P, P, C.c_int, C.c_float]
    L.orc_dot_f32.restype = C.c_float
    L.orc_dot_f32.argtypes = [P, P, C.c_int]
    L.orc_expf_batch.argtypes = [P, P, C.c_int64]
    L.orc_route_softmax.argtypes = [P, C.c_int, C.c_int, P, P, P]
    L.orc_route_sigmoid.argtypes = [P, P, C.c_int, C.c_int, C.c_float, P, P]
    L.orc_dispatch.argtypes = [P, C.c_int, C.c_int, C.c_int, P, P, P]
    L.orc_swiglu.argtypes = [P, P, C.c_int, C.c_float]
    L.orc_moe_forward.argtypes = [P, P, P, C.c_int, C.c_int, P, P, P, P, P, C.c_int]
    L.orc_moe_route.argtypes = [P, P, P, C.c_int, C.c_int, P, P, P, P, C.c_int]


def ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def tensor_bytes(n, fmt):
    bs, bb = BLOCK_SPEC[TRI if fmt == TRI_LEGACY else fmt]
    assert n % bs == 0
    return n // bs * bb


def quantize(fmt, x):
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    out = np.zeros(tensor_bytes(x.size, fmt), dtype=np.uint8)
    assert lib().orc_quantize(fmt, ptr(x), x.size, ptr(out)) == 0
    return out


def dequantize(fmt, b, n):
    b = np.ascontiguousarray(b, dtype=np.uint8)
    out = np.zeros(n, dtype=np.float32)
    assert lib().orc_dequantize(fmt, ptr(b), n, ptr(out)) == 0
    return out


def matvec(fmt, w, rows, cols, x, threads=1):
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.uint8)
    y = np.zeros(rows, dtype=np.float32)
    assert lib().orc_matvec_parallel(fmt, ptr(w), rows, cols, ptr(x), ptr(y), threads) == 0
    return y


def swiglu(g, u, limit):
    """TransformerOps.SiluMulInPlace / Glm5Ops.LimitedSwiglu (limit > 0) of g and u."""
    g = np.array(g, dtype=np.float32, copy=True)
    u = np.ascontiguousarray(u, dtype=np.float32)
    lib().orc_swiglu(ptr(g), ptr(u), g.size, limit)
    return g


def expf(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib().orc_expf_batch(ptr(x), ptr(y), x.size)
    return y


def rmsnorm(x, w, eps):
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    lib().orc_rmsnorm(ptr(x), ptr(w), ptr(out), x.size, eps)
    return out


def dispatch(sel, T, k, E):
    sel = np.ascontiguousarray(sel, dtype=np.int32).ravel()
    perm = np.zeros(T * k, dtype=np.int32)
    inv = np.zeros(T * k, dtype=np.int32)
    off = np.zeros(E + 1, dtype=np.int32)
    lib().orc_dispatch(ptr(sel), T, k, E, ptr(perm), ptr(inv), ptr(off))
    return perm, inv, off


class MoeDesc(C.Structure):
    _fields_ = [("d_model", C.c_int32), ("n_experts", C.c_int32), ("n_active", C.c_int32),
                ("expert_ffn", C.c_int32), ("moe_sigmoid", C.c_int32), ("routed_scale", C.c_float),
                ("n_shared", C.c_int32), ("swiglu_limit", C.c_float), ("rms_eps", C.c_float)]


class MoeWeights(C.Structure):
    _fields_ = [("norm_w", P), ("router", P), ("router_bias", P), ("logit_offset", P),
                ("gate", C.POINTER(P)), ("up", C.POINTER(P)), ("down", C.POINTER(P)),
                ("fmt_gate", C.c_int32), ("fmt_up", C.c_int32), ("fmt_down", C.c_int32),
                ("sh_gate", P), ("sh_up", P), ("sh_down", P),
                ("fmt_sh_gate", C.c_int32), ("fmt_sh_up", C.c_int32), ("fmt_sh_down", C.c_int32)]


def _moe_structs(layer):
    cfg = layer.cfg
    d, E = cfg["d_model"], cfg["n_experts"]
    desc = MoeDesc(d, E, cfg["n_active"], cfg["expert_ffn"], int(cfg["moe_sigmoid"]),
                   cfg["routed_scale"], cfg["n_shared"], cfg["swiglu_limit"], cfg["rms_eps"])
    arr = P * E
    gate = arr(*[ptr(b) for b in layer.gate])
    up = arr(*[ptr(b) for b in layer.up])
    down = arr(*[ptr(b) for b in layer.down])
    sh = layer.shared
    w = MoeWeights(ptr(layer.norm_w), ptr(layer.router), ptr(layer.router_bias), ptr(layer.logit_offset),
                   C.cast(gate, C.POINTER(P)), C.cast(up, C.POINTER(P)), C.cast(down, C.POINTER(P)),
                   layer.fmt_gate, layer.fmt_up, layer.fmt_down,
                   ptr(sh[0]) if sh else None, ptr(sh[1]) if sh else None, ptr(sh[2]) if sh else None,
                   layer.fmt_sh[0], layer.fmt_sh[1], layer.fmt_sh[2])
    return desc, w, (gate, up, down)


def moe_forward(layer, x, flags, threads=1):
    """Runs the oracle MoE layer.  `layer` is a tests.moe_case.MoeCase."""
    cfg = layer.cfg
    T = x.shape[0]
    d, E, k = cfg["d_model"], cfg["n_experts"], min(cfg["n_active"], 8)
    desc, w, keep = _moe_structs(layer)
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros((T, d), dtype=np.float32)
    idx = np.zeros((T, k), dtype=np.int32)
    wts = np.zeros((T, k), dtype=np.float32)
    logits = np.zeros((T, E), dtype=np.float32)
    xn = np.zeros((T, d), dtype=np.float32)
    rc = lib().orc_moe_forward(C.byref(desc), C.byref(w), ptr(x), T, flags, ptr(out), ptr(idx),
                               ptr(wts), ptr(logits), ptr(xn), threads)
    assert rc == 0
    return dict(out=out, topk_idx=idx, topk_w=wts, logits=logits, xn=xn)


def moe_route(layer, x, flags, threads=1):
    """The oracle's routing alone (xn, logits, top-k) for every token of x."""
    cfg = layer.cfg
    T = x.shape[0]
    d, E, k = cfg["d_model"], cfg["n_experts"], min(cfg["n_active"], 8)
    desc, w, keep = _moe_structs(layer)
    x = np.ascontiguousarray(x, dtype=np.float32)
    idx = np.zeros((T, k), dtype=np.int32)
    wts = np.zeros((T, k), dtype=np.float32)
    logits = np.zeros((T, E), dtype=np.float32)
    xn = np.zeros((T, d), dtype=np.float32)
    assert lib().orc_moe_route(C.byref(desc), C.byref(w), ptr(x), T, flags, ptr(idx), ptr(wts),
                               ptr(logits), ptr(xn), threads) == 0
    return dict(topk_idx=idx, topk_w=wts, logits=logits, xn=xn)


def _split(fn, layer, x, flags, workers):
    """fn over token chunks on `workers` threads (every token is independent:
    the results equal one call over all tokens)."""
    from concurrent.futures import ThreadPoolExecutor
    T = x.shape[0]
    workers = max(1, min(workers, T))
    if workers == 1:
        return fn(layer, x, flags, 1)
    bounds = np.linspace(0, T, workers + 1).astype(int)
    with ThreadPoolExecutor(workers) as ex:
        parts = list(ex.map(lambda i: fn(layer, x[bounds[i]:bounds[i + 1]], flags, 1), range(workers)))
    return {key: np.concatenate([p[key] for p in parts]) for key in parts[0]}


def moe_forward_par(layer, x, flags, workers=None):
    """moe_forward with the tokens spread over host threads."""
    return _split(moe_forward, layer, x, flags, workers or (os.cpu_count() or 1))


def moe_route_par(layer, x, flags, workers=None):
    return _split(moe_route, layer, x, flags, workers or (os.cpu_count() or 1))
