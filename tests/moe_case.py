"""Seeded synthetic MoE layers for the parity tests.

The weights follow the reference's synthetic-model recipe (src/QuantRunner.Cli/
Program.cs:357-362, Synth.cs:191-193): N(0, 0.02) floats quantised with the
reference quantiser (here: the oracle's restatement of BlockQuantizer).  Unlike
the reference's own synthetic models, whose router is all ones (every expert
ties), routers are drawn at random so that routing is decided by the data.
"""
from dataclasses import dataclass, field
from typing import List, Optional

import numpy as np

from tests import oracle_api as O

# Configs of BASELINE.json; full-size shapes and the smaller parity shapes.
CONFIGS = {
    "c1": dict(d_model=1024, expert_ffn=2816, n_experts=8, n_active=2, moe_sigmoid=0, n_shared=0,
               routed_scale=1.0, swiglu_limit=0.0, rms_eps=1e-5, fmt=(O.Q4_0, O.Q4_0, O.Q4_0)),
    "c2": dict(d_model=4096, expert_ffn=14336, n_experts=8, n_active=2, moe_sigmoid=0, n_shared=0,
               routed_scale=1.0, swiglu_limit=0.0, rms_eps=1e-5, fmt=(O.Q4_K, O.Q4_K, O.Q4_K)),
    "c3": dict(d_model=6144, expert_ffn=1536, n_experts=160, n_active=8, moe_sigmoid=1, n_shared=1,
               routed_scale=2.5, swiglu_limit=0.0, rms_eps=1e-5, fmt=(O.Q4_K, O.Q4_K, O.Q6_K),
               bias_sigma=0.01),
    "c4": dict(d_model=4096, expert_ffn=11008, n_experts=64, n_active=6, moe_sigmoid=0, n_shared=0,
               routed_scale=1.0, swiglu_limit=0.0, rms_eps=1e-5, fmt=(O.TRI_LEGACY,) * 3),
    "c5": dict(d_model=7168, expert_ffn=2048, n_experts=256, n_active=8, moe_sigmoid=1, n_shared=1,
               routed_scale=2.5, swiglu_limit=0.0, rms_eps=1e-5, fmt=(O.Q4_K, O.Q4_K, O.Q4_K),
               shared_fmt=(O.Q8_0, O.Q8_0, O.Q8_0), bias_sigma=0.01, offset_sigma=1.5),
}


def storage_fmt(f):
    return O.TRI if f == O.TRI_LEGACY else f


@dataclass
class MoeCase:
    cfg: dict
    norm_w: Optional[np.ndarray]
    router: np.ndarray
    router_bias: Optional[np.ndarray]
    logit_offset: Optional[np.ndarray]
    gate: List[np.ndarray]
    up: List[np.ndarray]
    down: List[np.ndarray]
    fmt_gate: int
    fmt_up: int
    fmt_down: int
    shared: Optional[tuple] = None
    fmt_sh: tuple = (0, 0, 0)
    float_weights: dict = field(default_factory=dict)


def make_case(name="c1", seed=1, d_model=None, expert_ffn=None, n_experts=None, n_active=None,
              router_sigma=0.02, weight_sigma=0.02, norm_random=False, **over):
    cfg = dict(CONFIGS[name])
    for k, v in dict(d_model=d_model, expert_ffn=expert_ffn, n_experts=n_experts,
                     n_active=n_active).items():
        if v is not None:
            cfg[k] = v
    cfg.update(over)
    rng = np.random.default_rng(seed)
    d, f, E = cfg["d_model"], cfg["expert_ffn"], cfg["n_experts"]
    fq = cfg["fmt"]

    def qmat(rows, cols, fmt):
        w = (rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(weight_sigma)).astype(np.float32)
        return O.quantize(fmt, w)

    gate = [qmat(f, d, fq[0]) for _ in range(E)]
    up = [qmat(f, d, fq[1]) for _ in range(E)]
    down = [qmat(d, f, fq[2]) for _ in range(E)]
    router = (rng.standard_normal((E, d), dtype=np.float32) * np.float32(router_sigma)).astype(np.float32)
    norm_w = (1.0 + 0.1 * rng.standard_normal(d)).astype(np.float32) if norm_random else np.ones(d, np.float32)
    bias = None
    if cfg.get("bias_sigma"):
        bias = (rng.standard_normal(E) * cfg["bias_sigma"]).astype(np.float32)
    offset = None
    if cfg.get("offset_sigma"):
        offset = (rng.standard_normal(E) * cfg["offset_sigma"]).astype(np.float32)
    shared = None
    fmt_sh = (0, 0, 0)
    if cfg["n_shared"] > 0:
        sf = cfg.get("shared_fmt", fq)
        shared = (qmat(f, d, sf[0]), qmat(f, d, sf[1]), qmat(d, f, sf[2]))
        fmt_sh = tuple(storage_fmt(x) for x in sf)
    return MoeCase(cfg=cfg, norm_w=norm_w, router=router, router_bias=bias, logit_offset=offset,
                   gate=gate, up=up, down=down, fmt_gate=storage_fmt(fq[0]), fmt_up=storage_fmt(fq[1]),
                   fmt_down=storage_fmt(fq[2]), shared=shared, fmt_sh=fmt_sh)


def make_input(case, T, seed=2):
    rng = np.random.default_rng(seed)
    return rng.standard_normal((T, case.cfg["d_model"]), dtype=np.float32)
