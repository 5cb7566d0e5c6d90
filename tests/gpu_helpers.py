"""Helpers of the GPU parity tests: load a tests.moe_case.MoeCase into a
qauntrunner_b200.MoeLayer (through the C ABI) and compare with the oracle."""
import numpy as np

import qauntrunner_b200 as Q
from tests import oracle_api as O

# Layer outputs must agree with the reference within max relative error 1e-3
# (f32 accumulation).  "Relative" is taken per token against the largest
# magnitude of the reference output row, so that outputs near zero are judged
# on the scale of their row rather than on their own.
OUT_TOL = 1e-3


def make_layer(case, max_tokens, device=0, rank=0, world=1, nccl_id=None):
    """The case's layer on `device`; an expert-parallel one (world > 1) gets
    only its own block of routed experts."""
    cfg = case.cfg
    shared_fmt = case.fmt_sh if case.shared else None
    fmt = (case.fmt_gate, case.fmt_up, case.fmt_down)
    L = Q.MoeLayer(cfg["d_model"], cfg["n_experts"], cfg["n_active"], cfg["expert_ffn"],
                   moe_sigmoid=bool(cfg["moe_sigmoid"]), routed_scale=cfg["routed_scale"],
                   n_shared=cfg["n_shared"], swiglu_limit=cfg["swiglu_limit"], rms_eps=cfg["rms_eps"],
                   fmt=fmt, shared_fmt=shared_fmt or fmt, max_tokens=max_tokens, device=device,
                   rank=rank, world=world, nccl_id=nccl_id)
    L.upload_norm(case.norm_w)
    L.upload_router(case.router, case.router_bias)
    if case.logit_offset is not None:
        L.upload_logit_offset(case.logit_offset)
    first, count = L.expert_range()
    for e in range(first, first + count):
        L.upload_expert(e, Q.GATE, case.fmt_gate, case.gate[e])
        L.upload_expert(e, Q.UP, case.fmt_up, case.up[e])
        L.upload_expert(e, Q.DOWN, case.fmt_down, case.down[e])
    if case.shared:
        for w in range(3):
            L.upload_expert(Q.SHARED_EXPERT, w, case.fmt_sh[w], case.shared[w])
    return L


def row_rel_err(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    scale = np.maximum(np.abs(ref).max(axis=-1, keepdims=True), 1e-30)
    return float((np.abs(got - ref) / scale).max())


def assert_parity(case, x, flags, L=None, check_out=True):
    """Runs the GPU layer and the oracle on x; routing must match bit for bit."""
    T = x.shape[0]
    ref = O.moe_forward(case, x, flags)
    own = L is None
    if own:
        L = make_layer(case, max_tokens=T)
    try:
        out, idx, w = L.forward(x, apply_norm=bool(flags & O.APPLY_NORM), add_residual=bool(flags & O.ADD_RESIDUAL))
        logits, xn = L.last_router(T)
        perm, off = L.last_dispatch(T)
    finally:
        if own:
            L.close()
    assert np.array_equal(xn.view(np.uint32), ref["xn"].view(np.uint32)), "RMSNorm output differs"
    assert np.array_equal(logits.view(np.uint32), ref["logits"].view(np.uint32)), "router logits differ"
    assert np.array_equal(idx, ref["topk_idx"]), "top-k indices differ"
    assert np.array_equal(w.view(np.uint32), ref["topk_w"].view(np.uint32)), "top-k weights differ"
    E = case.cfg["n_experts"]
    k = idx.shape[1]
    rperm, _, roff = O.dispatch(ref["topk_idx"], T, k, E)
    assert np.array_equal(perm, rperm), "dispatch permutation differs"
    assert np.array_equal(off, roff), "dispatch offsets differ"
    err = row_rel_err(out, ref["out"])
    if check_out:
        assert err <= OUT_TOL, f"output max relative error {err:.3e}"
    return dict(err=err, out=out, ref=ref)


def sample_tokens(idx, T, n=24, seed=0):
    """Tokens whose outputs are checked against the oracle when a batch is too
    large for the oracle to run whole: the first and last few, tokens of the
    most loaded expert (its group takes the large-group path) and random ones."""
    if T <= n:
        return np.arange(T)
    rng = np.random.default_rng(seed)
    counts = np.bincount(idx.ravel())
    top = int(np.argmax(counts))
    busy = np.nonzero((idx == top).any(axis=1))[0]
    pick = set(range(4)) | set(range(T - 4, T)) | set(busy[:: max(1, len(busy) // 8)][:8].tolist())
    pick |= set(rng.choice(T, size=n, replace=False).tolist())
    return np.array(sorted(pick))


def check_synth_batch(spec, L, x, flags, full_limit=64, workers=None, check_dispatch=True):
    """Runs the layer L (built from the tests.synth_layer.SynthLayer `spec`)
    on host tokens x and checks it against the oracle: routing (xn, logits,
    top-k, weights, dispatch) bit-exact for every token; outputs within
    OUT_TOL for every token when T <= full_limit, else for a sample of tokens
    (each token's output depends on that token alone).  Returns a summary."""
    import torch
    import qauntrunner_b200 as Q_
    T = x.shape[0]
    dev = L.desc.device
    out, idx, w = L.forward(x, apply_norm=bool(flags & O.APPLY_NORM), add_residual=bool(flags & O.ADD_RESIDUAL))
    logits, xn = L.last_router(T)
    perm, off = L.last_dispatch(T)
    case0 = spec.oracle_case(torch, Q_, dev, experts=())
    r = O.moe_route_par(case0, x, flags, workers)
    assert np.array_equal(xn.view(np.uint32), r["xn"].view(np.uint32)), "RMSNorm output differs"
    assert np.array_equal(logits.view(np.uint32), r["logits"].view(np.uint32)), "router logits differ"
    assert np.array_equal(idx, r["topk_idx"]), "top-k indices differ"
    assert np.array_equal(w.view(np.uint32), r["topk_w"].view(np.uint32)), "top-k weights differ"
    E = spec.cfg["n_experts"]
    k = idx.shape[1]
    rperm, _, roff = O.dispatch(r["topk_idx"], T, k, E)
    if check_dispatch:   # (an expert-parallel layer dispatches every rank's tokens)
        assert np.array_equal(perm, rperm), "dispatch permutation differs"
        assert np.array_equal(off, roff), "dispatch offsets differ"
    toks = np.arange(T) if T <= full_limit else sample_tokens(idx, T)
    case = spec.oracle_case(torch, Q_, dev, experts=np.unique(idx[toks]))
    ref = O.moe_forward_par(case, x[toks], flags, workers)
    err = row_rel_err(out[toks], ref["out"])
    return dict(err=err, tokens_checked=int(len(toks)), T=T, max_group=int(np.diff(roff).max()),
                routing_bit_exact=True, out=out)
