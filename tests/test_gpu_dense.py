"""Dense FFN (StreamingEngine.DenseFfn / DenseFfnOut, StreamingEngine.cs:
599-622) from three matrix operators, against the oracle's MatVecParallel,
SwiGLU and AxpyF32: within 1e-3 relative per token, for every expert format,
with and without the residual, plain and limited SwiGLU, and in place
(out aliasing x, as the engine adds into x)."""
import numpy as np
import pytest

import qauntrunner_b200 as Q
from tests import oracle_api as O
from tests.gpu_helpers import OUT_TOL, row_rel_err

pytestmark = pytest.mark.gpu


def _oracle(fmts, mats, d, f, xn, x, limit):
    out = np.zeros_like(xn)
    for t in range(xn.shape[0]):
        g = O.matvec(fmts[0], mats[0], f, d, xn[t])
        u = O.matvec(fmts[1], mats[1], f, d, xn[t])
        y = O.matvec(fmts[2], mats[2], d, f, O.swiglu(g, u, limit))
        out[t] = (x[t] + (np.float32(1.0) * y).astype(np.float32)).astype(np.float32) if x is not None else y
    return out


@pytest.mark.parametrize("fmt,d,f,limit,residual", [
    (O.Q4_K, 1024, 2816, 0.0, True),
    (O.Q8_0, 512, 1536, 10.0, False),
    (O.Q4_0, 1024, 2816, 0.0, True),
    (O.Q6_K, 768, 1536, 0.0, True),
    (O.TRI, 512, 1024, 7.0, False),
])
def test_dense_ffn(fmt, d, f, limit, residual):
    import torch
    rng = np.random.default_rng(7)
    qf = O.TRI_LEGACY if fmt == O.TRI else fmt
    shapes = [(f, d), (f, d), (d, f)]
    mats = [O.quantize(qf, rng.standard_normal(s, dtype=np.float32) * np.float32(0.02)) for s in shapes]
    T = 6
    xn = rng.standard_normal((T, d), dtype=np.float32)
    x = rng.standard_normal((T, d), dtype=np.float32) if residual else None
    ref = _oracle((fmt,) * 3, mats, d, f, xn, x, limit)
    ms = [Q.Matrix(fmt, s[0], s[1], m) for s, m in zip(shapes, mats)]
    ffn = Q.DenseFfn(*ms, max_tokens=T)
    try:
        xn_d = torch.from_numpy(xn).cuda()
        out_d = torch.empty((T, d), device="cuda")
        x_d = torch.from_numpy(x).cuda() if residual else None
        ffn.forward(xn_d.data_ptr(), x_d.data_ptr() if residual else None, T, out_d.data_ptr(), limit)
        torch.cuda.synchronize()
        err = row_rel_err(out_d.cpu().numpy(), ref)
        assert err <= OUT_TOL, f"relative error {err:.3e}"
        if residual:   # in place: out aliases x
            ffn.forward(xn_d.data_ptr(), x_d.data_ptr(), T, x_d.data_ptr(), limit)
            torch.cuda.synchronize()
            assert np.array_equal(x_d.cpu().numpy(), out_d.cpu().numpy())
    finally:
        ffn.close()
        for m in ms:
            m.close()


def test_dense_ffn_rejects_bad_shapes():
    rng = np.random.default_rng(8)
    a = Q.Matrix(O.Q8_0, 256, 512, O.quantize(O.Q8_0, rng.standard_normal((256, 512), dtype=np.float32)))
    b = Q.Matrix(O.Q8_0, 256, 512, O.quantize(O.Q8_0, rng.standard_normal((256, 512), dtype=np.float32)))
    try:
        with pytest.raises(Q.QrmError) as ei:
            Q.DenseFfn(a, a, b)          # down must be [d x f]
        assert ei.value.code == Q.E_INVALID
    finally:
        a.close()
        b.close()
