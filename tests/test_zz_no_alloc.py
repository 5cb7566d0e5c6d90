"""qrm_matrix_gemv_static (activation tables in the library's fixed per-device
scratch, no allocation) against qrm_matrix_gemv on the same inputs.  Collected
last so it also runs after every other GPU test in the same process."""
import numpy as np
import pytest

import qauntrunner_b200 as Q
from tests import oracle_api as O

pytestmark = pytest.mark.gpu

# both entry points run the same kernels; the bound only allows for a
# different launch order of the float reductions
TOL = 1e-6
SCRATCH_BYTES = 1 << 20


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    assert torch.cuda.is_available()
    return torch


def _matrix(fmt, rows, cols, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal(rows * cols) * 0.4).astype(np.float32)
    return Q.Matrix(fmt, rows, cols, O.quantize(fmt, w))


def _rel(a, b):
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


@pytest.mark.parametrize("fmt", [O.Q4_K, O.Q8_0, O.Q4_0, O.Q6_K])
def test_static_scratch_matches_allocating_gemv(torch_cuda, fmt):
    torch = torch_cuda
    rows, cols = 512, 2048
    m = _matrix(fmt, rows, cols, 100 + fmt)
    rng = np.random.default_rng(7)
    try:
        # two consecutive calls with different T and inputs
        for T in (3, 5):
            x = torch.from_numpy((rng.standard_normal((T, cols)) * 0.5).astype(np.float32)).cuda()
            y_ref = torch.zeros((T, rows), dtype=torch.float32, device="cuda")
            y_got = torch.full((T, rows), float("nan"), dtype=torch.float32, device="cuda")
            m.gemv(x.data_ptr(), T, y_ref.data_ptr())
            m.gemv_static(x.data_ptr(), T, y_got.data_ptr())
            torch.cuda.synchronize()
            got, ref = y_got.cpu().numpy(), y_ref.cpu().numpy()
            assert np.isfinite(got).all()
            assert _rel(got, ref) <= TOL
    finally:
        m.close()


def test_static_scratch_rejects_oversized_batch(torch_cuda):
    torch = torch_cuda
    rows, cols = 256, 1536
    stride = (2 * cols + 128 + 8 * (cols // 32) + 15) // 16 * 16
    T = SCRATCH_BYTES // stride + 1
    m = _matrix(O.Q4_K, rows, cols, 5)
    try:
        x = torch.zeros((T, cols), dtype=torch.float32, device="cuda")
        y = torch.zeros((T, rows), dtype=torch.float32, device="cuda")
        with pytest.raises(Q.QrmError) as ei:
            m.gemv_static(x.data_ptr(), T, y.data_ptr())
        assert ei.value.code == -9 and "static scratch" in str(ei.value)
        # the largest batch that fits still runs
        m.gemv_static(x.data_ptr(), T - 1, y.data_ptr())
        torch.cuda.synchronize()
        assert float(y[: T - 1].abs().max()) == 0.0
    finally:
        m.close()
