"""The device quantiser (qrm_synth_quantize) must produce the same bytes as
the CPU restatement of BlockQuantizer on the same floats."""
import numpy as np
import pytest

import qauntrunner_b200 as Q
from tests import oracle_api as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("fmt", [O.Q4_0, O.Q8_0, O.Q4_K, O.Q6_K, O.TRI, O.TRI_LEGACY])
@pytest.mark.parametrize("sigma", [0.02, 1.0])
def test_device_quantiser_is_byte_identical(fmt, sigma):
    import torch
    n = 256 * 2048
    xd = torch.empty(n, dtype=torch.float32, device="cuda")
    Q.synth_gaussian(xd.data_ptr(), n, 1234 + fmt, sigma)
    nbytes = O.tensor_bytes(n, fmt)
    qd = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    Q.synth_quantize(fmt, xd.data_ptr(), n, qd.data_ptr())
    torch.cuda.synchronize()
    x = xd.cpu().numpy()
    assert abs(float(x.std()) / sigma - 1.0) < 0.01 and abs(float(x.mean())) < 0.01 * sigma
    want = O.quantize(fmt, x)
    got = qd.cpu().numpy()
    assert np.array_equal(got, want)


def test_gaussian_is_seeded():
    import torch
    a = torch.empty(4096, dtype=torch.float32, device="cuda")
    b = torch.empty(4096, dtype=torch.float32, device="cuda")
    Q.synth_gaussian(a.data_ptr(), 4096, 7, 1.0)
    Q.synth_gaussian(b.data_ptr(), 4096, 7, 1.0)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    Q.synth_gaussian(b.data_ptr(), 4096, 8, 1.0)
    torch.cuda.synchronize()
    assert not torch.equal(a, b)
