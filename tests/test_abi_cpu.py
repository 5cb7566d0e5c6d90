"""C ABI checks that need no GPU: the library loads, exports every entry
point include/qrmoe.h declares, and fails cleanly (an error code and a
message, no crash) when no usable device is present."""
import ctypes as C
import os

import numpy as np
import pytest

import qauntrunner_b200 as Q


def test_library_loads_and_exports_header_symbols():
    L = Q.lib()
    names = Q.header_symbols()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    assert L.qrm_version() == 1


def test_header_and_python_signatures_agree():
    assert set(Q.header_symbols()) == set(Q._SIGS)


def test_tensor_bytes_matches_block_specs():
    assert Q.tensor_bytes(512, Q.QuantFormat.Q4_K) == 288
    assert Q.tensor_bytes(128, Q.QuantFormat.Q4_0) == 80
    assert Q.tensor_bytes(64, Q.QuantFormat.TRI) == 18
    assert Q.tensor_bytes(64, Q.TRI_LEGACY) == 18
    with pytest.raises(ValueError):
        Q.tensor_bytes(100, Q.QuantFormat.Q4_K)


def _no_gpu():
    try:
        import torch
        return not torch.cuda.is_available()
    except Exception:
        return True


@pytest.mark.skipif(not _no_gpu(), reason="checks the no-device error path")
def test_create_without_device_is_a_clean_error():
    with pytest.raises(Q.QrmError) as ei:
        Q.MoeLayer(1024, 8, 2, 2816, fmt=(3, 3, 3))
    assert ei.value.code in (-5, -1)


def test_invalid_descriptions_are_rejected_before_touching_a_device():
    # format / shape validation happens first, so these errors are the same with or without a GPU
    with pytest.raises(Q.QrmError) as ei:
        Q.MoeLayer(1024, 8, 2, 2816, fmt=(1, 1, 1))
    assert ei.value.code == -2
    with pytest.raises(Q.QrmError) as ei:
        Q.MoeLayer(1000, 8, 2, 2816, fmt=(3, 3, 3))
    assert ei.value.code == -1
    with pytest.raises(Q.QrmError) as ei:
        Q.MoeLayer(1024, 4, 6, 2816, fmt=(3, 3, 3))
    assert ei.value.code == -1
    with pytest.raises(Q.QrmError) as ei:
        Q.MoeLayer(1024, 8, 2, 2848, fmt=(6, 6, 6))   # 2848 % 256 != 0 for the Q4_K down matrix
    assert ei.value.code == -1
    with pytest.raises(Q.QrmError) as ei:
        Q.MoeLayer(1024, 8, 2, 2048, fmt=(6, 3, 6))   # gate and up formats differ
    assert ei.value.code == -2
