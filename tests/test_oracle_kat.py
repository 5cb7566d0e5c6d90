"""Pins the CPU oracle against the reference's own known answers and
tolerance checks before anything is compared with it.

- decoder known-answer blocks (tests/golden/kat_blocks.json, transcribed from
  src/QuantRunner.Cli/Commands.cs:2257-2325, plus formula blocks for the .qw
  Q4_0 and TRI layouts that the reference never pinned);
- f16 decode/encode cases of tests/QuantRunner.Tests/Program.cs:60-83;
- quantise->dequantise relative-RMS bounds of Program.cs:96-127;
- fused dot == dequantised fp32 matvec to 2e-4, Program.cs:129-165 and
  Commands.cs:1188-1234 (incl. MatVecParallel "must not corrupt y");
- RowPtr strides of Program.cs:225-238.
"""
import json
import math
import os

import numpy as np
import pytest

from tests import oracle_api as O

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "kat_blocks.json")


def load_gold():
    with open(GOLD) as fh:
        return json.load(fh)


@pytest.mark.parametrize("kat", load_gold()["kats"], ids=lambda k: k["name"])
def test_decoder_known_answers(kat):
    bs, bb = O.BLOCK_SPEC[kat["fmt"]]
    blk = np.array(kat["bytes"], dtype=np.uint8)
    assert blk.size == bb
    y = O.dequantize(kat["fmt"], blk, bs)
    for idx, want in kat["expect"].items():
        assert abs(float(y[int(idx)]) - want) <= 1e-6, (kat["name"], idx, y[int(idx)], want)


def test_decoder_kat_through_dot():
    # the fused dot must see the same values as the decoder on the KAT blocks
    for kat in load_gold()["kats"]:
        bs, _ = O.BLOCK_SPEC[kat["fmt"]]
        blk = np.array(kat["bytes"], dtype=np.uint8)
        y = O.dequantize(kat["fmt"], blk, bs)
        for idx in kat["expect"]:
            x = np.zeros(bs, np.float32)
            x[int(idx)] = 1.0
            got = O.matvec(kat["fmt"], blk, 1, bs, x)[0]
            assert got == y[int(idx)], kat["name"]


def test_f16_edge_cases():
    L = O.lib()
    for case in load_gold()["f16"]:
        got = L.orc_f16_to_f32(case["h"])
        want = math.inf if case["v"] == "inf" else case["v"]
        if case["h"] == 0x0001:
            assert abs(got - want) <= 1e-13
        else:
            assert got == want
            if want == 0.0:
                assert math.copysign(1.0, got) == math.copysign(1.0, want)
    # Program.cs:71-83 round trip with the reference's tolerances
    rng = np.random.default_rng(1)
    v = ((rng.random(100000) * 2 - 1) * np.exp2(rng.integers(-14, 15, 100000))).astype(np.float32)
    h = np.zeros(v.size, np.uint16)
    L.orc_f32_to_f16_batch(O.ptr(v), O.ptr(h), v.size)
    back = np.array([L.orc_f16_to_f32(int(x)) for x in h[:20000]], np.float32)
    vv = v[:20000]
    tol = np.where(np.abs(vv) < 6.1e-5, 6e-8, np.abs(vv) * 0.0005 + 1e-30)
    assert np.all(np.abs(back - vv) <= tol)
    assert L.orc_f16_to_f32(L.orc_f32_to_f16(65504.0)) == 65504.0
    # half-up mantissa rounding quirk (Dtypes.cs:111): 1 + 2^-11 rounds up to 1 + 2^-10
    assert L.orc_f32_to_f16(1.0 + 2.0 ** -11) == 0x3C01


RMS_TOL = [(O.Q8_0, 0.02), (O.Q6_K, 0.03), (O.Q4_0, 0.11), (O.Q4_K, 0.09), (O.TRI, 0.55)]


@pytest.mark.parametrize("fmt,tol", RMS_TOL)
def test_quant_roundtrip_rms(fmt, tol):
    bs, _ = O.BLOCK_SPEC[fmt]
    n = bs * 32
    x = (np.random.default_rng(7).standard_normal(n) * 0.5).astype(np.float32)
    b = O.quantize(fmt, x)
    y = O.dequantize(fmt, b, n)
    rms = math.sqrt(np.mean((y.astype(np.float64) - x) ** 2)) / math.sqrt(max(np.mean(x.astype(np.float64) ** 2), 1e-12))
    assert rms <= tol, (fmt, rms)


def test_tri_legacy_zero_fraction_and_bound():
    x = (np.random.default_rng(3).standard_normal(64 * 512) * 0.02).astype(np.float32)
    b = O.quantize(O.TRI_LEGACY, x)
    y = O.dequantize(O.TRI, b, x.size)
    zero_frac = float(np.mean(y == 0))
    assert 0.25 < zero_frac < 0.45  # "about 1/3 zeros"
    rms = math.sqrt(np.mean((y.astype(np.float64) - x) ** 2)) / math.sqrt(np.mean(x.astype(np.float64) ** 2))
    assert rms <= 0.7


@pytest.mark.parametrize("fmt", [O.Q4_0, O.Q8_0, O.Q4_K, O.Q6_K, O.TRI, O.F32, O.F16, O.BF16])
def test_dot_matches_dequantised_reference(fmt):
    rng = np.random.default_rng(11)
    bs, _ = O.BLOCK_SPEC[fmt]
    cols = max(bs * 4, 64)
    rows = 12
    w = (rng.standard_normal(rows * cols) * 0.4).astype(np.float32)
    x = (rng.standard_normal(cols) * 0.5).astype(np.float32)
    wq = O.quantize(fmt, w)
    wdq = O.dequantize(fmt, wq, rows * cols).reshape(rows, cols)
    yk = O.matvec(fmt, wq, rows, cols, x, threads=1)
    yp = O.matvec(fmt, wq, rows, cols, x, threads=4)
    assert np.array_equal(yk, yp)
    for r in range(rows):
        s = np.float32(0)
        for c in range(cols):
            s = np.float32(s + np.float32(wdq[r, c] * x[c]))
        scale = max(abs(float(s)), 1e-3)
        assert abs(float(yk[r]) - float(s)) / scale <= 2e-4, (fmt, r, yk[r], s)


def test_row_strides():
    assert O.tensor_bytes(512, O.Q4_K) == 512 // 256 * 144
    assert O.tensor_bytes(128, O.Q4_0) == 128 // 32 * 20
    assert O.lib().orc_tensor_bytes(100, O.Q4_K) == -1


def test_matvec_parallel_large_matches_serial():
    rng = np.random.default_rng(5)
    rows, cols = 2048, 1024  # above the 1 MiB / 16-row threshold
    w = O.quantize(O.Q4_K, (rng.standard_normal(rows * cols) * 0.02).astype(np.float32))
    x = rng.standard_normal(cols).astype(np.float32)
    assert np.array_equal(O.matvec(O.Q4_K, w, rows, cols, x, 1), O.matvec(O.Q4_K, w, rows, cols, x, 7))


def test_softmax_topk_known_answer():
    # E=8 (insertion-sort regime of Array.Sort: ties keep index order)
    L = O.lib()
    logits = np.array([0.5, 2.0, -1.0, 2.0, 0.0, 1.0, -3.0, 0.25], np.float32)
    sel = np.zeros(2, np.int32)
    w = np.zeros(2, np.float32)
    probs = np.zeros(8, np.float32)
    L.orc_route_softmax(O.ptr(logits), 8, 2, O.ptr(sel), O.ptr(w), O.ptr(probs))
    assert list(sel) == [1, 3]
    assert w[0] == w[1] == np.float32(0.5)
    ex = O.expf((logits - np.float32(2.0)).astype(np.float32))
    s = np.float32(0)
    for v in ex:
        s = np.float32(s + v)
    assert np.array_equal(probs, (ex * np.float32(np.float32(1) / s)).astype(np.float32))


def test_sigmoid_topk_known_answer():
    L = O.lib()
    E, k = 6, 2
    logits = np.array([0.0, 1.0, -1.0, 3.0, 0.5, 2.0], np.float32)
    bias = np.array([0.0, 0.0, 0.0, -0.5, 0.6, 0.0], np.float32)
    sel = np.zeros(k, np.int32)
    w = np.zeros(k, np.float32)
    L.orc_route_sigmoid(O.ptr(logits), O.ptr(bias), E, k, 2.5, O.ptr(sel), O.ptr(w))
    sig = (np.float32(1) / (np.float32(1) + O.expf(-logits))).astype(np.float32)
    choice = sig + bias
    order = sorted(range(E), key=lambda i: (-choice[i], i))[:k]
    assert list(sel) == order  # e4 (0.622+0.6) beats e3 (0.953-0.5)
    wsum = np.float32(sig[order[0]] + sig[order[1]])
    inv = np.float32(1) / np.float32(wsum + np.float32(1e-20))
    assert np.array_equal(w, np.array([sig[i] * inv * np.float32(2.5) for i in order], np.float32))


def test_dispatch_is_stable_counting_sort():
    sel = np.array([[3, 1], [1, 0], [3, 2], [0, 1]], np.int32)
    perm, inv, off = O.dispatch(sel, 4, 2, 4)
    assert list(off) == [0, 2, 5, 6, 8]
    assert list(perm) == [3, 6, 1, 2, 7, 5, 0, 4]
    assert all(perm[inv[a]] == a for a in range(8))
