"""The oracle's restatement of the formats QuantRunner stores that have no
GPU-specific layout (Q2_K, Q3_K, Q5_K, I8_BLK, B1, B1X, T1E, T1E_LO): decoders
pinned by hand-computed known answers from the BlockDequantizer.cs formulas,
T1E streams round-trip through EntropyCoder's encode / decode pair, and the
fused dots agree with dot(dequantised row, x) within 2e-4 (the reference's own
fused-dot check, Commands.cs:1188-1234)."""
import numpy as np
import pytest

from tests import oracle_api as O
from tests.raw_blocks import make_blocks, rans_encode3


def _h(v):
    return int(np.array([v], np.float16).view(np.uint16)[0])


def test_q2_k_known_answer():
    b = np.zeros(84, np.uint8)
    b[0] = 0x35                  # sub-block 0: sc 5, m 3
    b[1] = 0x21                  # sub-block 1: sc 1, m 2
    b[16] = 0b11100100           # weight 0: code 0 (shift 0); weight 32: code 1 (shift 2); 64: 2; 96: 3
    b[17] = 3                    # weight 1: code 3
    b[16 + 1] |= 0               # (weight 1 keeps code 3)
    d, dmin = 0.5, 0.25
    b[80:82] = np.frombuffer(np.array([d], np.float16).tobytes(), np.uint8)
    b[82:84] = np.frombuffer(np.array([dmin], np.float16).tobytes(), np.uint8)
    y = O.dequantize(O.Q2_K, b, 256)
    assert y[0] == np.float32(d * 5 * 0 - dmin * 3)
    assert y[1] == np.float32(d * 5 * 3 - dmin * 3)
    assert y[32] == np.float32(d * (b[2] & 15) * 1 - dmin * (b[2] >> 4))    # sub-block 2 (all-zero scale byte)
    assert y[16] == np.float32(d * 1 * 0 - dmin * 2)


def test_q3_k_and_q5_k_known_answers():
    b = np.zeros(110, np.uint8)
    b[0] = 0b1                   # hmask: weight 0 keeps its high bit (no -4)
    b[32] = 0b10                 # weight 0: code 2
    b[96] = 0x07                 # scale 0 low nibble 7, high bits from byte 104 = 0 -> 7 - 32 = -25
    b[108:110] = np.frombuffer(np.array([0.5], np.float16).tobytes(), np.uint8)
    y = O.dequantize(O.Q3_K, b, 256)
    assert y[0] == np.float32(0.5 * -25 * 2)
    assert y[1] == np.float32(0.5 * -25 * (0 - 4))          # code 0, hmask bit clear: -4
    c = np.zeros(176, np.uint8)
    c[0:2] = np.frombuffer(np.array([0.25], np.float16).tobytes(), np.uint8)
    c[2:4] = np.frombuffer(np.array([0.125], np.float16).tobytes(), np.uint8)
    c[4] = 3                     # sub-block 0: sc 3
    c[8] = 2                     # sub-block 0: m 2
    c[16] = 0x9A                 # weight 0: low nibble 10; weight 32 (sub 1): high nibble 9
    c[144] = 0b1                 # weight 0: +16
    y = O.dequantize(O.Q5_K, c, 256)
    assert y[0] == np.float32(np.float32(0.25 * 3) * 26 - np.float32(0.125 * 2))


def test_i8_b1_b1x_known_answers():
    b = np.zeros(258, np.uint8)
    b[0:2] = np.frombuffer(np.array([0.5], np.float16).tobytes(), np.uint8)
    b[2] = 0xFE                  # -2
    b[3] = 5
    y = O.dequantize(O.I8_BLK, b, 256)
    assert (y[0], y[1], y[2]) == (np.float32(-1.0), np.float32(2.5), np.float32(0.0))
    m = np.zeros(47, np.uint8)
    m[0:2] = np.frombuffer(np.array([0.75], np.float16).tobytes(), np.uint8)
    m[2] = 0b101
    y = O.dequantize(O.B1, m[:34], 256)
    assert (y[0], y[1], y[2], y[255]) == (np.float32(0.75), np.float32(-0.75), np.float32(0.75), np.float32(-0.75))
    m[34] = 1
    m[35] = 1
    m[36:38] = np.frombuffer(np.array([3.0], np.float16).tobytes(), np.uint8)
    y = O.dequantize(O.B1X, m, 256)
    assert (y[0], y[1]) == (np.float32(0.75), np.float32(3.0))


@pytest.mark.parametrize("fmt,sb", [(O.T1E, 34), (O.T1E_LO, 26)])
def test_t1e_round_trip(fmt, sb):
    rng = np.random.default_rng(3)
    for _ in range(20):
        f0 = int(rng.integers(170, 230))
        f1 = int(rng.integers(1, 256 - f0))
        syms = rng.choice(3, size=256, p=np.array([f0, f1, 256 - f0 - f1]) / 256)
        enc = rans_encode3(syms, f0, f1, sb)
        if enc is None:
            continue
        blk = np.zeros(6 + sb, np.uint8)
        blk[0:2] = [f0 & 0xFF, f0 >> 8]
        blk[2:4] = [f1 & 0xFF, f1 >> 8]
        blk[4:6] = np.frombuffer(np.array([0.5], np.float16).tobytes(), np.uint8)
        blk[6:] = np.frombuffer(enc, np.uint8)
        y = O.dequantize(fmt, blk, 256)
        want = np.where(syms == 1, 0.5, np.where(syms == 2, -0.5, 0.0)).astype(np.float32)
        assert np.array_equal(y, want)


@pytest.mark.parametrize("fmt", O.RAW_FORMATS)
def test_fused_dot_matches_dequantised(fmt):
    rng = np.random.default_rng(int(fmt))
    rows, cols = 6, 1024
    w = make_blocks(fmt, rows * cols // 256, rng)
    x = rng.standard_normal(cols, dtype=np.float32)
    y = O.matvec(fmt, w, rows, cols, x)
    rb = O.tensor_bytes(cols, fmt)
    for r in range(rows):
        deq = O.dequantize(fmt, w[r * rb:(r + 1) * rb], cols).astype(np.float64)
        ref = float(deq @ x.astype(np.float64))
        scale = float(np.abs(deq).sum() * np.abs(x).max()) + 1e-12
        assert abs(float(y[r]) - ref) <= 2e-4 * scale, (fmt, r, float(y[r]), ref)
