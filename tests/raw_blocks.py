"""Seeded blocks of the formats the reference stores without a GPU-specific
layout (Q2_K, Q3_K, Q5_K, I8_BLK, B1, B1X, T1E, T1E_LO), with the byte layouts
of src/QuantRunner.Core/Dtypes.cs:6-26 and BlockDequantizer.cs.  Codes are
random; scale fields hold f16 values of a realistic magnitude; T1E streams are
encoded with a restatement of EntropyCoder.Encode3 (EntropyCoder.cs:43-79)
from ternary symbols drawn with the block's stated counts."""
import numpy as np

from tests import oracle_api as O

L_RANS = 1 << 23


def rans_encode3(syms, f0, f1, cap):
    """EntropyCoder.Encode3: bytes (front-aligned, zero-padded to cap) or None
    when the stream does not fit."""
    f2 = 256 - f0 - f1
    out = bytearray(cap)
    ptr, x = cap, L_RANS
    for s in reversed(list(syms)):
        f, c = (f0, 0) if s == 0 else ((f1, f0) if s == 1 else (f2, f0 + f1))
        assert f > 0
        while x >= L_RANS * f:
            if ptr == 0:
                return None
            ptr -= 1
            out[ptr] = x & 0xFF
            x >>= 8
        x = ((x // f) << 8) + (x % f) + c
    for _ in range(4):
        if ptr == 0:
            return None
        ptr -= 1
        out[ptr] = x & 0xFF
        x >>= 8
    used = cap - ptr
    return bytes(out[ptr:]) + bytes(cap - used)


def _f16(v):
    return np.array([v], np.float16).view(np.uint16)[0]


def _put16(b, off, v):
    b[off] = int(v) & 0xFF
    b[off + 1] = (int(v) >> 8) & 0xFF


def make_blocks(fmt, nblocks, rng, scale=0.02):
    """nblocks blocks of `fmt` as one byte array."""
    bs, bb = O.BLOCK_SPEC[fmt]
    out = np.zeros((nblocks, bb), np.uint8)
    for i in range(nblocks):
        b = out[i]
        if fmt == O.Q2_K:
            b[:80] = rng.integers(0, 256, 80)
            _put16(b, 80, _f16(scale * rng.uniform(0.05, 0.15)))
            _put16(b, 82, _f16(scale * rng.uniform(0.05, 0.2)))
        elif fmt == O.Q3_K:
            b[:108] = rng.integers(0, 256, 108)
            _put16(b, 108, _f16(scale * rng.uniform(0.005, 0.02)))
        elif fmt == O.Q5_K:
            _put16(b, 0, _f16(scale * rng.uniform(0.002, 0.006)))
            _put16(b, 2, _f16(scale * rng.uniform(0.002, 0.006)))
            b[4:] = rng.integers(0, 256, bb - 4)
        elif fmt == O.I8_BLK:
            _put16(b, 0, _f16(scale * rng.uniform(0.005, 0.02)))
            b[2:] = rng.integers(0, 256, 256)
        elif fmt in (O.B1, O.B1X):
            _put16(b, 0, _f16(scale * rng.uniform(0.5, 1.5)))
            b[2:34] = rng.integers(0, 256, 32)
            if fmt == O.B1X:
                k = int(rng.integers(0, 5))
                b[34] = k
                for e, idx in enumerate(rng.choice(256, size=k, replace=False)):
                    b[35 + 3 * e] = idx
                    _put16(b, 35 + 3 * e + 1, _f16(scale * rng.normal() * 3))
        elif fmt in (O.T1E, O.T1E_LO):
            cap = bb - 6
            for _ in range(100):
                f0 = int(rng.integers(150, 230))
                f1 = int(rng.integers(1, 256 - f0))
                p = np.array([f0, f1, 256 - f0 - f1], np.float64) / 256
                syms = rng.choice(3, size=256, p=p)
                enc = rans_encode3(syms, f0, f1, cap)
                if enc is not None:
                    break
            else:
                raise RuntimeError("no T1E stream fitted")
            _put16(b, 0, f0)
            _put16(b, 2, f1)
            _put16(b, 4, _f16(scale * rng.uniform(0.5, 1.5)))
            b[6:] = np.frombuffer(enc, np.uint8)
        else:
            raise ValueError(fmt)
    return out.reshape(-1)


def make_matrix(fmt, rows, cols, rng, scale=0.02):
    return make_blocks(fmt, rows * cols // 256, rng, scale)
