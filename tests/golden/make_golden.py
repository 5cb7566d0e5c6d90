"""Writes tests/golden/kat_blocks.json: known-answer decoder blocks.

The blocks marked "reference" are transcribed from the reference's own selftest
(src/QuantRunner.Cli/Commands.cs:2257-2325, GgmlLegacyCompat) and its f16 edge
cases (tests/QuantRunner.Tests/Program.cs:60-69).  The reference has no known
answer for the 20-byte .qw Q4_0 block or for TRI; the blocks marked "formula"
are hand-built here and their expected values follow directly from the decoder
formulas (BlockDequantizer.cs:52-69 for Q4_0: y = d*(q-8), low nibble = weight
i, high nibble = weight i+16; BlockDequantizer.cs:258-276 for TRI: code of
weight i at byte 2+i/4, bits 2*(i&3), 01 -> +s, 10 -> -s, else 0).

Run:  python tests/golden/make_golden.py
"""
import json
import os


def block(nbytes, sets):
    b = [0] * nbytes
    for off, val in sets:
        b[off] = val & 0xFF
    return b


def main():
    kats = []
    # Commands.cs:2257-2265: Q8_0, d=0.25 (f16 0x3400), qs[0]=-8 -> y0=-2
    kats.append(dict(name="q8_0", src="reference Commands.cs:2257-2265", fmt=4,
                     bytes=block(34, [(0, 0x00), (1, 0x34), (2, -8)]),
                     expect={"0": -2.0}))
    # Commands.cs:2299-2311: Q4_K, d=2, dmin=1, scales[0]=3, [1]=2, [4]=1, [5]=1,
    # qs[0]=0x5F -> y0 = 2*3*15 - 1, y32 = 2*2*5 - 1
    kats.append(dict(name="q4_k", src="reference Commands.cs:2299-2311", fmt=6,
                     bytes=block(144, [(0, 0x00), (1, 0x40), (2, 0x00), (3, 0x3C),
                                       (4, 3), (5, 2), (8, 1), (9, 1), (16, 0x5F)]),
                     expect={"0": 89.0, "32": 19.0}))
    # Commands.cs:2313-2325: Q6_K, d=0.5, ql[0]=0x21, ql[32]=0x43, qh[0]=0b00011001,
    # scales[0]=2, [2]=1, [4]=3, [6]=-1 -> y0=-15, y32=1.5, y64=-21, y96=14
    kats.append(dict(name="q6_k", src="reference Commands.cs:2313-2325", fmt=7,
                     bytes=block(210, [(208, 0x00), (209, 0x38), (0, 0x21), (32, 0x43),
                                       (128, 0b00011001), (192, 2), (194, 1), (196, 3), (198, -1)]),
                     expect={"0": -15.0, "32": 1.5, "64": -21.0, "96": 14.0}))
    # formula KAT, .qw Q4_0 (20 B): d=0.5 (f16 0x3800); qs[0]=0x08 -> y0=(8-8)*0.5=0,
    # y16=(0-8)*0.5=-4; qs[1]=0xF2 -> y1=(2-8)*0.5=-3, y17=(15-8)*0.5=3.5; pad bytes 18-19 ignored
    kats.append(dict(name="q4_0", src="formula BlockDequantizer.cs:52-69", fmt=3,
                     bytes=block(20, [(0, 0x00), (1, 0x38), (2, 0x08), (3, 0xF2), (18, 0xAA), (19, 0x55)]),
                     expect={"0": 0.0, "16": -4.0, "1": -3.0, "17": 3.5, "2": -4.0, "18": -4.0}))
    # formula KAT, TRI (18 B): s=1.5 (f16 0x3E00); byte2=0b10_01_00_01 -> w0=+s, w1=0, w2=+s, w3=-s;
    # byte17=0b11_00_10_01 -> w60=+s, w61=-s, w62=0, w63=0 (code 11 decodes to 0)
    kats.append(dict(name="tri", src="formula BlockDequantizer.cs:258-276", fmt=8,
                     bytes=block(18, [(0, 0x00), (1, 0x3E), (2, 0b10010001), (17, 0b11001001)]),
                     expect={"0": 1.5, "1": 0.0, "2": 1.5, "3": -1.5, "60": 1.5, "61": -1.5,
                             "62": 0.0, "63": 0.0, "4": 0.0}))
    # tests/QuantRunner.Tests/Program.cs:62-69: f16 decode edge cases
    f16 = [
        dict(h=0x0000, v=0.0), dict(h=0x8000, v=-0.0), dict(h=0x3C00, v=1.0),
        dict(h=0xBC00, v=-1.0), dict(h=0x7BFF, v=65504.0), dict(h=0x7C00, v="inf"),
        dict(h=0x0001, v=5.9604645e-8),
    ]
    out = dict(kats=kats, f16=f16)
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "kat_blocks.json")
    with open(path, "w") as fh:
        json.dump(out, fh, indent=1)
    print("wrote", path)


if __name__ == "__main__":
    main()
