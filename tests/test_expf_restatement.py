"""Pins the product's binary32 exp (qauntrunner_b200/csrc/glibc_expf.cuh)
against the host C runtime expf -- what .NET's MathF.Exp calls -- on every
binary32 input, on the CPU."""
import os
import subprocess
import tempfile

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

PROG = r"""
#include "glibc_expf.cuh"
#include <math.h>
#include <stdio.h>
#include <string.h>
#include <thread>
#include <vector>
int main() {
    const int nt = (int)std::thread::hardware_concurrency() > 0 ? (int)std::thread::hardware_concurrency() : 4;
    std::vector<long long> bad(nt, 0);
    std::vector<std::thread> th;
    for (int t = 0; t < nt; t++)
        th.emplace_back([&, t]() {
            for (unsigned long long u = t; u < 0x100000000ull; u += nt) {
                float x; unsigned int b = (unsigned int)u; memcpy(&x, &b, 4);
                float a = expf(x), c = qrm::expf_glibc(x);
                unsigned int ua, uc; memcpy(&ua, &a, 4); memcpy(&uc, &c, 4);
                if (ua != uc && !(isnan(a) && isnan(c))) { if (bad[t] < 3) printf("x=%a glibc=%a mine=%a\n", x, a, c); bad[t]++; }
            }
        });
    long long tot = 0;
    for (int t = 0; t < nt; t++) { th[t].join(); tot += bad[t]; }
    printf("mismatches %lld\n", tot);
    return tot == 0 ? 0 : 1;
}
"""


def test_expf_matches_c_runtime_on_all_floats():
    with tempfile.TemporaryDirectory() as td:
        src = os.path.join(td, "p.cpp")
        exe = os.path.join(td, "p")
        with open(src, "w") as fh:
            fh.write(PROG)
        inc = os.path.join(ROOT, "qauntrunner_b200", "csrc")
        subprocess.run(["g++", "-O2", "-ffp-contract=off", "-std=c++17", "-pthread", "-I", inc, src,
                        "-o", exe, "-lm"], check=True)
        r = subprocess.run([exe], capture_output=True, text=True, timeout=600)
        assert r.returncode == 0, r.stdout + r.stderr
        assert "mismatches 0" in r.stdout
