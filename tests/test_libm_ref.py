"""The device expf (csrc/libm_ref.cuh) against the host C library's expf.

The reference computes every exponential of the forward pass (softmax, silu)
with the C library's expf, which is not correctly rounded.  libm_ref.cuh
restates that method; this test compiles the header for the host and compares
it with the C library over all 2^32 float arguments (a few seconds on all host
threads).  The GPU build of the same header is compared in test_decoder_gpu.py.
"""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.timeout(600)
def test_expf_ref_matches_c_library_everywhere(tmp_path):
    exe = tmp_path / "libm_ref_check"
    src = os.path.join(ROOT, "tests", "libm_ref_check.cpp")
    inc = os.path.join(ROOT, "quantr-in-c_b200", "csrc")
    subprocess.run(["g++", "-O2", "-std=c++17", "-ffp-contract=off", "-fopenmp",
                    "-B/usr/lib/gcc/x86_64-linux-gnu/13/", "-I", inc, src, "-o", str(exe), "-lm"], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=540)
    assert r.stdout.strip() == "mismatches 0", r.stdout + r.stderr
