"""Generates tests/golden/quant_golden.npz from the reference's own code.

    make -C oracle ref            # compiles the reference's src/quant.c into oracle/_ref/
    python tests/golden/make_golden.py

Every expected output in the fixture comes from oracle/_ref/libquantr_ref_scalar.so,
i.e. the reference's src/quant.c compiled with its default Makefile flags
(-O3 -std=c99, scalar paths), plus its header-inline fp16 helpers
(include/quant.h:53-77) exported by oracle/ref_shim.c.  Inputs are seeded
(numpy PCG64) and stored alongside.  The fixture pins both this repository's
C restatement (tests/test_oracle.py) and the CUDA path (tests/test_gemv_gpu.py).

Cases:
  fp16_all      all 65536 halves through fp16_to_fp32 (exhaustive)
  f2h_*         special and random floats through fp32_to_fp16
  qz_*          quantize_row_q8_0 on the reference unit-test inputs
                (tests/tests.c:59, :292-293), random, tiny/huge/non-finite, tails
  dq_*          dequantize_row per type, incl. the unit-test blocks (tests/tests.c:72-123)
  vd_*          vec_dot_{q8_0,q5K,q6K}_q8_0; vd_q4k_ref_broken records what the
                reference's Q4_K kernel returns (not a parity target)
  mm_*          matmul_q_fused for Q8_0 / Q5_K / Q6_K / F32, incl. ragged d
  sm_*          KernelOps softmax (src/kernels.c:191-207): router-sized vectors,
                ties, a wide range, one element
  mr_*          KernelOps matmul_ref (src/kernels.c:18-28), the MoE router GEMV
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "quantr-in-c_b200"))

import oracle  # noqa: E402
import synth  # noqa: E402

OUT = os.path.join(HERE, "quant_golden.npz")


def main():
    ref = oracle.RefLib("scalar")
    rng = synth.rng_for(20261201)
    G = {}

    # fp16 helpers -------------------------------------------------------
    G["fp16_all"] = np.array([ref.fp16_to_fp32(h) for h in range(65536)], dtype=np.float32)
    specials = np.array([0.0, -0.0, 1.0, -1.0, 3.14159, 1e-4, 65504.0, 65519.0, 65520.0, 1e6, 6.1035156e-05,
                         6.0e-05, 1e-5, 1e-8, np.inf, -np.inf, np.nan, 2.0 ** -14, -2.0 ** -15, 0.007874016],
                        dtype=np.float32)
    f2h_in = np.concatenate([specials, rng.standard_normal(200).astype(np.float32) * 10.0,
                             (rng.standard_normal(100) * 1e-3).astype(np.float32)])
    G["f2h_in"] = f2h_in
    G["f2h_out"] = np.array([ref.fp32_to_fp16(v) for v in f2h_in], dtype=np.uint16)

    # quantize_row_q8_0 --------------------------------------------------
    qcases = {
        "ramp": ((np.arange(32, dtype=np.float32) - 16.0) * 0.125),             # tests/tests.c:59
        "sin": np.sin(np.arange(256, dtype=np.float32) * np.float32(0.05)).astype(np.float32),  # :292
        "cos": np.cos(np.arange(256, dtype=np.float32) * np.float32(0.03)).astype(np.float32),  # :293
        "randn": rng.standard_normal(2048).astype(np.float32),
        "tail100": rng.standard_normal(100).astype(np.float32),
        "zeros": np.zeros(64, dtype=np.float32),
        "tiny": (rng.standard_normal(64) * 1e-39).astype(np.float32),
        "huge": (rng.standard_normal(64) * 1e36).astype(np.float32),
        "halves": (rng.integers(-8, 9, 128).astype(np.float32) * 0.5 * np.float32(127.0 / 4.0)),
        "nonfinite": np.array([1.0, np.inf, -2.0, np.nan] + [0.5] * 28 + [np.nan] + [0.25] * 31,
                              dtype=np.float32),
    }
    for k, x in qcases.items():
        G[f"qz_{k}_x"] = x
        G[f"qz_{k}_y"] = ref.quantize_row_q8_0(x)

    # dequantize_row -----------------------------------------------------
    for t, n in [(8, 256), (12, 512), (13, 512), (14, 512)]:
        src = synth.matrix(rng, t, 1, n)[0]
        G[f"dq_{t}_src"] = src
        G[f"dq_{t}_out"] = ref.dequantize_row(src, t, n)
    # The reference's own unit-test blocks (tests/tests.c:72-123).
    b4 = np.zeros(144, np.uint8)
    b4[0:2] = np.array([ref.fp32_to_fp16(0.5)], np.uint16).view(np.uint8)
    b4[2:4] = np.array([ref.fp32_to_fp16(0.1)], np.uint16).view(np.uint8)
    b4[4:16] = 1
    b4[16:] = 0x21
    b5 = np.zeros(176, np.uint8)
    b5[0:2] = np.array([ref.fp32_to_fp16(0.25)], np.uint16).view(np.uint8)
    b5[2:4] = np.array([ref.fp32_to_fp16(0.05)], np.uint16).view(np.uint8)
    b5[4:16] = 1
    b5[16:48] = 0x01
    b5[48:] = 0x43
    b6 = np.zeros(210, np.uint8)
    b6[192:200] = 1
    b6[208:210] = np.array([ref.fp32_to_fp16(0.5)], np.uint16).view(np.uint8)
    b6[:128] = 0x55
    for name, t, b in [("unit12", 12, b4), ("unit13", 13, b5), ("unit14", 14, b6)]:
        G[f"dq_{name}_src"] = b
        G[f"dq_{name}_out"] = ref.dequantize_row(b, t, 256)

    # vec_dot ------------------------------------------------------------
    for t, k in [(8, 2048), (13, 2048), (14, 1408), (12, 896)]:
        a = synth.matrix(rng, t, 1, k)[0]
        x = rng.standard_normal(k).astype(np.float32)
        b = ref.quantize_row_q8_0(x)
        G[f"vd_{t}_a"], G[f"vd_{t}_b"], G[f"vd_{t}_k"] = a, b, np.int32(k)
        key = "vd_q4k_ref_broken" if t == 12 else f"vd_{t}_out"
        G[key] = np.float32(ref.vec_dot(t, a, b, k))
    # tests/tests.c:125-140 and :284-307 inputs, through the Q8_0 dot.
    a_in = np.arange(32, dtype=np.float32) * np.float32(0.1)
    b_in = (32 - np.arange(32, dtype=np.float32)) * np.float32(0.1)
    G["vd_unit_a"], G["vd_unit_b"] = ref.quantize_row_q8_0(a_in), ref.quantize_row_q8_0(b_in)
    G["vd_unit_out"] = np.float32(ref.vec_dot(8, G["vd_unit_a"], G["vd_unit_b"], 32))

    # matmul_q_fused -----------------------------------------------------
    for name, t, n, d in [("q8_0", 8, 96, 2048), ("q8_0_tail", 8, 17, 100), ("q5k", 13, 48, 2048),
                          ("q6k", 14, 40, 1408), ("q6k_wide", 14, 8, 5632), ("q5k_tail", 13, 9, 1400)]:
        w = synth.matrix(rng, t, n, d)
        x = rng.standard_normal(d).astype(np.float32)
        G[f"mm_{name}_w"], G[f"mm_{name}_x"] = w, x
        G[f"mm_{name}_shape"] = np.array([t, n, d], np.int32)
        G[f"mm_{name}_out"] = ref.matmul_q_fused(x, w, t, n, d)
    wf = rng.standard_normal((16, 300)).astype(np.float32)
    xf = rng.standard_normal(300).astype(np.float32)
    G["mm_f32_w"], G["mm_f32_x"] = wf.view(np.uint8).reshape(16, -1), xf
    G["mm_f32_shape"] = np.array([0, 16, 300], np.int32)
    G["mm_f32_out"] = ref.matmul_q_fused(xf, wf, 0, 16, 300)

    # KernelOps softmax / matmul_ref (reference src/kernels.c), own seed so the
    # arrays above do not move --------------------------------------------
    r2 = synth.rng_for(20261202)
    sm = {
        "e60": r2.standard_normal(60, dtype=np.float32),
        "e128w": (r2.standard_normal(128, dtype=np.float32) * np.float32(8.0)).astype(np.float32),
        "ties": np.full(12, 0.5, np.float32),
        "e256": (r2.uniform(-90, 20, 256)).astype(np.float32),
        "one": np.array([3.25], np.float32),
    }
    for key, v in sm.items():
        G[f"sm_{key}_in"] = v
        G[f"sm_{key}_out"] = ref.softmax(v)
    wr = (r2.standard_normal((24, 300), dtype=np.float32) * np.float32(0.05)).astype(np.float32)
    xr = r2.standard_normal(300, dtype=np.float32)
    G["mr_w"], G["mr_x"] = wr, xr
    G["mr_out"] = ref.matmul_f32(xr, wr, 24, 300, backend=0)

    np.savez_compressed(OUT, **G)
    print(f"wrote {OUT}: {os.path.getsize(OUT)} bytes, {len(G)} arrays")


if __name__ == "__main__":
    main()
