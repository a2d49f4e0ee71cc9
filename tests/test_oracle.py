"""CPU: the C restatement (oracle/quant_oracle.c) against the reference.

Pins: (1) the golden fixture, produced by the reference's own src/quant.c
(tests/golden/make_golden.py); (2) the reference's unit-test gates
(tests/tests.c) restated; (3) live comparison with oracle/_ref when built.
Every comparison of integer/byte data and of scalar-build fp32 outputs is bit
for bit.
"""
import numpy as np
import pytest

import oracle
import synth


def bits(a):
    return np.asarray(a, dtype=np.float32).view(np.uint32)


def test_fp16_to_fp32_exhaustive(golden, orc):
    got = np.array([orc.fp16_to_fp32(h) for h in range(65536)], dtype=np.float32)
    assert np.array_equal(bits(got), bits(golden["fp16_all"]))


def test_fp32_to_fp16_cases(golden, orc):
    got = np.array([orc.fp32_to_fp16(v) for v in golden["f2h_in"]], dtype=np.uint16)
    assert np.array_equal(got, golden["f2h_out"])
    # The vectorised generator helper is the same recipe.
    assert np.array_equal(synth.fp32_to_fp16_trunc(golden["f2h_in"]), golden["f2h_out"])


@pytest.mark.parametrize("case", ["ramp", "sin", "cos", "randn", "tail100", "zeros", "tiny", "huge",
                                  "halves", "nonfinite"])
def test_quantize_row_q8_0(golden, orc, case):
    x = golden[f"qz_{case}_x"]
    assert np.array_equal(orc.quantize_row_q8_0(x), golden[f"qz_{case}_y"])


@pytest.mark.parametrize("key,type_,n", [("8", 8, 256), ("12", 12, 512), ("13", 13, 512), ("14", 14, 512),
                                         ("unit12", 12, 256), ("unit13", 13, 256), ("unit14", 14, 256)])
def test_dequantize_row(golden, orc, key, type_, n):
    got = orc.dequantize_row(golden[f"dq_{key}_src"], type_, n)
    assert np.array_equal(bits(got), bits(golden[f"dq_{key}_out"]))


@pytest.mark.parametrize("type_", [8, 13, 14])
def test_vec_dot(golden, orc, type_):
    got = orc.vec_dot(type_, golden[f"vd_{type_}_a"], golden[f"vd_{type_}_b"], int(golden[f"vd_{type_}_k"]))
    assert bits(got) == bits(golden[f"vd_{type_}_out"])


def test_q4k_restatement_matches_dequantize_semantics(golden, orc):
    """Q4_K: the reference kernel is broken (fp16 fields read as integers,
    src/quant.c:302-303); the restatement must equal the dot product that the
    reference's dequantize_row defines, up to fp32 rounding."""
    a, b, k = golden["vd_12_a"], golden["vd_12_b"], int(golden["vd_12_k"])
    got = float(orc.vec_dot(12, a, b, k))
    w = orc.dequantize_row(a, 12, k).astype(np.float64)
    x = orc.dequantize_row(b, 8, k).astype(np.float64)
    exact = float(w[: (k // 256) * 256] @ x[: (k // 256) * 256])
    assert abs(got - exact) <= 1e-5 * abs(exact) + 1e-6
    # ...and is nothing like what the broken reference function returns.
    assert abs(float(golden["vd_q4k_ref_broken"]) - exact) > 1e3 * abs(exact)


@pytest.mark.parametrize("name", ["q8_0", "q8_0_tail", "q5k", "q6k", "q6k_wide", "q5k_tail", "f32"])
def test_matmul_q_fused(golden, orc, name):
    t, n, d = (int(v) for v in golden[f"mm_{name}_shape"])
    w = golden[f"mm_{name}_w"]
    got = orc.matmul_q_fused(golden[f"mm_{name}_x"], w, t, n, d)
    assert np.array_equal(bits(got), bits(golden[f"mm_{name}_out"]))


def test_matmul_null_weights_give_zeros(orc):
    x = np.ones(64, np.float32)
    assert np.array_equal(orc.matmul_q_fused(x, None, 8, 5, 64), np.zeros(5, np.float32))


# --- the reference's own unit-test gates (tests/tests.c), on the restatement --

def test_gate_fp16_conversion(orc):  # tests/tests.c:42-52
    for v in [0.0, 1.0, -1.0, 3.14159, 0.0001]:
        f = orc.fp16_to_fp32(orc.fp32_to_fp16(v))
        assert abs(v - f) <= abs(v) * 0.01 + 1e-4


def test_gate_q8_0_round_trip(orc):  # tests/tests.c:54-70
    x = (np.arange(32, dtype=np.float32) - 16.0) * np.float32(0.125)
    y = orc.dequantize_row(orc.quantize_row_q8_0(x), 8, 32)
    assert np.max(np.abs(x - y)) < 0.05


def test_gate_vec_dot_q8_0(orc):  # tests/tests.c:125-140
    a_in = np.arange(32, dtype=np.float32) * np.float32(0.1)
    b_in = (32 - np.arange(32, dtype=np.float32)) * np.float32(0.1)
    ref = float(np.sum(a_in * b_in, dtype=np.float32))
    got = float(orc.vec_dot(8, orc.quantize_row_q8_0(a_in), orc.quantize_row_q8_0(b_in), 32))
    assert abs(ref - got) < ref * 0.05


def test_gate_kv_cache_parity(orc):  # tests/tests.c:284-307
    i = np.arange(256, dtype=np.float32)
    k = np.sin(i * np.float32(0.05)).astype(np.float32)
    q = np.cos(i * np.float32(0.03)).astype(np.float32)
    dot = float(np.sum(k * q, dtype=np.float32))
    got = float(orc.vec_dot(8, orc.quantize_row_q8_0(k), orc.quantize_row_q8_0(q), 256))
    assert abs(dot - got) / (abs(dot) + 1e-6) < 0.02


@pytest.mark.parametrize("key,type_", [("unit12", 12), ("unit13", 13), ("unit14", 14)])
def test_gate_kquant_dequant_finite(golden, orc, key, type_):  # tests/tests.c:72-123
    assert np.all(np.isfinite(orc.dequantize_row(golden[f"dq_{key}_src"], type_, 256)))


# --- live comparison with the compiled reference, where it was built -------

@pytest.mark.skipif(not oracle.ref_available("scalar"), reason="oracle/_ref not built")
@pytest.mark.parametrize("type_,n,d", [(8, 33, 2048), (8, 7, 1000), (13, 21, 2048), (13, 5, 1408),
                                       (14, 19, 1408), (14, 3, 5632)])
def test_live_reference_scalar(orc, type_, n, d):
    ref = oracle.RefLib("scalar")
    rng = synth.rng_for(1000 + type_ * 100 + n)
    w = synth.matrix(rng, type_, n, d)
    x = synth.activations(rng, 1, d)[0]
    assert np.array_equal(bits(orc.matmul_q_fused(x, w, type_, n, d)), bits(ref.matmul_q_fused(x, w, type_, n, d)))


@pytest.mark.skipif(not oracle.ref_available("avx2"), reason="oracle/_ref not built")
def test_avx2_build_within_tolerance(orc):
    """The reference's AVX2 build sums Q8_0 in 8 lanes: different order, same
    values within the north-star tolerance (1e-5 rel / 1e-6 abs)."""
    ref = oracle.RefLib("avx2")
    rng = synth.rng_for(77)
    w = synth.matrix(rng, 8, 64, 2048)
    x = synth.activations(rng, 1, 2048)[0]
    a = orc.matmul_q_fused(x, w, 8, 64, 2048)
    b = ref.matmul_q_fused(x, w, 8, 64, 2048)
    assert np.all(np.abs(a - b) <= 1e-6 + 1e-5 * np.abs(b))


def test_unit_partials_reconstruct_dot(orc):
    """The per-unit int32 partials recombined in order give the row dot."""
    rng = synth.rng_for(5)
    for t, d in [(8, 512), (13, 512), (14, 512), (12, 512)]:
        w = synth.matrix(rng, t, 3, d)
        x = synth.activations(rng, 1, d)[0]
        xq = orc.quantize_row_q8_0(x)
        isum, bsum = orc.unit_partials(w, t, 3, d, xq)
        xd = np.array([orc.fp16_to_fp32(h) for h in xq.reshape(-1, 34)[:, :2].copy().view(np.uint16)[:, 0]])
        assert np.array_equal(bsum[0], xq.reshape(-1, 34)[:, 2:].view(np.int8).astype(np.int32).sum(1)[: isum.shape[1]])
        if t == 8:
            wd = np.array([orc.fp16_to_fp32(h) for h in w[0].reshape(-1, 34)[:, :2].copy().view(np.uint16)[:, 0]])
            acc = np.float32(0)
            for u in range(isum.shape[1]):
                acc = np.float32(acc + np.float32(np.float32(np.float32(isum[0, u]) * np.float32(wd[u])) * np.float32(xd[u])))
            assert bits(acc) == bits(orc.matmul_q_fused(x, w, t, 3, d)[0])


# ---- router pieces of the MoE block (src/runtime.c:202-229) ----

@pytest.mark.parametrize("key", ["e60", "e128w", "ties", "e256", "one"])
def test_softmax_golden(golden, orc, key):
    """qo_softmax against the reference's KernelOps softmax (src/kernels.c:191-207)."""
    got = orc.softmax(golden[f"sm_{key}_in"])
    np.testing.assert_array_equal(got.view(np.uint32), golden[f"sm_{key}_out"].view(np.uint32))


def test_matmul_ref_golden(golden, orc):
    """qo_matmul_f32 against KernelOps matmul_ref (src/kernels.c:18-28)."""
    got = orc.matmul_f32(golden["mr_x"], golden["mr_w"], 24, 300)
    np.testing.assert_array_equal(got.view(np.uint32), golden["mr_out"].view(np.uint32))


def _route(probs, k):
    """src/runtime.c:208-229 restated in Python on already-softmaxed probs."""
    p = probs.astype(np.float32).copy()
    sel, w = [], []
    for _ in range(k):
        best, arg = np.float32(-1e9), -1
        for e in range(p.size):
            if p[e] > best:
                best, arg = p[e], e
        sel.append(arg)
        w.append(best)
        p[arg] = np.float32(-1e9)
    tot = np.float32(0.0)
    for v in w:
        tot = np.float32(tot + v)
    return np.array(sel, np.int32), np.array([np.float32(v / tot) for v in w], np.float32)


@pytest.mark.parametrize("key,k", [("e60", 4), ("e128w", 8), ("ties", 4), ("e256", 16), ("one", 1)])
def test_moe_token_routing(golden, orc, key, k):
    """qo_moe_token's routing (softmax, strict arg-max top-k, renormalisation)
    against the reference softmax output plus a direct restatement; the expert
    weights are zero so the FFN part only has to run."""
    logits = golden[f"sm_{key}_in"]
    E = logits.size
    dim, hidden = 32, 32
    w = np.zeros((E, hidden, 34), np.uint8)  # Q8_0 rows of zeros
    w2 = np.zeros((E, dim, 34), np.uint8)
    xb = np.ones(dim, np.float32)
    out, sel, wts = orc.moe_token(xb, E, k, w, 8, hidden * 34, w, 8, hidden * 34, w2, 8, dim * 34, dim, hidden,
                                  logits=logits)
    want_sel, want_w = _route(golden[f"sm_{key}_out"], k)
    np.testing.assert_array_equal(sel, want_sel)
    np.testing.assert_array_equal(wts.view(np.uint32), want_w.view(np.uint32))
    assert np.all(out == 0.0)
    if key == "ties":
        assert list(sel) == [0, 1, 2, 3]


@pytest.mark.skipif(not oracle.ref_available("scalar"), reason="oracle/_ref not built")
def test_live_reference_softmax_and_matmul(orc):
    ref = oracle.RefLib("scalar")
    rng = np.random.Generator(np.random.PCG64(77))
    for E in (1, 7, 60, 128, 256):
        v = (rng.standard_normal(E) * 4).astype(np.float32)
        np.testing.assert_array_equal(orc.softmax(v).view(np.uint32), ref.softmax(v).view(np.uint32))
    w = rng.standard_normal((60, 2048)).astype(np.float32)
    x = rng.standard_normal(2048).astype(np.float32)
    np.testing.assert_array_equal(orc.matmul_f32(x, w, 60, 2048).view(np.uint32),
                                  ref.matmul_f32(x, w, 60, 2048, backend=0).view(np.uint32))
