"""GPU parity: the CUDA path (through the C ABI) against the reference.

Bar: bit-exact.  Quantized activations and int32 unit partials are integer
data; the fp32 outputs are also required to be bit-identical to the
reference's scalar build (the kernels reproduce its operation order), which is
stronger than the north-star tolerance of 1e-5 relative / 1e-6 absolute that
`assert_close_ns` additionally checks.
"""
import ctypes
import zlib

import numpy as np
import pytest

import synth

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-5, 1e-6  # north-star tolerance (accumulation-order allowance)


def bits(a):
    return np.asarray(a, dtype=np.float32).view(np.uint32)


def assert_bit_exact(got, want):
    got = np.asarray(got, np.float32)
    want = np.asarray(want, np.float32)
    assert got.shape == want.shape
    bad = np.flatnonzero(bits(got).ravel() != bits(want).ravel())
    assert bad.size == 0, f"{bad.size} mismatches, first at {bad[:5]}: {got.ravel()[bad[:5]]} vs {want.ravel()[bad[:5]]}"
    assert np.all(np.abs(got - want) <= ATOL + RTOL * np.abs(want))


# ------------------------------------------------ golden fixtures (Part 1) --

@pytest.mark.parametrize("case", ["ramp", "sin", "cos", "randn", "tail100", "zeros", "tiny", "huge",
                                  "halves", "nonfinite"])
def test_quantize_row_q8_0_golden(qr_gpu, golden, case):
    got = qr_gpu.quantize_row_q8_0(golden[f"qz_{case}_x"])
    assert np.array_equal(got, golden[f"qz_{case}_y"])


@pytest.mark.parametrize("key,type_,n", [("8", 8, 256), ("12", 12, 512), ("13", 13, 512), ("14", 14, 512),
                                         ("unit12", 12, 256), ("unit13", 13, 256), ("unit14", 14, 256)])
def test_dequantize_row_golden(qr_gpu, golden, key, type_, n):
    assert_bit_exact(qr_gpu.dequantize_row(golden[f"dq_{key}_src"], type_, n), golden[f"dq_{key}_out"])


@pytest.mark.parametrize("type_", [8, 13, 14])
def test_vec_dot_golden(qr_gpu, golden, type_):
    got = qr_gpu.vec_dot(type_, golden[f"vd_{type_}_a"], golden[f"vd_{type_}_b"], int(golden[f"vd_{type_}_k"]))
    assert_bit_exact(np.array([got]), np.array([golden[f"vd_{type_}_out"]]))


def test_vec_dot_q4k_restated(qr_gpu, golden, orc):
    a, b, k = golden["vd_12_a"], golden["vd_12_b"], int(golden["vd_12_k"])
    assert_bit_exact(np.array([qr_gpu.vec_dot(12, a, b, k)]), np.array([orc.vec_dot(12, a, b, k)]))


def test_vec_dot_unit_gate(qr_gpu, golden):  # tests/tests.c:125-140 inputs
    got = qr_gpu.vec_dot(8, golden["vd_unit_a"], golden["vd_unit_b"], 32)
    assert_bit_exact(np.array([got]), np.array([golden["vd_unit_out"]]))


@pytest.mark.parametrize("name", ["q8_0", "q8_0_tail", "q5k", "q6k", "q6k_wide", "q5k_tail", "f32"])
def test_matmul_q_fused_golden(qr_gpu, golden, name):
    t, n, d = (int(v) for v in golden[f"mm_{name}_shape"])
    got = qr_gpu.matmul_q_fused(golden[f"mm_{name}_x"], golden[f"mm_{name}_w"], t, n, d)
    assert_bit_exact(got, golden[f"mm_{name}_out"])


# ------------------------------------- BASELINE shapes against the oracle --

CONFIG_SHAPES = [
    ("c1_q8_0", 8, 5632, 2048),
    ("c2_gate_up_q4k", 12, 4864, 896),
    ("c2_down_q4k", 12, 896, 4864),
    ("c4_expert_gate_up_q5k", 13, 1408, 2048),
    ("c4_expert_down_q6k", 14, 2048, 1408),
    ("c4_shared_gate_up_q5k", 13, 5632, 2048),
    ("c4_shared_down_q6k", 14, 2048, 5632),
    ("c3_head_q6k", 14, 32000, 2048),
    ("c5_expert_down_q4k", 12, 2048, 768),
]


@pytest.mark.parametrize("name,type_,n,d", CONFIG_SHAPES)
def test_config_shapes_b1(qr_gpu, orc, name, type_, n, d):
    rng = synth.rng_for(zlib.crc32(name.encode()))
    w = synth.matrix(rng, type_, n, d)
    x = synth.activations(rng, 1, d)[0]
    assert_bit_exact(qr_gpu.matmul_q_fused(x, w, type_, n, d), orc.matmul_q_fused(x, w, type_, n, d))


@pytest.mark.parametrize("B", [1, 2, 3, 4, 5, 8, 16, 17])
@pytest.mark.parametrize("type_,n,d", [(12, 4864, 896), (12, 896, 4864), (8, 512, 2048), (13, 300, 2048),
                                       (14, 300, 1408)])
def test_batched(qr_gpu, orc, B, type_, n, d):
    rng = synth.rng_for(B * 7919 + n)
    w = synth.matrix(rng, type_, n, d)
    x = synth.activations(rng, B, d)
    assert_bit_exact(qr_gpu.matmul_q_fused_batch(x, w, type_, n, d), orc.matmul_q_fused_batch(x, w, type_, n, d))


def test_registered_weights_path(qr_gpu, orc):
    rng = synth.rng_for(31)
    w = synth.matrix(rng, 12, 4864, 896)
    x = synth.activations(rng, 1, 896)[0]
    want = orc.matmul_q_fused(x, w, 12, 4864, 896)
    qr_gpu.register_weights(w)
    try:
        assert qr_gpu.lib().quantr_gpu_device_ptr(w.ctypes.data_as(ctypes.c_void_p)) is not None
        assert_bit_exact(qr_gpu.matmul_q_fused(x, w, 12, 4864, 896), want)
        # A sub-range (like one expert's slice of a stacked tensor) resolves too.
        sub = w[1000:2000]
        assert_bit_exact(qr_gpu.matmul_q_fused(x, sub, 12, 1000, 896), want[1000:2000])
    finally:
        qr_gpu.unregister_weights(w)


# ------------------------------------------------------------- edge cases --

def test_null_weights_zero_output(qr_gpu):
    out = qr_gpu.matmul_q_fused(np.ones(64, np.float32), None, 8, 7, 64)
    assert np.array_equal(out, np.zeros(7, np.float32))


def test_fewer_columns_than_a_block(qr_gpu, orc):
    rng = synth.rng_for(3)
    x = synth.activations(rng, 1, 200)[0]
    w = np.zeros(16, np.uint8)  # row_bytes(Q4_K, 200) == 0
    assert_bit_exact(qr_gpu.matmul_q_fused(x, w, 12, 4, 200), orc.matmul_q_fused(x, w, 12, 4, 200))


def test_unsupported_type_zeros_and_error(qr_gpu):
    L = qr_gpu.lib()
    x = np.ones(64, np.float32)
    w = np.ones(64 * 4 * 3, np.uint8)
    out = np.full(3, 7.0, np.float32)
    L.matmul_q_fused(out.ctypes.data_as(ctypes.c_void_p), x.ctypes.data_as(ctypes.c_void_p),
                     w.ctypes.data_as(ctypes.c_void_p), 2, 3, 64, 1)
    assert L.quantr_gpu_last_error() == 4
    L.quantr_gpu_clear_error()
    assert np.array_equal(out, np.zeros(3, np.float32))


@pytest.mark.parametrize("type_,n,d", [(8, 1, 32), (8, 3, 64), (12, 1, 256), (13, 2, 256), (14, 1, 256),
                                       (14, 5, 257), (8, 9, 31), (12, 6, 511)])
def test_small_and_ragged(qr_gpu, orc, type_, n, d):
    rng = synth.rng_for(n * 1000 + d)
    w = synth.matrix(rng, type_, n, d) if d >= synth.BLOCK_ELEMS[type_] else np.zeros((n, 1), np.uint8)
    x = synth.activations(rng, 1, d)[0]
    assert_bit_exact(qr_gpu.matmul_q_fused(x, w, type_, n, d), orc.matmul_q_fused(x, w, type_, n, d))


# ----------------------------------------------------- device API (torch) --

torch = pytest.importorskip("torch")


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("type_,n,d", [(8, 700, 2048), (12, 333, 896), (13, 128, 2048), (14, 97, 1408)])
def test_unit_partials_bit_exact(qr_gpu, orc, type_, n, d):
    rng = synth.rng_for(type_ * 31 + n)
    w = synth.matrix(rng, type_, n, d)
    x = synth.activations(rng, 1, d)[0]
    U = d // 32 if type_ == 8 else 8 * (d // 256)
    wd, xd = _dev(w), _dev(x)
    out = torch.empty(n, device="cuda")
    isum = torch.empty(n * U, dtype=torch.int32, device="cuda")
    bsum = torch.empty(n * U, dtype=torch.int32, device="cuda")
    ws = torch.empty(qr_gpu.workspace_bytes(d, 1), dtype=torch.uint8, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    qr_gpu.gemv_partials_dev(out.data_ptr(), isum.data_ptr(), bsum.data_ptr(), xd.data_ptr(), wd.data_ptr(),
                             type_, n, d, 1, ws.data_ptr(), ws.numel(), s)
    torch.cuda.synchronize()
    wi, wb = orc.unit_partials(w, type_, n, d, orc.quantize_row_q8_0(x))
    assert np.array_equal(isum.cpu().numpy().reshape(n, U), wi)
    assert np.array_equal(bsum.cpu().numpy().reshape(n, U), wb)
    assert_bit_exact(out.cpu().numpy(), orc.matmul_q_fused(x, w, type_, n, d))


@pytest.mark.parametrize("offset", [1, 2, 3, 7, 15])
@pytest.mark.parametrize("type_", [8, 12, 14])
def test_unaligned_weight_pointer(qr_gpu, orc, offset, type_):
    """Rows at any byte alignment (e.g. a tensor inside a GGUF mapping)."""
    n, d = 77, 1024
    rng = synth.rng_for(offset + type_)
    w = synth.matrix(rng, type_, n, d)
    x = synth.activations(rng, 2, d)
    buf = torch.zeros(w.nbytes + 64, dtype=torch.uint8, device="cuda")
    buf[offset:offset + w.nbytes] = _dev(w.ravel())
    xd = _dev(x)
    out = torch.empty(2, n, device="cuda")
    ws = torch.empty(qr_gpu.workspace_bytes(d, 2), dtype=torch.uint8, device="cuda")
    qr_gpu.gemv_dev(out.data_ptr(), n, xd.data_ptr(), d, buf.data_ptr() + offset, type_, n, d, 2, ws.data_ptr(),
                    ws.numel(), torch.cuda.current_stream().cuda_stream)
    assert_bit_exact(out.cpu().numpy(), orc.matmul_q_fused_batch(x, w, type_, n, d))


def test_strided_io_and_stream(qr_gpu, orc):
    n, d, B = 300, 2048, 3
    rng = synth.rng_for(99)
    w = synth.matrix(rng, 13, n, d)
    x = synth.activations(rng, B, d)
    xpad = np.zeros((B, d + 96), np.float32)
    xpad[:, :d] = x
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        wd, xd = _dev(w), _dev(xpad)
        out = torch.full((B, n + 5), -1.0, device="cuda")
        ws = torch.empty(qr_gpu.workspace_bytes(d, B), dtype=torch.uint8, device="cuda")
        qr_gpu.gemv_dev(out.data_ptr(), n + 5, xd.data_ptr(), d + 96, wd.data_ptr(), 13, n, d, B, ws.data_ptr(),
                        ws.numel(), s.cuda_stream)
    s.synchronize()
    o = out.cpu().numpy()
    assert_bit_exact(o[:, :n], orc.matmul_q_fused_batch(x, w, 13, n, d))
    assert np.all(o[:, n:] == -1.0)


def test_q8act_device_api(qr_gpu, orc):
    n, d = 64, 2048
    rng = synth.rng_for(5)
    w = synth.matrix(rng, 14, n, d)
    x = synth.activations(rng, 2, d)
    xq = np.stack([orc.quantize_row_q8_0(x[t]) for t in range(2)])
    wd, xqd = _dev(w), _dev(xq)
    out = torch.empty(2, n, device="cuda")
    ws = torch.empty(qr_gpu.workspace_bytes(d, 2), dtype=torch.uint8, device="cuda")
    qr_gpu.gemv_q8act_dev(out.data_ptr(), n, xqd.data_ptr(), wd.data_ptr(), 14, n, d, 2, ws.data_ptr(), ws.numel(),
                          torch.cuda.current_stream().cuda_stream)
    assert_bit_exact(out.cpu().numpy(), orc.matmul_q_fused_batch(x, w, 14, n, d))


def test_quantize_dev_matches_reference_blocks(qr_gpu, orc):
    B, k = 5, 4864
    rng = synth.rng_for(8)
    x = synth.activations(rng, B, k) * np.float32(3.0)
    xd = _dev(x)
    y = torch.zeros(B * (k // 32) * 34, dtype=torch.uint8, device="cuda")
    qr_gpu.quantize_q8_0_dev(y.data_ptr(), xd.data_ptr(), k, k, B, torch.cuda.current_stream().cuda_stream)
    want = np.concatenate([orc.quantize_row_q8_0(x[t]) for t in range(B)])
    assert np.array_equal(y.cpu().numpy(), want)


def test_chained_gemvs_with_pdl(qr_gpu, orc):
    """Back-to-back dependent GEMVs on one stream (programmatic dependent
    launch): each consumes the previous output; equals the sequential oracle."""
    rng = synth.rng_for(2024)
    shapes = [(12, 4864, 896), (12, 896, 4864), (14, 2048, 896), (8, 896, 2048)]
    ws_bytes = max(qr_gpu.workspace_bytes(d, 1) for _, _, d in shapes)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    x = synth.activations(rng, 1, 896)[0]
    ws_ = [synth.matrix(rng, t, n, d) for t, n, d in shapes]
    cur = _dev(x)
    s = torch.cuda.current_stream().cuda_stream
    want = x
    for (t, n, d), w in zip(shapes, ws_):
        out = torch.empty(n, device="cuda")
        qr_gpu.gemv_dev(out.data_ptr(), n, cur.data_ptr(), d, _dev(w).data_ptr(), t, n, d, 1, ws.data_ptr(),
                        ws_bytes, s)
        cur = out
        want = orc.matmul_q_fused(want, w, t, n, d)
    assert_bit_exact(cur.cpu().numpy(), want)
    assert qr_gpu.device_status(s) == 0


def test_batch_independence_and_determinism_full_size(qr_gpu):
    """Size-independent properties at the c2 down shape: a batch equals its
    single-token calls, rows permute with W, repeated runs are identical."""
    t, n, d = 12, 896, 4864
    rng = synth.rng_for(4242)
    w = synth.matrix(rng, t, n, d)
    x = synth.activations(rng, 16, d)
    batch = qr_gpu.matmul_q_fused_batch(x, w, t, n, d)
    for i in (0, 7, 15):
        assert np.array_equal(bits(batch[i]), bits(qr_gpu.matmul_q_fused(x[i], w, t, n, d)))
    perm = rng.permutation(n)
    pb = qr_gpu.matmul_q_fused_batch(x, w[perm], t, n, d)
    assert np.array_equal(bits(pb), bits(batch[:, perm]))
    assert np.array_equal(bits(qr_gpu.matmul_q_fused_batch(x, w, t, n, d)), bits(batch))


def test_launch_counter_moves(qr_gpu):
    before = qr_gpu.launch_count()
    qr_gpu.matmul_q_fused(np.ones(256, np.float32), np.zeros((4, 144), np.uint8), 12, 4, 256)
    assert qr_gpu.launch_count() >= before + 2  # quantizer + GEMV


@pytest.mark.parametrize("n,d,B,ldx_pad,xoff", [(128, 2048, 64, 0, 0), (1, 2048, 64, 0, 0), (60, 2048, 1, 0, 0),
                                                (200, 2048, 1, 0, 0), (37, 1001, 5, 3, 1), (130, 333, 7, 0, 2),
                                                (64, 64, 3, 4, 0)])
def test_f32_gemv_shapes(qr_gpu, orc, n, d, B, ldx_pad, xoff):
    """F32 weights (routers, the shared-expert gate): the reference's
    matmul_ref order per (row, token), bit for bit, for aligned rows (16-byte
    copies), odd widths and misaligned or padded activations (plain loads)."""
    rng = synth.rng_for(n * 131 + d + B)
    w = (rng.standard_normal((n, d), dtype=np.float32) * np.float32(0.05)).astype(np.float32)
    x = synth.activations(rng, B, d)
    ldx = d + ldx_pad
    xbuf = np.zeros(xoff + B * ldx, np.float32)
    for t in range(B):
        xbuf[xoff + t * ldx:xoff + t * ldx + d] = x[t]
    wd, xd = _dev(w), _dev(xbuf)
    out = torch.full((B, n), float("nan"), device="cuda")
    ws = torch.empty(max(256, qr_gpu.workspace_bytes(d, B)), dtype=torch.uint8, device="cuda")
    qr_gpu.gemv_dev(out.data_ptr(), n, xd.data_ptr() + 4 * xoff, ldx, wd.data_ptr(), 0, n, d, B, ws.data_ptr(),
                    ws.numel(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    want = np.stack([orc.matmul_f32(x[t], w, n, d) for t in range(B)])
    assert_bit_exact(out.cpu().numpy(), want)
