"""GPU: programs of 2..64-token GEMVs, which run on the tensor cores
(tcgen05.mma kind::i8 per 32-element unit, exact terms and running sums from
TMEM), against the oracle.  Bit-identical to the reference's scalar build, like
every other path (the north-star tolerance 1e-5 rel / 1e-6 abs is asserted too).
"""
import numpy as np
import pytest

import synth

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

Q8_0, Q4_K, Q5_K, Q6_K = 8, 12, 13, 14
RTOL, ATOL = 1e-5, 1e-6


def assert_bit_exact(got, want):
    got = np.asarray(got, np.float32)
    want = np.asarray(want, np.float32)
    assert got.shape == want.shape
    bad = np.flatnonzero(got.view(np.uint32).ravel() != want.view(np.uint32).ravel())
    assert bad.size == 0, f"{bad.size} mismatches, first at {bad[:5]}"
    assert np.all(np.abs(got - want) <= ATOL + RTOL * np.abs(want))


def build(qr, specs, seed, share_x=False):
    rng = synth.rng_for(seed)
    jobs, keep, host, shared = [], [], [], {}
    for type_, n, d, B in specs:
        w = synth.matrix(rng, type_, n, d)
        if share_x and (d, B) in shared:
            x, xd = shared[(d, B)]
        else:
            x = synth.activations(rng, B, d)
            xd = torch.from_numpy(x).cuda()
            shared[(d, B)] = (x, xd)
        wd = torch.from_numpy(np.ascontiguousarray(w)).cuda()
        out = torch.full((B, n), float("nan"), device="cuda")
        keep += [wd, xd, out]
        host.append((w, x, type_, n, d, out))
        jobs.append((wd.data_ptr(), type_, n, d, B, xd.data_ptr(), d, out.data_ptr(), n))
    return qr.Program(jobs), host, keep


def check(orc, host):
    for w, x, type_, n, d, out in host:
        assert_bit_exact(out.cpu().numpy(), orc.matmul_q_fused_batch(x, w, type_, n, d))


def run(prog):
    prog.run(torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()


@pytest.mark.parametrize("type_,n,d", [(Q4_K, 257, 2048), (Q5_K, 130, 2048), (Q6_K, 200, 1408), (Q8_0, 129, 288),
                                       (Q8_0, 300, 2048), (Q6_K, 64, 256)])
@pytest.mark.parametrize("B", [2, 3, 4, 5, 9, 16, 33, 64])
def test_tc_types_and_batches(qr_gpu, orc, type_, n, d, B):
    """Ragged row tiles (n not a multiple of 128), Q6_K/Q8_0 rows that are
    not 16-byte aligned, a partial last stage (Q8_0 d=288: 9 blocks)."""
    prog, host, keep = build(qr_gpu, [(type_, n, d, B)], 100 + B)
    run(prog)
    check(orc, host)
    assert qr_gpu.device_status() == 0


def test_tc_c2_ffn_batch16(qr_gpu, orc):
    """Two layers of the c2 FFN (gate/up 4864x896, down 896x4864, Q4_K) at 16
    tokens, inputs shared by gate and up."""
    specs = [(Q4_K, 4864, 896, 16), (Q4_K, 4864, 896, 16), (Q4_K, 896, 4864, 16)] * 2
    prog, host, keep = build(qr_gpu, specs, 7, share_x=True)
    run(prog)
    check(orc, host)


def test_tc_and_engine_in_one_program(qr_gpu, orc):
    specs = [(Q4_K, 1000, 2048, 1), (Q5_K, 700, 2048, 4), (Q6_K, 512, 2048, 16), (Q8_0, 333, 4096, 40),
             (Q4_K, 896, 4864, 12), (Q5_K, 256, 2048, 8)]
    prog, host, keep = build(qr_gpu, specs, 8)
    run(prog)
    check(orc, host)
    info = prog.info()
    assert info["items"] > 0 and info["grid"] > 0


def test_tc_rerun_new_inputs_and_graph(qr_gpu, orc):
    specs = [(Q4_K, 384, 1024, 16), (Q6_K, 256, 1024, 24)]
    prog, host, keep = build(qr_gpu, specs, 9)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        prog.run(s.cuda_stream)
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            prog.run(s.cuda_stream)
    rng = synth.rng_for(99)
    new = []
    for k, (w, x, type_, n, d, out) in enumerate(host):
        x2 = synth.activations(rng, x.shape[0], d)
        keep[3 * k + 1].copy_(torch.from_numpy(x2))
        out.fill_(float("nan"))
        new.append((w, x2, type_, n, d, out))
    g.replay()
    torch.cuda.synchronize()
    check(orc, new)
    del g


@pytest.mark.parametrize("B", [2, 3, 4])
def test_tc_small_batches_strided_x(qr_gpu, orc, B):
    """Few-token jobs on the tensor cores with rows of x that are not 16-byte
    aligned (ldx = d + 1: the quantizer's scalar loads), and jobs of different
    token counts (and epilogue widths) sharing one launch."""
    rng = synth.rng_for(300 + B)
    specs = [(Q4_K, 300, 1024, B), (Q6_K, 130, 512, 1 + (B % 2)), (Q8_0, 200, 320, B), (Q5_K, 64, 256, 2)]
    jobs, keep, host = [], [], []
    for type_, n, d, b in specs:
        w = synth.matrix(rng, type_, n, d)
        x = synth.activations(rng, b, d)
        xs = np.zeros((b, d + 1), np.float32)
        xs[:, :d] = x
        xd = torch.from_numpy(xs).cuda()
        wd = torch.from_numpy(np.ascontiguousarray(w)).cuda()
        out = torch.full((b, n), float("nan"), device="cuda")
        keep += [wd, xd, out]
        host.append((w, x, type_, n, d, out))
        jobs.append((wd.data_ptr(), type_, n, d, b, xd.data_ptr(), d + 1, out.data_ptr(), n))
    prog = qr_gpu.Program(jobs)
    run(prog)
    check(orc, host)
    assert qr_gpu.device_status() == 0


@pytest.mark.parametrize("type_,B", [(Q4_K, 150), (Q6_K, 65), (Q8_0, 128)])
def test_tc_wide_jobs_as_slices(qr_gpu, orc, type_, B):
    """A job wider than 64 tokens (a prefill chunk) runs as 64-token slices of
    the same weights; every token's outputs are the reference's."""
    prog, host, keep = build(qr_gpu, [(type_, 200, 512, B), (Q4_K, 128, 256, 3)], 200 + B)
    run(prog)
    check(orc, host)
    assert qr_gpu.device_status() == 0
