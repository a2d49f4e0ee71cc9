"""GPU: the persistent GEMV engine (quantr_program_*) against the oracle.

Every job's output must be bit-identical to the reference's scalar build, as
for the single-GEMV entry points (north-star tolerance 1e-5 rel / 1e-6 abs is
asserted too).
"""
import numpy as np
import pytest

import synth

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-5, 1e-6
torch = pytest.importorskip("torch")


def bits(a):
    return np.asarray(a, dtype=np.float32).view(np.uint32)


def assert_bit_exact(got, want):
    got = np.asarray(got, np.float32)
    want = np.asarray(want, np.float32)
    assert got.shape == want.shape
    bad = np.flatnonzero(bits(got).ravel() != bits(want).ravel())
    assert bad.size == 0, f"{bad.size} mismatches, first at {bad[:5]}"
    assert np.all(np.abs(got - want) <= ATOL + RTOL * np.abs(want))


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def build_program(qr, specs, seed, share_x=False):
    """specs: list of (type, n, d, B).  Returns (program, host data, outputs)."""
    rng = synth.rng_for(seed)
    jobs, keep, host = [], [], []
    shared = {}
    for type_, n, d, B in specs:
        w = synth.matrix(rng, type_, n, d)
        if share_x and (d, B) in shared:
            x, xd = shared[(d, B)]
        else:
            x = synth.activations(rng, B, d)
            xd = _dev(x)
            shared[(d, B)] = (x, xd)
        wd = _dev(w)
        out = torch.full((B, n), float("nan"), device="cuda")
        keep += [wd, xd, out]
        host.append((w, x, type_, n, d))
        jobs.append((wd.data_ptr(), type_, n, d, B, xd.data_ptr(), d, out.data_ptr(), n))
    prog = qr.Program(jobs)
    return prog, host, keep


def check_outputs(orc, host, keep):
    outs = keep[2::3]
    for (w, x, type_, n, d), out in zip(host, outs):
        assert_bit_exact(out.cpu().numpy(), orc.matmul_q_fused_batch(x, w, type_, n, d))


def test_program_c2_ffn_layers(qr_gpu, orc):
    """Three layers of the c2 FFN shapes (Q4_K), batch 1."""
    specs = [(12, 4864, 896, 1), (12, 4864, 896, 1), (12, 896, 4864, 1)] * 3
    prog, host, keep = build_program(qr_gpu, specs, 1)
    prog.run(torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    check_outputs(orc, host, keep)
    assert qr_gpu.device_status() == 0
    info = prog.info()
    assert info["items"] >= info["grid"] > 0


def test_program_mixed_types_and_batches(qr_gpu, orc):
    specs = [(8, 1000, 2048, 1), (13, 1408, 2048, 2), (14, 2048, 1408, 3), (12, 896, 4864, 4),
             (14, 700, 2048, 1), (8, 333, 4096, 8), (13, 257, 2048, 16), (12, 2048, 768, 5)]
    prog, host, keep = build_program(qr_gpu, specs, 2)
    prog.run(torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    check_outputs(orc, host, keep)


def test_program_shared_inputs_dedupe(qr_gpu, orc):
    """Jobs reading one x with different weight types (different activation
    layouts) and with the same type (one quantization)."""
    specs = [(12, 512, 2048, 2), (13, 384, 2048, 2), (14, 256, 2048, 2), (8, 128, 2048, 2), (12, 64, 2048, 2)]
    prog, host, keep = build_program(qr_gpu, specs, 3, share_x=True)
    prog.run(torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    check_outputs(orc, host, keep)


@pytest.mark.parametrize("spec", [(8, 17, 100, 1), (14, 13, 1408, 2), (14, 5, 5632, 1), (8, 9, 3200, 3),
                                  (12, 1, 256, 1), (13, 3, 512, 7)])
def test_program_ragged_tiles(qr_gpu, orc, spec):
    """Row sizes that are not multiples of 16 bytes: the last tile carries a
    ragged tail copied without the bulk engine."""
    prog, host, keep = build_program(qr_gpu, [spec, spec], 4)
    prog.run(torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    check_outputs(orc, host, keep)


def test_program_split_over_launches(qr_gpu, orc):
    """More jobs than one launch keeps in its shared-memory job table: the
    program runs as several engine launches after one quantizer launch."""
    specs = [(12, 64, 512, 1), (14, 32, 512, 2), (8, 48, 256, 1), (13, 40, 512, 3)] * 52  # 208 jobs
    prog, host, keep = build_program(qr_gpu, specs, 9)
    prog.run(torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    check_outputs(orc, host, keep)


def test_program_single_job(qr_gpu, orc):
    prog, host, keep = build_program(qr_gpu, [(14, 2048, 5632, 1)], 10)
    prog.run(torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    check_outputs(orc, host, keep)


def test_program_rerun_sees_new_inputs(qr_gpu, orc):
    specs = [(12, 1024, 2048, 2), (14, 512, 2048, 1)]
    prog, host, keep = build_program(qr_gpu, specs, 5)
    s = torch.cuda.current_stream().cuda_stream
    prog.run(s)
    rng = synth.rng_for(55)
    new_host = []
    for k, (w, x, type_, n, d) in enumerate(host):
        x2 = synth.activations(rng, x.shape[0], d)
        keep[3 * k + 1].copy_(torch.from_numpy(x2))
        new_host.append((w, x2, type_, n, d))
    prog.run(s)
    torch.cuda.synchronize()
    check_outputs(orc, new_host, keep)


def test_program_in_cuda_graph(qr_gpu, orc):
    specs = [(12, 4864, 896, 1), (12, 896, 4864, 1)]
    prog, host, keep = build_program(qr_gpu, specs, 6)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        prog.run(s.cuda_stream)  # first run outside capture
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            prog.run(s.cuda_stream)
    for o in keep[2::3]:
        o.fill_(float("nan"))
    g.replay()
    torch.cuda.synchronize()
    check_outputs(orc, host, keep)
    del g


def test_program_rejects_bad_jobs(qr_gpu):
    import ctypes
    w = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    x = torch.zeros(256, device="cuda")
    o = torch.zeros(4, device="cuda")
    with pytest.raises(qr_gpu.QuantrError):  # misaligned weights
        qr_gpu.Program([(w.data_ptr() + 1, 12, 4, 256, 1, x.data_ptr(), 256, o.data_ptr(), 4)])
    with pytest.raises(qr_gpu.QuantrError):  # unsupported type
        qr_gpu.Program([(w.data_ptr(), 2, 4, 256, 1, x.data_ptr(), 256, o.data_ptr(), 4)])
    with pytest.raises(qr_gpu.QuantrError):  # no tokens
        qr_gpu.Program([(w.data_ptr(), 12, 4, 256, 0, x.data_ptr(), 256, o.data_ptr(), 4)])
    with pytest.raises(qr_gpu.QuantrError):  # output rows overlap (ldo < n), sliced wide job
        qr_gpu.Program([(w.data_ptr(), 12, 4, 256, 65, x.data_ptr(), 256, o.data_ptr(), 3)])
    with pytest.raises(qr_gpu.QuantrError):  # misaligned weights on the tensor-core path
        qr_gpu.Program([(w.data_ptr() + 1, 12, 4, 256, 16, x.data_ptr(), 256, o.data_ptr(), 4)])
    assert ctypes is not None


@pytest.mark.parametrize("type_,d", [(12, 512), (12, 768), (13, 512), (13, 768), (14, 1024), (8, 2048), (8, 288)])
def test_program_single_type_one_token(qr_gpu, orc, type_, d):
    """Programs whose one-token jobs share one weight type run the engine
    kernel built for that type (and, for Q4_K/Q5_K rows of an odd number of
    16-byte units - d = 768 - for the row-fastest order only; d = 512 gives an
    even number and the other order).  A second run sees new inputs."""
    specs = [(type_, 300, d, 1), (type_, 129, d, 1), (type_, 64, d, 1)]
    prog, host, keep = build_program(qr_gpu, specs, 40 + type_)
    prog.run(torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    check_outputs(orc, host, keep)
    rng = synth.rng_for(99)
    for k, (w, x, t, n, dd) in enumerate(host):
        x2 = synth.activations(rng, 1, dd)
        keep[3 * k + 1].copy_(torch.from_numpy(x2))
        host[k] = (w, x2, t, n, dd)
    prog.run(torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    check_outputs(orc, host, keep)
