"""GPU: the allocation-free GEMV entry point, quantr_gemv_noalloc_dev.

It exists for callers that cannot call cudaMalloc (an embedder's memory
manager owns all device memory, a plugin host passes only input and output
buffers, or the path cannot take cudaMalloc's implicit synchronisation).  It
must give the same results as the allocating entry point quantr_gemv_dev,
including on a second call that finds the previous call's data still in the
shared scratch array.  This file sorts last so that a run stopping at the first
failure has already run every other test; it also passes alone in a fresh
process.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-5, 1e-6  # the tolerance the other parity tests state


def test_noalloc_matches_allocating_entry_point_twice():
    import torch

    import quantr
    import synth

    L = quantr.lib()  # the C ABI, loaded directly
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream().cuda_stream
    # Two consecutive calls with different shapes and inputs: the second one
    # runs over whatever the first left in the scratch array.
    for call, (type_, n, d, B) in enumerate([(12, 896, 4864, 3), (14, 333, 1408, 2)]):
        rng = synth.rng_for(900 + call)
        w = torch.from_numpy(synth.matrix(rng, type_, n, d)).to(dev)
        x = torch.from_numpy(synth.activations(rng, B, d)).to(dev)
        got = torch.full((B, n), float("nan"), device=dev)
        want = torch.full((B, n), float("nan"), device=dev)
        rc = L.quantr_gemv_noalloc_dev(ctypes.c_void_p(got.data_ptr()), n, ctypes.c_void_p(x.data_ptr()), d,
                                       ctypes.c_void_p(w.data_ptr()), type_, n, d, B, ctypes.c_void_p(stream))
        assert rc == 0, f"quantr_gemv_noalloc_dev returned {rc}"
        ws = torch.empty(quantr.workspace_bytes(d, B), dtype=torch.uint8, device=dev)
        rc = L.quantr_gemv_dev(ctypes.c_void_p(want.data_ptr()), n, ctypes.c_void_p(x.data_ptr()), d,
                               ctypes.c_void_p(w.data_ptr()), type_, n, d, B, ctypes.c_void_p(ws.data_ptr()),
                               ws.numel(), ctypes.c_void_p(stream))
        assert rc == 0
        torch.cuda.synchronize()
        g, e = got.cpu().numpy(), want.cpu().numpy()
        assert np.all(np.isfinite(g))
        assert np.all(np.abs(g - e) <= ATOL + RTOL * np.abs(e))
        assert np.array_equal(g.view(np.uint32), e.view(np.uint32))
    # No bounded wait gave up on either path: the status call reads the
    # allocation-free path's own error word as well and reports it clean.
    assert L.quantr_gpu_device_status(ctypes.c_void_p(stream), 1) == 0


def test_noalloc_rejects_oversized_shape():
    import quantr

    L = quantr.lib()
    # 16 tokens x 65536 columns needs 2.6 MB of scratch, above the 1 MiB array;
    # the size check happens before any pointer is touched.
    rc = L.quantr_gemv_noalloc_dev(ctypes.c_void_p(16), 4, ctypes.c_void_p(16), 65536, ctypes.c_void_p(16), 12, 4,
                                   65536, 16, None)
    assert rc == 7  # QUANTR_ERR_TOO_LARGE
