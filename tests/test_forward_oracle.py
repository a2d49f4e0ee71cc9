"""CPU: pins the restated decoder step (oracle/forward_oracle.c) against the
reference's own forward_runtime / prefill_runtime / sample_next, compiled from
its sources with the restated Q4_K dot product interposed (oracle/Makefile,
libquantr_ref_forward_scalar.so).  Logits must be bit-identical at every step
and the greedy tokens identical, for dense and MoE models, fp32 and fp16 KV
caches and every weight type.  Also checks that the link-time interposition
took: the reference build's matmul_q_fused gives the restated Q4_K results.
"""
import numpy as np
import pytest

import forward
import model_synth as ms
import oracle
import synth

pytestmark = pytest.mark.skipif(not forward.reference_available("scalar"),
                                reason="reference forward build (oracle/_ref) not present")


def small_dense(kv_type=0, wtype=ms.Q4_K, head=ms.Q6_K, embd=ms.Q8_0, layers=2):
    return ms.Spec(dim=512, hidden_dim=768, n_layers=layers, n_heads=8, n_kv_heads=2, vocab_size=1000,
                   seq_len=48, kv_type=kv_type, wtype=wtype, head_type=head, embd_type=embd)


def small_moe(kv_type=0):
    return ms.Spec(dim=512, hidden_dim=256, n_layers=2, n_heads=8, n_kv_heads=4, vocab_size=700, seq_len=40,
                   expert_count=8, expert_used_count=2, exp_types=(ms.Q5_K, ms.Q5_K, ms.Q6_K),
                   wtype=ms.Q8_0, head_type=ms.Q4_K, embd_type=ms.Q4_K, kv_type=kv_type)


def test_interposed_q4k_is_the_restatement():
    ref = forward.Reference.__new__(forward.Reference)  # library handle only
    import ctypes
    import os
    L = ctypes.CDLL(os.path.join(oracle.REF_DIR, "libquantr_ref_forward_scalar.so"))
    L.matmul_q_fused.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_uint32, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    rng = synth.rng_for(5)
    n, d = 64, 768
    w = synth.matrix(rng, ms.Q4_K, n, d)
    x = synth.activations(rng, 1, d)[0]
    got = np.zeros(n, np.float32)
    L.matmul_q_fused(got.ctypes.data, x.ctypes.data, w.ctypes.data, ms.Q4_K, n, d, 1)
    want = oracle.Oracle().matmul_q_fused(x, w, ms.Q4_K, n, d)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    del ref


@pytest.mark.parametrize("spec", [
    small_dense(),
    small_dense(kv_type=1),
    small_dense(wtype=ms.Q5_K, head=ms.Q8_0, embd=ms.F32),
    small_dense(wtype=ms.Q6_K, head=ms.Q4_K, embd=ms.Q5_K, layers=1),
    small_moe(),
    small_moe(kv_type=1),
], ids=["q4k", "q4k-fp16kv", "q5k-f32embd", "q6k", "moe", "moe-fp16kv"])
def test_restated_forward_matches_reference(spec):
    model = ms.build(spec, seed=11)
    prompt = ms.prompt(spec, 9, seed=3)[0]
    steps = 12
    want_t, want_l = forward.Reference(model).generate(prompt, steps, want_logits=True)
    got_t, got_l = forward.Restated(model).generate(prompt, steps, want_logits=True)
    assert np.all(np.isfinite(want_l))
    assert np.array_equal(got_l.view(np.uint32), want_l.view(np.uint32))
    np.testing.assert_array_equal(got_t, want_t)
    # the synthetic model is not degenerate: the greedy tokens vary
    assert len(set(want_t.tolist())) > 3


def test_explicit_head_dim_equal_to_derived_is_identity():
    spec = small_dense()
    model = ms.build(spec, seed=2)
    spec2 = ms.Spec(**{**spec.__dict__, "head_dim": spec.dim // spec.n_heads})
    model2 = ms.Model(spec2, model.buf, model.off)
    p = ms.prompt(spec, 5, seed=1)[0]
    a, _ = forward.Restated(model).generate(p, 6)
    b, _ = forward.Restated(model2).generate(p, 6)
    np.testing.assert_array_equal(a, b)
