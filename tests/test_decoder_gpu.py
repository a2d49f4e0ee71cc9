"""GPU: the device-resident decoder (quantr_decoder_*) against the decoder-step
oracles.

The decoder runs the reference's forward_runtime on the device with every
floating-point operation in the reference's order and rounding, so the bar is
bit-identity: every step's logits must equal the oracle's bit for bit and the
greedy tokens must be identical (1e-5 rel / 1e-6 abs, is
asserted too).  The oracle is the restatement in oracle/forward_oracle.c, which
tests/test_forward_oracle.py pins to the reference's own forward_runtime; the
full c3 configuration is compared with tokens and logit digests produced by
the reference itself (tests/golden/decode_c3.npz).
"""
import hashlib
import os

import numpy as np
import pytest

import model_synth as ms

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

RTOL, ATOL = 1e-5, 1e-6
GOLDEN_C3 = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "decode_c3.npz")


def _oracle(model):
    import forward
    return forward.Restated(model)


def _decoder(qr_gpu, model, batch=1):
    import quantr
    return quantr.Decoder(model, batch=batch)


def _same(got, want):
    got = np.asarray(got, np.float32)
    want = np.asarray(want, np.float32)
    assert got.shape == want.shape
    assert np.all(np.isfinite(want))
    assert np.all(np.abs(got - want) <= ATOL + RTOL * np.abs(want)), float(np.abs(got - want).max())
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), \
        f"{int((got.view(np.uint32) != want.view(np.uint32)).sum())} logits differ in their bits"


def dense(kv_type=0, wtype=ms.Q4_K, head=ms.Q6_K, embd=ms.Q8_0, layers=2, **kw):
    base = dict(dim=512, hidden_dim=768, n_layers=layers, n_heads=8, n_kv_heads=2, vocab_size=1000, seq_len=64,
                kv_type=kv_type, wtype=wtype, head_type=head, embd_type=embd)
    base.update(kw)
    return ms.Spec(**base)


def run_generate(qr_gpu, spec, seed=3, n_prompt=9, steps=12, batch=1):
    model = ms.build(spec, seed=seed)
    prompt = ms.prompt(spec, n_prompt, seed=seed + 1, batch=batch)
    dec = _decoder(qr_gpu, model, batch)
    try:
        got = dec.generate(prompt, steps)
    finally:
        dec.close()
    for b in range(batch):
        want, _ = _oracle(model).generate(prompt[b], steps)
        np.testing.assert_array_equal(got[b], want)
    return got


def test_device_expf_matches_c_library_on_every_float(qr_gpu, orc):
    import quantr
    n = 1 << 28
    buf = torch.empty(n, dtype=torch.float32, device="cuda")
    host = torch.empty(n, dtype=torch.float32, pin_memory=True)
    bad = 0
    for chunk in range(16):
        first = chunk * n
        rc = quantr.lib().quantr_debug_expf_dev(buf.data_ptr(), first, n, None)
        assert rc == 0
        host.copy_(buf)
        bad += orc.expf_mismatches(host.numpy(), first)
    assert bad == 0, f"{bad} floats where the device expf differs from the C library"


def test_forward_runtime_logits_bit_exact(qr_gpu):
    """quantr_forward_runtime at consecutive positions == qo_forward."""
    spec = dense()
    model = ms.build(spec, seed=5)
    orc = _oracle(model)
    dec = _decoder(qr_gpu, model)
    try:
        toks = ms.prompt(spec, 10, seed=9)[0]
        for pos, t in enumerate(toks):
            _same(dec.forward_runtime(int(t), pos), orc.forward(int(t), pos))
    finally:
        dec.close()


def test_prefill_runtime_then_forward(qr_gpu):
    spec = dense(layers=1)
    model = ms.build(spec, seed=6)
    orc = _oracle(model)
    dec = _decoder(qr_gpu, model)
    try:
        p = ms.prompt(spec, 7, seed=2)[0]
        dec.prefill_runtime(p)
        for i, t in enumerate(p):
            orc.forward(int(t), i)
        _same(dec.forward_runtime(int(p[-1]), 7), orc.forward(int(p[-1]), 7))
    finally:
        dec.close()


@pytest.mark.parametrize("spec", [
    dense(),
    dense(kv_type=1),
    dense(wtype=ms.Q5_K, head=ms.Q8_0, embd=ms.F32),
    dense(wtype=ms.Q8_0, head=ms.Q4_K, embd=ms.Q5_K),
    dense(wtype=ms.Q6_K, head=ms.Q6_K, embd=ms.Q4_K, layers=1),
    dense(head_dim=128, n_heads=8, n_kv_heads=2),  # explicit head_dim: q_dim 1024 != dim 512
], ids=["q4k", "q4k-fp16kv", "q5k-f32embd", "q8_0", "q6k", "headdim128"])
def test_generate_matches_oracle(qr_gpu, spec):
    """src/main.c:305-317 on the device: identical greedy tokens."""
    toks = run_generate(qr_gpu, spec)
    assert len(set(toks[0].tolist())) > 3


@pytest.mark.parametrize("kv_type,seq_len,n_prompt", [(0, 640, 530), (1, 1024, 900)], ids=["fp32kv", "fp16kv"])
def test_generate_long_context_value_ring(qr_gpu, kv_type, seq_len, n_prompt):
    """One sequence at a context longer than the value ring of the
    one-head-per-CTA softmax-V kernel holds (head_dim 128: 13 fp32 or 27 fp16
    stages of 32 positions), so stages are refilled while the running sums
    advance, over full tiles and a partial last tile: identical tokens."""
    spec = dense(kv_type=kv_type, head_dim=128, n_heads=4, n_kv_heads=2, seq_len=seq_len)
    run_generate(qr_gpu, spec, n_prompt=n_prompt, steps=6)


def test_persistent_one_token_kernel(qr_gpu, monkeypatch):
    """The persistent single-launch step (csrc/decode_persist.cu, opt-in with
    QUANTR_DECODE_PERSIST=1): identical tokens and bit-identical logits."""
    monkeypatch.setenv("QUANTR_DECODE_PERSIST", "1")
    spec = dense(layers=3)
    run_generate(qr_gpu, spec)
    model = ms.build(spec, seed=21)
    dec = _decoder(qr_gpu, model)
    try:
        assert dec.info()["launches_per_decode_step"] <= 8  # feed, barrier reset, persistent kernel, head
        orc = _oracle(model)
        for pos, t in enumerate(ms.prompt(spec, 6, seed=5)[0]):
            _same(dec.forward_runtime(int(t), pos), orc.forward(int(t), pos))
    finally:
        dec.close()


def test_generate_batched_sequences(qr_gpu):
    """Three independent sequences with their own prompts and KV caches; the
    GEMVs run as 3-token tensor-core jobs."""
    run_generate(qr_gpu, dense(), batch=3, steps=10)


def test_generate_wraps_positions(qr_gpu):
    """Positions wrap at seq_len (pos++ % seq_len, src/main.c:315)."""
    run_generate(qr_gpu, dense(seq_len=16, layers=1), n_prompt=6, steps=14)


def test_generate_moe_with_shared_expert(qr_gpu):
    spec = ms.Spec(dim=512, hidden_dim=256, n_layers=2, n_heads=8, n_kv_heads=4, vocab_size=700, seq_len=40,
                   expert_count=8, expert_used_count=2, exp_types=(ms.Q5_K, ms.Q5_K, ms.Q6_K), wtype=ms.Q8_0,
                   head_type=ms.Q4_K, embd_type=ms.Q4_K, shexp_hidden_dim=512, shexp_types=(ms.Q5_K, ms.Q5_K, ms.Q6_K))
    run_generate(qr_gpu, spec)


def test_generate_moe_batched_tensor_cores(qr_gpu):
    """c5-like shapes scaled down: explicit head_dim 128, 16 experts top-4,
    20 sequences (the experts stage runs on the tensor cores from 16 tokens)."""
    spec = ms.Spec(dim=512, hidden_dim=256, n_layers=2, n_heads=8, n_kv_heads=2, vocab_size=600, seq_len=32,
                   head_dim=128, expert_count=16, expert_used_count=4, wtype=ms.Q4_K, head_type=ms.Q4_K,
                   embd_type=ms.Q4_K)
    run_generate(qr_gpu, spec, batch=20, n_prompt=5, steps=6)


def test_c5_layer_shapes_batch64(qr_gpu):
    """BASELINE config c5's layer at full width (hidden 2048, 32/4 heads of
    head_dim 128, 128 experts top-8 of intermediate 768, all Q4_K), 2 layers,
    64 sequences: every sequence's greedy tokens identical to the per-sequence
    restated forward_runtime (the oracle c5 names)."""
    spec = ms.qwen3_moe(layers=2, vocab=1024, seq_len=16)
    run_generate(qr_gpu, spec, seed=12, n_prompt=4, steps=4, batch=64)


def test_step_dev_matches_forward(qr_gpu):
    """quantr_decoder_step_dev with device tokens/positions, two sequences at
    different positions."""
    spec = dense(layers=1)
    model = ms.build(spec, seed=8)
    dec = _decoder(qr_gpu, model, batch=2)
    orcs = [_oracle(model), _oracle(model)]
    try:
        p = ms.prompt(spec, 6, seed=4, batch=2)
        logits = torch.empty((2, spec.vocab_size), device="cuda")
        nxt = torch.empty(2, dtype=torch.int32, device="cuda")
        stream = torch.cuda.current_stream().cuda_stream
        for step in range(6):
            pos = [step, (step + 3) % spec.seq_len]
            tok = torch.tensor([int(p[0][step]), int(p[1][step])], dtype=torch.int32, device="cuda")
            posd = torch.tensor(pos, dtype=torch.int32, device="cuda")
            dec.step_dev(tok.data_ptr(), posd.data_ptr(), logits.data_ptr(), spec.vocab_size, nxt.data_ptr(), stream)
            torch.cuda.synchronize()
            got = logits.cpu().numpy()
            for b in range(2):
                want = orcs[b].forward(int(p[b][step]), pos[b])
                _same(got[b], want)
                assert int(nxt[b]) == int(np.argmax(want))
    finally:
        dec.close()


@pytest.mark.timeout(900)
def test_c3_tinyllama_decode_matches_reference():
    """BASELINE config c3 at full size: 22 layers, 512 prefill tokens, 128
    greedy tokens; token ids identical to the reference's own decode and the
    logits of every step bit-identical (SHA-256 of each step's 32000 logits)."""
    import quantr
    if not os.path.exists(GOLDEN_C3):
        pytest.skip("tests/golden/decode_c3.npz not generated")
    g = np.load(GOLDEN_C3)
    spec = ms.tinyllama()
    model = ms.build(spec, seed=int(g["model_seed"]))
    prompt = ms.prompt(spec, int(g["n_prompt"]), seed=int(g["prompt_seed"]))
    L = quantr.lib()
    assert L.quantr_gpu_init(0) == 0
    dec = quantr.Decoder(model)
    try:
        toks = dec.generate(prompt, int(g["steps"]))[0]
        np.testing.assert_array_equal(toks, g["tokens"])
        # replay with explicit positions to read every step's logits
        dec.prefill_runtime(prompt[0])
        tok, pos = int(prompt[0][-1]), int(g["n_prompt"])
        for i in range(int(g["steps"])):
            lg = dec.forward_runtime(tok, pos)
            if i == 0:
                _same(lg, g["logits_first"])
            d = np.frombuffer(hashlib.sha256(np.ascontiguousarray(lg).tobytes()).digest(), np.uint8)
            assert np.array_equal(d, g["logits_sha256"][i]), f"step {i}: logits differ"
            tok, pos = int(g["tokens"][i]), pos + 1
    finally:
        dec.close()
