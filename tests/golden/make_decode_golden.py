"""Generates tests/golden/decode_c3.npz: the reference's own greedy decode of
BASELINE config c3 (TinyLlama-1.1B shape, 22 layers, Q4_K linears, Q6_K head,
Q8_0 embedding, RoPE theta 10000, fp32 KV cache) on the seeded synthetic model
of model_synth.tinyllama(), from a seeded 512-token prompt, 128 greedy tokens
(src/main.c:305-317 through the reference's forward_runtime, prefill_runtime
and sample_next, compiled from its sources by oracle/Makefile with the
restated Q4_K dot product interposed).

Stored: the 128 token ids, the SHA-256 of every step's logits (bit-exact
check of all 128 x 32000 values) and the full logits of the first and last
step (for diagnosis).  Run from the repository root:

    python tests/golden/make_decode_golden.py
"""
import hashlib
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path[:0] = [os.path.join(ROOT, "quantr-in-c_b200"), os.path.join(ROOT, "oracle")]

import forward  # noqa: E402
import model_synth as ms  # noqa: E402

MODEL_SEED, PROMPT_SEED, N_PROMPT, STEPS = 1, 7, 512, 128
OUT = os.path.join(ROOT, "tests", "golden", "decode_c3.npz")


def main():
    spec = ms.tinyllama()
    t0 = time.time()
    model = ms.build(spec, seed=MODEL_SEED)
    prompt = ms.prompt(spec, N_PROMPT, seed=PROMPT_SEED)[0]
    ref = forward.Reference(model, variant="scalar")
    toks, logits = ref.generate(prompt, STEPS, want_logits=True)
    digests = np.array([np.frombuffer(hashlib.sha256(l.tobytes()).digest(), np.uint8) for l in logits])
    np.savez_compressed(OUT, tokens=toks, logits_sha256=digests, logits_first=logits[0], logits_last=logits[-1],
                        model_seed=MODEL_SEED, prompt_seed=PROMPT_SEED, n_prompt=N_PROMPT, steps=STEPS)
    print(f"wrote {OUT} in {time.time() - t0:.0f} s; tokens {toks[:16]} ...")


if __name__ == "__main__":
    main()
