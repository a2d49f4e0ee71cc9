"""Seeded synthetic decoder models (random-init weights with real architectures).

No checkpoints exist offline, so the decode configurations (TinyLlama-1.1B,
Qwen1.5-MoE-A2.7B, Qwen3-30B-A3B shapes) are built here from a seed.  The
weights are packed straight into the reference's block layouts (no fp32
intermediate) with scales chosen so every linear layer has roughly
N(0, 1/d_in) weights: activations stay O(1) through the layers, attention is
not one-hot, and greedy tokens vary.  fp16 fields use the reference's
truncating fp32->fp16 recipe (include/quant.h:68-77).

All tensors live in ONE contiguous host buffer with 32-byte aligned offsets,
like the GGUF mapping the reference loads (src/gguf.c:130-140,
src/model.c:253-449): the device decoder registers that buffer once and is
handed host pointers into it, exactly as the reference runtime would be.
"""
from dataclasses import dataclass, field

import numpy as np

import synth

F32, Q8_0, Q4_K, Q5_K, Q6_K = 0, 8, 12, 13, 14
ALIGN = 32


@dataclass
class Spec:
    dim: int
    hidden_dim: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    vocab_size: int
    seq_len: int
    rope_freq_base: float = 10000.0
    head_dim: int = 0            # 0: dim // n_heads (the reference's rule)
    expert_count: int = 0
    expert_used_count: int = 0
    shexp_hidden_dim: int = 0    # shared expert (Qwen1.5-MoE); 0 = none
    kv_type: int = 0             # 0 fp32, 1 fp16
    wtype: int = Q4_K            # attention and dense FFN linears
    w2type: int = -1             # FFN down projection (-1: wtype)
    exp_types: tuple = (Q4_K, Q4_K, Q4_K)  # expert W1 (=ffn_up), W3, W2
    shexp_types: tuple = (Q5_K, Q5_K, Q6_K)
    head_type: int = Q6_K
    embd_type: int = Q8_0

    @property
    def hd(self):
        return self.head_dim or self.dim // self.n_heads

    @property
    def q_dim(self):
        return self.n_heads * self.hd

    @property
    def kv_dim(self):
        return self.n_kv_heads * self.hd


def tinyllama(layers=22, vocab=32000, seq_len=1024):
    """BASELINE config c3: TinyLlama-1.1B (22 layers, dim 2048, 32/4 heads,
    head_dim 64, SwiGLU 5632, vocab 32000, RoPE theta 10000), Q4_K linears,
    Q6_K head."""
    return Spec(dim=2048, hidden_dim=5632, n_layers=layers, n_heads=32, n_kv_heads=4, vocab_size=vocab,
                seq_len=seq_len, rope_freq_base=10000.0, wtype=Q4_K, head_type=Q6_K, embd_type=Q8_0)


def qwen3_moe(layers=48, vocab=151936, seq_len=1152, experts=128):
    """BASELINE config c5: Qwen3-30B-A3B shape (48 layers, hidden 2048, 32/4
    heads with head_dim 128, 128 experts top-8 of intermediate 768, vocab
    151936), all Q4_K."""
    return Spec(dim=2048, hidden_dim=768, n_layers=layers, n_heads=32, n_kv_heads=4, vocab_size=vocab,
                seq_len=seq_len, rope_freq_base=10000.0, head_dim=128, expert_count=experts, expert_used_count=8,
                wtype=Q4_K, exp_types=(Q4_K, Q4_K, Q4_K), head_type=Q4_K, embd_type=Q4_K)


def qwen15_moe_layer_spec():
    """BASELINE config c4 shapes: hidden 2048, 60 experts top-4 of intermediate
    1408 (gate/up Q5_K, down Q6_K) plus a shared expert of 5632 with a sigmoid
    gate (one layer)."""
    return Spec(dim=2048, hidden_dim=1408, n_layers=1, n_heads=16, n_kv_heads=16, vocab_size=256, seq_len=64,
                expert_count=60, expert_used_count=4, shexp_hidden_dim=5632, exp_types=(Q5_K, Q5_K, Q6_K),
                shexp_types=(Q5_K, Q5_K, Q6_K), wtype=Q5_K, head_type=Q6_K, embd_type=Q8_0)


def row_bytes(t, d):
    if t == F32:
        return 4 * d
    return (d // synth.BLOCK_ELEMS[t]) * synth.BLOCK_BYTES[t]


def _f16(a):
    return synth.fp32_to_fp16_trunc(np.asarray(a, np.float32))


def _put16(blk, off, vals):
    n, nsb = vals.shape
    blk[:, :, off:off + 2] = vals.reshape(n, nsb, 1).view(np.uint8).reshape(n, nsb, 2)


def pack(rng, t, n, d, sigma):
    """n x d matrix of type t whose decoded values have std ~sigma."""
    if t == F32:
        return rng.normal(0.0, sigma, size=(n, d)).astype(np.float32).view(np.uint8).reshape(n, 4 * d)
    if t == Q8_0:
        nb = d // 32
        qs = rng.integers(-127, 128, size=(n, nb, 32), dtype=np.int16).astype(np.int8)
        # uniform [-127, 127] has std 73.3
        dd = _f16(np.full((n, nb), sigma / 73.3, np.float32) * (1.0 + 0.1 * rng.standard_normal((n, nb),
                                                                                               np.float32)))
        out = np.empty((n, nb, 34), np.uint8)
        _put16(out, 0, dd)
        out[:, :, 2:] = qs.view(np.uint8)
        return out.reshape(n, nb * 34)
    nsb = d // 256
    bb = synth.BLOCK_BYTES[t]
    nbytes = n * nsb * bb
    blk = rng.bit_generator.random_raw((nbytes + 7) // 8).view(np.uint8)[:nbytes].reshape(n, nsb, bb)
    jit = (1.0 + 0.1 * rng.standard_normal((n, nsb), np.float32)).astype(np.float32)
    if t in (Q4_K, Q5_K):
        levels = 16 if t == Q4_K else 32
        qmean, qstd = (levels - 1) / 2.0, np.sqrt((levels * levels - 1) / 12.0)
        # scale code c in [16, 47] (mean 31.5), min code mc in 0..3 (mean 1.5):
        c = rng.integers(16, 48, size=(n, nsb, 8), dtype=np.uint8)
        mc = rng.integers(0, 4, size=(n, nsb, 8), dtype=np.uint8)
        blk[:, :, 4:12] = c | (mc << 6)
        dd = np.float32(sigma / (31.5 * qstd)) * jit
        dmin = dd * np.float32(qmean * 31.5 / 1.5)
        _put16(blk, 0, _f16(dd))
        _put16(blk, 2, _f16(dmin))
    elif t == Q6_K:
        # quants uniform in [-32, 31] (std 18.5), scales int8 uniform in [-32, 31]
        sc = rng.integers(-32, 32, size=(n, nsb, 16), dtype=np.int16).astype(np.int8)
        blk[:, :, 192:208] = sc.view(np.uint8)
        dd = np.float32(sigma / (18.5 * 18.5)) * jit
        _put16(blk, 208, _f16(dd))
    else:
        raise ValueError(t)
    return blk.reshape(n, nsb * bb)


@dataclass
class Model:
    spec: Spec
    buf: np.ndarray                           # the whole "mapping" (uint8)
    off: dict = field(default_factory=dict)   # name -> (offset, nbytes, type)

    def ptr(self, name):
        return self.buf.ctypes.data + self.off[name][0]

    def array(self, name):
        o, nb, _ = self.off[name]
        return self.buf[o:o + nb]

    def type_of(self, name):
        return self.off[name][2]

    def expert_ptr(self, proj, layer, e):
        """Host address of expert e of merged projection proj ("exp_w1", ...)."""
        o, nb, _ = self.off[f"{proj}.{layer}"]
        return self.buf.ctypes.data + o + e * (nb // self.spec.expert_count)


def tensor_list(s):
    """(name, type, rows, cols, sigma) in load order."""
    out = [("token_embd", s.embd_type, s.vocab_size, s.dim, 1.0)]
    sig = lambda d: 1.0 / np.sqrt(d)  # noqa: E731
    w2t = s.w2type if s.w2type >= 0 else s.wtype
    for l in range(s.n_layers):
        out += [(f"rms_att.{l}", F32, 1, s.dim, None), (f"rms_ffn.{l}", F32, 1, s.dim, None),
                (f"wq.{l}", s.wtype, s.q_dim, s.dim, sig(s.dim)), (f"wk.{l}", s.wtype, s.kv_dim, s.dim, sig(s.dim)),
                (f"wv.{l}", s.wtype, s.kv_dim, s.dim, sig(s.dim)), (f"wo.{l}", s.wtype, s.dim, s.q_dim, sig(s.q_dim))]
        if s.expert_count:
            # merged expert tensors (GGUF *_exps, src/model.c:409-419): expert e
            # of a projection is rows [e*n, (e+1)*n)
            t1, t3, t2 = s.exp_types
            E = s.expert_count
            out += [(f"router.{l}", F32, E, s.dim, sig(s.dim)),
                    (f"exp_w1.{l}", t1, E * s.hidden_dim, s.dim, sig(s.dim)),
                    (f"exp_w3.{l}", t3, E * s.hidden_dim, s.dim, sig(s.dim)),
                    (f"exp_w2.{l}", t2, E * s.dim, s.hidden_dim, sig(s.hidden_dim))]
            if s.shexp_hidden_dim:
                a, b, c = s.shexp_types
                sh = s.shexp_hidden_dim
                out += [(f"shexp_w1.{l}", a, sh, s.dim, sig(s.dim)), (f"shexp_w3.{l}", b, sh, s.dim, sig(s.dim)),
                        (f"shexp_w2.{l}", c, s.dim, sh, sig(sh)), (f"shexp_gate.{l}", F32, 1, s.dim, sig(s.dim))]
        else:
            out += [(f"w1.{l}", s.wtype, s.hidden_dim, s.dim, sig(s.dim)),
                    (f"w3.{l}", s.wtype, s.hidden_dim, s.dim, sig(s.dim)),
                    (f"w2.{l}", w2t, s.dim, s.hidden_dim, sig(s.hidden_dim))]
    out += [("rms_final", F32, 1, s.dim, None), ("wcls", s.head_type, s.vocab_size, s.dim, 0.05)]
    return out


def build(spec, seed=0, threads=None):
    """The model's tensors packed into one 32-byte aligned host buffer.

    Tensor i is drawn from its own PCG64 stream seeded by (seed, i), so the
    tensors can be generated on all host cores and the bytes do not depend
    on the thread count."""
    import os
    from concurrent.futures import ThreadPoolExecutor
    tl = tensor_list(spec)
    off, pos = {}, 0
    for name, t, n, d, _ in tl:
        nb = n * row_bytes(t, d)
        off[name] = (pos, nb, t)
        pos = (pos + nb + ALIGN - 1) // ALIGN * ALIGN
    buf = np.zeros(pos + ALIGN, np.uint8)

    def one(i):
        name, t, n, d, sigma = tl[i]
        rng = np.random.Generator(np.random.PCG64(np.random.SeedSequence([seed, i])))
        o, nb, _ = off[name]
        if sigma is None:  # RMSNorm weight: 1 + N(0, 0.02)
            w = (1.0 + 0.02 * rng.standard_normal(d, dtype=np.float32)).astype(np.float32)
            buf[o:o + nb] = w.view(np.uint8)
        else:
            buf[o:o + nb] = pack(rng, t, n, d, sigma).reshape(-1)

    with ThreadPoolExecutor(max_workers=threads or os.cpu_count() or 1) as ex:
        list(ex.map(one, range(len(tl))))
    return Model(spec, buf, off)


def prompt(spec, n, seed=0, batch=1):
    """Seeded random prompt token ids, batch x n."""
    rng = synth.rng_for(10_000 + seed)
    return rng.integers(0, spec.vocab_size, size=(batch, n), dtype=np.int32)
