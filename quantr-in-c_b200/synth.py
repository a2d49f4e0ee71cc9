"""Seeded synthetic weights and activations with the shapes and value
distributions of the benchmark configurations (no checkpoints exist offline).

All generators use numpy's PCG64 with an explicit seed, so a (config, seed)
pair names one exact byte string; the parity tests and the benchmark build
their inputs from here.

Layouts are the reference's packed blocks (include/quant.h:28-50,
src/quant.c:216-236).  fp16 fields are produced with the reference's own
truncating fp32->fp16 recipe (include/quant.h:68-77).
"""
import numpy as np

Q8_0, Q4_K, Q5_K, Q6_K = 8, 12, 13, 14
BLOCK_BYTES = {Q8_0: 34, Q4_K: 144, Q5_K: 176, Q6_K: 210}
BLOCK_ELEMS = {Q8_0: 32, Q4_K: 256, Q5_K: 256, Q6_K: 256}


def fp32_to_fp16_trunc(a):
    """Vectorised reference fp32->fp16: truncate mantissa, FTZ, saturate."""
    x = np.asarray(a, dtype=np.float32).view(np.uint32).astype(np.int64)
    s = (x >> 16) & 0x8000
    e = ((x >> 23) & 0xFF) - 112
    m = (x >> 13) & 0x3FF
    h = np.where(e <= 0, s, np.where(e >= 31, s | 0x7C00, s | (np.clip(e, 0, 31) << 10) | m))
    return h.astype(np.uint16)


def rng_for(seed):
    return np.random.Generator(np.random.PCG64(seed))


def activations(rng, B, d):
    """x ~ N(0, 1), float32[B, d]."""
    return rng.standard_normal((B, d), dtype=np.float32)


def q8_0_matrix(rng, n, d, sigma=0.02):
    """Config-1 Q8_0 weights: per 32-block w ~ N(0, sigma), d = fp16(max|w|/127),
    quants uniform integers in [-127, 127].  Returns uint8[n, row_bytes]."""
    nb = d // 32
    w = rng.normal(0.0, sigma, size=(n, nb, 32)).astype(np.float32)
    scale = fp32_to_fp16_trunc(np.abs(w).max(axis=2) / np.float32(127.0))
    qs = rng.integers(-127, 128, size=(n, nb, 32), dtype=np.int16).astype(np.int8)
    out = np.empty((n, nb, 34), dtype=np.uint8)
    out[:, :, 0:2] = scale.reshape(n, nb, 1).view(np.uint8).reshape(n, nb, 2)
    out[:, :, 2:] = qs.view(np.uint8)
    return out.reshape(n, nb * 34)


def kquant_matrix(rng, type_, n, d, d_sigma=0.002, dmin_sigma=0.001):
    """Config-2 style K-quant super-blocks: fp16 d ~ |N(0, d_sigma)|, fp16
    dmin ~ |N(0, dmin_sigma)| (Q4_K/Q5_K), every other byte (scale codes,
    quants, high bits) uniform random.  Returns uint8[n, row_bytes]."""
    nsb = d // 256
    bb = BLOCK_BYTES[type_]
    blk = rng.integers(0, 256, size=(n, nsb, bb), dtype=np.uint8)
    dd = fp32_to_fp16_trunc(np.abs(rng.normal(0.0, d_sigma, size=(n, nsb))).astype(np.float32))
    if type_ in (Q4_K, Q5_K):
        dm = fp32_to_fp16_trunc(np.abs(rng.normal(0.0, dmin_sigma, size=(n, nsb))).astype(np.float32))
        blk[:, :, 0:2] = dd.reshape(n, nsb, 1).view(np.uint8).reshape(n, nsb, 2)
        blk[:, :, 2:4] = dm.reshape(n, nsb, 1).view(np.uint8).reshape(n, nsb, 2)
    elif type_ == Q6_K:
        blk[:, :, 208:210] = dd.reshape(n, nsb, 1).view(np.uint8).reshape(n, nsb, 2)
    else:
        raise ValueError(type_)
    return blk.reshape(n, nsb * bb)


def matrix(rng, type_, n, d):
    return q8_0_matrix(rng, n, d) if type_ == Q8_0 else kquant_matrix(rng, type_, n, d)


def random_bytes(rng, n):
    return rng.integers(0, 256, size=n, dtype=np.uint8)
