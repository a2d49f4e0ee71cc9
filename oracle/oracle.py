"""ctypes access to the oracle libraries.  TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
arm may import this module; it is the checker (or the timed CPU baseline),
never part of the product path.

  Oracle(...)      -> _build/libquant_oracle.so, this repo's C restatement
                      (quant_oracle.c), bit-identical to the reference's scalar
                      build and pinned by tests/golden/.
  RefLib(variant)  -> _ref/libquantr_ref_<variant>.so, the reference's own
                      src/quant.c compiled by oracle/Makefile (scalar, avx2,
                      avx512).  Present wherever it was built (the built
                      libraries travel with the tree; the reference's sources
                      are needed only to build them).
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libquant_oracle.so")
REF_DIR = os.path.join(HERE, "_ref")

_vp, _i, _u32, _f, _l = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint32, ctypes.c_float, ctypes.c_long


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def ref_root():
    """The reference checkout: $REF, else ../reference beside this repository."""
    return os.environ.get("REF") or os.path.abspath(os.path.join(HERE, "..", "..", "reference"))


def build(ref=True):
    """Builds the restatement (and, if the reference sources exist, _ref)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    if ref and os.path.isdir(os.path.join(ref_root(), "src")):
        subprocess.run(["make", "-s", "-C", HERE, "ref"], check=True)


def row_bytes(type_, d):
    return {0: 4 * d, 8: (d // 32) * 34, 12: (d // 256) * 144, 13: (d // 256) * 176,
            14: (d // 256) * 210}.get(type_, 4 * d)


class _QuantLib:
    """Common wrapper: both libraries export the reference's function set."""

    PREFIX = ""

    def __init__(self, path):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        self.path = path
        L = ctypes.CDLL(path)
        pre = self.PREFIX
        sig = {
            "quantize_row_q8_0": (None, [_vp, _vp, _i]),
            "dequantize_row": (None, [_vp, _vp, _u32, _i]),
            "vec_dot_q8_0_q8_0": (_f, [_vp, _vp, _i]),
            "vec_dot_q4K_q8_0": (_f, [_vp, _vp, _i]),
            "vec_dot_q5K_q8_0": (_f, [_vp, _vp, _i]),
            "vec_dot_q6K_q8_0": (_f, [_vp, _vp, _i]),
            "matmul_q_fused": (None, [_vp, _vp, _vp, _u32, _i, _i, _i]),
        }
        self.fn = {}
        for name, (res, args) in sig.items():
            f = getattr(L, pre + name)
            f.restype = res
            f.argtypes = args
            self.fn[name] = f
        self.L = L

    def quantize_row_q8_0(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.zeros((x.size // 32) * 34, dtype=np.uint8)
        self.fn["quantize_row_q8_0"](_p(x), _p(y), x.size)
        return y

    def dequantize_row(self, src, type_, n):
        out = np.zeros(n, dtype=np.float32)
        s = None if src is None else np.ascontiguousarray(src)
        self.fn["dequantize_row"](_p(out), _p(s), type_, n)
        return out

    def vec_dot(self, type_, a, b, k):
        name = {8: "vec_dot_q8_0_q8_0", 12: "vec_dot_q4K_q8_0", 13: "vec_dot_q5K_q8_0",
                14: "vec_dot_q6K_q8_0"}[type_]
        a = np.ascontiguousarray(a, dtype=np.uint8)
        b = np.ascontiguousarray(b, dtype=np.uint8)
        return np.float32(self.fn[name](_p(a), _p(b), k))

    def matmul_q_fused(self, x, w, type_, n, d, threads=1):
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty(n, dtype=np.float32)
        self.fn["matmul_q_fused"](_p(out), _p(x), None if w is None else _p(np.ascontiguousarray(w)),
                                  type_, n, d, threads)
        return out

    def matmul_q_fused_batch(self, x, w, type_, n, d, threads=1):
        x = np.ascontiguousarray(x, dtype=np.float32)
        return np.stack([self.matmul_q_fused(x[t], w, type_, n, d, threads) for t in range(x.shape[0])])


class Oracle(_QuantLib):
    """This repository's restatement (oracle/quant_oracle.c)."""

    PREFIX = "qo_"

    def __init__(self, path=ORACLE_SO):
        if not os.path.exists(path):
            build(ref=False)
        super().__init__(path)
        L = self.L
        L.qo_fp16_to_fp32.restype = _f
        L.qo_fp16_to_fp32.argtypes = [ctypes.c_uint16]
        L.qo_fp32_to_fp16.restype = ctypes.c_uint16
        L.qo_fp32_to_fp16.argtypes = [_f]
        L.qo_unit_partials.restype = _i
        L.qo_unit_partials.argtypes = [_vp, _vp, _vp, _u32, _i, _i, _vp]
        L.qo_softmax.restype = None
        L.qo_softmax.argtypes = [_vp, _i]
        L.qo_matmul_f32.restype = None
        L.qo_matmul_f32.argtypes = [_vp, _vp, _vp, _i, _i]
        L.qo_expf_mismatches.restype = _l
        L.qo_expf_mismatches.argtypes = [_vp, _u32, _l]
        L.qo_shared_expert.restype = None
        L.qo_shared_expert.argtypes = [_vp, _vp, _vp, _vp, _u32, _vp, _u32, _vp, _u32, _i, _i, _i]
        L.qo_moe_token.restype = _i
        L.qo_moe_token.argtypes = [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _vp, _u32, _l, _vp, _u32, _l,
                                   _vp, _u32, _l, _i, _i]

    def fp16_to_fp32(self, h):
        return np.float32(self.L.qo_fp16_to_fp32(int(h)))

    def fp32_to_fp16(self, f):
        return int(self.L.qo_fp32_to_fp16(float(f)))

    def expf_mismatches(self, got, first):
        """Entries of got (float32[n]) that differ from the C library's expf
        of the floats with bit patterns first, first + 1, ..."""
        got = np.ascontiguousarray(got, np.float32)
        return int(self.L.qo_expf_mismatches(_p(got), first, got.size))

    def shared_expert(self, out, xb, gate, w1, t1, w3, t3, w2, t2, dim, hidden):
        """out (float32[dim], updated in place) += the gated shared expert of xb."""
        self.L.qo_shared_expert(_p(out), _p(np.ascontiguousarray(xb, np.float32)),
                                _p(np.ascontiguousarray(gate, np.float32)), _p(w1), t1, _p(w3), t3, _p(w2), t2, dim,
                                hidden, os.cpu_count() or 1)
        return out

    def unit_partials(self, w, type_, n, d, xq):
        units = (d // 32) if type_ == 8 else 8 * (d // 256)
        isum = np.zeros((n, units), dtype=np.int32)
        bsum = np.zeros((n, units), dtype=np.int32)
        self.L.qo_unit_partials(_p(isum), _p(bsum), _p(np.ascontiguousarray(w)), type_, n, d,
                                _p(np.ascontiguousarray(xq)))
        return isum, bsum

    def softmax(self, x):
        y = np.array(x, dtype=np.float32, copy=True)
        self.L.qo_softmax(_p(y), y.size)
        return y

    def matmul_f32(self, x, w, n, d):
        out = np.zeros(n, dtype=np.float32)
        self.L.qo_matmul_f32(_p(out), _p(np.ascontiguousarray(x, np.float32)),
                             _p(np.ascontiguousarray(w, np.float32)), n, d)
        return out

    def moe_token(self, xb, E, k, w1, t1, b1, w3, t3, b3, w2, t2, b2, dim, hidden, router=None, logits=None):
        out = np.zeros(dim, dtype=np.float32)
        sel = np.zeros(k, dtype=np.int32)
        wts = np.zeros(k, dtype=np.float32)
        rc = self.L.qo_moe_token(_p(out), _p(sel), _p(wts), _p(np.ascontiguousarray(xb, np.float32)),
                                 _p(router), _p(logits), E, k, _p(w1), t1, b1, _p(w3), t3, b3, _p(w2), t2, b2,
                                 dim, hidden)
        if rc:
            raise ValueError("qo_moe_token rejected the shape")
        return out, sel, wts


class RefLib(_QuantLib):
    """The reference's own src/quant.c, compiled by oracle/Makefile."""

    def __init__(self, variant="scalar"):
        super().__init__(os.path.join(REF_DIR, f"libquantr_ref_{variant}.so"))
        self.variant = variant
        L = self.L
        L.ref_fp16_to_fp32.restype = _f
        L.ref_fp16_to_fp32.argtypes = [ctypes.c_uint16]
        L.ref_fp32_to_fp16.restype = ctypes.c_uint16
        L.ref_fp32_to_fp16.argtypes = [_f]
        L.ref_softmax.restype = None
        L.ref_softmax.argtypes = [_vp, _i]
        L.ref_matmul_f32.restype = None
        L.ref_matmul_f32.argtypes = [_vp, _vp, _vp, _i, _i, _i]

    def softmax(self, x):
        """KernelOps softmax of the scalar backend (src/kernels.c:191-207)."""
        y = np.array(x, dtype=np.float32, copy=True)
        self.L.ref_softmax(_p(y), y.size)
        return y

    def matmul_f32(self, x, w, n, d, backend=0):
        """KernelOps matmul of `backend` (0 = matmul_ref, src/kernels.c:18-28)."""
        out = np.zeros(n, dtype=np.float32)
        self.L.ref_matmul_f32(_p(out), _p(np.ascontiguousarray(x, np.float32)),
                              _p(np.ascontiguousarray(w, np.float32)), n, d, backend)
        return out

    def fp16_to_fp32(self, h):
        return np.float32(self.L.ref_fp16_to_fp32(int(h)))

    def fp32_to_fp16(self, f):
        return int(self.L.ref_fp32_to_fp16(float(f)))


def ref_available(variant="scalar"):
    return os.path.exists(os.path.join(REF_DIR, f"libquantr_ref_{variant}.so"))


def best_cpu_variant():
    """Fastest reference build this host's CPU can run."""
    try:
        flags = open("/proc/cpuinfo").read()
    except OSError:
        flags = ""
    if " avx512f" in flags and ref_available("avx512"):
        return "avx512"
    if " avx2" in flags and ref_available("avx2"):
        return "avx2"
    return "scalar"
