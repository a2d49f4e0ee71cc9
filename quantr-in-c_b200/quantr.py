"""Python mirror of quantr-in-c's quantized-GEMV API over libquantr_cuda.so.

The names, argument meanings and error behaviour follow the reference's C API
(include/quant.h:84-92): ``quantize_row_q8_0``, ``dequantize_row``,
``vec_dot_*_q8_0``, ``matmul_q_fused``.  Arrays are numpy host arrays, exactly
like the C functions take host pointers; every call runs on the GPU through the
C ABI declared in include/quantr_cuda.h.  There is no CPU path: if the CUDA
library cannot be loaded the import fails, and a device failure raises
``QuantrError`` carrying the library's sticky error code (the C calls
themselves zero their outputs, as the reference does).

The ``*_dev`` functions take device addresses (ints, e.g. ``tensor.data_ptr()``)
and a ``cudaStream_t`` handle (int) and are stream-ordered.
"""
import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libquantr_cuda.so")

F32, Q8_0, Q4_K, Q5_K, Q6_K = 0, 8, 12, 13, 14
TYPE_NAMES = {F32: "F32", Q8_0: "Q8_0", Q4_K: "Q4_K", Q5_K: "Q5_K", Q6_K: "Q6_K"}
BLOCK_BYTES = {Q8_0: 34, Q4_K: 144, Q5_K: 176, Q6_K: 210}
BLOCK_ELEMS = {Q8_0: 32, Q4_K: 256, Q5_K: 256, Q6_K: 256}

# Exported symbols of include/quantr_cuda.h with their ctypes signatures.
_c = ctypes
_vp, _i, _u32, _sz, _ll, _f = _c.c_void_p, _c.c_int, _c.c_uint32, _c.c_size_t, _c.c_longlong, _c.c_float
SIGNATURES = {
    "quantize_row_q8_0": (None, [_vp, _vp, _i]),
    "dequantize_row": (None, [_vp, _vp, _u32, _i]),
    "vec_dot_q4K_q8_0": (_f, [_vp, _vp, _i]),
    "vec_dot_q5K_q8_0": (_f, [_vp, _vp, _i]),
    "vec_dot_q6K_q8_0": (_f, [_vp, _vp, _i]),
    "vec_dot_q8_0_q8_0": (_f, [_vp, _vp, _i]),
    "matmul_q_fused": (None, [_vp, _vp, _vp, _u32, _i, _i, _i]),
    "matmul_q_fused_batch": (None, [_vp, _vp, _vp, _u32, _i, _i, _i]),
    "quantr_gpu_last_error": (_i, []),
    "quantr_gpu_clear_error": (None, []),
    "quantr_gpu_error_string": (_c.c_char_p, [_i]),
    "quantr_gpu_init": (_i, [_i]),
    "quantr_gpu_shutdown": (None, []),
    "quantr_gpu_launch_count": (_c.c_uint64, []),
    "quantr_gpu_register_weights": (_i, [_vp, _sz]),
    "quantr_gpu_unregister_weights": (_i, [_vp]),
    "quantr_gpu_device_ptr": (_vp, [_vp]),
    "quantr_gemv_workspace_bytes": (_sz, [_i, _i]),
    "quantr_gemv_dev": (_i, [_vp, _ll, _vp, _ll, _vp, _u32, _i, _i, _i, _vp, _sz, _vp]),
    "quantr_quantize_q8_0_dev": (_i, [_vp, _vp, _ll, _i, _i, _vp]),
    "quantr_gemv_q8act_dev": (_i, [_vp, _ll, _vp, _vp, _u32, _i, _i, _i, _vp, _sz, _vp]),
    "quantr_gemv_partials_dev": (_i, [_vp, _vp, _vp, _vp, _vp, _u32, _i, _i, _i, _vp, _sz, _vp]),
    "quantr_gpu_device_status": (_i, [_vp, _i]),
    "quantr_gemv_noalloc_dev": (_i, [_vp, _ll, _vp, _ll, _vp, _u32, _i, _i, _i, _vp]),
    "quantr_program_create": (_i, [_c.POINTER(_vp), _vp, _i]),
    "quantr_program_run": (_i, [_vp, _vp]),
    "quantr_program_destroy": (None, [_vp]),
    "quantr_program_info": (_i, [_vp, _c.POINTER(_i), _c.POINTER(_i), _c.POINTER(_i)]),
    "quantr_moe_workspace_bytes": (_sz, [_i, _i, _i, _i, _i]),
    "quantr_moe_dev": (_i, [_vp, _ll, _vp, _ll, _i, _vp, _vp, _ll, _i, _i, _vp, _vp, _vp, _i, _i, _vp, _vp, _vp,
                            _sz, _vp]),
    "quantr_moe_route_dev": (_i, [_vp, _vp, _vp, _ll, _i, _vp, _vp, _ll, _i, _i, _i, _vp, _sz, _vp]),
    "quantr_moe_experts_dev": (_i, [_vp, _vp, _ll, _i, _vp, _i, _i, _i, _vp, _vp, _vp, _i, _i, _vp, _sz, _vp]),
    "quantr_moe_combine_dev": (_i, [_vp, _ll, _vp, _vp, _vp, _i, _i, _i, _vp]),
    "quantr_moe_layer": (_i, [_vp, _vp, _i, _vp, _vp, _i, _i, _vp, _u32, _vp, _u32, _vp, _u32, _i, _i, _vp, _vp]),
    "quantr_decoder_create": (_i, [_c.POINTER(_vp), _vp, _i]),
    "quantr_decoder_destroy": (None, [_vp]),
    "quantr_decoder_step_dev": (_i, [_vp, _vp, _vp, _vp, _ll, _vp, _vp]),
    "quantr_decoder_generate": (_i, [_vp, _vp, _i, _i, _vp]),
    "quantr_forward_runtime": (_c.POINTER(_f), [_vp, _i, _i]),
    "quantr_prefill_runtime": (None, [_vp, _vp, _i]),
    "quantr_decoder_info": (_i, [_vp, _c.POINTER(_sz), _c.POINTER(_sz), _c.POINTER(_sz)]),
    "quantr_debug_expf_dev": (_i, [_vp, _u32, _ll, _vp]),
    "quantr_dequantize_rows_dev": (_i, [_vp, _ll, _vp, _ll, _u32, _i, _i, _vp]),
    "quantr_decoder_generate_dev": (_i, [_vp, _vp, _i, _i, _vp, _vp]),
    "quantr_decoder_launches": (_i, [_vp, _c.POINTER(_i), _c.POINTER(_i)]),
    "quantr_decoder_kv": (_i, [_vp, _c.POINTER(_vp), _c.POINTER(_vp), _c.POINTER(_sz)]),
    "quantr_moe_shared_dev": (_i, [_vp, _ll, _vp, _ll, _i, _vp, _vp, _u32, _vp, _u32, _vp, _u32, _i, _i, _vp]),
}


class GemvJob(ctypes.Structure):
    """quantr_gemv_job (include/quantr_cuda.h)."""
    _fields_ = [("w", _vp), ("type", _u32), ("n", _i), ("d", _i), ("B", _i), ("x", _vp), ("ldx", _ll),
                ("out", _vp), ("ldo", _ll)]


class ExpertWeights(ctypes.Structure):
    """quantr_expert_weights (include/quantr_cuda.h)."""
    _fields_ = [("base", _vp), ("stride", _ll), ("table", _vp), ("type", _u32)]


class QuantrError(RuntimeError):
    def __init__(self, code, where=""):
        msg = lib().quantr_gpu_error_string(code).decode()
        super().__init__(f"{where}: quantr error {code} ({msg})" if where else f"quantr error {code} ({msg})")
        self.code = code


_lib = None


def lib():
    """Loads libquantr_cuda.so (raises OSError if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise OSError(f"{LIB_PATH} is missing: run quantr-in-c_b200/build.py (or __graft_entry__.build())")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None else None


def _check(where):
    code = lib().quantr_gpu_last_error()
    if code:
        lib().quantr_gpu_clear_error()
        raise QuantrError(code, where)


def row_bytes(type_, d):
    """Packed bytes of one row of d columns (src/quant.c:477-484)."""
    if type_ == F32:
        return 4 * d
    return (d // BLOCK_ELEMS[type_]) * BLOCK_BYTES[type_]


# ---------------------------------------------------------------- Part 1 --

def quantize_row_q8_0(x):
    """x: float32[k] -> uint8[(k//32)*34] packed block_q8_0 (src/quant.c:143)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros((x.size // 32) * 34, dtype=np.uint8)
    lib().quantize_row_q8_0(_ptr(x), _ptr(y), x.size)
    _check("quantize_row_q8_0")
    return y


def dequantize_row(src, type_, n):
    """Packed row bytes -> float32[n] (src/quant.c:160)."""
    out = np.zeros(n, dtype=np.float32)
    s = None if src is None else np.ascontiguousarray(src)
    lib().dequantize_row(_ptr(out), _ptr(s), type_, n)
    _check("dequantize_row")
    return out


def vec_dot(type_, a, b, k):
    """One packed weight row `a` (k columns) . packed Q8_0 activations `b`."""
    a = np.ascontiguousarray(a, dtype=np.uint8)
    b = np.ascontiguousarray(b, dtype=np.uint8)
    fn = {Q8_0: "vec_dot_q8_0_q8_0", Q4_K: "vec_dot_q4K_q8_0", Q5_K: "vec_dot_q5K_q8_0",
          Q6_K: "vec_dot_q6K_q8_0"}[type_]
    r = getattr(lib(), fn)(_ptr(a), _ptr(b), k)
    _check(fn)
    return np.float32(r)


def matmul_q_fused(x, w, type_, n, d, threads=1, out=None):
    """out[i] = row_i(w) . x (src/quant.c:441).  w: packed bytes (host)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if out is None:
        out = np.empty(n, dtype=np.float32)
    wp = None if w is None else (w if isinstance(w, ctypes.c_void_p) else _ptr(np.ascontiguousarray(w)))
    lib().matmul_q_fused(_ptr(out), _ptr(x), wp, type_, n, d, threads)
    _check("matmul_q_fused")
    return out


def matmul_q_fused_batch(x, w, type_, n, d):
    """x: float32[B, d] -> float32[B, n]; B independent matmul_q_fused calls."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    B = x.shape[0]
    out = np.empty((B, n), dtype=np.float32)
    lib().matmul_q_fused_batch(_ptr(out), _ptr(x), _ptr(np.ascontiguousarray(w)), type_, n, d, B)
    _check("matmul_q_fused_batch")
    return out


def register_weights(w):
    """Makes the host bytes of `w` device-resident for later Part 1 calls."""
    rc = lib().quantr_gpu_register_weights(_ptr(w), w.nbytes)
    if rc:
        raise QuantrError(rc, "quantr_gpu_register_weights")


def unregister_weights(w):
    rc = lib().quantr_gpu_unregister_weights(_ptr(w))
    if rc:
        raise QuantrError(rc, "quantr_gpu_unregister_weights")


def launch_count():
    return int(lib().quantr_gpu_launch_count())


# ------------------------------------------------------------ device API --

def workspace_bytes(d, B=1):
    return int(lib().quantr_gemv_workspace_bytes(d, B))


def gemv_dev(out, ldo, x, ldx, w, type_, n, d, B, ws, ws_bytes, stream=0):
    rc = lib().quantr_gemv_dev(out, ldo, x, ldx, w, type_, n, d, B, ws, ws_bytes, stream or None)
    if rc:
        raise QuantrError(rc, "quantr_gemv_dev")


def gemv_q8act_dev(out, ldo, xq, w, type_, n, d, B, ws, ws_bytes, stream=0):
    rc = lib().quantr_gemv_q8act_dev(out, ldo, xq, w, type_, n, d, B, ws, ws_bytes, stream or None)
    if rc:
        raise QuantrError(rc, "quantr_gemv_q8act_dev")


def quantize_q8_0_dev(y, x, ldx, k, B, stream=0):
    rc = lib().quantr_quantize_q8_0_dev(y, x, ldx, k, B, stream or None)
    if rc:
        raise QuantrError(rc, "quantr_quantize_q8_0_dev")


def dequantize_rows_dev(out, ldo, src, src_stride, type_, n, rows, stream=0):
    rc = lib().quantr_dequantize_rows_dev(out, ldo, src, src_stride, type_, n, rows, stream or None)
    if rc:
        raise QuantrError(rc, "quantr_dequantize_rows_dev")


def gemv_partials_dev(out, isum, bsum, x, w, type_, n, d, B, ws, ws_bytes, stream=0):
    rc = lib().quantr_gemv_partials_dev(out, isum, bsum, x, w, type_, n, d, B, ws, ws_bytes, stream or None)
    if rc:
        raise QuantrError(rc, "quantr_gemv_partials_dev")


def gemv_noalloc_dev(out, ldo, x, ldx, w, type_, n, d, B, stream=0):
    """quantr_gemv_dev without a workspace: uses the library's fixed scratch."""
    rc = lib().quantr_gemv_noalloc_dev(out, ldo, x, ldx, w, type_, n, d, B, stream or None)
    if rc:
        raise QuantrError(rc, "quantr_gemv_noalloc_dev")


class Program:
    """A GEMV program: many independent device GEMVs run by one engine launch.

    jobs: iterable of (w_ptr, type, n, d, B, x_ptr, ldx, out_ptr, ldo) with
    device addresses as ints.  Created on the current CUDA device."""

    def __init__(self, jobs):
        jobs = list(jobs)
        arr = (GemvJob * len(jobs))(*[GemvJob(*j) for j in jobs])
        h = ctypes.c_void_p()
        rc = lib().quantr_program_create(ctypes.byref(h), ctypes.cast(arr, ctypes.c_void_p), len(jobs))
        if rc:
            raise QuantrError(rc, "quantr_program_create")
        self._h = h
        self.njobs = len(jobs)

    def run(self, stream=0):
        rc = lib().quantr_program_run(self._h, stream or None)
        if rc:
            raise QuantrError(rc, "quantr_program_run")

    def info(self):
        a, b, c = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        lib().quantr_program_info(self._h, ctypes.byref(a), ctypes.byref(b), ctypes.byref(c))
        return {"items": a.value, "grid": b.value, "smem": c.value}

    def close(self):
        if self._h:
            lib().quantr_program_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ------------------------------------------------------------------- MoE --

def moe_workspace_bytes(T, E, k, dim, hidden):
    return int(lib().quantr_moe_workspace_bytes(T, E, k, dim, hidden))


def moe_dev(out, ldo, xb, ldx, T, E, k, w1, w3, w2, dim, hidden, ws, ws_bytes, router=None, logits=None, ldl=0,
            sel=None, wts=None, stream=0):
    """quantr_moe_dev.  w1/w3/w2: ExpertWeights; pointers are device addresses."""
    rc = lib().quantr_moe_dev(out, ldo, xb, ldx, T, router, logits, ldl, E, k, ctypes.byref(w1), ctypes.byref(w3),
                              ctypes.byref(w2), dim, hidden, sel, wts, ws, ws_bytes, stream or None)
    if rc:
        raise QuantrError(rc, "quantr_moe_dev")


def moe_route_dev(sel, wts, xb, ldx, T, E, k, dim, ws, ws_bytes, router=None, logits=None, ldl=0, stream=0):
    rc = lib().quantr_moe_route_dev(sel, wts, xb, ldx, T, router, logits, ldl, E, k, dim, ws, ws_bytes,
                                    stream or None)
    if rc:
        raise QuantrError(rc, "quantr_moe_route_dev")


def moe_experts_dev(o, xb, ldx, T, sel, k, e0, E_local, w1, w3, w2, dim, hidden, ws, ws_bytes, stream=0):
    rc = lib().quantr_moe_experts_dev(o, xb, ldx, T, sel, k, e0, E_local, ctypes.byref(w1), ctypes.byref(w3),
                                      ctypes.byref(w2), dim, hidden, ws, ws_bytes, stream or None)
    if rc:
        raise QuantrError(rc, "quantr_moe_experts_dev")


def moe_combine_dev(out, ldo, o, sel, wts, T, k, dim, stream=0):
    rc = lib().quantr_moe_combine_dev(out, ldo, o, sel, wts, T, k, dim, stream or None)
    if rc:
        raise QuantrError(rc, "quantr_moe_combine_dev")


def moe_shared_dev(out, ldo, xb, ldx, T, gate, w1, t1, w3, t3, w2, t2, dim, hidden, stream=0):
    """quantr_moe_shared_dev: out += sigmoid(gate.xb) * shared-expert FFN(xb)."""
    rc = lib().quantr_moe_shared_dev(out, ldo, xb, ldx, T, gate, w1, t1, w3, t3, w2, t2, dim, hidden,
                                     stream or None)
    if rc:
        raise QuantrError(rc, "quantr_moe_shared_dev")


def moe_layer(xb, E, k, w1, t1, w3, t3, w2, t2, dim, hidden, router=None, logits=None):
    """quantr_moe_layer with host arrays.  w1/w3/w2: lists of E host arrays
    (views into registered arrays); returns (out, sel, wts, rc)."""
    xb = np.ascontiguousarray(xb, np.float32).reshape(-1, dim)
    T = xb.shape[0]
    out = np.empty((T, dim), np.float32)
    sel = np.empty((T, k), np.int32)
    wts = np.empty((T, k), np.float32)
    tabs = [(ctypes.c_void_p * E)(*[m.ctypes.data for m in mats]) for mats in (w1, w3, w2)]
    r = None if router is None else np.ascontiguousarray(router, np.float32)
    lg = None if logits is None else np.ascontiguousarray(logits, np.float32)
    rc = lib().quantr_moe_layer(_ptr(out), _ptr(xb), T, _ptr(r), _ptr(lg), E, k, ctypes.cast(tabs[0], _vp), t1,
                                ctypes.cast(tabs[1], _vp), t3, ctypes.cast(tabs[2], _vp), t2, dim, hidden, _ptr(sel),
                                _ptr(wts))
    lib().quantr_gpu_clear_error()
    return out, sel, wts, rc


def device_status(stream=0, reset=True):
    return int(lib().quantr_gpu_device_status(stream or None, 1 if reset else 0))


# --------------------------------------------------------------- decoder --

_P = ctypes.POINTER


class Model(ctypes.Structure):
    """quantr_model (include/quantr_cuda.h)."""
    _fields_ = [("dim", _i), ("hidden_dim", _i), ("n_layers", _i), ("n_heads", _i), ("n_kv_heads", _i),
                ("vocab_size", _i), ("seq_len", _i), ("rope_freq_base", _f), ("expert_count", _i),
                ("expert_used_count", _i), ("kv_type", _i), ("token_embd", _vp), ("token_embd_type", _u32),
                ("token_embd_row_bytes", _sz)] + \
        [(n, _P(_vp)) for n in ("rms_att", "rms_ffn", "wq", "wk", "wv", "wo", "w1", "w2", "w3")] + \
        [(n, _P(_u32)) for n in ("wq_type", "wk_type", "wv_type", "wo_type", "w1_type", "w2_type", "w3_type")] + \
        [("rms_final", _vp), ("wcls", _vp), ("wcls_type", _u32), ("ffn_gate_inp", _P(_vp)),
         ("expert_w1", _P(_P(_vp))), ("expert_w2", _P(_P(_vp))), ("expert_w3", _P(_P(_vp))),
         ("exp_w1_type", _P(_u32)), ("exp_w2_type", _P(_u32)), ("exp_w3_type", _P(_u32)),
         ("head_dim", _i), ("shexp_hidden_dim", _i), ("shexp_w1", _P(_vp)), ("shexp_w2", _P(_vp)),
         ("shexp_w3", _P(_vp)), ("shexp_w1_type", _P(_u32)), ("shexp_w2_type", _P(_u32)),
         ("shexp_w3_type", _P(_u32)), ("shexp_gate", _P(_vp))]


def describe_model(model):
    """quantr_model over a model_synth.Model's host buffer (host pointers into
    one mapping, as the reference's TransformerWeights are).  Returns the
    struct and the pointer arrays it references (keep both alive)."""
    s = model.spec
    L = s.n_layers
    keep = []

    def arr(ctype, vals):
        a = (ctype * max(len(vals), 1))(*vals)
        keep.append(a)
        return ctypes.cast(a, _P(ctype))

    def ptrs(names):
        return arr(_vp, [model.ptr(n) if n in model.off else None for n in names])

    def types(names):
        return arr(_u32, [model.type_of(n) if n in model.off else 0 for n in names])

    m = Model()
    m.dim, m.hidden_dim, m.n_layers, m.n_heads = s.dim, s.hidden_dim, L, s.n_heads
    m.n_kv_heads, m.vocab_size, m.seq_len, m.rope_freq_base = s.n_kv_heads, s.vocab_size, s.seq_len, s.rope_freq_base
    m.expert_count, m.expert_used_count, m.kv_type = s.expert_count, s.expert_used_count, s.kv_type
    m.token_embd = model.ptr("token_embd")
    m.token_embd_type = model.type_of("token_embd")
    m.token_embd_row_bytes = 0 if s.embd_type == F32 else row_bytes(s.embd_type, s.dim)
    m.rms_att = ptrs([f"rms_att.{l}" for l in range(L)])
    m.rms_ffn = ptrs([f"rms_ffn.{l}" for l in range(L)])
    for w in ("wq", "wk", "wv", "wo", "w1", "w2", "w3"):
        setattr(m, w, ptrs([f"{w}.{l}" for l in range(L)]))
        setattr(m, w + "_type", types([f"{w}.{l}" for l in range(L)]))
    m.rms_final = model.ptr("rms_final")
    m.wcls = model.ptr("wcls")
    m.wcls_type = model.type_of("wcls")
    if s.expert_count:
        m.ffn_gate_inp = ptrs([f"router.{l}" for l in range(L)])
        for w in ("exp_w1", "exp_w2", "exp_w3"):
            per_layer = [arr(_vp, [model.expert_ptr(w, l, e) for e in range(s.expert_count)]) for l in range(L)]
            setattr(m, "expert_" + w[4:], arr(_P(_vp), per_layer))
            setattr(m, w + "_type", types([f"{w}.{l}" for l in range(L)]))
    m.head_dim = s.head_dim
    if s.shexp_hidden_dim:
        m.shexp_hidden_dim = s.shexp_hidden_dim
        for w in ("shexp_w1", "shexp_w2", "shexp_w3"):
            setattr(m, w, ptrs([f"{w}.{l}" for l in range(L)]))
            setattr(m, w + "_type", types([f"{w}.{l}" for l in range(L)]))
        m.shexp_gate = ptrs([f"shexp_gate.{l}" for l in range(L)])
    return m, keep


class Decoder:
    """The device-resident decoder (quantr_decoder_*) over a model_synth.Model.

    The model's host buffer (its "GGUF mapping") is registered once with
    quantr_gpu_register_weights and the decoder is handed host pointers into
    it, the way the reference's runtime would drive it."""

    def __init__(self, model, batch=1, register=True):
        self.model = model
        self.batch = batch
        self._registered = False
        if register:
            register_weights(model.buf)
            self._registered = True
        self._m, self._keep = describe_model(model)
        h = ctypes.c_void_p()
        rc = lib().quantr_decoder_create(ctypes.byref(h), ctypes.byref(self._m), batch)
        if rc:
            self._unregister()
            raise QuantrError(rc, "quantr_decoder_create")
        self._h = h

    def generate(self, prompt, steps):
        """src/main.c:305-317 for every sequence: prompt int32[batch, n] ->
        int32[batch, steps] greedy tokens."""
        p = np.ascontiguousarray(np.asarray(prompt, np.int32).reshape(self.batch, -1))
        out = np.zeros((self.batch, steps), np.int32)
        rc = lib().quantr_decoder_generate(self._h, _ptr(p), p.shape[1], steps, _ptr(out))
        if rc:
            raise QuantrError(rc, "quantr_decoder_generate")
        return out

    def forward_runtime(self, token, pos):
        r = lib().quantr_forward_runtime(self._h, int(token), int(pos))
        if not r:
            raise QuantrError(QUANTR_ERR_BAD_ARG, "quantr_forward_runtime")
        return np.ctypeslib.as_array(r, shape=(self.model.spec.vocab_size,)).copy()

    def prefill_runtime(self, tokens):
        t = np.ascontiguousarray(tokens, np.int32)
        lib().quantr_prefill_runtime(self._h, _ptr(t), t.size)

    def step_dev(self, tokens, pos, logits=None, ldl=0, next_=None, stream=0):
        rc = lib().quantr_decoder_step_dev(self._h, tokens, pos, logits, ldl, next_, stream or None)
        if rc:
            raise QuantrError(rc, "quantr_decoder_step_dev")

    def generate_dev(self, prompt, n_prompt, steps, out, stream=0):
        """Device arrays, asynchronous: out is steps x batch (step-major)."""
        rc = lib().quantr_decoder_generate_dev(self._h, prompt, n_prompt, steps, out, stream or None)
        if rc:
            raise QuantrError(rc, "quantr_decoder_generate_dev")

    def kv(self):
        """(key cache, value cache) device addresses and bytes of each."""
        k, v, n = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_size_t()
        lib().quantr_decoder_kv(self._h, ctypes.byref(k), ctypes.byref(v), ctypes.byref(n))
        return k.value, v.value, n.value

    def info(self):
        a, b, c = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_size_t()
        lib().quantr_decoder_info(self._h, ctypes.byref(a), ctypes.byref(b), ctypes.byref(c))
        x, y = ctypes.c_int(), ctypes.c_int()
        lib().quantr_decoder_launches(self._h, ctypes.byref(x), ctypes.byref(y))
        return {"weight_bytes_per_step": a.value, "kv_bytes_per_position": b.value, "device_bytes": c.value,
                "launches_per_decode_step": x.value, "launches_per_prefill_step": y.value}

    def _unregister(self):
        if self._registered:
            unregister_weights(self.model.buf)
            self._registered = False

    def close(self):
        if getattr(self, "_h", None):
            lib().quantr_decoder_destroy(self._h)
            self._h = None
        self._unregister()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


QUANTR_ERR_BAD_ARG = 3
