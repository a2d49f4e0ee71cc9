"""ctypes driver of the decoder-step oracles.  TEST INFRASTRUCTURE ONLY.

Only tests/ and bench.py's CPU-baseline leg may import this module.

  Restated(model)        -> qo_open/qo_forward/qo_generate of
                            _build/libquant_oracle.so (forward_oracle.c), the
                            restatement of src/runtime.c:94-289 that also
                            takes an explicit head_dim and a shared expert.
  Reference(model, ...)  -> ref_open/ref_forward/ref_generate of
                            _ref/libquantr_ref_forward_<variant>.so: the
                            reference's own forward_runtime, prefill_runtime
                            and sample_next compiled from its sources
                            (oracle/Makefile), Q4_K dot product restated in
                            the "scalar" build, unmodified in "avx512".

`model` is a model_synth.Model: one host buffer holding every tensor, the
same bytes the device decoder registers.
"""
import ctypes
import os

import numpy as np

import oracle

_vp, _i, _u32, _f, _sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint32, ctypes.c_float, ctypes.c_size_t
_P = ctypes.POINTER


class QoModel(ctypes.Structure):
    """qo_model (oracle/quant_oracle.h); its prefix is ref_forward.c's ref_model."""
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


def describe(model):
    """QoModel over model.buf (host pointers); the return keeps every pointer
    array alive while the struct is in use."""
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

    m = QoModel()
    m.dim, m.hidden_dim, m.n_layers, m.n_heads = s.dim, s.hidden_dim, L, s.n_heads
    m.n_kv_heads, m.vocab_size, m.seq_len, m.rope_freq_base = s.n_kv_heads, s.vocab_size, s.seq_len, s.rope_freq_base
    m.expert_count, m.expert_used_count, m.kv_type = s.expert_count, s.expert_used_count, s.kv_type
    m.token_embd = model.ptr("token_embd")
    m.token_embd_type = model.type_of("token_embd")
    m.token_embd_row_bytes = 0 if s.embd_type == 0 else (s.dim // (32 if s.embd_type == 8 else 256)) * \
        {8: 34, 12: 144, 13: 176, 14: 210}[s.embd_type]
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


class _Runner:
    OPEN = CLOSE = FWD = GEN = None

    def __init__(self, L, model, open_args):
        self.L = L
        self.model = model
        self.m, self._keep = describe(model)
        self.h = getattr(L, self.OPEN)(ctypes.byref(self.m), *open_args)
        if not self.h:
            raise MemoryError("oracle state allocation failed")

    def close(self):
        if self.h:
            getattr(self.L, self.CLOSE)(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def generate(self, prompt, steps, want_logits=False):
        """src/main.c:305-317 greedy loop: (tokens[steps], logits[steps, vocab] or None)."""
        p = np.ascontiguousarray(prompt, np.int32)
        toks = np.zeros(steps, np.int32)
        logits = np.zeros((steps, self.model.spec.vocab_size), np.float32) if want_logits else None
        getattr(self.L, self.GEN)(self.h, p.ctypes.data_as(_vp), p.size, steps, toks.ctypes.data_as(_vp),
                                  None if logits is None else logits.ctypes.data_as(_vp))
        return toks, logits


class Restated(_Runner):
    OPEN, CLOSE, GEN = "qo_open", "qo_close", "qo_generate"

    def __init__(self, model, threads=None):
        L = ctypes.CDLL(oracle.ORACLE_SO)
        L.qo_open.restype = _vp
        L.qo_open.argtypes = [_vp, _i]
        L.qo_close.argtypes = [_vp]
        L.qo_forward.restype = _P(_f)
        L.qo_forward.argtypes = [_vp, _i, _i]
        L.qo_generate.argtypes = [_vp, _vp, _i, _i, _vp, _vp]
        super().__init__(L, model, (threads or os.cpu_count(),))

    def forward(self, token, pos):
        p = self.L.qo_forward(self.h, int(token), int(pos))
        return np.ctypeslib.as_array(p, shape=(self.model.spec.vocab_size,)).copy()


class Reference(_Runner):
    OPEN, CLOSE, GEN = "ref_open", "ref_close", "ref_generate"

    def __init__(self, model, variant="scalar", threads=None, backend=0):
        path = os.path.join(oracle.REF_DIR, f"libquantr_ref_forward_{variant}.so")
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        if model.spec.head_dim and model.spec.head_dim != model.spec.dim // model.spec.n_heads:
            raise ValueError("the reference derives head_dim = dim / n_heads")
        if model.spec.shexp_hidden_dim:
            raise ValueError("the reference has no shared expert")
        L = ctypes.CDLL(path)
        L.ref_open.restype = _vp
        L.ref_open.argtypes = [_vp, _i, _i]
        L.ref_close.argtypes = [_vp]
        L.ref_forward.argtypes = [_vp, _i, _i, _vp]
        L.ref_generate.argtypes = [_vp, _vp, _i, _i, _vp, _vp]
        self.variant = variant
        super().__init__(L, model, (backend, threads or os.cpu_count()))

    def forward(self, token, pos):
        out = np.zeros(self.model.spec.vocab_size, np.float32)
        self.L.ref_forward(self.h, int(token), int(pos), out.ctypes.data_as(_vp))
        return out


def reference_available(variant="scalar"):
    return os.path.exists(os.path.join(oracle.REF_DIR, f"libquantr_ref_forward_{variant}.so"))
