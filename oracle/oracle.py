"""ctypes bindings for the parity checkers.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline / reference legs -- never by the product path.

Two libraries share one Python surface:

* ``liboracle.so``      -- oracle/attn_oracle.c, the C restatement of the
  reference's rope()/softmax()/attention() (src/ops.cpp:1072-1515), and
  oracle/forward_oracle.c: matmul() of every weight format, rmsnorm(),
  ffn_swiglu(), vec_add(), sample_argmax() and forward()
  (src/ops.cpp:119-1597, src/forward.cpp:178-265).
* ``_ref/libref_attn.so`` -- the reference's own src/ops.cpp compiled
  unmodified (oracle/Makefile) with oracle/ref_harness.cpp.

All arrays are float32 numpy arrays; functions mutate exactly what the
reference mutates (q/k rotated in place, cache rows appended).
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libref_attn.so")

_f = ctypes.POINTER(ctypes.c_float)
_pp = ctypes.POINTER(ctypes.c_void_p)
_i = ctypes.c_int


def _fp(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"], (a.dtype, a.flags)
    return a.ctypes.data_as(_f)


_u8p = ctypes.POINTER(ctypes.c_uint8)


class FwWeight(ctypes.Structure):
    _fields_ = [("type", ctypes.c_int32), ("pad", ctypes.c_int32), ("data", ctypes.c_void_p)]


class FwLayer(ctypes.Structure):
    _fields_ = [(n, FwWeight) for n in ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down")] + \
               [("attn_norm", ctypes.c_void_p), ("ffn_norm", ctypes.c_void_p)]


class FwModel(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("n_layers", "n_embd", "n_head", "n_head_kv",
                                               "n_ff", "n_vocab", "n_ctx")] + \
               [("rope_freq_base", ctypes.c_float), ("rms_norm_eps", ctypes.c_float),
                ("pad", ctypes.c_int32), ("token_embd", FwWeight), ("output", FwWeight),
                ("output_norm", ctypes.c_void_p), ("layers", ctypes.POINTER(FwLayer))]


class FwState(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in ("x", "xb", "xb2", "q", "k", "v", "hb", "hb2",
                                                "logits", "key_cache", "value_cache", "att")]


class HostForward:
    """A synthetic model (tinyllama-engine_b200/synth.py) and a RunState on
    the host, for the oracle's (or the reference's) forward()."""

    _LAYER = (("wq", "attn_q"), ("wk", "attn_k"), ("wv", "attn_v"), ("wo", "attn_output"),
              ("w_gate", "ffn_gate"), ("w_up", "ffn_up"), ("w_down", "ffn_down"))

    def __init__(self, model):
        m = model
        self.model = m
        z = lambda n: np.zeros(n, np.float32)  # noqa: E731
        kv = m.kv_dim
        self.bufs = {"x": z(m.n_embd), "xb": z(m.n_embd), "xb2": z(m.n_embd), "q": z(m.n_embd),
                     "k": z(kv), "v": z(kv), "hb": z(m.n_ff), "hb2": z(m.n_ff),
                     "logits": z(m.n_vocab), "key_cache": z(m.n_layers * m.n_ctx * kv),
                     "value_cache": z(m.n_layers * m.n_ctx * kv), "att": z(m.n_ctx)}
        self.state = FwState(**{k: v.ctypes.data for k, v in self.bufs.items()})
        w = lambda W: FwWeight(W.wtype, 0, W.data.ctypes.data)  # noqa: E731
        self.layers = (FwLayer * m.n_layers)()
        for i, L in enumerate(m.layers):
            for f, n in self._LAYER:
                setattr(self.layers[i], f, w(L[n]))
            self.layers[i].attn_norm = L["attn_norm"].ctypes.data
            self.layers[i].ffn_norm = L["ffn_norm"].ctypes.data
        out = w(m.output) if m.output is not None else FwWeight(0, 0, None)
        self.fw = FwModel(m.n_layers, m.n_embd, m.n_head, m.n_head_kv, m.n_ff, m.n_vocab,
                          m.n_ctx, m.rope_freq_base, m.rms_norm_eps, 0, w(m.token_embd), out,
                          m.output_norm.ctypes.data, self.layers)

    @property
    def logits(self) -> np.ndarray:
        return self.bufs["logits"]


class _Lib:
    def __init__(self, path: str, prefix: str):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} not built (run `make -C oracle`)")
        self.path = path
        self.lib = ctypes.CDLL(path)
        self.prefix = prefix
        L, p = self.lib, prefix
        getattr(L, p + "rope").argtypes = [_f, _f, _i, _i, _i, _i, ctypes.c_float]
        getattr(L, p + "softmax").argtypes = [_f, _i]
        getattr(L, p + "prefill").argtypes = (
            [_f, _f, _f, _f, _f, _f] + [_i] * (8 if p == "ref_" else 7) + [ctypes.c_float])
        getattr(L, p + "decode_batch").argtypes = (
            [_i, _pp, _pp, ctypes.POINTER(_i), ctypes.POINTER(_i), _f, _f, _f, _f]
            + [_i] * (5 if p == "ref_" else 4) + [ctypes.c_float, _i])

    def _fn(self, name, argtypes, restype=None):
        f = getattr(self.lib, self.prefix + name)
        f.argtypes = argtypes
        f.restype = restype
        return f

    # ops.h:39
    def fp16_to_f32(self, h: np.ndarray) -> np.ndarray:
        f = self._fn("fp16_to_f32", [ctypes.c_uint16], ctypes.c_float)
        return np.array([f(int(x)) for x in np.asarray(h, np.uint16).ravel()], np.float32)

    # ops.h:64-66: W is a flat uint8 array in the GGUF layout of `wtype`
    def matmul(self, out, W, x, rows, cols, wtype):
        f = self._fn("matmul", [_f, ctypes.c_void_p, _f, _i, _i, _i], _i)
        if f(_fp(out), W.ctypes.data, _fp(x), rows, cols, wtype):
            raise ValueError(f"unsupported weight type {wtype}")

    # ops.h:95-96
    def rmsnorm(self, out, x, weight, eps=1e-5):
        self._fn("rmsnorm", [_f, _f, _f, _i, ctypes.c_float])(_fp(out), _fp(x), _fp(weight),
                                                               x.size, ctypes.c_float(eps))

    def silu(self, x):
        self._fn("silu", [_f, _i])(_fp(x), x.size)

    def elementwise_mul(self, a, b):
        self._fn("elementwise_mul", [_f, _f, _i])(_fp(a), _fp(b), a.size)

    def vec_add(self, out, x):
        self._fn("vec_add", [_f, _f, _i])(_fp(out), _fp(x), out.size)

    # ops.h:232-235
    def ffn_swiglu(self, out, inp, W_gate, W_up, W_down, n_ff, n_embd, wtype):
        hb = np.zeros(n_ff, np.float32)
        hb2 = np.zeros(n_ff, np.float32)
        f = self._fn("ffn_swiglu", [_f, _f, _f, _f] + [ctypes.c_void_p] * 3 + [_i] * 3, _i)
        if f(_fp(out), _fp(inp), _fp(hb), _fp(hb2), W_gate.ctypes.data, W_up.ctypes.data,
             W_down.ctypes.data, n_ff, n_embd, wtype):
            raise ValueError(f"unsupported weight type {wtype}")

    # ops.h:249
    def sample_argmax(self, logits) -> int:
        return int(self._fn("sample_argmax", [_f, _i], _i)(_fp(logits), logits.size))

    # ops.h:262 / 278 with the uniform draw r given (port only: the reference
    # draws r from its own unseeded generator, see sample_top_p_reference)
    def sample_temperature(self, logits, temperature, r) -> int:
        f = self._fn("sample_temperature", [_f, _i, ctypes.c_float, ctypes.c_float], _i)
        return int(f(_fp(logits), logits.size, temperature, r))

    def sample_top_p(self, logits, temperature, top_p, r) -> int:
        f = self._fn("sample_top_p", [_f, _i, ctypes.c_float, ctypes.c_float, ctypes.c_float], _i)
        return int(f(_fp(logits), logits.size, temperature, top_p, r))

    # the reference's own sample_top_p (its internal random draw)
    def sample_top_p_reference(self, logits, temperature, top_p) -> int:
        f = self._fn("sample_top_p", [_f, _i, ctypes.c_float, ctypes.c_float], _i)
        return int(f(_fp(logits), logits.size, temperature, top_p))

    # forward.cpp:178-265 on a HostForward (logits in hf.logits)
    def forward(self, hf: "HostForward", token: int, pos: int):
        f = self._fn("forward", [ctypes.POINTER(FwModel), ctypes.POINTER(FwState), _i, _i], _i)
        if f(ctypes.byref(hf.fw), ctypes.byref(hf.state), token, pos):
            raise ValueError("unsupported model format")
        return hf.logits

    # ops.h:175-176
    def rope(self, q, k, pos, head_dim=64, n_head=32, n_head_kv=4, freq_base=10000.0):
        getattr(self.lib, self.prefix + "rope")(_fp(q), _fp(k), pos, head_dim, n_head,
                                                n_head_kv, ctypes.c_float(freq_base))

    # ops.h:107
    def softmax(self, x):
        getattr(self.lib, self.prefix + "softmax")(_fp(x), x.size)

    # ops.h:204-206 (q, k already rotated, as in the reference)
    def attention(self, out, q, k, v, key_cache, value_cache, layer, pos, n_ctx,
                  n_head=32, n_head_kv=4, head_dim=64, n_layers=None):
        att = np.zeros(n_ctx, np.float32)
        if self.prefix == "ref_":
            if n_layers is None:
                n_layers = key_cache.size // (n_ctx * n_head_kv * head_dim)
            self.lib.ref_attention(_fp(out), _fp(q), _fp(k), _fp(v), _fp(key_cache),
                                   _fp(value_cache), _fp(att), layer, pos, n_layers, n_ctx,
                                   n_head, n_head_kv, head_dim)
        else:
            self.lib.oracle_attention(_fp(out), _fp(q), _fp(k), _fp(v), _fp(key_cache),
                                      _fp(value_cache), _fp(att), layer, pos, n_ctx, n_head,
                                      n_head_kv, head_dim)
        return att

    # S successive rope+attention steps (generate.cpp:56-59)
    def prefill(self, out, q, k, v, key_cache, value_cache, layer, pos0, n_ctx,
                n_head=32, n_head_kv=4, head_dim=64, freq_base=10000.0):
        n_tokens = q.shape[0]
        if self.prefix == "ref_":
            n_layers = key_cache.size // (n_ctx * n_head_kv * head_dim)
            self.lib.ref_prefill(_fp(out), _fp(q), _fp(k), _fp(v), _fp(key_cache),
                                 _fp(value_cache), layer, pos0, n_tokens, n_layers, n_ctx,
                                 n_head, n_head_kv, head_dim, ctypes.c_float(freq_base))
        else:
            self.lib.oracle_prefill(_fp(out), _fp(q), _fp(k), _fp(v), _fp(key_cache),
                                    _fp(value_cache), layer, pos0, n_tokens, n_ctx, n_head,
                                    n_head_kv, head_dim, ctypes.c_float(freq_base))

    # one fused rope+attention step for each of several independent sequences
    def decode_batch(self, key_caches, value_caches, n_ctx, pos, q, k, v, out, layer,
                     n_head=32, n_head_kv=4, head_dim=64, freq_base=10000.0, n_threads=1,
                     n_layers=None):
        n = len(key_caches)
        kp = (ctypes.c_void_p * n)(*[c.ctypes.data for c in key_caches])
        vp = (ctypes.c_void_p * n)(*[c.ctypes.data for c in value_caches])
        nc = np.ascontiguousarray(n_ctx, dtype=np.int32)
        ps = np.ascontiguousarray(pos, dtype=np.int32)
        ip = ctypes.POINTER(_i)
        common = [n, ctypes.cast(kp, _pp), ctypes.cast(vp, _pp), nc.ctypes.data_as(ip),
                  ps.ctypes.data_as(ip), _fp(q), _fp(k), _fp(v), _fp(out), layer]
        if self.prefix == "ref_":
            if n_layers is None:
                n_layers = key_caches[0].size // (int(nc[0]) * n_head_kv * head_dim)
            self.lib.ref_decode_batch(*common, n_layers, n_head, n_head_kv, head_dim,
                                      ctypes.c_float(freq_base), n_threads)
        else:
            self.lib.oracle_decode_batch(*common, n_head, n_head_kv, head_dim,
                                         ctypes.c_float(freq_base), n_threads)


_cache: dict = {}


def port() -> _Lib:
    """The C restatement (always available once `make -C oracle` ran)."""
    if "port" not in _cache:
        _cache["port"] = _Lib(ORACLE_SO, "oracle_")
    return _cache["port"]


def reference() -> _Lib:
    """The reference's own ops.cpp, compiled unmodified."""
    if "ref" not in _cache:
        _cache["ref"] = _Lib(REF_SO, "ref_")
    return _cache["ref"]


def have_reference() -> bool:
    return os.path.exists(REF_SO)
