"""ctypes bindings for the parity checkers.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline / reference legs -- never by the product path.

Two libraries share one Python surface:

* ``liboracle.so``      -- oracle/attn_oracle.c, the C restatement of the
  reference's rope()/softmax()/attention() (src/ops.cpp:1072-1515).
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
