"""Python plumbing over the C ABI in include/tle_attn.h (libtle_attn.so).

The product is the C ABI and the sm_100a kernels behind it; this module only
marshals torch CUDA tensors (device memory, streams) into those calls, the
way the reference's callers pass raw float pointers (src/ops.h:175-206).
There is no fallback: if libtle_attn.so is missing or a call fails, an
exception is raised.

Names follow the reference: ``rope`` (ops.h:175), ``attention`` (ops.h:204),
``rope_attention`` (forward.cpp:192-208 fused), ``DecodeBatch`` (attention()
for many sequences), ``prefill`` (generate.cpp:56-59 as one causal kernel).
"""
from __future__ import annotations

import ctypes
import os
from typing import Iterable, List, Optional, Sequence

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libtle_attn.so")

TLE_OK = 0
TLE_ERR_INVALID = 1
TLE_ERR_UNSUPPORTED = 2
TLE_ERR_WORKSPACE = 3
TLE_ERR_CUDA = 4
TLE_ERR_DEVICE = 5

TLE_DECODE_ROTATE = 1
TLE_DECODE_KV_READY = 2


def _decode_flags(rotate: bool, kv_ready: bool) -> int:
    return (TLE_DECODE_ROTATE if rotate else 0) | (TLE_DECODE_KV_READY if kv_ready else 0)

# Every symbol include/tle_attn.h declares (tests check the .so exports them).
EXPORTED = (
    "tle_last_error", "tle_version", "tle_rope", "tle_attention_workspace_bytes",
    "tle_attention", "tle_rope_attention", "tle_rope_attention_flags", "tle_decode_desc_bytes", "tle_decode_desc",
    "tle_decode_workspace_bytes", "tle_decode_batch", "tle_prefill_workspace_bytes",
    "tle_prefill", "tle_partition_lpt", "tle_device_error", "tle_decode_batch_noalloc",
    "tle_selftest_wait_timeout", "tle_attention_lse", "tle_merge_lse",
    "tle_decode_desc_paged", "tle_decode_batch_paged", "tle_decode_bf16_workspace_bytes",
    "tle_decode_batch_bf16", "tle_decode_batch_bf16_paged", "tle_decode_batch_short",
    # include/tle_forward.h
    "tle_matmul", "tle_rmsnorm", "tle_vec_add", "tle_ffn_swiglu", "tle_sample_argmax",
    "tle_forward_workspace_bytes", "tle_forward", "tle_forward_layers_one_launch", "tle_sample_temperature", "tle_sample_top_p",
    "tle_prompt_weights_bytes", "tle_prompt_pack_weights", "tle_prompt_scratch_bytes",
    "tle_prompt_forward",
)


class TleError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"tle error {code}: {msg}")
        self.code = code


class Shape(ctypes.Structure):
    """tle_shape_t: the llama_config_t fields attention reads (gguf.h:139-168)."""
    _fields_ = [("n_layers", ctypes.c_int32), ("n_head", ctypes.c_int32),
                ("n_head_kv", ctypes.c_int32), ("head_dim", ctypes.c_int32),
                ("rope_freq_base", ctypes.c_float)]


# DecodeBatch takes the cluster decode up to this many attended rows in all
# (measured on B200, 22-layer steps: one sequence of 2018 rows 11.5 against
# 18.1 us per layer for the split-K decode; 4 sequences of 5106 rows 22.1
# against 17.4; 64 sequences 202 against 33).
SHORT_MAX_ROWS = 2048


class Seq(ctypes.Structure):
    """tle_seq_t: one sequence's device KV cache and decode position."""
    _fields_ = [("key_cache", ctypes.c_void_p), ("value_cache", ctypes.c_void_p),
                ("n_ctx", ctypes.c_int32), ("pos", ctypes.c_int32)]


class PagePoolBf16(ctypes.Structure):
    """tle_page_pool_bf16_t: bf16 page pools."""
    _fields_ = [("key_pool", ctypes.c_void_p), ("value_pool", ctypes.c_void_p),
                ("n_pages", ctypes.c_int32), ("page_rows", ctypes.c_int32)]


class SeqBf16(ctypes.Structure):
    """tle_seq_bf16_t: the same record for a bf16 cache."""
    _fields_ = [("key_cache", ctypes.c_void_p), ("value_cache", ctypes.c_void_p),
                ("n_ctx", ctypes.c_int32), ("pos", ctypes.c_int32)]


class PagePool(ctypes.Structure):
    """tle_page_pool_t: the key/value page pools of a paged batch."""
    _fields_ = [("key_pool", ctypes.c_void_p), ("value_pool", ctypes.c_void_p),
                ("n_pages", ctypes.c_int32), ("page_rows", ctypes.c_int32)]


class PagedSeq(ctypes.Structure):
    """tle_paged_seq_t: one sequence's device page table and decode position."""
    _fields_ = [("pages", ctypes.c_void_p), ("n_pages", ctypes.c_int32), ("pos", ctypes.c_int32)]


class Weight(ctypes.Structure):
    """tle_weight_t: a device tensor in GGUF layout and its ggml type."""
    _fields_ = [("type", ctypes.c_int32), ("reserved", ctypes.c_int32), ("data", ctypes.c_void_p)]


class Layer(ctypes.Structure):
    """tle_layer_t: the tensors of one block (forward.cpp blk.l.*)."""
    _fields_ = [(n, Weight) for n in ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate",
                                      "ffn_up", "ffn_down")] + \
               [("attn_norm", ctypes.c_void_p), ("ffn_norm", ctypes.c_void_p)]


class Model(ctypes.Structure):
    """tle_model_t: llama_config_t fields and the global tensors."""
    _fields_ = [(n, ctypes.c_int32) for n in ("n_layers", "n_embd", "n_head", "n_head_kv", "n_ff",
                                               "n_vocab", "n_ctx")] + \
               [("rope_freq_base", ctypes.c_float), ("rms_norm_eps", ctypes.c_float),
                ("reserved", ctypes.c_int32), ("token_embd", Weight), ("output", Weight),
                ("output_norm", ctypes.c_void_p), ("layers", ctypes.POINTER(Layer))]


class State(ctypes.Structure):
    """tle_state_t: RunState buffers in device memory."""
    _fields_ = [(n, ctypes.c_void_p) for n in ("x", "xb", "xb2", "q", "k", "v", "hb", "hb2",
                                                "logits", "key_cache", "value_cache",
                                                "workspace")] + [("workspace_bytes", ctypes.c_size_t)]


def tinyllama_shape(n_layers: int = 22) -> Shape:
    return Shape(n_layers, 32, 4, 64, 10000.0)


_lib = None


def lib() -> ctypes.CDLL:
    """Loads libtle_attn.so (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(f"{LIB_PATH} missing: run `make` (or __graft_entry__.build())")
        L = ctypes.CDLL(LIB_PATH)
        vp, i, f, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t
        P = ctypes.POINTER
        L.tle_last_error.restype = ctypes.c_char_p
        L.tle_version.restype = ctypes.c_char_p
        L.tle_rope.argtypes = [vp, vp, i, i, i, i, f, vp]
        L.tle_attention_workspace_bytes.argtypes = [P(Shape), i]
        L.tle_attention_workspace_bytes.restype = sz
        for name in ("tle_attention", "tle_rope_attention"):
            getattr(L, name).argtypes = [vp, vp, vp, vp, vp, vp, i, i, i, P(Shape), vp, sz, vp]
        L.tle_rope_attention_flags.argtypes = [vp, vp, vp, vp, vp, vp, i, i, i, P(Shape), i, vp, sz, vp]
        L.tle_decode_desc_bytes.argtypes = [i, i]
        L.tle_decode_desc_bytes.restype = sz
        L.tle_decode_desc.argtypes = [P(Shape), P(Seq), i, i, vp, sz, P(i)]
        L.tle_decode_workspace_bytes.argtypes = [P(Shape), i, i]
        L.tle_decode_workspace_bytes.restype = sz
        L.tle_decode_batch.argtypes = [P(Shape), vp, i, i, vp, vp, vp, vp, i, i, vp, sz, vp]
        L.tle_decode_batch_short.argtypes = [P(Shape), vp, i, i, vp, vp, vp, vp, i, i, vp]
        L.tle_decode_bf16_workspace_bytes.argtypes = [i, i]
        L.tle_decode_bf16_workspace_bytes.restype = sz
        L.tle_decode_batch_bf16.argtypes = [P(Shape), vp, i, i, vp, vp, vp, vp, i, i, vp, sz, vp]
        L.tle_decode_batch_bf16_paged.argtypes = [P(Shape), vp, vp, i, i, vp, vp, vp, vp, i, i, vp, sz, vp]
        L.tle_prefill_workspace_bytes.argtypes = [P(Shape), i, i]
        L.tle_prefill_workspace_bytes.restype = sz
        L.tle_prefill.argtypes = [vp, vp, vp, vp, vp, vp, i, i, i, i, P(Shape), vp, sz, vp]
        L.tle_partition_lpt.argtypes = [P(ctypes.c_int32), i, i, P(ctypes.c_int32)]
        L.tle_device_error.argtypes = [i, P(ctypes.c_uint32)]
        L.tle_selftest_wait_timeout.argtypes = [ctypes.c_uint32, ctypes.c_void_p]
        L.tle_attention_lse.argtypes = [vp, vp, vp, vp, vp, vp, vp, i, i, i, P(Shape), vp, sz, vp]
        L.tle_merge_lse.argtypes = [vp, vp, vp, i, vp]
        L.tle_decode_batch_noalloc.argtypes = [P(Shape), P(Seq), i, vp, vp, vp, vp, i, i, vp]
        L.tle_matmul.argtypes = [vp, vp, vp, i, i, i, vp]
        L.tle_rmsnorm.argtypes = [vp, vp, vp, i, f, vp]
        L.tle_vec_add.argtypes = [vp, vp, i, vp]
        L.tle_ffn_swiglu.argtypes = [vp, vp, vp, vp, vp, vp, vp, i, i, i, vp]
        L.tle_sample_argmax.argtypes = [vp, i, vp, vp]
        L.tle_forward_workspace_bytes.argtypes = [P(Model)]
        L.tle_forward_workspace_bytes.restype = sz
        L.tle_forward_layers_one_launch.argtypes = [P(Model), P(State), i]
        L.tle_forward_layers_one_launch.restype = i
        L.tle_forward.argtypes = [P(Model), P(State), vp, i, vp]
        L.tle_sample_temperature.argtypes = [vp, i, f, f, vp, vp]
        L.tle_sample_top_p.argtypes = [vp, i, f, f, f, vp, vp]
        L.tle_decode_desc_paged.argtypes = [P(Shape), P(PagePool), P(PagedSeq), i, i, vp, sz, P(i)]
        L.tle_decode_batch_paged.argtypes = [P(Shape), P(PagePool), vp, i, i, vp, vp, vp, vp, i, i,
                                             vp, sz, vp]
        L.tle_prompt_weights_bytes.argtypes = [P(Model)]
        L.tle_prompt_weights_bytes.restype = sz
        L.tle_prompt_pack_weights.argtypes = [P(Model), vp, sz, vp]
        L.tle_prompt_scratch_bytes.argtypes = [P(Model), i, i]
        L.tle_prompt_scratch_bytes.restype = sz
        L.tle_prompt_forward.argtypes = [P(Model), vp, P(State), vp, i, i, vp, sz, vp]
        _lib = L
    return _lib


def _check(rc: int) -> None:
    if rc != TLE_OK:
        raise TleError(rc, lib().tle_last_error().decode())


def _ptr(t) -> int:
    return 0 if t is None else int(t.data_ptr())


def _stream(stream) -> int:
    import torch
    if stream is None:
        stream = torch.cuda.current_stream()
    return int(stream.cuda_stream)


def _want(t, numel: int, name: str):
    import torch
    if t.dtype != torch.float32 or not t.is_cuda or not t.is_contiguous():
        raise ValueError(f"{name}: need a contiguous float32 CUDA tensor")
    if t.numel() < numel:
        raise ValueError(f"{name}: need at least {numel} elements, got {t.numel()}")


def version() -> str:
    return lib().tle_version().decode()


# ---------------------------------------------------------------- ops.h:175
def rope(q, k, pos: int, head_dim: int = 64, n_head: int = 32, n_head_kv: int = 4,
         freq_base: float = 10000.0, stream=None) -> None:
    """In-place RoPE on device q [n_head*hd] and k [n_head_kv*hd] (ops.cpp:1223)."""
    _want(q, n_head * head_dim, "q")
    _want(k, n_head_kv * head_dim, "k")
    _check(lib().tle_rope(_ptr(q), _ptr(k), pos, head_dim, n_head, n_head_kv, freq_base,
                          _stream(stream)))


def attention_workspace(shape: Shape, n_ctx: int):
    import torch
    n = lib().tle_attention_workspace_bytes(ctypes.byref(shape), n_ctx)
    return torch.empty((n + 3) // 4, dtype=torch.float32, device="cuda")


def _single(fn, out, q, k, v, key_cache, value_cache, layer, pos, n_ctx, shape, workspace, stream):
    _want(out, 2048, "out"); _want(q, 2048, "q"); _want(k, 256, "k"); _want(v, 256, "v")
    _want(key_cache, (layer + 1) * n_ctx * 256, "key_cache")
    _want(value_cache, (layer + 1) * n_ctx * 256, "value_cache")
    if workspace is None:
        workspace = attention_workspace(shape, n_ctx)
    _check(fn(_ptr(out), _ptr(q), _ptr(k), _ptr(v), _ptr(key_cache), _ptr(value_cache), layer,
              pos, n_ctx, ctypes.byref(shape), _ptr(workspace), workspace.numel() * 4,
              _stream(stream)))


# ---------------------------------------------------------------- ops.h:204
def attention(out, q, k, v, key_cache, value_cache, layer: int, pos: int, n_ctx: int,
              shape: Optional[Shape] = None, workspace=None, stream=None) -> None:
    """attention() with device buffers; q, k already rotated (ops.cpp:1317)."""
    shape = shape or tinyllama_shape()
    _single(lib().tle_attention, out, q, k, v, key_cache, value_cache, layer, pos, n_ctx, shape,
            workspace, stream)


def rope_attention(out, q, k, v, key_cache, value_cache, layer: int, pos: int, n_ctx: int,
                   shape: Optional[Shape] = None, workspace=None, stream=None,
                   kv_ready: bool = False) -> None:
    """rope()+attention() (forward.cpp:192-208) in one launch; q, k unrotated.
    kv_ready: TLE_DECODE_KV_READY (the kernels still in flight on the stream
    write none of this layer's rows < pos), so the cached rows stream while
    the previous kernel finishes."""
    shape = shape or tinyllama_shape()
    if not kv_ready:
        _single(lib().tle_rope_attention, out, q, k, v, key_cache, value_cache, layer, pos, n_ctx,
                shape, workspace, stream)
        return
    flagged = lambda *a: lib().tle_rope_attention_flags(*a[:10], TLE_DECODE_KV_READY, *a[10:])  # noqa: E731
    _single(flagged, out, q, k, v, key_cache, value_cache, layer, pos, n_ctx, shape, workspace,
            stream)


def attention_lse(out, lse, q, k, v, key_cache, value_cache, layer: int, pos: int, n_ctx: int,
                  shape: Optional[Shape] = None, workspace=None, stream=None) -> None:
    """attention() plus each head's score log-sum-exp lse[32] (context split
    of one sequence over GPUs; see tle_attention_lse).  q, k already rotated."""
    shape = shape or tinyllama_shape()
    _want(lse, 32, "lse")
    _want(out, 2048, "out"); _want(q, 2048, "q"); _want(k, 256, "k"); _want(v, 256, "v")
    _want(key_cache, (layer + 1) * n_ctx * 256, "key_cache")
    _want(value_cache, (layer + 1) * n_ctx * 256, "value_cache")
    if workspace is None:
        workspace = attention_workspace(shape, n_ctx)
    _check(lib().tle_attention_lse(_ptr(out), _ptr(lse), _ptr(q), _ptr(k), _ptr(v), _ptr(key_cache),
                                   _ptr(value_cache), layer, pos, n_ctx, ctypes.byref(shape),
                                   _ptr(workspace), workspace.numel() * 4, _stream(stream)))


def merge_lse(out, parts, lses, stream=None) -> None:
    """out[2048] from parts[n][2048] and lses[n][32] (tle_merge_lse)."""
    n = int(parts.shape[0])
    _want(out, 2048, "out"); _want(parts, n * 2048, "parts"); _want(lses, n * 32, "lses")
    _check(lib().tle_merge_lse(_ptr(out), _ptr(parts), _ptr(lses), n, _stream(stream)))


# ----------------------------------------------------------- batched decode
class DecodeBatchBf16:
    """The decode step over bf16 caches (tle_decode_batch_bf16).

    ``caches`` is a list of (key_cache, value_cache, n_ctx) device tensors of
    dtype torch.bfloat16, each [n_layers][n_ctx][256].  The sequence records
    live in device memory; ``set_positions`` rewrites them (one H2D copy).
    """

    def __init__(self, caches: Sequence, positions: Sequence[int], shape: Optional[Shape] = None):
        import torch
        self.shape = shape or tinyllama_shape()
        self.caches = list(caches)
        self.n = len(self.caches)
        for kc, vc, _ in self.caches:
            if kc.dtype != torch.bfloat16 or vc.dtype != torch.bfloat16 or not kc.is_cuda:
                raise ValueError("bf16 CUDA caches expected")
        self._seqs_dev = torch.empty(self.n * ctypes.sizeof(SeqBf16), dtype=torch.uint8, device="cuda")
        self.workspace = None
        self.set_positions(positions)

    def set_positions(self, positions: Sequence[int]) -> None:
        import torch
        if len(positions) != self.n:
            raise ValueError("one position per sequence")
        self.positions = [int(p) for p in positions]
        self.max_rows = max(self.positions) + 1
        seqs = (SeqBf16 * self.n)()
        for i, (kc, vc, n_ctx) in enumerate(self.caches):
            seqs[i] = SeqBf16(_ptr(kc), _ptr(vc), int(n_ctx), self.positions[i])
        host = torch.frombuffer(bytearray(bytes(seqs)), dtype=torch.uint8)
        self._seqs_dev.copy_(host)
        nbytes = lib().tle_decode_bf16_workspace_bytes(self.n, self.max_rows)
        if self.workspace is None or self.workspace.numel() * 4 < nbytes:
            self.workspace = torch.empty((nbytes + 3) // 4, dtype=torch.float32, device="cuda")

    def run(self, q, k, v, out, layer: int, rotate: bool = True, stream=None) -> None:
        """q [n][2048], k/v [n][256], out [n][2048]: fp32 CUDA tensors."""
        for t, n, name in ((q, self.n * 2048, "q"), (k, self.n * 256, "k"), (v, self.n * 256, "v"),
                           (out, self.n * 2048, "out")):
            _want(t, n, name)
        _check(lib().tle_decode_batch_bf16(ctypes.byref(self.shape), self._seqs_dev.data_ptr(), self.n,
                                           self.max_rows, _ptr(q), _ptr(k), _ptr(v), _ptr(out), layer,
                                           1 if rotate else 0, _ptr(self.workspace),
                                           self.workspace.numel() * 4, _stream(stream)))


class PagedDecodeBatchBf16:
    """DecodeBatchBf16 over a bf16 PagedKVCache (tle_decode_batch_bf16_paged):
    one device page table per sequence; the sequence records (page table,
    entries, pos) live in device memory and ``set_positions`` rewrites them."""

    def __init__(self, cache: "PagedKVCache", tables: Sequence, positions: Sequence[int]):
        import torch
        if cache.dtype != torch.bfloat16:
            raise ValueError("a bfloat16 PagedKVCache expected")
        self.cache = cache
        self.tables = list(tables)
        self.n = len(self.tables)
        self.shape = cache.shape
        self._seqs_dev = torch.empty(self.n * ctypes.sizeof(PagedSeq), dtype=torch.uint8, device="cuda")
        self.workspace = None
        self.set_positions(positions)

    def set_positions(self, positions: Sequence[int]) -> None:
        import torch
        if len(positions) != self.n:
            raise ValueError("one position per sequence")
        self.positions = [int(p) for p in positions]
        self.max_rows = max(self.positions) + 1
        seqs = (PagedSeq * self.n)()
        for i, t in enumerate(self.tables):
            seqs[i] = PagedSeq(_ptr(t), int(t.numel()), self.positions[i])
        self._seqs_dev.copy_(torch.frombuffer(bytearray(bytes(seqs)), dtype=torch.uint8))
        nbytes = lib().tle_decode_bf16_workspace_bytes(self.n, self.max_rows)
        if self.workspace is None or self.workspace.numel() * 4 < nbytes:
            self.workspace = torch.empty((nbytes + 3) // 4, dtype=torch.float32, device="cuda")

    def run(self, q, k, v, out, layer: int, rotate: bool = True, stream=None) -> None:
        for t, n, name in ((q, self.n * 2048, "q"), (k, self.n * 256, "k"), (v, self.n * 256, "v"),
                           (out, self.n * 2048, "out")):
            _want(t, n, name)
        pool = self.cache.pool()
        _check(lib().tle_decode_batch_bf16_paged(ctypes.byref(self.shape), ctypes.byref(pool),
                                                 self._seqs_dev.data_ptr(), self.n, self.max_rows, _ptr(q),
                                                 _ptr(k), _ptr(v), _ptr(out), layer, 1 if rotate else 0,
                                                 _ptr(self.workspace), self.workspace.numel() * 4,
                                                 _stream(stream)))


class DecodeBatch:
    """attention() for many independent sequences in one launch per layer.

    ``caches`` is a list of (key_cache, value_cache, n_ctx) device tensors,
    each [n_layers][n_ctx][256] fp32.  ``set_positions`` re-plans the split
    of rows over CTAs (host) and uploads the descriptor (one H2D copy).
    """

    def __init__(self, caches: Sequence, positions: Sequence[int], shape: Optional[Shape] = None,
                 max_ctas: int = 0):
        import torch
        self.shape = shape or tinyllama_shape()
        self.caches = list(caches)
        self.n = len(self.caches)
        self.max_ctas = max_ctas
        L = lib()
        self.desc_bytes = L.tle_decode_desc_bytes(self.n, max_ctas)
        self._desc_host = torch.empty(self.desc_bytes, dtype=torch.uint8).pin_memory()
        self._desc_dev = torch.empty(self.desc_bytes, dtype=torch.uint8, device="cuda")
        self.workspace = None
        self.n_ctas = 0
        self.set_positions(positions)

    def build_host(self, positions: Sequence[int]) -> int:
        """Fills the pinned host descriptor; returns the CTA count."""
        if len(positions) != self.n:
            raise ValueError("one position per sequence")
        seqs = (Seq * self.n)()
        for i, (kc, vc, n_ctx) in enumerate(self.caches):
            seqs[i] = Seq(_ptr(kc), _ptr(vc), int(n_ctx), int(positions[i]))
        n_ctas = ctypes.c_int(0)
        _check(lib().tle_decode_desc(ctypes.byref(self.shape), seqs, self.n, self.max_ctas,
                                     self._desc_host.data_ptr(), self.desc_bytes,
                                     ctypes.byref(n_ctas)))
        return n_ctas.value

    def set_positions(self, positions: Sequence[int], stream=None) -> None:
        import torch
        self.positions = [int(p) for p in positions]
        self.n_ctas = self.build_host(self.positions)
        nbytes = lib().tle_decode_workspace_bytes(ctypes.byref(self.shape), self.n, self.n_ctas)
        if self.workspace is None or self.workspace.numel() * 4 < nbytes:
            self.workspace = torch.empty((nbytes + 3) // 4, dtype=torch.float32, device="cuda")
        self.upload(stream)

    def upload(self, stream=None) -> None:
        """H2D copy of the descriptor on `stream` (pinned -> device)."""
        import torch
        s = stream or torch.cuda.current_stream()
        with torch.cuda.stream(s):
            self._desc_dev.copy_(self._desc_host, non_blocking=True)

    def run(self, q, k, v, out, layer: int, rotate: bool = True, stream=None,
            kv_ready: bool = False, short: Optional[bool] = False) -> None:
        """kv_ready: TLE_DECODE_KV_READY (the previous kernel on the stream
        wrote none of the cached rows read here).  short: True runs the
        cluster decode (tle_decode_batch_short, every sequence <= 2048 rows),
        None picks it when it is the faster one (short_pays); the default
        keeps the split-K decode, which the paged call matches bit for bit."""
        n = self.n
        _want(q, n * 2048, "q"); _want(k, n * 256, "k"); _want(v, n * 256, "v")
        _want(out, n * 2048, "out")
        max_rows = max(self.positions) + 1
        if short is None:
            short = self.short_pays()
        if short:
            _check(lib().tle_decode_batch_short(ctypes.byref(self.shape), self._desc_dev.data_ptr(), n,
                                                max_rows, _ptr(q), _ptr(k), _ptr(v), _ptr(out), layer,
                                                _decode_flags(rotate, kv_ready), _stream(stream)))
            return
        _check(lib().tle_decode_batch(ctypes.byref(self.shape), self._desc_dev.data_ptr(), n,
                                      self.n_ctas, _ptr(q), _ptr(k), _ptr(v), _ptr(out), layer,
                                      _decode_flags(rotate, kv_ready), _ptr(self.workspace),
                                      self.workspace.numel() * 4, _stream(stream)))

    def short_pays(self) -> bool:
        """Whether the cluster decode applies (every sequence <= 2048 rows) and
        is the faster one (few rows per SM; measured crossover)."""
        rows = sum(p + 1 for p in self.positions)
        return max(self.positions) + 1 <= 2048 and rows <= SHORT_MAX_ROWS


# ------------------------------------------------------- paged KV cache
class PagedKVCache:
    """Key/value page pools shared by a batch of sequences.

    The pools are [n_layers][n_pages][page_rows][256] fp32; a sequence's row
    r lives in row r % page_rows of page ``table[r // page_rows]``.  Page ids
    are handed out from a free list (``alloc`` / ``free``); the page tables
    are int32 CUDA tensors the caller keeps per sequence.  The reference keeps
    one contiguous [n_layers][n_ctx][256] cache per sequence (run_state.h:20-25).
    """

    def __init__(self, n_pages: int, page_rows: int = 256, shape: Optional[Shape] = None,
                 device="cuda", dtype=None):
        import torch
        self.shape = shape or tinyllama_shape()
        self.n_pages = int(n_pages)
        self.page_rows = int(page_rows)
        self.dtype = dtype or torch.float32   # torch.bfloat16: pools for PagedDecodeBatchBf16
        dims = (self.shape.n_layers, self.n_pages, self.page_rows, 256)
        self.key_pool = torch.zeros(dims, dtype=self.dtype, device=device)
        self.value_pool = torch.zeros(dims, dtype=self.dtype, device=device)
        self._free = list(range(self.n_pages - 1, -1, -1))

    def pool(self):
        if self.dtype != __import__("torch").float32:
            return PagePoolBf16(_ptr(self.key_pool), _ptr(self.value_pool), self.n_pages, self.page_rows)
        return PagePool(_ptr(self.key_pool), _ptr(self.value_pool), self.n_pages, self.page_rows)

    def pages_for(self, n_rows: int) -> int:
        return -(-int(n_rows) // self.page_rows)

    def alloc(self, n: int) -> List[int]:
        if n > len(self._free):
            raise MemoryError(f"page pool exhausted: {n} pages wanted, {len(self._free)} free")
        return [self._free.pop() for _ in range(n)]

    def free(self, ids: Iterable[int]) -> None:
        self._free.extend(int(i) for i in ids)

    def table(self, ids: Sequence[int]):
        """The device page table for page ids ``ids``."""
        import torch
        return torch.tensor(list(ids), dtype=torch.int32, device=self.key_pool.device)


class PagedDecodeBatch:
    """DecodeBatch over a PagedKVCache: ``tables`` holds one int32 CUDA page
    table per sequence.  Same kernel, split and results as DecodeBatch on the
    same rows."""

    def __init__(self, cache: PagedKVCache, tables: Sequence, positions: Sequence[int],
                 max_ctas: int = 0):
        import torch
        self.cache = cache
        self.shape = cache.shape
        self.tables = list(tables)
        self.n = len(self.tables)
        self.max_ctas = max_ctas
        L = lib()
        self.desc_bytes = L.tle_decode_desc_bytes(self.n, max_ctas)
        self._desc_host = torch.empty(self.desc_bytes, dtype=torch.uint8).pin_memory()
        self._desc_dev = torch.empty(self.desc_bytes, dtype=torch.uint8, device="cuda")
        self.workspace = None
        self.n_ctas = 0
        self.set_positions(positions)

    def build_host(self, positions: Sequence[int]) -> int:
        import torch
        if len(positions) != self.n:
            raise ValueError("one position per sequence")
        seqs = (PagedSeq * self.n)()
        for i, t in enumerate(self.tables):
            if t.dtype != torch.int32 or not t.is_cuda or not t.is_contiguous():
                raise ValueError("page tables must be contiguous int32 CUDA tensors")
            seqs[i] = PagedSeq(_ptr(t), int(t.numel()), int(positions[i]))
        pool = self.cache.pool()
        n_ctas = ctypes.c_int(0)
        _check(lib().tle_decode_desc_paged(ctypes.byref(self.shape), ctypes.byref(pool), seqs,
                                           self.n, self.max_ctas, self._desc_host.data_ptr(),
                                           self.desc_bytes, ctypes.byref(n_ctas)))
        return n_ctas.value

    def set_positions(self, positions: Sequence[int], stream=None) -> None:
        import torch
        self.positions = [int(p) for p in positions]
        self.n_ctas = self.build_host(self.positions)
        nbytes = lib().tle_decode_workspace_bytes(ctypes.byref(self.shape), self.n, self.n_ctas)
        if self.workspace is None or self.workspace.numel() * 4 < nbytes:
            self.workspace = torch.empty((nbytes + 3) // 4, dtype=torch.float32, device="cuda")
        s = stream or torch.cuda.current_stream()
        with torch.cuda.stream(s):
            self._desc_dev.copy_(self._desc_host, non_blocking=True)

    def run(self, q, k, v, out, layer: int, rotate: bool = True, stream=None,
            kv_ready: bool = False) -> None:
        n = self.n
        _want(q, n * 2048, "q"); _want(k, n * 256, "k"); _want(v, n * 256, "v")
        _want(out, n * 2048, "out")
        pool = self.cache.pool()
        _check(lib().tle_decode_batch_paged(ctypes.byref(self.shape), ctypes.byref(pool),
                                            self._desc_dev.data_ptr(), n, self.n_ctas, _ptr(q),
                                            _ptr(k), _ptr(v), _ptr(out), layer,
                                            _decode_flags(rotate, kv_ready), _ptr(self.workspace),
                                            self.workspace.numel() * 4, _stream(stream)))


# ------------------------------------------------- decode without allocation
NOALLOC_MAX_SEQS = 256  # TLE_NOALLOC_MAX_SEQS


def decode_batch_noalloc(caches: Sequence, positions: Sequence[int], q, k, v, out, layer: int,
                         rotate: bool = True, shape: Optional[Shape] = None, stream=None) -> None:
    """tle_decode_batch_noalloc: the batched decode for callers that cannot
    allocate device memory (the library's fixed scratch array is used; see
    include/tle_attn.h).  ``caches`` as for DecodeBatch, records stay on the host."""
    shape = shape or tinyllama_shape()
    n = len(caches)
    _want(q, n * 2048, "q"); _want(k, n * 256, "k"); _want(v, n * 256, "v")
    _want(out, n * 2048, "out")
    seqs = (Seq * max(n, 1))()
    for i, (kc, vc, n_ctx) in enumerate(caches):
        seqs[i] = Seq(_ptr(kc), _ptr(vc), int(n_ctx), int(positions[i]))
    _check(lib().tle_decode_batch_noalloc(ctypes.byref(shape), seqs, n, _ptr(q), _ptr(k), _ptr(v),
                                          _ptr(out), layer, 1 if rotate else 0, _stream(stream)))


# ------------------------------------------------------------------ prefill
def prefill_workspace(n_tokens: int, pos0: int = 0, shape: Optional[Shape] = None):
    import torch
    shape = shape or tinyllama_shape()
    n = lib().tle_prefill_workspace_bytes(ctypes.byref(shape), n_tokens, pos0)
    # over-allocate by 1 KB so the buffer can start on a 1024-byte boundary
    raw = torch.empty(n + 1024, dtype=torch.uint8, device="cuda")
    off = (-raw.data_ptr()) % 1024
    return raw[off:off + n] if n > 0 else raw[off:off + 1024]


def prefill(out, q, k, v, key_cache, value_cache, layer: int, pos0: int, n_ctx: int,
            shape: Optional[Shape] = None, workspace=None, stream=None) -> None:
    """S successive rope+attention steps as one causal kernel (generate.cpp:56-59)."""
    shape = shape or tinyllama_shape()
    n_tokens = q.numel() // 2048
    _want(out, n_tokens * 2048, "out"); _want(k, n_tokens * 256, "k"); _want(v, n_tokens * 256, "v")
    if workspace is None:
        workspace = prefill_workspace(n_tokens, pos0, shape)
    _check(lib().tle_prefill(_ptr(out), _ptr(q), _ptr(k), _ptr(v), _ptr(key_cache),
                             _ptr(value_cache), layer, pos0, n_tokens, n_ctx, ctypes.byref(shape),
                             _ptr(workspace), workspace.numel() * workspace.element_size(),
                             _stream(stream)))


# ---------------------------------------------------------- multi-GPU plan
def partition_lpt(lengths: Iterable[int], n_ranks: int) -> List[int]:
    """Rank of each sequence under greedy longest-processing-time balancing."""
    lengths = [int(x) for x in lengths]
    n = len(lengths)
    arr = (ctypes.c_int32 * max(n, 1))(*lengths)
    out = (ctypes.c_int32 * max(n, 1))()
    _check(lib().tle_partition_lpt(arr, n, n_ranks, out))
    return [int(out[i]) for i in range(n)]


def device_error(clear: bool = True) -> int:
    code = ctypes.c_uint32(0)
    _check(lib().tle_device_error(1 if clear else 0, ctypes.byref(code)))
    return code.value


def selftest_wait_timeout(limit_us: int = 20000, stream=None) -> None:
    """Launches a block whose bounded wait is planted to expire after
    limit_us (tle_selftest_wait_timeout); read the result with device_error."""
    _check(lib().tle_selftest_wait_timeout(int(limit_us), _stream(stream)))


# ------------------------------------------------------------ forward pass
def _wptr(t) -> int:
    """Device pointer of a uint8 CUDA tensor holding GGUF-layout weights."""
    import torch
    if t.dtype != torch.uint8 or not t.is_cuda or not t.is_contiguous():
        raise ValueError("weights: need a contiguous uint8 CUDA tensor")
    return int(t.data_ptr())


def matmul(out, W, x, rows: int, cols: int, wtype: int, stream=None) -> None:
    """ops.h:64-66 matmul on the device; W: uint8 CUDA tensor, GGUF layout."""
    _want(out, rows, "out"); _want(x, cols, "x")
    _check(lib().tle_matmul(_ptr(out), _wptr(W), _ptr(x), rows, cols, wtype, _stream(stream)))


def rmsnorm(out, x, weight, eps: float = 1e-5, stream=None) -> None:
    n = x.numel()
    _want(out, n, "out"); _want(weight, n, "weight")
    _check(lib().tle_rmsnorm(_ptr(out), _ptr(x), _ptr(weight), n, eps, _stream(stream)))


def vec_add(out, x, stream=None) -> None:
    n = out.numel()
    _want(x, n, "x")
    _check(lib().tle_vec_add(_ptr(out), _ptr(x), n, _stream(stream)))


def ffn_swiglu(out, inp, hb, W_gate, W_up, W_down, n_ff: int, n_embd: int, wtype: int,
               stream=None) -> None:
    _want(out, n_embd, "out"); _want(inp, n_embd, "input"); _want(hb, n_ff, "hb")
    _check(lib().tle_ffn_swiglu(_ptr(out), _ptr(inp), _ptr(hb), None, _wptr(W_gate),
                                _wptr(W_up), _wptr(W_down), n_ff, n_embd, wtype, _stream(stream)))


def sample_argmax(logits, token_out, stream=None) -> None:
    """ops.h:249 on the device: writes the index into token_out (int32 CUDA)."""
    import torch
    _want(logits, 1, "logits")
    if token_out.dtype != torch.int32 or not token_out.is_cuda:
        raise ValueError("token_out: need an int32 CUDA tensor")
    _check(lib().tle_sample_argmax(_ptr(logits), logits.numel(), _ptr(token_out), _stream(stream)))


def sample_temperature(logits, token_out, temperature: float, r: float, stream=None) -> None:
    """ops.h:262 on the device with the uniform draw r; logits become probabilities."""
    _want(logits, 1, "logits")
    _check(lib().tle_sample_temperature(_ptr(logits), logits.numel(), temperature, r,
                                        _ptr(token_out), _stream(stream)))


def sample_top_p(logits, token_out, temperature: float, top_p: float, r: float, stream=None) -> None:
    """ops.h:278 on the device with the uniform draw r; logits become probabilities."""
    _want(logits, 1, "logits")
    _check(lib().tle_sample_top_p(_ptr(logits), logits.numel(), temperature, top_p, r,
                                  _ptr(token_out), _stream(stream)))


class DeviceModel:
    """A model (tinyllama-engine_b200/synth.py SynthModel, GGUF layouts)
    copied to device memory and described as a tle_model_t."""

    _LAYER = (("attn_q", "attn_q"), ("attn_k", "attn_k"), ("attn_v", "attn_v"),
              ("attn_output", "attn_output"), ("ffn_gate", "ffn_gate"), ("ffn_up", "ffn_up"),
              ("ffn_down", "ffn_down"))

    def __init__(self, model, device="cuda"):
        import torch
        self.src = model
        dev = torch.device(device)
        up = lambda a: torch.from_numpy(a).to(dev)  # noqa: E731
        self.keep = []

        def w(W):
            t = up(W.data)
            self.keep.append(t)
            return Weight(W.wtype, 0, t.data_ptr())

        def f32(a):
            t = up(a)
            self.keep.append(t)
            return t.data_ptr()

        self.layers = (Layer * model.n_layers)()
        for i, L in enumerate(model.layers):
            for f, n in self._LAYER:
                setattr(self.layers[i], f, w(L[n]))
            self.layers[i].attn_norm = f32(L["attn_norm"])
            self.layers[i].ffn_norm = f32(L["ffn_norm"])
        out = w(model.output) if model.output is not None else Weight(0, 0, None)
        self.desc = Model(model.n_layers, model.n_embd, model.n_head, model.n_head_kv, model.n_ff,
                          model.n_vocab, model.n_ctx, model.rope_freq_base, model.rms_norm_eps, 0,
                          w(model.token_embd), out, f32(model.output_norm), self.layers)


class DeviceState:
    """RunState (run_state.h) in device memory for a DeviceModel."""

    def __init__(self, dm: DeviceModel, device="cuda"):
        import torch
        m = dm.src
        z = lambda n: torch.zeros(n, dtype=torch.float32, device=device)  # noqa: E731
        kv = m.kv_dim
        self.t = {"x": z(m.n_embd), "xb": z(m.n_embd), "xb2": z(m.n_embd), "q": z(m.n_embd),
                  "k": z(kv), "v": z(kv), "hb": z(m.n_ff), "hb2": z(m.n_ff),
                  "logits": z(m.n_vocab), "key_cache": z(m.n_layers * m.n_ctx * kv),
                  "value_cache": z(m.n_layers * m.n_ctx * kv)}
        nbytes = lib().tle_forward_workspace_bytes(ctypes.byref(dm.desc))
        self.workspace = torch.zeros((nbytes + 3) // 4, dtype=torch.float32, device=device)
        self.desc = State(**{k: v.data_ptr() for k, v in self.t.items()},
                          workspace=self.workspace.data_ptr(), workspace_bytes=nbytes)

    @property
    def logits(self):
        return self.t["logits"]


class PromptWeights:
    """The fp16 copy of a DeviceModel's linear weights that the batched
    prompt reads (tle_prompt_pack_weights), made once on the device."""

    def __init__(self, dm: DeviceModel, stream=None):
        import torch
        nbytes = lib().tle_prompt_weights_bytes(ctypes.byref(dm.desc))
        if nbytes == 0:
            _check(TLE_ERR_UNSUPPORTED)
        self.buf = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        _check(lib().tle_prompt_pack_weights(ctypes.byref(dm.desc), _ptr(self.buf), nbytes,
                                             _stream(stream)))


def prompt_scratch(dm: DeviceModel, n_tokens: int, pos0: int = 0, device="cuda"):
    """A 1024-byte aligned uint8 CUDA tensor of tle_prompt_scratch_bytes (the
    caching allocator hands out 512-byte aligned blocks, so this
    over-allocates by 1 KB and offsets)."""
    import torch
    need = lib().tle_prompt_scratch_bytes(ctypes.byref(dm.desc), n_tokens, pos0)
    if need == 0:
        _check(TLE_ERR_INVALID)
    raw = torch.empty(need + 1024, dtype=torch.uint8, device=device)
    off = (-raw.data_ptr()) % 1024
    return raw[off:off + need]


def prompt_forward(dm: DeviceModel, ds: DeviceState, pw: PromptWeights, tokens, pos0: int = 0,
                   scratch=None, stream=None) -> None:
    """generate.cpp:52-59's prompt loop (forward() for tokens[i] at pos0 + i)
    as one batched pass: tokens is an int32 CUDA tensor; the caches get rows
    pos0.., ds.logits the last token's logits.  scratch: from prompt_scratch
    (allocated here when None)."""
    import torch
    if tokens.dtype != torch.int32 or not tokens.is_cuda or not tokens.is_contiguous():
        raise ValueError("tokens: need a contiguous int32 CUDA tensor")
    n = tokens.numel()
    if scratch is None:
        scratch = prompt_scratch(dm, n, pos0, tokens.device)
    _check(lib().tle_prompt_forward(ctypes.byref(dm.desc), _ptr(pw.buf), ctypes.byref(ds.desc),
                                    _ptr(tokens), n, pos0, _ptr(scratch),
                                    scratch.numel() * scratch.element_size(), _stream(stream)))


def forward_layers_one_launch(dm: DeviceModel, ds: DeviceState, pos: int) -> bool:
    """Whether forward() at this position runs every layer in one persistent
    launch (else one launch per product)."""
    return bool(lib().tle_forward_layers_one_launch(ctypes.byref(dm.desc), ctypes.byref(ds.desc), pos))


def forward(dm: DeviceModel, ds: DeviceState, token, pos: int, stream=None) -> None:
    """forward.h:16 on the device: token is an int32 CUDA tensor (its first
    element is read); logits land in ds.logits."""
    import torch
    if token.dtype != torch.int32 or not token.is_cuda:
        raise ValueError("token: need an int32 CUDA tensor")
    _check(lib().tle_forward(ctypes.byref(dm.desc), ctypes.byref(ds.desc), _ptr(token), pos,
                             _stream(stream)))
