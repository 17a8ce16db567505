"""Synthetic TinyLlama models in the reference's GGUF tensor layouts.

There is no checkpoint in this environment (and no network): the end-to-end
workload is defined on random-init weights.  This module
writes them in the byte layouts the reference reads (src/gguf.h:54-135):

* Q4_0: blocks of 32 weights, fp16 scale d ~ |N(0, 0.02)| then 16 bytes of
  nibbles, uniform 0..15 (element j in the low nibble of byte j, j + 16 in
  the high nibble; weight = (nibble - 8) * d).
* Q8_0: fp16 d ~ |N(0, 0.02)| then 32 int8 uniform in [-128, 127].
* Q6_K: super-blocks of 256 (ql[128], qh[64], int8 scales[16], fp16 d),
  random bytes, scales uniform in [-32, 31], d ~ |N(0, 0.002)|.
* F16 / F32: N(0, sigma) values.

Norm weights are 1.0 (config 2).  The model is a plain description: numpy
byte arrays plus their ggml type; ``tle.DeviceModel`` uploads it and the
oracle reads it on the host.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List

import numpy as np

F32, F16, Q4_0, Q8_0, Q6_K = 0, 1, 2, 8, 14
# (weights per block, bytes per block) of each format (reference gguf.h)
BLOCK = {F32: (1, 4), F16: (1, 2), Q4_0: (32, 18), Q8_0: (32, 34), Q6_K: (256, 210)}
LAYER_WEIGHTS = ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down")


def row_bytes(wtype: int, cols: int) -> int:
    n, b = BLOCK[wtype]
    if cols % n:
        raise ValueError(f"cols {cols} is not a multiple of the block size {n}")
    return cols // n * b


def _fp16(values: np.ndarray) -> np.ndarray:
    return values.astype(np.float16).view(np.uint16)


def random_weight(rng: np.random.Generator, wtype: int, rows: int, cols: int,
                  sigma: float = 0.02) -> np.ndarray:
    """rows x cols weights of format wtype as a flat uint8 array (row-major,
    row i at i * row_bytes)."""
    if wtype == F32:
        return (rng.standard_normal((rows, cols), dtype=np.float32) * sigma).view(np.uint8).ravel()
    if wtype == F16:
        w = rng.standard_normal((rows, cols), dtype=np.float32) * sigma
        return _fp16(w).view(np.uint8).ravel()
    nb = cols // BLOCK[wtype][0]
    if wtype == Q4_0:
        blk = np.empty((rows, nb, 18), np.uint8)
        d = np.abs(rng.standard_normal((rows, nb), dtype=np.float32) * sigma)
        blk[:, :, 0:2] = _fp16(d).view(np.uint8).reshape(rows, nb, 2)
        blk[:, :, 2:] = rng.integers(0, 256, (rows, nb, 16), dtype=np.uint8)
        return blk.ravel()
    if wtype == Q8_0:
        blk = np.empty((rows, nb, 34), np.uint8)
        d = np.abs(rng.standard_normal((rows, nb), dtype=np.float32) * sigma)
        blk[:, :, 0:2] = _fp16(d).view(np.uint8).reshape(rows, nb, 2)
        blk[:, :, 2:] = rng.integers(0, 256, (rows, nb, 32), dtype=np.uint8)
        return blk.ravel()
    if wtype == Q6_K:
        blk = np.empty((rows, nb, 210), np.uint8)
        blk[:, :, 0:192] = rng.integers(0, 256, (rows, nb, 192), dtype=np.uint8)
        blk[:, :, 192:208] = rng.integers(-32, 32, (rows, nb, 16)).astype(np.int8).view(np.uint8)
        d = np.abs(rng.standard_normal((rows, nb), dtype=np.float32) * sigma * 0.1)
        blk[:, :, 208:210] = _fp16(d).view(np.uint8).reshape(rows, nb, 2)
        return blk.ravel()
    raise ValueError(f"unsupported weight type {wtype}")


@dataclass
class Weight:
    wtype: int
    rows: int
    cols: int
    data: np.ndarray          # flat uint8, GGUF layout


@dataclass
class SynthModel:
    n_layers: int = 22
    n_embd: int = 2048
    n_head: int = 32
    n_head_kv: int = 4
    n_ff: int = 5632
    n_vocab: int = 32000
    n_ctx: int = 2048
    rope_freq_base: float = 10000.0
    rms_norm_eps: float = 1e-5
    token_embd: Weight = None
    output: Weight = None          # None: the LM head is token_embd (forward.cpp:253-260)
    output_norm: np.ndarray = None
    layers: List[Dict[str, object]] = field(default_factory=list)

    @property
    def head_dim(self) -> int:
        return self.n_embd // self.n_head

    @property
    def kv_dim(self) -> int:
        return self.n_head_kv * self.head_dim

    def weight_bytes_per_token(self) -> int:
        """Bytes of weights one forward() reads (all layers + LM head)."""
        total = sum(L[n].data.nbytes for L in self.layers for n in LAYER_WEIGHTS)
        head = self.output if self.output is not None else self.token_embd
        return total + head.data.nbytes


def make_model(seed: int = 0, n_layers: int = 22, wtype: int = Q4_0, output_type: int = Q4_0,
               embd_type: int = F16, n_vocab: int = 32000, n_ctx: int = 2048, n_embd: int = 2048,
               n_head: int = 32, n_head_kv: int = 4, n_ff: int = 5632) -> SynthModel:
    """TinyLlama-1.1B shapes with random weights (config 2: Q4_0 linear
    weights, fp16 embedding table, RMSNorm weights 1.0).  output_type None
    ties the LM head to the embedding table."""
    rng = np.random.default_rng(seed)
    m = SynthModel(n_layers=n_layers, n_embd=n_embd, n_head=n_head, n_head_kv=n_head_kv,
                   n_ff=n_ff, n_vocab=n_vocab, n_ctx=n_ctx)
    m.token_embd = Weight(embd_type, n_vocab, n_embd,
                          random_weight(rng, embd_type, n_vocab, n_embd, sigma=1.0))
    if output_type is not None:
        m.output = Weight(output_type, n_vocab, n_embd,
                          random_weight(rng, output_type, n_vocab, n_embd))
    m.output_norm = np.ones(n_embd, np.float32)
    kv = m.kv_dim
    shapes = {"attn_q": (n_embd, n_embd), "attn_k": (kv, n_embd), "attn_v": (kv, n_embd),
              "attn_output": (n_embd, n_embd), "ffn_gate": (n_ff, n_embd),
              "ffn_up": (n_ff, n_embd), "ffn_down": (n_embd, n_ff)}
    for _ in range(n_layers):
        L: Dict[str, object] = {}
        for name in LAYER_WEIGHTS:
            r, c = shapes[name]
            L[name] = Weight(wtype, r, c, random_weight(rng, wtype, r, c))
        L["attn_norm"] = np.ones(n_embd, np.float32)
        L["ffn_norm"] = np.ones(n_embd, np.float32)
        m.layers.append(L)
    return m
