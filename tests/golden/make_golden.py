"""Generates the golden fixtures in tests/golden/ from the reference itself.

Runs the reference's own rope()/attention() (src/ops.cpp compiled unmodified
into oracle/_ref/libref_attn.so by oracle/Makefile) on seeded inputs with
TinyLlama shapes and stores inputs and outputs.  The fixtures pin both the C
restatement (oracle/attn_oracle.c) and the CUDA kernels.

Inputs are N(0,1) values rounded to float16 precision and stored as float16
(exactly representable in float32) to keep the files small; outputs are
stored as float32 bit patterns.

    python tests/golden/make_golden.py        # needs oracle/_ref built
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle  # noqa: E402

NH, NKV, HD = 32, 4, 64
QD, KVD = NH * HD, NKV * HD


def normal16(rng, shape):
    return rng.standard_normal(shape, dtype=np.float32).astype(np.float16)


def decode_case(ref, name, seed, n_layers, n_ctx, layer, pos):
    rng = np.random.default_rng(seed)
    kc = normal16(rng, (n_layers, n_ctx, KVD))
    vc = normal16(rng, (n_layers, n_ctx, KVD))
    q = normal16(rng, QD)
    k = normal16(rng, KVD)
    v = normal16(rng, KVD)
    kc32, vc32 = kc.astype(np.float32), vc.astype(np.float32)
    q32, k32 = q.astype(np.float32), k.astype(np.float32)
    ref.rope(q32, k32, pos)
    out = np.zeros(QD, np.float32)
    ref.attention(out, q32, k32, v.astype(np.float32), kc32, vc32, layer, pos, n_ctx)
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), kind="decode", n_layers=n_layers,
                        n_ctx=n_ctx, layer=layer, pos=pos, key_cache=kc, value_cache=vc, q=q, k=k,
                        v=v, q_rot=q32, k_rot=k32, out=out)


def prefill_case(ref, name, seed, n_ctx, pos0, n_tokens):
    rng = np.random.default_rng(seed)
    kc = np.zeros((1, n_ctx, KVD), np.float16)
    vc = np.zeros((1, n_ctx, KVD), np.float16)
    kc[0, :pos0] = normal16(rng, (pos0, KVD))
    vc[0, :pos0] = normal16(rng, (pos0, KVD))
    q = normal16(rng, (n_tokens, QD))
    k = normal16(rng, (n_tokens, KVD))
    v = normal16(rng, (n_tokens, KVD))
    kc32, vc32 = kc.astype(np.float32), vc.astype(np.float32)
    out = np.zeros((n_tokens, QD), np.float32)
    ref.prefill(out, q.astype(np.float32), k.astype(np.float32), v.astype(np.float32), kc32, vc32,
                0, pos0, n_ctx)
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), kind="prefill", n_ctx=n_ctx, pos0=pos0,
                        key_cache=kc, value_cache=vc, q=q, k=k, v=v, out=out,
                        key_cache_after=kc32[0, : pos0 + n_tokens],
                        value_cache_after=vc32[0, : pos0 + n_tokens])


def batch_case(ref, name, seed, n_ctx_list, pos_list, layer, n_layers):
    rng = np.random.default_rng(seed)
    n = len(pos_list)
    kcs = [normal16(rng, (n_layers, c, KVD)) for c in n_ctx_list]
    vcs = [normal16(rng, (n_layers, c, KVD)) for c in n_ctx_list]
    q = normal16(rng, (n, QD))
    k = normal16(rng, (n, KVD))
    v = normal16(rng, (n, KVD))
    out = np.zeros((n, QD), np.float32)
    ref.decode_batch([c.astype(np.float32) for c in kcs], [c.astype(np.float32) for c in vcs],
                     n_ctx_list, pos_list, q.astype(np.float32), k.astype(np.float32),
                     v.astype(np.float32), out, layer, n_layers=n_layers)
    arrays = {f"key_cache_{i}": kcs[i] for i in range(n)}
    arrays.update({f"value_cache_{i}": vcs[i] for i in range(n)})
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), kind="batch", n_layers=n_layers,
                        layer=layer, n_ctx=np.array(n_ctx_list, np.int32),
                        pos=np.array(pos_list, np.int32), q=q, k=k, v=v, out=out, **arrays)


def rope_cases(ref, name, seed, positions):
    rng = np.random.default_rng(seed)
    q = normal16(rng, (len(positions), QD))
    k = normal16(rng, (len(positions), KVD))
    q_out = q.astype(np.float32)
    k_out = k.astype(np.float32)
    for i, p in enumerate(positions):
        qi, ki = q_out[i].copy(), k_out[i].copy()
        ref.rope(qi, ki, int(p))
        q_out[i], k_out[i] = qi, ki
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), kind="rope",
                        pos=np.array(positions, np.int32), q=q, k=k, q_out=q_out, k_out=k_out)


def softmax_case(ref, name):
    rows = [np.array(r, np.float32) for r in (
        [1, 1, 1, 1], [10, 0, 0], [2, 1, 0.1, -1, 3], [1000, 1000, 999], [-50.5, 3.25, 88.0, -1e3])]
    outs = []
    for r in rows:
        x = r.copy()
        ref.softmax(x)
        outs.append(x)
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), kind="softmax",
                        **{f"in_{i}": r for i, r in enumerate(rows)},
                        **{f"out_{i}": o for i, o in enumerate(outs)})


def main():
    if not oracle.have_reference():
        sys.exit("oracle/_ref/libref_attn.so missing: run `make -C oracle` with the reference tree")
    ref = oracle.reference()
    decode_case(ref, "decode_mid", 101, n_layers=2, n_ctx=40, layer=1, pos=29)
    decode_case(ref, "decode_pos0", 102, n_layers=2, n_ctx=16, layer=0, pos=0)
    decode_case(ref, "decode_full", 103, n_layers=1, n_ctx=70, layer=0, pos=69)
    prefill_case(ref, "prefill_fresh", 201, n_ctx=48, pos0=0, n_tokens=40)
    prefill_case(ref, "prefill_chunk", 202, n_ctx=64, pos0=21, n_tokens=19)
    batch_case(ref, "batch_ragged", 301, n_ctx_list=[9, 33, 64, 5, 40],
               pos_list=[8, 0, 63, 2, 37], layer=1, n_layers=2)
    rope_cases(ref, "rope_positions", 401, [0, 1, 5, 42, 100, 511, 2047, 32767])
    softmax_case(ref, "softmax_cases")
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
