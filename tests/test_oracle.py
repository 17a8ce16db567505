"""CPU tests: the C restatement (oracle/attn_oracle.c) is pinned to the reference.

* known-answer tests of the reference's own suite (src/test_ops.cpp:130-162
  softmax, 295-431 attention, 433-546 rope), run on the restatement and, when
  built, on the reference itself;
* bit-exact agreement with the golden fixtures made from the reference
  (tests/golden/make_golden.py);
* bit-exact agreement with the compiled reference on fresh seeded inputs.
"""
import math

import numpy as np
import pytest

import oracle
from conftest import load_golden

LIBS = ["port"] + (["ref"] if oracle.have_reference() else [])
NH, NKV, HD = 32, 4, 64
QD, KVD = NH * HD, NKV * HD


def get(which):
    return oracle.port() if which == "port" else oracle.reference()


def approx(a, b, tol=1e-4):  # test_ops.cpp:17-19
    return abs(a - b) < tol


# ------------------------------------------------ test_ops.cpp:130-162
@pytest.mark.parametrize("which", LIBS)
def test_softmax_known_answers(which):
    L = get(which)
    x1 = np.ones(4, np.float32); L.softmax(x1)
    assert approx(x1[0], 0.25)
    x2 = np.array([10, 0, 0], np.float32); L.softmax(x2)
    assert x2[0] > 0.99 and x2[1] < 0.01 and x2[2] < 0.01
    x3 = np.array([2, 1, 0.1, -1, 3], np.float32); L.softmax(x3)
    assert approx(float(x3.sum()), 1.0, 1e-5)
    x4 = np.array([1000, 1000, 999], np.float32); L.softmax(x4)
    assert np.all(np.isfinite(x4))


# ------------------------------------------------ test_ops.cpp:295-431
@pytest.mark.parametrize("which", LIBS)
def test_attention_known_answers(which):
    L = get(which)
    n_ctx, n_layers = 64, 2
    kc = np.zeros((n_layers, n_ctx, KVD), np.float32)
    vc = np.zeros_like(kc)
    out = np.zeros(QD, np.float32)
    # T1: single token -> output == v (test_ops.cpp:326-351)
    q = np.ones(QD, np.float32); k = np.ones(KVD, np.float32)
    v = (np.arange(KVD) % HD).astype(np.float32)
    L.attention(out, q, k, v, kc, vc, 0, 0, n_ctx)
    assert np.allclose(out[:HD], np.arange(HD), atol=1e-3)
    # T2: two equal keys, v=1 then v=3 -> 2.0 (test_ops.cpp:354-376)
    kc[:] = 0; vc[:] = 0
    L.attention(out, q, k, np.ones(KVD, np.float32), kc, vc, 0, 0, n_ctx)
    L.attention(out, q, k, np.full(KVD, 3.0, np.float32), kc, vc, 0, 1, n_ctx)
    assert approx(out[0], 2.0, 0.01)
    # T3: 10 tokens of modular patterns -> finite (test_ops.cpp:379-400)
    kc[:] = 0; vc[:] = 0
    for p in range(10):
        qq = ((np.arange(QD) + p) % 11 - 5).astype(np.float32)
        kk = ((np.arange(KVD) + 3 * p) % 7 - 3).astype(np.float32)
        vv = ((np.arange(KVD) + 5 * p) % 9 - 4).astype(np.float32)
        L.attention(out, qq, kk, vv, kc, vc, 0, p, n_ctx)
    assert np.all(np.isfinite(out))
    # T4: GQA mapping, q head 0 -> kv head 0, q head 8 -> kv head 1 (test_ops.cpp:405-430)
    kc[:] = 0; vc[:] = 0
    v = np.zeros(KVD, np.float32); v[:HD] = 10.0; v[HD:2 * HD] = 20.0
    L.attention(out, q, k, v, kc, vc, 0, 0, n_ctx)
    assert approx(out[0], 10.0, 0.01) and approx(out[8 * HD], 20.0, 0.01)


# ------------------------------------------------ test_ops.cpp:433-546
@pytest.mark.parametrize("which", LIBS)
def test_rope_known_answers(which):
    L = get(which)
    q = np.ones(QD, np.float32); k = np.ones(KVD, np.float32)
    L.rope(q, k, 0)
    assert np.all(np.abs(q - 1) < 1e-4) and np.all(np.abs(k - 1) < 1e-4)
    q = ((np.arange(QD) % 7) - 3).astype(np.float32)
    k = ((np.arange(KVD) % 5) - 2).astype(np.float32)
    n0 = math.sqrt(float(np.sum(q[:HD].astype(np.float64) ** 2)))
    L.rope(q, k, 42)
    n1 = math.sqrt(float(np.sum(q[:HD].astype(np.float64) ** 2)))
    assert approx(n0, n1, 1e-3)
    q1 = np.ones(QD, np.float32); k1 = np.ones(KVD, np.float32)
    q2 = np.ones(QD, np.float32); k2 = np.ones(KVD, np.float32)
    L.rope(q1, k1, 5); L.rope(q2, k2, 100)
    assert np.any(np.abs(q1[:HD] - q2[:HD]) >= 1e-4)
    q1 = np.full(QD, 2.5, np.float32); k1 = np.full(KVD, 2.5, np.float32)
    q2 = q1.copy(); k2 = k1.copy()
    L.rope(q1, k1, 17); L.rope(q2, k2, 17)
    assert np.array_equal(q1, q2)
    q = np.zeros(QD, np.float32); k = np.zeros(KVD, np.float32)
    q[0], q[1] = 3.0, 4.0
    L.rope(q, k, 1)
    c, s = np.cos(np.float32(1.0)), np.sin(np.float32(1.0))
    assert approx(q[0], 3 * c - 4 * s) and approx(q[1], 3 * s + 4 * c)


# ------------------------------------------------ golden fixtures (bit-exact)
def test_golden_decode_bitexact():
    P = oracle.port()
    for name in ("decode_mid", "decode_pos0", "decode_full"):
        g = load_golden(name)
        kc = g["key_cache"].astype(np.float32); vc = g["value_cache"].astype(np.float32)
        q = g["q"].astype(np.float32); k = g["k"].astype(np.float32)
        v = g["v"].astype(np.float32)
        P.rope(q, k, int(g["pos"]))
        assert np.array_equal(q, g["q_rot"]) and np.array_equal(k, g["k_rot"]), name
        out = np.zeros(QD, np.float32)
        P.attention(out, q, k, v, kc, vc, int(g["layer"]), int(g["pos"]), int(g["n_ctx"]))
        assert np.array_equal(out, g["out"]), name
        assert np.array_equal(kc[int(g["layer"]), int(g["pos"])], g["k_rot"]), name


def test_golden_prefill_bitexact():
    P = oracle.port()
    for name in ("prefill_fresh", "prefill_chunk"):
        g = load_golden(name)
        kc = g["key_cache"].astype(np.float32); vc = g["value_cache"].astype(np.float32)
        out = np.zeros_like(g["out"])
        P.prefill(out, g["q"].astype(np.float32), g["k"].astype(np.float32),
                  g["v"].astype(np.float32), kc, vc, 0, int(g["pos0"]), int(g["n_ctx"]))
        assert np.array_equal(out, g["out"]), name
        n = g["key_cache_after"].shape[0]
        assert np.array_equal(kc[0, :n], g["key_cache_after"]), name
        assert np.array_equal(vc[0, :n], g["value_cache_after"]), name


def test_golden_batch_bitexact():
    g = load_golden("batch_ragged")
    n = len(g["pos"])
    kcs = [g[f"key_cache_{i}"].astype(np.float32) for i in range(n)]
    vcs = [g[f"value_cache_{i}"].astype(np.float32) for i in range(n)]
    out = np.zeros_like(g["out"])
    oracle.port().decode_batch(kcs, vcs, g["n_ctx"], g["pos"], g["q"].astype(np.float32),
                               g["k"].astype(np.float32), g["v"].astype(np.float32), out,
                               int(g["layer"]), n_threads=2)
    assert np.array_equal(out, g["out"])


def test_golden_rope_and_softmax_bitexact():
    P = oracle.port()
    g = load_golden("rope_positions")
    for i, p in enumerate(g["pos"]):
        q = g["q"][i].astype(np.float32); k = g["k"][i].astype(np.float32)
        P.rope(q, k, int(p))
        assert np.array_equal(q, g["q_out"][i]) and np.array_equal(k, g["k_out"][i]), int(p)
    s = load_golden("softmax_cases")
    for i in range(5):
        x = s[f"in_{i}"].copy()
        P.softmax(x)
        assert np.array_equal(x, s[f"out_{i}"])


@pytest.mark.skipif(not oracle.have_reference(), reason="reference not compiled here")
def test_port_matches_reference_random():
    P, R = oracle.port(), oracle.reference()
    rng = np.random.default_rng(7)
    for n_ctx, pos, layer in ((128, 127, 0), (300, 211, 2), (1, 0, 0)):
        kc = rng.standard_normal((3, n_ctx, KVD), dtype=np.float32)
        vc = rng.standard_normal((3, n_ctx, KVD), dtype=np.float32)
        q = rng.standard_normal(QD, dtype=np.float32); k = rng.standard_normal(KVD, dtype=np.float32)
        v = rng.standard_normal(KVD, dtype=np.float32)
        res = []
        for L in (P, R):
            kc2, vc2, q2, k2 = kc.copy(), vc.copy(), q.copy(), k.copy()
            L.rope(q2, k2, pos)
            o = np.zeros(QD, np.float32)
            L.attention(o, q2, k2, v, kc2, vc2, layer, pos, n_ctx)
            res.append((o, kc2, vc2))
        assert np.array_equal(res[0][0], res[1][0])
        assert np.array_equal(res[0][1], res[1][1]) and np.array_equal(res[0][2], res[1][2])
