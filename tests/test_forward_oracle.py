"""CPU pins of the forward-pass oracle (oracle/forward_oracle.c): the
reference suite's known-answer tests (src/test_ops.cpp) on both the
restatement and the reference's own ops.cpp compiled unmodified
(oracle/_ref), and bit-for-bit agreement of the two on seeded inputs for
every weight format, RMSNorm, SiLU, SwiGLU, argmax and whole forward()
steps (src/forward.cpp:178-265)."""
import sys
import os

import numpy as np
import pytest

import oracle
from forward_cases import F16, F32, Q4_0, Q6_K, Q8_0, matmul_kats

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                "tinyllama-engine_b200"))
import synth  # noqa: E402

BACKENDS = ["port"] + (["reference"] if oracle.have_reference() else [])


def backend(name):
    return oracle.port() if name == "port" else oracle.reference()


@pytest.mark.parametrize("name", BACKENDS)
def test_matmul_known_answers(name):
    B = backend(name)
    for label, W, x, rows, cols, t, want, tol in matmul_kats():
        out = np.zeros(rows, np.float32)
        B.matmul(out, np.ascontiguousarray(W), np.ascontiguousarray(x, np.float32), rows, cols, t)
        assert np.all(np.abs(out - np.asarray(want, np.float32)) < tol), (label, out)


@pytest.mark.parametrize("name", BACKENDS)
def test_elementwise_known_answers(name):
    """rmsnorm test_ops.cpp:92-127, silu 164-186, elementwise_mul 189-200,
    vec_add 202-213, ffn_swiglu 215-268, argmax 583-596."""
    B = backend(name)
    o = np.zeros(4, np.float32)
    B.rmsnorm(o, np.ones(4, np.float32), np.ones(4, np.float32), 1e-5)
    assert abs(o[0] - 1.0) < 1e-3
    r = 1.0 / np.sqrt(12.5)
    o2 = np.zeros(2, np.float32)
    B.rmsnorm(o2, np.array([3, 4], np.float32), np.ones(2, np.float32), 0.0)
    assert np.allclose(o2, [3 * r, 4 * r], atol=1e-4)
    B.rmsnorm(o2, np.array([3, 4], np.float32), np.array([2, 0.5], np.float32), 0.0)
    assert np.allclose(o2, [3 * r * 2, 4 * r * 0.5], atol=1e-4)
    for v, want, tol in ((0.0, 0.0, 1e-4), (10.0, 10.0, 0.01), (-10.0, 0.0, 0.01),
                         (1.0, 1.0 / (1.0 + np.exp(-1.0)), 1e-4)):
        a = np.array([v], np.float32)
        B.silu(a)
        assert abs(a[0] - want) < tol
    a = np.array([2, 3, 4], np.float32)
    B.elementwise_mul(a, np.array([5, 0.5, -1], np.float32))
    assert np.allclose(a, [10, 1.5, -4], atol=1e-4)
    a = np.array([1, 2, 3], np.float32)
    B.vec_add(a, np.array([10, 20, 30], np.float32))
    assert np.allclose(a, [11, 22, 33], atol=1e-4)
    gate = np.array([1, 0, 0, 1, 1, 1], np.float32).view(np.uint8)
    up = np.array([1, 1, 0, 1, 1, 0], np.float32).view(np.uint8)
    down = np.array([1, 0, 1, 0, 1, 0], np.float32).view(np.uint8)
    out = np.zeros(2, np.float32)
    B.ffn_swiglu(out, np.array([1, 2], np.float32), gate, up, down, 3, 2, F32)
    s = lambda v: v / (1 + np.exp(-v))  # noqa: E731
    assert np.allclose(out, [s(1.0) * 3 + s(3.0), s(2.0) * 2], atol=1e-3)
    B.ffn_swiglu(out, np.zeros(2, np.float32), gate, up, down, 3, 2, F32)
    assert np.allclose(out, 0, atol=1e-4)
    assert B.sample_argmax(np.array([1, 5, 3, 2], np.float32)) == 1
    assert B.sample_argmax(np.array([-1, -5, -0.5, -2], np.float32)) == 2


@pytest.mark.skipif(not oracle.have_reference(), reason="reference not built")
@pytest.mark.parametrize("wtype,rows,cols", [(F32, 33, 256), (F16, 40, 512), (Q8_0, 70, 2048),
                                             (Q4_0, 64, 2048), (Q4_0, 16, 5632),
                                             (Q6_K, 24, 2048)])
def test_matmul_bit_exact_vs_reference(wtype, rows, cols):
    rng = np.random.default_rng(wtype * 1000 + cols)
    W = synth.random_weight(rng, wtype, rows, cols)
    x = rng.standard_normal(cols, dtype=np.float32)
    a, b = np.zeros(rows, np.float32), np.zeros(rows, np.float32)
    oracle.port().matmul(a, W, x, rows, cols, wtype)
    oracle.reference().matmul(b, W, x, rows, cols, wtype)
    assert np.array_equal(a, b)


@pytest.mark.skipif(not oracle.have_reference(), reason="reference not built")
def test_fp16_conversion_and_elementwise_bit_exact_vs_reference():
    P, R = oracle.port(), oracle.reference()
    h = np.arange(0, 65536, 257, dtype=np.uint16)   # every exponent, subnormals, inf/NaN
    h = np.concatenate([h, np.array([0x0001, 0x03FF, 0x7C00, 0xFC00, 0x7E00, 0x8001], np.uint16)])
    assert np.array_equal(P.fp16_to_f32(h).view(np.uint32), R.fp16_to_f32(h).view(np.uint32))
    rng = np.random.default_rng(3)
    x = rng.standard_normal(2048, dtype=np.float32) * 3
    w = rng.standard_normal(2048, dtype=np.float32)
    a, b = np.zeros_like(x), np.zeros_like(x)
    P.rmsnorm(a, x, w, 1e-5)
    R.rmsnorm(b, x, w, 1e-5)
    assert np.array_equal(a, b)
    a, b = x.copy(), x.copy()
    P.silu(a)
    R.silu(b)
    assert np.array_equal(a, b)
    for logits in (rng.standard_normal(32000, dtype=np.float32),
                   np.array([1, 7, 7, 3], np.float32),                 # tie: first index
                   np.array([np.nan, 1, 2], np.float32),               # NaN first: index 0
                   np.array([1, np.nan, 2, np.nan], np.float32),
                   np.full(5, -np.inf, np.float32)):
        assert P.sample_argmax(logits) == R.sample_argmax(logits)


@pytest.mark.skipif(not oracle.have_reference(), reason="reference not built")
@pytest.mark.parametrize("wtype,out_type", [(Q4_0, Q4_0), (Q8_0, None), (Q6_K, Q6_K)])
def test_forward_bit_exact_vs_reference(wtype, out_type):
    """Two layers of TinyLlama width (q/k/v/o, SwiGLU 5632) with a small
    vocabulary, four tokens: the restated forward() equals the reference's
    ops composed in forward.cpp's order, logits bit for bit."""
    m = synth.make_model(seed=wtype, n_layers=2, wtype=wtype, output_type=out_type, n_vocab=512,
                         n_ctx=16)
    hp, hr = oracle.HostForward(m), oracle.HostForward(m)
    P, R = oracle.port(), oracle.reference()
    for pos, tok in enumerate([1, 511, 77, 1]):
        P.forward(hp, tok, pos)
        R.forward(hr, tok, pos)
        assert np.all(np.isfinite(hp.logits))
        assert np.array_equal(hp.logits, hr.logits), pos
    assert np.array_equal(hp.bufs["key_cache"], hr.bufs["key_cache"])


def _probs(logits, temperature):
    x = logits.astype(np.float32).copy()
    if temperature != 1.0 and temperature > 0:
        x *= np.float32(1.0) / np.float32(temperature)
    e = np.exp(x - x.max(), dtype=np.float32)
    return e / e.sum(dtype=np.float32)


def test_sampling_known_answers_and_reference_draws():
    """test_ops.cpp:598-633: temperature and top-p give valid ids, and top-p
    with a dominant logit keeps picking it; the oracle (uniform draw passed
    in) agrees with the reference's own draws: every reference top-p token
    lies in the oracle's nucleus (nuclei of at most 100 tokens, which the
    reference sorts fully)."""
    P = oracle.port()
    rng = np.random.default_rng(9)
    for r in rng.random(10):
        tok = P.sample_temperature(np.array([1.0, 10.0, 2.0, 0.5, 0.1], np.float32), 1.0, float(r))
        assert 0 <= tok < 5                                        # test_ops.cpp:601-610
        tok = P.sample_top_p(np.array([1.0, 10.0, 2.0, 0.5, 0.1], np.float32), 0.8, 0.9, float(r))
        assert 0 <= tok < 5                                        # test_ops.cpp:613-621
        dom = np.array([0.0, 100.0, 0.0, 0.0, 0.0], np.float32)
        assert P.sample_top_p(dom, 0.5, 0.1, float(r)) == 1       # test_ops.cpp:624-633
    lg = np.array([1.0, 2.0, 3.0], np.float32)
    p = _probs(lg, 1.0)
    assert P.sample_temperature(lg.copy(), 1.0, float(p[0] / 2)) == 0
    assert P.sample_temperature(lg.copy(), 1.0, float(p[0] + p[1] / 2)) == 1
    assert P.sample_temperature(lg.copy(), 1.0, 0.99999) == 2
    if not oracle.have_reference():
        return
    R = oracle.reference()
    for scale in (4.5, 6.0):
        lg = rng.standard_normal(32000).astype(np.float32) * scale
        p = _probs(lg, 0.8)
        order = np.argsort(-p, kind="stable")
        m = int(np.searchsorted(np.cumsum(p[order]), 0.9) + 1)
        assert m <= 100
        nucleus = set(order[:m].tolist())
        for _ in range(100):
            assert R.sample_top_p_reference(lg.copy(), 0.8, 0.9) in nucleus
