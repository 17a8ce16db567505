"""GPU parity of the device forward pass around attention
(include/tle_forward.h): the reference suite's known-answer tests
(src/test_ops.cpp) through the CUDA path, every weight format against the
oracle on seeded inputs, greedy sampling (exact), and whole forward()
steps against the oracle's forward() (src/forward.cpp:178-265).

Tolerances (written here): a matrix-vector product differs from the
oracle's only in fp32 summation order, so each output row is checked
against a float64 evaluation of the same dequantised weights with a bound
of 3e-5 x sum_j |w_j x_j| (the row's error scale), which the oracle itself
also meets; silu/RMSNorm use expf/sqrtf and differ by a few ulps.  Argmax
is exact.  Forward logits after L layers are compared with max-abs
<= 2e-3 x max|logit| and the greedy token must agree whenever the top two
logits are further apart than that.
"""
import os
import sys

import numpy as np
import pytest

import oracle
from forward_cases import F16, F32, Q4_0, Q6_K, Q8_0, matmul_kats, matmul_truth

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                "tinyllama-engine_b200"))
import synth  # noqa: E402

pytestmark = pytest.mark.gpu
ROW_TOL = 3e-5


def host(t):
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


def dev(a, dtype=None):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(a))
    return t.cuda() if dtype is None else t.to(dtype).cuda()


class Gpu:
    """The oracle's method names over the CUDA path (inputs/outputs numpy)."""

    def matmul(self, out, W, x, rows, cols, wtype):
        import tle
        o = dev(np.zeros(rows, np.float32))
        tle.matmul(o, dev(W), dev(x), rows, cols, wtype)
        out[:] = host(o)

    def rmsnorm(self, out, x, w, eps=1e-5):
        import tle
        o = dev(np.zeros_like(out))
        tle.rmsnorm(o, dev(x), dev(w), eps)
        out[:] = host(o)

    def vec_add(self, out, x):
        import tle
        o = dev(out)
        tle.vec_add(o, dev(x))
        out[:] = host(o)

    def ffn_swiglu(self, out, inp, W_gate, W_up, W_down, n_ff, n_embd, wtype):
        import tle
        o = dev(np.zeros(n_embd, np.float32))
        hb = dev(np.zeros(n_ff, np.float32))
        tle.ffn_swiglu(o, dev(inp), hb, dev(W_gate), dev(W_up), dev(W_down), n_ff, n_embd, wtype)
        out[:] = host(o)

    def sample_argmax(self, logits):
        import torch
        import tle
        t = torch.zeros(1, dtype=torch.int32, device="cuda")
        tle.sample_argmax(dev(logits), t)
        return int(host(t)[0])


def test_matmul_known_answers(cuda):
    G = Gpu()
    for label, W, x, rows, cols, t, want, tol in matmul_kats():
        out = np.zeros(rows, np.float32)
        G.matmul(out, np.ascontiguousarray(W), np.ascontiguousarray(x, np.float32), rows, cols, t)
        assert np.all(np.abs(out - np.asarray(want, np.float32)) < tol), (label, out)


def test_elementwise_known_answers(cuda):
    """rmsnorm test_ops.cpp:92-127, vec_add 202-213, ffn_swiglu 215-268
    (F32 weights, 3x2), argmax 583-596."""
    G = Gpu()
    o = np.zeros(4, np.float32)
    G.rmsnorm(o, np.ones(4, np.float32), np.ones(4, np.float32), 1e-5)
    assert abs(o[0] - 1.0) < 1e-3
    r = 1.0 / np.sqrt(12.5)
    o2 = np.zeros(2, np.float32)
    G.rmsnorm(o2, np.array([3, 4], np.float32), np.array([2, 0.5], np.float32), 0.0)
    assert np.allclose(o2, [3 * r * 2, 4 * r * 0.5], atol=1e-4)
    a = np.array([1, 2, 3], np.float32)
    G.vec_add(a, np.array([10, 20, 30], np.float32))
    assert np.allclose(a, [11, 22, 33], atol=1e-4)
    gate = np.array([1, 0, 0, 1, 1, 1], np.float32).view(np.uint8)
    up = np.array([1, 1, 0, 1, 1, 0], np.float32).view(np.uint8)
    down = np.array([1, 0, 1, 0, 1, 0], np.float32).view(np.uint8)
    out = np.zeros(2, np.float32)
    G.ffn_swiglu(out, np.array([1, 2], np.float32), gate, up, down, 3, 2, F32)
    s = lambda v: v / (1 + np.exp(-v))  # noqa: E731
    assert np.allclose(out, [s(1.0) * 3 + s(3.0), s(2.0) * 2], atol=1e-3)
    assert G.sample_argmax(np.array([1, 5, 3, 2], np.float32)) == 1
    assert G.sample_argmax(np.array([-1, -5, -0.5, -2], np.float32)) == 2


@pytest.mark.parametrize("wtype,rows,cols", [
    (F32, 100, 2048), (F32, 7, 3), (F16, 96, 2048), (F16, 5, 10), (Q8_0, 300, 2048),
    (Q4_0, 2560, 2048), (Q4_0, 2048, 5632), (Q4_0, 33, 64), (Q6_K, 256, 2048),
    (Q4_0, 32000, 2048),
])
def test_matmul_matches_oracle(cuda, wtype, rows, cols):
    rng = np.random.default_rng(rows + cols + wtype)
    W = synth.random_weight(rng, wtype, rows, cols)
    x = rng.standard_normal(cols, dtype=np.float32)
    got = np.zeros(rows, np.float32)
    Gpu().matmul(got, W, x, rows, cols, wtype)
    want = np.zeros(rows, np.float32)
    oracle.port().matmul(want, W, x, rows, cols, wtype)
    truth, scale = matmul_truth(W, x, rows, cols, wtype)
    bound = ROW_TOL * scale + 1e-7
    assert np.all(np.abs(want - truth) <= bound)          # the oracle meets the bound
    err = np.abs(got - truth)
    assert np.all(err <= bound), float(np.max(err / bound))
    assert np.max(np.abs(got - want)) <= 2 * np.max(bound)


def test_argmax_exact(cuda):
    G = Gpu()
    rng = np.random.default_rng(1)
    P = oracle.port()
    cases = [rng.standard_normal(32000, dtype=np.float32) for _ in range(5)]
    tie = rng.standard_normal(32000, dtype=np.float32)
    tie[[100, 20000, 31999]] = 50.0                        # first of three equal maxima
    cases += [tie, np.array([np.nan, 1, 2], np.float32), np.array([1, np.nan, 2, np.nan], np.float32),
              np.full(33, -np.inf, np.float32), np.array([3.0], np.float32)]
    late = np.zeros(32000, np.float32)
    late[31999] = 1.0
    cases.append(late)
    for c in cases:
        assert G.sample_argmax(c) == P.sample_argmax(c)


def test_ffn_swiglu_q4_matches_oracle(cuda):
    rng = np.random.default_rng(7)
    n_embd, n_ff = 2048, 5632
    Wg = synth.random_weight(rng, Q4_0, n_ff, n_embd)
    Wu = synth.random_weight(rng, Q4_0, n_ff, n_embd)
    Wd = synth.random_weight(rng, Q4_0, n_embd, n_ff)
    x = rng.standard_normal(n_embd, dtype=np.float32)
    got = np.zeros(n_embd, np.float32)
    Gpu().ffn_swiglu(got, x, Wg, Wu, Wd, n_ff, n_embd, Q4_0)
    want = np.zeros(n_embd, np.float32)
    oracle.port().ffn_swiglu(want, x, Wg, Wu, Wd, n_ff, n_embd, Q4_0)
    # error scale: the down product's sum |w h| with h from float64
    g, _ = matmul_truth(Wg, x, n_ff, n_embd, Q4_0)
    u, _ = matmul_truth(Wu, x, n_ff, n_embd, Q4_0)
    h = g / (1 + np.exp(-g)) * u
    _, scale = matmul_truth(Wd, h.astype(np.float32), n_embd, n_ff, Q4_0)
    assert np.all(np.abs(got - want) <= 1e-4 * scale + 1e-6), float(np.max(np.abs(got - want) / scale))


@pytest.mark.parametrize("wtype,out_type,n_layers,vocab", [
    (Q4_0, Q4_0, 2, 32000), (Q8_0, None, 2, 4096), (Q6_K, Q6_K, 1, 2048), (F16, F16, 1, 1024),
])
def test_forward_matches_oracle(cuda, wtype, out_type, n_layers, vocab):
    """Teacher-forced tokens through tle_forward and the oracle's forward():
    logits close at every step, same greedy token whenever it is decided by
    more than the tolerance, identical K/V cache rows within tolerance."""
    import torch
    import tle
    m = synth.make_model(seed=5 + wtype, n_layers=n_layers, wtype=wtype, output_type=out_type,
                         n_vocab=vocab, n_ctx=64)
    dm = tle.DeviceModel(m)
    ds = tle.DeviceState(dm)
    hf = oracle.HostForward(m)
    P = oracle.port()
    tokens = [1, vocab - 1, 17, 17, 300 % vocab, 2]
    tok_dev = torch.tensor(tokens, dtype=torch.int32, device="cuda")
    # Q4_0 models run every layer in one persistent launch, the others per product
    assert tle.forward_layers_one_launch(dm, ds, 0) == (wtype == Q4_0)
    for pos, tok in enumerate(tokens):
        tle.forward(dm, ds, tok_dev[pos:pos + 1], pos)
        want = P.forward(hf, tok, pos)
        got = host(ds.logits)
        assert np.all(np.isfinite(got))
        tol = 2e-3 * float(np.max(np.abs(want)))
        assert float(np.max(np.abs(got - want))) <= tol, (pos, float(np.max(np.abs(got - want))), tol)
        top2 = np.sort(want)[-2:]
        if top2[1] - top2[0] > 2 * tol:
            assert int(np.argmax(got)) == int(np.argmax(want))
    kc = host(ds.t["key_cache"]).reshape(n_layers, 64, -1)[:, :len(tokens)]
    kw = hf.bufs["key_cache"].reshape(n_layers, 64, -1)[:, :len(tokens)]
    assert float(np.max(np.abs(kc - kw))) <= 2e-3 * float(np.max(np.abs(kw)))
    assert tle.device_error() == 0


def test_forward_persistent_attention_chunks_match_oracle(cuda):
    """The one-launch forward over 576 positions: the attention split grows
    from 1 to 9 chunks of 64 rows per KV head (the record fold takes its
    one-pass form up to 8 chunks, its two-pass form at 9), checked against
    the oracle's forward() at chunk edges."""
    import torch
    import tle
    n = 576
    m = synth.make_model(seed=21, n_layers=1, n_vocab=512, n_ctx=n)
    dm = tle.DeviceModel(m)
    ds = tle.DeviceState(dm)
    hf = oracle.HostForward(m)
    P = oracle.port()
    tokens = np.random.default_rng(21).integers(0, 512, n)
    tok_dev = torch.tensor(tokens.astype(np.int32), device="cuda")
    checks = {0, 63, 64, 127, 200, 511, 512, 575}
    for pos in range(n):
        assert tle.forward_layers_one_launch(dm, ds, pos)
        tle.forward(dm, ds, tok_dev[pos:pos + 1], pos)
        want = P.forward(hf, int(tokens[pos]), pos)
        if pos in checks:
            got = host(ds.logits)
            tol = 2e-3 * float(np.max(np.abs(want)))
            assert float(np.max(np.abs(got - want))) <= tol, (pos, float(np.max(np.abs(got - want))), tol)
    assert tle.device_error() == 0


def test_forward_bad_token_is_reported(cuda):
    import torch
    import tle
    m = synth.make_model(seed=1, n_layers=1, n_vocab=256, n_ctx=8)
    dm = tle.DeviceModel(m)
    ds = tle.DeviceState(dm)
    tle.forward(dm, ds, torch.tensor([256], dtype=torch.int32, device="cuda"), 0)
    assert tle.device_error() == 0x106
    tle.forward(dm, ds, torch.tensor([3], dtype=torch.int32, device="cuda"), 1)
    assert np.all(np.isfinite(host(ds.logits)))
    assert tle.device_error() == 0


def test_greedy_generation_device_fed_matches_synced_and_oracle(cuda):
    """Greedy generation with the token of step t+1 written by the device
    sampler and read by the next step's embedding, no host sync in between
    (every launch a programmatic dependent of the one before): the same
    tokens as a run synchronised after every step, and as the oracle's own
    greedy loop (forward() then sample_argmax, generate.cpp:76-102)."""
    import torch
    import tle
    prompt, gen = 6, 18
    n = prompt + gen
    m = synth.make_model(seed=11, n_layers=2, n_vocab=32000, n_ctx=n)
    dm = tle.DeviceModel(m)
    ids = np.random.default_rng(11).integers(0, m.n_vocab, prompt).astype(np.int32)

    def generate(sync):
        ds = tle.DeviceState(dm)
        toks = torch.zeros(n + 1, dtype=torch.int32, device="cuda")
        toks[:prompt] = torch.from_numpy(ids).cuda()
        for pos in range(n):
            tle.forward(dm, ds, toks[pos:pos + 1], pos)
            if pos >= prompt - 1:
                tle.sample_argmax(ds.logits, toks[pos + 1:pos + 2])
            if sync:
                torch.cuda.synchronize()
        return host(toks)[prompt:n + 1]

    fast, synced = generate(False), generate(True)
    assert np.array_equal(fast, synced)
    hf = oracle.HostForward(m)
    P = oracle.port()
    want, tok = [], int(ids[0])
    for pos in range(n):
        tok = int(ids[pos]) if pos < prompt else tok
        P.forward(hf, tok, pos)
        if pos >= prompt - 1:
            tok = P.sample_argmax(hf.logits)
            want.append(tok)
    assert list(synced) == want
    assert tle.device_error() == 0


def _probs(logits, temperature):
    x = logits.astype(np.float32).copy()
    if temperature != 1.0 and temperature > 0:
        x *= np.float32(1.0) / np.float32(temperature)
    e = np.exp(x - x.max(), dtype=np.float32)
    return e / e.sum(dtype=np.float32)


@pytest.mark.parametrize("scale,temperature", [(1.0, 1.0), (3.0, 0.7), (0.2, 1.5)])
def test_temperature_sampling_matches_oracle(cuda, scale, temperature):
    """With the same uniform draw r the device picks the oracle's token.  The
    draws sit in the middle of a token's cumulative-probability interval
    (sequential fp32 sums, as the reference's), away from the summation-
    order differences; the logits are left as the probabilities, like the
    reference."""
    import torch
    import tle
    rng = np.random.default_rng(int(scale * 10))
    lg = (rng.standard_normal(32000) * scale).astype(np.float32)
    p = _probs(lg, temperature)
    c = np.cumsum(p, dtype=np.float32)
    P = oracle.port()
    picks = [int(i) for i in np.argsort(-p)[:6]] + [int(x) for x in rng.integers(0, 32000, 6)]
    tested = 0
    for i in picks:
        lo = float(c[i - 1]) if i else 0.0
        if float(c[i]) - lo < 2e-5 or float(c[i]) >= 1.0:
            continue
        r = (lo + float(c[i])) / 2
        want = P.sample_temperature(lg.copy(), temperature, r)
        dl = dev(lg)
        t = torch.zeros(1, dtype=torch.int32, device="cuda")
        tle.sample_temperature(dl, t, temperature, r)
        assert int(host(t)[0]) == want, (i, want)
        assert np.allclose(host(dl), p, rtol=1e-5, atol=1e-9)
        tested += 1
    assert tested >= 3


@pytest.mark.parametrize("scale,top_p", [(6.0, 0.9), (4.5, 0.9), (3.0, 0.5), (9.0, 0.95)])
def test_top_p_sampling_matches_oracle(cuda, scale, top_p):
    import torch
    import tle
    rng = np.random.default_rng(int(scale * 100))
    lg = (rng.standard_normal(32000) * scale).astype(np.float32)
    temperature = 0.8
    p = _probs(lg, temperature)
    order = np.argsort(-p, kind="stable")
    cs = np.cumsum(p[order].astype(np.float64))
    m = int(np.searchsorted(cs, top_p) + 1)
    total = cs[m - 1]
    P = oracle.port()
    for k in range(min(m, 5)):
        lo = cs[k - 1] if k else 0.0
        if cs[k] - lo < 1e-4 * total:
            continue
        r = float((lo + cs[k]) / 2 / total)
        want = P.sample_top_p(lg.copy(), temperature, top_p, r)
        t = torch.zeros(1, dtype=torch.int32, device="cuda")
        tle.sample_top_p(dev(lg), t, temperature, top_p, r)
        assert int(host(t)[0]) == want, (k, m, want)
        assert want == int(order[k])
