"""GPU parity of tle_prefill (tcgen05 causal attention) against the reference's
token-at-a-time prefill (generate.cpp:56-59 -> rope + attention per token).

Tolerance: max-abs 2e-2 on outputs (bf16 tensor-core operands with fp32
accumulation, the north-star prefill bound); the appended fp32 cache rows are
rotated in fp32 and must match within 1e-5.
"""
import numpy as np
import pytest

import oracle
from conftest import load_golden

pytestmark = pytest.mark.gpu

NH, NKV, HD = 32, 4, 64
QD, KVD = NH * HD, NKV * HD
ATOL = 2e-2
ROT_ATOL = 1e-5


def dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()


def host(t):
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


def maxabs(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64))))


@pytest.mark.parametrize("name", ["prefill_fresh", "prefill_chunk"])
def test_golden_prefill(cuda, name):
    import tle
    g = load_golden(name)
    pos0, n_ctx = int(g["pos0"]), int(g["n_ctx"])
    kc, vc = dev(g["key_cache"]), dev(g["value_cache"])
    out = dev(np.full(g["out"].shape, np.nan, np.float32))
    tle.prefill(out, dev(g["q"]), dev(g["k"]), dev(g["v"]), kc, vc, 0, pos0, n_ctx,
                tle.tinyllama_shape(1))
    assert maxabs(host(out), g["out"]) <= ATOL
    n = g["key_cache_after"].shape[0]
    assert maxabs(host(kc)[0, :n], g["key_cache_after"]) <= ROT_ATOL
    assert maxabs(host(vc)[0, :n], g["value_cache_after"]) <= 0.0
    assert tle.device_error() == 0


@pytest.mark.parametrize("n_tokens,pos0,n_ctx", [(1, 0, 8), (129, 0, 140), (300, 77, 400),
                                                 (1024, 0, 1024), (2048, 0, 2048)])
def test_prefill_matches_oracle(cuda, n_tokens, pos0, n_ctx):
    """Every output row and cache row against the oracle's token-at-a-time
    loop (rope + attention per token, bit-exact to the reference's own
    ops.cpp); (2048, 0, 2048) is config 3's shape (about 6 s of oracle)."""
    import tle
    rng = np.random.default_rng(n_tokens + pos0)
    n_layers, layer = 2, 1
    kc = np.zeros((n_layers, n_ctx, KVD), np.float32)
    vc = np.zeros_like(kc)
    kc[:, :pos0] = rng.standard_normal((n_layers, pos0, KVD), dtype=np.float32)
    vc[:, :pos0] = rng.standard_normal((n_layers, pos0, KVD), dtype=np.float32)
    q = rng.standard_normal((n_tokens, QD), dtype=np.float32)
    k = rng.standard_normal((n_tokens, KVD), dtype=np.float32)
    v = rng.standard_normal((n_tokens, KVD), dtype=np.float32)
    dkc, dvc = dev(kc), dev(vc)
    out = dev(np.full((n_tokens, QD), np.nan, np.float32))
    tle.prefill(out, dev(q), dev(k), dev(v), dkc, dvc, layer, pos0, n_ctx,
                tle.tinyllama_shape(n_layers))
    want = np.zeros((n_tokens, QD), np.float32)
    oracle.port().prefill(want, q.copy(), k.copy(), v, kc, vc, layer, pos0, n_ctx)
    got = host(out)
    assert np.all(np.isfinite(got))
    assert maxabs(got, want) <= ATOL
    assert maxabs(host(dkc)[layer, :pos0 + n_tokens], kc[layer, :pos0 + n_tokens]) <= ROT_ATOL
    assert np.array_equal(host(dvc)[layer], vc[layer])
    assert np.array_equal(host(dkc)[0], kc[0])  # other layers untouched


def test_prefill_config3_against_torch_fp32(cuda):
    """North-star config 3 (S=2048, pos0=0) against a torch fp32 causal GQA
    attention of the same rotated inputs: an independent second check of the
    shape the oracle test above also covers."""
    import torch
    import tle
    S, n_ctx = 2048, 2048
    g = torch.Generator(device="cuda").manual_seed(3)
    q = torch.randn((S, QD), generator=g, device="cuda")
    k = torch.randn((S, KVD), generator=g, device="cuda")
    v = torch.randn((S, KVD), generator=g, device="cuda")
    kc = torch.zeros((1, n_ctx, KVD), device="cuda")
    vc = torch.zeros_like(kc)
    out = torch.full((S, QD), float("nan"), device="cuda")
    tle.prefill(out, q, k, v, kc, vc, 0, 0, n_ctx, tle.tinyllama_shape(1))
    torch.cuda.synchronize()
    # torch fp32 reference: rope on q and k (ops.cpp:1223 expression), causal GQA
    half = HD // 2
    inv = torch.tensor([1.0 / np.power(np.float32(10000.0), np.float32(2 * i) / np.float32(HD))
                        for i in range(half)], dtype=torch.float32, device="cuda")
    ang = torch.arange(S, device="cuda", dtype=torch.float32)[:, None] * inv[None, :]
    cs, sn = torch.cos(ang), torch.sin(ang)

    def rot(x, nh):
        x = x.view(S, nh, half, 2)
        x0, x1 = x[..., 0], x[..., 1]
        return torch.stack([x0 * cs[:, None] - x1 * sn[:, None],
                            x0 * sn[:, None] + x1 * cs[:, None]], -1).view(S, nh, HD)

    qr, kr, vv = rot(q, NH), rot(k, NKV), v.view(S, NKV, HD)
    kr_e = kr.repeat_interleave(NH // NKV, dim=1)
    vv_e = vv.repeat_interleave(NH // NKV, dim=1)
    scores = torch.einsum("qhd,khd->hqk", qr, kr_e) / 8.0
    mask = torch.triu(torch.ones(S, S, dtype=torch.bool, device="cuda"), 1)
    scores.masked_fill_(mask, float("-inf"))
    ref = torch.einsum("hqk,khd->qhd", torch.softmax(scores, -1), vv_e).reshape(S, QD)
    err = float((out - ref).abs().max())
    assert err <= ATOL, err
    # appended rows against the reference rope (glibc sinf/cosf; torch's GPU
    # sin/cos of angles up to 2047 rad differ by ~2e-4 and are not the oracle)
    k_h = k.cpu().numpy()
    P = oracle.port()
    want = np.empty_like(k_h)
    qdummy = np.zeros(QD, np.float32)
    for i in range(S):
        kk = k_h[i].copy()
        P.rope(qdummy, kk, i)
        want[i] = kk
    assert maxabs(kc[0].cpu().numpy(), want) <= ROT_ATOL


def test_prefill_rejects_bad_arguments(cuda):
    import tle
    kc = dev(np.zeros((1, 16, KVD)))
    vc = dev(np.zeros((1, 16, KVD)))
    with pytest.raises(tle.TleError) as e:   # pos0 + n_tokens > n_ctx
        tle.prefill(dev(np.zeros((10, QD))), dev(np.zeros((10, QD))), dev(np.zeros((10, KVD))),
                    dev(np.zeros((10, KVD))), kc, vc, 0, 8, 16, tle.tinyllama_shape(1))
    assert e.value.code == tle.TLE_ERR_INVALID


def test_prefill_long_with_prefix_many_items_per_cta(cuda):
    """S = 3000 new tokens after a 1000-row cached prefix: 24 query tiles x 16
    head pairs = 384 work items, so every persistent CTA walks two or three
    items (the Q double buffer is reused) with ragged causal tile counts.
    Checked against a torch fp32 causal GQA attention of the same rows."""
    import torch
    import tle
    S, pos0, n_ctx = 3000, 1000, 4096
    g = torch.Generator(device="cuda").manual_seed(17)
    kc = torch.zeros((1, n_ctx, KVD), device="cuda")
    vc = torch.zeros_like(kc)
    kc[0, :pos0] = torch.randn((pos0, KVD), generator=g, device="cuda")
    vc[0, :pos0] = torch.randn((pos0, KVD), generator=g, device="cuda")
    prefix_k, prefix_v = kc[0, :pos0].clone(), vc[0, :pos0].clone()
    q = torch.randn((S, QD), generator=g, device="cuda")
    k = torch.randn((S, KVD), generator=g, device="cuda")
    v = torch.randn((S, KVD), generator=g, device="cuda")
    out = torch.full((S, QD), float("nan"), device="cuda")
    tle.prefill(out, q, k, v, kc, vc, 0, pos0, n_ctx, tle.tinyllama_shape(1))
    torch.cuda.synchronize()
    assert tle.device_error() == 0
    half = HD // 2
    inv = torch.tensor([1.0 / np.power(np.float32(10000.0), np.float32(2 * i) / np.float32(HD))
                        for i in range(half)], dtype=torch.float32, device="cuda")
    ang = torch.arange(pos0, pos0 + S, device="cuda", dtype=torch.float32)[:, None] * inv[None, :]
    cs, sn = torch.cos(ang), torch.sin(ang)

    def rot(x, nh):
        x = x.view(S, nh, half, 2)
        x0, x1 = x[..., 0], x[..., 1]
        return torch.stack([x0 * cs[:, None] - x1 * sn[:, None],
                            x0 * sn[:, None] + x1 * cs[:, None]], -1).view(S, nh, HD)

    R = pos0 + S
    keys = torch.cat([prefix_k.view(pos0, NKV, HD), rot(k, NKV)], 0)       # [R][4][64]
    vals = torch.cat([prefix_v, v], 0).view(R, NKV, HD)
    qr = rot(q, NH)
    scores = torch.einsum("qhd,khd->hqk", qr, keys.repeat_interleave(NH // NKV, 1)) / 8.0
    allowed = torch.arange(R, device="cuda")[None, :] <= (pos0 + torch.arange(S, device="cuda"))[:, None]
    scores.masked_fill_(~allowed, float("-inf"))
    ref = torch.einsum("hqk,khd->qhd", torch.softmax(scores, -1),
                       vals.repeat_interleave(NH // NKV, 1)).reshape(S, QD)
    err = float((out - ref).abs().max())
    assert err <= ATOL, err
    # prefix rows untouched, new v rows appended as given
    assert torch.equal(kc[0, :pos0], prefix_k) and torch.equal(vc[0, :pos0], prefix_v)
    assert torch.equal(vc[0, pos0:R], v)
