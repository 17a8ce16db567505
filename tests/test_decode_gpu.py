"""GPU parity of the decode path (tle_rope, tle_attention, tle_rope_attention,
tle_decode_batch) against the reference: golden fixtures made by the
reference itself, the reference suite's known-answer tests
(src/test_ops.cpp:295-546) run through the CUDA path, and the C oracle on
seeded inputs up to the north-star shapes.

Tolerance: max-abs 1e-4 on attention outputs (fp32 accumulation, the
north-star bound); 1e-5 on rotated q/k and appended cache rows (device
sincosf vs glibc sinf/cosf).
"""
import numpy as np
import pytest

import oracle
from conftest import load_golden

pytestmark = pytest.mark.gpu

NH, NKV, HD = 32, 4, 64
QD, KVD = NH * HD, NKV * HD
ATOL = 1e-4
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


# --------------------------------------------------------------- golden
@pytest.mark.parametrize("name", ["decode_mid", "decode_pos0", "decode_full"])
@pytest.mark.parametrize("fused", [True, False])
def test_golden_decode(cuda, name, fused):
    import tle
    g = load_golden(name)
    layer, pos, n_ctx = int(g["layer"]), int(g["pos"]), int(g["n_ctx"])
    shape = tle.tinyllama_shape(int(g["n_layers"]))
    kc, vc = dev(g["key_cache"]), dev(g["value_cache"])
    q, k, v = dev(g["q"]), dev(g["k"]), dev(g["v"])
    out = dev(np.full(QD, np.nan, np.float32))
    if fused:
        tle.rope_attention(out, q, k, v, kc, vc, layer, pos, n_ctx, shape)
        assert np.array_equal(host(q), g["q"].astype(np.float32))  # fused call leaves q untouched
    else:
        tle.rope(q, k, pos)
        assert maxabs(host(q), g["q_rot"]) <= ROT_ATOL
        tle.attention(out, q, k, v, kc, vc, layer, pos, n_ctx, shape)
    assert maxabs(host(out), g["out"]) <= ATOL
    kc_h, vc_h = host(kc), host(vc)
    assert maxabs(kc_h[layer, pos], g["k_rot"]) <= ROT_ATOL
    assert np.array_equal(vc_h[layer, pos], g["v"].astype(np.float32))
    # every other row untouched
    ref_kc = g["key_cache"].astype(np.float32)
    mask = np.ones(ref_kc.shape[:2], bool); mask[layer, pos] = False
    assert np.array_equal(kc_h[mask], ref_kc[mask])
    assert tle.device_error() == 0


def test_golden_rope_positions(cuda):
    import tle
    g = load_golden("rope_positions")
    for i, p in enumerate(g["pos"]):
        q, k = dev(g["q"][i]), dev(g["k"][i])
        tle.rope(q, k, int(p))
        assert maxabs(host(q), g["q_out"][i]) <= ROT_ATOL, int(p)
        assert maxabs(host(k), g["k_out"][i]) <= ROT_ATOL, int(p)


def test_golden_batch(cuda):
    import tle
    g = load_golden("batch_ragged")
    n = len(g["pos"])
    caches = [(dev(g[f"key_cache_{i}"]), dev(g[f"value_cache_{i}"]), int(g["n_ctx"][i]))
              for i in range(n)]
    for max_ctas in (1, 3, 0):
        cs = [(a.clone(), b.clone(), c) for a, b, c in caches]
        batch = tle.DecodeBatch(cs, g["pos"], tle.tinyllama_shape(int(g["n_layers"])), max_ctas)
        out = dev(np.full((n, QD), np.nan, np.float32))
        batch.run(dev(g["q"]), dev(g["k"]), dev(g["v"]), out, int(g["layer"]), rotate=True)
        assert maxabs(host(out), g["out"]) <= ATOL, max_ctas


# ----------------------------------------- reference known-answer tests
def test_known_answers_through_cuda(cuda):
    """test_ops.cpp:295-431 with the CUDA attention (q, k pre-rotated = unrotated at pos 0)."""
    import tle
    n_ctx = 64
    shape = tle.tinyllama_shape(2)
    kc = dev(np.zeros((2, n_ctx, KVD))); vc = dev(np.zeros((2, n_ctx, KVD)))
    out = dev(np.zeros(QD))
    q = dev(np.ones(QD)); k = dev(np.ones(KVD))
    tle.attention(out, q, k, dev(np.arange(KVD) % HD), kc, vc, 0, 0, n_ctx, shape)   # T1
    assert np.allclose(host(out)[:HD], np.arange(HD), atol=1e-3)
    kc.zero_(); vc.zero_()
    tle.attention(out, q, k, dev(np.ones(KVD)), kc, vc, 0, 0, n_ctx, shape)           # T2
    tle.attention(out, q, k, dev(np.full(KVD, 3.0)), kc, vc, 0, 1, n_ctx, shape)
    assert abs(host(out)[0] - 2.0) < 0.01
    kc.zero_(); vc.zero_()
    for p in range(10):                                                               # T3
        tle.attention(out, dev((np.arange(QD) + p) % 11 - 5), dev((np.arange(KVD) + 3 * p) % 7 - 3),
                      dev((np.arange(KVD) + 5 * p) % 9 - 4), kc, vc, 0, p, n_ctx, shape)
    assert np.all(np.isfinite(host(out)))
    kc.zero_(); vc.zero_()
    v = np.zeros(KVD); v[:HD] = 10; v[HD:2 * HD] = 20                                # T4
    tle.attention(out, q, k, dev(v), kc, vc, 0, 0, n_ctx, shape)
    o = host(out)
    assert abs(o[0] - 10) < 0.01 and abs(o[8 * HD] - 20) < 0.01


def test_rope_known_answers_through_cuda(cuda):
    """test_ops.cpp:433-546 with tle_rope."""
    import tle
    q, k = dev(np.ones(QD)), dev(np.ones(KVD))
    tle.rope(q, k, 0)
    assert np.all(np.abs(host(q) - 1) < 1e-4) and np.all(np.abs(host(k) - 1) < 1e-4)
    qh = (np.arange(QD) % 7 - 3).astype(np.float32)
    q, k = dev(qh), dev(np.arange(KVD) % 5 - 2)
    tle.rope(q, k, 42)
    assert abs(np.linalg.norm(host(q)[:HD]) - np.linalg.norm(qh[:HD])) < 1e-3
    q1, k1, q2, k2 = dev(np.ones(QD)), dev(np.ones(KVD)), dev(np.ones(QD)), dev(np.ones(KVD))
    tle.rope(q1, k1, 5); tle.rope(q2, k2, 100)
    assert np.any(np.abs(host(q1)[:HD] - host(q2)[:HD]) >= 1e-4)
    q1, k1 = dev(np.full(QD, 2.5)), dev(np.full(KVD, 2.5))
    q2, k2 = dev(np.full(QD, 2.5)), dev(np.full(KVD, 2.5))
    tle.rope(q1, k1, 17); tle.rope(q2, k2, 17)
    assert np.array_equal(host(q1), host(q2))
    qz = np.zeros(QD, np.float32); qz[0], qz[1] = 3, 4
    q, k = dev(qz), dev(np.zeros(KVD))
    tle.rope(q, k, 1)
    c, s = np.cos(np.float32(1)), np.sin(np.float32(1))
    assert abs(host(q)[0] - (3 * c - 4 * s)) < 1e-4 and abs(host(q)[1] - (3 * s + 4 * c)) < 1e-4


# ------------------------------------------------- seeded, oracle-checked
def run_batch_case(lengths, n_layers, layer, max_ctas, seed, check=None):
    """Random caches/q/k/v for sequences of the given attended lengths; runs the
    CUDA batch decode and the oracle on the sequences in `check` (all by default)."""
    import torch
    import tle
    rng = np.random.default_rng(seed)
    n = len(lengths)
    gen = torch.Generator(device="cuda").manual_seed(seed)
    caches, n_ctx, pos = [], [], []
    for L in lengths:
        cap = int(L + rng.integers(0, 5))
        kc = torch.randn((n_layers, cap, KVD), generator=gen, device="cuda")
        vc = torch.randn((n_layers, cap, KVD), generator=gen, device="cuda")
        caches.append((kc, vc, cap)); n_ctx.append(cap); pos.append(int(L) - 1)
    q = rng.standard_normal((n, QD), dtype=np.float32)
    k = rng.standard_normal((n, KVD), dtype=np.float32)
    v = rng.standard_normal((n, KVD), dtype=np.float32)
    check = list(range(n)) if check is None else list(check)
    kc_h = [caches[i][0].cpu().numpy() for i in check]
    vc_h = [caches[i][1].cpu().numpy() for i in check]
    batch = tle.DecodeBatch(caches, pos, tle.tinyllama_shape(n_layers), max_ctas)
    out = torch.full((n, QD), float("nan"), device="cuda")
    batch.run(dev(q), dev(k), dev(v), out, layer, rotate=True)
    got = host(out)
    want = np.zeros((len(check), QD), np.float32)
    oracle.port().decode_batch(kc_h, vc_h, [n_ctx[i] for i in check], [pos[i] for i in check],
                               q[check].copy(), k[check].copy(), v[check].copy(), want, layer,
                               n_threads=8)
    err = maxabs(got[check], want)
    # appended rows: the oracle appended into its host copies
    for j, i in enumerate(check):
        row_dev = caches[i][0][layer, pos[i]].cpu().numpy()
        assert maxabs(row_dev, kc_h[j][layer, pos[i]]) <= ROT_ATOL
        assert np.array_equal(caches[i][1][layer, pos[i]].cpu().numpy(), v[i])
    return err, batch.n_ctas


@pytest.mark.parametrize("lengths,max_ctas", [
    ([1], 0), ([2], 0), ([31], 0), ([32], 0), ([33], 0), ([64], 1), ([1000], 0),
    ([1, 1, 1, 1, 1], 3),                       # many tiny sequences per CTA
    ([5, 4097, 33, 1, 640], 0),                 # ragged, split across CTAs
    ([300, 300, 300, 300], 7),                  # CTA boundaries inside sequences
    ([2048] * 6, 148),
])
def test_batch_decode_matches_oracle(cuda, lengths, max_ctas):
    err, _ = run_batch_case(lengths, n_layers=2, layer=1, max_ctas=max_ctas, seed=sum(lengths))
    assert err <= ATOL, err


def test_single_long_context_matches_oracle(cuda):
    """One sequence, 16384 cached rows, split over ~148 CTAs and merged."""
    import torch
    import tle
    rng = np.random.default_rng(11)
    n_ctx, pos, layer = 16400, 16383, 0
    kc_h = rng.standard_normal((1, n_ctx, KVD), dtype=np.float32)
    vc_h = rng.standard_normal((1, n_ctx, KVD), dtype=np.float32)
    q = rng.standard_normal(QD, dtype=np.float32)
    k = rng.standard_normal(KVD, dtype=np.float32)
    v = rng.standard_normal(KVD, dtype=np.float32)
    kc, vc = dev(kc_h), dev(vc_h)
    out = dev(np.zeros(QD))
    tle.rope_attention(out, dev(q), dev(k), dev(v), kc, vc, layer, pos, n_ctx, tle.tinyllama_shape(1))
    want = np.zeros(QD, np.float32)
    P = oracle.port()
    q2, k2 = q.copy(), k.copy()
    P.rope(q2, k2, pos)
    P.attention(want, q2, k2, v, kc_h, vc_h, layer, pos, n_ctx)
    assert maxabs(host(out), want) <= ATOL


_SHARED_WS = {}


@pytest.mark.parametrize("L", [1, 2, 31, 32, 33, 64, 65, 255, 256, 257, 512, 513, 1000, 2047,
                               2048, 2049])
def test_single_sequence_lengths_match_oracle(cuda, L):
    """rope + attention of one sequence at lengths across the chunk
    boundaries: up to 2048 rows one launch splits the rows over a cluster of
    up to 8 CTAs per KV head (32 to 256 rows each) merged in distributed
    shared memory; 2049 takes the SM split and its second launch.  Three
    calls on one workspace give identical outputs, and the appended row is
    the rotated k / v."""
    import tle
    rng = np.random.default_rng(1000 + L)
    n_layers, layer, n_ctx = 2, 1, L + 5
    kc_h = rng.standard_normal((n_layers, n_ctx, KVD), dtype=np.float32)
    vc_h = rng.standard_normal((n_layers, n_ctx, KVD), dtype=np.float32)
    q = rng.standard_normal(QD, dtype=np.float32)
    k = rng.standard_normal(KVD, dtype=np.float32)
    v = rng.standard_normal(KVD, dtype=np.float32)
    shape = tle.tinyllama_shape(n_layers)
    if "ws" not in _SHARED_WS:
        _SHARED_WS["ws"] = tle.attention_workspace(shape, 4096)
    kc, vc = dev(kc_h), dev(vc_h)
    out, lse = dev(np.full(QD, np.nan, np.float32)), dev(np.zeros(32))
    pos = L - 1
    for _ in range(2):   # twice on the same workspace: identical outputs
        tle.rope_attention(out, dev(q), dev(k), dev(v), kc, vc, layer, pos, n_ctx, shape, _SHARED_WS["ws"])
        first = host(out).copy()
    tle.rope_attention(out, dev(q), dev(k), dev(v), kc, vc, layer, pos, n_ctx, shape, _SHARED_WS["ws"])
    assert np.array_equal(host(out), first)
    want = np.zeros(QD, np.float32)
    P = oracle.port()
    q2, k2 = q.copy(), k.copy()
    P.rope(q2, k2, pos)
    P.attention(want, q2, k2, v, kc_h, vc_h, layer, pos, n_ctx)   # appends row pos of kc_h / vc_h
    assert maxabs(first, want) <= ATOL
    got_kc, got_vc = host(kc), host(vc)
    assert maxabs(got_kc[layer, pos], kc_h[layer, pos]) <= ROT_ATOL
    assert np.array_equal(got_vc[layer, pos], v)
    mask = np.ones((n_layers, n_ctx), bool)
    mask[layer, pos] = False
    assert np.array_equal(got_kc[mask], kc_h[mask]) and np.array_equal(got_vc[mask], vc_h[mask])
    # the log-sum-exp variant (context split) on the same rows: same output
    # and lse = log sum_p exp(q.K_p / 8) per head
    out2 = dev(np.full(QD, np.nan, np.float32))
    tle.attention_lse(out2, lse, dev(q2), dev(k2), dev(v), kc, vc, layer, pos, n_ctx, shape, _SHARED_WS["ws"])
    assert maxabs(host(out2), want) <= ATOL
    K = kc_h[layer, :L].reshape(L, 4, 64)
    sc = np.einsum("hd,phd->hp", q2.reshape(32, 64).astype(np.float64) / 8.0,
                   np.repeat(K.astype(np.float64), 8, axis=1))
    mx = sc.max(1)
    want_lse = mx + np.log(np.exp(sc - mx[:, None]).sum(1))
    assert maxabs(host(lse), want_lse) <= 1e-4
    assert tle.device_error() == 0


def test_config4_shapes_all_sequences(cuda):
    """North-star config 4: 64 sequences, lengths U[128, 2048], 22-layer caches;
    layer 13 checked for every sequence."""
    rng = np.random.default_rng(4)
    lengths = rng.integers(128, 2049, 64)
    err, n_ctas = run_batch_case(lengths, n_layers=22, layer=13, max_ctas=0, seed=4)
    assert n_ctas > 1
    assert err <= ATOL, err


def test_repeat_call_is_idempotent(cuda):
    """Decoding the same token twice rewrites the same row and gives the same output."""
    import torch
    import tle
    rng = np.random.default_rng(5)
    kc = dev(rng.standard_normal((1, 700, KVD), dtype=np.float32))
    vc = dev(rng.standard_normal((1, 700, KVD), dtype=np.float32))
    q, k, v = (dev(rng.standard_normal(n, dtype=np.float32)) for n in (QD, KVD, KVD))
    o1, o2 = dev(np.zeros(QD)), dev(np.zeros(QD))
    shape = tle.tinyllama_shape(1)
    tle.rope_attention(o1, q, k, v, kc, vc, 0, 650, 700, shape)
    tle.rope_attention(o2, q, k, v, kc, vc, 0, 650, 700, shape)
    assert np.array_equal(host(o1), host(o2))


def test_invalid_arguments_fail_loudly(cuda):
    import tle
    shape = tle.tinyllama_shape(1)
    kc, vc = dev(np.zeros((2, 8, KVD))), dev(np.zeros((2, 8, KVD)))
    out, q, k, v = dev(np.zeros(QD)), dev(np.zeros(QD)), dev(np.zeros(KVD)), dev(np.zeros(KVD))
    with pytest.raises(tle.TleError) as e:
        tle.attention(out, q, k, v, kc, vc, 0, 8, 8, shape)   # pos == n_ctx
    assert e.value.code == tle.TLE_ERR_INVALID
    with pytest.raises(tle.TleError) as e:
        tle.attention(out, q, k, v, kc, vc, 1, 3, 8, shape)   # layer >= shape.n_layers
    assert e.value.code == tle.TLE_ERR_INVALID


def test_batch_replay_without_upload(cuda):
    """The split-K merge runs in the last CTA of each sequence, counted in the
    descriptor's arrival words; the merging CTA resets them, so running the
    same uploaded descriptor again (as a CUDA graph replay does) gives the same
    output and leaves every count at zero."""
    import torch
    import tle
    rng = np.random.default_rng(21)
    lengths = [3000, 17, 900, 2500, 64, 1]
    n = len(lengths)
    caches, pos = [], []
    for L in lengths:
        kc = dev(rng.standard_normal((1, L + 2, KVD), dtype=np.float32))
        vc = dev(rng.standard_normal((1, L + 2, KVD), dtype=np.float32))
        caches.append((kc, vc, L + 2)); pos.append(L - 1)
    batch = tle.DecodeBatch(caches, pos, tle.tinyllama_shape(1), 40)
    assert batch.n_ctas > n
    q = dev(rng.standard_normal((n, QD), dtype=np.float32))
    k = dev(rng.standard_normal((n, KVD), dtype=np.float32))
    v = dev(rng.standard_normal((n, KVD), dtype=np.float32))
    outs = []
    for _ in range(3):
        o = torch.full((n, QD), float("nan"), device="cuda")
        batch.run(q, k, v, o, 0, rotate=True)
        outs.append(host(o))
    assert np.all(np.isfinite(outs[0]))
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[0], outs[2])
    off = 32 + 24 * n + 8 * (batch.n_ctas + 1) + 8 * n
    arrivals = batch._desc_dev[off:off + 4 * n].cpu().numpy()
    assert not arrivals.any(), arrivals


def test_bounded_wait_expiry_is_reported_and_context_survives(cuda):
    """The kernels' bounded mbarrier wait, planted on a barrier nothing
    arrives at (tle_selftest_wait_timeout, 20 ms limit), records 0x1ff in
    the device error word and returns; the context then runs a decode that
    matches the oracle."""
    import tle
    assert tle.device_error() == 0
    tle.selftest_wait_timeout(20000)
    assert tle.device_error() == 0x1FF
    assert tle.device_error() == 0            # cleared by the read above
    err, _ = run_batch_case([300, 40], n_layers=1, layer=0, max_ctas=4, seed=99)
    assert err <= ATOL, err
    assert tle.device_error() == 0


@pytest.mark.parametrize("n_rows,world", [(10000, 3), (700, 2), (4096, 8)])
def test_context_split_matches_oracle(cuda, n_rows, world):
    """One sequence whose rows are split over `world` shards (shard.context_plan),
    each decoded with tle_attention_lse on its own cache, the (out, lse) pairs
    merged with tle_merge_lse: equals the oracle's rope + attention over all
    rows, and the shard holding the new row appends it as the oracle does."""
    import torch
    import tle
    import shard
    rng = np.random.default_rng(n_rows + world)
    n_layers, layer = 2, 1
    pos = n_rows - 1
    kc = rng.standard_normal((n_layers, n_rows + 3, KVD), dtype=np.float32)
    vc = rng.standard_normal((n_layers, n_rows + 3, KVD), dtype=np.float32)
    q = rng.standard_normal(QD, dtype=np.float32)
    k = rng.standard_normal(KVD, dtype=np.float32)
    v = rng.standard_normal(KVD, dtype=np.float32)
    plan = shard.context_plan(n_rows, world)
    shape = tle.tinyllama_shape(n_layers)
    qd, kd = dev(q), dev(k)
    tle.rope(qd, kd, pos)                             # global position, in place
    parts = torch.empty((world, QD), device="cuda")
    lses = torch.empty((world, 32), device="cuda")
    shards = []
    for r, (r0, r1) in enumerate(plan.bounds):
        cap = r1 - r0 + 1
        skc = dev(np.ascontiguousarray(kc[:, r0:r0 + cap]))
        svc = dev(np.ascontiguousarray(vc[:, r0:r0 + cap]))
        shards.append((skc, svc))
        if r == world - 1:
            tle.attention_lse(parts[r], lses[r], qd, kd, dev(v), skc, svc, layer, pos - r0, cap, shape)
        else:
            row = r1 - r0 - 1
            tle.attention_lse(parts[r], lses[r], qd, skc[layer, row], svc[layer, row], skc, svc,
                              layer, row, cap, shape)
    out = torch.empty(QD, device="cuda")
    tle.merge_lse(out, parts, lses)
    want = np.zeros(QD, np.float32)
    P = oracle.port()
    q2, k2 = q.copy(), k.copy()
    P.rope(q2, k2, pos)
    P.attention(want, q2, k2, v, kc, vc, layer, pos, n_rows + 3)
    assert maxabs(host(out), want) <= ATOL
    r0 = plan.bounds[-1][0]
    assert maxabs(host(shards[-1][0])[layer, pos - r0], kc[layer, pos]) <= ROT_ATOL
    assert np.array_equal(host(shards[-1][1])[layer, pos - r0], v)
    for r in range(world - 1):                         # earlier shards unchanged
        a, b = plan.bounds[r]
        assert np.array_equal(host(shards[r][0])[layer, :b - a], kc[layer, a:b])
    assert tle.device_error() == 0


def test_many_short_sequences_per_cta(cuda):
    """2000 sequences of 1..120 rows: far more sequences than CTAs, so every
    CTA walks dozens of whole-sequence segments (q prefetch across segments,
    the tile ring running ahead over segment boundaries); a sample of 300
    sequences is checked against the oracle."""
    rng = np.random.default_rng(77)
    lengths = rng.integers(1, 121, 2000)
    check = sorted(rng.choice(2000, 300, replace=False).tolist())
    err, n_ctas = run_batch_case(lengths, n_layers=1, layer=0, max_ctas=0, seed=77, check=check)
    assert n_ctas >= 100
    assert err <= ATOL, err


def test_kv_ready_flag_gives_identical_results(cuda):
    """TLE_DECODE_KV_READY only moves the first tile copies before the wait
    on the previous kernel: two back-to-back layers decoded with it (the
    previous kernel writes a different layer) give bit-identical outputs and
    appended rows to the strict ordering."""
    import torch
    import tle
    rng = np.random.default_rng(31)
    lengths = [3000, 17, 900, 2500, 64, 1, 1500]
    n = len(lengths)
    caches = []
    for L in lengths:
        kc = dev(rng.standard_normal((2, L + 3, KVD), dtype=np.float32))
        vc = dev(rng.standard_normal((2, L + 3, KVD), dtype=np.float32))
        caches.append((kc, vc, L + 3))
    pos = [L - 1 for L in lengths]
    batch = tle.DecodeBatch(caches, pos, tle.tinyllama_shape(2), 60)
    q = [dev(rng.standard_normal((n, QD), dtype=np.float32)) for _ in range(2)]
    k = [dev(rng.standard_normal((n, KVD), dtype=np.float32)) for _ in range(2)]
    v = [dev(rng.standard_normal((n, KVD), dtype=np.float32)) for _ in range(2)]
    res = {}
    for kvr in (False, True, False):
        outs = [torch.full((n, QD), float("nan"), device="cuda") for _ in range(2)]
        for layer in range(2):
            batch.run(q[layer], k[layer], v[layer], outs[layer], layer, True, kv_ready=kvr)
        res.setdefault(kvr, []).append([host(o) for o in outs])
    assert tle.device_error() == 0
    base = res[False][0]
    assert np.all(np.isfinite(base[0])) and np.all(np.isfinite(base[1]))
    for got in res[True] + res[False][1:]:
        assert np.array_equal(got[0], base[0]) and np.array_equal(got[1], base[1])


@pytest.mark.parametrize("L", [1, 65, 512, 2048, 3000])
def test_single_kv_ready_gives_identical_results(cuda, L):
    """tle_rope_attention_flags with TLE_DECODE_KV_READY over a chain of
    layers (each call's previous kernel writes another layer's row) gives
    bit-identical outputs and cache contents to tle_rope_attention, on the
    cluster path (L <= 2048) and the SM split (3000); unknown flag bits are
    rejected."""
    import ctypes
    import torch
    import tle
    rng = np.random.default_rng(77 + L)
    n_layers, n_ctx = 3, L + 2
    pos = L - 1
    shape = tle.tinyllama_shape(n_layers)
    kc_h = rng.standard_normal((n_layers, n_ctx, KVD), dtype=np.float32)
    vc_h = rng.standard_normal((n_layers, n_ctx, KVD), dtype=np.float32)
    q, k, v = (dev(rng.standard_normal((n_layers, n), dtype=np.float32)) for n in (QD, KVD, KVD))
    ws = tle.attention_workspace(shape, n_ctx)
    res = []
    for kvr in (False, True):
        kc, vc = dev(kc_h), dev(vc_h)
        outs = torch.full((n_layers, QD), float("nan"), device="cuda")
        for layer in range(n_layers):
            tle.rope_attention(outs[layer], q[layer], k[layer], v[layer], kc, vc, layer, pos, n_ctx,
                               shape, ws, kv_ready=kvr)
        res.append((host(outs), host(kc), host(vc)))
    assert tle.device_error() == 0
    assert np.all(np.isfinite(res[0][0]))
    for a, b in zip(res[0], res[1]):
        assert np.array_equal(a, b)
    rc = tle.lib().tle_rope_attention_flags(
        ctypes.c_void_p(outs.data_ptr()), ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(k.data_ptr()),
        ctypes.c_void_p(v.data_ptr()), ctypes.c_void_p(kc.data_ptr()), ctypes.c_void_p(vc.data_ptr()),
        0, pos, n_ctx, ctypes.byref(shape), 4, ctypes.c_void_p(ws.data_ptr()), ws.numel() * 4, None)
    assert rc != 0


def test_short_batch_matches_split_and_oracle(cuda):
    """tle_decode_batch_short (one cluster per sequence and KV head, every
    sequence <= 2048 rows) agrees with the split-K batch decode to fp32
    rounding and with the oracle to 1e-4, appended rows included."""
    import torch
    import oracle
    import tle
    rng = np.random.default_rng(77)
    lengths = [1, 33, 640, 2048, 1500]
    n = len(lengths)
    hk = [rng.standard_normal((2, L + 2, KVD), dtype=np.float32) for L in lengths]
    hv = [rng.standard_normal((2, L + 2, KVD), dtype=np.float32) for L in lengths]
    q = rng.standard_normal((n, QD), dtype=np.float32)
    k = rng.standard_normal((n, KVD), dtype=np.float32)
    v = rng.standard_normal((n, KVD), dtype=np.float32)
    outs = []
    for short in (False, True):
        caches = [(dev(a), dev(b), L + 2) for a, b, L in zip(hk, hv, lengths)]
        batch = tle.DecodeBatch(caches, [L - 1 for L in lengths], tle.tinyllama_shape(2))
        o = dev(np.full((n, QD), np.nan, np.float32))
        batch.run(dev(q), dev(k), dev(v), o, 1, True, short=short)
        outs.append((host(o), [(host(a), host(b)) for a, b, _ in caches]))
    assert tle.device_error() == 0
    assert float(np.max(np.abs(outs[0][0] - outs[1][0]))) <= 1e-5
    for (ka, va), (kb, vb) in zip(outs[0][1], outs[1][1]):
        assert np.array_equal(va, vb) and float(np.max(np.abs(ka - kb))) <= 1e-6
    P = oracle.port()
    want = np.zeros((n, QD), np.float32)
    P.decode_batch([a.copy() for a in hk], [b.copy() for b in hv], [L + 2 for L in lengths],
                   [L - 1 for L in lengths], q.copy(), k.copy(), v, want, 1)
    assert float(np.max(np.abs(outs[1][0] - want))) <= ATOL


def test_short_batch_record_beyond_max_rows_is_reported(cuda):
    """A record longer than the launch's max_rows (more chunks than the
    cluster has CTAs) is skipped and reported as 0x10a: its output and cache
    are untouched, the other sequences decode as with a correct max_rows
    (to fp32 rounding)."""
    import ctypes
    import torch
    import tle
    rng = np.random.default_rng(78)
    lengths = [100, 700, 300]
    n = len(lengths)
    shape = tle.tinyllama_shape(1)
    hk = [rng.standard_normal((1, L, KVD), dtype=np.float32) for L in lengths]
    hv = [rng.standard_normal((1, L, KVD), dtype=np.float32) for L in lengths]
    q, k, v = (dev(rng.standard_normal((n, d), dtype=np.float32)) for d in (QD, KVD, KVD))
    res = []
    for max_rows in (700, 512):   # 512 rows: 8 chunks of 64, short of the second record
        caches = [(dev(a), dev(b), L) for a, b, L in zip(hk, hv, lengths)]
        batch = tle.DecodeBatch(caches, [L - 1 for L in lengths], shape)
        out = torch.zeros((n, QD), device="cuda")
        tle.device_error(clear=True)
        rc = tle.lib().tle_decode_batch_short(ctypes.byref(shape), batch._desc_dev.data_ptr(), n, max_rows,
                                              ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(k.data_ptr()),
                                              ctypes.c_void_p(v.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                                              0, 1, None)
        assert rc == 0
        res.append((tle.device_error(clear=True), host(out), [host(c[0]) for c in caches]))
    assert res[0][0] == 0 and res[1][0] == 0x10a
    good, bad = res[0][1], res[1][1]
    # (another max_rows gives other chunk sizes, so a different fold order)
    assert maxabs(bad[0], good[0]) <= 1e-5 and maxabs(bad[2], good[2]) <= 1e-5
    assert np.all(bad[1] == 0)
    assert np.array_equal(res[1][2][1], hk[1])   # the skipped record's cache was not touched
