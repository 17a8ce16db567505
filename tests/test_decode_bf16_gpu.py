"""Decode over a bf16 KV cache (tle_decode_batch_bf16) against the oracle.

The oracle runs the reference's rope() and attention() in fp32 over the
same caches converted from bf16, with the appended row rounded to bf16 as
the kernel stores it; the kernel's query and softmax weights are bf16 on the
tensor cores, so the bound is bf16's (2e-2, the prefill contract).
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "tinyllama-engine_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

pytestmark = pytest.mark.gpu

ATOL = 2e-2


def bf16(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(torch.bfloat16).float().numpy()


def run_case(lengths, seed, layer=1, n_layers=2, rotate=True):
    import torch
    import oracle
    import tle
    rng = np.random.default_rng(seed)
    n = len(lengths)
    caches, host = [], []
    for L in lengths:
        n_ctx = L + 3
        kc = torch.randn(n_layers, n_ctx, 256, generator=torch.Generator().manual_seed(int(rng.integers(1 << 30))))
        vc = torch.randn(n_layers, n_ctx, 256, generator=torch.Generator().manual_seed(int(rng.integers(1 << 30))))
        kb, vb = kc.to(torch.bfloat16).cuda(), vc.to(torch.bfloat16).cuda()
        caches.append((kb, vb, n_ctx))
        host.append((kb.float().cpu().numpy(), vb.float().cpu().numpy(), n_ctx))
    q = rng.standard_normal((n, 2048), dtype=np.float32)
    k = rng.standard_normal((n, 256), dtype=np.float32)
    v = rng.standard_normal((n, 256), dtype=np.float32)
    pos = [L - 1 for L in lengths]
    batch = tle.DecodeBatchBf16(caches, pos, tle.tinyllama_shape(n_layers))
    out = torch.full((n, 2048), float("nan"), device="cuda")
    dev = lambda a: torch.from_numpy(a.copy()).cuda()  # noqa: E731
    batch.run(dev(q), dev(k), dev(v), out, layer, rotate=rotate)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    P = oracle.port()
    worst = 0.0
    for i, (kh, vh, n_ctx) in enumerate(host):
        q2, k2 = q[i].copy(), k[i].copy()
        if rotate:
            P.rope(q2, k2, pos[i])
        kr, vr = bf16(k2), bf16(v[i])
        want = np.zeros(2048, np.float32)
        kc_o, vc_o = kh.copy(), vh.copy()
        P.attention(want, q2, kr, vr, kc_o, vc_o, layer, pos[i], n_ctx)
        worst = max(worst, float(np.max(np.abs(got[i] - want))))
        # the appended row: bf16 of the rotated k (one bf16 step of slack for
        # the rotation's last-bit differences) and bf16(v) exactly
        kg = caches[i][0][layer, pos[i]].float().cpu().numpy()
        vg = caches[i][1][layer, pos[i]].float().cpu().numpy()
        assert np.array_equal(vg, vr)
        assert np.all(np.abs(kg - kr) <= np.abs(kr) * 2.0 ** -7 + 1e-30)
        # other rows untouched
        kgl = caches[i][0][layer].float().cpu().numpy()
        mask = np.ones(n_ctx, bool)
        mask[pos[i]] = False
        assert np.array_equal(kgl[mask], kh[layer][mask])
    assert tle.device_error() == 0
    return worst


@pytest.mark.parametrize("lengths", [
    [1, 2, 33, 64, 65],                 # inside one tile, tile edges, a single row
    [700, 2047, 2048, 2049, 4100],      # chunk edges (2048 rows) and a three-chunk merge
])
def test_bf16_decode_matches_oracle(lengths):
    worst = run_case(lengths, seed=len(lengths) + lengths[-1])
    assert worst <= ATOL, worst


def test_bf16_decode_without_rotation():
    worst = run_case([130, 2100], seed=7, rotate=False)
    assert worst <= ATOL, worst


def test_bf16_decode_reports_bad_record():
    """A record whose pos is outside its cache is skipped and reported
    (0x10a); the others are still decoded."""
    import torch
    import tle
    kc = torch.randn(1, 100, 256).to(torch.bfloat16).cuda()
    vc = torch.randn(1, 100, 256).to(torch.bfloat16).cuda()
    kc2, vc2 = kc.clone(), vc.clone()
    kc2_before = kc2.clone()
    batch = tle.DecodeBatchBf16([(kc, vc, 100), (kc2, vc2, 100)], [50, 60], tle.tinyllama_shape(1))
    # corrupt the second record's n_ctx on the device side: pos 60 >= n_ctx 40
    seqs = (tle.SeqBf16 * 2)()
    seqs[0] = tle.SeqBf16(kc.data_ptr(), vc.data_ptr(), 100, 50)
    seqs[1] = tle.SeqBf16(kc2.data_ptr(), vc2.data_ptr(), 40, 60)
    batch._seqs_dev.copy_(torch.frombuffer(bytearray(bytes(seqs)), dtype=torch.uint8))
    q = torch.randn(2, 2048, device="cuda")
    k = torch.randn(2, 256, device="cuda")
    v = torch.randn(2, 256, device="cuda")
    out = torch.zeros(2, 2048, device="cuda")
    tle.device_error(clear=True)
    batch.run(q, k, v, out, 0)
    assert tle.device_error(clear=True) == 0x10a
    assert torch.isfinite(out[0]).all() and bool((out[1] == 0).all())
    assert torch.equal(kc2, kc2_before)   # the bad record's cache was not touched


@pytest.mark.parametrize("page_rows", [64, 256])
def test_bf16_paged_matches_contiguous(page_rows):
    """The same rows in shuffled bf16 page pools give bit-identical outputs
    and appended rows to the contiguous bf16 caches."""
    import torch
    import tle
    rng = np.random.default_rng(page_rows)
    lengths = [70, 2100, 300, 1]
    n = len(lengths)
    shape = tle.tinyllama_shape(2)
    layer = 1
    cont, tables = [], []
    pc = tle.PagedKVCache(sum(-(-L // page_rows) for L in lengths) + 5, page_rows, shape, dtype=torch.bfloat16)
    pc._free = [int(i) for i in rng.permutation(pc.n_pages)]
    for L in lengths:
        kc = torch.randn(2, L, 256).to(torch.bfloat16).cuda()
        vc = torch.randn(2, L, 256).to(torch.bfloat16).cuda()
        cont.append((kc, vc, L))
        ids = pc.alloc(-(-L // page_rows))
        for j, pid in enumerate(ids):
            r0, r1 = page_rows * j, min(page_rows * (j + 1), L)
            pc.key_pool[:, pid, :r1 - r0] = kc[:, r0:r1]
            pc.value_pool[:, pid, :r1 - r0] = vc[:, r0:r1]
        tables.append(pc.table(ids))
    pos = [L - 1 for L in lengths]
    q = torch.randn(n, 2048, device="cuda")
    k = torch.randn(n, 256, device="cuda")
    v = torch.randn(n, 256, device="cuda")
    o1 = torch.full((n, 2048), float("nan"), device="cuda")
    o2 = torch.full((n, 2048), float("nan"), device="cuda")
    tle.DecodeBatchBf16(cont, pos, shape).run(q, k, v, o1, layer)
    tle.PagedDecodeBatchBf16(pc, tables, pos).run(q, k, v, o2, layer)
    torch.cuda.synchronize()
    assert tle.device_error() == 0
    assert torch.isfinite(o1).all() and torch.equal(o1, o2)
    for (kc, vc, L), t in zip(cont, tables):
        p = L - 1
        pid = int(t[p // page_rows])
        assert torch.equal(pc.key_pool[layer, pid, p % page_rows], kc[layer, p])
        assert torch.equal(pc.value_pool[layer, pid, p % page_rows], vc[layer, p])


def test_bf16_paged_bad_page_is_reported():
    """A page id outside the pool is never dereferenced: 0x105."""
    import torch
    import tle
    shape = tle.tinyllama_shape(1)
    pc = tle.PagedKVCache(4, 64, shape, dtype=torch.bfloat16)
    pc.key_pool.normal_()
    pc.value_pool.normal_()
    tables = [pc.table([0, 1]), pc.table([2, 1000])]   # the second table's page 1 is out of the pool
    out = torch.zeros(2, 2048, device="cuda")
    tle.device_error(clear=True)
    tle.PagedDecodeBatchBf16(pc, tables, [100, 100]).run(
        torch.randn(2, 2048, device="cuda"), torch.randn(2, 256, device="cuda"),
        torch.randn(2, 256, device="cuda"), out, 0)
    assert tle.device_error(clear=True) == 0x105
    assert torch.isfinite(out[0]).all()
