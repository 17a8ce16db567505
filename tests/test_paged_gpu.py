"""GPU parity of the paged batched decode (tle_decode_desc_paged +
tle_decode_batch_paged) against the contiguous batched decode and the C
oracle.

The reference keeps one contiguous [n_layers][n_ctx][256] cache per
sequence (src/run_state.h:20-25, 134-138); the paged variant stores the
same rows in shared page pools behind per-sequence page tables.  The paged
and contiguous paths use the same kernel and the same split of rows over
CTAs, so their outputs and appended rows must be bit-identical; the oracle
bound is max-abs 1e-4 as for every decode output.

Pool pages that hold no row of a sequence, and the rows past each
sequence's position, are filled with NaN: a read of any row the kernel must
not touch shows up as a NaN output.
"""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

NH, NKV, HD = 32, 4, 64
QD, KVD = NH * HD, NKV * HD
ATOL = 1e-4


def host(t):
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


def maxabs(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64))))


class PagedCase:
    """Contiguous caches for `lengths` (attended rows, pos = L - 1) and the
    same rows scattered over a shuffled page pool."""

    def __init__(self, lengths, n_layers, page_rows, seed, spare_rows=0, extra_pages=7):
        import torch
        import tle
        self.rng = np.random.default_rng(seed)
        gen = torch.Generator(device="cuda").manual_seed(seed)
        self.n = len(lengths)
        self.n_layers = n_layers
        self.shape = tle.tinyllama_shape(n_layers)
        self.pos = [int(L) - 1 for L in lengths]
        self.caps = [int(L) + spare_rows for L in lengths]
        self.caches = []
        for cap in self.caps:
            kc = torch.randn((n_layers, cap, KVD), generator=gen, device="cuda")
            vc = torch.randn((n_layers, cap, KVD), generator=gen, device="cuda")
            self.caches.append((kc, vc, cap))
        need = [-(-cap // page_rows) for cap in self.caps]
        n_pages = sum(need) + extra_pages
        self.pc = tle.PagedKVCache(n_pages, page_rows, self.shape)
        self.pc.key_pool.fill_(float("nan"))
        self.pc.value_pool.fill_(float("nan"))
        # hand out pages in a shuffled order so neighbours in a table are not
        # neighbours in the pool
        self.pc._free = [int(i) for i in self.rng.permutation(n_pages)]
        self.ids, self.tables = [], []
        for s, cap in enumerate(self.caps):
            ids = self.pc.alloc(need[s])
            self.ids.append(ids)
            self.tables.append(self.pc.table(ids))
            kc, vc, _ = self.caches[s]
            # rows 0 .. pos-1 are the cached history; row pos and later stay NaN
            L = self.pos[s]
            for j, pid in enumerate(ids):
                a, b = j * page_rows, min((j + 1) * page_rows, L)
                if b > a:
                    self.pc.key_pool[:, pid, :b - a] = kc[:, a:b]
                    self.pc.value_pool[:, pid, :b - a] = vc[:, a:b]

    def inputs(self):
        import torch
        q = self.rng.standard_normal((self.n, QD), dtype=np.float32)
        k = self.rng.standard_normal((self.n, KVD), dtype=np.float32)
        v = self.rng.standard_normal((self.n, KVD), dtype=np.float32)
        return q, k, v, (torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda(),
                         torch.from_numpy(v).cuda())

    def pool_rows(self, s, layer, upto):
        """Rows 0..upto-1 of sequence s, layer `layer`, gathered from the pools."""
        import torch
        pr = self.pc.page_rows
        ks, vs = [], []
        for j, pid in enumerate(self.ids[s]):
            a, b = j * pr, min((j + 1) * pr, upto)
            if b > a:
                ks.append(self.pc.key_pool[layer, pid, :b - a])
                vs.append(self.pc.value_pool[layer, pid, :b - a])
        return torch.cat(ks), torch.cat(vs)


def run_both(case, layer, max_ctas, rotate=True):
    import torch
    import tle
    q, k, v, (dq, dk, dv) = case.inputs()
    cont = tle.DecodeBatch(case.caches, case.pos, case.shape, max_ctas)
    paged = tle.PagedDecodeBatch(case.pc, case.tables, case.pos, max_ctas)
    assert cont.n_ctas == paged.n_ctas
    o_c = torch.full((case.n, QD), float("nan"), device="cuda")
    o_p = torch.full((case.n, QD), float("nan"), device="cuda")
    cont.run(dq, dk, dv, o_c, layer, rotate)
    paged.run(dq, dk, dv, o_p, layer, rotate)
    return q, k, v, host(o_c), host(o_p), paged


@pytest.mark.parametrize("lengths,page_rows,max_ctas", [
    ([1], 16, 0),
    ([16], 16, 0), ([17], 16, 0), ([33], 32, 0),
    ([5, 4097, 33, 1, 640], 16, 0),          # ragged; 32-row tiles straddle 16-row pages
    ([5, 4097, 33, 1, 640], 64, 0),
    ([300, 300, 300, 300], 256, 7),          # CTA boundaries inside pages
    ([2048] * 6, 1024, 148),
    ([1, 1, 1, 1, 1], 16, 3),                # many one-row sequences per CTA
])
def test_paged_matches_contiguous_bit_for_bit_and_oracle(cuda, lengths, page_rows, max_ctas):
    import tle
    layer, n_layers = 1, 2
    case = PagedCase(lengths, n_layers, page_rows, seed=sum(lengths) + page_rows)
    q, k, v, o_c, o_p, _ = run_both(case, layer, max_ctas)
    assert tle.device_error() == 0
    assert np.all(np.isfinite(o_p))
    assert np.array_equal(o_c, o_p)
    # the appended row, read back through the page table, equals the
    # contiguous cache's appended row
    for s in range(case.n):
        kp, vp = case.pool_rows(s, layer, case.pos[s] + 1)
        kc, vc, _ = case.caches[s]
        assert np.array_equal(host(kp), host(kc[layer, :case.pos[s] + 1]))
        assert np.array_equal(host(vp), host(vc[layer, :case.pos[s] + 1]))
    # the other layer's rows were not touched
    for s in range(case.n):
        kp, _ = case.pool_rows(s, 0, case.pos[s] + 1)
        assert np.all(np.isnan(host(kp)[case.pos[s]]))
    # oracle on the contiguous copies (made before the decode appended)
    check = list(range(min(case.n, 6)))
    kc_h = [host(case.caches[s][0]) for s in check]
    vc_h = [host(case.caches[s][1]) for s in check]
    for j, s in enumerate(check):   # the oracle appends row pos itself
        kc_h[j][layer, case.pos[s]] = np.nan
        vc_h[j][layer, case.pos[s]] = np.nan
    want = np.zeros((len(check), QD), np.float32)
    oracle.port().decode_batch(kc_h, vc_h, [case.caps[s] for s in check],
                               [case.pos[s] for s in check], q[check].copy(), k[check].copy(),
                               v[check].copy(), want, layer, n_threads=8)
    assert maxabs(o_p[check], want) <= ATOL


def test_paged_decode_steps_cross_page_boundaries(cuda):
    """Thirty decode steps in which every sequence grows across page
    boundaries (16-row pages), alternating layers; after every step the paged
    output equals the contiguous one bit for bit, and at the end every cached
    row matches."""
    import torch
    import tle
    lengths = [10, 31, 200, 47, 1]
    steps = 30
    case = PagedCase(lengths, 2, 16, seed=7, spare_rows=steps)
    cont = tle.DecodeBatch(case.caches, case.pos, case.shape, 9)
    paged = tle.PagedDecodeBatch(case.pc, case.tables, case.pos, 9)
    for t in range(steps):
        layer = t & 1                  # both layers of a token, then the next token
        pos = [p + (t >> 1) for p in case.pos]
        if t and layer == 0:
            cont.set_positions(pos)
            paged.set_positions(pos)
        _, _, _, (dq, dk, dv) = case.inputs()
        o_c = torch.empty((case.n, QD), device="cuda")
        o_p = torch.empty((case.n, QD), device="cuda")
        cont.run(dq, dk, dv, o_c, layer)
        paged.run(dq, dk, dv, o_p, layer)
        a, b = host(o_c), host(o_p)
        assert np.all(np.isfinite(b)), t
        assert np.array_equal(a, b), t
    assert tle.device_error() == 0
    for s in range(case.n):
        for layer in (0, 1):
            kp, vp = case.pool_rows(s, layer, pos[s] + 1)
            kc, vc, _ = case.caches[s]
            assert np.array_equal(host(kp), host(kc[layer, :pos[s] + 1]))
            assert np.array_equal(host(vp), host(vc[layer, :pos[s] + 1]))


def test_paged_config4_shapes_match_oracle(cuda):
    """North-star config 4 (64 sequences, lengths U[128, 2048], 22 layers) on
    256-row pages: bit-identical to the contiguous cache, every sequence
    checked against the oracle on layer 13."""
    import tle
    lengths = np.random.default_rng(4).integers(128, 2049, 64)
    case = PagedCase(lengths, 22, 256, seed=4, extra_pages=0)
    layer = 13
    kc_h = [host(c[0][layer:layer + 1]) for c in case.caches]
    vc_h = [host(c[1][layer:layer + 1]) for c in case.caches]
    q, k, v, o_c, o_p, paged = run_both(case, layer, 0)
    assert paged.n_ctas > 1
    assert tle.device_error() == 0
    assert np.array_equal(o_c, o_p)
    want = np.zeros((case.n, QD), np.float32)
    oracle.port().decode_batch(kc_h, vc_h, case.caps, case.pos, q, k, v, want, 0, n_threads=8)
    assert maxabs(o_p, want) <= ATOL


def test_bad_page_id_is_reported_not_dereferenced(cuda):
    """A page id outside the pool is never used as an address: the kernel
    skips that copy (and that append), records 0x105 and returns; the
    sequences with valid tables in the same launch are still exact, and the
    context runs a clean decode afterwards."""
    import torch
    import tle
    case = PagedCase([700, 300, 90], 1, 64, seed=13)
    bad = case.tables[0].clone()
    bad[3] = case.pc.n_pages          # one past the pool
    bad[-1] = -1                      # the page that receives row pos
    tables = [bad] + case.tables[1:]
    q, k, v, (dq, dk, dv) = case.inputs()
    cont = tle.DecodeBatch(case.caches, case.pos, case.shape, 0)
    paged = tle.PagedDecodeBatch(case.pc, tables, case.pos, 0)
    o_c = torch.empty((case.n, QD), device="cuda")
    o_p = torch.empty((case.n, QD), device="cuda")
    cont.run(dq, dk, dv, o_c, 0)
    paged.run(dq, dk, dv, o_p, 0)
    assert tle.device_error() == 0x105
    assert np.array_equal(host(o_c)[1:], host(o_p)[1:])
    # context still usable: a clean paged decode of the other sequences
    case2 = PagedCase([700, 300, 90], 1, 64, seed=14)
    _, _, _, a, b, _ = run_both(case2, 0, 0)
    assert tle.device_error() == 0
    assert np.array_equal(a, b)


def test_paged_kv_ready_flag_gives_identical_results(cuda):
    """Paged decode with TLE_DECODE_KV_READY (first tiles and page-table
    reads before the wait on the previous kernel) equals the strict order."""
    import torch
    import tle
    case = PagedCase([700, 3000, 90, 1, 257], 2, 64, seed=17)
    _, _, _, (dq, dk, dv) = case.inputs()
    paged = tle.PagedDecodeBatch(case.pc, case.tables, case.pos, 40)
    got = {}
    for kvr in (False, True):
        outs = [torch.empty((case.n, QD), device="cuda") for _ in range(2)]
        for layer in range(2):
            paged.run(dq, dk, dv, outs[layer], layer, kv_ready=kvr)
        got[kvr] = [host(o) for o in outs]
    assert tle.device_error() == 0
    assert np.all(np.isfinite(got[False][0]))
    assert np.array_equal(got[False][0], got[True][0]) and np.array_equal(got[False][1], got[True][1])
