"""tle_decode_batch_noalloc: the batched decode for callers that cannot call
cudaMalloc (a host framework that owns all device memory through its own
pool, or a per-token loop that must not pay cudaMalloc/cudaFree's implicit
synchronisation).  Its scratch lives in the library's fixed device array, so
the caller passes only inputs and outputs.

Checked through the C ABI against tle_decode_batch (the entry point that
takes a caller workspace) on two calls in a row, within the decode tolerance
of the other tests.  Named test_zz_* so pytest collects it last; it also
passes on its own in a fresh process.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

QD, KVD = 2048, 256
ATOL = 1e-4  # the decode parity bound used throughout tests/


def _case(seed, lengths, n_layers):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    rng = np.random.default_rng(seed)
    caches = []
    for L in lengths:
        cap = int(L) + int(rng.integers(0, 4))
        caches.append((torch.randn((n_layers, cap, KVD), generator=g, device="cuda"),
                       torch.randn((n_layers, cap, KVD), generator=g, device="cuda"), cap))
    n = len(lengths)
    q = torch.randn((n, QD), generator=g, device="cuda")
    k = torch.randn((n, KVD), generator=g, device="cuda")
    v = torch.randn((n, KVD), generator=g, device="cuda")
    return caches, [int(L) - 1 for L in lengths], q, k, v


def _clone(caches):
    return [(a.clone(), b.clone(), c) for a, b, c in caches]


def _noalloc_via_cabi(caches, pos, q, k, v, out, layer, n_layers):
    """Calls tle_decode_batch_noalloc directly through ctypes."""
    import torch
    import tle
    L = tle.lib()
    n = len(caches)
    seqs = (tle.Seq * n)()
    for i, (kc, vc, cap) in enumerate(caches):
        seqs[i] = tle.Seq(kc.data_ptr(), vc.data_ptr(), cap, pos[i])
    shape = tle.tinyllama_shape(n_layers)
    rc = L.tle_decode_batch_noalloc(ctypes.byref(shape), seqs, n, q.data_ptr(), k.data_ptr(),
                                    v.data_ptr(), out.data_ptr(), layer, 1,
                                    torch.cuda.current_stream().cuda_stream)
    assert rc == tle.TLE_OK, L.tle_last_error().decode()


def test_noalloc_matches_workspace_entry_point_twice(cuda):
    import torch
    import tle
    # call 1: ragged batch split over many CTAs; call 2: a different batch,
    # layer and size, so stale scratch from call 1 would show up
    for seed, lengths, n_layers, layer in ((71, [5, 3000, 33, 1, 700, 129], 2, 1),
                                           (72, list(np.random.default_rng(9).integers(1, 2500, 40)),
                                            3, 2)):
        caches, pos, q, k, v = _case(seed, lengths, n_layers)
        n = len(lengths)
        want = torch.full((n, QD), float("nan"), device="cuda")
        batch = tle.DecodeBatch(_clone(caches), pos, tle.tinyllama_shape(n_layers))
        batch.run(q, k, v, want, layer, rotate=True)
        got = torch.full((n, QD), float("nan"), device="cuda")
        mine = _clone(caches)
        _noalloc_via_cabi(mine, pos, q, k, v, got, layer, n_layers)
        torch.cuda.synchronize()
        err = float((got - want).abs().max())
        assert err <= ATOL, (seed, err)
        # the appended rows are the same as the workspace path's
        for (kc, vc, _), (kw, vw, _), p in zip(mine, batch.caches, pos):
            assert torch.equal(kc[layer, p], kw[layer, p]) and torch.equal(vc[layer, p], vw[layer, p])
    assert tle.device_error() == 0


def test_noalloc_rejects_too_many_sequences(cuda):
    import torch
    import tle
    n = tle.NOALLOC_MAX_SEQS + 1
    kc = torch.zeros((1, 4, KVD), device="cuda")
    seqs = (tle.Seq * n)()
    for i in range(n):
        seqs[i] = tle.Seq(kc.data_ptr(), kc.data_ptr(), 4, 0)
    buf = torch.zeros((n, QD), device="cuda")
    rc = tle.lib().tle_decode_batch_noalloc(ctypes.byref(tle.tinyllama_shape(1)), seqs, n,
                                            buf.data_ptr(), buf.data_ptr(), buf.data_ptr(),
                                            buf.data_ptr(), 0, 1, 0)
    assert rc == tle.TLE_ERR_INVALID
    assert "exceeds" in tle.lib().tle_last_error().decode()
