"""CPU tests of the C ABI: the library loads, exports every symbol the header
declares, and its host-side logic (argument checks, the decode work plan,
the multi-GPU partition) behaves as documented.  No kernel is launched."""
import ctypes
import os
import re

import numpy as np
import pytest

import tle

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    text = "".join(open(os.path.join(ROOT, "include", h)).read()
                   for h in ("tle_attn.h", "tle_forward.h"))
    return sorted(set(re.findall(r"\b(tle_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_header_symbol():
    L = tle.lib()
    declared = header_functions()
    assert set(declared) == set(tle.EXPORTED), declared
    for name in declared:
        assert hasattr(L, name), name
    assert "sm_100a" in tle.version()


def test_header_compiles_as_c():
    # the boundary is plain C: the header must compile with a C compiler
    import subprocess
    import tempfile
    with tempfile.TemporaryDirectory() as d:
        src = os.path.join(d, "t.c")
        with open(src, "w") as f:
            f.write('#include "tle_attn.h"\n#include "tle_forward.h"\n'
                    'int main(void){tle_shape_t s; tle_model_t m; (void)s; (void)m; return 0;}\n')
        r = subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
                            src, "-c", "-o", os.path.join(d, "t.o")], capture_output=True, text=True)
        assert r.returncode == 0, r.stderr


def parse_desc(buf, n_seqs, n_ctas):
    b = bytes(buf)
    magic, ns, nc, _ = np.frombuffer(b[:16], np.int32)
    total = int(np.frombuffer(b[16:24], np.int64)[0])
    off = 32 + 24 * n_seqs
    cs = np.frombuffer(b[off:off + 8 * (n_ctas + 1)], np.int32).reshape(-1, 2)
    off2 = off + 8 * (n_ctas + 1)
    sc = np.frombuffer(b[off2:off2 + 8 * n_seqs], np.int32).reshape(-1, 2)
    return magic, ns, nc, total, cs, sc


def build_desc(positions, n_ctx, max_ctas):
    n = len(positions)
    shape = tle.tinyllama_shape()
    seqs = (tle.Seq * n)()
    for i, p in enumerate(positions):
        seqs[i] = tle.Seq(0x1000 * (i + 1), 0x100000 * (i + 1), n_ctx[i], p)
    nbytes = tle.lib().tle_decode_desc_bytes(n, max_ctas)
    buf = (ctypes.c_uint8 * nbytes)()
    n_ctas = ctypes.c_int(0)
    rc = tle.lib().tle_decode_desc(ctypes.byref(shape), seqs, n, max_ctas, buf, nbytes,
                                   ctypes.byref(n_ctas))
    return rc, buf, n_ctas.value


SEG_COST = 128  # rows of streaming time charged per sequence segment by the planner
START_ALIGN = 32  # CTA starts inside a sequence fall on the decode kernel's pipeline tile


@pytest.mark.parametrize("seed", [0, 1, 2, 3, 4, 5, 6, 7])
def test_decode_plan_covers_every_row_once(seed):
    rng = np.random.default_rng(seed)
    n = int(rng.integers(1, 70))
    n_ctx = rng.integers(1, 3000, n).astype(int)
    if seed == 3:
        n_ctx[:] = rng.integers(1, 6, n)  # many tiny sequences
    pos = [int(rng.integers(0, c)) for c in n_ctx]
    max_ctas = int(rng.integers(1, 300))
    rc, buf, G = build_desc(pos, list(n_ctx), max_ctas)
    assert rc == 0, tle.lib().tle_last_error()
    magic, ns, nc, total, cs, sc = parse_desc(buf, n, G)
    L = np.array(pos) + 1
    assert ns == n and nc == G and total == int(L.sum())
    assert 1 <= G <= max_ctas and G <= max(1, -(-total // 128))   # at least 128 rows per CTA
    prefix = np.concatenate([[0], np.cumsum(L)])
    row = lambda c: prefix[cs[c, 0]] + cs[c, 1] if cs[c, 0] < n else total
    # CTA ranges are contiguous and monotone, and cover every row exactly once
    assert row(0) == 0 and row(G) == total
    covered = np.zeros(total, np.int32)
    owner = np.full(total, -1)
    cost = np.zeros(G)
    for c in range(G):
        a, b = row(c), row(c + 1)
        assert b >= a
        assert cs[c, 0] == n or cs[c, 1] < L[cs[c, 0]]
        assert cs[c, 1] % START_ALIGN == 0
        covered[a:b] += 1
        owner[a:b] = c
        if b > a:
            segs = len(set(np.searchsorted(prefix, np.arange(a, b), side="right") - 1))
            cost[c] = (b - a) + SEG_COST * segs
    assert np.all(covered == 1)
    # per-sequence CTA range = first and last owner of its rows, all in between own rows of it
    for s in range(n):
        lo, hi = sc[s]
        own = owner[prefix[s]:prefix[s + 1]]
        assert lo == own.min() and hi == own.max()
        assert set(range(lo, hi + 1)) == set(own.tolist())
    # cost balance: no CTA above the even share by more than two segment
    # overheads and the rounding of its two ends to the tile
    share = (total + SEG_COST * n) / G
    assert cost.max() <= share + 2 * SEG_COST + 2 * (START_ALIGN - 1) + 1


def test_decode_plan_rejects_bad_sequences():
    rc, _, _ = build_desc([5], [5], 8)  # pos == n_ctx
    assert rc == tle.TLE_ERR_INVALID
    assert "pos" in tle.lib().tle_last_error().decode()
    rc, _, _ = build_desc([-1], [5], 8)
    assert rc == tle.TLE_ERR_INVALID


def test_unsupported_shape_is_rejected_without_gpu():
    shape = tle.Shape(22, 16, 4, 64, 10000.0)
    seqs = (tle.Seq * 1)(tle.Seq(0x1000, 0x2000, 8, 3))
    buf = (ctypes.c_uint8 * 4096)()
    n = ctypes.c_int(0)
    rc = tle.lib().tle_decode_desc(ctypes.byref(shape), seqs, 1, 4, buf, 4096, ctypes.byref(n))
    assert rc == tle.TLE_ERR_UNSUPPORTED


def test_partition_lpt_balances_and_is_deterministic():
    rng = np.random.default_rng(3)
    lengths = rng.integers(128, 2049, 64)
    for ranks in (1, 2, 4, 8):
        r = tle.partition_lpt(lengths, ranks)
        assert r == tle.partition_lpt(lengths, ranks)
        loads = np.bincount(r, weights=lengths, minlength=ranks)
        assert len(loads) == ranks
        # LPT bound: max load <= mean + max item
        assert loads.max() <= loads.sum() / ranks + lengths.max()
    # equal lengths: round robin in sequence order
    assert tle.partition_lpt([7] * 8, 4) == [0, 1, 2, 3, 0, 1, 2, 3]


# ------------------------------------------------------- paged descriptor
def build_desc_paged(positions, n_pages, page_rows, max_ctas, pool_pages=1 << 20,
                     table_ptr=lambda i: 0x4000 * (i + 1)):
    n = len(positions)
    shape = tle.tinyllama_shape()
    pool = tle.PagePool(0x10000000, 0x20000000, pool_pages, page_rows)
    seqs = (tle.PagedSeq * n)()
    for i, p in enumerate(positions):
        seqs[i] = tle.PagedSeq(table_ptr(i), n_pages[i], p)
    nbytes = tle.lib().tle_decode_desc_bytes(n, max_ctas)
    buf = (ctypes.c_uint8 * nbytes)()
    n_ctas = ctypes.c_int(0)
    rc = tle.lib().tle_decode_desc_paged(ctypes.byref(shape), ctypes.byref(pool), seqs, n,
                                         max_ctas, buf, nbytes, ctypes.byref(n_ctas))
    return rc, buf, n_ctas.value


@pytest.mark.parametrize("seed", [0, 1])
def test_paged_plan_equals_contiguous_plan(seed):
    """The paged descriptor splits rows over CTAs exactly like the contiguous
    one for the same positions (so the two give bit-identical outputs); its
    sequence slots carry {page table, 0, n_pages, pos}."""
    rng = np.random.default_rng(seed)
    n = int(rng.integers(1, 60))
    page_rows = 64
    pos = [int(x) for x in rng.integers(0, 5000, n)]
    n_pages = [p // page_rows + 1 + int(rng.integers(0, 3)) for p in pos]
    max_ctas = int(rng.integers(1, 300))
    rc, buf, G = build_desc_paged(pos, n_pages, page_rows, max_ctas)
    assert rc == 0, tle.lib().tle_last_error()
    rc2, buf2, G2 = build_desc(pos, [p + 1 for p in pos], max_ctas)
    assert rc2 == 0 and G2 == G
    m1, ns, nc, total, cs, sc = parse_desc(buf, n, G)
    m2, _, _, total2, cs2, sc2 = parse_desc(buf2, n, G)
    assert m1 == 0x544C4550 and m2 == 0x544C4544
    assert total == total2 and np.array_equal(cs, cs2) and np.array_equal(sc, sc2)
    slots = np.frombuffer(bytes(buf)[32:32 + 24 * n], np.uint8).reshape(n, 24)
    for i in range(n):
        ptrs = np.frombuffer(slots[i, :16].tobytes(), np.uint64)
        ints = np.frombuffer(slots[i, 16:].tobytes(), np.int32)
        assert ptrs[0] == 0x4000 * (i + 1) and ptrs[1] == 0
        assert ints[0] == n_pages[i] and ints[1] == pos[i]


@pytest.mark.parametrize("page_rows,n_pages,pos,table,what", [
    (48, [4], [10], None, "power of two"),
    (8, [4], [10], None, "power of two"),
    (32, [1], [32], None, "n_pages"),        # row 32 needs a second page
    (32, [2], [-1], None, "pos"),
    (32, [2], [5], lambda i: 0, "page table"),
    (32, [2], [5], lambda i: 0x4002, "aligned"),
])
def test_paged_desc_rejects_bad_arguments(page_rows, n_pages, pos, table, what):
    kw = {} if table is None else {"table_ptr": table}
    rc, _, _ = build_desc_paged(pos, n_pages, page_rows, 8, **kw)
    assert rc == tle.TLE_ERR_INVALID
    assert what in tle.lib().tle_last_error().decode()


def test_paged_desc_rejects_empty_pool():
    rc, _, _ = build_desc_paged([3], [1], 32, 8, pool_pages=0)
    assert rc == tle.TLE_ERR_INVALID


def test_decode_batch_rejects_unknown_flags():
    # checked before any device work: fake (aligned, never dereferenced) pointers
    shape = tle.tinyllama_shape()
    p = 0x100000
    rc = tle.lib().tle_decode_batch(ctypes.byref(shape), p, 1, 1, p, p, p, p, 0, 4, p, 1 << 20, None)
    assert rc == tle.TLE_ERR_INVALID
    assert "flags" in tle.lib().tle_last_error().decode()


# ------------------------------------------------- forward-pass arguments
def test_matmul_rejects_bad_arguments_without_gpu():
    """Checked before any device work (fake, never dereferenced pointers)."""
    L = tle.lib()
    p = 0x200000
    assert L.tle_matmul(p, p, p, 0, 64, tle_w("Q4_0"), None) == tle.TLE_ERR_INVALID       # rows 0
    assert L.tle_matmul(p, p, p, 8, 33, tle_w("Q4_0"), None) == tle.TLE_ERR_UNSUPPORTED   # cols % 32
    assert L.tle_matmul(p, p, p, 8, 300, tle_w("Q6_K"), None) == tle.TLE_ERR_UNSUPPORTED  # cols % 256
    assert L.tle_matmul(p, p, p, 8, 64, 3, None) == tle.TLE_ERR_UNSUPPORTED               # Q4_1
    assert L.tle_matmul(p, p + 2, p, 8, 64, tle_w("Q4_0"), None) == tle.TLE_ERR_INVALID   # unaligned W
    assert L.tle_matmul(p, p, p, 8, 16385, tle_w("F32"), None) == tle.TLE_ERR_UNSUPPORTED # too wide
    assert "cols" in L.tle_last_error().decode()


def tle_w(name):
    return {"F32": 0, "F16": 1, "Q4_0": 2, "Q8_0": 8, "Q6_K": 14}[name]


def fake_model(**kw):
    layers = (tle.Layer * 2)()
    p = 0x400000
    for i in range(2):
        for f in ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"):
            setattr(layers[i], f, tle.Weight(2, 0, p))
        layers[i].attn_norm = p
        layers[i].ffn_norm = p
    args = dict(n_layers=2, n_embd=2048, n_head=32, n_head_kv=4, n_ff=5632, n_vocab=32000,
                n_ctx=64, rope_freq_base=10000.0, rms_norm_eps=1e-5, reserved=0,
                token_embd=tle.Weight(1, 0, p), output=tle.Weight(2, 0, p), output_norm=p,
                layers=layers)
    args.update(kw)
    return tle.Model(**args), layers


def test_forward_rejects_bad_models_without_gpu():
    L = tle.lib()
    p = 0x400000
    st = tle.State(*([p] * 12), workspace_bytes=1 << 20)
    m, keep = fake_model(n_head=16)                       # attention kernels need 32 heads
    assert L.tle_forward(ctypes.byref(m), ctypes.byref(st), p, 0, None) == tle.TLE_ERR_UNSUPPORTED
    m, keep = fake_model()
    assert L.tle_forward(ctypes.byref(m), ctypes.byref(st), p, 64, None) == tle.TLE_ERR_INVALID  # pos
    m, keep = fake_model(token_embd=tle.Weight(2, 0, p))  # Q4_0 embedding table
    assert L.tle_forward(ctypes.byref(m), ctypes.byref(st), p, 0, None) == tle.TLE_ERR_UNSUPPORTED
    m, keep = fake_model()
    assert L.tle_forward(None, ctypes.byref(st), p, 0, None) == tle.TLE_ERR_INVALID
    assert L.tle_forward(ctypes.byref(m), ctypes.byref(st), None, 0, None) == tle.TLE_ERR_INVALID
    assert L.tle_forward_workspace_bytes(ctypes.byref(m)) > 0


def test_prompt_sizes_and_argument_checks_without_gpu():
    """Batched prompt: the fp16 weight copy and scratch sizes follow the
    documented layouts, and bad arguments are refused before any device
    work (fake, never dereferenced pointers)."""
    L = tle.lib()
    p = 0x400000
    m, keep = fake_model(n_ctx=512)
    e, kv, ff = 2048, 256, 5632
    layer_halves = (e + 2 * kv) * e + e * e + 2 * ff * e + e * ff
    assert L.tle_prompt_weights_bytes(ctypes.byref(m)) == 2 * 2 * layer_halves

    def a(n):
        return (n + 1023) // 1024 * 1024
    for S, pos0 in ((1, 0), (200, 0), (128, 300)):
        sp = (S + 127) // 128 * 128
        attn_ws = L.tle_prefill_workspace_bytes(ctypes.byref(tle.tinyllama_shape(2)), S, pos0)
        want = (2 * a(S * e * 4) + 2 * a(S * kv * 4) + a(S * e * 4) + 2 * a(sp * e * 2) + a(sp * ff * 2)
                + a(attn_ws))
        assert L.tle_prompt_scratch_bytes(ctypes.byref(m), S, pos0) == want, (S, pos0)

    bad, keep2 = fake_model(n_ff=5600)                     # not a multiple of the 128-row tile
    assert L.tle_prompt_weights_bytes(ctypes.byref(bad)) == 0
    assert "n_ff" in L.tle_last_error().decode()
    bad, keep2 = fake_model(n_head=16)
    assert L.tle_prompt_scratch_bytes(ctypes.byref(bad), 8, 0) == 0

    st = tle.State(*([p] * 12), workspace_bytes=0)
    big = 1 << 40
    fwd = L.tle_prompt_forward
    assert fwd(ctypes.byref(m), p, ctypes.byref(st), p, 0, 0, p, big, None) == tle.TLE_ERR_INVALID
    assert fwd(ctypes.byref(m), p, ctypes.byref(st), p, 500, 13, p, big, None) == tle.TLE_ERR_INVALID
    assert fwd(ctypes.byref(m), p, ctypes.byref(st), p, 8, 0, p + 512, big, None) == tle.TLE_ERR_INVALID
    assert fwd(ctypes.byref(m), p, ctypes.byref(st), p, 8, 0, p, 1024, None) == tle.TLE_ERR_WORKSPACE
    assert fwd(ctypes.byref(m), None, ctypes.byref(st), p, 8, 0, p, big, None) == tle.TLE_ERR_INVALID
    q4_table, keep3 = fake_model(n_ctx=512, token_embd=tle.Weight(2, 0, p))
    assert fwd(ctypes.byref(q4_table), p, ctypes.byref(st), p, 8, 0, p, big, None) == tle.TLE_ERR_UNSUPPORTED
    assert L.tle_prompt_pack_weights(ctypes.byref(m), None, big, None) == tle.TLE_ERR_INVALID
    assert L.tle_prompt_pack_weights(ctypes.byref(m), p, 1024, None) == tle.TLE_ERR_WORKSPACE


def test_sampling_rejects_bad_arguments_without_gpu():
    """Checked before any device work (fake, never dereferenced pointers)."""
    L = tle.lib()
    p = 0x200000
    assert L.tle_sample_temperature(p, 0, 1.0, 0.5, p, None) == tle.TLE_ERR_UNSUPPORTED     # empty row
    assert L.tle_sample_temperature(p, 50000, 1.0, 0.5, p, None) == tle.TLE_ERR_UNSUPPORTED  # > 40960
    assert L.tle_sample_top_p(p, 32000, 1.0, 0.9, 1.0, p, None) == tle.TLE_ERR_INVALID      # r == 1
    assert L.tle_sample_top_p(p, 32000, 1.0, 0.9, -0.1, p, None) == tle.TLE_ERR_INVALID
    assert L.tle_sample_temperature(p, 32000, 1.0, float("nan"), p, None) == tle.TLE_ERR_INVALID
    assert "r must be" in L.tle_last_error().decode()
    assert L.tle_sample_top_p(None, 32000, 1.0, 0.9, 0.5, p, None) == tle.TLE_ERR_INVALID


def test_paged_cache_allocator_host_logic():
    """PagedKVCache's free list (host side; built on the CPU here): pages
    come out in pool order, exhaustion raises, freed pages are reused, and
    page counts round up."""
    import torch
    pc = tle.PagedKVCache(6, 32, tle.tinyllama_shape(1), device="cpu")
    assert pc.key_pool.shape == (1, 6, 32, 256)
    assert pc.pages_for(1) == 1 and pc.pages_for(32) == 1 and pc.pages_for(33) == 2
    a = pc.alloc(4)
    assert a == [0, 1, 2, 3]
    with pytest.raises(MemoryError):
        pc.alloc(3)
    pc.free(a[:2])
    b = pc.alloc(4)
    assert sorted(b) == [0, 1, 4, 5]
    t = pc.table(b)
    assert t.dtype == torch.int32 and t.tolist() == b
    pool = pc.pool()
    assert pool.n_pages == 6 and pool.page_rows == 32
