// decode.cu -- fused RoPE + KV append + split-K flash-decoding for TinyLlama
// GQA (32 query heads, 4 KV heads, head_dim 64, fp32 cache).
//
// Reference semantics: rope() src/ops.cpp:1223-1281 followed by attention()
// src/ops.cpp:1317-1515, per sequence:
//   append k,v at row pos (ops.cpp:1370-1371); for each query head qh with KV
//   head qh/8 (ops.cpp:1383): s_p = (q.K_p)/sqrt(64) for p <= pos
//   (ops.cpp:1425-1433), softmax (ops.cpp:1445), out = sum_p w_p V_p
//   (ops.cpp:1494-1508).
//
// Design (B200): the rows of all sequences in a batch are concatenated and
// split over the CTAs (one per SM), balanced in rows plus a fixed cost per
// segment.  A CTA walks its row range as segments of one sequence each.
// Warp 0 lane 0 streams 32-row K and V tiles
// (1 KB per row: all 4 KV heads) into a 3-stage shared-memory ring with 1-D
// bulk copies (refilling a stage once all warps released it), and prefetches
// each segment's q and new k/v rows one segment ahead.
// The 8 warps each own 4 rows of every tile and all 32 query heads (lane =
// head), so every K/V element read from HBM serves its 8 query heads.
// Scores, an online softmax and the PV accumulation run in fp32 (TF32 tensor
// cores would miss the 1e-4 parity bound), as packed f32x2 FMAs: the same
// FLOPs in half the instructions, which keeps the SM below its power cap
// (4-5 % more HBM throughput than scalar FFMA).  Each lane reads its KV
// head's 16-byte chunks in an order rotated by the KV-head index, so the four
// distinct addresses of a warp-wide load fall in four different bank groups
// (conflict-free broadcast).  At the end of a segment the warps merge in a
// 3-level tree (8 -> 4 through tensor memory, which the kernel otherwise
// does not use, 4 -> 2 -> 1 through shared memory); warp 0 writes the output
// of a segment that is a whole sequence, otherwise its (m, l, o) partial goes
// to the workspace and the last CTA to finish a partial of that sequence
// combines them (batch mode; merge_kernel does it for the single-sequence
// entry points).
#include <math.h>

#include <cooperative_groups.h>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace cg = cooperative_groups;

namespace tle {

namespace {

__device__ uint32_t g_tle_error = 0;


constexpr int HD = kHeadDim;
constexpr int NH = kNHead;
constexpr int NKV_HEADS = kNHeadKv;
constexpr int ROWF = kRowFloats;   // 256 floats per cache row
constexpr int ROWB = ROWF * 4;     // 1024 bytes
constexpr int TILE = 32;           // rows per pipeline stage
constexpr int NSTAGE = 3;
constexpr int NCW = 8;             // warps (all consume; warp 0 lane 0 also issues the copies)
constexpr int NCT = NCW * 32;      // threads per CTA
constexpr int RPW = TILE / NCW;    // rows per warp per tile (4)
constexpr int QS = HD + 4;         // padded row of the q / tree buffers: 64 floats, m, l, pad
constexpr uint32_t kTmemCols = 128;  // tree-merge exchange: acc[64], m, l per lane
constexpr float kScale = 0.125f;   // 1/sqrt(64), exact in fp32

struct __align__(128) DecodeSmem {
    float k[NSTAGE][TILE * ROWF];
    float v[NSTAGE][TILE * ROWF];
    // q of a segment's sequence (one 8 KB bulk copy), double-buffered by
    // segment; after the prologue it is the tree merge's buffer A (chunk c of
    // row h stored at chunk (c + h) & 15: conflict-free), m and l in mlA.
    float qraw[2][NH * HD];
    float kvraw[2 * ROWF];      // that sequence's new k row and v row (segments holding row pos)
    float newk[ROWF];           // rotated k of the token being decoded
    float newv[ROWF];
    // Rotated, scaled q of the current segment in padded rows (stride 68:
    // the rotated-order reads are conflict-free); once the q registers are
    // loaded it is the tree merge's buffer B (m, l in the row padding).
    float qo[NH * QS];
    float mlA[2 * NH];
    int32_t apage[2];           // paged mode: page id of row pos of the segment's sequence
    int32_t npage[2];           // paged mode: the issuer's prefetched next page ids (ring)
    const int32_t* cur_pages;   // paged mode: page table of the issuer's current sequence
    uint32_t tmem_base;
    uint64_t full[NSTAGE];
    uint64_t empty[NSTAGE];
    uint64_t qfull[2];
    uint64_t csync;             // all-warp barrier (bounded waits)
    int merge_last;             // wide merge: this CTA arrived last for the segment's sequence
};

// CTA c's row range as (start seq, start off) .. (end seq, end off), exclusive end.
__device__ __forceinline__ void cta_range(const DecodeArgs& A, int c, int& s0, int& o0, int& s1,
                                          int& o1) {
    if (A.seqs) {
        const CtaStart b = A.cta_start[c], e = A.cta_start[c + 1];
        s0 = b.seq; o0 = b.off; s1 = e.seq; o1 = e.off;
    } else {
        // boundaries rounded down to the pipeline tile (the planner gives
        // each CTA >= 128 rows, so no range becomes empty)
        const int L = A.single.pos + 1;
        s0 = 0;
        o0 = static_cast<int>(static_cast<int64_t>(c) * L / A.n_ctas) / TILE * TILE;
        const int e = c + 1 == A.n_ctas ? L : static_cast<int>(static_cast<int64_t>(c + 1) * L / A.n_ctas) / TILE * TILE;
        if (e >= L) { s1 = 1; o1 = 0; } else { s1 = 0; o1 = e; }
    }
}

__device__ __forceinline__ tle_seq_t load_seq(const DecodeArgs& A, int s) {
    return A.seqs ? A.seqs[s] : A.single;
}

__device__ __forceinline__ bool in_range(int s, int off, int s1, int o1) {
    return s < s1 || (s == s1 && off < o1);
}

// The copy issuer's position in the CTA's sequence of tiles (it runs up to
// NSTAGE tiles ahead of the consumers).  kb/vb: K and V bases such that row
// r of the sequence is at kb + 256 r (paged mode: valid while r is in page
// cpi).  Paged mode keeps the index of the page being read (cpi) and
// prefetches the id of the page after it when the
// cursor enters a page: a 4-byte cp.async into npage[slot], so the table
// read is in flight for a page's worth of tiles and no register waits on it
// (the issuer is also a consumer thread: a load it waits on stalls its warp
// and, through the stage barriers, the CTA).  pst bit 0: a prefetch of page
// cpi + 1 is pending; bit 1: its slot.  The page-table pointer itself sits
// in shared memory (read at page switches only): every register the cursor
// holds is live through the consumer loop of a kernel at the register limit.
struct TileCursor {
    int s, ta, b;
    bool done;
    const float* kb;
    const float* vb;
    int pos;
    int cpi, pst;
};

// Paged mode: a sequence record's key_cache slot holds its page table (the
// host builds the descriptor that way, see tle_decode_desc_paged).
__device__ __forceinline__ const int32_t* seq_pages(const tle_seq_t& sq) {
    return reinterpret_cast<const int32_t*>(sq.key_cache);
}

// Offset (floats) of row r of page `id` of the current layer in a pool
// [n_layers][pool_pages][1 << page_shift][256].
__device__ __forceinline__ size_t pool_row(const DecodeArgs& A, int id, int r) {
    return ((static_cast<size_t>(A.layer) * A.pool_pages + id) << A.page_shift |
            static_cast<size_t>(r & ((1 << A.page_shift) - 1))) * ROWF;
}

// Checked page id: -1 (and the error word set) for an id outside the pool.
__device__ __forceinline__ int check_page(const DecodeArgs& A, int id) {
    if (static_cast<unsigned>(id) >= static_cast<unsigned>(A.pool_pages)) {
        record_error(A.err, kErrBadPage);
        return -1;
    }
    return id;
}

// Page id of page pi of the cursor's sequence; advances the one-page-ahead
// prefetch.  Rows below min(b, pos) are the only ones read, so the prefetch
// never reads past the entries the host checked (n_pages * page_rows > pos).
__device__ __forceinline__ int cursor_page(TileCursor& c, const DecodeArgs& A, DecodeSmem& S, int pi) {
    if (pi == c.cpi) return 0;
    const int32_t* pages = S.cur_pages;
    int id;
    if ((c.pst & 1) && pi == c.cpi + 1) {
        cp_async_wait_all();
        id = S.npage[c.pst >> 1];
        c.pst ^= 2;           // the next prefetch goes to the other slot
    } else {
        if (c.pst & 1) cp_async_wait_all();   // an unused prefetch must land before its slot is reused
        id = ld_cg_s32(pages + pi);
    }
    c.pst &= ~1;
    id = check_page(A, id);
    // A bad page is never made current, so no tile takes the fast path on it.
    c.cpi = id >= 0 ? pi : INT_MIN;
    if (id >= 0) {
        // bases such that kb + r * 256 is row r of the sequence while r is
        // in page pi (the offset of page pi's row 0 minus pi's first row)
        const size_t o = pool_row(A, id, 0) - (static_cast<size_t>(pi) << A.page_shift) * ROWF;
        c.kb = A.key_pool + o;
        c.vb = A.value_pool + o;
    }
    if (((pi + 1) << A.page_shift) < min(c.b, c.pos)) {
        cp_async_4(&S.npage[c.pst >> 1], pages + pi + 1);
        c.pst |= 1;
    }
    return id;
}

// Paged mode: starts the page-table read of the cursor's first page.
// (The first page is announced as "the page after cpi"; tiles only move
// forward from ta, so page cpi itself is never asked for.)
__device__ __forceinline__ void cursor_prefetch(TileCursor& c, const DecodeArgs& A, DecodeSmem& S) {
    if (!c.done && c.ta < min(c.b, c.pos)) {
        const int first = c.ta >> A.page_shift;
        c.cpi = first - 1;
        cp_async_4(&S.npage[c.pst >> 1], S.cur_pages + first);
        c.pst |= 1;
    }
}

// Moves the cursor to row `off` of sequence s (done once past the CTA's
// range).  Paged mode also starts the read of the first page's id unless
// `table` is false (the kernel's first call, made before the wait on the
// previous grid: page tables may be that grid's output).
template <bool PAGED>
__device__ __forceinline__ void cursor_load(TileCursor& c, const DecodeArgs& A, DecodeSmem& S, int s,
                                            int off, int s1, int o1, bool table = true) {
    c.s = s;
    c.ta = off;
    c.done = !in_range(s, off, s1, o1);
    if (!c.done) {
        const tle_seq_t sq = load_seq(A, s);
        c.b = (s == s1) ? o1 : sq.pos + 1;
        c.pos = sq.pos;
        if (PAGED) {
            S.cur_pages = seq_pages(sq);
            c.cpi = INT_MIN;   // no page yet (pages are >= 0, so cpi + 1 matches none)
            c.pst &= ~1;
            if (table) cursor_prefetch(c, A, S);
        } else {
            const size_t base = (static_cast<size_t>(A.layer) * sq.n_ctx) * ROWF;
            c.kb = sq.key_cache + base;
            c.vb = sq.value_cache + base;
        }
    }
}

// Issues the cursor's tile into stage st (1-D bulk copies of whole 1 KB rows)
// and advances the cursor.  Row `pos` (the token being decoded) is never read
// from the cache: the consumers take it from newk/newv.  Paged mode copies
// the tile as one piece per page it touches (a row of the stage is the same
// row whichever layout it came from).
template <bool PAGED>
__device__ __forceinline__ void cursor_issue(TileCursor& c, const DecodeArgs& A, DecodeSmem& S,
                                             int st, int s1, int o1, uint64_t pol) {
    const int tb = min(c.ta + TILE, c.b);
    const int te = min(tb, c.pos);
    const int n = te - c.ta;
    if (n > 0) {
        const uint32_t bytes = static_cast<uint32_t>(n) * ROWB;
        mbar_arrive_expect_tx(&S.full[st], 2 * bytes);
        // Paged mode: a tile inside the current (valid) page is issued like a
        // contiguous one, from the page-relative bases kb/vb; a tile that
        // enters a new page goes piece by piece (one per page it touches).
        const bool whole_page = !PAGED || ((c.ta >> A.page_shift) == c.cpi &&
                                           ((te - 1) >> A.page_shift) == c.cpi);
        if (!whole_page) {
            for (int r = c.ta; r < te;) {
                const int pi = r >> A.page_shift;
                const int e = min(te, (pi + 1) << A.page_shift);
                const uint32_t pb = static_cast<uint32_t>(e - r) * ROWB;
                if (cursor_page(c, A, S, pi) >= 0) {
                    bulk_g2s(S.k[st] + (r - c.ta) * ROWF, c.kb + static_cast<size_t>(r) * ROWF, pb,
                             &S.full[st], pol);
                    bulk_g2s(S.v[st] + (r - c.ta) * ROWF, c.vb + static_cast<size_t>(r) * ROWF, pb,
                             &S.full[st], pol);
                } else {
                    // bad page id (reported): the stage completes without
                    // this piece, its rows keep stale contents
                    mbar_tx_complete(&S.full[st], 2 * pb);
                }
                r = e;
            }
        } else {
            bulk_g2s(S.k[st], c.kb + static_cast<size_t>(c.ta) * ROWF, bytes, &S.full[st], pol);
            bulk_g2s(S.v[st], c.vb + static_cast<size_t>(c.ta) * ROWF, bytes, &S.full[st], pol);
        }
    } else {
        mbar_arrive(&S.full[st]);
    }
    c.ta = tb;
    if (c.ta >= c.b) cursor_load<PAGED>(c, A, S, c.s + 1, 0, s1, o1);
}

// Bulk copies of segment n's per-sequence inputs into buffer n & 1, issued by
// warp 0: q of its sequence and, when the segment holds row pos, the new k and
// v rows (paged mode: also the page id of row pos, by a 4-byte cp.async that
// the same barrier waits for, so no thread stalls on the page-table read).
// Segment n of a CTA is sequence s0 + n.  Returns false (nothing issued) when
// the CTA has no segment n; warp-uniform.
template <bool PAGED>
__device__ __forceinline__ bool issue_q(const DecodeArgs& A, DecodeSmem& S, int n, int s0, int o0,
                                        int s1, int o1, int lane) {
    const int s = s0 + n;
    if (!in_range(s, n == 0 ? o0 : 0, s1, o1)) return false;
    const tle_seq_t sq = load_seq(A, s);
    const int L = sq.pos + 1;
    const bool has_new = ((s == s1) ? o1 : L) == L;
    const int b = n & 1;
    if (lane == 0) {
        if (PAGED && has_new) {
            cp_async_4(&S.apage[b], seq_pages(sq) + (sq.pos >> A.page_shift));
            cp_async_mbar_arrive(&S.qfull[b]);
        }
        mbar_arrive_expect_tx(&S.qfull[b], NH * HD * 4 + (has_new ? 2 * ROWB : 0));
        bulk_g2s_plain(S.qraw[b], A.q + static_cast<size_t>(s) * NH * HD, NH * HD * 4, &S.qfull[b]);
        if (has_new) {
            bulk_g2s_plain(S.kvraw, A.k + static_cast<size_t>(s) * ROWF, ROWB, &S.qfull[b]);
            bulk_g2s_plain(S.kvraw + ROWF, A.v + static_cast<size_t>(s) * ROWF, ROWB, &S.qfull[b]);
        }
    }
    __syncwarp();
    return true;
}

// Folds (m2, l2, a2) of the same query head into (m, l, acc[c0 .. c0+7]) /
// computes the factors; split so TMEM can be read 32 columns at a time.
struct FoldFactors {
    float f1, f2;
};
__device__ __forceinline__ FoldFactors fold_factors(float& m, float& l, float m2, float l2) {
    const float mn = fmaxf(m, m2);
    FoldFactors f;
    f.f1 = (m == -INFINITY) ? 0.f : expf(m - mn);
    f.f2 = (m2 == -INFINITY) ? 0.f : expf(m2 - mn);
    l = fmaf(l, f.f1, l2 * f.f2);
    m = mn;
    return f;
}
__device__ __forceinline__ void fold4(float4& a, float4 b, FoldFactors f) {
    a.x = fmaf(a.x, f.f1, b.x * f.f2);
    a.y = fmaf(a.y, f.f1, b.y * f.f2);
    a.z = fmaf(a.z, f.f1, b.z * f.f2);
    a.w = fmaf(a.w, f.f1, b.w * f.f2);
}

// Shared-memory tree steps: another warp's (acc, m, l) of the same query
// head, acc in the lanes' shared chunk order.  Buffer B: row h of a [32][QS]
// buffer (m, l in the padding).
__device__ __forceinline__ void merge_in(float& m, float& l, float4 (&acc)[16], const float* row) {
    const FoldFactors f = fold_factors(m, l, row[HD], row[HD + 1]);
#pragma unroll
    for (int c = 0; c < 16; ++c) fold4(acc[c], *reinterpret_cast<const float4*>(row + 4 * c), f);
}
__device__ __forceinline__ void merge_out(float m, float l, const float4 (&acc)[16], float* row) {
#pragma unroll
    for (int c = 0; c < 16; ++c) *reinterpret_cast<float4*>(row + 4 * c) = acc[c];
    row[HD] = m;
    row[HD + 1] = l;
}
// Buffer A: dense [32][64] with chunk c of row h at chunk (c + h) & 15, m and l in ml.
__device__ __forceinline__ void merge_in_a(float& m, float& l, float4 (&acc)[16], const float* O,
                                           const float* ml, int h) {
    const FoldFactors f = fold_factors(m, l, ml[h], ml[NH + h]);
#pragma unroll
    for (int c = 0; c < 16; ++c)
        fold4(acc[c], *reinterpret_cast<const float4*>(O + h * HD + 4 * ((c + h) & 15)), f);
}
__device__ __forceinline__ void merge_out_a(float m, float l, const float4 (&acc)[16], float* O, float* ml,
                                            int h) {
#pragma unroll
    for (int c = 0; c < 16; ++c) *reinterpret_cast<float4*>(O + h * HD + 4 * ((c + h) & 15)) = acc[c];
    ml[h] = m;
    ml[NH + h] = l;
}

// Tensor-memory tree step: warp w + 4 stores its (acc, m, l) in its TMEM lane
// quadrant (w & 3), warp w reads it (a warp reaches only its own quadrant).
__device__ __forceinline__ void tmem_put(uint32_t tq, float m, float l, const float4 (&acc)[16]) {
    uint32_t r[32];
#pragma unroll
    for (int half = 0; half < 2; ++half) {
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const float4 a = acc[8 * half + c];
            r[4 * c] = __float_as_uint(a.x);
            r[4 * c + 1] = __float_as_uint(a.y);
            r[4 * c + 2] = __float_as_uint(a.z);
            r[4 * c + 3] = __float_as_uint(a.w);
        }
        tmem_st32(tq + 32 * half, r);
    }
    tmem_st2(tq + 64, m, l);
    tmem_wait_st();
}
__device__ __forceinline__ void tmem_merge_in(uint32_t tq, float& m, float& l, float4 (&acc)[16]) {
    float m2, l2;
    tmem_ld2(tq + 64, m2, l2);
    tmem_wait_ld();
    const FoldFactors f = fold_factors(m, l, m2, l2);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        float v[32];
        tmem_ld32(tq + 32 * half, v);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 8; ++c)
            fold4(acc[8 * half + c], make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]), f);
    }
}

// Batch mode, warp 0 (lane = query head h), after this CTA wrote its partial
// of sequence s covered by CTAs sc.lo..sc.hi: counts the arrival and returns
// true in the CTA whose arrival completes the count (the fence + atomic "last
// block" pattern; no CTA ever waits).  That CTA resets the count for the next
// call.  The release fence orders the whole warp's partial stores (made
// visible to lane 0 by __syncwarp) before the count.
__device__ __forceinline__ bool arrive_last(const DecodeArgs& A, int s, int lane, SeqCtas sc) {
    __syncwarp();
    int last = 0;
    if (lane == 0) {
        asm volatile("fence.acq_rel.gpu;" ::: "memory");
        last = (atomicAdd(&A.arrivals[s], 1) == sc.hi - sc.lo);
        if (last) {
            A.arrivals[s] = 0;
            asm volatile("fence.acq_rel.gpu;" ::: "memory");
        }
    }
    return __shfl_sync(0xffffffffu, last, 0) != 0;
}

// Warp-wide coalesced view of a [32 heads][64] block: float4 number 32 i + lane
// holds head 2 i + (lane >> 4), chunk lane & 15.
__device__ __forceinline__ int coalesced_head(int i, int lane) { return 2 * i + (lane >> 4); }

// Loads the partial of CTA c: m, l of head `lane`, o in the coalesced view.
__device__ __forceinline__ void load_partial(const DecodeArgs& A, int s, int c, int lane,
                                             float& m, float& l, float4 (&o)[16]) {
    const float* P = A.partials + static_cast<size_t>(s + c) * kPartialFloats;
    m = ld_cg(P + NH * HD + lane);
    l = ld_cg(P + NH * HD + NH + lane);
    const float4* src = reinterpret_cast<const float4*>(P) + lane;
#pragma unroll
    for (int i = 0; i < 16; ++i) o[i] = ld_cg4(src + 32 * i);
}

// The last CTA of sequence s combines the partials of CTAs sc.lo..sc.hi (its
// own included, re-read from L2) into out[s].  The fold order is fixed, CTA
// lo first and then two partials per round, so the output does not depend on
// which CTA finished last; the loads of a round are issued together.  Every
// partial covers at least one row, so every m is finite.
__device__ __forceinline__ void merge_partials(const DecodeArgs& A, int s, int lane, SeqCtas sc) {
    float m, l;
    float4 acc[16];
    load_partial(A, s, sc.lo, lane, m, l, acc);
    for (int c = sc.lo + 1; c <= sc.hi; c += 2) {
        const bool two = c + 1 <= sc.hi;
        float m1, l1, m2 = -INFINITY, l2 = 0.f;
        float4 o1[16], o2[16];
        load_partial(A, s, c, lane, m1, l1, o1);
        if (two) {
            load_partial(A, s, c + 1, lane, m2, l2, o2);
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) o2[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        const float mn = fmaxf(m, fmaxf(m1, m2));
        const float f0 = expf(m - mn), f1 = expf(m1 - mn), f2 = two ? expf(m2 - mn) : 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int hh = coalesced_head(i, lane);
            const float a0 = __shfl_sync(0xffffffffu, f0, hh);
            const float a1 = __shfl_sync(0xffffffffu, f1, hh);
            const float a2 = __shfl_sync(0xffffffffu, f2, hh);
            acc[i].x = fmaf(acc[i].x, a0, fmaf(o1[i].x, a1, o2[i].x * a2));
            acc[i].y = fmaf(acc[i].y, a0, fmaf(o1[i].y, a1, o2[i].y * a2));
            acc[i].z = fmaf(acc[i].z, a0, fmaf(o1[i].z, a1, o2[i].z * a2));
            acc[i].w = fmaf(acc[i].w, a0, fmaf(o1[i].w, a1, o2[i].w * a2));
        }
        l = fmaf(l, f0, fmaf(l1, f1, l2 * f2));
        m = mn;
    }
    const float inv = 1.0f / l;
    float4* dst = reinterpret_cast<float4*>(A.out + static_cast<size_t>(s) * NH * HD) + lane;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const float f = __shfl_sync(0xffffffffu, inv, coalesced_head(i, lane));
        dst[32 * i] = make_float4(acc[i].x * f, acc[i].y * f, acc[i].z * f, acc[i].w * f);
    }
}

// A sequence split over at least kWideMergeParts CTAs is folded by all eight
// warps of its last CTA: warp w takes heads 4w .. 4w+3, lane = (head 4w +
// lane / 8, dimensions 8 (lane % 8) .. +7), and the partials are folded in
// CTA order, eight per round with all their loads in flight (one warp alone
// needs a round trip per two partials).  Deterministic like merge_partials;
// the fold order, and so the last bits, differ from it.
constexpr int kWideMergeParts = 4;
__device__ __forceinline__ void merge_partials_wide(const DecodeArgs& A, int s, int warp, int lane, SeqCtas sc) {
    const int hh = 4 * warp + (lane >> 3), d0 = 8 * (lane & 7);
    float m = -INFINITY, l = 0.f;
    float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0;
    for (int c0 = sc.lo; c0 <= sc.hi; c0 += 8) {
        float mc[8], lc[8];
        float4 o0[8], o1[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            mc[j] = -INFINITY;
            lc[j] = 0.f;
            o0[j] = o1[j] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (c0 + j <= sc.hi) {
                const float* P = A.partials + static_cast<size_t>(s + c0 + j) * kPartialFloats;
                mc[j] = ld_cg(P + NH * HD + hh);
                lc[j] = ld_cg(P + NH * HD + NH + hh);
                o0[j] = ld_cg4(reinterpret_cast<const float4*>(P + hh * HD + d0));
                o1[j] = ld_cg4(reinterpret_cast<const float4*>(P + hh * HD + d0 + 4));
            }
        }
        float mn = m;
#pragma unroll
        for (int j = 0; j < 8; ++j) mn = fmaxf(mn, mc[j]);
        const float fr = (m == -INFINITY) ? 0.f : expf(m - mn);
        l *= fr;
        a0 = make_float4(a0.x * fr, a0.y * fr, a0.z * fr, a0.w * fr);
        a1 = make_float4(a1.x * fr, a1.y * fr, a1.z * fr, a1.w * fr);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            if (c0 + j <= sc.hi) {   // every partial covers a row, so its m is finite
                const float f = expf(mc[j] - mn);
                l = fmaf(lc[j], f, l);
                a0 = make_float4(fmaf(o0[j].x, f, a0.x), fmaf(o0[j].y, f, a0.y), fmaf(o0[j].z, f, a0.z),
                                 fmaf(o0[j].w, f, a0.w));
                a1 = make_float4(fmaf(o1[j].x, f, a1.x), fmaf(o1[j].y, f, a1.y), fmaf(o1[j].z, f, a1.z),
                                 fmaf(o1[j].w, f, a1.w));
            }
        }
        m = mn;
    }
    const float inv = 1.0f / l;
    float4* dst = reinterpret_cast<float4*>(A.out + static_cast<size_t>(s) * NH * HD + hh * HD + d0);
    dst[0] = make_float4(a0.x * inv, a0.y * inv, a0.z * inv, a0.w * inv);
    dst[1] = make_float4(a1.x * inv, a1.y * inv, a1.z * inv, a1.w * inv);
}

// e^x on the SFU: ex2.approx.ftz(x log2 e), relative error ~2^-22 (far inside
// the 1e-4 output bound); e^-inf = 0.
__device__ __forceinline__ float exp_sfu(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x * 1.4426950408889634f));
    return y;
}

__device__ __forceinline__ uint64_t pk2(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void up2(uint64_t v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}

// All-warp barrier on an mbarrier (bounded wait; false on timeout).
__device__ __forceinline__ bool cta_sync(DecodeSmem& S, uint32_t& phase, int lane) {
    __syncwarp();
    if (lane == 0) mbar_arrive(&S.csync);
    const bool ok = __all_sync(0xffffffffu, mbar_wait(&S.csync, phase));  // warp-uniform
    phase ^= 1u;
    __syncwarp();
    return ok;
}

template <bool PAGED>
__global__ void __launch_bounds__(NCT, 1) decode_kernel(const __grid_constant__ DecodeArgs A) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    DecodeSmem& S = *reinterpret_cast<DecodeSmem*>(smem_raw);
    // The next kernel on the stream (merge_kernel in single-sequence mode,
    // the next decode launch in batch mode) is a programmatic dependent: it
    // may be scheduled now and runs its prologue while this grid finishes.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int cta = blockIdx.x;
    const bool issuer = (tid == 0);

    int s0, o0, s1, o1;
    cta_range(A, cta, s0, o0, s1, o1);

    // Prologue: thread 0 (the tile issuer) initialises the barriers and
    // reads its first sequence record while warp 1 allocates the tensor
    // memory.  Up to here only the descriptor is read, which the host wrote
    // before the launch; everything else (q/k/v, the caches, page tables,
    // outputs, partials, arrival counts) may belong to the previous kernel
    // on the stream, so it is touched only after griddepcontrol.wait --
    // except with kv_ready, where the caller guarantees that the previous
    // kernel wrote no cached row this launch reads and no page table: the
    // first NSTAGE tiles are then streamed while that kernel drains.  Then
    // warp 0 starts segment 0's q copy (and thread 0 the first tiles); the
    // other warps touch none of it before the __syncthreads below.
    TileCursor cur;
    uint64_t pol = 0;
    int issued = 0;
    int q_issued = 0;   // (warp 0) segments 0 .. q_issued-1 have their q copy issued
    if (issuer) {
        for (int i = 0; i < NSTAGE; ++i) {
            mbar_init(&S.full[i], 1);
            mbar_init(&S.empty[i], NCW);
        }
        mbar_init(&S.qfull[0], 1);
        mbar_init(&S.qfull[1], 1);
        mbar_init(&S.csync, NCW);
        fence_barrier_init();
        cur.pst = 0;
        cursor_load<PAGED>(cur, A, S, s0, o0, s1, o1, /*table=*/A.kv_ready != 0);
        pol = l2_evict_first_policy();
    }
    if (warp == 1) {
        tmem_alloc(&S.tmem_base, kTmemCols);
        tmem_relinquish();
    }
    if (!A.kv_ready) {
        asm volatile("griddepcontrol.wait;" ::: "memory");
        if (warp == 0) {
            __syncwarp();
            if (issue_q<PAGED>(A, S, 0, s0, o0, s1, o1, lane)) q_issued = 1;
        }
        if (PAGED && issuer) cursor_prefetch(cur, A, S);
    }
    if (issuer) {
        while (!cur.done && issued < NSTAGE) {
            cursor_issue<PAGED>(cur, A, S, issued, s1, o1, pol);
            ++issued;
        }
    }
    if (A.kv_ready) {
        asm volatile("griddepcontrol.wait;" ::: "memory");
        if (warp == 0) {
            __syncwarp();
            if (issue_q<PAGED>(A, S, 0, s0, o0, s1, o1, lane)) q_issued = 1;
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tq = S.tmem_base + (static_cast<uint32_t>((warp & 3) * 32) << 16);

    const int g = lane >> 3;       // KV head of this lane's query head
    const int h = lane;            // query head
    uint32_t cphase = 0;
    int it = 0;
    int n = 0;                     // segment index within this CTA
    bool ok = true;

    for (int s = s0, off = o0; ok && in_range(s, off, s1, o1); ++s, off = 0, ++n) {
        const tle_seq_t sq = load_seq(A, s);
        const int L = sq.pos + 1;
        const int seg_a = off;
        const int seg_b = (s == s1) ? o1 : L;
        const int qb = n & 1;
        if (!__all_sync(0xffffffffu, mbar_wait(&S.qfull[qb], (n >> 1) & 1))) {
            record_error(A.err, kErrWaitFull);
            ok = false;
            break;
        }

        // q: rotate (rope, ops.cpp:1229-1260), pre-scale by 1/sqrt(64) (exact
        // power of two, so (q/8).k == (q.k)/8 bit for bit).  Every pair this
        // thread rotates (j = tid + 256 i, here and for the new k row) has
        // rotation index j & 31 == lane, so one sincosf serves them all.
        float sn = 0.f, cs = 1.f;
        if (A.rotate) sincosf(static_cast<float>(sq.pos) * A.inv_freq[lane], &sn, &cs);
        {
            // Pair `lane` of heads warp + 8 i.
            const float2* Q = reinterpret_cast<const float2*>(S.qraw[qb]);
#pragma unroll
            for (int i = 0; i < NH / NCW; ++i) {
                const int hh = warp + NCW * i;
                const float2 x = Q[hh * (HD / 2) + lane];
                float y0 = x.x, y1 = x.y;
                if (A.rotate) {
                    y0 = x.x * cs - x.y * sn;
                    y1 = x.x * sn + x.y * cs;
                }
                *reinterpret_cast<float2*>(&S.qo[hh * QS + 2 * lane]) = make_float2(y0 * kScale, y1 * kScale);
            }
        }
        // The new token's k (rotated) and v: append to the cache at row pos
        // (ops.cpp:1370-1371) and keep a copy for this CTA's last tile.
        if (seg_b == L) {
            // row pos of the contiguous cache, or of the pool page holding it
            // (a bad page id is reported and the row not written)
            float* kdst = nullptr;
            float* vdst = nullptr;
            if (PAGED) {
                const int id = check_page(A, S.apage[qb]);
                if (id >= 0) {
                    const size_t row = pool_row(A, id, sq.pos);
                    kdst = A.key_pool + row;
                    vdst = A.value_pool + row;
                }
            } else {
                const size_t row = (static_cast<size_t>(A.layer) * sq.n_ctx + sq.pos) * ROWF;
                kdst = sq.key_cache + row;
                vdst = sq.value_cache + row;
            }
            if (tid < ROWF / 2) {
                const float2 x = reinterpret_cast<const float2*>(S.kvraw)[tid];
                float y0 = x.x, y1 = x.y;
                if (A.rotate) {
                    y0 = x.x * cs - x.y * sn;
                    y1 = x.x * sn + x.y * cs;
                }
                const float2 y = make_float2(y0, y1);
                reinterpret_cast<float2*>(S.newk)[tid] = y;
                if (!PAGED || kdst) reinterpret_cast<float2*>(kdst)[tid] = y;
            } else {
                const int t2 = tid - ROWF / 2;
                const float2 x = reinterpret_cast<const float2*>(S.kvraw + ROWF)[t2];
                reinterpret_cast<float2*>(S.newv)[t2] = x;
                if (!PAGED || vdst) reinterpret_cast<float2*>(vdst)[t2] = x;
            }
        }
        // Shared memory written by this thread through the generic proxy
        // (qraw, kvraw, the tree buffers) is rewritten by later bulk copies.
        fence_proxy_async_smem();
        if (!cta_sync(S, cphase, lane)) { record_error(A.err, kErrWaitFull); ok = false; break; }
        // qraw[(n+1)&1] was last used in segment n-1 and kvraw was consumed
        // above: prefetch the next segment's q (and new rows) while this
        // segment streams.
        if (warp == 0 && q_issued == n + 1 && issue_q<PAGED>(A, S, n + 1, s0, o0, s1, o1, lane)) q_issued = n + 2;

        // This lane's query head, its 16-byte chunks in KV-head-rotated order.
        // q and the accumulator as f32x2 pairs: chunk c is pairs 2c (x, y)
        // and 2c + 1 (z, w)
        uint64_t q2[32];
#pragma unroll
        for (int c = 0; c < 16; ++c) {
            const float4 qc = *reinterpret_cast<const float4*>(&S.qo[h * QS + 4 * ((c + g) & 15)]);
            q2[2 * c] = pk2(qc.x, qc.y);
            q2[2 * c + 1] = pk2(qc.z, qc.w);
        }

        float m_run = -INFINITY, l_run = 0.f;
        uint64_t a2[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) a2[i] = 0ull;

        for (int ta = seg_a; ta < seg_b; ta += TILE) {
            // Refill: the stage of tile it-1 takes tile it-1+NSTAGE once all
            // warps have released it.
            if (issuer && it >= 1 && !cur.done) {
                const int ps = (it - 1) % NSTAGE;
                if (!mbar_wait(&S.empty[ps], ((it - 1) / NSTAGE) & 1)) {
                    record_error(A.err, kErrWaitEmpty);
                    cur.done = true;
                } else {
                    cursor_issue<PAGED>(cur, A, S, ps, s1, o1, pol);
                    ++issued;
                }
            }
            const int nrows = min(ta + TILE, seg_b) - ta;
            const int st = it % NSTAGE;
            if (!__all_sync(0xffffffffu, mbar_wait(&S.full[st], (it / NSTAGE) & 1))) {
                record_error(A.err, kErrWaitFull);
                ok = false;
                break;
            }
            const int r0 = warp * RPW;
            // One tile: scores, online softmax and PV for this warp's RPW rows
            // at kp[r] / vp[r] (already offset to the lane's KV head).
            auto tile_rows = [&](const float* const (&kp)[RPW], const float* const (&vp)[RPW],
                                 const bool (&valid)[RPW]) __attribute__((always_inline)) {
                    // scores s_r = (q/8) . K_r, as (even, odd) dimension partial
                    // sums in f32x2 lanes, added at the end
                    float sc[RPW];
                    uint64_t sc2[RPW];
#pragma unroll
                    for (int r = 0; r < RPW; ++r) sc2[r] = 0ull;
#pragma unroll
                    for (int c = 0; c < 16; ++c) {
                        const int o = 4 * ((c + g) & 15);
                        const uint64_t qa = q2[2 * c], qb2 = q2[2 * c + 1];
#pragma unroll
                        for (int r = 0; r < RPW; ++r) {
                            const float4 kv = *reinterpret_cast<const float4*>(kp[r] + o);
                            sc2[r] = fma2(qa, pk2(kv.x, kv.y), sc2[r]);
                            sc2[r] = fma2(qb2, pk2(kv.z, kv.w), sc2[r]);
                        }
                    }
#pragma unroll
                    for (int r = 0; r < RPW; ++r) {
                        float a0, a1;
                        up2(sc2[r], a0, a1);
                        sc[r] = a0 + a1;
                    }
                    // online softmax over this warp's rows
                    float mb = -INFINITY;
#pragma unroll
                    for (int r = 0; r < RPW; ++r) {
                        if (!valid[r]) sc[r] = -INFINITY;
                        mb = fmaxf(mb, sc[r]);
                    }
                    if (mb > m_run) {
                        const float f = exp_sfu(m_run - mb);
                        l_run *= f;
#pragma unroll
                        for (int i = 0; i < 32; ++i) a2[i] = fma2(a2[i], pk2(f, f), 0ull);
                        m_run = mb;
                    }
                    float p[RPW];
#pragma unroll
                    for (int r = 0; r < RPW; ++r) {
                        p[r] = exp_sfu(sc[r] - m_run);
                        l_run += p[r];
                    }
                    // out += p_r * V_r
#pragma unroll
                    for (int c = 0; c < 16; ++c) {
                        const int o = 4 * ((c + g) & 15);
                        uint64_t axy = a2[2 * c], azw = a2[2 * c + 1];
#pragma unroll
                        for (int r = 0; r < RPW; ++r) {
                            const float4 vv = *reinterpret_cast<const float4*>(vp[r] + o);
                            const uint64_t pp = pk2(p[r], p[r]);
                            axy = fma2(pp, pk2(vv.x, vv.y), axy);
                            azw = fma2(pp, pk2(vv.z, vv.w), azw);
                        }
                        a2[2 * c] = axy;
                        a2[2 * c + 1] = azw;
                    }
            };
            if (nrows == TILE && !(ta <= sq.pos && sq.pos < ta + TILE)) {
                // full tile without the new row: rows at a constant stride
                // from one base, so the loads use immediate offsets
                const float* kb = &S.k[st][r0 * ROWF] + g * HD;
                const float* vb = &S.v[st][r0 * ROWF] + g * HD;
                const float* kp[RPW];
                const float* vp[RPW];
                bool valid[RPW];
#pragma unroll
                for (int r = 0; r < RPW; ++r) {
                    kp[r] = kb + r * ROWF;
                    vp[r] = vb + r * ROWF;
                    valid[r] = true;
                }
                tile_rows(kp, vp, valid);
            } else if (r0 < nrows) {
                const float* kp[RPW];
                const float* vp[RPW];
                bool valid[RPW];
#pragma unroll
                for (int r = 0; r < RPW; ++r) {
                    valid[r] = (r0 + r) < nrows;
                    const int rr = valid[r] ? r0 + r : r0;  // invalid rows alias a valid one
                    const bool is_new = (ta + rr) == sq.pos;
                    kp[r] = (is_new ? S.newk : &S.k[st][rr * ROWF]) + g * HD;
                    vp[r] = (is_new ? S.newv : &S.v[st][rr * ROWF]) + g * HD;
                }
                tile_rows(kp, vp, valid);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.empty[st]);
            ++it;
        }
        if (!ok) break;
        float4 acc[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) {
            up2(a2[2 * c], acc[c].x, acc[c].y);
            up2(a2[2 * c + 1], acc[c].z, acc[c].w);
        }

        // ---- tree merge of the 8 warps' (m, l, acc): 8 -> 4 -> 2 -> 1 ----
        // (every lane of a pair of warps holds the same query head with the
        // same chunk rotation, so rows are merged in place).  8 -> 4 through
        // TMEM.  Then buffers A (qraw[qb], free since the prologue barrier,
        // next rewritten by segment n + 2's q copy) and B (qo, free once
        // every warp has loaded its q registers, which the first barrier
        // guarantees; B's last reader passes the third barrier before any
        // warp rotates the next segment's q into it).
        if (warp >= 4) {
            tc_fence_after();
            tmem_put(tq, m_run, l_run, acc);
            tc_fence_before();
        }
        if (!cta_sync(S, cphase, lane)) { record_error(A.err, kErrWaitFull); ok = false; break; }
        float* OA = S.qraw[qb];
        if (warp < 4) {
            tc_fence_after();
            tmem_merge_in(tq, m_run, l_run, acc);
            tc_fence_before();
        }
        if (warp == 2) merge_out(m_run, l_run, acc, S.qo + h * QS);
        if (warp == 3) merge_out_a(m_run, l_run, acc, OA, S.mlA, h);
        if (!cta_sync(S, cphase, lane)) { record_error(A.err, kErrWaitFull); ok = false; break; }
        if (warp == 0) merge_in(m_run, l_run, acc, S.qo + h * QS);
        if (warp == 1) {
            merge_in_a(m_run, l_run, acc, OA, S.mlA, h);
            __syncwarp();
            merge_out_a(m_run, l_run, acc, OA, S.mlA, h);
        }
        // CTAs sharing this sequence (every warp: the wide merge needs them)
        const bool split = A.arrivals && !(seg_a == 0 && seg_b == L);
        const SeqCtas sc = split ? A.seq_ctas[s] : SeqCtas{0, 0};
        const bool wide = split && sc.hi - sc.lo + 1 >= kWideMergeParts;
        if (!cta_sync(S, cphase, lane)) { record_error(A.err, kErrWaitFull); ok = false; break; }
        if (warp == 0) {
            merge_in_a(m_run, l_run, acc, OA, S.mlA, h);
            // ---- write: whole sequence -> output; otherwise a partial ----
            // Staged through buffer A (only warp 0 touches it from here to
            // the next segment's prologue) so the global stores are coalesced.
            __syncwarp();
#pragma unroll
            for (int c = 0; c < 16; ++c)
                *reinterpret_cast<float4*>(OA + h * HD + 4 * ((((c + g) & 15) + h) & 15)) = acc[c];
            __syncwarp();
            const bool whole = (seg_a == 0 && seg_b == L);
            const float scale = whole ? 1.0f / l_run : 1.0f;
            float* dst = whole ? A.out + static_cast<size_t>(s) * NH * HD
                               : A.partials + static_cast<size_t>(s + cta) * kPartialFloats;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const int hh = coalesced_head(i, lane);
                const float f = __shfl_sync(0xffffffffu, scale, hh);
                const float4 v = *reinterpret_cast<const float4*>(OA + hh * HD + 4 * (((lane & 15) + hh) & 15));
                reinterpret_cast<float4*>(dst)[32 * i + lane] = make_float4(v.x * f, v.y * f, v.z * f, v.w * f);
            }
            if (whole && A.lse) A.lse[h] = m_run + logf(l_run);   // single mode only
            if (!whole) {
                dst[NH * HD + h] = m_run;
                dst[NH * HD + NH + h] = l_run;
                if (wide) {
                    const bool last = arrive_last(A, s, lane, sc);
                    if (lane == 0) S.merge_last = last ? 1 : 0;
                } else if (A.arrivals && arrive_last(A, s, lane, sc)) {
                    merge_partials(A, s, lane, sc);
                }
            }
            __syncwarp();
        }
        if (wide) {   // the same value in every warp
            if (!cta_sync(S, cphase, lane)) { record_error(A.err, kErrWaitFull); ok = false; break; }
            if (S.merge_last) merge_partials_wide(A, s, warp, lane, sc);
        }
    }

    // Exit: every copy the issuer started must land before the CTA's shared
    // memory is released (tiles and q copies remain only on the error path;
    // a page-id prefetch can remain in paged mode).
    if (issuer) {
        if (PAGED) cp_async_wait_all();
        for (int t = it; t < issued; ++t)
            if (!mbar_wait(&S.full[t % NSTAGE], (t / NSTAGE) & 1)) { record_error(A.err, kErrDrain); break; }
        for (int m = n; m < q_issued; ++m)
            if (!mbar_wait(&S.qfull[m & 1], (m >> 1) & 1)) { record_error(A.err, kErrDrain); break; }
    }
    // Every warp gets here (all waits are bounded); the allocating warp frees
    // the tensor memory once no warp can touch it.
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(S.tmem_base, kTmemCols);
    }
}

// Single-sequence mode: combines the split-K partials of the CTAs.  Thread
// t owns query head t / 8, dims 8 (t % 8) .. +8.  The partials are folded in
// chunks of 8 with every load of a chunk issued before any is used (one L2
// round trip per chunk), with an online rescale between chunks.  Launched as
// a programmatic dependent of decode_kernel: it may start while the decode
// grid runs and waits (griddepcontrol.wait) for its partials.
constexpr int kMergeChunk = 8;
__global__ void __launch_bounds__(256) merge_kernel(const __grid_constant__ DecodeArgs A) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int s = blockIdx.x;
    const int lo = 0, hi = A.n_ctas - 1;
    if (lo >= hi) return;
    const int t = threadIdx.x;
    const int h = t >> 3;
    const int d0 = (t & 7) * 8;
    float m_run = -INFINITY, l_run = 0.f;
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = 0.f;
    for (int c0 = lo; c0 <= hi; c0 += kMergeChunk) {
        float mc[kMergeChunk], lc[kMergeChunk];
        float4 a0[kMergeChunk], a1[kMergeChunk];
#pragma unroll
        for (int u = 0; u < kMergeChunk; ++u) {
            mc[u] = -INFINITY;
            lc[u] = 0.f;
            a0[u] = a1[u] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (c0 + u <= hi) {
                const float* P = A.partials + static_cast<size_t>(s + c0 + u) * kPartialFloats;
                mc[u] = ld_cg(P + NH * HD + h);
                lc[u] = ld_cg(P + NH * HD + NH + h);
                a0[u] = ld_cg4(reinterpret_cast<const float4*>(P + h * HD + d0));
                a1[u] = ld_cg4(reinterpret_cast<const float4*>(P + h * HD + d0 + 4));
            }
        }
        float mn = m_run;
#pragma unroll
        for (int u = 0; u < kMergeChunk; ++u) mn = fmaxf(mn, mc[u]);
        const float fr = (m_run == -INFINITY) ? 0.f : expf(m_run - mn);
        l_run *= fr;
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] *= fr;
#pragma unroll
        for (int u = 0; u < kMergeChunk; ++u) {
            const float f = (mc[u] == -INFINITY) ? 0.f : expf(mc[u] - mn);
            l_run = fmaf(lc[u], f, l_run);
            o[0] = fmaf(a0[u].x, f, o[0]); o[1] = fmaf(a0[u].y, f, o[1]);
            o[2] = fmaf(a0[u].z, f, o[2]); o[3] = fmaf(a0[u].w, f, o[3]);
            o[4] = fmaf(a1[u].x, f, o[4]); o[5] = fmaf(a1[u].y, f, o[5]);
            o[6] = fmaf(a1[u].z, f, o[6]); o[7] = fmaf(a1[u].w, f, o[7]);
        }
        m_run = mn;
    }
    float4* dst = reinterpret_cast<float4*>(A.out + static_cast<size_t>(s) * NH * HD + h * HD + d0);
    dst[0] = make_float4(o[0] / l_run, o[1] / l_run, o[2] / l_run, o[3] / l_run);
    dst[1] = make_float4(o[4] / l_run, o[5] / l_run, o[6] / l_run, o[7] / l_run);
    if (A.lse && (t & 7) == 0) A.lse[h] = m_run + logf(l_run);
}

// Context-split combine: thread t owns head t / 8, dims 8 (t % 8) .. +8;
// all parts' loads of a head are independent (one round trip per 8 parts).
__global__ void __launch_bounds__(256) merge_lse_kernel(float* out, const float* parts, const float* lses,
                                                        int n_parts) {
    const int t = threadIdx.x;
    const int h = t >> 3;
    const int d0 = (t & 7) * 8;
    float mx = -INFINITY;
    for (int r = 0; r < n_parts; ++r) mx = fmaxf(mx, lses[static_cast<size_t>(r) * NH + h]);
    float wsum = 0.f;
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = 0.f;
    for (int r = 0; r < n_parts; ++r) {
        const float lr = lses[static_cast<size_t>(r) * NH + h];
        const float w = (lr == -INFINITY) ? 0.f : expf(lr - mx);
        wsum += w;
        const float4* src = reinterpret_cast<const float4*>(parts + static_cast<size_t>(r) * NH * HD + h * HD + d0);
        const float4 a0 = src[0], a1 = src[1];
        o[0] = fmaf(a0.x, w, o[0]); o[1] = fmaf(a0.y, w, o[1]);
        o[2] = fmaf(a0.z, w, o[2]); o[3] = fmaf(a0.w, w, o[3]);
        o[4] = fmaf(a1.x, w, o[4]); o[5] = fmaf(a1.y, w, o[5]);
        o[6] = fmaf(a1.z, w, o[6]); o[7] = fmaf(a1.w, w, o[7]);
    }
    float4* dst = reinterpret_cast<float4*>(out + h * HD + d0);
    dst[0] = make_float4(o[0] / wsum, o[1] / wsum, o[2] / wsum, o[3] / wsum);
    dst[1] = make_float4(o[4] / wsum, o[5] / wsum, o[6] / wsum, o[7] / wsum);
}

// ---- short single-sequence decode ------------------------------------------
// attention() for one sequence with L = pos + 1 <= kSeqMaxRows rows, built for
// latency: one thread-block cluster per KV head g, its C CTAs (C <= 8) taking
// consecutive chunks of R rows (R a multiple of 32, C R >= L).  CTA (c, g)
// copies its rows of KV head g into shared memory with 16-byte cp.async, warp
// w computes query head 8 g + w over them (lane = row for the scores, lane = a
// pair of dimensions for P V) and keeps the chunk's (o, m, l) of its eight
// heads in shared memory.  After a cluster barrier CTA c folds head 8 g + c
// (and + C, + 2C, ... when C < 8) over the C chunks in chunk order
// (deterministic) through distributed shared memory and writes the output: no
// workspace, no global atomics, one launch.  A second barrier keeps every
// CTA's shared memory alive until its peers have read it.  The last chunk's
// CTAs rotate the new k (every CTA rotates q for its own heads) and append
// their KV head's slice of k and v at row pos (ops.cpp:1350-1371).
constexpr int SEQ_THREADS = 256;
constexpr int SEQ_KP = HD + 4;   // padded row (floats): lane-per-row float4 reads hit all banks
constexpr int SEQ_PF = HD + 4;   // one head's partial in shared memory: o[64], m, l (+ pad)

__global__ void __launch_bounds__(SEQ_THREADS) seq_decode_kernel(const __grid_constant__ SeqArgs A) {
    extern __shared__ __align__(16) float seq_smem[];
    float* ks = seq_smem;                                    // [R][SEQ_KP]
    float* vs = ks + A.chunk_rows * SEQ_KP;                  // [R][SEQ_KP]
    float* qs = vs + A.chunk_rows * SEQ_KP;                  // [8][64]
    float* comb = qs + 8 * HD;                               // [8][SEQ_PF]: the second row half's
    float* recv = comb + 8 * SEQ_PF;                         // [n_chunks][8][SEQ_PF]: the chunk records
                                                             // of the heads this CTA folds
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    cg::cluster_group cl = cg::this_cluster();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int c = blockIdx.x, g = blockIdx.y;   // cluster = the n_chunks CTAs of KV head g
    // this cluster's sequence (batch mode: record blockIdx.z, written by the
    // host before the launch)
    const int sz = blockIdx.z;
    const bool batch = A.seqs != nullptr;
    const tle_seq_t sq = batch ? A.seqs[sz] : tle_seq_t{A.key_cache, A.value_cache, A.n_ctx, A.pos};
    const float* qin = A.q + (batch ? static_cast<size_t>(sz) * NH * HD : 0);
    const float* kin = A.k + (batch ? static_cast<size_t>(sz) * ROWF : 0);
    const float* vin = A.v + (batch ? static_cast<size_t>(sz) * ROWF : 0);
    float* outp = A.out + (batch ? static_cast<size_t>(sz) * NH * HD : 0);
    float* const key_cache = sq.key_cache;
    float* const value_cache = sq.value_cache;
    const int L = sq.pos + 1;
    // batch mode: a record outside its cache, or longer than the launch's
    // max_rows (more chunks than the cluster has CTAs), is reported and
    // skipped by every CTA of its cluster alike (no access, no cluster sync)
    if (batch && (sq.pos < 0 || sq.pos >= sq.n_ctx || L > static_cast<int>(gridDim.x) * A.chunk_rows ||
                  !key_cache || !value_cache)) {
        if (c == 0 && g == 0 && tid == 0) record_error(A.err, kErrBadSeq);
        return;
    }
    // this CTA has started: the cluster's CTAs wait for it (below) before
    // they store into its shared memory
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
    const int C = (L + A.chunk_rows - 1) / A.chunk_rows;   // this sequence's chunks (<= n_chunks)
    const int r0 = c * A.chunk_rows;
    const int nrows = max(0, min(A.chunk_rows, L - r0));
    const bool has_new = nrows > 0 && (r0 + nrows == L);
    const size_t layer_base = static_cast<size_t>(A.layer) * sq.n_ctx * ROWF;
    // cached rows of this chunk (row pos comes from the new k and v)
    const int ncached = has_new ? nrows - 1 : nrows;
    auto load_rows = [&]() {
        for (int e = tid; e < ncached * 32; e += SEQ_THREADS) {
            const int r = e >> 5, piece = e & 31;           // 16 pieces of K then 16 of V
            const float* src = (piece < 16 ? key_cache : value_cache) + layer_base +
                               static_cast<size_t>(r0 + r) * ROWF + g * HD + 4 * (piece & 15);
            float* dst = (piece < 16 ? ks : vs) + r * SEQ_KP + 4 * (piece & 15);
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    // q, k, v and the cache may be the previous kernel's output; with
    // kv_ready the caller guarantees that kernel wrote none of the cached
    // rows read here (in a forward pass it is the q/k/v projection), so they
    // stream while it drains
    if (A.kv_ready) {
        load_rows();
        asm volatile("griddepcontrol.wait;" ::: "memory");
    } else {
        asm volatile("griddepcontrol.wait;" ::: "memory");
        load_rows();
    }
    // q of this cluster's heads (rotated, x 1/8) and, in the last chunk, the new row
    {
        const int p = lane;   // rotation pair
        float sn = A.rope_sin[p], cs = A.rope_cos[p];
        if (batch && A.rotate) sincosf(static_cast<float>(sq.pos) * A.inv_freq[p], &sn, &cs);
        const float2 x = reinterpret_cast<const float2*>(qin + static_cast<size_t>(8 * g + warp) * HD)[p];
        float y0 = x.x, y1 = x.y;
        if (A.rotate) {
            y0 = x.x * cs - x.y * sn;
            y1 = x.x * sn + x.y * cs;
        }
        *reinterpret_cast<float2*>(&qs[warp * HD + 2 * p]) = make_float2(y0 * kScale, y1 * kScale);
        if (has_new && warp < 2) {
            const size_t row = layer_base + static_cast<size_t>(sq.pos) * ROWF + g * HD;
            if (warp == 0) {   // k: rotate, keep, append (ops.cpp:1370)
                const float2 kx = reinterpret_cast<const float2*>(kin + g * HD)[p];
                float k0 = kx.x, k1 = kx.y;
                if (A.rotate) {
                    k0 = kx.x * cs - kx.y * sn;
                    k1 = kx.x * sn + kx.y * cs;
                }
                *reinterpret_cast<float2*>(&ks[(nrows - 1) * SEQ_KP + 2 * p]) = make_float2(k0, k1);
                reinterpret_cast<float2*>(key_cache + row)[p] = make_float2(k0, k1);
            } else {           // v: keep, append (ops.cpp:1371)
                const float2 vx = reinterpret_cast<const float2*>(vin + g * HD)[p];
                *reinterpret_cast<float2*>(&vs[(nrows - 1) * SEQ_KP + 2 * p]) = vx;
                reinterpret_cast<float2*>(value_cache + row)[p] = vx;
            }
        }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();

    // warp w: query heads 2 hp, 2 hp + 1 of the cluster's eight (hp = w & 3)
    // over the row blocks 32 half, 32 half + 64, ... (half = w >> 2): scores
    // lane = row, online softmax across blocks, P V with lane = dimensions
    // 2 lane, 2 lane + 1; each K/V row read from shared memory serves both
    // heads.  The halves are folded in shared memory below.
    const int hp = warp & 3, half = warp >> 2;
    const float4* qa = reinterpret_cast<const float4*>(&qs[(2 * hp) * HD]);   // broadcast reads
    const float4* qb = reinterpret_cast<const float4*>(&qs[(2 * hp + 1) * HD]);
    float ma = -INFINITY, la = 0.f, oa0 = 0.f, oa1 = 0.f;
    float mb = -INFINITY, lb = 0.f, ob0 = 0.f, ob1 = 0.f;
    for (int rb = 32 * half; rb < nrows; rb += 64) {
        const int r = rb + lane;
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f, b0 = 0.f, b1 = 0.f, b2 = 0.f, b3 = 0.f;
        if (r < nrows) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const float4 kk = *reinterpret_cast<const float4*>(&ks[r * SEQ_KP + 4 * i]);
                const float4 x = qa[i], y = qb[i];
                a0 = fmaf(x.x, kk.x, a0);
                a1 = fmaf(x.y, kk.y, a1);
                a2 = fmaf(x.z, kk.z, a2);
                a3 = fmaf(x.w, kk.w, a3);
                b0 = fmaf(y.x, kk.x, b0);
                b1 = fmaf(y.y, kk.y, b1);
                b2 = fmaf(y.z, kk.z, b2);
                b3 = fmaf(y.w, kk.w, b3);
            }
        }
        const float sa = (r < nrows) ? (a0 + a1) + (a2 + a3) : -INFINITY;
        const float sb = (r < nrows) ? (b0 + b1) + (b2 + b3) : -INFINITY;
        float xa = sa, xb = sb;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            xa = fmaxf(xa, __shfl_xor_sync(0xffffffffu, xa, o));
            xb = fmaxf(xb, __shfl_xor_sync(0xffffffffu, xb, o));
        }
        const float na = fmaxf(ma, xa), nb_ = fmaxf(mb, xb);
        const float fa = (ma == -INFINITY) ? 0.f : expf(ma - na);
        const float fb = (mb == -INFINITY) ? 0.f : expf(mb - nb_);
        const float pa = (sa == -INFINITY) ? 0.f : expf(sa - na);
        const float pb = (sb == -INFINITY) ? 0.f : expf(sb - nb_);
        float ta = pa, tb = pb;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            ta += __shfl_xor_sync(0xffffffffu, ta, o);
            tb += __shfl_xor_sync(0xffffffffu, tb, o);
        }
        la = fmaf(la, fa, ta);
        lb = fmaf(lb, fb, tb);
        oa0 *= fa;
        oa1 *= fa;
        ob0 *= fb;
        ob1 *= fb;
        ma = na;
        mb = nb_;
        const int nb = min(32, nrows - rb);
        for (int j0 = 0; j0 < nb; j0 += 8) {   // eight rows' shuffles and loads in flight
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) {
                const int j = j0 + jj;   // < 32
                const float wa = __shfl_sync(0xffffffffu, pa, j), wb = __shfl_sync(0xffffffffu, pb, j);
                const float2 vv = *reinterpret_cast<const float2*>(&vs[(rb + j) * SEQ_KP + 2 * lane]);
                if (j < nb) {
                    oa0 = fmaf(wa, vv.x, oa0);
                    oa1 = fmaf(wa, vv.y, oa1);
                    ob0 = fmaf(wb, vv.x, ob0);
                    ob1 = fmaf(wb, vv.y, ob1);
                }
            }
        }
    }
    // the second half's (o, m, l) to comb; the first folds it (a half
    // without rows: m = -inf, l = 0) and writes this chunk's partial of its
    // two heads (an empty chunk: m = -inf, l = 0)
    if (half == 1) {
        float* ca = comb + (2 * hp) * SEQ_PF;
        float* cb = comb + (2 * hp + 1) * SEQ_PF;
        reinterpret_cast<float2*>(ca)[lane] = make_float2(oa0, oa1);
        reinterpret_cast<float2*>(cb)[lane] = make_float2(ob0, ob1);
        if (lane == 0) {
            ca[HD] = ma;
            ca[HD + 1] = la;
            cb[HD] = mb;
            cb[HD + 1] = lb;
        }
    }
    __syncthreads();
    // Records of this chunk, pushed into the folding CTA of each head (head
    // hl: CTA hl mod C, warp hl / C) with remote stores, slot (chunk, head);
    // after the cluster barrier every fold reads its own shared memory, and
    // no CTA touches another's afterwards (no second barrier).
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");   // every CTA of the cluster has started
    if (half == 0 && c < C) {
        auto fold = [&](int hl, float m0, float l0, float o0, float o1) {
            const float* cc = comb + hl * SEQ_PF;
            const float m1 = cc[HD], l1 = cc[HD + 1];
            const float2 p1 = reinterpret_cast<const float2*>(cc)[lane];
            const float mt = fmaxf(m0, m1);
            const float f0 = (m0 == -INFINITY) ? 0.f : expf(m0 - mt);
            const float f1 = (m1 == -INFINITY) ? 0.f : expf(m1 - mt);
            float* dst = cl.map_shared_rank(recv, hl % C) + (c * 8 + hl) * SEQ_PF;
            reinterpret_cast<float2*>(dst)[lane] = make_float2(o0 * f0 + p1.x * f1, o1 * f0 + p1.y * f1);
            if (lane == 0) {
                dst[HD] = mt;
                dst[HD + 1] = l0 * f0 + l1 * f1;
            }
        };
        fold(2 * hp, ma, la, oa0, oa1);
        fold(2 * hp + 1, mb, lb, ob0, ob1);
    }
    cl.sync();
    // fold: CTA c takes heads c, c + C, ... of this KV head, one warp each
    // (the sequence's C chunks: CTAs c >= C of a shorter sequence of the batch fold nothing)
    for (int hl = c + C * warp; c < C && warp < 8 && hl < 8; hl += C * 8) {
        // every chunk's record in flight at once (C <= 8), then the fold in chunk order
        float mc[kSeqMaxChunks], lc[kSeqMaxChunks];
        float2 oc[kSeqMaxChunks];
#pragma unroll
        for (int cc = 0; cc < kSeqMaxChunks; ++cc) {
            mc[cc] = -INFINITY;
            lc[cc] = 0.f;
            oc[cc] = make_float2(0.f, 0.f);
            if (cc < C) {
                const float* pp = recv + (cc * 8 + hl) * SEQ_PF;
                mc[cc] = pp[HD];
                lc[cc] = pp[HD + 1];
                oc[cc] = reinterpret_cast<const float2*>(pp)[lane];
            }
        }
        float mt = -INFINITY;
#pragma unroll
        for (int cc = 0; cc < kSeqMaxChunks; ++cc) mt = fmaxf(mt, mc[cc]);
        float acc0 = 0.f, acc1 = 0.f, lt = 0.f;
#pragma unroll
        for (int cc = 0; cc < kSeqMaxChunks; ++cc) {
            if (cc < C) {
                const float f = (mc[cc] == -INFINITY) ? 0.f : expf(mc[cc] - mt);
                lt = fmaf(lc[cc], f, lt);
                acc0 = fmaf(oc[cc].x, f, acc0);
                acc1 = fmaf(oc[cc].y, f, acc1);
            }
        }
        const int h = 8 * g + hl;
        const float inv = 1.0f / lt;
        reinterpret_cast<float2*>(outp + h * HD)[lane] = make_float2(acc0 * inv, acc1 * inv);
        if (!batch && A.lse && lane == 0) A.lse[h] = mt + logf(lt);
    }
}

// rope() (ops.cpp:1223-1281): one thread per (head, pair); q heads then k heads.
__global__ void rope_kernel(const __grid_constant__ RopeArgs A) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    const int total = (A.n_head + A.n_head_kv) * A.half;
    if (j >= total) return;
    const int hh = j / A.half, i = j - hh * A.half;
    float* x = hh < A.n_head ? A.q + static_cast<size_t>(hh) * 2 * A.half
                             : A.k + static_cast<size_t>(hh - A.n_head) * 2 * A.half;
    float sn, cs;
    sincosf(static_cast<float>(A.pos) * A.inv_freq[i], &sn, &cs);
    const float x0 = x[2 * i], x1 = x[2 * i + 1];
    x[2 * i] = x0 * cs - x1 * sn;
    x[2 * i + 1] = x0 * sn + x1 * cs;
}

}  // namespace

// Failure-path self-test: the planted barrier (count 1) never receives an
// arrival, so every thread's bounded wait expires after limit_ns; thread 0
// records the code.  Nothing asynchronous is in flight when the block exits.
__global__ void __launch_bounds__(32) selftest_wait_kernel(uint32_t* err, uint64_t limit_ns) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
    }
    __syncwarp();
    const bool ok = mbar_wait_for(&bar, 0, limit_ns);
    if (!__all_sync(0xffffffffu, ok) && threadIdx.x == 0) record_error(err, kErrSelfTest);
}

cudaError_t launch_decode(const DecodeArgs& a, cudaStream_t stream) {
    static PerDeviceOnce once;
    const int smem = static_cast<int>(sizeof(DecodeSmem));
    cudaError_t e = once.run([&](int) {
        cudaError_t r = cudaFuncSetAttribute(decode_kernel<false>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (r != cudaSuccess) return r;
        return cudaFuncSetAttribute(decode_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    smem);
    });
    if (e != cudaSuccess) return e;
    // Launched as a programmatic dependent of the previous kernel on the
    // stream: its CTAs may start (barrier init, tensor-memory allocation,
    // descriptor reads) as the previous grid drains; griddepcontrol.wait in
    // the kernel orders everything else after that grid.
    cudaLaunchConfig_t dcfg{};
    dcfg.gridDim = dim3(a.n_ctas);
    dcfg.blockDim = dim3(NCT);
    dcfg.dynamicSmemBytes = static_cast<size_t>(smem);
    dcfg.stream = stream;
    cudaLaunchAttribute dattr[1];
    dattr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    dattr[0].val.programmaticStreamSerializationAllowed = 1;
    dcfg.attrs = dattr;
    dcfg.numAttrs = 1;
    if (a.key_pool)
        e = cudaLaunchKernelEx(&dcfg, decode_kernel<true>, a);
    else
        e = cudaLaunchKernelEx(&dcfg, decode_kernel<false>, a);
    if (e != cudaSuccess) return e;
    if (a.n_ctas > 1 && a.seqs == nullptr) {   // batch mode merges inside decode_kernel
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(a.n_seqs);
        cfg.blockDim = dim3(256);
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, merge_kernel, a);
    }
    return e;
}

cudaError_t launch_seq_decode(const SeqArgs& a, cudaStream_t stream) {
    const size_t smem =
        static_cast<size_t>(2 * a.chunk_rows * SEQ_KP + 8 * HD + (8 + 8 * a.n_chunks) * SEQ_PF) * sizeof(float);
    static PerDeviceOnce once;
    cudaError_t e = once.run([&](int) {
        return cudaFuncSetAttribute(seq_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(2 * kSeqMaxChunkRows * SEQ_KP * sizeof(float) +
                                                     (8 * HD + (8 + 8 * kSeqMaxChunks) * SEQ_PF) * sizeof(float)));
    });
    if (e != cudaSuccess) return e;
    // one cluster of n_chunks CTAs per KV head; a programmatic dependent of
    // the previous kernel (its CTAs may be scheduled while that grid drains;
    // griddepcontrol.wait orders the reads)
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(a.n_chunks, NKV_HEADS, a.seqs ? a.n_seqs : 1);
    cfg.blockDim = dim3(SEQ_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = a.n_chunks;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, seq_decode_kernel, a);
}

cudaError_t launch_rope(const RopeArgs& a, cudaStream_t stream) {
    const int total = (a.n_head + a.n_head_kv) * a.half;
    rope_kernel<<<(total + 255) / 256, 256, 0, stream>>>(a);
    return cudaGetLastError();
}

cudaError_t error_word(uint32_t** word) {
    static std::atomic<uint32_t*> cached[kMaxDevices] = {};   // thread-safe lazy lookup
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    uint32_t* w = cached[dev].load(std::memory_order_acquire);
    if (!w) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_tle_error);
        if (e != cudaSuccess) return e;
        w = static_cast<uint32_t*>(p);
        cached[dev].store(w, std::memory_order_release);
    }
    *word = w;
    return cudaSuccess;
}

cudaError_t read_device_error(int clear, uint32_t* code) {
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return e;
    e = cudaMemcpyFromSymbol(code, g_tle_error, sizeof(uint32_t));
    if (e != cudaSuccess) return e;
    if (clear && *code) {
        const uint32_t zero = 0;
        e = cudaMemcpyToSymbol(g_tle_error, &zero, sizeof(uint32_t));
    }
    return e;
}

cudaError_t launch_selftest_wait(uint32_t* err, uint64_t limit_ns, cudaStream_t stream) {
    selftest_wait_kernel<<<1, 32, 0, stream>>>(err, limit_ns);
    return cudaGetLastError();
}

cudaError_t launch_merge_lse(float* out, const float* parts, const float* lses, int n_parts,
                             cudaStream_t stream) {
    merge_lse_kernel<<<1, 256, 0, stream>>>(out, parts, lses, n_parts);
    return cudaGetLastError();
}

}  // namespace tle
