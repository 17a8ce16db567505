// abi.cu -- the extern "C" boundary (include/tle_attn.h): argument checks,
// the decode work plan and kernel launches.  No exceptions leave this file;
// every entry point returns a TLE_* status and records a message for
// tle_last_error().
#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <numeric>
#include <string>
#include <vector>

#include "kernels.h"
#include "tle_attn.h"
#include "tle_forward.h"

namespace {

thread_local std::string g_last_error;

int set_error(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int cuda_error(cudaError_t e, const char* what) {
    return set_error(TLE_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

int ok() {
    g_last_error.clear();
    return TLE_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// 1/freq_base^(2i/head_dim) with the reference's exact float expression
// (ops.cpp:1244-1245): std::pow on floats resolves to powf.
void fill_inv_freq(float* dst, int half, float freq_base) {
    const int head_dim = 2 * half;
    for (int i = 0; i < half; ++i)
        dst[i] = 1.0f / std::pow(freq_base, static_cast<float>(2 * i) / static_cast<float>(head_dim));
}

int check_shape(const tle_shape_t* shape) {
    if (!shape) return set_error(TLE_ERR_INVALID, "shape is NULL");
    if (shape->n_head != tle::kNHead || shape->n_head_kv != tle::kNHeadKv ||
        shape->head_dim != tle::kHeadDim)
        return set_error(TLE_ERR_UNSUPPORTED,
                         "attention kernels are built for n_head=32, n_head_kv=4, head_dim=64 "
                         "(got %d, %d, %d)",
                         shape->n_head, shape->n_head_kv, shape->head_dim);
    if (shape->n_layers <= 0) return set_error(TLE_ERR_INVALID, "n_layers must be > 0");
    if (!(shape->rope_freq_base > 0.f)) return set_error(TLE_ERR_INVALID, "rope_freq_base must be > 0");
    return TLE_OK;
}

int sm_count() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
        return 148;
    return n;
}

// Number of CTAs for `rows` attended rows: about one per SM, but never fewer
// than kMinRowsPerCta rows per CTA.
int choose_ctas(int64_t rows, int max_ctas) {
    if (max_ctas <= 0) max_ctas = sm_count();
    max_ctas = std::min(max_ctas, tle::kMaxCtas);
    const int64_t by_rows = (rows + tle::kMinRowsPerCta - 1) / tle::kMinRowsPerCta;
    return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(max_ctas, by_rows)));
}

// Splits a batch over G CTAs in "cost" units: every sequence costs its rows
// plus kSegCostRows (the per-segment setup of the decode kernel: q rotation,
// warp merge, output write: about three microseconds of streaming time; 128
// measured best on a 64-sequence ragged batch against 32 .. 256, and again
// against 96 and 160 with the tile-aligned starts below), so a
// CTA that holds several short segments gets fewer rows.  CTA boundaries are
// cost positions mapped to (sequence, row); a boundary inside a sequence's
// overhead lands on its first row, and a boundary inside a sequence is
// rounded down to a multiple of kStartAlignRows, the decode kernel's
// pipeline tile, so no CTA starts or ends a segment with a partial tile
// (config 4: 1.1 % faster contiguous, 1.7 % paged).  seq_ctas[t] = first and
// last CTA owning a row of t.  No allocation (shared by the no-allocation
// entry point).
constexpr int64_t kSegCostRows = 128;
constexpr int64_t kStartAlignRows = 32;

void plan_ctas(const tle_seq_t* seqs, int n, int G, tle::CtaStart* cs, tle::SeqCtas* sc) {
    int64_t T = 0;
    for (int t = 0; t < n; ++t) T += seqs[t].pos + 1 + kSegCostRows;
    int s = 0;
    int64_t X = 0;  // cost position where sequence s starts
    for (int c = 0; c <= G; ++c) {
        const int64_t x = (c == G) ? T : static_cast<int64_t>(c) * T / G;
        while (s < n && X + seqs[s].pos + 1 + kSegCostRows <= x) {
            X += seqs[s].pos + 1 + kSegCostRows;
            ++s;
        }
        if (s >= n) {
            cs[c].seq = n;
            cs[c].off = 0;
            continue;
        }
        const int64_t r = x - X - kSegCostRows;
        cs[c].seq = s;
        cs[c].off = r > 0 ? static_cast<int32_t>(r / kStartAlignRows * kStartAlignRows) : 0;
    }
    for (int t = 0; t < n; ++t) {
        sc[t].lo = G;
        sc[t].hi = -1;
    }
    for (int c = 0; c < G; ++c) {
        const tle::CtaStart b = cs[c], e = cs[c + 1];
        if (b.seq == e.seq && b.off == e.off) continue;  // empty CTA
        const int last = (e.off > 0) ? e.seq : e.seq - 1;
        for (int t = b.seq; t <= last && t < n; ++t) {
            if (c < sc[t].lo) sc[t].lo = c;
            if (c > sc[t].hi) sc[t].hi = c;
        }
    }
}

size_t partial_bytes(int n_slots) {
    return static_cast<size_t>(n_slots) * tle::kPartialFloats * sizeof(float);
}

int single_decode(float* out, const float* q, const float* k, const float* v, float* key_cache,
                  float* value_cache, int layer, int pos, int n_ctx, const tle_shape_t* shape,
                  void* workspace, size_t workspace_bytes, void* stream, int rotate,
                  float* lse = nullptr, int kv_ready = 0) {
    if (int rc = check_shape(shape)) return rc;
    if (!out || !q || !k || !v || !key_cache || !value_cache)
        return set_error(TLE_ERR_INVALID, "null buffer pointer");
    if (!aligned16(out) || !aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(key_cache) ||
        !aligned16(value_cache))
        return set_error(TLE_ERR_INVALID, "buffers must be 16-byte aligned");
    if (n_ctx <= 0 || pos < 0 || pos >= n_ctx)
        return set_error(TLE_ERR_INVALID, "need 0 <= pos < n_ctx (pos=%d, n_ctx=%d)", pos, n_ctx);
    if (layer < 0 || layer >= shape->n_layers)
        return set_error(TLE_ERR_INVALID, "layer %d outside [0, %d)", layer, shape->n_layers);
    const int L = pos + 1;
    if (L <= tle::kSeqMaxRows) {
        // short sequence: one launch, a cluster of up to 8 CTAs per KV head
        // taking chunks of 32 .. 256 rows (a multiple of 32)
        tle::SeqArgs s{};
        const int chunks = std::min(tle::kSeqMaxChunks, (L + 31) / 32);
        s.chunk_rows = ((L + chunks - 1) / chunks + 31) / 32 * 32;
        s.n_chunks = (L + s.chunk_rows - 1) / s.chunk_rows;
        (void)workspace;
        (void)workspace_bytes;
        s.q = q;
        s.k = k;
        s.v = v;
        s.out = out;
        s.lse = lse;
        s.key_cache = key_cache;
        s.value_cache = value_cache;
        s.layer = layer;
        s.pos = pos;
        s.n_ctx = n_ctx;
        s.rotate = rotate;
        s.kv_ready = kv_ready;
        // the rotation angles as the reference computes them (ops.cpp:1233-1238:
        // float angle, std::cos / std::sin), once per call on the host
        float inv_freq[tle::kHeadDim / 2];
        fill_inv_freq(inv_freq, tle::kHeadDim / 2, shape->rope_freq_base);
        for (int i = 0; i < tle::kHeadDim / 2; ++i) {
            const float angle = static_cast<float>(pos) * inv_freq[i];
            s.rope_cos[i] = std::cos(angle);
            s.rope_sin[i] = std::sin(angle);
        }
        cudaError_t e = tle::error_word(&s.err);
        if (e != cudaSuccess) return cuda_error(e, "device error word");
        e = tle::launch_seq_decode(s, static_cast<cudaStream_t>(stream));
        if (e != cudaSuccess) return cuda_error(e, "decode launch");
        return ok();
    }
    tle::DecodeArgs a{};
    a.seqs = nullptr;
    a.cta_start = nullptr;
    a.seq_ctas = nullptr;
    a.arrivals = nullptr;
    a.single.key_cache = key_cache;
    a.single.value_cache = value_cache;
    a.single.n_ctx = n_ctx;
    a.single.pos = pos;
    a.n_seqs = 1;
    a.n_ctas = choose_ctas(static_cast<int64_t>(pos) + 1, 0);
    if (a.n_ctas > 1) {
        if (!workspace) return set_error(TLE_ERR_WORKSPACE, "workspace is NULL");
        if (workspace_bytes < partial_bytes(a.n_ctas + 1))
            return set_error(TLE_ERR_WORKSPACE, "workspace %zu bytes < %zu needed", workspace_bytes,
                             partial_bytes(a.n_ctas + 1));
        if (!aligned16(workspace)) return set_error(TLE_ERR_INVALID, "workspace must be 16-byte aligned");
    }
    a.q = q;
    a.k = k;
    a.v = v;
    a.out = out;
    a.partials = static_cast<float*>(workspace);
    a.lse = lse;
    a.layer = layer;
    a.rotate = rotate;
    a.kv_ready = kv_ready;
    fill_inv_freq(a.inv_freq, tle::kHeadDim / 2, shape->rope_freq_base);
    cudaError_t e = tle::error_word(&a.err);
    if (e != cudaSuccess) return cuda_error(e, "device error word");
    e = tle::launch_decode(a, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_error(e, "decode launch");
    return ok();
}

}  // namespace

extern "C" {

const char* tle_last_error(void) { return g_last_error.c_str(); }

const char* tle_version(void) { return "tle_attn 0.1 (sm_100a)"; }

int tle_rope(float* q, float* k, int pos, int head_dim, int n_head, int n_head_kv, float freq_base,
             void* stream) {
    if (!q || (n_head_kv > 0 && !k)) return set_error(TLE_ERR_INVALID, "null q/k");
    if (head_dim <= 0 || (head_dim & 1) || head_dim > 256)
        return set_error(TLE_ERR_UNSUPPORTED, "head_dim must be even and <= 256 (got %d)", head_dim);
    if (n_head <= 0 || n_head_kv < 0) return set_error(TLE_ERR_INVALID, "bad head counts");
    if (pos < 0) return set_error(TLE_ERR_INVALID, "pos must be >= 0");
    tle::RopeArgs a{};
    a.q = q;
    a.k = k;
    a.pos = pos;
    a.half = head_dim / 2;
    a.n_head = n_head;
    a.n_head_kv = n_head_kv;
    fill_inv_freq(a.inv_freq, a.half, freq_base);
    cudaError_t e = tle::launch_rope(a, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_error(e, "rope launch");
    return ok();
}

size_t tle_attention_workspace_bytes(const tle_shape_t* shape, int n_ctx) {
    (void)shape;
    (void)n_ctx;
    return partial_bytes(tle::kMaxCtas + 1);
}

int tle_attention(float* out, const float* q, const float* k, const float* v, float* key_cache,
                  float* value_cache, int layer, int pos, int n_ctx, const tle_shape_t* shape,
                  void* workspace, size_t workspace_bytes, void* stream) {
    return single_decode(out, q, k, v, key_cache, value_cache, layer, pos, n_ctx, shape, workspace,
                         workspace_bytes, stream, 0);
}

int tle_attention_lse(float* out, float* lse, const float* q, const float* k, const float* v,
                      float* key_cache, float* value_cache, int layer, int pos, int n_ctx,
                      const tle_shape_t* shape, void* workspace, size_t workspace_bytes,
                      void* stream) {
    if (!lse || !aligned16(lse)) return set_error(TLE_ERR_INVALID, "lse must be a 16-byte aligned buffer");
    return single_decode(out, q, k, v, key_cache, value_cache, layer, pos, n_ctx, shape, workspace,
                         workspace_bytes, stream, 0, lse);
}

int tle_merge_lse(float* out, const float* parts, const float* lses, int n_parts, void* stream) {
    if (!out || !parts || !lses) return set_error(TLE_ERR_INVALID, "null buffer pointer");
    if (!aligned16(out) || !aligned16(parts)) return set_error(TLE_ERR_INVALID, "buffers must be 16-byte aligned");
    if (n_parts < 1) return set_error(TLE_ERR_INVALID, "n_parts %d < 1", n_parts);
    cudaError_t e = tle::launch_merge_lse(out, parts, lses, n_parts, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_error(e, "merge launch");
    return ok();
}

int tle_rope_attention(float* out, const float* q, const float* k, const float* v,
                       float* key_cache, float* value_cache, int layer, int pos, int n_ctx,
                       const tle_shape_t* shape, void* workspace, size_t workspace_bytes,
                       void* stream) {
    return single_decode(out, q, k, v, key_cache, value_cache, layer, pos, n_ctx, shape, workspace,
                         workspace_bytes, stream, 1);
}

int tle_rope_attention_flags(float* out, const float* q, const float* k, const float* v,
                             float* key_cache, float* value_cache, int layer, int pos, int n_ctx,
                             const tle_shape_t* shape, int flags, void* workspace, size_t workspace_bytes,
                             void* stream) {
    if (flags & ~TLE_DECODE_KV_READY) return set_error(TLE_ERR_INVALID, "unknown flags 0x%x", flags);
    return single_decode(out, q, k, v, key_cache, value_cache, layer, pos, n_ctx, shape, workspace,
                         workspace_bytes, stream, 1, nullptr, (flags & TLE_DECODE_KV_READY) ? 1 : 0);
}

size_t tle_decode_desc_bytes(int n_seqs, int max_ctas) {
    if (n_seqs < 0) n_seqs = 0;
    if (max_ctas <= 0 || max_ctas > tle::kMaxCtas) max_ctas = tle::kMaxCtas;
    return tle::desc_total_bytes(n_seqs, max_ctas);
}

namespace {

// Writes the descriptor for `n_seqs` validated records (their pos fields
// drive the plan; the records are copied as they are).
int write_desc(const tle_seq_t* seqs, int n_seqs, int max_ctas, int32_t magic, void* desc_host,
               size_t desc_bytes, int* n_ctas_out) {
    int64_t total = 0;
    for (int s = 0; s < n_seqs; ++s) total += static_cast<int64_t>(seqs[s].pos) + 1;
    const int G = choose_ctas(total, max_ctas);
    const size_t need = tle::desc_total_bytes(n_seqs, G);
    if (desc_bytes < need)
        return set_error(TLE_ERR_INVALID, "descriptor buffer %zu bytes < %zu needed", desc_bytes, need);
    unsigned char* base = static_cast<unsigned char*>(desc_host);
    tle::DescHeader hdr{};
    hdr.magic = magic;
    hdr.n_seqs = n_seqs;
    hdr.n_ctas = G;
    hdr.total_rows = total;
    std::memcpy(base, &hdr, sizeof hdr);
    std::memcpy(base + tle::desc_seqs_offset(), seqs, sizeof(tle_seq_t) * static_cast<size_t>(n_seqs));
    auto* cs = reinterpret_cast<tle::CtaStart*>(base + tle::desc_cta_offset(n_seqs));
    auto* sc = reinterpret_cast<tle::SeqCtas*>(base + tle::desc_seqctas_offset(n_seqs, G));
    plan_ctas(seqs, n_seqs, G, cs, sc);
    std::memset(base + tle::desc_arrivals_offset(n_seqs, G), 0, sizeof(int32_t) * static_cast<size_t>(n_seqs));
    *n_ctas_out = G;
    return ok();
}

int check_pool(const tle_shape_t* shape, const tle_page_pool_t* pool, int* shift) {
    if (!pool || !pool->key_pool || !pool->value_pool)
        return set_error(TLE_ERR_INVALID, "page pool and both pools must be non-null");
    if (!aligned16(pool->key_pool) || !aligned16(pool->value_pool))
        return set_error(TLE_ERR_INVALID, "page pools must be 16-byte aligned");
    const int pr = pool->page_rows;
    if (pr < 16 || pr > 65536 || (pr & (pr - 1)) != 0)
        return set_error(TLE_ERR_INVALID, "page_rows %d is not a power of two in [16, 65536]", pr);
    if (pool->n_pages <= 0) return set_error(TLE_ERR_INVALID, "pool n_pages %d <= 0", pool->n_pages);
    // row offsets are formed in 64 bits; keep the pool below 2^62 floats
    const double rows = static_cast<double>(shape->n_layers) * pool->n_pages * pr;
    if (rows * tle::kRowFloats > 4.0e18) return set_error(TLE_ERR_INVALID, "page pool too large");
    int sh = 0;
    while ((1 << sh) < pr) ++sh;
    *shift = sh;
    return 0;
}

// Fills the kernel arguments shared by the contiguous and paged batch calls.
int batch_args(const tle_shape_t* shape, const void* desc_dev, int n_seqs, int n_ctas, const float* q,
               const float* k, const float* v, float* out, int layer, int flags, void* workspace,
               size_t workspace_bytes, tle::DecodeArgs& a) {
    if (int rc = check_shape(shape)) return rc;
    if (!desc_dev || !q || !k || !v || !out) return set_error(TLE_ERR_INVALID, "null pointer argument");
    if (n_seqs <= 0 || n_ctas <= 0 || n_ctas > tle::kMaxCtas)
        return set_error(TLE_ERR_INVALID, "bad n_seqs/n_ctas (%d, %d)", n_seqs, n_ctas);
    if (!aligned16(desc_dev) || !aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out))
        return set_error(TLE_ERR_INVALID, "buffers must be 16-byte aligned");
    if (layer < 0 || layer >= shape->n_layers)
        return set_error(TLE_ERR_INVALID, "layer %d outside [0, %d)", layer, shape->n_layers);
    const size_t need = partial_bytes(n_ctas + n_seqs);
    if (!workspace || workspace_bytes < need || !aligned16(workspace))
        return set_error(TLE_ERR_WORKSPACE, "workspace %zu bytes < %zu needed (or unaligned)",
                         workspace_bytes, need);
    const unsigned char* base = static_cast<const unsigned char*>(desc_dev);
    a = tle::DecodeArgs{};
    a.seqs = reinterpret_cast<const tle_seq_t*>(base + tle::desc_seqs_offset());
    a.cta_start = reinterpret_cast<const tle::CtaStart*>(base + tle::desc_cta_offset(n_seqs));
    a.seq_ctas = reinterpret_cast<const tle::SeqCtas*>(base + tle::desc_seqctas_offset(n_seqs, n_ctas));
    a.arrivals = reinterpret_cast<int32_t*>(const_cast<unsigned char*>(base) + tle::desc_arrivals_offset(n_seqs, n_ctas));
    a.n_seqs = n_seqs;
    a.n_ctas = n_ctas;
    a.q = q;
    a.k = k;
    a.v = v;
    a.out = out;
    a.partials = static_cast<float*>(workspace);
    if (flags & ~(TLE_DECODE_ROTATE | TLE_DECODE_KV_READY))
        return set_error(TLE_ERR_INVALID, "unknown decode flags 0x%x", flags);
    a.layer = layer;
    a.rotate = (flags & TLE_DECODE_ROTATE) ? 1 : 0;
    a.kv_ready = (flags & TLE_DECODE_KV_READY) ? 1 : 0;
    fill_inv_freq(a.inv_freq, tle::kHeadDim / 2, shape->rope_freq_base);
    cudaError_t e = tle::error_word(&a.err);
    if (e != cudaSuccess) return cuda_error(e, "device error word");
    return 0;
}

}  // namespace

int tle_decode_desc(const tle_shape_t* shape, const tle_seq_t* seqs, int n_seqs, int max_ctas,
                    void* desc_host, size_t desc_bytes, int* n_ctas_out) {
    if (int rc = check_shape(shape)) return rc;
    if (n_seqs <= 0 || !seqs || !desc_host || !n_ctas_out)
        return set_error(TLE_ERR_INVALID, "need n_seqs > 0 and non-null seqs/desc/n_ctas");
    for (int s = 0; s < n_seqs; ++s) {
        const tle_seq_t& q = seqs[s];
        if (!q.key_cache || !q.value_cache || !aligned16(q.key_cache) || !aligned16(q.value_cache))
            return set_error(TLE_ERR_INVALID, "sequence %d: caches must be non-null and 16-byte aligned", s);
        if (q.n_ctx <= 0 || q.pos < 0 || q.pos >= q.n_ctx)
            return set_error(TLE_ERR_INVALID, "sequence %d: need 0 <= pos < n_ctx (pos=%d, n_ctx=%d)", s,
                             q.pos, q.n_ctx);
    }
    return write_desc(seqs, n_seqs, max_ctas, tle::kDescMagic, desc_host, desc_bytes, n_ctas_out);
}

int tle_decode_desc_paged(const tle_shape_t* shape, const tle_page_pool_t* pool,
                          const tle_paged_seq_t* seqs, int n_seqs, int max_ctas, void* desc_host,
                          size_t desc_bytes, int* n_ctas_out) {
    if (int rc = check_shape(shape)) return rc;
    int shift = 0;
    if (int rc = check_pool(shape, pool, &shift)) return rc;
    if (n_seqs <= 0 || !seqs || !desc_host || !n_ctas_out)
        return set_error(TLE_ERR_INVALID, "need n_seqs > 0 and non-null seqs/desc/n_ctas");
    // The descriptor's 24-byte sequence slots carry {page table, -, n_pages, pos}.
    // (a byte vector: nvcc's front end rejects std::vector of the C ABI's
    // unnamed struct types)
    std::vector<unsigned char> rec_bytes(sizeof(tle_seq_t) * static_cast<size_t>(n_seqs));
    tle_seq_t* recs = reinterpret_cast<tle_seq_t*>(rec_bytes.data());
    for (int s = 0; s < n_seqs; ++s) {
        const tle_paged_seq_t& q = seqs[s];
        if (!q.pages || (reinterpret_cast<uintptr_t>(q.pages) & 3u) != 0)
            return set_error(TLE_ERR_INVALID, "sequence %d: page table must be non-null and 4-byte aligned", s);
        if (q.n_pages <= 0 || q.pos < 0 ||
            static_cast<int64_t>(q.n_pages) * pool->page_rows <= q.pos)
            return set_error(TLE_ERR_INVALID,
                             "sequence %d: need 0 <= pos < n_pages * page_rows (pos=%d, n_pages=%d)", s,
                             q.pos, q.n_pages);
        recs[s].key_cache = const_cast<float*>(reinterpret_cast<const float*>(q.pages));
        recs[s].value_cache = nullptr;
        recs[s].n_ctx = q.n_pages;
        recs[s].pos = q.pos;
    }
    return write_desc(recs, n_seqs, max_ctas, tle::kDescMagicPaged, desc_host, desc_bytes,
                      n_ctas_out);
}

size_t tle_decode_workspace_bytes(const tle_shape_t* shape, int n_seqs, int n_ctas) {
    (void)shape;
    if (n_ctas <= 0) n_ctas = tle::kMaxCtas;
    return partial_bytes(n_ctas + std::max(n_seqs, 0));
}

int tle_decode_batch(const tle_shape_t* shape, const void* desc_dev, int n_seqs, int n_ctas,
                     const float* q, const float* k, const float* v, float* out, int layer, int flags,
                     void* workspace, size_t workspace_bytes, void* stream) {
    tle::DecodeArgs a;
    if (int rc = batch_args(shape, desc_dev, n_seqs, n_ctas, q, k, v, out, layer, flags, workspace,
                            workspace_bytes, a))
        return rc;
    cudaError_t e = tle::launch_decode(a, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_error(e, "decode launch");
    return ok();
}

int tle_decode_batch_short(const tle_shape_t* shape, const void* desc_dev, int n_seqs, int max_rows,
                           const float* q, const float* k, const float* v, float* out, int layer,
                           int flags, void* stream) {
    if (int rc = check_shape(shape)) return rc;
    if (!desc_dev || !q || !k || !v || !out) return set_error(TLE_ERR_INVALID, "null pointer");
    if (n_seqs <= 0 || n_seqs > 65535 || max_rows <= 0 || max_rows > tle::kSeqMaxRows || layer < 0 ||
        layer >= shape->n_layers)
        return set_error(TLE_ERR_INVALID, "n_seqs %d, max_rows %d (<= %d), layer %d", n_seqs, max_rows,
                         tle::kSeqMaxRows, layer);
    if (flags & ~(TLE_DECODE_ROTATE | TLE_DECODE_KV_READY))
        return set_error(TLE_ERR_INVALID, "unknown flags 0x%x", flags);
    tle::SeqArgs s{};
    const int chunks = std::min(tle::kSeqMaxChunks, (max_rows + 31) / 32);
    s.chunk_rows = ((max_rows + chunks - 1) / chunks + 31) / 32 * 32;
    s.n_chunks = (max_rows + s.chunk_rows - 1) / s.chunk_rows;
    s.seqs = reinterpret_cast<const tle_seq_t*>(static_cast<const unsigned char*>(desc_dev) +
                                                sizeof(tle::DescHeader));
    s.n_seqs = n_seqs;
    s.q = q;
    s.k = k;
    s.v = v;
    s.out = out;
    s.layer = layer;
    s.rotate = (flags & TLE_DECODE_ROTATE) != 0;
    s.kv_ready = (flags & TLE_DECODE_KV_READY) != 0;
    fill_inv_freq(s.inv_freq, tle::kHeadDim / 2, shape->rope_freq_base);
    cudaError_t e = tle::error_word(&s.err);
    if (e != cudaSuccess) return cuda_error(e, "device error word");
    e = tle::launch_seq_decode(s, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_error(e, "short batch decode launch");
    return ok();
}

size_t tle_decode_bf16_workspace_bytes(int n_seqs, int max_rows) {
    if (n_seqs <= 0 || max_rows <= 0) return 0;
    return tle::decode_bf16_workspace_bytes(n_seqs, max_rows);
}

}  // extern "C"

namespace {

// Checks and fills the arguments shared by the contiguous and paged bf16 calls.
int bf16_args(const tle_shape_t* shape, const void* seqs_dev, int n_seqs, int max_rows, const float* q,
              const float* k, const float* v, float* out, int layer, int flags, void* workspace,
              size_t workspace_bytes, tle::BfArgs& a) {
    if (int rc = check_shape(shape)) return rc;
    if (!seqs_dev || !q || !k || !v || !out) return set_error(TLE_ERR_INVALID, "null pointer");
    if (n_seqs <= 0 || n_seqs > 65535 || max_rows <= 0 || layer < 0 || layer >= shape->n_layers)
        return set_error(TLE_ERR_INVALID, "n_seqs %d, max_rows %d, layer %d", n_seqs, max_rows, layer);
    if (flags & ~TLE_DECODE_ROTATE) return set_error(TLE_ERR_INVALID, "unknown flags 0x%x", flags);
    const size_t need = tle::decode_bf16_workspace_bytes(n_seqs, max_rows);
    const int chunk = tle::bf16_chunk_rows(n_seqs, max_rows);
    const int max_chunks = (max_rows + chunk - 1) / chunk;
    if (max_chunks > 1 && (!workspace || workspace_bytes < need))
        return set_error(TLE_ERR_INVALID, "workspace %zu bytes, need %zu", workspace_bytes, need);
    a = tle::BfArgs{};
    a.n_seqs = n_seqs;
    a.chunk = chunk;
    a.max_chunks = max_chunks;
    a.q = q;
    a.k = k;
    a.v = v;
    a.out = out;
    a.parts = static_cast<float*>(workspace);
    a.lses = a.parts ? a.parts + static_cast<size_t>(n_seqs) * max_chunks * tle::kNHead * tle::kHeadDim : nullptr;
    a.layer = layer;
    a.rotate = (flags & TLE_DECODE_ROTATE) != 0;
    fill_inv_freq(a.inv_freq, tle::kHeadDim / 2, shape->rope_freq_base);
    cudaError_t e = tle::error_word(&a.err);
    if (e != cudaSuccess) return cuda_error(e, "device error word");
    return 0;
}

}  // namespace

extern "C" {

int tle_decode_batch_bf16(const tle_shape_t* shape, const tle_seq_bf16_t* seqs_dev, int n_seqs,
                          int max_rows, const float* q, const float* k, const float* v, float* out,
                          int layer, int flags, void* workspace, size_t workspace_bytes, void* stream) {
    tle::BfArgs a;
    if (int rc = bf16_args(shape, seqs_dev, n_seqs, max_rows, q, k, v, out, layer, flags, workspace,
                           workspace_bytes, a))
        return rc;
    a.seqs = seqs_dev;
    cudaError_t e = tle::launch_decode_bf16(a, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_error(e, "bf16 decode launch");
    return ok();
}

int tle_decode_batch_bf16_paged(const tle_shape_t* shape, const tle_page_pool_bf16_t* pool,
                                const tle_paged_seq_t* seqs_dev, int n_seqs, int max_rows, const float* q,
                                const float* k, const float* v, float* out, int layer, int flags,
                                void* workspace, size_t workspace_bytes, void* stream) {
    tle::BfArgs a;
    if (int rc = bf16_args(shape, seqs_dev, n_seqs, max_rows, q, k, v, out, layer, flags, workspace,
                           workspace_bytes, a))
        return rc;
    if (!pool || !pool->key_pool || !pool->value_pool)
        return set_error(TLE_ERR_INVALID, "page pool and both pools must be non-null");
    if (!aligned16(pool->key_pool) || !aligned16(pool->value_pool))
        return set_error(TLE_ERR_INVALID, "page pools must be 16-byte aligned");
    const int pr = pool->page_rows;
    if (pr < 64 || pr > 65536 || (pr & (pr - 1)) != 0)
        return set_error(TLE_ERR_INVALID, "page_rows %d is not a power of two in [64, 65536]", pr);
    if (pool->n_pages <= 0) return set_error(TLE_ERR_INVALID, "pool n_pages %d <= 0", pool->n_pages);
    int shift = 0;
    while ((1 << shift) < pr) ++shift;
    a.pseqs = seqs_dev;
    a.key_pool = pool->key_pool;
    a.value_pool = pool->value_pool;
    a.pool_pages = pool->n_pages;
    a.page_shift = shift;
    cudaError_t e = tle::launch_decode_bf16(a, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_error(e, "paged bf16 decode launch");
    return ok();
}

int tle_decode_batch_paged(const tle_shape_t* shape, const tle_page_pool_t* pool,
                           const void* desc_dev, int n_seqs, int n_ctas, const float* q,
                           const float* k, const float* v, float* out, int layer, int flags,
                           void* workspace, size_t workspace_bytes, void* stream) {
    tle::DecodeArgs a;
    if (int rc = batch_args(shape, desc_dev, n_seqs, n_ctas, q, k, v, out, layer, flags, workspace,
                            workspace_bytes, a))
        return rc;
    int shift = 0;
    if (int rc = check_pool(shape, pool, &shift)) return rc;
    a.key_pool = pool->key_pool;
    a.value_pool = pool->value_pool;
    a.pool_pages = pool->n_pages;
    a.page_shift = shift;
    cudaError_t e = tle::launch_decode(a, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_error(e, "paged decode launch");
    return ok();
}

size_t tle_prefill_workspace_bytes(const tle_shape_t* shape, int n_tokens, int pos0) {
    (void)shape;
    return tle::prefill_workspace_bytes(n_tokens, pos0);
}

int tle_prefill(float* out, const float* q, const float* k, const float* v, float* key_cache,
                float* value_cache, int layer, int pos0, int n_tokens, int n_ctx,
                const tle_shape_t* shape, void* workspace, size_t workspace_bytes, void* stream) {
    if (int rc = check_shape(shape)) return rc;
    if (!out || !q || !k || !v || !key_cache || !value_cache)
        return set_error(TLE_ERR_INVALID, "null buffer pointer");
    if (!aligned16(out) || !aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(key_cache) ||
        !aligned16(value_cache))
        return set_error(TLE_ERR_INVALID, "buffers must be 16-byte aligned");
    if (n_tokens <= 0 || pos0 < 0 || static_cast<int64_t>(pos0) + n_tokens > n_ctx)
        return set_error(TLE_ERR_INVALID, "need n_tokens > 0 and pos0 + n_tokens <= n_ctx");
    if (layer < 0 || layer >= shape->n_layers)
        return set_error(TLE_ERR_INVALID, "layer %d outside [0, %d)", layer, shape->n_layers);
    const size_t need = tle::prefill_workspace_bytes(n_tokens, pos0);
    if (!workspace || workspace_bytes < need)
        return set_error(TLE_ERR_WORKSPACE, "workspace %zu bytes < %zu needed", workspace_bytes, need);
    if ((reinterpret_cast<uintptr_t>(workspace) & 1023u) != 0)
        return set_error(TLE_ERR_INVALID, "prefill workspace must be 1024-byte aligned");
    tle::PrefillArgs a{};
    a.q = q;
    a.k = k;
    a.v = v;
    a.out = out;
    a.key_cache = key_cache;
    a.value_cache = value_cache;
    a.layer = layer;
    a.pos0 = pos0;
    a.n_tokens = n_tokens;
    a.n_ctx = n_ctx;
    a.workspace = workspace;
    fill_inv_freq(a.inv_freq, tle::kHeadDim / 2, shape->rope_freq_base);
    cudaError_t e = tle::error_word(&a.err);
    if (e != cudaSuccess) return cuda_error(e, "device error word");
    e = tle::launch_prefill(a, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_error(e, "prefill launch");
    return ok();
}

int tle_partition_lpt(const int32_t* lengths, int n_seqs, int n_ranks, int32_t* rank_of_seq) {
    if (n_seqs < 0 || n_ranks <= 0 || (n_seqs > 0 && (!lengths || !rank_of_seq)))
        return set_error(TLE_ERR_INVALID, "bad partition arguments");
    std::vector<int> order(static_cast<size_t>(n_seqs));
    std::iota(order.begin(), order.end(), 0);
    // Longest first; equal lengths keep sequence order.
    std::stable_sort(order.begin(), order.end(),
                     [&](int a, int b) { return lengths[a] > lengths[b]; });
    std::vector<int64_t> load(static_cast<size_t>(n_ranks), 0);
    for (int s : order) {
        int best = 0;
        for (int r = 1; r < n_ranks; ++r)
            if (load[r] < load[best]) best = r;
        rank_of_seq[s] = best;
        load[best] += lengths[s];
    }
    return ok();
}

int tle_device_error(int clear, uint32_t* code) {
    if (!code) return set_error(TLE_ERR_INVALID, "code is NULL");
    cudaError_t e = tle::read_device_error(clear, code);
    if (e != cudaSuccess) return cuda_error(e, "device error read");
    return ok();
}

int tle_selftest_wait_timeout(uint32_t limit_us, void* stream) {
    if (limit_us < 1 || limit_us > 1000000)
        return set_error(TLE_ERR_INVALID, "limit_us %u outside [1, 1000000]", limit_us);
    uint32_t* err = nullptr;
    cudaError_t e = tle::error_word(&err);
    if (e != cudaSuccess) return cuda_error(e, "error word");
    e = tle::launch_selftest_wait(err, static_cast<uint64_t>(limit_us) * 1000u,
                                  static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_error(e, "selftest launch");
    return ok();
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Decode without allocation (tle_decode_batch_noalloc).
//
// For callers that cannot call cudaMalloc -- a host framework that owns all
// device memory through its own pool, or a per-token loop that must not pay
// cudaMalloc/cudaFree's implicit device synchronisation.  Its scratch (the
// batch descriptor and the split-K partials) lives in this fixed-size
// file-scope device array, which every GPU that loads the library keeps until
// the process exits.
// ---------------------------------------------------------------------------
namespace {

constexpr int kNoAllocMaxSeqs = TLE_NOALLOC_MAX_SEQS;
constexpr int kNoAllocMaxCtas = 256;
constexpr size_t kNoAllocDescBytes = 32768;
constexpr size_t kNoAllocPartialBytes =
    static_cast<size_t>(kNoAllocMaxSeqs + kNoAllocMaxCtas) * tle::kPartialFloats * sizeof(float);
constexpr size_t kNoAllocBytes = kNoAllocDescBytes + kNoAllocPartialBytes;
static_assert(sizeof(tle::DescHeader) + sizeof(tle_seq_t) * kNoAllocMaxSeqs +
                      sizeof(tle::CtaStart) * (kNoAllocMaxCtas + 1) +
                      (sizeof(tle::SeqCtas) + sizeof(int32_t)) * kNoAllocMaxSeqs <=
                  kNoAllocDescBytes,
              "descriptor region too small");
constexpr int kNoAllocMaxDevices = 64;

std::mutex g_noalloc_mu;
unsigned char* g_noalloc_ptr[kNoAllocMaxDevices] = {};

// Host staging for the descriptor: fixed size, per host thread, no malloc.
thread_local unsigned char t_noalloc_desc[kNoAllocDescBytes];

}  // namespace

// The scratch itself.  In host code this name is only a stand-in for the
// symbol: its device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_tle_noalloc_scratch[kNoAllocBytes];

namespace {

// Device address of the scratch on the current device; looked up once per
// device (the first call on a device) and cached.
int noalloc_scratch(unsigned char** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_error(e, "cudaGetDevice");
    if (dev < 0 || dev >= kNoAllocMaxDevices)
        return set_error(TLE_ERR_UNSUPPORTED, "device %d beyond the no-allocation table", dev);
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_tle_noalloc_scratch);
        if (e != cudaSuccess) return cuda_error(e, "cudaGetSymbolAddress(no-allocation scratch)");
        g_noalloc_ptr[dev] = static_cast<unsigned char*>(p);
    }
    *out = g_noalloc_ptr[dev];
    return TLE_OK;
}

// The descriptor of tle_decode_desc, written into a caller-provided buffer
// (plan_ctas allocates nothing).
void fill_desc_noalloc(const tle_seq_t* seqs, int n_seqs, int G, int64_t total, unsigned char* base) {
    tle::DescHeader hdr{};
    hdr.magic = tle::kDescMagic;
    hdr.n_seqs = n_seqs;
    hdr.n_ctas = G;
    hdr.total_rows = total;
    std::memcpy(base, &hdr, sizeof hdr);
    std::memcpy(base + tle::desc_seqs_offset(), seqs, sizeof(tle_seq_t) * static_cast<size_t>(n_seqs));
    auto* cs = reinterpret_cast<tle::CtaStart*>(base + tle::desc_cta_offset(n_seqs));
    auto* sc = reinterpret_cast<tle::SeqCtas*>(base + tle::desc_seqctas_offset(n_seqs, G));
    plan_ctas(seqs, n_seqs, G, cs, sc);
    std::memset(base + tle::desc_arrivals_offset(n_seqs, G), 0, sizeof(int32_t) * static_cast<size_t>(n_seqs));
}

}  // namespace

extern "C" int tle_decode_batch_noalloc(const tle_shape_t* shape, const tle_seq_t* seqs, int n_seqs,
                                        const float* q, const float* k, const float* v, float* out,
                                        int layer, int rotate, void* stream) {
    if (int rc = check_shape(shape)) return rc;
    if (!seqs || !q || !k || !v || !out) return set_error(TLE_ERR_INVALID, "null pointer argument");
    if (n_seqs <= 0) return set_error(TLE_ERR_INVALID, "n_seqs must be > 0");
    if (n_seqs > kNoAllocMaxSeqs)
        return set_error(TLE_ERR_INVALID,
                         "n_seqs=%d exceeds the no-allocation scratch limit of %d sequences "
                         "(TLE_NOALLOC_MAX_SEQS); use tle_decode_batch with a workspace",
                         n_seqs, kNoAllocMaxSeqs);
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out))
        return set_error(TLE_ERR_INVALID, "buffers must be 16-byte aligned");
    if (layer < 0 || layer >= shape->n_layers)
        return set_error(TLE_ERR_INVALID, "layer %d outside [0, %d)", layer, shape->n_layers);
    int64_t total = 0;
    for (int s = 0; s < n_seqs; ++s) {
        const tle_seq_t& r = seqs[s];
        if (!r.key_cache || !r.value_cache || !aligned16(r.key_cache) || !aligned16(r.value_cache))
            return set_error(TLE_ERR_INVALID, "sequence %d: caches must be non-null and 16-byte aligned", s);
        if (r.n_ctx <= 0 || r.pos < 0 || r.pos >= r.n_ctx)
            return set_error(TLE_ERR_INVALID, "sequence %d: need 0 <= pos < n_ctx (pos=%d, n_ctx=%d)", s,
                             r.pos, r.n_ctx);
        total += static_cast<int64_t>(r.pos) + 1;
    }
    unsigned char* scratch = nullptr;
    if (int rc = noalloc_scratch(&scratch)) return rc;
    const int G = choose_ctas(total, std::min(sm_count(), kNoAllocMaxCtas));
    fill_desc_noalloc(seqs, n_seqs, G, total, t_noalloc_desc);
    const size_t desc_bytes = tle::desc_total_bytes(n_seqs, G);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // Pageable source: the copy is staged before this call returns, so the
    // host buffer may be refilled by the next call.
    cudaError_t e = cudaMemcpyAsync(scratch, t_noalloc_desc, desc_bytes, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return cuda_error(e, "descriptor upload");
    tle::DecodeArgs a{};
    a.seqs = reinterpret_cast<const tle_seq_t*>(scratch + tle::desc_seqs_offset());
    a.cta_start = reinterpret_cast<const tle::CtaStart*>(scratch + tle::desc_cta_offset(n_seqs));
    a.seq_ctas = reinterpret_cast<const tle::SeqCtas*>(scratch + tle::desc_seqctas_offset(n_seqs, G));
    a.arrivals = reinterpret_cast<int32_t*>(scratch + tle::desc_arrivals_offset(n_seqs, G));
    a.n_seqs = n_seqs;
    a.n_ctas = G;
    a.q = q;
    a.k = k;
    a.v = v;
    a.out = out;
    a.partials = reinterpret_cast<float*>(scratch + kNoAllocDescBytes);
    a.layer = layer;
    a.rotate = rotate ? 1 : 0;
    fill_inv_freq(a.inv_freq, tle::kHeadDim / 2, shape->rope_freq_base);
    e = tle::error_word(&a.err);
    if (e != cudaSuccess) return cuda_error(e, "device error word");
    e = tle::launch_decode(a, st);
    if (e != cudaSuccess) return cuda_error(e, "decode launch");
    return ok();
}

// ===================== forward pass around attention (tle_forward.h) =====================

namespace {

int check_weight(const void* W, int type, int cols, int* row_bytes, const char* what) {
    if (!W || !aligned16(W)) return set_error(TLE_ERR_INVALID, "%s: weights must be non-null and 16-byte aligned", what);
    if (cols <= 0 || cols > tle::kGemvMaxCols)
        return set_error(TLE_ERR_UNSUPPORTED, "%s: cols %d outside [1, %d]", what, cols, tle::kGemvMaxCols);
    const int rb = tle::weight_row_bytes(type, cols);
    if (rb < 0) return set_error(TLE_ERR_UNSUPPORTED, "%s: weight type %d with %d cols is not supported", what, type, cols);
    *row_bytes = rb;
    return 0;
}

// Rows per warp: enough CTAs for two per SM on small matrices, fewer and
// longer CTAs on big ones (the LM head), where each CTA's input staging
// (and RMSNorm) is amortised over more rows.
int rows_per_warp(int rows) {
    const int per = rows / (2 * std::max(sm_count(), 1) * 8);
    return std::max(1, std::min(8, per));
}

int gemv(int type, int epi, const tle::GemvSeg* segs, int n_seg, const uint8_t* W2, int cols,
         const float* x, const float* norm_w, float eps, cudaStream_t st, const char* what) {
    int rb = 0;
    if (int rc = check_weight(segs[0].W, type, cols, &rb, what)) return rc;
    tle::GemvArgs a{};
    int rows = 0;
    for (int i = 0; i < n_seg; ++i) {
        a.seg[i] = segs[i];
        rows += segs[i].rows;
    }
    a.n_seg = n_seg;
    a.W2 = W2;
    a.cols = cols;
    a.row_bytes = rb;
    a.rpw = rows_per_warp(rows);
    a.x = x;
    a.norm_w = norm_w;
    a.eps = eps;
    cudaError_t e = tle::launch_gemv(type, epi, a, st);
    if (e != cudaSuccess) return cuda_error(e, what);
    return 0;
}

}  // namespace

extern "C" {

int tle_matmul(float* out, const void* W, const float* x, int rows, int cols, int type, void* stream) {
    if (!out || !x) return set_error(TLE_ERR_INVALID, "null pointer argument");
    if (rows <= 0) return set_error(TLE_ERR_INVALID, "rows %d <= 0", rows);
    tle::GemvSeg seg{static_cast<const uint8_t*>(W), out, rows, 0};
    if (int rc = gemv(type, tle::kEpiStore, &seg, 1, nullptr, cols, x, nullptr, 0.f,
                      static_cast<cudaStream_t>(stream), "matmul"))
        return rc;
    return ok();
}

int tle_rmsnorm(float* out, const float* x, const float* weight, int size, float eps, void* stream) {
    if (!out || !x || !weight) return set_error(TLE_ERR_INVALID, "null pointer argument");
    if (size <= 0) return set_error(TLE_ERR_INVALID, "size %d <= 0", size);
    cudaError_t e = tle::launch_rmsnorm(out, x, weight, size, eps, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_error(e, "rmsnorm");
    return ok();
}

int tle_vec_add(float* out, const float* x, int size, void* stream) {
    if (!out || !x) return set_error(TLE_ERR_INVALID, "null pointer argument");
    if (size <= 0) return set_error(TLE_ERR_INVALID, "size %d <= 0", size);
    cudaError_t e = tle::launch_vec_add(out, x, size, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_error(e, "vec_add");
    return ok();
}

int tle_ffn_swiglu(float* out, const float* input, float* hb, float* hb2, const void* W_gate,
                   const void* W_up, const void* W_down, int n_ff, int n_embd, int type,
                   void* stream) {
    (void)hb2;
    if (!out || !input || !hb || !W_up) return set_error(TLE_ERR_INVALID, "null pointer argument");
    if (n_ff <= 0 || n_embd <= 0) return set_error(TLE_ERR_INVALID, "bad n_ff/n_embd (%d, %d)", n_ff, n_embd);
    int rb = 0;
    if (int rc = check_weight(W_up, type, n_embd, &rb, "ffn_up")) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    tle::GemvSeg g{static_cast<const uint8_t*>(W_gate), hb, n_ff, 0};
    if (int rc = gemv(type, tle::kEpiSwiGLU, &g, 1, static_cast<const uint8_t*>(W_up), n_embd, input,
                      nullptr, 0.f, st, "ffn_gate/up"))
        return rc;
    tle::GemvSeg d{static_cast<const uint8_t*>(W_down), out, n_embd, 0};
    if (int rc = gemv(type, tle::kEpiStore, &d, 1, nullptr, n_ff, hb, nullptr, 0.f, st, "ffn_down"))
        return rc;
    return ok();
}

int tle_sample_argmax(const float* logits, int n_vocab, int32_t* token, void* stream) {
    if (!logits || !token) return set_error(TLE_ERR_INVALID, "null pointer argument");
    if (n_vocab <= 0) return set_error(TLE_ERR_INVALID, "n_vocab %d <= 0", n_vocab);
    cudaError_t e = tle::launch_argmax(logits, n_vocab, token, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_error(e, "argmax");
    return ok();
}

}  // extern "C"

namespace {
int sample_common(float* logits, int n_vocab, float temperature, float top_p, float r, bool use_top_p,
                  int32_t* token, void* stream) {
    if (!logits || !token) return set_error(TLE_ERR_INVALID, "null pointer argument");
    if (n_vocab <= 0 || n_vocab > tle::kSampleMaxVocab)
        return set_error(TLE_ERR_UNSUPPORTED, "n_vocab %d outside [1, %d]", n_vocab, tle::kSampleMaxVocab);
    if (!(r >= 0.0f && r < 1.0f)) return set_error(TLE_ERR_INVALID, "r must be in [0, 1)");
    cudaError_t e = tle::launch_sample(logits, n_vocab, temperature, top_p, r, use_top_p, token,
                                       static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_error(e, "sample");
    return ok();
}
}  // namespace

extern "C" {

int tle_sample_temperature(float* logits, int n_vocab, float temperature, float r, int32_t* token,
                           void* stream) {
    return sample_common(logits, n_vocab, temperature, 1.0f, r, false, token, stream);
}

int tle_sample_top_p(float* logits, int n_vocab, float temperature, float top_p, float r,
                     int32_t* token, void* stream) {
    return sample_common(logits, n_vocab, temperature, top_p, r, true, token, stream);
}

}  // extern "C"

namespace {

// Every layer of the token in one persistent cooperative launch, when the
// model allows it: all linear weights Q4_0 (16-byte aligned), at most
// kPersistMaxLayers layers, widths that are multiples of 256, the attention
// of pos + 1 rows in at most SMs / 4 chunks of 64 rows per KV head, the
// workspace large enough, cooperative launch supported.  Otherwise *used
// stays false and the caller launches product by product.
bool persist_plan(const tle_model_t* m, const tle_state_t* s, int pos, int* grid, size_t* smem, int* chunks,
                  tle::PersistArgs* a) {
    if (m->n_layers > tle::kPersistMaxLayers) return false;
    for (int l = 0; l < m->n_layers; ++l) {
        const tle_layer_t& L = m->layers[l];
        const tle_weight_t* w[7] = {&L.attn_q, &L.attn_k, &L.attn_v, &L.attn_output, &L.ffn_gate, &L.ffn_up,
                                    &L.ffn_down};
        for (const tle_weight_t* x : w)
            if (x->type != TLE_W_Q4_0 || !x->data || !aligned16(x->data)) return false;
        if (!L.attn_norm || !L.ffn_norm) return false;
    }
    int dev = 0, coop = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev) != cudaSuccess || !coop)
        return false;
    *grid = sm_count();
    *smem = tle::persist_smem_bytes(m->n_embd, m->n_ff, *grid, a);
    if (!*smem) return false;
    *chunks = (pos + 1 + tle::kPersistAttRows - 1) / tle::kPersistAttRows;
    if (*chunks > tle::persist_max_chunks(*grid)) return false;
    return s->workspace && s->workspace_bytes >= tle::persist_workspace_bytes(*grid) &&
           (reinterpret_cast<uintptr_t>(s->workspace) & 255u) == 0;
}

int forward_layers_persistent(const tle_model_t* m, const tle_state_t* s, int pos, uint32_t* err,
                              cudaStream_t st, bool* used) {
    *used = false;
    int grid = 0, chunks = 0;
    size_t smem = 0;
    tle::PersistArgs a{};
    if (!persist_plan(m, s, pos, &grid, &smem, &chunks, &a)) return 0;
    for (int l = 0; l < m->n_layers; ++l) {
        const tle_layer_t& Ly = m->layers[l];
        const tle_weight_t* w[7] = {&Ly.attn_q, &Ly.attn_k, &Ly.attn_v, &Ly.attn_output, &Ly.ffn_gate, &Ly.ffn_up,
                                    &Ly.ffn_down};
        for (int i = 0; i < 7; ++i) a.layer[l].w[i] = static_cast<const uint8_t*>(w[i]->data);
        a.layer[l].attn_norm = Ly.attn_norm;
        a.layer[l].ffn_norm = Ly.ffn_norm;
    }
    a.n_layers = m->n_layers;
    a.n_embd = m->n_embd;
    a.n_ff = m->n_ff;
    a.n_ctx = m->n_ctx;
    a.pos = pos;
    a.eps = m->rms_norm_eps;
    a.x = s->x;
    a.q = s->q;
    a.k = s->k;
    a.v = s->v;
    a.hb = s->hb;
    a.key_cache = s->key_cache;
    a.value_cache = s->value_cache;
    a.sync = static_cast<uint32_t*>(s->workspace);
    a.partials = reinterpret_cast<float*>(static_cast<unsigned char*>(s->workspace) + 256);
    a.err = err;
    a.att_chunks = chunks;
    fill_inv_freq(a.inv_freq, tle::kHeadDim / 2, m->rope_freq_base);
    cudaError_t e = cudaMemsetAsync(a.sync, 0, sizeof(uint32_t), st);   // the barrier count
    if (e != cudaSuccess) return cuda_error(e, "persistent forward: barrier count");
    e = tle::launch_forward_persistent(a, grid, smem, st);
    if (e == cudaErrorCooperativeLaunchTooLarge) {   // SMs held elsewhere: product by product
        (void)cudaGetLastError();
        return 0;
    }
    if (e != cudaSuccess) return cuda_error(e, "persistent forward launch");
    *used = true;
    return 0;
}

}  // namespace

extern "C" {

int tle_forward_layers_one_launch(const tle_model_t* m, const tle_state_t* s, int pos) {
    if (!m || !s || pos < 0 || pos >= m->n_ctx) return 0;
    int grid = 0, chunks = 0;
    size_t smem = 0;
    tle::PersistArgs a{};
    return persist_plan(m, s, pos, &grid, &smem, &chunks, &a) ? 1 : 0;
}

size_t tle_forward_workspace_bytes(const tle_model_t* model) {
    if (!model || model->n_ctx <= 0) return 0;
    return std::max(partial_bytes(tle::kMaxCtas + 1), tle::persist_workspace_bytes(tle::kMaxCtas));
}

int tle_forward(const tle_model_t* m, const tle_state_t* s, const int32_t* token, int pos, void* stream) {
    if (!m || !s || !token) return set_error(TLE_ERR_INVALID, "null model/state/token");
    if (!m->layers || m->n_layers <= 0) return set_error(TLE_ERR_INVALID, "model has no layers");
    tle_shape_t shape{m->n_layers, m->n_head, m->n_head_kv,
                      m->n_head > 0 ? m->n_embd / m->n_head : 0, m->rope_freq_base};
    if (int rc = check_shape(&shape)) return rc;
    if (m->n_embd != m->n_head * shape.head_dim)
        return set_error(TLE_ERR_UNSUPPORTED, "n_embd %d != n_head * 64", m->n_embd);
    if (pos < 0 || pos >= m->n_ctx) return set_error(TLE_ERR_INVALID, "need 0 <= pos < n_ctx (pos=%d)", pos);
    if (m->n_vocab <= 0 || m->n_ff <= 0) return set_error(TLE_ERR_INVALID, "bad n_vocab/n_ff");
    if (!s->x || !s->xb2 || !s->q || !s->k || !s->v || !s->hb || !s->logits || !s->key_cache ||
        !s->value_cache)
        return set_error(TLE_ERR_INVALID, "null state buffer");
    if (m->token_embd.type != TLE_W_F16 && m->token_embd.type != TLE_W_F32)
        return set_error(TLE_ERR_UNSUPPORTED, "token_embd type %d (F16 or F32 supported)", m->token_embd.type);
    if (!m->token_embd.data || !m->output_norm) return set_error(TLE_ERR_INVALID, "null global tensor");
    const int n_embd = m->n_embd, kv_dim = m->n_head_kv * shape.head_dim, n_ff = m->n_ff;
    const float eps = m->rms_norm_eps;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    uint32_t* err = nullptr;
    cudaError_t e = tle::error_word(&err);
    if (e != cudaSuccess) return cuda_error(e, "device error word");

    e = tle::launch_embed(m->token_embd.type, s->x, m->token_embd.data, token, m->n_vocab, n_embd, err, st);
    if (e != cudaSuccess) return cuda_error(e, "embedding");
    bool persistent = false;
    if (int rc = forward_layers_persistent(m, s, pos, err, st, &persistent)) return rc;
    for (int l = 0; !persistent && l < m->n_layers; ++l) {
        const tle_layer_t& L = m->layers[l];
        if (!L.attn_norm || !L.ffn_norm) return set_error(TLE_ERR_INVALID, "layer %d: null norm weight", l);
        // rmsnorm + q, k, v (forward.cpp:184-196): one launch when the three share a format
        tle::GemvSeg qkv[3] = {{static_cast<const uint8_t*>(L.attn_q.data), s->q, n_embd, 0},
                               {static_cast<const uint8_t*>(L.attn_k.data), s->k, kv_dim, 0},
                               {static_cast<const uint8_t*>(L.attn_v.data), s->v, kv_dim, 0}};
        if (L.attn_q.type == L.attn_k.type && L.attn_q.type == L.attn_v.type) {
            int rb = 0;
            if (int rc = check_weight(L.attn_k.data, L.attn_k.type, n_embd, &rb, "attn_k")) return rc;
            if (int rc = check_weight(L.attn_v.data, L.attn_v.type, n_embd, &rb, "attn_v")) return rc;
            if (int rc = gemv(L.attn_q.type, tle::kEpiStore, qkv, 3, nullptr, n_embd, s->x, L.attn_norm,
                              eps, st, "attn_qkv"))
                return rc;
        } else {
            const tle_weight_t* w[3] = {&L.attn_q, &L.attn_k, &L.attn_v};
            for (int i = 0; i < 3; ++i)
                if (int rc = gemv(w[i]->type, tle::kEpiStore, &qkv[i], 1, nullptr, n_embd, s->x,
                                  L.attn_norm, eps, st, "attn_q/k/v"))
                    return rc;
        }
        // rope + attention (forward.cpp:198-208), appending row pos
        if (int rc = single_decode(s->xb2, s->q, s->k, s->v, s->key_cache, s->value_cache, l, pos,
                                   m->n_ctx, &shape, s->workspace, s->workspace_bytes, stream, 1))
            return rc;
        // output projection + residual (forward.cpp:210-214)
        tle::GemvSeg wo{static_cast<const uint8_t*>(L.attn_output.data), s->x, n_embd, 0};
        if (int rc = gemv(L.attn_output.type, tle::kEpiAdd, &wo, 1, nullptr, n_embd, s->xb2, nullptr,
                          0.f, st, "attn_output"))
            return rc;
        // rmsnorm + SwiGLU (forward.cpp:216-227; all three read as the gate's type)
        int rb = 0;
        if (int rc = check_weight(L.ffn_up.data, L.ffn_gate.type, n_embd, &rb, "ffn_up")) return rc;
        tle::GemvSeg gate{static_cast<const uint8_t*>(L.ffn_gate.data), s->hb, n_ff, 0};
        if (int rc = gemv(L.ffn_gate.type, tle::kEpiSwiGLU, &gate, 1,
                          static_cast<const uint8_t*>(L.ffn_up.data), n_embd, s->x, L.ffn_norm, eps, st,
                          "ffn_gate/up"))
            return rc;
        // down projection + residual (forward.cpp:227-229)
        tle::GemvSeg down{static_cast<const uint8_t*>(L.ffn_down.data), s->x, n_embd, 0};
        if (int rc = gemv(L.ffn_gate.type, tle::kEpiAdd, &down, 1, nullptr, n_ff, s->hb, nullptr, 0.f, st,
                          "ffn_down"))
            return rc;
    }
    // final rmsnorm + LM head (forward.cpp:245-265)
    const tle_weight_t& head = m->output.data ? m->output : m->token_embd;
    tle::GemvSeg lm{static_cast<const uint8_t*>(head.data), s->logits, m->n_vocab, 0};
    if (int rc = gemv(head.type, tle::kEpiStore, &lm, 1, nullptr, n_embd, s->x, m->output_norm, eps, st,
                      "lm_head"))
        return rc;
    return ok();
}

}  // extern "C"

// ===================== batched prompt (tle_forward.h) =====================

namespace {

constexpr size_t kSegAlign = 1024;
size_t align_up(size_t n) { return (n + kSegAlign - 1) / kSegAlign * kSegAlign; }

// Element offsets (fp16) of one layer's weights in the packed copy.
struct PackedLayer {
    size_t qkv, o, gu, down, total;
};
PackedLayer packed_layer(const tle_model_t* m) {
    const size_t e = static_cast<size_t>(m->n_embd), kv = static_cast<size_t>(m->n_head_kv) * tle::kHeadDim,
                 ff = static_cast<size_t>(m->n_ff);
    PackedLayer p;
    p.qkv = 0;
    p.o = p.qkv + (e + 2 * kv) * e;
    p.gu = p.o + e * e;
    p.down = p.gu + 2 * ff * e;
    p.total = p.down + e * ff;
    return p;
}

// Byte offsets of tle_prompt_forward's scratch (each segment 1024-aligned).
struct PromptScratch {
    size_t x, q, k, v, att, xb16, att16, h16, attn_ws, total;
    int s_pad;
};
PromptScratch prompt_scratch(const tle_model_t* m, int n_tokens, int pos0) {
    const size_t S = static_cast<size_t>(n_tokens), e = static_cast<size_t>(m->n_embd),
                 kv = static_cast<size_t>(m->n_head_kv) * tle::kHeadDim, ff = static_cast<size_t>(m->n_ff);
    PromptScratch p{};
    p.s_pad = (n_tokens + tle::kGemmTileTokens - 1) / tle::kGemmTileTokens * tle::kGemmTileTokens;
    const size_t sp = static_cast<size_t>(p.s_pad);
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t at = off;
        off += align_up(bytes);
        return at;
    };
    p.x = take(S * e * 4);
    p.q = take(S * e * 4);
    p.k = take(S * kv * 4);
    p.v = take(S * kv * 4);
    p.att = take(S * e * 4);
    p.xb16 = take(sp * e * 2);
    p.att16 = take(sp * e * 2);
    p.h16 = take(sp * ff * 2);
    p.attn_ws = take(tle::prefill_workspace_bytes(n_tokens, pos0));
    p.total = off;
    return p;
}

// The model shapes the batched prompt supports; 0 or a TLE_* error.
int check_prompt_model(const tle_model_t* m) {
    if (!m) return set_error(TLE_ERR_INVALID, "model is NULL");
    if (!m->layers || m->n_layers <= 0) return set_error(TLE_ERR_INVALID, "model has no layers");
    tle_shape_t shape{m->n_layers, m->n_head, m->n_head_kv, m->n_head > 0 ? m->n_embd / m->n_head : 0,
                      m->rope_freq_base};
    if (int rc = check_shape(&shape)) return rc;
    if (m->n_embd != m->n_head * tle::kHeadDim)
        return set_error(TLE_ERR_UNSUPPORTED, "n_embd %d != n_head * 64", m->n_embd);
    if (m->n_ff <= 0 || m->n_ff % tle::kGemmTileRows)
        return set_error(TLE_ERR_UNSUPPORTED, "n_ff %d is not a positive multiple of %d", m->n_ff,
                         tle::kGemmTileRows);
    if (m->n_vocab <= 0 || m->n_ctx <= 0) return set_error(TLE_ERR_INVALID, "bad n_vocab/n_ctx");
    const int kv = m->n_head_kv * tle::kHeadDim;
    for (int l = 0; l < m->n_layers; ++l) {
        const tle_layer_t& L = m->layers[l];
        const struct {
            const tle_weight_t* w;
            int type, cols;
            const char* name;
        } ws[7] = {{&L.attn_q, L.attn_q.type, m->n_embd, "attn_q"},
                   {&L.attn_k, L.attn_k.type, m->n_embd, "attn_k"},
                   {&L.attn_v, L.attn_v.type, m->n_embd, "attn_v"},
                   {&L.attn_output, L.attn_output.type, m->n_embd, "attn_output"},
                   {&L.ffn_gate, L.ffn_gate.type, m->n_embd, "ffn_gate"},
                   {&L.ffn_up, L.ffn_gate.type, m->n_embd, "ffn_up"},
                   {&L.ffn_down, L.ffn_gate.type, m->n_ff, "ffn_down"}};
        for (const auto& w : ws) {
            if (!w.w->data) return set_error(TLE_ERR_INVALID, "layer %d: %s is NULL", l, w.name);
            if (tle::weight_row_bytes(w.type, w.cols) < 0)
                return set_error(TLE_ERR_UNSUPPORTED, "layer %d: %s type %d with %d cols is not supported", l,
                                 w.name, w.type, w.cols);
        }
        if (!L.attn_norm || !L.ffn_norm) return set_error(TLE_ERR_INVALID, "layer %d: null norm weight", l);
    }
    (void)kv;
    return 0;
}

}  // namespace

extern "C" {

size_t tle_prompt_weights_bytes(const tle_model_t* model) {
    if (check_prompt_model(model)) return 0;
    return packed_layer(model).total * 2 * static_cast<size_t>(model->n_layers);
}

int tle_prompt_pack_weights(const tle_model_t* m, void* dst, size_t dst_bytes, void* stream) {
    if (int rc = check_prompt_model(m)) return rc;
    if (!dst || !aligned16(dst)) return set_error(TLE_ERR_INVALID, "dst must be non-null and 16-byte aligned");
    const PackedLayer P = packed_layer(m);
    const size_t need = P.total * 2 * static_cast<size_t>(m->n_layers);
    if (dst_bytes < need) return set_error(TLE_ERR_WORKSPACE, "dst %zu bytes < %zu needed", dst_bytes, need);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int e = m->n_embd, kv = m->n_head_kv * tle::kHeadDim, ff = m->n_ff;
    const size_t ee = static_cast<size_t>(e);
    for (int l = 0; l < m->n_layers; ++l) {
        const tle_layer_t& L = m->layers[l];
        uint16_t* base = static_cast<uint16_t*>(dst) + P.total * static_cast<size_t>(l);
        const struct {
            const tle_weight_t* w;
            int type, rows, cols;
            size_t at;
        } parts[7] = {{&L.attn_q, L.attn_q.type, e, e, P.qkv},
                      {&L.attn_k, L.attn_k.type, kv, e, P.qkv + ee * e},
                      {&L.attn_v, L.attn_v.type, kv, e, P.qkv + (ee + kv) * e},
                      {&L.attn_output, L.attn_output.type, e, e, P.o},
                      {&L.ffn_gate, L.ffn_gate.type, ff, e, P.gu},
                      {&L.ffn_up, L.ffn_gate.type, ff, e, P.gu + static_cast<size_t>(ff) * e},
                      {&L.ffn_down, L.ffn_gate.type, e, ff, P.down}};
        for (const auto& p : parts) {
            cudaError_t err = tle::launch_pack_f16(p.type, base + p.at, p.w->data, p.rows, p.cols, st);
            if (err != cudaSuccess) return cuda_error(err, "pack weights");
        }
    }
    return ok();
}

size_t tle_prompt_scratch_bytes(const tle_model_t* model, int n_tokens, int pos0) {
    if (check_prompt_model(model) || n_tokens <= 0 || pos0 < 0) return 0;
    return prompt_scratch(model, n_tokens, pos0).total;
}

namespace {
// K splits of one prompt product: enough CTAs for the SMs when the output
// tiles are few (short prompts).
int gemm_splits(const tle::GemmLaunch& g) {
    const int s_pad = (g.n_tokens + tle::kGemmTileTokens - 1) / tle::kGemmTileTokens;
    return tle::gemm_split_for((g.tile_rows / tle::kGemmTileRows) * s_pad, g.K / tle::kGemmTileK, sm_count());
}
}  // namespace

int tle_prompt_forward(const tle_model_t* m, const void* packed, const tle_state_t* s, const int32_t* tokens,
                       int n_tokens, int pos0, void* scratch, size_t scratch_bytes, void* stream) {
    if (int rc = check_prompt_model(m)) return rc;
    if (!packed || !s || !tokens || !scratch) return set_error(TLE_ERR_INVALID, "null packed/state/tokens/scratch");
    if (!aligned16(packed)) return set_error(TLE_ERR_INVALID, "packed weights must be 16-byte aligned");
    if (n_tokens <= 0 || n_tokens > 65535 || pos0 < 0 || static_cast<int64_t>(pos0) + n_tokens > m->n_ctx)
        return set_error(TLE_ERR_INVALID, "need 0 < n_tokens <= 65535 and 0 <= pos0, pos0 + n_tokens <= n_ctx");
    if (!s->x || !s->logits || !s->key_cache || !s->value_cache) return set_error(TLE_ERR_INVALID, "null state buffer");
    if (!aligned16(s->key_cache) || !aligned16(s->value_cache) || !aligned16(s->x))
        return set_error(TLE_ERR_INVALID, "state buffers must be 16-byte aligned");
    if (m->token_embd.type != TLE_W_F16 && m->token_embd.type != TLE_W_F32)
        return set_error(TLE_ERR_UNSUPPORTED, "token_embd type %d (F16 or F32 supported)", m->token_embd.type);
    if (!m->token_embd.data || !m->output_norm) return set_error(TLE_ERR_INVALID, "null global tensor");
    if ((reinterpret_cast<uintptr_t>(scratch) & (kSegAlign - 1)) != 0)
        return set_error(TLE_ERR_INVALID, "scratch must be 1024-byte aligned");
    const PromptScratch W = prompt_scratch(m, n_tokens, pos0);
    if (scratch_bytes < W.total)
        return set_error(TLE_ERR_WORKSPACE, "scratch %zu bytes < %zu needed", scratch_bytes, W.total);
    const PackedLayer P = packed_layer(m);
    const int e = m->n_embd, kv = m->n_head_kv * tle::kHeadDim, ff = m->n_ff, S = n_tokens;
    const float eps = m->rms_norm_eps;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    unsigned char* ws = static_cast<unsigned char*>(scratch);
    float* X = reinterpret_cast<float*>(ws + W.x);
    float* Q = reinterpret_cast<float*>(ws + W.q);
    float* K = reinterpret_cast<float*>(ws + W.k);
    float* V = reinterpret_cast<float*>(ws + W.v);
    float* ATT = reinterpret_cast<float*>(ws + W.att);
    uint16_t* XB16 = reinterpret_cast<uint16_t*>(ws + W.xb16);
    uint16_t* ATT16 = reinterpret_cast<uint16_t*>(ws + W.att16);
    uint16_t* H16 = reinterpret_cast<uint16_t*>(ws + W.h16);
    uint32_t* err = nullptr;
    cudaError_t ce = tle::error_word(&err);
    if (ce != cudaSuccess) return cuda_error(ce, "device error word");

    ce = tle::launch_embed_rows(m->token_embd.type, X, m->token_embd.data, tokens, S, m->n_vocab, e, err, st);
    if (ce != cudaSuccess) return cuda_error(ce, "embedding");
    for (int l = 0; l < m->n_layers; ++l) {
        const tle_layer_t& L = m->layers[l];
        const uint16_t* Wl = static_cast<const uint16_t*>(packed) + P.total * static_cast<size_t>(l);
        // rmsnorm + q/k/v for all tokens (forward.cpp:184-196)
        ce = tle::launch_rmsnorm_rows_f16(XB16, X, L.attn_norm, e, eps, S, err, st);
        if (ce != cudaSuccess) return cuda_error(ce, "attn_norm");
        tle::GemmLaunch g{};
        g.W = Wl + P.qkv;
        g.w_rows = e + 2 * kv;
        g.X = XB16;
        g.n_tokens = S;
        g.K = e;
        g.tile_rows = g.w_rows;
        g.seg[0] = {0, e, Q};
        g.seg[1] = {e, kv, K};
        g.seg[2] = {e + kv, kv, V};
        g.n_seg = 3;
        g.err = err;
        g.n_split = gemm_splits(g);
        ce = tle::launch_gemm_f16(tle::kEpiStore, g, st);
        if (ce != cudaSuccess) return cuda_error(ce, "attn_qkv");
        // rope + attention of every token (forward.cpp:198-208), appending rows pos0..
        tle::PrefillArgs a{};
        a.q = Q;
        a.k = K;
        a.v = V;
        a.out = ATT;
        a.key_cache = s->key_cache;
        a.value_cache = s->value_cache;
        a.layer = l;
        a.pos0 = pos0;
        a.n_tokens = S;
        a.n_ctx = m->n_ctx;
        a.workspace = ws + W.attn_ws;
        a.err = err;
        a.f16 = 1;   // fp16 operands: the errors of one layer's attention feed the next layer
        fill_inv_freq(a.inv_freq, tle::kHeadDim / 2, m->rope_freq_base);
        ce = tle::launch_prefill(a, st);
        if (ce != cudaSuccess) return cuda_error(ce, "attention");
        // output projection + residual (forward.cpp:210-214)
        ce = tle::launch_to_f16(ATT16, ATT, static_cast<size_t>(S) * e, err, st);
        if (ce != cudaSuccess) return cuda_error(ce, "attention output");
        g = tle::GemmLaunch{};
        g.W = Wl + P.o;
        g.w_rows = e;
        g.X = ATT16;
        g.n_tokens = S;
        g.K = e;
        g.tile_rows = e;
        g.seg[0] = {0, e, X};
        g.n_seg = 1;
        g.err = err;
        g.n_split = gemm_splits(g);
        ce = tle::launch_gemm_f16(tle::kEpiAdd, g, st);
        if (ce != cudaSuccess) return cuda_error(ce, "attn_output");
        // rmsnorm + gate/up + SwiGLU (forward.cpp:216-227)
        ce = tle::launch_rmsnorm_rows_f16(XB16, X, L.ffn_norm, e, eps, S, err, st);
        if (ce != cudaSuccess) return cuda_error(ce, "ffn_norm");
        g = tle::GemmLaunch{};
        g.W = Wl + P.gu;
        g.w_rows = 2 * ff;
        g.X = XB16;
        g.n_tokens = S;
        g.K = e;
        g.tile_rows = ff;
        g.h_out = H16;
        g.err = err;
        g.n_split = gemm_splits(g);
        ce = tle::launch_gemm_f16(tle::kEpiSwiGLU, g, st);
        if (ce != cudaSuccess) return cuda_error(ce, "ffn_gate/up");
        // down projection + residual (forward.cpp:227-229)
        g = tle::GemmLaunch{};
        g.W = Wl + P.down;
        g.w_rows = e;
        g.X = H16;
        g.n_tokens = S;
        g.K = ff;
        g.tile_rows = e;
        g.seg[0] = {0, e, X};
        g.n_seg = 1;
        g.err = err;
        g.n_split = gemm_splits(g);
        ce = tle::launch_gemm_f16(tle::kEpiAdd, g, st);
        if (ce != cudaSuccess) return cuda_error(ce, "ffn_down");
    }
    // the last token's residual, final rmsnorm + LM head (forward.cpp:245-265)
    ce = cudaMemcpyAsync(s->x, X + static_cast<size_t>(S - 1) * e, sizeof(float) * e, cudaMemcpyDeviceToDevice, st);
    if (ce != cudaSuccess) return cuda_error(ce, "last residual");
    const tle_weight_t& head = m->output.data ? m->output : m->token_embd;
    tle::GemvSeg lm{static_cast<const uint8_t*>(head.data), s->logits, m->n_vocab, 0};
    if (int rc = gemv(head.type, tle::kEpiStore, &lm, 1, nullptr, e, s->x, m->output_norm, eps, st, "lm_head"))
        return rc;
    return ok();
}

}  // extern "C"
