// kernels.h -- internal interface between the C ABI (abi.cu) and the kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>

#include "tle_attn.h"

namespace tle {

// TinyLlama attention geometry the decode/prefill kernels are built for.
constexpr int kHeadDim = 64;
constexpr int kNHead = 32;
constexpr int kNHeadKv = 4;
constexpr int kRowFloats = kNHeadKv * kHeadDim;          // one cache row, all kv heads
constexpr int kPartialFloats = kNHead * (kHeadDim + 2);  // o[32][64], m[32], l[32]
constexpr int kMaxCtas = 1024;                            // upper bound on decode CTAs
constexpr int kMinRowsPerCta = 128;                       // smallest split worth a CTA

// Batch descriptor (built on the host by tle_decode_desc, read by the kernels):
//   DescHeader | tle_seq_t seqs[n_seqs] | CtaStart cta_start[n_ctas+1] | SeqCtas seq_ctas[n_seqs]
//   | int32 arrivals[n_seqs]
// arrivals[] are zero in every upload; the decode kernel counts the CTAs that
// finished a partial of each sequence there and the last one merges them and
// resets the count to zero.
struct DescHeader {
    int32_t magic;
    int32_t n_seqs;
    int32_t n_ctas;
    int32_t reserved;
    int64_t total_rows;
    int64_t reserved2;
};
static_assert(sizeof(DescHeader) == 32, "descriptor header is 32 bytes");
static_assert(sizeof(tle_seq_t) == 24, "tle_seq_t is 24 bytes");
constexpr int32_t kDescMagic = 0x544c4544;  // "TLED"
constexpr int32_t kDescMagicPaged = 0x544c4550;  // "TLEP": slots hold {page table, -, n_pages, pos}

// CTA c processes the concatenated rows [cta_start[c], cta_start[c+1]) of the
// batch, each start given as (sequence, row offset in that sequence).
struct CtaStart {
    int32_t seq;
    int32_t off;
};
// Sequence s is covered by CTAs lo..hi; lo == hi means one CTA wrote the
// final output directly and no merge is needed.
struct SeqCtas {
    int32_t lo;
    int32_t hi;
};

inline size_t desc_seqs_offset() { return sizeof(DescHeader); }
inline size_t desc_cta_offset(int n_seqs) {
    return sizeof(DescHeader) + sizeof(tle_seq_t) * static_cast<size_t>(n_seqs);
}
inline size_t desc_seqctas_offset(int n_seqs, int n_ctas) {
    return desc_cta_offset(n_seqs) + sizeof(CtaStart) * static_cast<size_t>(n_ctas + 1);
}
inline size_t desc_arrivals_offset(int n_seqs, int n_ctas) {
    return desc_seqctas_offset(n_seqs, n_ctas) + sizeof(SeqCtas) * static_cast<size_t>(n_seqs);
}
inline size_t desc_total_bytes(int n_seqs, int n_ctas) {
    return desc_arrivals_offset(n_seqs, n_ctas) + sizeof(int32_t) * static_cast<size_t>(n_seqs);
}

struct DecodeArgs {
    const tle_seq_t* seqs;       // batch mode: device array; nullptr = single mode
    const CtaStart* cta_start;   // batch mode: [n_ctas+1]
    const SeqCtas* seq_ctas;     // batch mode: [n_seqs]
    int32_t* arrivals;           // batch mode: [n_seqs] partial-arrival counts (merge in the last CTA)
    tle_seq_t single;            // single mode: the one sequence
    int n_seqs;
    int n_ctas;
    const float* q;              // [n_seqs][32*64]
    const float* k;              // [n_seqs][4*64]
    const float* v;              // [n_seqs][4*64]
    float* out;                  // [n_seqs][32*64]
    float* partials;             // [n_ctas + n_seqs][kPartialFloats]
    float* lse;                  // single mode, optional: [32] log-sum-exp of each head's scores
    int layer;
    int rotate;
    int kv_ready;                // batch mode: stream the first tiles before waiting on the previous grid
    uint32_t* err;               // device error word
    // Paged batch mode (key_pool != nullptr): each sequence record's
    // key_cache slot holds its page table (int32 page ids), and row r of a
    // sequence is row r % page_rows of page pages[r / page_rows] in the pools
    // [n_layers][pool_pages][page_rows][256], page_rows = 1 << page_shift.
    float* key_pool;
    float* value_pool;
    int pool_pages;
    int page_shift;
    float inv_freq[kHeadDim / 2];
};

cudaError_t launch_decode(const DecodeArgs& a, cudaStream_t stream);

// Short single-sequence decode (tle_attention, tle_rope_attention,
// tle_attention_lse with at most kSeqMaxRows attended rows): one cluster of
// n_chunks (<= 8) CTAs per KV head, one warp per query head, the chunks'
// partials folded through distributed shared memory (no workspace, one
// launch).
constexpr int kSeqMaxChunks = 8;
constexpr int kSeqMaxChunkRows = 256;
constexpr int kSeqMaxRows = kSeqMaxChunkRows * kSeqMaxChunks;            // 2048
struct SeqArgs {
    const float* q;              // [32*64]
    const float* k;              // [4*64]
    const float* v;              // [4*64]
    float* out;                  // [32*64]
    float* lse;                  // optional [32]
    float* key_cache;            // [n_layers][n_ctx][256]
    float* value_cache;
    uint32_t* err;
    int layer, pos, n_ctx, rotate;
    int chunk_rows, n_chunks;    // n_chunks * chunk_rows >= pos + 1, chunk_rows a multiple of 32
    float rope_cos[kHeadDim / 2], rope_sin[kHeadDim / 2];   // of pos * inv_freq[i], from the host
    // Batch mode (seqs != nullptr): grid z = sequence s of seqs[0..n_seqs)
    // (device records; pos + 1 <= n_chunks * chunk_rows for every s), q/k/v/out
    // [n_seqs][...], angles from inv_freq on the device; the fields above
    // that describe one sequence (pos, n_ctx, caches, lse, angles) are unused.
    const tle_seq_t* seqs;
    int n_seqs;
    int kv_ready;                // TLE_DECODE_KV_READY: the cached rows are read before the wait
    float inv_freq[kHeadDim / 2];
};
cudaError_t launch_seq_decode(const SeqArgs& a, cudaStream_t stream);

// Decode over bf16 caches (decode_bf16.cu): CTA (c, s) takes rows
// [c chunk, (c + 1) chunk) of sequence s; chunk partials (o / l and the
// log-sum-exp) of sequences with more than one chunk are merged by a second
// launch.  The chunk (a multiple of 64 rows, at most kBfMaxChunk) is chosen
// from the batch shape so that a launch has about kBfTargetCtas CTAs.
constexpr int kBfMaxChunk = 2048;
constexpr int kBfTargetCtas = 2 * 148;
inline int bf16_chunk_rows(int n_seqs, int max_rows) {
    const long long per = (static_cast<long long>(n_seqs) * max_rows + kBfTargetCtas - 1) / kBfTargetCtas;
    const long long c = (per + 63) / 64 * 64;
    return static_cast<int>(c < 64 ? 64 : (c > kBfMaxChunk ? kBfMaxChunk : c));
}
struct BfArgs {
    const tle_seq_bf16_t* seqs;  // device [n_seqs] (contiguous caches), or
    const tle_paged_seq_t* pseqs;   // device [n_seqs] (paged: rows in the pools below)
    void* key_pool;              // paged: bf16 [n_layers][pool_pages][1 << page_shift][256]
    void* value_pool;
    int pool_pages, page_shift;
    int n_seqs, chunk, max_chunks;   // max_chunks = ceil(max_rows / chunk)
    const float* q;              // [n_seqs][32*64]
    const float* k;              // [n_seqs][256]
    const float* v;
    float* out;                  // [n_seqs][32*64]
    float* parts;                // [n_seqs][max_chunks][32][64]
    float* lses;                 // [n_seqs][max_chunks][32]
    int layer, rotate;
    uint32_t* err;
    float inv_freq[kHeadDim / 2];
};
size_t decode_bf16_workspace_bytes(int n_seqs, int max_rows);
cudaError_t launch_decode_bf16(const BfArgs& a, cudaStream_t stream);
// out[32*64] = sum_r w_r parts[r] with w_r = exp(lses[r][h] - LSE_h),
// LSE_h = log sum_r exp(lses[r][h]): the attention over the union of the
// parts' key sets, each part normalised over its own keys.
cudaError_t launch_merge_lse(float* out, const float* parts, const float* lses, int n_parts,
                             cudaStream_t stream);

struct RopeArgs {
    float* q;
    float* k;
    int pos;
    int half;  // head_dim / 2
    int n_head;
    int n_head_kv;
    float inv_freq[128];
};
cudaError_t launch_rope(const RopeArgs& a, cudaStream_t stream);

struct PrefillArgs {
    const float* q;       // [n_tokens][32*64] unrotated
    const float* k;       // [n_tokens][4*64]  unrotated
    const float* v;       // [n_tokens][4*64]
    float* out;           // [n_tokens][32*64]
    float* key_cache;     // [n_layers][n_ctx][256]
    float* value_cache;
    int layer;
    int pos0;
    int n_tokens;
    int n_ctx;
    void* workspace;
    uint32_t* err;        // device error word
    int f16;              // tensor-core operands fp16 (batched prompt) instead of bf16 (tle_prefill)
    float inv_freq[kHeadDim / 2];
};
size_t prefill_workspace_bytes(int n_tokens, int pos0);
cudaError_t launch_prefill(const PrefillArgs& a, cudaStream_t stream);

cudaError_t read_device_error(int clear, uint32_t* code);

// Runs `configure` (kernel attributes) once per device, thread-safe; later
// calls cost one atomic load.
// ---- forward pass around attention (forward.cu) ----
// Weight formats: the ggml type numbers (reference src/gguf.h:23-33).
constexpr int kWF32 = 0, kWF16 = 1, kWQ4_0 = 2, kWQ8_0 = 8, kWQ6_K = 14;
// What a GEMV does with row r's product y.
constexpr int kEpiStore = 0;    // out[r] = y
constexpr int kEpiAdd = 1;      // out[r] += y (residual)
constexpr int kEpiSwiGLU = 2;   // out[r] = silu(gate_r) * up_r (gate rows seg[0].W, up rows W2)
constexpr int kGemvMaxCols = 16384;   // input vector in shared memory (64 KB)
constexpr int kGemvMaxSmem = 160 * 1024;   // input vector + TMA-staged weight rows per CTA

struct GemvSeg {
    const uint8_t* W;   // rows x cols, GGUF layout, row r at r * row_bytes
    float* out;
    int rows;
    int tile0;          // first CTA of the segment (set by launch_gemv)
};
struct GemvArgs {
    GemvSeg seg[3];
    int n_seg;
    const uint8_t* W2;      // SwiGLU: the up-projection rows (gate's layout)
    int cols;
    int row_bytes;
    int rpw;                // rows per warp (generic path)
    int rpc;                // (set by launch_gemv) rows per CTA
    int ks;                 // (set by launch_gemv) column chunks per row group (shared-memory Q4_0 path)
    const float* x;         // input [cols]
    const float* norm_w;    // RMSNorm weight applied to x first (nullptr: none)
    float eps;
    int xs_bytes;           // (set by launch_gemv) shared bytes of the input vector
    int tile_bytes;         // (set by launch_gemv) TMA-staged rows per CTA; 0: rows read from global
    uint32_t* err;          // device error word
};
// Bytes of one row of `cols` weights of format `type`; -1 if unsupported.
int weight_row_bytes(int type, int cols);

// The layers of one token in one persistent cooperative launch (models
// whose linear weights are all Q4_0): per layer five phases separated by
// grid barriers -- RMSNorm + q/k/v, rope + attention + append, output
// projection + residual, RMSNorm + gate/up + SwiGLU, down + residual -- with
// each CTA's weight rows of the next products bulk-copied into shared
// memory ahead of the barrier before the phase that reads them.
constexpr int kPersistMaxLayers = 32;
constexpr int kPersistAttRows = 64;   // attention rows per chunk
constexpr int kPersistMaxBlocks = 256;   // 32-input blocks of the widest input (n_ff <= 8192)
struct PersistLayer {
    const uint8_t* w[7];         // q, k, v, output, gate, up, down (Q4_0, 16-byte aligned)
    const float* attn_norm;
    const float* ffn_norm;
};
struct PersistArgs {
    PersistLayer layer[kPersistMaxLayers];
    int n_layers, n_embd, n_ff, n_ctx, pos;
    float eps;
    float* x;                    // [n_embd] residual stream
    float* q;                    // [n_embd]
    float* k;                    // [256]
    float* v;                    // [256]
    float* hb;                   // [n_ff]
    float* key_cache;            // [n_layers][n_ctx][256]
    float* value_cache;
    float* partials;             // [att_chunks][32][68] attention records (o[64], max, sum)
    uint32_t* sync;              // grid barrier count, zero at launch
    uint32_t* err;
    int att_chunks;              // chunks of 64 rows per KV head (ceil((pos + 1) / 64))
    int stride_e, stride_f;      // shared-memory row strides of n_embd- and n_ff-column rows (bytes)
    int off_a, off_b, off_kv, off_part;   // shared-memory offsets (bytes): buffers A, B, K/V, partials
    float inv_freq[kHeadDim / 2];
};
// Shared memory a persistent launch over `grid` CTAs needs (fills the
// strides and offsets of *a); 0 when the shape does not fit (then the
// per-product launches are used).
size_t persist_smem_bytes(int n_embd, int n_ff, int grid, PersistArgs* a);
// Most attention chunks per KV head, and the workspace (barrier count and
// attention records) a launch over `grid` CTAs needs.
int persist_max_chunks(int grid);
size_t persist_workspace_bytes(int grid);
cudaError_t launch_forward_persistent(const PersistArgs& a, int grid, size_t smem, cudaStream_t stream);
cudaError_t launch_gemv(int type, int epi, GemvArgs a, cudaStream_t stream);
cudaError_t launch_embed(int type, float* x, const void* table, const int32_t* token, int n_vocab,
                         int n_embd, uint32_t* err, cudaStream_t stream);
cudaError_t launch_argmax(const float* logits, int n, int32_t* out, cudaStream_t stream);
// Temperature or top-p sampling of one row with the uniform draw r.
constexpr int kSampleMaxVocab = 40960;
constexpr int kSampleMaxSmem = (kSampleMaxVocab + 2 * 2048) * 4;
cudaError_t launch_sample(float* logits, int n, float temperature, float top_p, float r, bool use_top_p,
                          int32_t* out, cudaStream_t stream);
cudaError_t launch_rmsnorm(float* out, const float* x, const float* w, int n, float eps,
                           cudaStream_t stream);
cudaError_t launch_vec_add(float* out, const float* x, int n, cudaStream_t stream);

// ---- batched prompt forward (gemm.cu) ----
// Y[t][r] = sum_k W[r][k] X[t][k] on the tensor cores, W and X fp16
// row-major, fp32 accumulation; tiles of 128 weight rows x 128 tokens.
constexpr int kGemmTileRows = 128;
constexpr int kGemmTileTokens = 128;
constexpr int kGemmTileK = 64;
struct GemmSegment {
    int row0;     // first weight row of the segment
    int rows;     // its rows (a multiple of kGemmTileRows)
    float* out;   // [n_tokens][rows]: out[t][r - row0]
};
struct GemmLaunch {
    const uint16_t* W;   // fp16 [w_rows][K]
    int w_rows;
    const uint16_t* X;   // fp16 [round_up(n_tokens, 128)][K] (pad rows are read, their results dropped)
    int n_tokens;
    int K;               // a multiple of kGemmTileK
    int tile_rows;       // output rows: w_rows (store/add), n_ff (SwiGLU: gate rows 0.., up rows n_ff..)
    GemmSegment seg[3];  // store/add outputs by weight row
    int n_seg;
    uint16_t* h_out;     // SwiGLU: fp16 [round_up(n_tokens, 128)][tile_rows]
    uint32_t* err;
    // Split of K over the CTAs of a cluster when the output tiles alone leave
    // SMs idle (few tokens): 1, 2, 4 or 8 splits.
    int n_split;
};
// Number of K splits (clusters of 1, 2 or 4 CTAs) for a product of `tiles`
// output tiles and `nk` 64-wide K blocks on `sms` SMs: the most that keeps
// every cluster resident in one wave (at most 7/8 of the SMs busy, as whole
// clusters must fit in a GPC) with at least 4 K blocks per split.  (Clusters
// of 8 of these 197 KB CTAs measured slower than 4.)
inline int gemm_split_for(int tiles, int nk, int sms) {
    int s = 1;
    while (s < 4 && tiles * 2 * s * 8 <= sms * 7 && nk / (2 * s) >= 4) s *= 2;
    return s;
}
cudaError_t launch_gemm_f16(int epi, const GemmLaunch& g, cudaStream_t stream);
// fp16 copy of a GGUF weight (rows x cols of `type`): dst[r][c] = the
// reference's dequantised value, rounded to nearest fp16.
cudaError_t launch_pack_f16(int type, uint16_t* dst, const void* W, int rows, int cols, cudaStream_t stream);
// out[t][:] = fp16(rmsnorm(x[t][:]) * w) for t < n_tokens.
cudaError_t launch_rmsnorm_rows_f16(uint16_t* out, const float* x, const float* w, int n, float eps,
                                    int n_tokens, uint32_t* err, cudaStream_t stream);
// out[i] = fp16(x[i]), i < n.
cudaError_t launch_to_f16(uint16_t* out, const float* x, size_t n, uint32_t* err, cudaStream_t stream);
// x[t][:] = row tokens[t] of the table (F16 or F32), t < n_tokens.
cudaError_t launch_embed_rows(int type, float* x, const void* table, const int32_t* tokens, int n_tokens,
                             int n_vocab, int n_embd, uint32_t* err, cudaStream_t stream);

constexpr int kMaxDevices = 64;
struct PerDeviceOnce {
    std::atomic<bool> done[kMaxDevices] = {};
    std::mutex mu;
    template <class F>
    cudaError_t run(F&& configure) {
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return e;
        if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
        if (done[dev].load(std::memory_order_acquire)) return cudaSuccess;
        std::lock_guard<std::mutex> lock(mu);
        if (done[dev].load(std::memory_order_relaxed)) return cudaSuccess;
        e = configure(dev);
        if (e == cudaSuccess) done[dev].store(true, std::memory_order_release);
        return e;
    }
};
// One block waiting (bounded by limit_ns) on a barrier nothing arrives at;
// records kErrSelfTest in err when the limit expires.
cudaError_t launch_selftest_wait(uint32_t* err, uint64_t limit_ns, cudaStream_t stream);
// Device address of the error word on the current device.
cudaError_t error_word(uint32_t** word);

}  // namespace tle
