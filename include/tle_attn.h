/*
 * tle_attn.h -- C ABI of the B200 grouped-query-attention hot path of
 * tinyllama-engine (RoPE on Q/K, KV-cache append, QK^T, causal softmax, PV).
 *
 * Plain C: device pointers, sizes, an opaque stream handle (a cudaStream_t
 * passed as void*; NULL = legacy default stream) and an int status.  No
 * exceptions cross this boundary; tle_last_error() gives the message of the
 * last failing call on the calling host thread.  Every kernel is sm_100a
 * only; there is no CPU fallback -- calls fail with TLE_ERR_CUDA when no
 * B200 is present.
 *
 * Shapes follow llama_config_t (reference src/gguf.h:139-168).  The kernels
 * are specialised for TinyLlama-1.1B attention: n_head = 32, n_head_kv = 4,
 * head_dim = 64 (tle_rope accepts any even head_dim).  Other shapes return
 * TLE_ERR_UNSUPPORTED.
 *
 * KV-cache layout is the reference's (run_state.h:100-101, ops.cpp:1350):
 * one fp32 array per sequence per K/V, [n_layers][n_ctx][n_head_kv*head_dim],
 * device-resident, 16-byte aligned.
 */
#ifndef TLE_ATTN_H
#define TLE_ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    TLE_OK = 0,
    TLE_ERR_INVALID = 1,     /* bad argument (null pointer, range, alignment) */
    TLE_ERR_UNSUPPORTED = 2, /* shape outside the specialised kernels */
    TLE_ERR_WORKSPACE = 3,   /* workspace smaller than the *_workspace_bytes() result */
    TLE_ERR_CUDA = 4,        /* CUDA runtime error (message in tle_last_error) */
    TLE_ERR_DEVICE = 5       /* a kernel recorded a device-side error (bounded wait expired) */
};

/* The fields of llama_config_t (gguf.h:139-168) that attention reads. */
typedef struct {
    int32_t n_layers;      /* llama.block_count                  (22)    */
    int32_t n_head;        /* llama.attention.head_count         (32)    */
    int32_t n_head_kv;     /* llama.attention.head_count_kv      (4)     */
    int32_t head_dim;      /* n_embd / n_head, gguf.h:165-167    (64)    */
    float rope_freq_base;  /* llama.rope.freq_base               (10000) */
} tle_shape_t;

/* One decoding sequence: its device KV cache and the position of the token
 * being decoded (the call appends row `pos` and attends to rows 0..pos,
 * exactly like attention(..., layer, pos, cfg) with cfg.n_ctx = n_ctx). */
typedef struct {
    float* key_cache;   /* device [n_layers][n_ctx][n_head_kv*head_dim] */
    float* value_cache; /* device, same layout                           */
    int32_t n_ctx;      /* rows per layer (RunState capacity)            */
    int32_t pos;        /* 0 <= pos < n_ctx                              */
} tle_seq_t;

/* Message for the last failing call on this host thread ("" if none). */
const char* tle_last_error(void);

/* Library version string. */
const char* tle_version(void);

/* Replaces rope() (reference src/ops.h:175-176, src/ops.cpp:1223-1281):
 * rotates pairs (2i, 2i+1) of q [n_head*head_dim] and k [n_head_kv*head_dim]
 * in place by pos * 1/freq_base^(2i/head_dim).  Device pointers. */
int tle_rope(float* q, float* k, int pos, int head_dim, int n_head, int n_head_kv,
             float freq_base, void* stream);

/* Workspace for tle_attention / tle_rope_attention / tle_attention_lse
 * (split-K partials of sequences longer than 2048 rows; no initialisation
 * needed).  Calls that share a workspace must not overlap on the GPU (calls
 * on one stream never do). */
size_t tle_attention_workspace_bytes(const tle_shape_t* shape, int n_ctx);

/* Replaces attention() (reference src/ops.h:204-206, src/ops.cpp:1317-1515)
 * for one sequence: appends k, v at row pos of layer `layer`, then writes
 * out [n_head*head_dim] = softmax(q.K^T/sqrt(hd)) V over rows 0..pos.  q and
 * k are already rotated, as in the reference.  The reference's `att` scratch
 * is replaced by `workspace` (device, tle_attention_workspace_bytes()).  Up
 * to 2048 attended rows one launch splits the rows into chunks of one
 * thread-block cluster per KV head, merged in distributed shared memory (the
 * workspace is not touched); longer sequences are split over the SMs and
 * merged by a second launch. */
int tle_attention(float* out, const float* q, const float* k, const float* v, float* key_cache,
                  float* value_cache, int layer, int pos, int n_ctx, const tle_shape_t* shape,
                  void* workspace, size_t workspace_bytes, void* stream);

/* Context split of one long sequence over several GPUs (no reference
 * counterpart; the reference is single-process).  tle_attention plus the
 * log-sum-exp of every head's scaled scores, lse[n_head] (device, 16-byte
 * aligned): a GPU holding rows [r0, r1) of the sequence calls it on its
 * shard (local rows, q and k rotated for the global position), and
 * tle_merge_lse combines the shards' (out, lse) into the attention over all
 * rows.  A shard that does not hold the new token passes its own last
 * cached row as k, v with pos = its last local row (the append rewrites the
 * row with itself). */
int tle_attention_lse(float* out, float* lse, const float* q, const float* k, const float* v,
                      float* key_cache, float* value_cache, int layer, int pos, int n_ctx,
                      const tle_shape_t* shape, void* workspace, size_t workspace_bytes,
                      void* stream);

/* out[32*64] = sum_r exp(lses[r][h] - LSE_h) parts[r][h][:], LSE_h =
 * log sum_r exp(lses[r][h]); parts [n_parts][32*64], lses [n_parts][32],
 * all device pointers.  TinyLlama geometry (32 heads x 64). */
int tle_merge_lse(float* out, const float* parts, const float* lses, int n_parts, void* stream);

/* forward.cpp:192-208 in one launch: rope(q, k, pos) then attention().
 * q and k are the UNROTATED projections and are left unmodified; the rotated
 * k is what lands in the cache, as in the reference. */
int tle_rope_attention(float* out, const float* q, const float* k, const float* v,
                       float* key_cache, float* value_cache, int layer, int pos, int n_ctx,
                       const tle_shape_t* shape, void* workspace, size_t workspace_bytes,
                       void* stream);

/* tle_rope_attention with flags: TLE_DECODE_KV_READY (defined below; the
 * same contract as for tle_decode_batch, for this call's layer and rows <
 * pos) lets the kernel stream the cached rows while the kernel launched
 * before it on the stream finishes.  0 gives tle_rope_attention; unknown
 * bits are rejected with TLE_ERR_INVALID. */
int tle_rope_attention_flags(float* out, const float* q, const float* k, const float* v,
                             float* key_cache, float* value_cache, int layer, int pos, int n_ctx,
                             const tle_shape_t* shape, int flags, void* workspace,
                             size_t workspace_bytes, void* stream);

/* ---- batched multi-sequence decode (no reference counterpart: the
 * reference decodes one sequence; this runs its attention() for many
 * independent sequences in one launch, ops.cpp:1317 per sequence) ---- */

/* Bytes of the batch descriptor for n_seqs sequences and up to max_ctas CTAs. */
size_t tle_decode_desc_bytes(int n_seqs, int max_ctas);

/* Builds the batch descriptor in HOST memory from host-side sequence
 * records: copies the records and splits the sum of (pos+1) over the
 * sequences evenly across *n_ctas CTAs (max_ctas <= 0: one per SM of the
 * current device).  The caller copies desc_host to device memory unchanged
 * and passes that copy and *n_ctas to tle_decode_batch. */
int tle_decode_desc(const tle_shape_t* shape, const tle_seq_t* seqs, int n_seqs, int max_ctas,
                    void* desc_host, size_t desc_bytes, int* n_ctas);

/* Workspace for tle_decode_batch. */
size_t tle_decode_workspace_bytes(const tle_shape_t* shape, int n_seqs, int n_ctas);

/* Flags of tle_decode_batch / tle_decode_batch_paged (a 0/1 `rotate` value
 * from older callers keeps its meaning). */
#define TLE_DECODE_ROTATE 1   /* rope(q_s, k_s, pos_s) before attending            */
/* The caller guarantees that no kernel that may still be running when this
 * call's kernel starts writes the cached rows this call reads (rows < pos_s)
 * or a page table.  Under programmatic dependent launch that is the kernel
 * launched just before this call and, in a chain of such launches, the ones
 * before it that have not finished.  The decode kernel then starts streaming
 * those rows while the previous kernels finish, and waits for them only
 * before reading q/k/v and writing anything.  Holds in a forward pass (the
 * kernels in flight are the projections and other layers' calls; a layer's
 * rows < pos are written only by that layer's call of an earlier token) and
 * in a loop over layers; does not hold for a prefill of the same layer
 * issued just before on the same stream. */
#define TLE_DECODE_KV_READY 2

/* One decode step of layer `layer` for every sequence in the descriptor:
 * per sequence s, with q [n_seqs][n_head*hd], k/v [n_seqs][n_head_kv*hd]:
 * if flags & TLE_DECODE_ROTATE, rope(q_s, k_s, pos_s) (not written back);
 * append k_s, v_s at row pos_s; out_s = attention over rows 0..pos_s.
 * desc_dev is the device copy of the tle_decode_desc() output.  Unknown
 * flag bits are rejected with TLE_ERR_INVALID. */
int tle_decode_batch(const tle_shape_t* shape, const void* desc_dev, int n_seqs, int n_ctas,
                     const float* q, const float* k, const float* v, float* out, int layer,
                     int flags, void* workspace, size_t workspace_bytes, void* stream);

/* tle_decode_batch for a batch whose every sequence attends to at most 2048
 * rows (pos + 1 <= max_rows <= 2048), built for latency: one thread-block
 * cluster of up to 8 CTAs per (sequence, KV head), the chunk partials folded
 * in distributed shared memory (no workspace, no atomics, one launch).
 * desc_dev as for tle_decode_batch (a contiguous-cache descriptor); only its
 * sequence records are read.  Same contract and tolerance as
 * tle_decode_batch; faster when the batch's rows leave the SMs short of work
 * (for example one rank's share of a sequence-partitioned batch).  A record
 * with pos outside [0, n_ctx), pos + 1 beyond max_rows or a null cache is
 * skipped and reported through tle_device_error as 0x10a. */
int tle_decode_batch_short(const tle_shape_t* shape, const void* desc_dev, int n_seqs, int max_rows,
                           const float* q, const float* k, const float* v, float* out, int layer,
                           int flags, void* stream);

/* ---- batched decode over a bf16 KV cache ----
 * No counterpart in the reference (its cache is fp32, run_state.h:134-138):
 * the same decode step with cache rows stored as bf16 (round to nearest
 * even), half the bytes per row.  The query and the softmax weights enter
 * the tensor cores as bf16 with fp32 accumulation, so outputs agree with
 * the fp32 reference to bf16 precision (the prefill contract, 2e-2), not
 * to the fp32 decode's 1e-4. */
typedef struct {
    void* key_cache;    /* device bf16 [n_layers][n_ctx][n_head_kv*head_dim] */
    void* value_cache;  /* device bf16, same layout                          */
    int32_t n_ctx;
    int32_t pos;
} tle_seq_bf16_t;

/* Scratch of tle_decode_batch_bf16 for n_seqs sequences of at most max_rows
 * rows (pos + 1). */
size_t tle_decode_bf16_workspace_bytes(int n_seqs, int max_rows);

/* One decode step of layer `layer` for sequences seqs_dev[0..n_seqs) (a
 * device array): per sequence s, if flags & TLE_DECODE_ROTATE, rope(q_s,
 * k_s, pos_s) (not written back); append bf16(k_s), bf16(v_s) at row pos_s;
 * out_s = attention over rows 0..pos_s.  q [n_seqs][n_head*hd], k/v
 * [n_seqs][n_head_kv*hd] fp32; max_rows >= every pos_s + 1 (a record with
 * pos outside [0, n_ctx) or beyond max_rows is skipped and reported through
 * tle_device_error as 0x10a).  Other flag bits are rejected with
 * TLE_ERR_INVALID. */
int tle_decode_batch_bf16(const tle_shape_t* shape, const tle_seq_bf16_t* seqs_dev, int n_seqs,
                          int max_rows, const float* q, const float* k, const float* v, float* out,
                          int layer, int flags, void* workspace, size_t workspace_bytes, void* stream);

/* The bf16 decode over page pools (the paged layout below, rows stored as
 * bf16): row r of page p of layer l is at
 *   pool + ((l * n_pages + p) * page_rows + r) * n_head_kv * head_dim
 * bf16 elements; page_rows a power of two in [64, 65536].  seqs_dev is a
 * device array of tle_paged_seq_t records, their page tables on the device too.
 * A record with pos outside its table is skipped (0x10a), a page id
 * outside the pool is not dereferenced (0x105).  Same results as
 * tle_decode_batch_bf16 on the same rows. */
typedef struct {
    void* key_pool;     /* device bf16 [n_layers][n_pages][page_rows][n_head_kv*head_dim] */
    void* value_pool;
    int32_t n_pages;
    int32_t page_rows;
} tle_page_pool_bf16_t;

/* ---- batched decode over a paged KV cache ----
 * No counterpart in the reference: run_state.h:20-25 sizes one contiguous
 * [n_layers][n_ctx][256] cache per sequence and names PagedAttention as the
 * next step.  Here the rows of all sequences live in one pair of page pools
 * shared by the batch; each sequence maps its rows to pool pages through a
 * page table.  Same kernel, same split of rows over CTAs and bit-identical
 * results to tle_decode_batch on the same rows (a tile of rows reaches
 * shared memory in the same order whichever layout it came from). */

/* The pools: row r of page p of layer l is at
 *   pool + ((l * n_pages + p) * page_rows + r) * n_head_kv * head_dim. */
typedef struct {
    float* key_pool;    /* device [n_layers][n_pages][page_rows][n_head_kv*head_dim] fp32 */
    float* value_pool;  /* device, same layout                                            */
    int32_t n_pages;    /* pages per layer in each pool                                   */
    int32_t page_rows;  /* rows per page: a power of two, 16 .. 65536                     */
} tle_page_pool_t;

/* One decoding sequence of a paged batch: its rows 0..pos are rows
 * r % page_rows of pool pages pages[r / page_rows]. */
typedef struct {
    const int32_t* pages; /* DEVICE int32 [n_pages]: page ids in [0, pool n_pages)   */
    int32_t n_pages;      /* entries in pages; need n_pages * page_rows > pos       */
    int32_t pos;          /* position of the token being decoded (appended at row pos) */
} tle_paged_seq_t;

/* tle_decode_batch_bf16 over bf16 page pools (see tle_page_pool_bf16_t);
 * workspace as tle_decode_bf16_workspace_bytes. */
int tle_decode_batch_bf16_paged(const tle_shape_t* shape, const tle_page_pool_bf16_t* pool,
                                const tle_paged_seq_t* seqs_dev, int n_seqs, int max_rows, const float* q,
                                const float* k, const float* v, float* out, int layer, int flags,
                                void* workspace, size_t workspace_bytes, void* stream);

/* tle_decode_desc for a paged batch (same tle_decode_desc_bytes size, same
 * split of rows over CTAs).  The page tables stay on the device and are
 * read by the kernel: they must hold valid ids when the decode runs.  An id
 * outside [0, pool n_pages) is not dereferenced; the kernel skips that
 * access and tle_device_error then reports 0x105. */
int tle_decode_desc_paged(const tle_shape_t* shape, const tle_page_pool_t* pool,
                          const tle_paged_seq_t* seqs, int n_seqs, int max_ctas, void* desc_host,
                          size_t desc_bytes, int* n_ctas);

/* tle_decode_batch over the pools: appends k_s, v_s at row pos_s of each
 * sequence (through its page table) and attends to rows 0..pos_s.  desc_dev
 * is the device copy of the tle_decode_desc_paged() output, workspace as
 * for tle_decode_batch (tle_decode_workspace_bytes). */
int tle_decode_batch_paged(const tle_shape_t* shape, const tle_page_pool_t* pool,
                           const void* desc_dev, int n_seqs, int n_ctas, const float* q,
                           const float* k, const float* v, float* out, int layer, int flags,
                           void* workspace, size_t workspace_bytes, void* stream);

/* ---- decode without allocation ----
 * No counterpart in the reference.  For callers that cannot call cudaMalloc:
 * a host framework that owns all device memory through its own pool, or a
 * per-token loop that must not pay cudaMalloc/cudaFree's implicit device
 * synchronisation.  Same kernels and results as tle_decode_batch, but the
 * batch descriptor is built from HOST records (seqs) and both it and the
 * split-K partials live in a fixed file-scope device array of about 4.2 MB
 * (TLE_NOALLOC_MAX_SEQS sequences, up to 256 CTAs) that every GPU loading
 * the library keeps until the process exits.  The caller passes only inputs
 * and outputs; nothing is allocated (no cudaMalloc/cudaFree, no allocating
 * library routine).
 *  - n_seqs > TLE_NOALLOC_MAX_SEQS is rejected with TLE_ERR_INVALID.
 *  - The first call on a device looks up the array's device address
 *    (cudaGetSymbolAddress); make that first call before any stream capture.
 *  - Every call shares the one array: calls that overlap on the GPU (other
 *    streams, other host threads on the same device) race.  Calls on one
 *    stream are ordered.  Nothing in the array needs to start at zero: each
 *    call rewrites the descriptor and every partial it reads.
 *  - The descriptor is copied from pageable host memory on `stream`, which
 *    makes the call wait for earlier work on that stream. */
#define TLE_NOALLOC_MAX_SEQS 256
int tle_decode_batch_noalloc(const tle_shape_t* shape, const tle_seq_t* seqs, int n_seqs,
                             const float* q, const float* k, const float* v, float* out, int layer,
                             int rotate, void* stream);

/* ---- prefill ---- */

/* Workspace for tle_prefill with n_rows = pos0 + n_tokens attended rows. */
size_t tle_prefill_workspace_bytes(const tle_shape_t* shape, int n_tokens, int pos0);

/* The reference's prefill (generate.cpp:56-59: one forward() per prompt
 * token, i.e. rope+attention at pos0, pos0+1, ..., pos0+n_tokens-1) as one
 * causal flash attention on the tcgen05 tensor cores: q [n_tokens][n_head*hd],
 * k/v [n_tokens][n_head_kv*hd] (unrotated, unmodified); rotated k and v are
 * appended at rows pos0.. of layer `layer`; out [n_tokens][n_head*hd].
 * Q, K and V enter the tensor cores as bf16 with fp32 accumulation and an
 * fp32 softmax; rows < pos0 are read from the fp32 cache. */
int tle_prefill(float* out, const float* q, const float* k, const float* v, float* key_cache,
                float* value_cache, int layer, int pos0, int n_tokens, int n_ctx,
                const tle_shape_t* shape, void* workspace, size_t workspace_bytes, void* stream);

/* ---- multi-GPU sequence partition ---- */

/* Greedy longest-processing-time assignment of sequences to n_ranks GPUs,
 * balancing sum(lengths) per rank (KV bytes are proportional to length).
 * rank_of_seq[s] receives the rank of sequence s; ties keep sequence order.
 * Host-only; no counterpart in the single-process reference. */
int tle_partition_lpt(const int32_t* lengths, int n_seqs, int n_ranks, int32_t* rank_of_seq);

/* ---- diagnostics ---- */

/* Reads (and clears if clear != 0) the device error word that kernels set;
 * 0 = no error.  Codes: 0x101-0x104 a bounded wait expired (0x101 a stage
 * never filled, 0x102 never drained, 0x103 a tensor-core commit never
 * arrived, 0x104 the exit-time drain), 0x105 a paged decode met a page id
 * outside the pool, 0x106 a token id outside the vocabulary, 0x108 a grid
 * barrier wait of the one-launch forward expired, 0x109 a finite activation
 * of the batched prompt overflowed fp16, 0x10a a bf16 or short-batch decode
 * record outside its cache or max_rows, 0x1ff the self-test below.  The first code recorded
 * stays until cleared.  Synchronises the device. */
int tle_device_error(int clear, uint32_t* code);

/* Exercises the failure path of the kernels' bounded waits without a fault:
 * launches one block that waits, through the same bounded mbarrier wait the
 * kernels use, on a barrier nothing ever arrives at, with a limit of
 * limit_us microseconds (1 .. 1000000).  When the limit expires the block
 * records code 0x1ff in the device error word and returns, leaving the
 * context usable; read it with tle_device_error.  No reference counterpart. */
int tle_selftest_wait_timeout(uint32_t limit_us, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TLE_ATTN_H */
