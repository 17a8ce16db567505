/*
 * attn_oracle.c -- CPU restatement of tinyllama-engine's attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * kernels in tinyllama-engine_b200/csrc.  Only tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline / reference legs may load it; the product path
 * never links or calls it (there is no CPU fallback).
 *
 * Parity is pinned: tests/test_oracle.py checks this restatement bit-for-bit
 * against the reference's own ops.cpp compiled unmodified into
 * oracle/_ref/libref_attn.so (fixtures in tests/golden/, made by
 * tests/golden/make_golden.py), and against the reference's known-answer
 * tests (src/test_ops.cpp:295-546).
 *
 * Every function keeps the reference's operation order for the x86 scalar
 * path (no __ARM_NEON on x86), so with the reference Makefile's flags
 * (-O2, no -ffast-math, no FMA contraction on baseline x86-64) the results
 * are bit-identical to the reference.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* rope(): reference src/ops.cpp:1223-1281 (declared ops.h:175-176).
 * Rotates interleaved pairs (2i, 2i+1) of every query head and every KV head
 * in place.  freq_i = 1/powf(base, 2i/hd) (ops.cpp:1244-1245), angle =
 * pos*freq_i in float (ops.cpp:1246), then the 2-D rotation
 * (ops.cpp:1257-1258).  std::pow/cos/sin on float arguments resolve to the
 * float overloads, i.e. powf/cosf/sinf. */
static void rope_heads(float *x, int n_heads, int pos, int head_dim, float freq_base)
{
    int n_pairs = head_dim / 2;
    for (int h = 0; h < n_heads; h++) {
        float *hx = x + h * head_dim;
        for (int i = 0; i < n_pairs; i++) {
            float freq = 1.0f / powf(freq_base, (float)(2 * i) / (float)head_dim);
            float angle = (float)pos * freq;
            float c = cosf(angle);
            float s = sinf(angle);
            float x0 = hx[2 * i];
            float x1 = hx[2 * i + 1];
            hx[2 * i] = x0 * c - x1 * s;
            hx[2 * i + 1] = x0 * s + x1 * c;
        }
    }
}

void oracle_rope(float *q, float *k, int pos, int head_dim, int n_head,
                 int n_head_kv, float freq_base)
{
    rope_heads(q, n_head, pos, head_dim, freq_base);    /* ops.cpp:1229-1260 */
    rope_heads(k, n_head_kv, pos, head_dim, freq_base); /* ops.cpp:1263-1280 */
}

/* softmax(): reference src/ops.cpp:1072-1091.  Max pass, exp-and-sum pass,
 * then multiply by 1/sum. */
void oracle_softmax(float *x, int size)
{
    float max_val = x[0];
    for (int i = 1; i < size; i++)
        if (x[i] > max_val) max_val = x[i];
    float sum = 0.0f;
    for (int i = 0; i < size; i++) {
        x[i] = expf(x[i] - max_val);
        sum += x[i];
    }
    float inv_sum = 1.0f / sum;
    for (int i = 0; i < size; i++) x[i] *= inv_sum;
}

/* attention(): reference src/ops.cpp:1317-1515, scalar branch.
 * Cache layout [n_layers][n_ctx][n_head_kv*head_dim]; the layer offset is
 * layer*n_ctx*kv_dim (ops.cpp:1350).  Step 1 appends k and v at row pos
 * (ops.cpp:1370-1371); step 2, per query head qh with kv head qh/gqa
 * (ops.cpp:1383): scores over p in [0,pos] scaled after the dot product
 * (ops.cpp:1425-1433), softmax (ops.cpp:1445), then the zero-initialised
 * weighted sum of cached values (ops.cpp:1494-1508). */
void oracle_attention(float *out, const float *q, const float *k, const float *v,
                      float *key_cache, float *value_cache, float *att,
                      int layer, int pos, int n_ctx, int n_head, int n_head_kv,
                      int head_dim)
{
    int kv_dim = n_head_kv * head_dim;
    int gqa_ratio = n_head / n_head_kv;
    float scale = 1.0f / sqrtf((float)head_dim);
    size_t layer_offset = (size_t)layer * (size_t)n_ctx * (size_t)kv_dim;

    memcpy(key_cache + layer_offset + (size_t)pos * kv_dim, k, sizeof(float) * kv_dim);
    memcpy(value_cache + layer_offset + (size_t)pos * kv_dim, v, sizeof(float) * kv_dim);

    for (int qh = 0; qh < n_head; qh++) {
        const float *q_head = q + qh * head_dim;
        int kvh = qh / gqa_ratio;
        for (int p = 0; p <= pos; p++) {
            const float *kc = key_cache + layer_offset + (size_t)p * kv_dim + kvh * head_dim;
            float score = 0.0f;
            for (int d = 0; d < head_dim; d++) score += q_head[d] * kc[d];
            att[p] = score * scale;
        }
        oracle_softmax(att, pos + 1);
        float *out_head = out + qh * head_dim;
        for (int d = 0; d < head_dim; d++) out_head[d] = 0.0f;
        for (int t = 0; t <= pos; t++) {
            const float *vc = value_cache + layer_offset + (size_t)t * kv_dim + kvh * head_dim;
            float w = att[t];
            for (int d = 0; d < head_dim; d++) out_head[d] += w * vc[d];
        }
    }
}

/* The per-token step that forward() performs for one layer:
 * rope (forward.cpp:192-196) followed by attention (forward.cpp:206-208).
 * q and k are rotated in place, as in the reference. */
void oracle_rope_attention(float *out, float *q, float *k, const float *v,
                           float *key_cache, float *value_cache, float *att,
                           int layer, int pos, int n_ctx, int n_head,
                           int n_head_kv, int head_dim, float freq_base)
{
    oracle_rope(q, k, pos, head_dim, n_head, n_head_kv, freq_base);
    oracle_attention(out, q, k, v, key_cache, value_cache, att, layer, pos,
                     n_ctx, n_head, n_head_kv, head_dim);
}

/* Prefill as the reference performs it: one forward() per prompt token
 * (generate.cpp:56-59), so S successive rope+attention steps at positions
 * pos0 .. pos0+S-1.  q [S][n_head*hd], k/v [S][n_head_kv*hd] are the
 * unrotated projections; q and k are rotated in place; out [S][n_head*hd]. */
void oracle_prefill(float *out, float *q, float *k, const float *v,
                    float *key_cache, float *value_cache, int layer, int pos0,
                    int n_tokens, int n_ctx, int n_head, int n_head_kv,
                    int head_dim, float freq_base)
{
    int q_dim = n_head * head_dim, kv_dim = n_head_kv * head_dim;
    float *att = (float *)malloc(sizeof(float) * (size_t)n_ctx);
    for (int i = 0; i < n_tokens; i++)
        oracle_rope_attention(out + (size_t)i * q_dim, q + (size_t)i * q_dim,
                              k + (size_t)i * kv_dim, v + (size_t)i * kv_dim,
                              key_cache, value_cache, att, layer, pos0 + i,
                              n_ctx, n_head, n_head_kv, head_dim, freq_base);
    free(att);
}

/* ---- batched decode over independent sequences (multi-threaded) ----------
 * One fused rope+attention step per sequence for one layer.  Sequences are
 * independent (each owns its cache), so they are spread over threads; each
 * thread has its own att scratch, as the reference requires (the shared att
 * buffer makes attention() non-reentrant, run_state.h:64). */
typedef struct {
    int n_seqs, n_head, n_head_kv, head_dim, layer;
    float freq_base;
    float *const *kc;
    float *const *vc;
    const int *n_ctx;
    const int *pos;
    float *q, *k;
    const float *v;
    float *out;
    int next;
    pthread_mutex_t mu;
} batch_job;

static void *batch_worker(void *arg)
{
    batch_job *j = (batch_job *)arg;
    int max_ctx = 0;
    for (int s = 0; s < j->n_seqs; s++)
        if (j->n_ctx[s] > max_ctx) max_ctx = j->n_ctx[s];
    float *att = (float *)malloc(sizeof(float) * (size_t)(max_ctx > 0 ? max_ctx : 1));
    int q_dim = j->n_head * j->head_dim, kv_dim = j->n_head_kv * j->head_dim;
    for (;;) {
        pthread_mutex_lock(&j->mu);
        int s = j->next++;
        pthread_mutex_unlock(&j->mu);
        if (s >= j->n_seqs) break;
        oracle_rope_attention(j->out + (size_t)s * q_dim, j->q + (size_t)s * q_dim,
                              j->k + (size_t)s * kv_dim, j->v + (size_t)s * kv_dim,
                              j->kc[s], j->vc[s], att, j->layer, j->pos[s],
                              j->n_ctx[s], j->n_head, j->n_head_kv, j->head_dim,
                              j->freq_base);
    }
    free(att);
    return NULL;
}

void oracle_decode_batch(int n_seqs, float *const *key_caches,
                         float *const *value_caches, const int *n_ctx,
                         const int *pos, float *q, float *k, const float *v,
                         float *out, int layer, int n_head, int n_head_kv,
                         int head_dim, float freq_base, int n_threads)
{
    batch_job j;
    j.n_seqs = n_seqs; j.n_head = n_head; j.n_head_kv = n_head_kv;
    j.head_dim = head_dim; j.layer = layer; j.freq_base = freq_base;
    j.kc = key_caches; j.vc = value_caches; j.n_ctx = n_ctx; j.pos = pos;
    j.q = q; j.k = k; j.v = v; j.out = out; j.next = 0;
    pthread_mutex_init(&j.mu, NULL);
    if (n_threads < 1) n_threads = 1;
    if (n_threads > n_seqs) n_threads = n_seqs > 0 ? n_seqs : 1;
    pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)n_threads);
    for (int t = 1; t < n_threads; t++) pthread_create(&th[t], NULL, batch_worker, &j);
    batch_worker(&j);
    for (int t = 1; t < n_threads; t++) pthread_join(th[t], NULL);
    free(th);
    pthread_mutex_destroy(&j.mu);
}
