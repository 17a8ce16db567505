/*
 * forward_oracle.c -- CPU restatement of the rest of tinyllama-engine's
 * forward pass around attention: the matrix-vector products of every weight
 * format, RMSNorm, the SwiGLU feed-forward block, the residual add, greedy
 * sampling, the embedding lookup and forward()'s call sequence.
 *
 * TEST INFRASTRUCTURE ONLY, like attn_oracle.c: the parity checker for the
 * device forward pass (tinyllama-engine_b200/csrc/forward.cu).  Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU legs may load it.
 *
 * Every function keeps the operation order of the reference's x86 (naive,
 * no __ARM_NEON) path, so with the reference Makefile's flags the results
 * are bit-identical to src/ops.cpp compiled unmodified
 * (tests/test_forward_oracle.py checks that against oracle/_ref).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* Weight formats: the ggml type numbers of reference src/gguf.h:23-33. */
enum { FW_F32 = 0, FW_F16 = 1, FW_Q4_0 = 2, FW_Q8_0 = 8, FW_Q6_K = 14 };

/* Block sizes and byte layouts of reference src/gguf.h:54-135. */
#define QK8_0 32  /* block_q8_0: fp16 d, int8 qs[32]               (34 B)  */
#define QK4_0 32  /* block_q4_0: fp16 d, uint8 qs[16]              (18 B)  */
#define QK_K 256  /* block_q6_K: ql[128], qh[64], int8 sc[16], d   (210 B) */

/* fp16_to_f32(): reference src/ops.cpp:119-156, bit manipulation of an IEEE
 * half (subnormals normalised, NaN quietened). */
float oracle_fp16_to_f32(uint16_t h)
{
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t exp = ((uint32_t)h >> 10) & 0x1Fu;
    uint32_t mant = (uint32_t)h & 0x3FFu;
    uint32_t bits;
    if (exp == 0) {
        if (mant == 0) {
            bits = sign;
        } else {
            int e = -14;
            while ((mant & 0x400u) == 0) {
                mant <<= 1;
                --e;
            }
            mant &= 0x3FFu;
            bits = sign | ((uint32_t)(e + 127) << 23) | (mant << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7F800000u | (mant << 13);
        if (mant != 0) bits |= 0x00400000u;
    } else {
        bits = sign | ((exp + (127 - 15)) << 23) | (mant << 13);
    }
    float out;
    memcpy(&out, &bits, sizeof out);
    return out;
}

static uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* matmul_f32 naive path: ops.cpp:251-262. */
static void mm_f32(float *out, const float *W, const float *x, int rows, int cols)
{
    for (int i = 0; i < rows; i++) {
        float sum = 0.0f;
        const float *row = W + (size_t)i * cols;
        for (int j = 0; j < cols; j++) sum += row[j] * x[j];
        out[i] = sum;
    }
}

/* matmul_f16 naive path: ops.cpp:342-356. */
static void mm_f16(float *out, const uint16_t *W, const float *x, int rows, int cols)
{
    for (int i = 0; i < rows; i++) {
        float sum = 0.0f;
        const uint16_t *row = W + (size_t)i * cols;
        for (int j = 0; j < cols; j++) {
            float w = oracle_fp16_to_f32(row[j]);
            sum += w * x[j];
        }
        out[i] = sum;
    }
}

/* matmul_q8_0 naive path: ops.cpp:442-473 (block sum, then scale * sum). */
static void mm_q8_0(float *out, const uint8_t *W, const float *x, int rows, int cols)
{
    int nb = cols / QK8_0;
    for (int i = 0; i < rows; i++) {
        const uint8_t *row = W + (size_t)i * nb * 34;
        float sum = 0.0f;
        for (int b = 0; b < nb; b++) {
            const uint8_t *blk = row + (size_t)b * 34;
            float scale = oracle_fp16_to_f32(rd16(blk));
            const int8_t *qs = (const int8_t *)(blk + 2);
            const float *xb = x + b * QK8_0;
            float block_sum = 0.0f;
            for (int j = 0; j < QK8_0; j++) block_sum += (float)qs[j] * xb[j];
            sum += scale * block_sum;
        }
        out[i] = sum;
    }
}

/* matmul_q4_0 naive path: ops.cpp:616-655.  Byte j holds element j (low
 * nibble) and element j + 16 (high nibble), both offset by -8. */
static void mm_q4_0(float *out, const uint8_t *W, const float *x, int rows, int cols)
{
    int nb = cols / QK4_0;
    for (int i = 0; i < rows; i++) {
        const uint8_t *row = W + (size_t)i * nb * 18;
        float sum = 0.0f;
        for (int b = 0; b < nb; b++) {
            const uint8_t *blk = row + (size_t)b * 18;
            float scale = oracle_fp16_to_f32(rd16(blk));
            const uint8_t *qs = blk + 2;
            const float *xb = x + b * QK4_0;
            float block_sum = 0.0f;
            for (int j = 0; j < QK4_0 / 2; j++) {
                int v0 = (int)(qs[j] & 0x0F) - 8;
                int v1 = (int)(qs[j] >> 4) - 8;
                block_sum += (float)v0 * xb[j];
                block_sum += (float)v1 * xb[j + QK4_0 / 2];
            }
            sum += scale * block_sum;
        }
        out[i] = sum;
    }
}

/* matmul_q6_k naive path: ops.cpp:882-948.  Super-block of 256: ql[128]
 * low nibbles, qh[64] high 2-bit pairs, int8 scales[16], fp16 d (last).
 * Every product is accumulated straight into the row sum, in the
 * reference's order (two halves of 128, l = 0..31, four values each). */
static void mm_q6_k(float *out, const uint8_t *W, const float *x, int rows, int cols)
{
    int nb = cols / QK_K;
    for (int i = 0; i < rows; i++) {
        const uint8_t *row = W + (size_t)i * nb * 210;
        float sum = 0.0f;
        for (int b = 0; b < nb; b++) {
            const uint8_t *blk = row + (size_t)b * 210;
            const uint8_t *ql = blk;
            const uint8_t *qh = blk + 128;
            const int8_t *sc = (const int8_t *)(blk + 192);
            float d = oracle_fp16_to_f32(rd16(blk + 208));
            const float *xb = x + b * QK_K;
            for (int half = 0; half < 2; half++) {
                const uint8_t *L = ql + 64 * half;
                const uint8_t *H = qh + 32 * half;
                const int8_t *S = sc + 8 * half;
                const float *X = xb + 128 * half;
                for (int l = 0; l < 32; l++) {
                    int is = l / 16;
                    int q1 = ((int)(L[l] & 0x0F) | ((int)((H[l] >> 0) & 3) << 4)) - 32;
                    int q2 = ((int)(L[l + 32] & 0x0F) | ((int)((H[l] >> 2) & 3) << 4)) - 32;
                    int q3 = ((int)(L[l] >> 4) | ((int)((H[l] >> 4) & 3) << 4)) - 32;
                    int q4 = ((int)(L[l + 32] >> 4) | ((int)((H[l] >> 6) & 3) << 4)) - 32;
                    sum += d * (float)S[is + 0] * (float)q1 * X[l + 0];
                    sum += d * (float)S[is + 2] * (float)q2 * X[l + 32];
                    sum += d * (float)S[is + 4] * (float)q3 * X[l + 64];
                    sum += d * (float)S[is + 6] * (float)q4 * X[l + 96];
                }
            }
        }
        out[i] = sum;
    }
}

/* matmul(): the type dispatch of ops.cpp:959-981.  Returns -1 for a type
 * the reference does not support (it throws). */
int oracle_matmul(float *out, const void *W, const float *x, int rows, int cols, int type)
{
    switch (type) {
    case FW_F32: mm_f32(out, (const float *)W, x, rows, cols); return 0;
    case FW_F16: mm_f16(out, (const uint16_t *)W, x, rows, cols); return 0;
    case FW_Q8_0: mm_q8_0(out, (const uint8_t *)W, x, rows, cols); return 0;
    case FW_Q4_0: mm_q4_0(out, (const uint8_t *)W, x, rows, cols); return 0;
    case FW_Q6_K: mm_q6_k(out, (const uint8_t *)W, x, rows, cols); return 0;
    default: return -1;
    }
}

/* rmsnorm() naive path: ops.cpp:1040-1054.  out may alias x. */
void oracle_rmsnorm(float *out, const float *x, const float *weight, int size, float eps)
{
    float ss = 0.0f;
    for (int i = 0; i < size; i++) ss += x[i] * x[i];
    float rms = 1.0f / sqrtf(ss / (float)size + eps);
    for (int i = 0; i < size; i++) out[i] = x[i] * rms * weight[i];
}

/* silu(): ops.cpp:1107-1113; elementwise_mul(): ops.cpp:1129-1146 (naive);
 * vec_add(): ops.cpp:1165-1184 (naive). */
void oracle_silu(float *x, int size)
{
    for (int i = 0; i < size; i++) {
        float val = x[i];
        float sigmoid = 1.0f / (1.0f + expf(-val));
        x[i] = val * sigmoid;
    }
}

void oracle_elementwise_mul(float *a, const float *b, int size)
{
    for (int i = 0; i < size; i++) a[i] *= b[i];
}

void oracle_vec_add(float *out, const float *x, int size)
{
    for (int i = 0; i < size; i++) out[i] += x[i];
}

/* ffn_swiglu(): ops.cpp:1535-1564 -- gate and up projections, silu(gate) *
 * up, down projection; all three weights have the gate's type. */
int oracle_ffn_swiglu(float *out, const float *input, float *hb, float *hb2, const void *W_gate,
                      const void *W_up, const void *W_down, int n_ff, int n_embd, int type)
{
    if (oracle_matmul(hb, W_gate, input, n_ff, n_embd, type)) return -1;
    oracle_matmul(hb2, W_up, input, n_ff, n_embd, type);
    oracle_silu(hb, n_ff);
    oracle_elementwise_mul(hb, hb2, n_ff);
    return oracle_matmul(out, W_down, hb, n_embd, n_ff, type);
}

/* sample_argmax(): ops.cpp:1587-1597 -- the first index of the maximum
 * under '>' (a NaN never replaces the running best; a NaN at index 0 stays). */
int oracle_sample_argmax(const float *logits, int n_vocab)
{
    int best = 0;
    float best_val = logits[0];
    for (int i = 1; i < n_vocab; i++) {
        if (logits[i] > best_val) {
            best_val = logits[i];
            best = i;
        }
    }
    return best;
}

/* softmax(): ops.cpp:1072-1091 (max, exp and sum, multiply by 1/sum). */
int oracle_softmax_inplace(float *x, int size)
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
    return 0;
}

/* sample_temperature(): ops.cpp:1624-1651 with the uniform draw r passed in
 * (the reference draws it from an unseeded mt19937, ops.cpp:1571-1574,
 * 1642-1643).  Scales logits by 1/T when T != 1 and T > 0, softmax in place,
 * then the first index whose running sum exceeds r; n_vocab - 1 if none. */
int oracle_sample_temperature(float *logits, int n_vocab, float temperature, float r)
{
    if (temperature != 1.0f && temperature > 0.0f) {
        float inv_temp = 1.0f / temperature;
        for (int i = 0; i < n_vocab; i++) logits[i] *= inv_temp;
    }
    oracle_softmax_inplace(logits, n_vocab);
    float cumsum = 0.0f;
    for (int i = 0; i < n_vocab; i++) {
        cumsum += logits[i];
        if (cumsum > r) return i;
    }
    return n_vocab - 1;
}

/* sample_top_p(): ops.cpp:1677-1722 with r passed in.  The reference sorts
 * the min(n, 100) most probable indices (std::partial_sort, descending; the
 * rest stay in an unspecified order); here all indices are sorted by
 * (probability descending, index ascending), which is the reference's order
 * whenever the nucleus has at most 100 tokens and no tied probabilities. */
static const float *g_sort_p;
static int cmp_desc(const void *a, const void *b)
{
    int i = *(const int *)a, j = *(const int *)b;
    float pi = g_sort_p[i], pj = g_sort_p[j];
    if (pi > pj) return -1;
    if (pi < pj) return 1;
    return (i > j) - (i < j);
}
int oracle_sample_top_p(float *logits, int n_vocab, float temperature, float top_p, float r)
{
    if (temperature != 1.0f && temperature > 0.0f) {
        float inv_temp = 1.0f / temperature;
        for (int i = 0; i < n_vocab; i++) logits[i] *= inv_temp;
    }
    oracle_softmax_inplace(logits, n_vocab);
    int *idx = (int *)malloc(sizeof(int) * (size_t)n_vocab);
    if (!idx) return -1;
    for (int i = 0; i < n_vocab; i++) idx[i] = i;
    g_sort_p = logits;
    qsort(idx, (size_t)n_vocab, sizeof(int), cmp_desc);
    float cumsum = 0.0f;
    int cutoff = 0;
    for (int i = 0; i < n_vocab; i++) {
        cumsum += logits[idx[i]];
        cutoff = i + 1;
        if (cumsum >= top_p) break;
    }
    float rr = r * cumsum;
    float running = 0.0f;
    int tok = idx[0];
    for (int i = 0; i < cutoff; i++) {
        running += logits[idx[i]];
        if (running > rr) {
            tok = idx[i];
            break;
        }
    }
    free(idx);
    return tok;
}

/* ------------------------------------------------------------ forward() */

#include "fw_model.h"

void oracle_rope(float *q, float *k, int pos, int head_dim, int n_head, int n_head_kv,
                 float freq_base);
void oracle_attention(float *out, const float *q, const float *k, const float *v,
                      float *key_cache, float *value_cache, float *att, int layer, int pos,
                      int n_ctx, int n_head, int n_head_kv, int head_dim);

/* embed_token(): reference src/forward.cpp:35-60 for the F16 and F32
 * tables (the formats the synthetic models here use). */
static int embed_token(float *out, const fw_model_t *m, int token)
{
    int n = m->n_embd;
    if (m->token_embd.type == FW_F16) {
        const uint16_t *row = (const uint16_t *)m->token_embd.data + (size_t)token * n;
        for (int i = 0; i < n; i++) out[i] = oracle_fp16_to_f32(row[i]);
    } else if (m->token_embd.type == FW_F32) {
        const float *row = (const float *)m->token_embd.data + (size_t)token * n;
        for (int i = 0; i < n; i++) out[i] = row[i];
    } else {
        return -1;
    }
    return 0;
}

/* forward(): reference src/forward.cpp:178-265, one token at position pos;
 * logits in state->logits.  Returns -1 on an unsupported format. */
int oracle_forward(const fw_model_t *m, fw_state_t *s, int token, int pos)
{
    int n_embd = m->n_embd, kv_dim = m->n_head_kv * (m->n_embd / m->n_head);
    int hd = m->n_embd / m->n_head;
    if (embed_token(s->x, m, token)) return -1;
    for (int l = 0; l < m->n_layers; l++) {
        const fw_layer_t *L = &m->layers[l];
        oracle_rmsnorm(s->xb, s->x, L->attn_norm, n_embd, m->rms_norm_eps);
        if (oracle_matmul(s->q, L->wq.data, s->xb, n_embd, n_embd, L->wq.type)) return -1;
        if (oracle_matmul(s->k, L->wk.data, s->xb, kv_dim, n_embd, L->wk.type)) return -1;
        if (oracle_matmul(s->v, L->wv.data, s->xb, kv_dim, n_embd, L->wv.type)) return -1;
        oracle_rope(s->q, s->k, pos, hd, m->n_head, m->n_head_kv, m->rope_freq_base);
        oracle_attention(s->xb2, s->q, s->k, s->v, s->key_cache, s->value_cache, s->att, l, pos,
                         m->n_ctx, m->n_head, m->n_head_kv, hd);
        if (oracle_matmul(s->xb, L->wo.data, s->xb2, n_embd, n_embd, L->wo.type)) return -1;
        oracle_vec_add(s->x, s->xb, n_embd);
        oracle_rmsnorm(s->xb, s->x, L->ffn_norm, n_embd, m->rms_norm_eps);
        if (oracle_ffn_swiglu(s->xb2, s->xb, s->hb, s->hb2, L->w_gate.data, L->w_up.data,
                              L->w_down.data, m->n_ff, n_embd, L->w_gate.type))
            return -1;
        oracle_vec_add(s->x, s->xb2, n_embd);
    }
    oracle_rmsnorm(s->x, s->x, m->output_norm, n_embd, m->rms_norm_eps);
    const fw_weight_t *w = m->output.data ? &m->output : &m->token_embd;
    return oracle_matmul(s->logits, w->data, s->x, m->n_vocab, n_embd, w->type);
}
