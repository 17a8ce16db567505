// ref_harness.cpp -- C-ABI harness around the reference's own rope()/attention().
//
// TEST INFRASTRUCTURE ONLY.  It is compiled together with the reference's
// unmodified src/ops.cpp (taken from where it lies in the reference tree, never
// copied) into oracle/_ref/libref_attn.so by oracle/Makefile.  Tests use it
// to pin the C restatement (oracle/attn_oracle.c); bench.py uses it as the
// timed CPU baseline ("kind": "reference").  Nothing in the product links it.
//
// Every entry point builds an llama_config_t (reference src/gguf.h:139-168)
// and calls the reference functions exactly as forward.cpp:192-208 does.
#include <algorithm>
#include <atomic>
#include <cstddef>
#include <thread>
#include <vector>

#include "fw_model.h"
#include "ops.h"

namespace {
llama_config_t make_cfg(int n_layers, int n_head, int n_head_kv, int head_dim, int n_ctx,
                        float freq_base) {
    llama_config_t cfg;
    cfg.n_layers = static_cast<std::uint32_t>(n_layers);
    cfg.n_embd = static_cast<std::uint32_t>(n_head * head_dim);
    cfg.n_head = static_cast<std::uint32_t>(n_head);
    cfg.n_head_kv = static_cast<std::uint32_t>(n_head_kv);
    cfg.n_ctx = static_cast<std::uint32_t>(n_ctx);
    cfg.rope_freq_base = freq_base;
    return cfg;
}
}  // namespace

extern "C" {

// ops.h:175-176
void ref_rope(float* q, float* k, int pos, int head_dim, int n_head, int n_head_kv,
              float freq_base) {
    rope(q, k, pos, head_dim, n_head, n_head_kv, freq_base);
}

// ops.h:107
void ref_softmax(float* x, int size) { softmax(x, size); }

// ops.h:204-206
void ref_attention(float* out, const float* q, const float* k, const float* v, float* key_cache,
                   float* value_cache, float* att, int layer, int pos, int n_layers, int n_ctx,
                   int n_head, int n_head_kv, int head_dim) {
    llama_config_t cfg = make_cfg(n_layers, n_head, n_head_kv, head_dim, n_ctx, 10000.0f);
    attention(out, q, k, v, key_cache, value_cache, att, layer, pos, cfg);
}

// The reference's prefill: one rope+attention step per prompt token
// (generate.cpp:56-59 driving forward.cpp:192-208).
void ref_prefill(float* out, float* q, float* k, const float* v, float* key_cache,
                 float* value_cache, int layer, int pos0, int n_tokens, int n_layers, int n_ctx,
                 int n_head, int n_head_kv, int head_dim, float freq_base) {
    llama_config_t cfg = make_cfg(n_layers, n_head, n_head_kv, head_dim, n_ctx, freq_base);
    const int q_dim = n_head * head_dim, kv_dim = n_head_kv * head_dim;
    std::vector<float> att(static_cast<size_t>(n_ctx));
    for (int i = 0; i < n_tokens; i++) {
        float* qi = q + static_cast<size_t>(i) * q_dim;
        float* ki = k + static_cast<size_t>(i) * kv_dim;
        rope(qi, ki, pos0 + i, head_dim, n_head, n_head_kv, freq_base);
        attention(out + static_cast<size_t>(i) * q_dim, qi, ki, v + static_cast<size_t>(i) * kv_dim,
                  key_cache, value_cache, att.data(), layer, pos0 + i, cfg);
    }
}

// Batched decode over independent sequences for one layer, spread over
// n_threads std::threads (attention() itself is single-threaded and needs a
// private att scratch per caller, run_state.h:64).  Each sequence s has its
// own cache [n_layers][n_ctx[s]][kv_dim].
void ref_decode_batch(int n_seqs, float* const* key_caches, float* const* value_caches,
                      const int* n_ctx, const int* pos, float* q, float* k, const float* v,
                      float* out, int layer, int n_layers, int n_head, int n_head_kv,
                      int head_dim, float freq_base, int n_threads) {
    const int q_dim = n_head * head_dim, kv_dim = n_head_kv * head_dim;
    int max_ctx = 1;
    for (int s = 0; s < n_seqs; s++) max_ctx = std::max(max_ctx, n_ctx[s]);
    std::atomic<int> next{0};
    auto worker = [&]() {
        std::vector<float> att(static_cast<size_t>(max_ctx));
        for (;;) {
            int s = next.fetch_add(1);
            if (s >= n_seqs) break;
            llama_config_t cfg =
                make_cfg(n_layers, n_head, n_head_kv, head_dim, n_ctx[s], freq_base);
            float* qs = q + static_cast<size_t>(s) * q_dim;
            float* ks = k + static_cast<size_t>(s) * kv_dim;
            rope(qs, ks, pos[s], head_dim, n_head, n_head_kv, freq_base);
            attention(out + static_cast<size_t>(s) * q_dim, qs, ks,
                      v + static_cast<size_t>(s) * kv_dim, key_caches[s], value_caches[s],
                      att.data(), layer, pos[s], cfg);
        }
    };
    n_threads = std::max(1, std::min(n_threads, n_seqs));
    std::vector<std::thread> th;
    for (int t = 1; t < n_threads; t++) th.emplace_back(worker);
    worker();
    for (auto& t : th) t.join();
}

// ---- the forward pass around attention (ops.h:39-143, 232-249) ----

// ops.h:39
float ref_fp16_to_f32(std::uint16_t h) { return fp16_to_f32(h); }

// ops.h:64-66 (matmul throws on an unsupported type: -1 here)
int ref_matmul(float* out, const void* W, const float* x, int rows, int cols, int type) {
    try {
        matmul(out, W, x, rows, cols, static_cast<ggml_type>(type));
    } catch (...) {
        return -1;
    }
    return 0;
}

// ops.h:95-96, 118, 130, 143
void ref_rmsnorm(float* out, const float* x, const float* weight, int size, float eps) {
    rmsnorm(out, x, weight, size, eps);
}
void ref_silu(float* x, int size) { silu(x, size); }
void ref_elementwise_mul(float* a, const float* b, int size) { elementwise_mul(a, b, size); }
void ref_vec_add(float* out, const float* x, int size) { vec_add(out, x, size); }

// ops.h:232-235
int ref_ffn_swiglu(float* out, const float* input, float* hb, float* hb2, const void* W_gate,
                   const void* W_up, const void* W_down, int n_ff, int n_embd, int type) {
    try {
        ffn_swiglu(out, input, hb, hb2, W_gate, W_up, W_down, n_ff, n_embd,
                   static_cast<ggml_type>(type));
    } catch (...) {
        return -1;
    }
    return 0;
}

// ops.h:249
int ref_sample_argmax(const float* logits, int n_vocab) { return sample_argmax(logits, n_vocab); }

void ref_set_num_threads(int n) { set_num_threads(n); }

// ops.h:262, 278 as the reference runs them: the uniform draw comes from its
// own unseeded generator (ops.cpp:1571), so these are nondeterministic.
int ref_sample_temperature(float* logits, int n_vocab, float temperature) {
    return sample_temperature(logits, n_vocab, temperature);
}
int ref_sample_top_p(float* logits, int n_vocab, float temperature, float top_p) {
    return sample_top_p(logits, n_vocab, temperature, top_p);
}

// forward() (src/forward.cpp:178-265) composed from the reference's own ops
// in the same order, for one token at position pos.  The embedding lookup is
// embed_token() (forward.cpp:35-60, static there) for F16/F32 tables through
// the reference's fp16_to_f32.  Returns -1 on an unsupported format.
int ref_forward(const fw_model_t* m, fw_state_t* s, int token, int pos) {
    const int n_embd = m->n_embd, hd = m->n_embd / m->n_head, kv_dim = m->n_head_kv * hd;
    llama_config_t cfg = make_cfg(m->n_layers, m->n_head, m->n_head_kv, hd, m->n_ctx,
                                  m->rope_freq_base);
    cfg.n_ff = static_cast<std::uint32_t>(m->n_ff);
    cfg.n_vocab = static_cast<std::uint32_t>(m->n_vocab);
    cfg.rms_norm_eps = m->rms_norm_eps;
    try {
        if (m->token_embd.type == 1) {
            const auto* row = static_cast<const std::uint16_t*>(m->token_embd.data) +
                              static_cast<size_t>(token) * n_embd;
            for (int i = 0; i < n_embd; i++) s->x[i] = fp16_to_f32(row[i]);
        } else if (m->token_embd.type == 0) {
            const auto* row = static_cast<const float*>(m->token_embd.data) +
                              static_cast<size_t>(token) * n_embd;
            for (int i = 0; i < n_embd; i++) s->x[i] = row[i];
        } else {
            return -1;
        }
        for (int l = 0; l < m->n_layers; l++) {
            const fw_layer_t& L = m->layers[l];
            rmsnorm(s->xb, s->x, L.attn_norm, n_embd, cfg.rms_norm_eps);
            matmul(s->q, L.wq.data, s->xb, n_embd, n_embd, static_cast<ggml_type>(L.wq.type));
            matmul(s->k, L.wk.data, s->xb, kv_dim, n_embd, static_cast<ggml_type>(L.wk.type));
            matmul(s->v, L.wv.data, s->xb, kv_dim, n_embd, static_cast<ggml_type>(L.wv.type));
            rope(s->q, s->k, pos, hd, m->n_head, m->n_head_kv, cfg.rope_freq_base);
            attention(s->xb2, s->q, s->k, s->v, s->key_cache, s->value_cache, s->att, l, pos, cfg);
            matmul(s->xb, L.wo.data, s->xb2, n_embd, n_embd, static_cast<ggml_type>(L.wo.type));
            vec_add(s->x, s->xb, n_embd);
            rmsnorm(s->xb, s->x, L.ffn_norm, n_embd, cfg.rms_norm_eps);
            ffn_swiglu(s->xb2, s->xb, s->hb, s->hb2, L.w_gate.data, L.w_up.data, L.w_down.data,
                       m->n_ff, n_embd, static_cast<ggml_type>(L.w_gate.type));
            vec_add(s->x, s->xb2, n_embd);
        }
        rmsnorm(s->x, s->x, m->output_norm, n_embd, cfg.rms_norm_eps);
        const fw_weight_t& w = m->output.data ? m->output : m->token_embd;
        matmul(s->logits, w.data, s->x, m->n_vocab, n_embd, static_cast<ggml_type>(w.type));
    } catch (...) {
        return -1;
    }
    return 0;
}

}  // extern "C"
