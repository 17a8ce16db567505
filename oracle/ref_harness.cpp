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

}  // extern "C"
