// ops_gpu.h -- C++20 host layer above the C ABI, shaped like the reference's
// ops.h / run_state.h so forward.cpp changes only where its pointers live.
//
//   reference (src/ops.h)                      this header
//   rope(q, k, pos, hd, nh, nkv, base)          tle::rope_gpu(...)        ops.h:175-176
//   attention(out, q, k, v, Kc, Vc, att,        tle::attention_gpu(...)   ops.h:204-206
//             layer, pos, cfg)
//   rope + attention (forward.cpp:192-208)      tle::rope_attention_gpu(...)
//   RunState (run_state.h:27-182)               tle::DeviceRunState
//   matmul(out, W, x, rows, cols, type)         tle::matmul_gpu(...)      ops.h:64-66
//   rmsnorm / vec_add / ffn_swiglu              tle::rmsnorm_gpu, ...     ops.h:95-96, 143, 232-235
//   sample_argmax(logits, n_vocab)              tle::sample_argmax_gpu    ops.h:249
//   sample_temperature / sample_top_p           tle::sample_*_gpu         ops.h:262, 278
//   forward(model, state, token, pos)           tle::forward_gpu          forward.h:16
//
// All pointers are device pointers.  Errors throw std::runtime_error, the
// reference's convention (e.g. ops.cpp:978-979, forward.cpp:143-145).
#pragma once

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <type_traits>
#include <vector>

#include "tle_attn.h"
#include "tle_forward.h"

namespace tle {

// The llama_config_t fields (reference src/gguf.h:139-168) attention reads.
struct AttnConfig {
    std::uint32_t n_layers = 0;
    std::uint32_t n_embd = 0;
    std::uint32_t n_head = 0;
    std::uint32_t n_head_kv = 0;
    std::uint32_t n_ctx = 2048;
    float rope_freq_base = 10000.0f;
    std::uint32_t head_dim() const { return n_head > 0 ? n_embd / n_head : 0; }
};

// Accepts the reference's llama_config_t (or anything with the same fields).
template <class Cfg>
AttnConfig to_attn_config(const Cfg& c) {
    AttnConfig a;
    a.n_layers = c.n_layers;
    a.n_embd = c.n_embd;
    a.n_head = c.n_head;
    a.n_head_kv = c.n_head_kv;
    a.n_ctx = c.n_ctx;
    a.rope_freq_base = c.rope_freq_base;
    return a;
}

inline void check(int rc) {
    if (rc != TLE_OK) throw std::runtime_error(std::string("tle: ") + tle_last_error());
}

inline tle_shape_t shape_of(const AttnConfig& c) {
    tle_shape_t s;
    s.n_layers = static_cast<int32_t>(c.n_layers);
    s.n_head = static_cast<int32_t>(c.n_head);
    s.n_head_kv = static_cast<int32_t>(c.n_head_kv);
    s.head_dim = static_cast<int32_t>(c.head_dim());
    s.rope_freq_base = c.rope_freq_base;
    return s;
}

// ops.h:175-176, in place on device q/k.
void rope_gpu(float* q, float* k, int pos, int head_dim, int n_head, int n_head_kv, float freq_base,
              void* stream = nullptr);

// ops.h:204-206 with device pointers.  `att` is the reference's score
// scratch (run_state.h:64, 126: n_ctx floats); it is accepted so forward.cpp's
// call sites stay as they are, and it is never read or written (it may be
// null).  The split-K scratch of the call is owned by this layer instead:
// one device buffer per (device, stream), made by the first
// call on that pair (so make that call outside stream capture) and grown,
// after synchronising the device, when a larger n_ctx needs more; it lives
// until the process exits.  Calls on one stream are ordered and share it;
// calls from several host threads on the same stream race, as the
// reference's shared `att` does.
void attention_gpu(float* out, const float* q, const float* k, const float* v, float* key_cache,
                   float* value_cache, float* att, int layer, int pos, const AttnConfig& cfg,
                   void* stream = nullptr);

// forward.cpp:192-208 fused: q, k unrotated (left unmodified).
void rope_attention_gpu(float* out, const float* q, const float* k, const float* v,
                        float* key_cache, float* value_cache, float* att, int layer, int pos,
                        const AttnConfig& cfg, void* stream = nullptr);

// ---- the forward pass around attention (tle_forward.h) ----
// Weights are device copies of the GGUF tensor bytes; `type` is the ggml
// type (the reference's ggml_type enum converts implicitly through the
// template overloads).
void matmul_gpu(float* out, const void* W, const float* x, int rows, int cols, int type,
                void* stream = nullptr);
void rmsnorm_gpu(float* out, const float* x, const float* weight, int size, float eps,
                 void* stream = nullptr);
void vec_add_gpu(float* out, const float* x, int size, void* stream = nullptr);
void ffn_swiglu_gpu(float* out, const float* input, float* hb, float* hb2, const void* W_gate,
                    const void* W_up, const void* W_down, int n_ff, int n_embd, int type,
                    void* stream = nullptr);
// ops.h:249 returns the token on the host (synchronises); the tle_sample_argmax
// C call leaves it in device memory for a device-fed loop.
int sample_argmax_gpu(const float* logits, int n_vocab, void* stream = nullptr);
// ops.h:262 / 278: the uniform draw comes from a std::mt19937 this layer
// holds, seeded by std::random_device like the reference's get_rng()
// (ops.cpp:1571-1574), drawn with std::uniform_real_distribution<float>;
// logits become probabilities; the token is returned on the host.
int sample_temperature_gpu(float* logits, int n_vocab, float temperature, void* stream = nullptr);
int sample_top_p_gpu(float* logits, int n_vocab, float temperature, float top_p,
                     void* stream = nullptr);
template <class E, class = std::enable_if_t<std::is_enum_v<E>>>
void matmul_gpu(float* out, const void* W, const float* x, int rows, int cols, E type,
                void* stream = nullptr) {
    matmul_gpu(out, W, x, rows, cols, static_cast<int>(type), stream);
}
template <class E, class = std::enable_if_t<std::is_enum_v<E>>>
void ffn_swiglu_gpu(float* out, const float* input, float* hb, float* hb2, const void* W_gate,
                    const void* W_up, const void* W_down, int n_ff, int n_embd, E type,
                    void* stream = nullptr) {
    ffn_swiglu_gpu(out, input, hb, hb2, W_gate, W_up, W_down, n_ff, n_embd, static_cast<int>(type),
                   stream);
}
// forward.h:16 for the token *token (device int32) at position pos.
void forward_gpu(const tle_model_t& model, const tle_state_t& state, const int32_t* token, int pos,
                 void* stream = nullptr);

// Device-memory helpers so C++ callers need no CUDA headers of their own.
float* device_alloc_floats(std::size_t n);
void* device_alloc_bytes(std::size_t n);
void copy_bytes_to_device(void* dst, const void* src, std::size_t n);
void copy_bytes_to_host(void* dst, const void* src, std::size_t n);
void device_free(void* p);
void copy_to_device(float* dst, const float* src, std::size_t n);
void copy_to_host(float* dst, const float* src, std::size_t n);
void device_zero(float* p, std::size_t n);
void device_sync();

// run_state.h:27-182 for the attention block, in HBM: q/k/v/xb2 activations,
// the [n_layers][n_ctx][kv_dim] fp32 KV cache (zeroed, run_state.h:152-153)
// and `att`, n_ctx floats as the reference allocates it (run_state.h:126;
// attention_gpu leaves it untouched).
struct DeviceRunState {
    float* xb2 = nullptr;  // attention output [n_embd]
    float* q = nullptr;    // [n_embd]
    float* k = nullptr;    // [kv_dim]
    float* v = nullptr;    // [kv_dim]
    float* att = nullptr;  // [n_ctx], the reference's score scratch
    float* key_cache = nullptr;
    float* value_cache = nullptr;
    int pos = 0;

    DeviceRunState() = default;
    DeviceRunState(const DeviceRunState&) = delete;
    DeviceRunState& operator=(const DeviceRunState&) = delete;
    ~DeviceRunState() { free_buffers(); }

    void allocate(const AttnConfig& cfg);
    void free_buffers();
};

// Many independent sequences decoded together (batched decode).
class DecodeBatch {
public:
    DecodeBatch(const AttnConfig& cfg, std::vector<tle_seq_t> seqs, int max_ctas = 0);
    ~DecodeBatch();
    DecodeBatch(const DecodeBatch&) = delete;
    DecodeBatch& operator=(const DecodeBatch&) = delete;

    // Re-plans after positions change (e.g. every decode step: pos += 1).
    void set_positions(const std::vector<int32_t>& pos);
    // One layer of decode for all sequences; q/k/v/out are device arrays
    // [n][n_embd], [n][kv_dim], [n][kv_dim], [n][n_embd].
    void run(const float* q, const float* k, const float* v, float* out, int layer, bool rotate,
             void* stream = nullptr);
    int n_ctas() const { return n_ctas_; }
    int n_seqs() const { return static_cast<int>(seqs_.size()); }

private:
    void upload();
    tle_shape_t shape_;
    std::vector<tle_seq_t> seqs_;
    int max_ctas_;
    int n_ctas_ = 0;
    std::vector<unsigned char> desc_host_;
    void* desc_dev_ = nullptr;
    std::size_t desc_cap_ = 0;
    void* ws_ = nullptr;
    std::size_t ws_bytes_ = 0;
};

}  // namespace tle
