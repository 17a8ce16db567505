// ops_gpu.cpp -- implementation of the ops.h-shaped C++ layer (ops_gpu.h).
#include "ops_gpu.h"

#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <random>
#include <utility>

namespace tle {

namespace {
void cuda_check(cudaError_t e, const char* what) {
    if (e != cudaSuccess)
        throw std::runtime_error(std::string("tle: ") + what + ": " + cudaGetErrorString(e));
}
}  // namespace

namespace {
// Split-K scratch of attention_gpu / rope_attention_gpu, one per (device,
// stream): the caller's `att` (n_ctx floats in the reference) is smaller
// than the partials of a split over the SMs, so it is never used.
struct SplitScratch {
    void* p = nullptr;
    std::size_t bytes = 0;
};
std::mutex& scratch_mutex() {
    static std::mutex m;
    return m;
}
std::map<std::pair<int, void*>, SplitScratch>& scratch_map() {
    static std::map<std::pair<int, void*>, SplitScratch> m;
    return m;
}
void* split_scratch(const tle_shape_t& s, int n_ctx, void* stream, std::size_t* bytes) {
    const std::size_t need = tle_attention_workspace_bytes(&s, n_ctx);
    int dev = 0;
    cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
    std::lock_guard<std::mutex> lock(scratch_mutex());
    SplitScratch& w = scratch_map()[{dev, stream}];
    if (w.bytes < need) {
        if (w.p) {
            // an earlier call may still read it
            cuda_check(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
            cudaFree(w.p);
            w = SplitScratch{};
        }
        cuda_check(cudaMalloc(&w.p, need), "cudaMalloc split-K scratch");
        w.bytes = need;
    }
    *bytes = w.bytes;
    return w.p;
}
}  // namespace

void rope_gpu(float* q, float* k, int pos, int head_dim, int n_head, int n_head_kv, float freq_base,
              void* stream) {
    check(tle_rope(q, k, pos, head_dim, n_head, n_head_kv, freq_base, stream));
}

void attention_gpu(float* out, const float* q, const float* k, const float* v, float* key_cache,
                   float* value_cache, float* /*att*/, int layer, int pos, const AttnConfig& cfg,
                   void* stream) {
    const tle_shape_t s = shape_of(cfg);
    std::size_t ws_bytes = 0;
    void* ws = split_scratch(s, static_cast<int>(cfg.n_ctx), stream, &ws_bytes);
    check(tle_attention(out, q, k, v, key_cache, value_cache, layer, pos, static_cast<int>(cfg.n_ctx),
                        &s, ws, ws_bytes, stream));
}

void rope_attention_gpu(float* out, const float* q, const float* k, const float* v,
                        float* key_cache, float* value_cache, float* /*att*/, int layer, int pos,
                        const AttnConfig& cfg, void* stream) {
    const tle_shape_t s = shape_of(cfg);
    std::size_t ws_bytes = 0;
    void* ws = split_scratch(s, static_cast<int>(cfg.n_ctx), stream, &ws_bytes);
    check(tle_rope_attention(out, q, k, v, key_cache, value_cache, layer, pos,
                             static_cast<int>(cfg.n_ctx), &s, ws, ws_bytes, stream));
}

void matmul_gpu(float* out, const void* W, const float* x, int rows, int cols, int type, void* stream) {
    check(tle_matmul(out, W, x, rows, cols, type, stream));
}

void rmsnorm_gpu(float* out, const float* x, const float* weight, int size, float eps, void* stream) {
    check(tle_rmsnorm(out, x, weight, size, eps, stream));
}

void vec_add_gpu(float* out, const float* x, int size, void* stream) {
    check(tle_vec_add(out, x, size, stream));
}

void ffn_swiglu_gpu(float* out, const float* input, float* hb, float* hb2, const void* W_gate,
                    const void* W_up, const void* W_down, int n_ff, int n_embd, int type,
                    void* stream) {
    check(tle_ffn_swiglu(out, input, hb, hb2, W_gate, W_up, W_down, n_ff, n_embd, type, stream));
}

int sample_argmax_gpu(const float* logits, int n_vocab, void* stream) {
    int32_t* d = static_cast<int32_t*>(device_alloc_bytes(sizeof(int32_t)));
    int32_t h = 0;
    try {
        check(tle_sample_argmax(logits, n_vocab, d, stream));
        cuda_check(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "sync");
        copy_bytes_to_host(&h, d, sizeof h);
    } catch (...) {
        device_free(d);
        throw;
    }
    device_free(d);
    return h;
}

namespace {
std::mt19937& layer_rng() {
    static std::mt19937 rng(std::random_device{}());
    return rng;
}
template <class F>
int sample_to_host(F&& launch, void* stream) {
    int32_t* d = static_cast<int32_t*>(device_alloc_bytes(sizeof(int32_t)));
    int32_t h = 0;
    try {
        check(launch(d));
        cuda_check(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "sync");
        copy_bytes_to_host(&h, d, sizeof h);
    } catch (...) {
        device_free(d);
        throw;
    }
    device_free(d);
    return h;
}
}  // namespace

int sample_temperature_gpu(float* logits, int n_vocab, float temperature, void* stream) {
    std::uniform_real_distribution<float> dist(0.0f, 1.0f);
    const float r = dist(layer_rng());
    return sample_to_host(
        [&](int32_t* d) { return tle_sample_temperature(logits, n_vocab, temperature, r, d, stream); }, stream);
}

int sample_top_p_gpu(float* logits, int n_vocab, float temperature, float top_p, void* stream) {
    std::uniform_real_distribution<float> dist(0.0f, 1.0f);
    const float r = dist(layer_rng());
    return sample_to_host(
        [&](int32_t* d) { return tle_sample_top_p(logits, n_vocab, temperature, top_p, r, d, stream); }, stream);
}

void forward_gpu(const tle_model_t& model, const tle_state_t& state, const int32_t* token, int pos,
                 void* stream) {
    check(tle_forward(&model, &state, token, pos, stream));
}

void* device_alloc_bytes(std::size_t n) {
    void* p = nullptr;
    cuda_check(cudaMalloc(&p, std::max<std::size_t>(n, 1)), "cudaMalloc");
    return p;
}
void copy_bytes_to_device(void* dst, const void* src, std::size_t n) {
    cuda_check(cudaMemcpy(dst, src, n, cudaMemcpyHostToDevice), "cudaMemcpy H2D");
}
void copy_bytes_to_host(void* dst, const void* src, std::size_t n) {
    cuda_check(cudaMemcpy(dst, src, n, cudaMemcpyDeviceToHost), "cudaMemcpy D2H");
}

float* device_alloc_floats(std::size_t n) {
    void* p = nullptr;
    cuda_check(cudaMalloc(&p, std::max<std::size_t>(n, 1) * sizeof(float)), "cudaMalloc");
    return static_cast<float*>(p);
}
void device_free(void* p) {
    if (p) cudaFree(p);
}
void copy_to_device(float* dst, const float* src, std::size_t n) {
    cuda_check(cudaMemcpy(dst, src, n * sizeof(float), cudaMemcpyHostToDevice), "cudaMemcpy H2D");
}
void copy_to_host(float* dst, const float* src, std::size_t n) {
    cuda_check(cudaMemcpy(dst, src, n * sizeof(float), cudaMemcpyDeviceToHost), "cudaMemcpy D2H");
}
void device_zero(float* p, std::size_t n) {
    cuda_check(cudaMemset(p, 0, n * sizeof(float)), "cudaMemset");
}
void device_sync() { cuda_check(cudaDeviceSynchronize(), "cudaDeviceSynchronize"); }

void DeviceRunState::allocate(const AttnConfig& cfg) {
    free_buffers();
    const std::size_t hd = cfg.head_dim(), kv_dim = cfg.n_head_kv * hd;
    const std::size_t cache = static_cast<std::size_t>(cfg.n_layers) * cfg.n_ctx * kv_dim;
    xb2 = device_alloc_floats(cfg.n_embd);
    q = device_alloc_floats(cfg.n_embd);
    k = device_alloc_floats(kv_dim);
    v = device_alloc_floats(kv_dim);
    att = device_alloc_floats(cfg.n_ctx);
    key_cache = device_alloc_floats(cache);
    value_cache = device_alloc_floats(cache);
    for (auto [p, n] : {std::pair{xb2, std::size_t(cfg.n_embd)}, std::pair{q, std::size_t(cfg.n_embd)},
                        std::pair{k, kv_dim}, std::pair{v, kv_dim}, std::pair{att, std::size_t(cfg.n_ctx)},
                        std::pair{key_cache, cache},
                        std::pair{value_cache, cache}})
        device_zero(p, n);
    pos = 0;
}

void DeviceRunState::free_buffers() {
    for (float** p : {&xb2, &q, &k, &v, &att, &key_cache, &value_cache}) {
        device_free(*p);
        *p = nullptr;
    }
}

DecodeBatch::DecodeBatch(const AttnConfig& cfg, std::vector<tle_seq_t> seqs, int max_ctas)
    : shape_(shape_of(cfg)), seqs_(std::move(seqs)), max_ctas_(max_ctas) {
    if (seqs_.empty()) throw std::runtime_error("tle: DecodeBatch needs at least one sequence");
    upload();
}

DecodeBatch::~DecodeBatch() {
    device_free(desc_dev_);
    device_free(ws_);
}

void DecodeBatch::set_positions(const std::vector<int32_t>& pos) {
    if (pos.size() != seqs_.size()) throw std::runtime_error("tle: position count mismatch");
    for (std::size_t i = 0; i < pos.size(); ++i) seqs_[i].pos = pos[i];
    upload();
}

void DecodeBatch::upload() {
    const int n = static_cast<int>(seqs_.size());
    const std::size_t bytes = tle_decode_desc_bytes(n, max_ctas_);
    desc_host_.assign(bytes, 0);
    check(tle_decode_desc(&shape_, seqs_.data(), n, max_ctas_, desc_host_.data(), bytes, &n_ctas_));
    if (bytes > desc_cap_) {
        device_free(desc_dev_);
        desc_dev_ = nullptr;
        cuda_check(cudaMalloc(&desc_dev_, bytes), "cudaMalloc desc");
        desc_cap_ = bytes;
    }
    cuda_check(cudaMemcpy(desc_dev_, desc_host_.data(), bytes, cudaMemcpyHostToDevice), "desc upload");
    const std::size_t ws = tle_decode_workspace_bytes(&shape_, n, n_ctas_);
    if (ws > ws_bytes_) {
        device_free(ws_);
        ws_ = nullptr;
        cuda_check(cudaMalloc(&ws_, ws), "cudaMalloc workspace");
        ws_bytes_ = ws;
    }
}

void DecodeBatch::run(const float* q, const float* k, const float* v, float* out, int layer,
                      bool rotate, void* stream) {
    check(tle_decode_batch(&shape_, desc_dev_, static_cast<int>(seqs_.size()), n_ctas_, q, k, v, out,
                           layer, rotate ? 1 : 0, ws_, ws_bytes_, stream));
}

}  // namespace tle
