// test_ops_gpu.cpp -- the reference's attention and rope test groups
// (src/test_ops.cpp:295-546) run through the C++ layer of this library
// (tinyllama-engine_b200/host/ops_gpu.h), i.e. the call surface a forward.cpp
// built on device buffers uses.  Same check()/approx_equal() conventions and
// the same exit status contract (non-zero on failure) as the reference suite.
#include <cmath>
#include <cstdio>
#include <iostream>
#include <vector>

#include "ops_gpu.h"

namespace {

int tests_passed = 0;
int tests_failed = 0;

bool approx_equal(float a, float b, float tol = 1e-4f) { return std::fabs(a - b) < tol; }

void check(const char* name, bool condition) {
    if (condition) {
        std::cout << "  ok   " << name << "\n";
        ++tests_passed;
    } else {
        std::cout << "  FAIL " << name << "\n";
        ++tests_failed;
    }
}

struct Dev {
    float* p = nullptr;
    std::size_t n = 0;
    explicit Dev(std::size_t count) : p(tle::device_alloc_floats(count)), n(count) { tle::device_zero(p, n); }
    ~Dev() { tle::device_free(p); }
    void put(const std::vector<float>& h) { tle::copy_to_device(p, h.data(), h.size()); }
    std::vector<float> get() const {
        std::vector<float> h(n);
        tle::copy_to_host(h.data(), p, n);
        return h;
    }
};

tle::AttnConfig tinyllama(std::uint32_t n_layers, std::uint32_t n_ctx) {
    tle::AttnConfig c;
    c.n_layers = n_layers;
    c.n_embd = 2048;
    c.n_head = 32;
    c.n_head_kv = 4;
    c.n_ctx = n_ctx;
    return c;
}

void test_attention() {
    std::cout << "\n=== attention (device) ===\n";
    const tle::AttnConfig cfg = tinyllama(2, 64);
    const int head_dim = 64, kv_dim = 256, n_embd = 2048;
    tle::DeviceRunState st;
    st.allocate(cfg);
    Dev out(n_embd);
    std::vector<float> q(n_embd), k(kv_dim), v(kv_dim);
    const std::size_t cache = 2ull * 64 * kv_dim;

    // T1 single token -> output == v (test_ops.cpp:326-351)
    for (auto& x : q) x = 1.0f;
    for (auto& x : k) x = 1.0f;
    for (int i = 0; i < kv_dim; ++i) v[i] = static_cast<float>(i % head_dim);
    Dev dq(n_embd), dk(kv_dim), dv(kv_dim);
    dq.put(q); dk.put(k); dv.put(v);
    tle::attention_gpu(out.p, dq.p, dk.p, dv.p, st.key_cache, st.value_cache, st.att, 0, 0, cfg);
    std::vector<float> o = out.get();
    bool ok = true;
    for (int d = 0; d < head_dim; ++d) ok = ok && approx_equal(o[d], static_cast<float>(d), 1e-3f);
    check("single token: output = value (100% self-attention)", ok);

    // T2 two equal keys -> 50/50 blend (test_ops.cpp:354-376)
    tle::device_zero(st.key_cache, cache);
    tle::device_zero(st.value_cache, cache);
    for (auto& x : v) x = 1.0f;
    dv.put(v);
    tle::attention_gpu(out.p, dq.p, dk.p, dv.p, st.key_cache, st.value_cache, st.att, 0, 0, cfg);
    for (auto& x : v) x = 3.0f;
    dv.put(v);
    tle::attention_gpu(out.p, dq.p, dk.p, dv.p, st.key_cache, st.value_cache, st.att, 0, 1, cfg);
    o = out.get();
    check("uniform attention: 50/50 blend -> 2.0", approx_equal(o[0], 2.0f, 0.01f));

    // T3 10 tokens -> no NaN/Inf (test_ops.cpp:379-400)
    tle::device_zero(st.key_cache, cache);
    tle::device_zero(st.value_cache, cache);
    for (int p = 0; p < 10; ++p) {
        for (int i = 0; i < n_embd; ++i) q[i] = static_cast<float>((i + p) % 11) - 5.0f;
        for (int i = 0; i < kv_dim; ++i) {
            k[i] = static_cast<float>((i + p * 3) % 7) - 3.0f;
            v[i] = static_cast<float>((i + p * 5) % 9) - 4.0f;
        }
        dq.put(q); dk.put(k); dv.put(v);
        tle::attention_gpu(out.p, dq.p, dk.p, dv.p, st.key_cache, st.value_cache, st.att, 0, p, cfg);
    }
    o = out.get();
    ok = true;
    for (float x : o) ok = ok && std::isfinite(x);
    check("10 tokens: no NaN/Inf in output", ok);

    // T4 GQA mapping (test_ops.cpp:405-430)
    tle::device_zero(st.key_cache, cache);
    tle::device_zero(st.value_cache, cache);
    for (auto& x : q) x = 1.0f;
    for (auto& x : k) x = 1.0f;
    for (auto& x : v) x = 0.0f;
    for (int d = 0; d < head_dim; ++d) {
        v[d] = 10.0f;
        v[head_dim + d] = 20.0f;
    }
    dq.put(q); dk.put(k); dv.put(v);
    tle::attention_gpu(out.p, dq.p, dk.p, dv.p, st.key_cache, st.value_cache, st.att, 0, 0, cfg);
    o = out.get();
    check("GQA: head 0 uses KV head 0 (val=10)", approx_equal(o[0], 10.0f, 0.01f));
    check("GQA: head 8 uses KV head 1 (val=20)", approx_equal(o[8 * head_dim], 20.0f, 0.01f));

    // Fused rope+attention equals rope then attention (forward.cpp:192-208)
    tle::device_zero(st.key_cache, cache);
    tle::device_zero(st.value_cache, cache);
    Dev out2(n_embd);
    for (int p = 0; p < 40; ++p) {
        for (int i = 0; i < n_embd; ++i) q[i] = std::sin(0.37f * static_cast<float>(i + 7 * p));
        for (int i = 0; i < kv_dim; ++i) {
            k[i] = std::cos(0.11f * static_cast<float>(i + 3 * p));
            v[i] = std::sin(0.05f * static_cast<float>(i * p + 1));
        }
        dq.put(q); dk.put(k); dv.put(v);
        tle::rope_attention_gpu(out2.p, dq.p, dk.p, dv.p, st.key_cache, st.value_cache, st.att, 1, p, cfg);
    }
    std::vector<float> fused = out2.get();
    tle::DeviceRunState st2;
    st2.allocate(cfg);
    for (int p = 0; p < 40; ++p) {
        for (int i = 0; i < n_embd; ++i) q[i] = std::sin(0.37f * static_cast<float>(i + 7 * p));
        for (int i = 0; i < kv_dim; ++i) {
            k[i] = std::cos(0.11f * static_cast<float>(i + 3 * p));
            v[i] = std::sin(0.05f * static_cast<float>(i * p + 1));
        }
        dq.put(q); dk.put(k); dv.put(v);
        tle::rope_gpu(dq.p, dk.p, p, 64, 32, 4, 10000.0f);
        tle::attention_gpu(out.p, dq.p, dk.p, dv.p, st2.key_cache, st2.value_cache, st2.att, 1, p, cfg);
    }
    o = out.get();
    ok = true;
    for (int i = 0; i < n_embd; ++i) ok = ok && approx_equal(o[i], fused[i], 1e-5f);
    check("fused rope+attention == rope then attention", ok);
}

void test_rope() {
    std::cout << "\n=== rope (device) ===\n";
    const int head_dim = 64, n_head = 32, n_head_kv = 4;
    const float base = 10000.0f;
    Dev dq(n_head * head_dim), dk(n_head_kv * head_dim);
    std::vector<float> q(n_head * head_dim, 1.0f), k(n_head_kv * head_dim, 1.0f);
    dq.put(q); dk.put(k);
    tle::rope_gpu(dq.p, dk.p, 0, head_dim, n_head, n_head_kv, base);
    std::vector<float> qo = dq.get(), ko = dk.get();
    bool qu = true, ku = true;
    for (float x : qo) qu = qu && approx_equal(x, 1.0f);
    for (float x : ko) ku = ku && approx_equal(x, 1.0f);
    check("position 0: Q unchanged", qu);
    check("position 0: K unchanged", ku);

    for (int i = 0; i < n_head * head_dim; ++i) q[i] = static_cast<float>(i % 7) - 3.0f;
    float nb = 0.f;
    for (int i = 0; i < head_dim; ++i) nb += q[i] * q[i];
    dq.put(q);
    tle::rope_gpu(dq.p, dk.p, 42, head_dim, n_head, n_head_kv, base);
    qo = dq.get();
    float na = 0.f;
    for (int i = 0; i < head_dim; ++i) na += qo[i] * qo[i];
    check("rotation preserves vector length", approx_equal(std::sqrt(nb), std::sqrt(na), 1e-3f));

    std::vector<float> zq(n_head * head_dim, 0.0f), zk(n_head_kv * head_dim, 0.0f);
    zq[0] = 3.0f;
    zq[1] = 4.0f;
    dq.put(zq); dk.put(zk);
    tle::rope_gpu(dq.p, dk.p, 1, head_dim, n_head, n_head_kv, base);
    qo = dq.get();
    check("manual rotation q[0]", approx_equal(qo[0], 3.0f * std::cos(1.0f) - 4.0f * std::sin(1.0f)));
    check("manual rotation q[1]", approx_equal(qo[1], 3.0f * std::sin(1.0f) + 4.0f * std::cos(1.0f)));
}

void test_errors() {
    std::cout << "\n=== error reporting ===\n";
    const tle::AttnConfig cfg = tinyllama(1, 8);
    tle::DeviceRunState st;
    st.allocate(cfg);
    bool threw = false;
    try {
        tle::attention_gpu(st.xb2, st.q, st.k, st.v, st.key_cache, st.value_cache, st.att, 0, 8, cfg);
    } catch (const std::runtime_error&) {
        threw = true;
    }
    check("pos >= n_ctx throws std::runtime_error", threw);
    tle::AttnConfig bad = cfg;
    bad.n_head = 16;
    bad.n_embd = 1024;
    threw = false;
    try {
        tle::attention_gpu(st.xb2, st.q, st.k, st.v, st.key_cache, st.value_cache, st.att, 0, 1, bad);
    } catch (const std::runtime_error&) {
        threw = true;
    }
    check("unsupported head count throws", threw);
}

}  // namespace

int main() {
    try {
        test_attention();
        test_rope();
        test_errors();
        tle::device_sync();
    } catch (const std::exception& e) {
        std::cerr << "error: " << e.what() << "\n";
        return 2;
    }
    std::cout << "\n" << tests_passed << " passed, " << tests_failed << " failed\n";
    return tests_failed == 0 ? 0 : 1;
}
