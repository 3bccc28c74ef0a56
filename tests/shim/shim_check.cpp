// Test driver of include/jieyu_b200_shim.hpp (built by tests/test_gpu_shim.py
// into a scratch shared library and called through ctypes).
//
// The structs below have the members and layouts of the reference's WMat,
// LayerWeights, __KVq and __KVcache (libs/date_libs/wmat.h:32-44,
// libs/date_libs/date.h:75-147, libs/model_libs/attention/attention_q8.h:12-19),
// so every shim entry point is called exactly as the reference's code calls
// its own; each extern "C" wrapper turns the C ABI's plain arguments into
// those structs and returns 0, or -1 with the exception's message kept for
// shim_last_error().
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "jieyu_b200_shim.hpp"

namespace {

struct WMat {
    const float* f = nullptr;
    const uint16_t* h = nullptr;
    const void* q = nullptr;
    uint8_t qt = 0;
};
struct LayerWeights {
    const float* rms1_weight;
    WMat Wq, Wk, Wv, Wo;
    const float* bq;
    const float* bk;
    const float* bv;
    const float* rms2_weight;
    WMat W1, W2, W3;
};
struct KVq {
    int8_t* k;
    float* ks;
    int8_t* v;
    float* vs;
    int cap;
};
struct KVcache {
    int num_layers, max_seq, num_kv_heads, head_dim, current_len;
    std::vector<int8_t> k, v;
    std::vector<float> ks, vs;
    void init(int l, int ms, int nkh, int hd) {
        num_layers = l;
        max_seq = ms;
        num_kv_heads = nkh;
        head_dim = hd;
        current_len = 0;
        k.assign((size_t)l * ms * nkh * hd, 0);
        v.assign(k.size(), 0);
        ks.assign((size_t)l * ms * nkh, 0.0f);
        vs.assign(ks.size(), 0.0f);
    }
    int8_t* k_ptr(int l, int p) { return k.data() + ((size_t)l * max_seq + p) * num_kv_heads * head_dim; }
    int8_t* v_ptr(int l, int p) { return v.data() + ((size_t)l * max_seq + p) * num_kv_heads * head_dim; }
    float* ks_ptr(int l, int p) { return ks.data() + ((size_t)l * max_seq + p) * num_kv_heads; }
    float* vs_ptr(int l, int p) { return vs.data() + ((size_t)l * max_seq + p) * num_kv_heads; }
};

std::string g_err;

WMat wm(const jyc_wmat& w) {
    WMat m;
    m.f = w.f;
    m.h = w.h;
    m.q = w.q;
    m.qt = w.qt;
    return m;
}

template <class F>
int guarded(F f) {
    try {
        f();
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

std::vector<LayerWeights> layers_of(const jyc_model_desc* d) {
    std::vector<LayerWeights> v((size_t)d->num_layers);
    for (int l = 0; l < d->num_layers; l++) {
        const jyc_layer_weights& s = d->layers[l];
        LayerWeights& t = v[(size_t)l];
        t.rms1_weight = s.rms1_weight;
        t.Wq = wm(s.Wq);
        t.Wk = wm(s.Wk);
        t.Wv = wm(s.Wv);
        t.Wo = wm(s.Wo);
        t.bq = s.bq;
        t.bk = s.bk;
        t.bv = s.bv;
        t.rms2_weight = s.rms2_weight;
        t.W1 = wm(s.W1);
        t.W2 = wm(s.W2);
        t.W3 = wm(s.W3);
    }
    return v;
}

struct StopAfter {
    int n, seen;
};
bool stop_after(int, void* ud) {
    StopAfter* s = static_cast<StopAfter*>(ud);
    return ++s->seen >= s->n;
}

}  // namespace

extern "C" {

const char* shim_last_error() { return g_err.c_str(); }

int shim_matmul_q(const float* a, const void* b, float* c, int m, int n, int k, int t) {
    return guarded([&] { jieyu_b200::qmat::matmul_q(a, b, c, m, n, k, (uint8_t)t); });
}

int shim_matmul(int m, int n, int k, const float* A, const float* B, float* C) {
    return guarded([&] { jieyu_b200::matmul(m, n, k, A, B, C); });
}

// matmul_w over a WMat holding either fp32 [k][n] (f) or blocks of type qt (q)
int shim_matmul_w(const float* f, const void* q, int qt, int m, int n, int k, const float* A, float* C) {
    WMat w;
    w.f = f;
    w.q = q;
    w.qt = (uint8_t)qt;
    return guarded([&] { jieyu_b200::matmul_w(w, m, n, k, A, C); });
}

int shim_rmsnorm(float* x, float* y, const float* w, int n, float eps) {
    return guarded([&] { jieyu_b200::rmsnorm(x, y, w, n, eps); });
}

int shim_rope_pos(float* q, int seq, int start_pos, int heads, int hd, const float* cos_t, const float* sin_t) {
    return guarded([&] { jieyu_b200::rope_pos(q, seq, start_pos, heads, hd, cos_t, sin_t); });
}

int shim_kv_pack_q8(const float* src, int8_t* dst, float* sc, int heads, int hd, int n) {
    return guarded([&] { jieyu_b200::kv_pack_q8(src, dst, sc, heads, hd, n); });
}

int shim_attention_q8(float* Q, float* K, float* V, float* out, int seq, int start_pos, int H, int KVh, int hd,
                      int8_t* kc, float* ks, int8_t* vc, float* vs, int cap) {
    const KVq kvq{kc, ks, vc, vs, cap};
    return guarded([&] { jieyu_b200::attention_q8(Q, K, V, out, seq, start_pos, H, KVh, hd, kvq); });
}

int shim_silu(float* x, float* y, int n) {
    return guarded([&] { jieyu_b200::silu(x, y, n); });
}

int shim_ffn(float* x, const jyc_wmat* w1, const jyc_wmat* w2, const jyc_wmat* w3, float* out, int seq, int hidden,
             int inter) {
    return guarded([&] { jieyu_b200::ffn(x, wm(*w1), wm(*w2), wm(*w3), out, seq, hidden, inter); });
}

// generate() with the reference's argument list; stop_after > 0 installs a
// token callback that stops after that many tokens
int shim_generate(const jyc_model_desc* d, const int* prompt, int prompt_len, const int* eos, int num_eos,
                  int max_new, float temperature, float penalty, int stop_after_n, int* out_ids) {
    static const jyc_model_desc none{};  // a null descriptor: only generate's early returns are reachable
    if (!d) d = &none;
    const std::vector<LayerWeights> L = layers_of(d);
    int n = -1;
    StopAfter sa{stop_after_n, 0};
    const int r = guarded([&] {
        n = jieyu_b200::generate(prompt, prompt_len, eos, num_eos, wm(d->embed), wm(d->lm_head), L.data(),
                                 d->num_layers, d->final_rms_weight, d->cos_table, d->sin_table, d->max_seq,
                                 max_new, temperature, d->vocab_size, d->hidden, d->num_heads, d->num_kv_heads,
                                 d->head_dim, d->intermediate, out_ids, penalty,
                                 stop_after_n > 0 ? stop_after : nullptr, stop_after_n > 0 ? &sa : nullptr);
    });
    return r == 0 ? n : -1;
}

// generate_cached() into a __KVcache-like cache; copies layer `layer`'s rows
// [0, npos) out in the reference layout and returns the generated length
// (current_len in *cur_len)
int shim_generate_cached(const jyc_model_desc* d, const int* prompt, int prompt_len, int max_new, int* out_ids,
                         int layer, int8_t* k, float* ks, int8_t* v, float* vs, int* cur_len) {
    const std::vector<LayerWeights> L = layers_of(d);
    KVcache cache;
    cache.init(d->num_layers, d->max_seq, d->num_kv_heads, d->head_dim);
    int n = -1;
    const int r = guarded([&] {
        n = jieyu_b200::generate_cached(prompt, prompt_len, nullptr, 0, wm(d->embed), wm(d->lm_head), L.data(),
                                        d->num_layers, d->final_rms_weight, d->cos_table, d->sin_table,
                                        d->max_seq, max_new, 0.0f, d->vocab_size, d->hidden, d->num_heads,
                                        d->num_kv_heads, d->head_dim, d->intermediate, cache, out_ids);
    });
    if (r != 0) return -1;
    *cur_len = cache.current_len;
    const size_t kvd = (size_t)d->num_kv_heads * d->head_dim;
    std::memcpy(k, cache.k_ptr(layer, 0), (size_t)cache.current_len * kvd);
    std::memcpy(v, cache.v_ptr(layer, 0), (size_t)cache.current_len * kvd);
    std::memcpy(ks, cache.ks_ptr(layer, 0), (size_t)cache.current_len * d->num_kv_heads * 4);
    std::memcpy(vs, cache.vs_ptr(layer, 0), (size_t)cache.current_len * d->num_kv_heads * 4);
    return n;
}

void shim_release() { jieyu_b200::release_model(); }

}  // extern "C"
