/*
 * ref_harness.cpp — TEST INFRASTRUCTURE ONLY (the checker, never the product).
 *
 * Compiles the UNMODIFIED jieyu reference headers (from the reference source
 * tree, include path given by the Makefile) into oracle/_ref/libjyref.so and
 * exposes its hot-path functions through a plain C ABI so tests and the CPU
 * baseline can drive the reference's own code on in-memory weights:
 *   qmat::matmul_q      libs/matmul_libs/matmul_q.h:134-162
 *   matmul              libs/matmul_libs/matmul.h:7-76
 *   rmsnorm             libs/model_libs/rmsnorm/rmsnorm.h:8-78
 *   RoPETable::init     libs/date_libs/date.h:52-66
 *   rope_pos            libs/model_libs/rope/rope.h:108-110
 *   kv_pack_q8          libs/model_libs/attention/attention_q8.h:20-37
 *   attention_q8        libs/model_libs/attention/attention_q8.h:38-184
 *   silu                libs/model_libs/silu/silu.h:7-81
 *   ffn                 libs/model_libs/ffn/ffn.h:7-19
 *   forward_cached      libs/model_libs/forward.h:47-96
 *   generate            libs/model_libs/generate.h:90-112
 *   generate_cached's step body (generate.h:40-60) over a pre-filled cache
 *   bfile::write_bfile  libs/model_libs/bfile.h:393-411 (model.bf writer)
 *   bfile::View::open + bind_layers / bind_biases / bind_embed / bind_lm_head /
 *   bind_final_norm     libs/model_libs/bfile.h:141-204, load_weights.h:97-155
 *   json_libs::Tokenizer libs/tokenizer_libs/include/tokenizer.h (load, encode,
 *                       decode, add_special_token)
 * Nothing here changes the reference's arithmetic; the harness only builds
 * WMat / LayerWeights / __KVcache objects over caller buffers.
 */
#define JIEYU_HPP 1
/* the reference relies on libs.h having pulled these in first (libs/libs.h:15-28) */
#include <algorithm>
#include <cmath>
#include <math.h>
#include <cstdint>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <exception>
#include <string>
#include <vector>
#include <chrono>
#if defined(_OPENMP)
#include <omp.h>
#endif

#include "date_libs/date.h"
#include "date_libs/check_cpu.h"
#include "date_libs/info.h"
#include "matmul_libs/matmul.h"
#include "matmul_libs/matmul_q.h"
#include "model_libs/wmat_kernel.h"
#include "model_libs/prefetch.h"
#include "model_libs/silu/silu.h"
#include "model_libs/rmsnorm/rmsnorm.h"
#include "model_libs/rope/rope.h"
#include "model_libs/attention/attention_q8.h"
#include "model_libs/ffn/ffn.h"
#include "model_libs/transformer_layer.h"
#include "model_libs/forward.h"
#include "model_libs/generate.h"
#include "model_libs/bfile.h"
#include "model_libs/load_weights.h"
#include "tokenizer_libs/include/tokenizer.h"
#include "tokenizer_libs/include/byte_vocab.h"
#include <fstream>

#include "jieyu_b200.h"

#include <cstddef>
/* jyc_wmat / jyc_layer_weights must be layout-identical to WMat / LayerWeights. */
static_assert(sizeof(jyc_wmat) == sizeof(WMat), "WMat layout");
static_assert(offsetof(jyc_wmat, q) == offsetof(WMat, q), "WMat.q");
static_assert(offsetof(jyc_wmat, qt) == offsetof(WMat, qt), "WMat.qt");
static_assert(sizeof(jyc_layer_weights) == sizeof(LayerWeights), "LayerWeights layout");
static_assert(offsetof(jyc_layer_weights, bq) == offsetof(LayerWeights, bq), "LW.bq");
static_assert(offsetof(jyc_layer_weights, W3) == offsetof(LayerWeights, W3), "LW.W3");

static thread_local std::string g_err;

static WMat to_wmat(const jyc_wmat& w) {
    WMat m;
    m.f = w.f; m.h = w.h; m.q = w.q; m.qt = w.qt;
    return m;
}

extern "C" {

const char* jyref_last_error(void) { return g_err.c_str(); }

/* Reads JIEYU_ISA (check_cpu.h:54-68) and fills cpu_can; pins the ISA path. */
void jyref_init(const char* isa, int threads) {
    if (isa != nullptr) setenv("JIEYU_ISA", isa, 1);
    cpu_can.GetCpuCan();
#if defined(_OPENMP)
    if (threads > 0) omp_set_num_threads(threads);
#else
    (void)threads;
#endif
}

int jyref_threads(void) { return par_threads(); }

void jyref_matmul_q8(const float* a, const void* b, float* c, int m, int n, int k) {
    qmat::matmul_q(a, b, c, m, n, k, qmat::Q8_0);
}

/* qmat::matmul_q with a K-quant weight type (t = qmat::Q4K, Q5K or Q6K). */
void jyref_matmul_qk(const float* a, const void* b, float* c, int m, int n, int k, int t) {
    qmat::matmul_q(a, b, c, m, n, k, (uint8_t)t);
}

void jyref_matmul_f32(int m, int n, int k, const float* A, const float* B, float* C) {
    matmul(m, n, k, A, B, C);
}

void jyref_matmul_f16(const float* a, const uint16_t* b, float* c, int m, int n, int k) {
    WMat w{};
    w.h = b;
    matmul_w(w, m, n, k, a, c);  // the reference's own dispatch picks its f16 kernel
}

void jyref_rmsnorm(float* x, float* y, const float* w, int n, float eps) {
    rmsnorm(x, y, w, n, eps);
}

void jyref_rope_table(int max_seq, int head_dim, float theta, float* cos_out, float* sin_out) {
    RoPETable t;
    t.init(max_seq, head_dim, theta);
    std::memcpy(cos_out, t.cos.data(), t.cos.size() * sizeof(float));
    std::memcpy(sin_out, t.sin.data(), t.sin.size() * sizeof(float));
}

void jyref_rope_pos(float* q, int seq, int start_pos, int heads, int hd,
                    const float* cos_t, const float* sin_t) {
    rope_pos(q, seq, start_pos, heads, hd, cos_t, sin_t);
}

void jyref_kv_pack_q8(const float* src, int8_t* dst, float* sc, int heads, int hd, int n) {
    kv_pack_q8(src, dst, sc, heads, hd, n);
}

int jyref_attention_q8(float* Q, float* K, float* V, float* out, int seq, int start_pos,
                       int H, int KV, int hd, int8_t* kc, float* ks, int8_t* vc, float* vs,
                       int cap) {
    try {
        attention_q8(Q, K, V, out, seq, start_pos, H, KV, hd, __KVq{kc, ks, vc, vs, cap});
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
    return 0;
}

void jyref_silu(float* x, float* y, int n) { silu(x, y, n); }

void jyref_ffn(float* x, const jyc_wmat* w1, const jyc_wmat* w2, const jyc_wmat* w3,
               float* out, int seq, int hidden, int inter) {
    ffn(x, to_wmat(*w1), to_wmat(*w2), to_wmat(*w3), out, seq, hidden, inter);
}

/* ---- model level: a KV cache object plus teacher-forced forward ------- */
void* jyref_cache_create(int L, int max_seq, int KV, int hd) {
    __KVcache* c = new __KVcache();
    c->init(L, max_seq, KV, hd);
    return c;
}
void jyref_cache_free(void* c) { delete static_cast<__KVcache*>(c); }

/* Reads one layer of the cache in its native layout. */
void jyref_cache_read(void* cp, int layer, int npos, int8_t* k, float* ks, int8_t* v, float* vs) {
    __KVcache* c = static_cast<__KVcache*>(cp);
    const size_t row = (size_t)c->num_kv_heads * c->head_dim;
    std::memcpy(k, c->k_ptr(layer, 0), (size_t)npos * row);
    std::memcpy(v, c->v_ptr(layer, 0), (size_t)npos * row);
    std::memcpy(ks, c->ks_ptr(layer, 0), (size_t)npos * c->num_kv_heads * sizeof(float));
    std::memcpy(vs, c->vs_ptr(layer, 0), (size_t)npos * c->num_kv_heads * sizeof(float));
}

/* Writes one layer's first npos positions in the cache's native layout (the
 * inverse of jyref_cache_read): a context filled without running a prefill. */
void jyref_cache_write(void* cp, int layer, int npos, const int8_t* k, const float* ks, const int8_t* v,
                       const float* vs) {
    __KVcache* c = static_cast<__KVcache*>(cp);
    const size_t row = (size_t)c->num_kv_heads * c->head_dim;
    std::memcpy(c->k_ptr(layer, 0), k, (size_t)npos * row);
    std::memcpy(c->v_ptr(layer, 0), v, (size_t)npos * row);
    std::memcpy(c->ks_ptr(layer, 0), ks, (size_t)npos * c->num_kv_heads * sizeof(float));
    std::memcpy(c->vs_ptr(layer, 0), vs, (size_t)npos * c->num_kv_heads * sizeof(float));
}

/* n greedy decode steps of generate_cached's loop body (generate.h:40-60,
 * seq = 1) from a cache already holding positions [0, start_pos): the LM-head
 * prefetch, the embedding row of the last id, forward_cached, matmul_w of the
 * LM head and the greedy pick (first index of the maximum). first_id is the
 * token at start_pos; out_ids[i] receives the i-th new id. step_s (optional,
 * n doubles) receives each step's seconds. Returns n, or -1. */
int jyref_decode_steps(const jyc_model_desc* d, void* cache, int start_pos, int first_id, int n, int* out_ids,
                       double* step_s) {
    try {
        __KVcache& c = *static_cast<__KVcache*>(cache);
        std::vector<float> X((size_t)d->hidden), logits((size_t)d->vocab_size);
        const WMat embed = to_wmat(d->embed), head = to_wmat(d->lm_head);
        int id = first_id;
        for (int i = 0; i < n; i++) {
            const auto t0 = std::chrono::steady_clock::now();
            prefetch::range(prefetch::data_of(head), prefetch::bytes_of(head, (size_t)d->vocab_size, (size_t)d->hidden));
            wmat_row(embed, (size_t)id, d->hidden, X.data());
            forward_cached(X.data(), reinterpret_cast<const LayerWeights*>(d->layers), d->num_layers,
                           d->final_rms_weight, d->cos_table, d->sin_table, 1, start_pos + i, c, d->hidden,
                           d->num_heads, d->num_kv_heads, d->head_dim, d->intermediate);
            matmul_w(head, 1, d->vocab_size, d->hidden, X.data(), logits.data());
            int next = 0;
            for (int v = 1; v < d->vocab_size; v++)
                if (logits[(size_t)v] > logits[(size_t)next]) next = v;
            out_ids[i] = next;
            id = next;
            if (step_s) step_s[i] = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        }
        return n;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

/* The step body of generate_cached (generate.h:43-49): embedding rows,
 * forward_cached, LM head on the last row. */
int jyref_forward_logits(const jyc_model_desc* d, void* cache, const int* ids, int seq,
                         int start_pos, float* logits, float* hidden_out) {
    try {
        __KVcache& c = *static_cast<__KVcache*>(cache);
        std::vector<float> X((size_t)seq * d->hidden);
        const WMat embed = to_wmat(d->embed), head = to_wmat(d->lm_head);
        for (int i = 0; i < seq; i++)
            wmat_row(embed, (size_t)ids[i], d->hidden, X.data() + (size_t)i * d->hidden);
        forward_cached(X.data(), reinterpret_cast<const LayerWeights*>(d->layers), d->num_layers,
                       d->final_rms_weight, d->cos_table, d->sin_table, seq, start_pos, c,
                       d->hidden, d->num_heads, d->num_kv_heads, d->head_dim, d->intermediate);
        const float* last = X.data() + (size_t)(seq - 1) * d->hidden;
        if (hidden_out) std::memcpy(hidden_out, last, (size_t)d->hidden * sizeof(float));
        if (logits) matmul_w(head, 1, d->vocab_size, d->hidden, last, logits);
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
    return 0;
}

struct cb_timer {
    int count = 0;
    std::chrono::steady_clock::time_point first, last;
};
static bool timing_cb(int, void* ud) {
    cb_timer* t = static_cast<cb_timer*>(ud);
    const auto now = std::chrono::steady_clock::now();
    if (t->count == 0) t->first = now;
    t->last = now;
    t->count++;
    return false;
}

/* generate() (generate.h:90-112). times (optional, 3 doubles): seconds from
 * call start to first token, first to last token (the -tokenspeed split,
 * pipeline.h:356-367), whole call. */
int jyref_generate(const jyc_model_desc* d, const int* prompt, int prompt_len,
                   const int* eos, int num_eos, int max_new, float temperature,
                   int* out_ids, float rep_penalty, double* times) {
    try {
        cb_timer t;
        const auto t0 = std::chrono::steady_clock::now();
        const int n = generate(prompt, prompt_len, eos, num_eos, to_wmat(d->embed),
                               to_wmat(d->lm_head),
                               reinterpret_cast<const LayerWeights*>(d->layers), d->num_layers,
                               d->final_rms_weight, d->cos_table, d->sin_table, d->max_seq,
                               max_new, temperature, d->vocab_size, d->hidden, d->num_heads,
                               d->num_kv_heads, d->head_dim, d->intermediate, out_ids,
                               rep_penalty, timing_cb, &t);
        const auto t1 = std::chrono::steady_clock::now();
        if (times) {
            using sec = std::chrono::duration<double>;
            times[0] = t.count ? sec(t.first - t0).count() : sec(t1 - t0).count();
            times[1] = t.count > 1 ? sec(t.last - t.first).count() : 0.0;
            times[2] = sec(t1 - t0).count();
        }
        return n;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

/* Writes a model.bf through the reference's writer. hdr = {hidden, layers,
 * mode, num_heads, num_kv_heads, head_dim, intermediate, vocab}; tensor i has
 * name names[i], dtype dtypes[i] (bfile::dtype_t), ndims[i] dims in
 * shapes[4*i..], nbytes[i] bytes at data[i]. Returns 0, or -1 (message in
 * jyref_last_error) when the writer rejects it. */
int jyref_bfile_write(const char* path, const uint64_t* hdr, int n, const char* const* names,
                      const uint8_t* dtypes, const uint8_t* ndims, const uint32_t* shapes,
                      const void* const* data, const uint64_t* nbytes) {
    try {
        bfile::Header h;
        h.hidden = hdr[0]; h.layers = hdr[1]; h.mode = (uint8_t)hdr[2];
        h.num_heads = (uint8_t)hdr[3]; h.num_kv_heads = (uint8_t)hdr[4]; h.head_dim = (uint8_t)hdr[5];
        h.intermediate = (uint32_t)hdr[6]; h.vocab_size = hdr[7];
        std::vector<bfile::Tensor> ts((size_t)n);
        for (int i = 0; i < n; i++) {
            ts[i].name = names[i];
            ts[i].dtype = dtypes[i];
            ts[i].shape.assign(shapes + 4 * i, shapes + 4 * i + ndims[i]);
            const unsigned char* p = static_cast<const unsigned char*>(data[i]);
            ts[i].data.assign(p, p + nbytes[i]);
        }
        bfile::write_bfile(path, h, ts);
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

/* Opens a model.bf with the reference's reader (bfile::View::open over the
 * file's bytes) and binds it with load_weights.h's rules. Per layer l,
 * out[l*12 + k] = byte offset in the file of tensor k (0 input_layernorm,
 * 1..4 q/k/v/o, 5 post_attention_layernorm, 6 gate, 7 down, 8 up, 9..11 q/k/v
 * bias) or -1 when absent; then embed, lm_head, final norm at out[12 L ..].
 * dt[...] gets the matching dtype codes (bfile::dtype_t, 255 when absent).
 * Returns 0, 1 when the reader rejects the file, 2 when binding fails. */
int jyref_bfile_bind(const char* path, int num_layers, int hidden, int vocab, int64_t* out, uint8_t* dt) {
    static std::vector<unsigned char> bytes;
    std::ifstream f(path, std::ios::binary);
    if (!f) { g_err = "cannot open"; return 1; }
    bytes.assign(std::istreambuf_iterator<char>(f), std::istreambuf_iterator<char>());
    bfile::current().reset();
    if (!bfile::current().open(bytes.data(), bytes.size())) { g_err = "reader rejected the file"; return 1; }
    const unsigned char* base = bytes.data();
    std::vector<LayerWeights> lw((size_t)num_layers);
    std::string missing;
    if (!bind_layers(lw.data(), num_layers, &missing)) { g_err = "missing " + missing; return 2; }
    bind_biases(lw.data(), num_layers);
    auto off = [&](const void* p) -> int64_t {
        return p ? (int64_t)(static_cast<const unsigned char*>(p) - base) : -1;
    };
    auto wm = [&](const WMat& m, int64_t* o, uint8_t* d) {
        if (m.f) { *o = off(m.f); *d = bfile::F32; }
        else if (m.h) { *o = off(m.h); *d = bfile::F16; }
        else if (m.q) { *o = off(m.q); *d = m.qt == qmat::Q8_0 ? bfile::Q8_0 : m.qt == qmat::Q4K ? bfile::Q4K
                                       : m.qt == qmat::Q5K ? bfile::Q5K : bfile::Q6K; }
        else { *o = -1; *d = 255; }
    };
    for (int l = 0; l < num_layers; l++) {
        int64_t* o = out + 12 * l;
        uint8_t* d = dt + 12 * l;
        const LayerWeights& w = lw[(size_t)l];
        o[0] = off(w.rms1_weight); d[0] = bfile::F32;
        wm(w.Wq, o + 1, d + 1); wm(w.Wk, o + 2, d + 2); wm(w.Wv, o + 3, d + 3); wm(w.Wo, o + 4, d + 4);
        o[5] = off(w.rms2_weight); d[5] = bfile::F32;
        wm(w.W1, o + 6, d + 6); wm(w.W2, o + 7, d + 7); wm(w.W3, o + 8, d + 8);
        o[9] = off(w.bq); o[10] = off(w.bk); o[11] = off(w.bv);
        for (int b = 9; b < 12; b++) d[b] = o[b] < 0 ? 255 : bfile::F32;
    }
    int64_t* o = out + 12 * num_layers;
    uint8_t* d = dt + 12 * num_layers;
    const WMat emb = bind_embed();
    if (emb.empty()) { g_err = "missing embedding"; return 2; }
    wm(emb, o + 0, d + 0);
    const WMat head = bind_lm_head(hidden, vocab);
    if (head.empty()) { g_err = "lm_head missing or misshapen"; return 2; }
    wm(head, o + 1, d + 1);
    o[2] = off(bind_final_norm()); d[2] = o[2] < 0 ? 255 : bfile::F32;
    return 0;
}

/* The reference's tokenizer over vocab.json / merges.txt files. */
void* jyref_tok_load(const char* vocab, const char* merges) {
    json_libs::Tokenizer* t = new json_libs::Tokenizer();
    if (!t->load(vocab, merges)) {
        delete t;
        return nullptr;
    }
    return t;
}

void jyref_tok_free(void* t) { delete static_cast<json_libs::Tokenizer*>(t); }

/* ids of `text` (len bytes); returns their count (only the first `cap` are stored). */
int jyref_tok_encode(void* t, const char* text, int len, int* out, int cap) {
    const std::vector<int32_t> ids = static_cast<json_libs::Tokenizer*>(t)->encode(std::string(text, (size_t)len));
    for (size_t i = 0; i < ids.size() && (int)i < cap; i++) out[i] = ids[i];
    return (int)ids.size();
}

/* bytes of decode(ids); returns their count (only the first `cap` are stored). */
int jyref_tok_decode(void* t, const int* ids, int n, char* out, int cap) {
    const std::string s = static_cast<json_libs::Tokenizer*>(t)->decode(std::vector<int32_t>(ids, ids + n));
    memcpy(out, s.data(), std::min<size_t>(s.size(), (size_t)std::max(cap, 0)));
    return (int)s.size();
}

/* {bos, eos, unk, word_end, vocab_size} */
void jyref_tok_info(void* t, int* out) {
    const json_libs::Tokenizer* k = static_cast<json_libs::Tokenizer*>(t);
    out[0] = k->bos_id(); out[1] = k->eos_id(); out[2] = k->unk_id(); out[3] = k->word_end_id();
    out[4] = (int)k->vocab_size();
}

int jyref_tok_add_special(void* t, const char* piece) {
    return static_cast<json_libs::Tokenizer*>(t)->add_special_token(piece);
}

/* The reference's byte-level vocabulary files (byte_vocab.h write_byte_level_vocab). */
int jyref_write_byte_vocab(const char* vocab, const char* merges) {
    try {
        json_libs::write_byte_level_vocab(vocab, merges);
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

}  // extern "C"
