/*
 * jieyu_b200_shim.hpp — the reference's operator and generation entry points
 * under the reference's own names, argument lists and conventions (host
 * pointers in the reference's layouts, synchronous, std::runtime_error on
 * misuse), running on the B200 through libjieyu_b200.
 *
 * A caller of the reference's free functions swaps the namespace and keeps
 * every call: `jieyu_b200::qmat::matmul_q(a, b, c, m, n, k, t)` for
 * `qmat::matmul_q(...)`, `jieyu_b200::generate(...)` for `generate(...)`, and
 * so on. The functions that take the reference's structs (WMat, LayerWeights,
 * __KVq, __KVcache; libs/date_libs/wmat.h:32-44, libs/date_libs/date.h:75-147,
 * libs/model_libs/attention/attention_q8.h:12-19) are templates over them, so
 * the header compiles beside the reference's own headers (their layouts are
 * checked against the C ABI's with static_asserts) or with any structs of the
 * same members. Header only; link with -ljieyu_b200.
 *
 *   reference (file:line)                                  here
 *   qmat::matmul_q  libs/matmul_libs/matmul_q.h:134        jieyu_b200::qmat::matmul_q
 *   matmul          libs/matmul_libs/matmul.h:7            jieyu_b200::matmul
 *   matmul_f16_avx_fma libs/matmul_libs/matmul_f16.h:19     jieyu_b200::matmul_f16_avx_fma
 *   matmul_w        libs/model_libs/wmat_kernel.h:9        jieyu_b200::matmul_w
 *   rmsnorm         libs/model_libs/rmsnorm/rmsnorm.h:8    jieyu_b200::rmsnorm
 *   rope_pos        libs/model_libs/rope/rope.h:108        jieyu_b200::rope_pos
 *   kv_pack_q8      libs/model_libs/attention/attention_q8.h:20   jieyu_b200::kv_pack_q8
 *   attention_q8    libs/model_libs/attention/attention_q8.h:38   jieyu_b200::attention_q8
 *   silu            libs/model_libs/silu/silu.h:7          jieyu_b200::silu
 *   ffn             libs/model_libs/ffn/ffn.h:7            jieyu_b200::ffn
 *   generate        libs/model_libs/generate.h:90          jieyu_b200::generate
 *   generate_cached libs/model_libs/generate.h:9           jieyu_b200::generate_cached
 *
 * The operators copy their operands to the device on every call (unit-level
 * drop-ins). generate / generate_cached upload the weights once: the model
 * stays bound on the device while the same weights and shape come back
 * (the bind_model point, libs/model_libs/pipeline.h:63-153) — the weight
 * memory must not change while it is bound; release_model() unbinds it.
 * Like the reference, none of this is thread-safe.
 */
#ifndef JIEYU_B200_SHIM_HPP
#define JIEYU_B200_SHIM_HPP

#include <cstddef>
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <type_traits>

#include "jieyu_b200.h"

namespace jieyu_b200 {

namespace detail {

inline void check(int r, const char* what) {
    if (r < 0) throw std::runtime_error(std::string(what) + ": " + jyc_last_error());
}

template <class W>
inline jyc_wmat to_wmat(const W& w) {
    jyc_wmat m;
    m.f = w.f;
    m.h = w.h;
    m.q = w.q;
    m.qt = w.qt;
    return m;
}

// The reference's LayerWeights is passed to the library as an array, so its
// layout must be the C ABI's jyc_layer_weights (date.h:75-88 = jieyu_b200.h).
template <class LW>
inline const jyc_layer_weights* to_layers(const LW* layers) {
    static_assert(sizeof(LW) == sizeof(jyc_layer_weights), "LayerWeights layout differs from jyc_layer_weights");
    static_assert(std::is_standard_layout<LW>::value, "LayerWeights must be standard layout");
    static_assert(offsetof(LW, Wq) == offsetof(jyc_layer_weights, Wq) &&
                      offsetof(LW, bq) == offsetof(jyc_layer_weights, bq) &&
                      offsetof(LW, rms2_weight) == offsetof(jyc_layer_weights, rms2_weight) &&
                      offsetof(LW, W3) == offsetof(jyc_layer_weights, W3),
                  "LayerWeights field offsets differ from jyc_layer_weights");
    static_assert(sizeof(decltype(layers->Wq)) == sizeof(jyc_wmat), "WMat layout differs from jyc_wmat");
    return reinterpret_cast<const jyc_layer_weights*>(layers);
}

// The model generate() keeps bound on the device, and what it was bound from
// (no destructor: at exit the process's device memory goes with it, and the
// CUDA runtime may already be gone when static objects are destroyed).
struct Bound {
    jyc_model* model = nullptr;
    jyc_model_desc desc{};
};
inline Bound& bound() {
    static Bound b;
    return b;
}
inline bool same_wmat(const jyc_wmat& a, const jyc_wmat& b) {
    return a.f == b.f && a.h == b.h && a.q == b.q && a.qt == b.qt;
}
inline bool same_desc(const jyc_model_desc& a, const jyc_model_desc& b) {
    return a.layers == b.layers && a.num_layers == b.num_layers && same_wmat(a.embed, b.embed) &&
           same_wmat(a.lm_head, b.lm_head) && a.final_rms_weight == b.final_rms_weight &&
           a.cos_table == b.cos_table && a.sin_table == b.sin_table && a.max_seq == b.max_seq &&
           a.vocab_size == b.vocab_size && a.hidden == b.hidden && a.num_heads == b.num_heads &&
           a.num_kv_heads == b.num_kv_heads && a.head_dim == b.head_dim && a.intermediate == b.intermediate;
}
inline jyc_model* bind(const jyc_model_desc& d) {
    Bound& b = bound();
    if (b.model && same_desc(b.desc, d)) return b.model;
    if (b.model) {
        jyc_model_free(b.model);
        b.model = nullptr;
    }
    jyc_model* m = jyc_model_create(&d);
    if (!m) throw std::runtime_error(std::string("generate: ") + jyc_last_error());
    b.model = m;
    b.desc = d;
    return m;
}

typedef bool (*token_cb)(int id, void* ud);
struct CbPair {
    token_cb cb;
    void* ud;
};
inline int cb_trampoline(int id, void* ud) {
    const CbPair* p = static_cast<const CbPair*>(ud);
    return p->cb(id, p->ud) ? 1 : 0;
}

}  // namespace detail

/* Token callback of generate (generate.h:8): return true to stop. */
typedef detail::token_cb token_cb;

namespace qmat {
/* qmat::matmul_q (matmul_q.h:134-162): c[m][n] = a[m][k] . W^T, W [n][k]
 * in blocks of type t (Q4K 0, Q5K 1, Q6K 2, Q8_0 3: the reference's enum). */
inline void matmul_q(const float* a, const void* b, float* c, int m, int n, int k, uint8_t t) {
    detail::check(jyc_host_matmul_q(a, b, c, m, n, k, t), "matmul_q");
}
}  // namespace qmat

/* matmul (matmul.h:7-76): C[m][n] = A[m][k] . B[k][n], fp32. */
inline void matmul(const int m, const int n, const int k, const float* A, const float* B, float* C) {
    detail::check(jyc_host_matmul_f32(m, n, k, A, B, C), "matmul");
}

/* matmul_f16_avx_fma (matmul_f16.h:19-41): c[m][n] = a[m][k] . b[k][n], b fp16. */
inline void matmul_f16_avx_fma(const float* a, const uint16_t* b, float* c, int m, int n, int k) {
    detail::check(jyc_host_matmul_f16(a, b, c, m, n, k), "matmul_f16");
}

/* matmul_w (wmat_kernel.h:9-16): the WMat dispatch (fp32, fp16, blocks). */
template <class WMatT>
inline void matmul_w(const WMatT& B, const int m, const int n, const int k, const float* A, float* C) {
    const jyc_wmat w = detail::to_wmat(B);
    detail::check(jyc_host_matmul_w(&w, m, n, k, A, C), "matmul_w");
}

/* rmsnorm (rmsnorm.h:8-78): y = x / sqrt(mean(x^2) + eps) * weight. */
inline void rmsnorm(float* x, float* y, const float* weight, int n, float eps) {
    detail::check(jyc_host_rmsnorm(x, y, weight, n, eps), "rmsnorm");
}

/* rope_pos (rope.h:108-110), in place. */
inline void rope_pos(float* q, int seq, int start_pos, int num_heads, int head_dim, const float* cos_table,
                     const float* sin_table) {
    detail::check(jyc_host_rope_pos(q, seq, start_pos, num_heads, head_dim, cos_table, sin_table), "rope_pos");
}

/* kv_pack_q8 (attention_q8.h:20-37). */
inline void kv_pack_q8(const float* src, int8_t* dst, float* sc, int heads, int hd, int n) {
    detail::check(jyc_host_kv_pack_q8(src, dst, sc, heads, hd, n), "kv_pack_q8");
}

/* attention_q8 (attention_q8.h:38-184) over the caller's __KVq. */
template <class KVq>
inline void attention_q8(float* Q, float* K, float* V, float* out, int seq, int start_pos, int num_heads,
                         int num_kv_heads, int head_dim, const KVq& kvq) {
    detail::check(jyc_host_attention_q8(Q, K, V, out, seq, start_pos, num_heads, num_kv_heads, head_dim, kvq.k,
                                        kvq.ks, kvq.v, kvq.vs, kvq.cap),
                  "attention_q8");
}

/* silu (silu.h:7-81). */
inline void silu(float* x, float* y, int n) { detail::check(jyc_host_silu(x, y, n), "silu"); }

/* ffn (ffn.h:7-19): out = W2 (silu(W1 x) * (W3 x)). */
template <class WMatT>
inline void ffn(float* x, const WMatT& w1, const WMatT& w2, const WMatT& w3, float* out, int seq, int hidden,
                int intermediate) {
    const jyc_wmat a = detail::to_wmat(w1), b = detail::to_wmat(w2), c = detail::to_wmat(w3);
    detail::check(jyc_host_ffn(x, &a, &b, &c, out, seq, hidden, intermediate), "ffn");
}

namespace detail {
template <class WMatT, class LayerW>
inline jyc_model_desc make_desc(const WMatT& embed, const WMatT& lm_head, const LayerW* layers, int num_layers,
                                const float* final_rms_weight, const float* cos_table, const float* sin_table,
                                int max_seq, int vocab_size, int hidden, int num_heads, int num_kv_heads,
                                int head_dim, int intermediate) {
    jyc_model_desc d;
    std::memset(&d, 0, sizeof(d));
    d.layers = to_layers(layers);
    d.num_layers = num_layers;
    d.embed = to_wmat(embed);
    d.lm_head = to_wmat(lm_head);
    d.final_rms_weight = final_rms_weight;
    d.cos_table = cos_table;
    d.sin_table = sin_table;
    d.max_seq = max_seq;
    d.vocab_size = vocab_size;
    d.hidden = hidden;
    d.num_heads = num_heads;
    d.num_kv_heads = num_kv_heads;
    d.head_dim = head_dim;
    d.intermediate = intermediate;
    return d;
}

inline int run_generate(jyc_model* m, const int* prompt_ids, int prompt_len, const int* eos_ids, int num_eos,
                        int max_new_tokens, float temperature, int* out_ids, float repetition_penalty, token_cb cb,
                        void* cb_ud) {
    CbPair p{cb, cb_ud};
    const int n = jyc_generate(m, prompt_ids, prompt_len, eos_ids, eos_ids ? num_eos : 0, max_new_tokens,
                               temperature, out_ids, repetition_penalty, cb ? cb_trampoline : nullptr,
                               cb ? static_cast<void*>(&p) : nullptr);
    check(n, "generate");
    return n;
}
}  // namespace detail

/* generate (generate.h:90-112): greedy (temperature <= 0) or the reference's
 * LCG sampler, repetition penalty, EOS ids, token callback; out_ids receives
 * the prompt then the new ids; returns their count (0 if prompt_len <= 0 or
 * > max_seq). The weights are bound on the device at the first call. */
template <class WMatT, class LayerW>
inline int generate(const int* prompt_ids, int prompt_len, const int* eos_ids, int num_eos, const WMatT& embed,
                    const WMatT& lm_head, const LayerW* layers, int num_layers, const float* final_rms_weight,
                    const float* cos_table, const float* sin_table, int max_seq, int max_new_tokens,
                    float temperature, int vocab_size, int hidden, int num_heads, int num_kv_heads, int head_dim,
                    int intermediate, int* out_ids, float repetition_penalty = 1.0f, token_cb cb = nullptr,
                    void* cb_ud = nullptr) {
    if (prompt_len <= 0 || prompt_len > max_seq) return 0;
    const jyc_model_desc d = detail::make_desc(embed, lm_head, layers, num_layers, final_rms_weight, cos_table,
                                               sin_table, max_seq, vocab_size, hidden, num_heads, num_kv_heads,
                                               head_dim, intermediate);
    return detail::run_generate(detail::bind(d), prompt_ids, prompt_len, eos_ids, num_eos, max_new_tokens,
                                temperature, out_ids, repetition_penalty, cb, cb_ud);
}

/* generate_cached (generate.h:9-89) with the caller's __KVcache: the same
 * generation; afterwards the cache holds the int8 K/V rows of every
 * position the loop ran through (all but the last new token) and
 * current_len = their count, as forward_cached leaves it. */
template <class WMatT, class LayerW, class Cache>
inline int generate_cached(const int* prompt_ids, int prompt_len, const int* eos_ids, int num_eos,
                           const WMatT& embed, const WMatT& lm_head, const LayerW* layers, int num_layers,
                           const float* final_rms_weight, const float* cos_table, const float* sin_table,
                           int max_seq, int max_new_tokens, float temperature, int vocab_size, int hidden,
                           int num_heads, int num_kv_heads, int head_dim, int intermediate, Cache& cache,
                           int* out_ids, float repetition_penalty = 1.0f, token_cb cb = nullptr,
                           void* cb_ud = nullptr) {
    if (prompt_len <= 0 || prompt_len > max_seq) return 0;
    if (cache.num_layers < num_layers || cache.max_seq < max_seq || cache.num_kv_heads != num_kv_heads ||
        cache.head_dim != head_dim)
        throw std::runtime_error("generate: KV cache shape does not match the model");
    const jyc_model_desc d = detail::make_desc(embed, lm_head, layers, num_layers, final_rms_weight, cos_table,
                                               sin_table, max_seq, vocab_size, hidden, num_heads, num_kv_heads,
                                               head_dim, intermediate);
    jyc_model* m = detail::bind(d);
    cache.current_len = 0;
    const int n = detail::run_generate(m, prompt_ids, prompt_len, eos_ids, num_eos, max_new_tokens, temperature,
                                       out_ids, repetition_penalty, cb, cb_ud);
    const int npos = n > prompt_len ? n - 1 : 0;
    for (int l = 0; l < num_layers && npos > 0; l++)
        detail::check(jyc_model_read_kv(m, l, npos, cache.k_ptr(l, 0), cache.ks_ptr(l, 0), cache.v_ptr(l, 0),
                                        cache.vs_ptr(l, 0)),
                      "generate: KV cache read-back");
    cache.current_len = npos;
    return n;
}

/* Frees the model generate() keeps bound (the next call binds again). */
inline void release_model() {
    detail::Bound& b = detail::bound();
    if (b.model) jyc_model_free(b.model);
    b.model = nullptr;
}

}  // namespace jieyu_b200

#endif
