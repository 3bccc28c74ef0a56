/*
 * jieyu.h — the reference's text C ABI (JieyuAI_api.h:42-67, implemented
 * in main.hpp:85-227) served by the B200 decode path: a model directory
 * (model.bf + model_info.json + vocab.json / merges.txt) is bound once, its
 * weights uploaded to the GPU, and every jieyu_generate runs the prompt
 * through the byte-level BPE tokenizer, the device token loop and the
 * reference's output rules.
 *
 * Contract (same names, argument meaning and error behaviour as the
 * reference):
 *   - One model per process, shared by every handle (a handle records the
 *     directory, its last error and its context length). Loading another
 *     directory unbinds the previous model; the last jieyu_free unbinds it.
 *   - jieyu_load(dir, 0) takes model_info.json's max_position_embeddings
 *     clamped to [64, 4096]; NULL on failure, the reason in
 *     jieyu_last_error(NULL) (per thread).
 *   - jieyu_generate returns the number of new tokens, 0 when nothing was
 *     produced (empty prompt or full context; the handle's error says so),
 *     -1 on error (NULL handle / prompt, prompt ids outside the vocabulary,
 *     a device failure). The text is copied to out truncated to cap-1 bytes
 *     plus NUL; out == NULL copies nothing.
 *   - Not thread-safe, as the reference.
 */
#ifndef JIEYU_H
#define JIEYU_H

#if defined(_WIN32)
#define JIEYU_API __declspec(dllexport)
#else
#define JIEYU_API __attribute__((visibility("default")))
#endif

#define JIEYU_PATH_MAX 512
#define JIEYU_ERR_MAX  256

/* Handle data, laid out as the reference's jieyu_ctx (JieyuAI_api.h:42-46). */
struct jieyu_ctx {
    char dir[JIEYU_PATH_MAX];
    char error[JIEYU_ERR_MAX];
    int max_seq;
};
typedef struct jieyu_ctx* jieyu_model;

#ifdef __cplusplus
#define JIEYU_DEFAULT(v) = v
extern "C" {
#else
#define JIEYU_DEFAULT(v)
#endif

JIEYU_API jieyu_model jieyu_load(const char* dir, int max_seq JIEYU_DEFAULT(0));
JIEYU_API void jieyu_free(jieyu_model h);
JIEYU_API const char* jieyu_last_error(jieyu_model h);
JIEYU_API const char* jieyu_version(void);
JIEYU_API int jieyu_context_length(jieyu_model h);
JIEYU_API const char* jieyu_model_dir(jieyu_model h);
JIEYU_API int jieyu_generate(jieyu_model h, const char* prompt, char* out, int cap, int max_new,
                             float temperature, float repetition_penalty);
/* Chat prompt from a JSONL file (jsonl_ochat.h:7-34): every line's "name"
 * and "message" become qb + name + "\n" + message + qe + "\n" (qb / qe empty:
 * the model's message_start / message_end), then assistant_start (or, for
 * "<|im_start|>" models, "<|im_start|>assistant\n"); -1 with "no usable
 * name/message" when no line has either. */
JIEYU_API int jieyu_generate_jsonl(jieyu_model h, const char* jsonl, const char* qb, const char* qe, char* out,
                                   int cap, int max_new JIEYU_DEFAULT(256), float temperature JIEYU_DEFAULT(0.8f),
                                   float repetition_penalty JIEYU_DEFAULT(1.1f));

/* Tokenizer entry points (the reference's json_libs::Tokenizer,
 * tokenizer_libs/include/tokenizer.h: load :340-455, encode :602,
 * decode :645, add_special_token :457-481) for callers and tests that need
 * ids without a model. jyt_tok_encode / jyt_tok_decode return the full
 * count and fill at most cap entries; -1 on a bad argument. */
typedef struct jyt_tokenizer jyt_tokenizer;
JIEYU_API jyt_tokenizer* jyt_tok_load(const char* vocab_path, const char* merges_path);
JIEYU_API void jyt_tok_free(jyt_tokenizer* t);
JIEYU_API int jyt_tok_encode(const jyt_tokenizer* t, const char* text, int len, int* ids, int cap);
JIEYU_API int jyt_tok_decode(const jyt_tokenizer* t, const int* ids, int n, char* out, int cap);
JIEYU_API int jyt_tok_add_special(jyt_tokenizer* t, const char* piece, int len);
/* vocab_size, bos, eos, unk, "</w>" id (-1 if absent), merge count */
JIEYU_API int jyt_tok_info(const jyt_tokenizer* t, int* out6);
/* jieyu_load's directory binding without the device upload: 0 and
 * out13 = {layers, hidden, heads, kv heads, head dim, intermediate, vocab,
 * max_seq, QKV bias, tied head, bit mask of the layer weights' model.bf
 * dtypes, rope_theta, (head block-quantised) | 2 * (embedding
 * block-quantised)}, or -1 and the reason in err (cap bytes with NUL). */
JIEYU_API int jyt_model_dir_probe(const char* dir, int max_seq, int* out13, char* err, int cap);

#ifdef __cplusplus
}

#include <stdexcept>
#include <string>
#include <string_view>
#include <utility>
#include <vector>

/* RAII wrapper with the reference's `class jieyu` surface
 * (JieyuAI_api.h:74-142): move-only, throws jieyu::error. */
class jieyu {
public:
    class error : public std::runtime_error {
    public:
        explicit error(const std::string& msg) : std::runtime_error(msg) {}
    };
    struct options {
        int max_new = 256;
        float temperature = 0.7f;
        float repetition_penalty = 1.1f;
    };
    jieyu() noexcept = default;
    explicit jieyu(std::string_view dir, int max_seq = 0) { open(dir, max_seq); }
    ~jieyu() { close(); }
    jieyu(const jieyu&) = delete;
    jieyu& operator=(const jieyu&) = delete;
    jieyu(jieyu&& o) noexcept : h_(std::exchange(o.h_, nullptr)) {}
    jieyu& operator=(jieyu&& o) noexcept {
        if (this != &o) { close(); h_ = std::exchange(o.h_, nullptr); }
        return *this;
    }
    void open(std::string_view dir, int max_seq = 0) {
        close();
        h_ = jieyu_load(std::string(dir).c_str(), max_seq);
        if (!h_) throw error(std::string("load failed: ") + jieyu_last_error(nullptr));
    }
    void close() noexcept {
        if (h_) { jieyu_free(h_); h_ = nullptr; }
    }
    bool is_open() const noexcept { return h_ != nullptr; }
    explicit operator bool() const noexcept { return h_ != nullptr; }
    int context_length() const noexcept { return h_ ? jieyu_context_length(h_) : 0; }
    std::string dir() const { return h_ ? std::string(jieyu_model_dir(h_)) : std::string(); }
    std::string last_error() const { return std::string(jieyu_last_error(h_)); }
    std::string generate(std::string_view prompt) { return generate(prompt, options{}); }
    std::string generate(std::string_view prompt, const options& o) {
        check();
        std::vector<char> buf(buffer_bytes(o), 0);
        if (jieyu_generate(h_, std::string(prompt).c_str(), buf.data(), (int)buf.size(), o.max_new, o.temperature,
                           o.repetition_penalty) < 0)
            throw error(jieyu_last_error(h_));
        return std::string(buf.data());
    }
    std::string generate_jsonl(std::string_view jsonl, std::string_view qb = {}, std::string_view qe = {}) {
        return generate_jsonl(jsonl, qb, qe, options{});
    }
    std::string generate_jsonl(std::string_view jsonl, std::string_view qb, std::string_view qe, const options& o) {
        check();
        std::vector<char> buf(buffer_bytes(o), 0);
        if (jieyu_generate_jsonl(h_, std::string(jsonl).c_str(), std::string(qb).c_str(), std::string(qe).c_str(),
                                 buf.data(), (int)buf.size(), o.max_new, o.temperature, o.repetition_penalty) < 0)
            throw error(jieyu_last_error(h_));
        return std::string(buf.data());
    }
    static std::string version() { return std::string(jieyu_version()); }

private:
    static size_t buffer_bytes(const options& o) { return (size_t)(o.max_new > 0 ? o.max_new : 4096) * 16u + 256u; }
    void check() const {
        if (!h_) throw error("no model loaded (call open first)");
    }
    jieyu_model h_ = nullptr;
};
#endif /* __cplusplus */

#endif /* JIEYU_H */
