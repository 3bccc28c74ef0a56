/*
 * jieyu_b200.h — C ABI of the B200 (sm_100a) decode path for jieyu.
 *
 * Every entry point is `extern "C"`, takes plain pointers and sizes, and
 * returns a status code (JYC_OK == 0, negative on error; the message is in
 * jyc_last_error()). No C++ exception crosses this boundary.
 *
 * Two families:
 *   - operator entry points over DEVICE pointers on a caller stream
 *     (jyc_matmul_q8, jyc_rmsnorm, jyc_rope_pos, jyc_attention_q8, ...): one
 *     per reference operator, same argument meaning and order;
 *   - the model entry points (jyc_model_create, jyc_generate, ...) that take
 *     the reference's own host-side weight handles (WMat / LayerWeights are
 *     binary-compatible with jyc_wmat / jyc_layer_weights), upload them to HBM
 *     once, and run the whole token loop on the GPU.
 *
 * Reference paths below are relative to the jieyu source tree.
 */
#ifndef JIEYU_B200_H
#define JIEYU_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define JYC_API __attribute__((visibility("default")))
#else
#define JYC_API
#endif

/* ---- status codes ------------------------------------------------------ */
#define JYC_OK               0
#define JYC_ERR_ARG         -1   /* bad argument (reference: std::runtime_error on misuse) */
#define JYC_ERR_CUDA        -2   /* a CUDA runtime call failed */
#define JYC_ERR_KV_OOM      -3   /* start_pos+seq > KV capacity (reference: "KV cache 容量不足") */
#define JYC_ERR_UNSUPPORTED -4   /* weight type / shape this build does not handle */
#define JYC_ERR_NOMEM       -5   /* device allocation failed */

/* Quantised block types, same numbering as qmat's enum (libs/matmul_libs/matmul_q.h:15). */
enum { JYC_Q4K = 0, JYC_Q5K = 1, JYC_Q6K = 2, JYC_Q8_0 = 3 };

/* Weight handle. Field order and types equal `struct WMat`
 * (libs/date_libs/wmat.h:32-44): exactly one of f (fp32, row-major [in][out]),
 * h (fp16, [in][out]) or q (quantised blocks: [out][in/32] x 34 B for Q8_0,
 * [out][in/256] x 144 / 176 / 210 B for Q4_K / Q5_K / Q6_K) is non-null. */
typedef struct jyc_wmat {
    const float*    f;
    const uint16_t* h;
    const void*     q;
    uint8_t         qt;
} jyc_wmat;

/* Per-layer weights. Field order equals `struct LayerWeights`
 * (libs/date_libs/date.h:75-88); bq/bk/bv may be NULL (no QKV bias). */
typedef struct jyc_layer_weights {
    const float* rms1_weight;
    jyc_wmat Wq, Wk, Wv, Wo;
    const float* bq;
    const float* bk;
    const float* bv;
    const float* rms2_weight;
    jyc_wmat W1, W2, W3;
} jyc_layer_weights;

/* Everything `generate()` receives besides the prompt (libs/model_libs/generate.h:90-104),
 * all HOST pointers in the reference's layouts. cos/sin are RoPETable tables
 * [max_seq][head_dim/2] (libs/date_libs/date.h:52-66). */
typedef struct jyc_model_desc {
    const jyc_layer_weights* layers;
    int num_layers;
    jyc_wmat embed;
    jyc_wmat lm_head;
    const float* final_rms_weight;
    const float* cos_table;
    const float* sin_table;
    int max_seq;
    int vocab_size;
    int hidden;
    int num_heads;
    int num_kv_heads;
    int head_dim;
    int intermediate;
    /* Vocabulary-sharded LM head (tensor parallel; 0/0 otherwise): the
     * embedding has embed_rows rows (0: vocab_size) and the head's row i is
     * token vocab_offset + i. */
    int embed_rows;
    int vocab_offset;
} jyc_model_desc;

/* Token callback, same contract as `token_cb` (libs/model_libs/generate.h:8):
 * return non-zero to stop generation after this token. */
typedef int (*jyc_token_cb)(int id, void* ud);

/* ---- library ----------------------------------------------------------- */
JYC_API const char* jyc_version(void);
/* Message of the last failing call on this thread ("" if none). */
JYC_API const char* jyc_last_error(void);
/* Number of device kernels this library launched so far in this process
 * (every launch made by the library increments it). */
JYC_API long long jyc_kernel_launches(void);

/* ---- host helpers (no GPU needed) -------------------------------------- */
/* RoPE tables exactly as RoPETable::init (libs/date_libs/date.h:52-66):
 * freq = 1/powf(theta, 2j/hd), angle = i*freq, cosf/sinf, all in float. */
JYC_API int jyc_rope_table(int max_seq, int head_dim, float theta,
                           float* cos_out, float* sin_out);

/* Seeded synthetic data (no reference counterpart: the reference has no
 * quantiser, GGUF blocks are copied raw, libs/gguf_libs/gguf_convert.h:201-229).
 * Values are an exact integer function of (seed, stream, index):
 *   x = (u1+u2+u3+u4 - 2*65535) * scale, u_i 16-bit slices of splitmix64,
 * i.e. a zero-mean bell-shaped variable with std = std_dev.
 * Q8_0 quantisation: d = fp16(amax/127), q = lrintf(x / fp32(d)) clamped to
 * [-127,127]; block = 2-byte fp16 d then 32 int8 (34 bytes). */
JYC_API int jyc_synth_f32(uint64_t seed, uint64_t stream, float std_dev,
                          float* out, size_t n);
JYC_API int jyc_synth_q8_0(uint64_t seed, uint64_t stream, float std_dev,
                           void* out_blocks, size_t rows, size_t k);
JYC_API int jyc_synth_ids(uint64_t seed, uint64_t stream, int vocab,
                          int* out, size_t n);
/* fp32 -> Q8_0 blocks (same rule as jyc_synth_q8_0). k % 32 == 0. */
JYC_API int jyc_quantize_q8_0(const float* x, void* out_blocks, size_t rows, size_t k);

/* ---- operator entry points (DEVICE pointers, asynchronous on `stream`) - */
/* Device layout of a Q8_0 matrix [n][k]: qs = n*k bytes holding q+128
 * (row-major), d = n*(k/32) fp16 scales (row-major). Produced from the
 * reference block layout by jyc_q8_repack. */
JYC_API int jyc_q8_repack(const void* blocks, int n, int k,
                          uint8_t* qs, uint16_t* d, void* stream);

/* C[m][n] = A[m][k] . W^T for a Q8_0 weight W [n][k]; fp32 activations,
 * exact fp16->fp32 scale x int8 weight products, fp32 accumulation.
 * m == 1: GEMV kernel. 2 <= m < 16: the few-row matmul (8 rows of A per
 * launch, activations held in registers, split-K partial sums summed in a
 * fixed order), stream-ordered scratch (cudaMallocAsync on `stream`) for the
 * partial sums. m >= 16: tcgen05 tensor-core tiles over exact fp16 hi/lo
 * splits of the dequantised weights and of A (fp32 accumulation in tensor
 * memory, drained every 128 of K); takes stream-ordered scratch for the
 * split copy of A.
 * Replaces qmat::matmul_q(a,b,c,m,n,k,Q8_0) (libs/matmul_libs/matmul_q.h:134-162). */
JYC_API int jyc_matmul_q8(const float* A, const uint8_t* qs, const uint16_t* d,
                          float* C, int m, int n, int k, void* stream);

/* C[m][n] = A[m][k] . W^T for a K-quant weight W [n][k] given as the
 * reference's super-blocks of 256 weights, row after row, on the device
 * (qtype JYC_Q4K: 144 B per block, JYC_Q5K: 176 B, JYC_Q6K: 210 B; GGUF's
 * block layout, as model.bf stores it). Each block is dequantised to the
 * reference's fp32 values (Q4_K as its AVX2+FMA path: fma(q, d*sc, -dmin*m);
 * Q5_K d*sc*q - dmin*m; Q6_K (d*sc)*q), accumulated in fp32. k % 256 == 0;
 * A 16-byte aligned, blocks 4-byte aligned. One kernel launch per 8 rows of A.
 * Replaces qmat::matmul_q(a,b,c,m,n,k,Q4K|Q5K|Q6K) (libs/matmul_libs/matmul_q.h:134-162). */
JYC_API int jyc_matmul_qk(const float* A, const void* blocks, float* C, int m, int n, int k,
                          int qtype, void* stream);

/* C[m][n] = A[m][k] . B with B given TRANSPOSED on the device, Bt [n][k]
 * (jyc_f32_transpose makes it from the reference's [k][n]).
 * Replaces matmul(m,n,k,A,B,C) (libs/matmul_libs/matmul.h:7-76). */
JYC_API int jyc_matmul_f32(const float* A, const float* Bt, float* C,
                           int m, int n, int k, void* stream);
JYC_API int jyc_f32_transpose(const float* B, float* Bt, int k, int n, void* stream);

/* C[m][n] = A[m][k] . B for fp16 (IEEE half) weights given TRANSPOSED on the
 * device, Bt [n][k] (jyc_f16_transpose makes it from the reference's [k][n]):
 * each half is converted to fp32 exactly and accumulated with fp32 FMAs.
 * Replaces matmul_f16_avx_fma / matmul_f16_classic(a,b,c,m,n,k)
 * (libs/matmul_libs/matmul_f16.h:8-41). */
JYC_API int jyc_matmul_f16(const float* A, const uint16_t* Bt, float* C,
                           int m, int n, int k, void* stream);
JYC_API int jyc_f16_transpose(const uint16_t* B, uint16_t* Bt, int k, int n, void* stream);

/* y = x * (1/sqrtf(sum(x^2)/n + eps)) * w, for `rows` rows of n.
 * Replaces rmsnorm(x,y,w,n,eps) (libs/model_libs/rmsnorm/rmsnorm.h:8-78). */
JYC_API int jyc_rmsnorm(const float* x, float* y, const float* w, int rows, int n,
                        float eps, void* stream);

/* In-place interleaved-pair rotation from the tables.
 * Replaces rope_pos(q,seq,start_pos,heads,hd,cos,sin) (libs/model_libs/rope/rope.h:108-110). */
JYC_API int jyc_rope_pos(float* q, int seq, int start_pos, int num_heads, int head_dim,
                         const float* cos_table, const float* sin_table, void* stream);

/* Per (row, head) int8 quantisation with one fp32 scale, bit-exact with
 * kv_pack_q8 (libs/model_libs/attention/attention_q8.h:20-37). */
JYC_API int jyc_kv_pack_q8(const float* src, int8_t* dst, float* scale,
                           int heads, int head_dim, int n, void* stream);

/* Int8-KV GQA attention for `seq` new rows at start_pos: packs K,V into the
 * cache, quantises Q per (row, head), int32 q.k dot, fp32 causal softmax,
 * out = sum p*vs*v. KV cache layout equals __KVq (attention_q8.h:12-19):
 * k,v [cap][num_kv_heads][head_dim] int8, ks,vs [cap][num_kv_heads] fp32.
 * Replaces attention_q8 (libs/model_libs/attention/attention_q8.h:38-184). */
JYC_API int jyc_attention_q8(const float* Q, const float* K, const float* V, float* out,
                             int seq, int start_pos, int num_heads, int num_kv_heads,
                             int head_dim, int8_t* kc, float* ks, int8_t* vc, float* vs,
                             int cap, void* stream);

/* jyc_attention_q8 without any allocation (no counterpart in the reference):
 * same arguments, kernels and results, but its scratch (quantised queries,
 * split partials, arrival counters) lives in one fixed device array of the
 * library image instead of stream-ordered cudaMallocAsync memory, for callers
 * that must not allocate (a caller inside a memory-pool-free region, a
 * real-time thread). Limits: num_heads * head_dim <= 8192, num_kv_heads <= 256,
 * and 8 * num_heads * head_dim * splits <= 1,048,576 floats of split partials
 * (splits = ceil((start_pos + seq) / chunk), chunk as jyc_attention_q8 picks
 * it); larger calls return JYC_ERR_ARG before launching anything. The first
 * call on a device resolves the array's address (cudaGetSymbolAddress with
 * that device current): make that first call before any stream capture. The
 * address is kept per device for the life of the process; after
 * cudaDeviceReset (or anything else that tears down the device's primary
 * context) it is stale, so do not call this entry point again after a reset. The
 * arrival counters must be zero when a call starts: they are at load and
 * every completed call leaves them so. Calls overlapping in time (other
 * streams, other host threads) share the array and race: serialise them. */
JYC_API int jyc_attention_q8_noalloc(const float* Q, const float* K, const float* V, float* out,
                                     int seq, int start_pos, int num_heads, int num_kv_heads,
                                     int head_dim, int8_t* kc, float* ks, int8_t* vc, float* vs,
                                     int cap, void* stream);

/* y = x / (1 + e^-x), with the reference's own exp polynomial for the
 * vector body. Replaces silu(x,y,n) (libs/model_libs/silu/silu.h:7-81). */
JYC_API int jyc_silu(const float* x, float* y, int n, void* stream);

/* First index of the maximum (strict >, ties -> lowest id) over n logits.
 * Replaces the greedy loop of generate_cached (libs/model_libs/generate.h:57-60). */
JYC_API int jyc_argmax(const float* logits, int n, int* out_index, void* stream);

/* The token pick of one generate step, on the device (all pointers device
 * memory; one CTA). Replaces the pick of generate_cached
 * (libs/model_libs/generate.h:50-77): for every out_ids[i], i in
 * [prompt_len, len), a positive logits[id] is divided by repetition_penalty
 * and a non-positive one multiplied (once per occurrence, in order); then
 * temperature <= 0 takes the first index of the maximum, else logits[v]
 * becomes expf((logits[v] - max) / temperature), *rng advances one LCG step
 * (rng * 1664525 + 1013904223) and the pick is the first v where
 * (rng >> 8) / 2^24 * sum minus the running sum reaches <= 0 (vocab_size - 1
 * if none). logits is modified in place, as in the reference. The sum runs in
 * double over 512 contiguous chunks (the reference: one running sum), and
 * expf is CUDA's (within its 2-ulp bound of the reference's libm). */
JYC_API int jyc_sample(float* logits, int vocab_size, float temperature, float repetition_penalty,
                       const int* out_ids, int prompt_len, int len, unsigned int* rng, int* next, void* stream);

/* ---- operator entry points with the reference's calling convention ------
 * HOST pointers in the reference's own layouts, caller-owned, synchronous:
 * each call copies its operands to the device, runs the device entry point
 * above (same kernels, same results) and copies the result back; the
 * reference's weight blocks are used as they are (Q8_0 34-byte blocks are
 * re-laid on the device inside the call). include/jieyu_b200_shim.hpp binds
 * them under the reference's C++ names. Errors as the device entry points. */
/* qmat::matmul_q(a,b,c,m,n,k,t) (libs/matmul_libs/matmul_q.h:134-162):
 * C[m][n] = A[m][k] . W^T, W [n][k/block] blocks of qtype (JYC_Q8_0, JYC_Q4K,
 * JYC_Q5K, JYC_Q6K). */
JYC_API int jyc_host_matmul_q(const float* a, const void* b, float* c, int m, int n, int k, int qtype);
/* matmul(m,n,k,A,B,C) (libs/matmul_libs/matmul.h:7-76): B fp32 [k][n]. */
JYC_API int jyc_host_matmul_f32(int m, int n, int k, const float* A, const float* B, float* C);
/* matmul_f16_avx_fma(a,b,c,m,n,k) (libs/matmul_libs/matmul_f16.h:19-41): b fp16 [k][n]. */
JYC_API int jyc_host_matmul_f16(const float* a, const uint16_t* b, float* c, int m, int n, int k);
/* matmul_w(B,m,n,k,A,C) (libs/model_libs/wmat_kernel.h:9-16): the WMat
 * dispatch (fp32 -> matmul, blocks -> matmul_q, fp16 -> matmul_f16, none ->
 * C = 0). */
JYC_API int jyc_host_matmul_w(const jyc_wmat* B, int m, int n, int k, const float* A, float* C);
/* rmsnorm(x,y,w,n,eps) (libs/model_libs/rmsnorm/rmsnorm.h:8-78). */
JYC_API int jyc_host_rmsnorm(const float* x, float* y, const float* w, int n, float eps);
/* rope_pos(q,seq,start_pos,heads,hd,cos,sin) (libs/model_libs/rope/rope.h:108-110):
 * in place; tables [max_seq][hd/2] as RoPETable. */
JYC_API int jyc_host_rope_pos(float* q, int seq, int start_pos, int num_heads, int head_dim,
                              const float* cos_table, const float* sin_table);
/* kv_pack_q8(src,dst,sc,heads,hd,n) (libs/model_libs/attention/attention_q8.h:20-37). */
JYC_API int jyc_host_kv_pack_q8(const float* src, int8_t* dst, float* sc, int heads, int head_dim, int n);
/* attention_q8(Q,K,V,out,seq,start_pos,H,KV,hd,kvq) (attention_q8.h:38-184):
 * the cache is the caller's __KVq (k,v [cap][KV][hd] int8, ks,vs [cap][KV]
 * fp32); rows [start_pos, start_pos+seq) are appended to it. An incomplete
 * cache (a null pointer or cap <= 0) works on a temporary one of seq rows at
 * position 0, as the reference does. */
JYC_API int jyc_host_attention_q8(const float* Q, const float* K, const float* V, float* out, int seq,
                                  int start_pos, int num_heads, int num_kv_heads, int head_dim,
                                  int8_t* kc, float* ks, int8_t* vc, float* vs, int cap);
/* silu(x,y,n) (libs/model_libs/silu/silu.h:7-81). */
JYC_API int jyc_host_silu(const float* x, float* y, int n);
/* ffn(x,w1,w2,w3,out,seq,hidden,inter) (libs/model_libs/ffn/ffn.h:7-19):
 * out = W2 (silu(W1 x) * (W3 x)). */
JYC_API int jyc_host_ffn(const float* x, const jyc_wmat* w1, const jyc_wmat* w2, const jyc_wmat* w3,
                         float* out, int seq, int hidden, int intermediate);

/* ---- model entry points ------------------------------------------------ */
typedef struct jyc_model jyc_model;

/* Uploads every weight once (the bind_model point, libs/model_libs/pipeline.h:63-153):
 * Q8_0 blocks are re-laid into the device layout, fp32 [in][out] matrices are
 * transposed, Q4_K / Q5_K / Q6_K blocks (input dimensions multiples of 256)
 * stay as they are and the K-quant matmul reads them in place when every
 * layer matrix is K-quant (the LM head and embedding are dequantised once to
 * the reference's fp32 values); K-quant mixed with fp32 matrices is
 * dequantised once and runs on the fp32 kernels; fp16 [in][out] matrices (matmul_f16.h)
 * are transposed and stay fp16 (2 bytes per weight streamed, converted to fp32
 * exactly in the GEMV; an fp16 embedding becomes fp32 rows); Q/K/V and
 * gate/up are fused. The layer weights are all Q8_0, all fp16, or fp32 and
 * K-quant mixed.
 * Allocates a device KV cache of desc->max_seq positions. Returns NULL on error. */
JYC_API jyc_model* jyc_model_create(const jyc_model_desc* desc);
JYC_API void jyc_model_free(jyc_model* m);
/* Bytes of weights one decode token streams (algorithmic, for rooflines). */
JYC_API double jyc_model_weight_bytes_per_token(const jyc_model* m);
/* Bytes of KV cache one decode token reads at context `ctx`. */
JYC_API double jyc_model_kv_bytes_per_token(const jyc_model* m, int ctx);

/* Full token loop, same contract as generate() (libs/model_libs/generate.h:90-112)
 * with an internal KV cache: out_ids[0..ret) = prompt then new tokens;
 * returns 0 if prompt_len<=0 or > max_seq, prompt_len if max_new_tokens<=0,
 * negative on error. temperature > 0 samples and repetition_penalty != 1
 * penalises as jyc_sample describes (the reference's LCG, seeded 12345 per
 * call, generate.h:36 and 50-77), on the device; a tensor-parallel shard
 * (vocabulary-sliced head) returns JYC_ERR_UNSUPPORTED for them. cb (may be
 * NULL) gets every new id in order; a non-zero return stops generation. */
JYC_API int jyc_generate(jyc_model* m, const int* prompt_ids, int prompt_len,
                         const int* eos_ids, int num_eos, int max_new_tokens,
                         float temperature, int* out_ids, float repetition_penalty,
                         jyc_token_cb cb, void* cb_ud);

/* One forward pass of `seq` tokens at start_pos through the device KV cache,
 * then the LM head on the last row: the step body of generate_cached
 * (libs/model_libs/generate.h:40-49). logits: host fp32[vocab]
 * (may be NULL); hidden_out: host fp32[hidden] final-norm output of the last
 * row (may be NULL). For teacher-forced parity checks. */
JYC_API int jyc_forward_logits(jyc_model* m, const int* ids, int seq, int start_pos,
                               float* logits, float* hidden_out);

/* Device KV cache contents for parity checks, copied to host in the reference
 * layout of __KVcache (libs/date_libs/date.h:89-147) for one layer:
 * k,v [npos][num_kv_heads][head_dim] int8, ks,vs [npos][num_kv_heads] fp32. */
JYC_API int jyc_model_read_kv(jyc_model* m, int layer, int npos,
                              int8_t* k, float* ks, int8_t* v, float* vs);
/* The reverse: positions [0, npos) of one layer's device KV cache from host
 * arrays in the same __KVcache order, so that a long context can be set up
 * without prefilling it (the reference's cache is a plain host array that
 * its tests may fill the same way, date.h:89-147). Synchronous. */
JYC_API int jyc_model_write_kv(jyc_model* m, int layer, int npos,
                               const int8_t* k, const float* ks, const int8_t* v, const float* vs);

/* ---- device-resident stepping (bench / device loop) -------------------- */
/* `stream` is used as given (0 = the legacy default stream). */
/* Prefill `prompt_len` ids (DEVICE int32 pointer) from position 0 and emit the
 * first greedy token into the device token buffer. Asynchronous on `stream`. */
JYC_API int jyc_prefill_device(jyc_model* m, const int* prompt_ids_dev, int prompt_len,
                               void* stream);
/* Run `n_steps` greedy decode steps from the current device state (each
 * consumes the last token and appends the next): one cooperative launch of
 * the decode kernel per step on models in the tiled layout, a captured CUDA
 * graph of the generic kernels otherwise; asynchronous on `stream`. */
JYC_API int jyc_decode_device(jyc_model* m, int n_steps, void* stream);
/* Reset the device state to `len` tokens already in the buffer (and their KV
 * entries in the cache), so decode can be replayed from the same point. */
JYC_API int jyc_model_rewind(jyc_model* m, int len, void* stream);
/* Kernels one decode step launches. */
JYC_API int jyc_model_kernels_per_step(const jyc_model* m);
/* 2 when the model decodes with the single-launch TMA-streamed decode kernel
 * (Q8_0 weights in the tiled layout), 0 with the generic kernels. */
JYC_API int jyc_model_decode_path(const jyc_model* m);
/* Tensor-parallel stepping (no counterpart in the reference, which runs on
 * one host): a model built from one rank's shard (its query and kv heads, its
 * gate/up rows, the matching input columns of O and down; norms, embedding and
 * LM head whole) decodes one token as a sequence of phase windows of the
 * decode kernel: [2l, 2l+1) = QKV, attention and the O projection of layer l,
 * [2l+1, 2l+2) = gate/up and down, [2L, 2L+1) = the LM head. O and down leave
 * per-rank partial sums (jyc_model_partials: device pointers and float counts)
 * that the caller all-reduces (sum over ranks) between windows; the next
 * window adds them into the residual stream. */
JYC_API int jyc_model_decode_window(jyc_model* m, int first, int last, void* stream);
/* Tensor parallel inside the decode kernel (no NCCL in the token loop): each
 * rank opens a receive area (jyc_model_tp_open returns its 64-byte CUDA IPC
 * handle), the callers exchange the handles (all-gather in rank order) and
 * connect (jyc_model_tp_connect maps every peer's area over NVLink). From
 * then on every decode step on every rank stores its O and down partial rows
 * into all ranks' areas and waits (bounded, error word 8) for all ranks'
 * arrivals: the ranks must step together, on one node, one GPU each. */
JYC_API int jyc_model_tp_open(jyc_model* m, int size, int rank, void* handle_out);
JYC_API int jyc_model_tp_connect(jyc_model* m, const void* handles);
JYC_API int jyc_model_partials(jyc_model* m, float** o_part, int* o_count, float** d_part, int* d_count);
/* Tensor-parallel prefill on a shard (no counterpart in the reference): runs
 * half-layer phases [first, last) of the batched prefill for the token rows
 * [start, start + rows) (ids already in the device token buffer; rows at most
 * the batched prefill's pass, jyc_model_prefill_partial's max_rows): phase 2l =
 * RMSNorm, QKV, RoPE + int8 cache append and attention of layer l, then the O
 * projection; phase 2l+1 = RMSNorm, gate/up + SwiGLU, down projection. O and
 * down write this shard's partial rows [rows][hidden] to the buffer that
 * jyc_model_prefill_partial returns (no residual add); the caller sums it over
 * the ranks (all-reduce) between windows, and the next window adds the sum to
 * the residual stream. Phase 0 starts from the embedding. */
JYC_API int jyc_model_prefill_window(jyc_model* m, int start, int rows, int first, int last, void* stream);
JYC_API int jyc_model_prefill_partial(jyc_model* m, float** part, int* max_rows);

/* ---- batched decode (configs[4]; no counterpart in the reference, whose
 * generate_cached runs one sequence, libs/model_libs/generate.h:9-89) ------- */
/* num_seqs independent sequences over one model, each with its own int8 KV
 * cache slot of the model's max_seq positions (the layout of the model's own
 * cache) and its own token buffer; every step appends one greedy token to
 * every sequence, with the same arithmetic per sequence as jyc_generate's
 * greedy steps. The matmuls of a step run over all num_seqs rows together:
 * the few-row matmul up to 8 sequences, tcgen05 token tiles from 9 on. Needs a
 * Q8_0 model with the batched prefill; at most min(512, max_seq, 256)
 * sequences. While a batch runs, the model must not decode on its own (they
 * share the model's activation buffers). */
typedef struct jyc_batch jyc_batch;
JYC_API jyc_batch* jyc_batch_create(jyc_model* m, int num_seqs);
JYC_API void jyc_batch_free(jyc_batch* b);
/* Prefill sequence `seq` with prompt_ids (HOST int32[prompt_len]) from
 * position 0 and append its first greedy token (synchronous). */
JYC_API int jyc_batch_prefill(jyc_batch* b, int seq, const int* prompt_ids, int prompt_len);
/* n_steps batched greedy steps on `stream` (one captured CUDA graph per
 * step); a sequence whose buffer is full stops growing. */
JYC_API int jyc_batch_decode(jyc_batch* b, int n_steps, void* stream);
/* Every sequence back to `len` tokens (its cache entries before len kept). */
JYC_API int jyc_batch_rewind(jyc_batch* b, int len, void* stream);
/* Copies up to cap ids of sequence `seq` (prompt + generated) to out_ids
 * (host); returns its length. Synchronises the device. */
JYC_API int jyc_batch_tokens(jyc_batch* b, int seq, int* out_ids, int cap);
/* 2: matmuls on the tcgen05 tiles, 1: the few-row matmul. */
JYC_API int jyc_batch_path(const jyc_batch* b);
JYC_API int jyc_batch_kernels_per_step(const jyc_batch* b);
/* KV-cache bytes one batched step reads with every sequence at context ctx. */
JYC_API double jyc_batch_kv_bytes_per_step(const jyc_batch* b, int ctx);

/* Error word of the device kernels: non-zero if a bounded wait gave up
 * (reset != 0 clears it). */
JYC_API int jyc_device_error(int reset);
/* Tracing of the decode megakernel: phase boundaries per step and one traced
 * step. out receives [ctas][points] SM-clock stamps; returns the CTA count.
 * Point 0 = start; per layer l at 1+23l: QKV input ready, QKV done, barrier,
 * attention done, barrier, O input ready, O done, barrier, gate/up input
 * ready, gate/up done, barrier, down input ready, down done, barrier, then 9
 * points inside the CTA's first attention item (start, queries ready, K/V in,
 * scores, softmax, P.V, partials written, arrival counted, merge done; 0 when
 * the CTA had no item); then the LM head: input ready, done, barrier. */
JYC_API int jyc_model_trace_points(const jyc_model* m);
JYC_API int jyc_model_trace_decode(jyc_model* m, void* stream, long long* out, int cap);
/* Per-kernel timing of decode: replays the step graph with an event after
 * every kernel, n_steps times from the current state. Arrays of 8 kernel
 * classes (embed, qkv, rope_quant, attention, o_proj, gate_up, down, head):
 * summed device ms, launch counts, algorithmic bytes of one launch. */
JYC_API int jyc_model_profile_decode(jyc_model* m, int n_steps, void* stream, double* ms,
                                     int* launches, double* bytes);
/* Device pointer to the int32 token buffer [max_seq] and host read of the
 * current length (synchronises the stream). */
JYC_API int* jyc_model_tokens_device(jyc_model* m);
JYC_API int jyc_model_length(jyc_model* m, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* JIEYU_B200_H */
