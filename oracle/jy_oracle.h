/*
 * jy_oracle.h — TEST INFRASTRUCTURE ONLY: the CPU checker for the B200 path.
 *
 * A plain-C restatement of the jieyu reference hot path (the JIEYU_ISA=fma
 * code path: AVX2 + FMA, no AVX-VNNI), written so that every float operation
 * happens in the same order as the reference's 8-lane SIMD code. Pinned
 * against the reference itself (oracle/_ref) and the golden vectors under
 * tests/golden. Only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline use it; the product library never links it.
 */
#ifndef JY_ORACLE_H
#define JY_ORACLE_H
#include <stddef.h>
#include <stdint.h>
#include "jieyu_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

void jyo_set_threads(int n);
/* qmat::matmul_q Q8_0 (libs/matmul_libs/matmul_q.h:134-162): m==1 AVX2 lane order, m>1 scalar. */
void jyo_matmul_q8(const float* a, const void* b, float* c, int m, int n, int k);
/* K-quant weights (t = JYC_Q4K, JYC_Q5K, JYC_Q6K; k % 256 == 0); -1 for another t. */
int jyo_matmul_qk(const float* a, const void* b, float* c, int m, int n, int k, int t);
/* matmul (libs/matmul_libs/matmul.h:7-76), B = [k][n]. */
void jyo_matmul_f32(int m, int n, int k, const float* A, const float* B, float* C);
/* matmul_f16_avx_fma (libs/matmul_libs/matmul_f16.h:19-41): B fp16 [k][n]. */
void jyo_matmul_f16(const float* a, const uint16_t* b, float* c, int m, int n, int k);
/* rmsnorm (libs/model_libs/rmsnorm/x86/x86_classic.txt:1-27). */
void jyo_rmsnorm(const float* x, float* y, const float* w, int n, float eps);
/* RoPETable::init (libs/date_libs/date.h:52-66). */
void jyo_rope_table(int max_seq, int head_dim, float theta, float* cos_out, float* sin_out);
/* rope_pos (libs/model_libs/rope/x86/x86_classic.txt:1-39). */
void jyo_rope_pos(float* q, int seq, int start_pos, int heads, int hd, const float* cos_t,
                  const float* sin_t);
/* kv_pack_q8 (libs/model_libs/attention/attention_q8.h:20-37). */
void jyo_kv_pack_q8(const float* src, int8_t* dst, float* sc, int heads, int hd, int n);
/* attention_q8 (attention_q8.h:38-184 + attention/x86/x86_classic.txt:1-75).
 * Cache layout [cap][KV][hd] int8 + [cap][KV] fp32. Returns 0, or -1 on misuse. */
int jyo_attention_q8(const float* Q, const float* K, const float* V, float* out, int seq,
                     int start_pos, int H, int KV, int hd, int8_t* kc, float* ks, int8_t* vc,
                     float* vs, int cap);
/* silu (libs/model_libs/silu/x86/x86_classic.txt:1-32). */
void jyo_silu(const float* x, float* y, int n);

/* Model level: a KV cache like __KVcache (libs/date_libs/date.h:89-147). */
void* jyo_cache_create(int L, int max_seq, int KV, int hd);
void jyo_cache_free(void* c);
void jyo_cache_read(void* c, int layer, int npos, int8_t* k, float* ks, int8_t* v, float* vs);
void jyo_cache_write(void* c, int layer, int npos, const int8_t* k, const float* ks, const int8_t* v,
                     const float* vs);
/* generate_cached step body (generate.h:43-49): embed rows, forward_cached, LM head. */
int jyo_forward_logits(const jyc_model_desc* d, void* cache, const int* ids, int seq,
                       int start_pos, float* logits, float* hidden_out);
/* generate (generate.h:90-112), greedy or LCG sampling, repetition penalty. */
int jyo_sample(float* logits, int V, float temperature, float rep_penalty, const int* out_ids,
               int prompt_len, int len, unsigned* rng);
int jyo_generate(const jyc_model_desc* d, const int* prompt, int prompt_len, const int* eos,
                 int num_eos, int max_new, float temperature, int* out_ids, float rep_penalty);

/* Seeded synthetic weights / prompt ids (byte-identical to jyc_synth_*). */
void jyo_synth_f32(uint64_t seed, uint64_t stream, float std_dev, float* out, size_t n);
void jyo_synth_q8_0(uint64_t seed, uint64_t stream, float std_dev, void* out_blocks, size_t rows, size_t k);
void jyo_synth_ids(uint64_t seed, uint64_t stream, int vocab, int* out, size_t n);

#ifdef __cplusplus
}
#endif
#endif
