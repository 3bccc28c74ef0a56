// kernels.cuh — sm_100a kernels of the decode path and their launch helpers.
//
// Data layouts in HBM (the device copy is private, so it is laid out for the GPU):
//   Q8_0 matrix [n][k]   qs: n*k bytes, byte = q+128, row-major (16-byte vector loads);
//                        d : n*(k/32) fp16 scales, row-major.
//                        34 bytes per 32 weights, the same as the reference blocks.
//   fp32 matrix [n][k]   row-major (the reference's [k][n] transposed once at upload).
//   fp16 matrix [n][k]   row-major IEEE halves (the reference's [k][n] transposed once).
//   KV cache (model)     k8/v8 int8 [layer][kv_head][pos][head_dim], ks/vs fp32
//                        [layer][kv_head][pos]; the op-level entry uses the
//                        reference's [pos][kv_head][head_dim] through strides.
#pragma once
#include "common.cuh"

namespace jyc {

enum WType { W_Q8 = 0, W_F32 = 1, W_F16 = 2 };
enum Epi { EPI_STORE = 0, EPI_BIAS = 1, EPI_RESID = 2, EPI_SWIGLU = 3, EPI_ARGMAX = 4 };

// Step state shared by the kernels of one decode step (device memory).
struct DevState {
    int len;        // tokens in the token buffer (prompt + generated)
    int steps;      // tokens generated so far
    int max_new;    // stop after this many new tokens
    int max_len;    // stop when len reaches this (max_seq)
    int active;     // 0 -> every step kernel returns immediately
    int n_eos;
    int eos[16];
    unsigned long long amax;   // argmax slot (argmax_pack)
    unsigned int head_arrive;  // last-arriver counter of the LM-head grid
    unsigned int bar_base;     // grid-barrier counter value at the start of the next step
    unsigned int xbase;        // tensor-parallel exchanges of each kind completed (O / down, per step L each)
    float temperature;         // > 0: sample (the reference's sampler), else greedy
    float penalty;             // repetition penalty over the generated ids (1: none)
    unsigned int rng;          // the sampler's LCG state
    int prompt_len;            // generated ids start here (penalty range)
    int fresh;                 // the last head appended a token not yet re-picked by the sampler
    unsigned int apar;         // decode kernel: which half of its attention arrival counters this step uses
};

// Where a kernel finds its first position: from the step state (decode graph,
// pos0 = len-1, guarded by `active`) or from a host constant (prefill / ops).
struct PosSrc {
    const DevState* st;
    int pos0;
};
__device__ __forceinline__ bool pos_inactive(const PosSrc& p) {
    return p.st != nullptr && *(volatile const int*)&p.st->active == 0;
}
__device__ __forceinline__ int pos_first(const PosSrc& p) {
    return p.st != nullptr ? (*(volatile const int*)&p.st->len) - 1 : p.pos0;
}

struct GemvArgs {
    const float* x;        // activations [m][ldx]
    int ldx;
    int m, n, k;
    const uint8_t* qs;     // Q8 weights
    const uint16_t* d;
    const float* wt;       // fp32 weights [n][k]
    const uint16_t* wh;    // fp16 weights [n][k]
    const float* norm_w;   // optional fused RMSNorm of x (weights [k]); nullptr = off
    float eps;
    float* y;              // output [m][ldy]
    int ldy;
    const float* bias;     // EPI_BIAS
    DevState* st;          // EPI_ARGMAX: state updated by the last CTA; also the guard
    const int* tokens_ro;  // unused
    int* tokens;           // EPI_ARGMAX: token buffer
};

struct KVView {
    int8_t* k;
    float* ks;
    int8_t* v;
    float* vs;
    long long pos_stride;    // elements between positions (int8 arrays)
    long long head_stride;   // elements between kv heads (int8 arrays)
    long long spos_stride;   // scale arrays
    long long shead_stride;
    int cap;
};

struct RopeQuantArgs {
    const float* q;        // [rows][ldq] query heads
    const float* k;        // [rows][ldq] key heads
    const float* v;        // [rows][ldq] value heads
    int ldq;               // row stride of q/k/v (floats)
    int rows, H, KV, hd;
    const float* cos_t;    // nullptr: inputs are already rotated (quantise only)
    const float* sin_t;
    int8_t* q8;            // [rows][H][hd]
    float* qsc;            // [rows][H]
    float* q_roped;        // optional fp32 roped Q [rows][H*hd] (op-level parity), may be null
    float* k_roped;        // optional fp32 roped K [rows][KV*hd]
    KVView kv;
    PosSrc pos;
    // batched decode (row_len != null): row i is the last token of sequence i,
    // at position row_len[i] - 1, with its cache at kv + i * kv_row_stride
    const int* row_len;
    long long kv_row_stride;   // int8 elements between sequences' caches
    long long skv_row_stride;  // scale elements between sequences' caches
};

struct AttnArgs {
    const int8_t* q8;
    const float* qsc;
    KVView kv;
    int rows, H, KV, hd;
    int chunk;             // positions per split (multiple of 64)
    int nsplit;
    float scale;           // 1/sqrtf(hd)
    float* part_o;         // [rows][H][nsplit][hd]
    float* part_ml;        // [rows][H][nsplit][2]
    unsigned int* arrive;  // [KV] last-arriver counters (zero between launches)
    float* out;            // [rows][ldo]
    int ldo;
    PosSrc pos;
};

// ---- launchers (kernels.cu) ----------------------------------------------
int launch_gemv(const GemvArgs& a, int wtype, int epi, cudaStream_t s);
int launch_rmsnorm(const float* x, float* y, const float* w, int rows, int n, float eps,
                   cudaStream_t s);
int launch_add_rows(float* x, const float* p, size_t n, cudaStream_t s);
int launch_rope_quant(const RopeQuantArgs& a, cudaStream_t s);
int launch_rope(float* q, int seq, int start_pos, int heads, int hd, const float* cos_t,
                const float* sin_t, cudaStream_t s);
int attn_smem_bytes(int rows, int H, int KV, int hd);
int prepare_kernels();
int launch_attention(const AttnArgs& a, cudaStream_t s);
int launch_embed(const int* tokens, PosSrc pos, int rows, const float* ef, const uint8_t* eqs,
                 const uint16_t* ed, int hidden, float* X, cudaStream_t s);
int launch_q8_repack(const void* blocks, int n, int k, uint8_t* qs, uint16_t* d, int row_off,
                     int row_stride, cudaStream_t s);
int launch_transpose(const float* B, float* Bt, int k, int n, int row_off, int row_stride,
                     cudaStream_t s);
int launch_transpose_h(const uint16_t* B, uint16_t* Bt, int k, int n, int row_off, int row_stride, cudaStream_t s);
int launch_h2f(const uint16_t* h, float* f, size_t n, cudaStream_t s);
int launch_matmul_f16_generic(const float* A, const uint16_t* Bt, float* C, int m, int n, int k, cudaStream_t s);
int launch_silu(const float* x, float* y, int n, cudaStream_t s);
int launch_kv_pack(const float* src, int8_t* dst, float* sc, int heads, int hd, int n,
                   cudaStream_t s);
int launch_argmax(const float* v, int n, unsigned long long* slot, int* out, cudaStream_t s);
int launch_matmul_f32_generic(const float* A, const float* Bt, float* C, int m, int n, int k,
                              cudaStream_t s);
int launch_set_sampling(DevState* st, float temperature, float penalty, unsigned int rng, int prompt_len,
                        cudaStream_t s);
int launch_resample_last(DevState* st, float* logits, unsigned int* stag, int V, int* tokens, cudaStream_t s);
int launch_sample(float* logits, int V, float temperature, float penalty, const int* ids, int prompt_len, int len,
                  unsigned int* rng_dev, int* out_dev, cudaStream_t s);
int launch_set_state(DevState* st, int len, int max_new, int max_len, const int* eos, int n_eos,
                     cudaStream_t s);

// Matmul over K-quant weights in the reference's block layout (qtype
// JYC_Q4K / JYC_Q5K / JYC_Q6K, k % 256 == 0): y[m][n] = x[m][k] . W^T.
int launch_kquant_matmul(const float* x, int m, int n, int k, const uint8_t* wq, int qtype, float* y,
                         cudaStream_t s);
int launch_kquant_matmul_ld(const float* x, int ldx, int m, int n, int k, const uint8_t* wq, int qtype, float* y,
                            int ldy, cudaStream_t s);
// y[r][i] += bias[i] for rows r < rows (row stride ldy), i < n.
int launch_bias_rows(float* y, int ldy, const float* bias, int n, int rows, cudaStream_t s);
// h[i] = silu(g[i]) * u[i] (the reference's silu vector body, ffn.h:7-19).
int launch_swiglu_rows(const float* g, const float* u, float* h, size_t n, cudaStream_t s);
// K-quant rows [n][k/256 blocks] -> fp32 rows of `dst` ([.][k]), row r at
// row_off + r * row_stride, with the reference's dequantised values.
int launch_kquant_dequant(const uint8_t* blocks, int n, int k, int qtype, float* dst, int row_off, int row_stride,
                          cudaStream_t s);
// Bytes of one 256-weight super-block (0 for a type that is not a K-quant).
size_t kquant_block_bytes(int qtype);

}  // namespace jyc
