// prefill.cuh — batched-token kernels of prompt prefill (Q8_0 weights in the
// tiled decode layout; int8 KV cache).
#pragma once
#include "kernels.cuh"

namespace jyc {

constexpr int kPfTok = 64;   // tokens per token tile of the digit layout
constexpr int kPfRows = 64;  // weight rows per CTA tile
constexpr int kPfQT = 16;    // query tokens per attention CTA
constexpr int kPfChunk = 512;  // tokens per batched prefill pass

enum PfEpi { PF_STORE = 0, PF_BIAS, PF_RESID, PF_SWIGLU };

struct PfGemm {
    const uint8_t* qs;   // tiled weights (see mega.cuh)
    const uint16_t* d;
    int n, k;
    const int8_t* dig;   // token digits (pf_digitize)
    const float* sx;
    int T;               // tokens
    float* y;            // [T][ldy]
    int ldy;
    const float* bias;
    int* err;
};

struct PfAttn {
    const int8_t* q8;    // [T][H * hd] roped, quantised queries
    const float* qsc;    // [T][H]
    const int8_t* k8;    // this layer's cache [KV][max_seq][hd]
    const int8_t* v8;
    const float* ks;     // [KV][max_seq]
    const float* vs;
    int max_seq, H, KV, hd, T, pos0;
    float scale;
    float* out;          // [T][H * hd]
};

size_t pf_digit_bytes(int T, int k);
size_t pf_scale_floats(int T, int k);
int launch_pf_digitize(const float* x, int ldx, int T, int k, const float* w, float eps, int8_t* dig, float* sx,
                       cudaStream_t s);
int launch_pf_gemm(const PfGemm& p, int epi, cudaStream_t s);
int launch_pf_attention(const PfAttn& a, cudaStream_t s);
int prepare_pf_kernels();
bool pf_attention_supported(int H, int KV, int hd);

}  // namespace jyc
