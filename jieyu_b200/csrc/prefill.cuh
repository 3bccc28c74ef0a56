// prefill.cuh — causal attention of the batched prompt prefill (int8 KV cache).
#pragma once
#include "kernels.cuh"

namespace jyc {

constexpr int kPfQT = 16;    // query tokens per attention CTA
constexpr int kPfChunk = 4096;  // tokens per batched prefill pass (up to max_seq)
constexpr int kPfPartRows = 512;  // rows the K-split partial sums are sized for (fewer splits above)

struct PfAttn {
    const int8_t* q8;    // [T][H * hd] roped, quantised queries
    const float* qsc;    // [T][H]
    const int8_t* k8;    // this layer's cache [KV][max_seq][hd]
    const int8_t* v8;
    const float* ks;     // [KV][max_seq]
    const float* vs;
    int max_seq, H, KV, hd, T, pos0;
    int gc;              // query heads per CTA (set by launch_pf_attention)
    float scale;
    float* out;          // [T][H * hd]
};

int launch_pf_attention(const PfAttn& a, cudaStream_t s);
int prepare_pf_kernels();
bool pf_attention_supported(int H, int KV, int hd);

}  // namespace jyc
