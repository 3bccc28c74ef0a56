// batch.cuh — kernels of batched decode: B independent sequences, each with
// its own int8 KV cache slot and length, stepped together (one token each).
#pragma once
#include "kernels.cuh"

namespace jyc {

// X[b] = embedding of tokens[b * tok_stride + lens[b] - 1] (fp32 copy or exact
// Q8_0 dequantisation, as embed_kernel).
int launch_bd_embed(const int* tokens, int tok_stride, const int* lens, int nseq, const float* ef,
                    const uint8_t* eqs, const uint16_t* ed, int hidden, float* X, cudaStream_t s);
// Greedy pick per sequence over logits [nseq][V]: the first index of the
// maximum (NaN never wins) is appended at tokens[b * tok_stride + lens[b]]
// and lens[b] advances (a full buffer, lens[b] >= cap, is left unchanged).
// slots: [nseq] zeroed 64-bit scratch, left zeroed.
int launch_bd_argmax(const float* logits, int V, int nseq, unsigned long long* slots, int* tokens,
                     int tok_stride, int* lens, int cap, cudaStream_t s);
// lens[b] = st->len (after a prefill through the model's own state).
int launch_bd_take_len(const DevState* st, int* lens, int b, cudaStream_t s);
// lens[b] = len for every b.
int launch_bd_set_lens(int* lens, int nseq, int len, cudaStream_t s);

// Attention of one new row per sequence over its own int8 KV cache slot.
struct BdAttn {
    const int8_t* q8;     // [nseq][H][hd] roped, quantised queries
    const float* qsc;     // [nseq][H]
    const int8_t* k8;     // this layer's cache in slot 0: [KV][cap][hd]
    const int8_t* v8;
    const float* ks;      // [KV][cap]
    const float* vs;
    long long slot_q;     // int8 elements between sequences' caches
    long long slot_s;     // scale elements between sequences' caches
    int cap, H, KV, hd;
    int chunk, nsplit;    // positions per split (multiple of 128), splits
    const int* lens;      // [nseq]: the new row sits at lens[b] - 1
    float scale;          // 1/sqrtf(hd)
    float* part_o;        // [nseq][H][nsplit][hd]
    float* part_ml;       // [nseq][H][nsplit][2]
    unsigned int* arrive; // [nseq][KV], zero at rest
    float* out;           // [nseq][ldo]
    int ldo;
};
bool bd_attention_supported(int H, int KV, int hd);
int bd_attention_chunk(int cap, int nseq, int KV);
int launch_bd_attention(const BdAttn& a, int nseq, cudaStream_t s);

}  // namespace jyc
