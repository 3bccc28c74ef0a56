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

}  // namespace jyc
