// batch.cu — the small kernels of batched decode (embedding gather by
// per-sequence length, per-sequence greedy argmax + append, length updates).
// The matmuls, RoPE/KV append and attention of a batched step are the model
// kernels run over B rows (kernels.cu with row_len, tcgemm.cu).
#include "batch.cuh"

namespace jyc {

namespace {

__global__ void bd_embed_kernel(const int* tokens, int tok_stride, const int* lens, const float* ef,
                                const uint8_t* eqs, const uint16_t* ed, int hidden, float* X) {
    const int b = blockIdx.x;
    const int id = tokens[(size_t)b * tok_stride + lens[b] - 1];
    float* xr = X + (size_t)b * hidden;
    for (int c = threadIdx.x; c < hidden; c += blockDim.x) {
        if (ef) {
            xr[c] = ef[(size_t)id * hidden + c];
        } else {
            const float q = (float)((int)eqs[(size_t)id * hidden + c] - 128);
            xr[c] = __fmul_rn(q, h2f(ed[(size_t)id * (hidden >> 5) + (c >> 5)]));
        }
    }
}

constexpr int kArgThreads = 256, kArgPer = 8;  // logits per thread per CTA

// CTA (chunk, sequence): packed maximum of its chunk into slots[b]
__global__ void __launch_bounds__(kArgThreads) bd_argmax_kernel(const float* logits, int V,
                                                                unsigned long long* slots) {
    const int b = blockIdx.y, tid = threadIdx.x;
    const int c0 = blockIdx.x * kArgThreads * kArgPer;
    const float* row = logits + (size_t)b * V;
    unsigned long long best = 0ull;
#pragma unroll
    for (int i = 0; i < kArgPer; i++) {
        const int v = c0 + i * kArgThreads + tid;
        if (v < V) best = max(best, argmax_pack(row[v], v));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
    __shared__ unsigned long long s_best[kArgThreads / 32];
    if ((tid & 31) == 0) s_best[tid >> 5] = best;
    __syncthreads();
    if (tid == 0) {
        for (int w = 1; w < kArgThreads / 32; w++) best = max(best, s_best[w]);
        atomicMax(slots + b, best);
    }
}

__global__ void bd_append_kernel(unsigned long long* slots, int nseq, int* tokens, int tok_stride, int* lens,
                                 int cap) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nseq) return;
    const unsigned long long p = slots[b];
    slots[b] = 0ull;
    const int len = lens[b];
    if (len >= cap) return;
    tokens[(size_t)b * tok_stride + len] = argmax_index(p);
    lens[b] = len + 1;
}

__global__ void bd_take_len_kernel(const DevState* st, int* lens, int b) { lens[b] = st->len; }

__global__ void bd_set_lens_kernel(int* lens, int nseq, int len) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b < nseq) lens[b] = len;
}

}  // namespace

int launch_bd_embed(const int* tokens, int tok_stride, const int* lens, int nseq, const float* ef,
                    const uint8_t* eqs, const uint16_t* ed, int hidden, float* X, cudaStream_t s) {
    bd_embed_kernel<<<nseq, 256, 0, s>>>(tokens, tok_stride, lens, ef, eqs, ed, hidden, X);
    JYC_LAUNCHED();
    return JYC_OK;
}

int launch_bd_argmax(const float* logits, int V, int nseq, unsigned long long* slots, int* tokens, int tok_stride,
                     int* lens, int cap, cudaStream_t s) {
    const dim3 grid((V + kArgThreads * kArgPer - 1) / (kArgThreads * kArgPer), nseq);
    bd_argmax_kernel<<<grid, kArgThreads, 0, s>>>(logits, V, slots);
    JYC_LAUNCHED();
    bd_append_kernel<<<(nseq + 127) / 128, 128, 0, s>>>(slots, nseq, tokens, tok_stride, lens, cap);
    JYC_LAUNCHED();
    return JYC_OK;
}

int launch_bd_take_len(const DevState* st, int* lens, int b, cudaStream_t s) {
    bd_take_len_kernel<<<1, 1, 0, s>>>(st, lens, b);
    JYC_LAUNCHED();
    return JYC_OK;
}

int launch_bd_set_lens(int* lens, int nseq, int len, cudaStream_t s) {
    bd_set_lens_kernel<<<(nseq + 127) / 128, 128, 0, s>>>(lens, nseq, len);
    JYC_LAUNCHED();
    return JYC_OK;
}

}  // namespace jyc
