// tcgemm.cuh — tcgen05 (5th-generation tensor core) GEMM for Q8_0 weights
// over many tokens: prompt prefill and batched decode of 16+ sequences.
//
// Y[t][r] = sum_k W[r][k] x[t][k] with the reference's numerics (fp32
// activations times exactly dequantised weights, qmat::matmul_q,
// libs/matmul_libs/matmul_q.h:101-143). The tensor cores take fp16 operands,
// so both sides are split exactly into two fp16 planes:
//   w = q * d is an 18-bit product: scaled by a power of two per row,
//       hi = fp16(w), lo = fp16(w - hi) holds the rest exactly;
//   x is scaled by a power of two per token and split the same way (22 of its
//       24 bits kept; the dropped part is below 2^-22 of each element).
// Three MMAs per K step (hi.hi + hi.lo + lo.hi) accumulate in fp32 in tensor
// memory; the epilogue undoes both power-of-two scales exactly.
#pragma once
#include <cuda_fp16.h>

#include "kernels.cuh"

namespace jyc {

enum TcEpi { TC_STORE = 0, TC_BIAS, TC_RESID, TC_SWIGLU };

struct TcGemm {
    const uint8_t* qs;   // Q8_0 weights [n][k], byte = q + 128 (row-major device copy)
    const uint16_t* d;   // fp16 scales [n][k/32]
    const uint8_t* rexp; // [n] fp16 exponent field of each row's max |d| (launch_tc_rowexp)
    int n, k;
    const __half* xs;    // split activations in the tc_split layout for token tile N
    const int* xe;       // per-token power-of-two exponents [token tiles * N]
    int T, N;            // tokens; token tile (16, 32, 64 or 128)
    float* y;            // [T][ldy]
    int ldy;
    const float* bias;   // TC_BIAS: [n]
    int splits;          // K splits (1: no partial sums)
    float* part;         // splits > 1: [splits][T][n] partial sums
    unsigned int* cnt;   // splits > 1: [row tiles * token tiles] arrival counters, zero at rest
    int* err;            // device error word (bounded waits)
};

constexpr int kTcRows = 128;  // weight rows per CTA tile (UMMA M)
constexpr int kTcKC = 64;     // K elements per pipeline chunk
constexpr int kTcMaxSplits = 16; // K splits at most
constexpr int kTcMinRows = 16;  // activation rows from which a matmul runs on the tensor cores

// Token tile width used for T tokens.
int tc_token_tile(int T);
// Halves of the split-activation buffer for T tokens of k columns at tile N.
size_t tc_split_halves(int T, int N, int k);
// Token rows (T padded to the tile) = entries of the exponent array.
int tc_padded_tokens(int T, int N);
// Token tile N and K splits (1 = none, at most max_splits) for an n x k
// weight over T tokens: the pair with the least modelled time.
void tc_plan(int n, int k, int T, int max_splits, int* N, int* splits);

// x [T][ldx] (optionally RMSNorm'd with weights norm_w) -> fp16 hi/lo planes
// in the swizzled tile layout the GEMM copies with one bulk copy per chunk.
int launch_tc_split(const float* x, int ldx, int T, int k, const float* norm_w, float eps, int N, __half* xs,
                    int* xe, cudaStream_t s);
int launch_tc_gemm(const TcGemm& p, int epi, cudaStream_t s);
// rexp[r] = exponent field of max_b |d[r][b]| (the GEMM scales row r by
// 2^(22 - rexp[r]) before splitting it into fp16 hi/lo).
int launch_tc_rowexp(const uint16_t* d, int n, int k, uint8_t* rexp, cudaStream_t s);
int prepare_tc_kernels();

}  // namespace jyc
