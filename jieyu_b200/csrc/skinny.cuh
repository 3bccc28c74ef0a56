// skinny.cuh — Q8_0 matmul over a few activation rows (2..15 sequences of a
// batched decode step, or a short C-ABI matmul): y[t][r] = sum_k W[r][k] x[t][k]
// with the reference's numerics (fp32 activations times exactly dequantised
// weights, qmat::matmul_q, libs/matmul_libs/matmul_q.h:101-143).
//
// The work is split into warp units of RW weight rows x one 512-column K
// slice. A lane owns 16 columns of the slice and keeps the (optionally
// RMSNorm'd) activations of all rows for them in registers, so every weight
// byte that arrives through the warp's cp.async copies meets its activations
// without another load; products are formed with packed f32x2 FMAs, and the
// per-lane partial sums of 32/MT rows x MT activation rows are folded across
// the warp by a transposing butterfly (one result per lane). Slices of a row
// unit are summed in slice order by the last unit to arrive (deterministic).
#pragma once
#include "kernels.cuh"

namespace jyc {

constexpr int kSkMaxRows = 8;    // activation rows per launch
constexpr int kSkSlice = 512;    // K columns per warp unit
constexpr int kSkWarps = 4;      // warps (row units) per CTA, all on one slice

struct SkinnyGemm {
    const float* x;        // activations [m][ldx]
    int ldx, m, n, k;      // 1 <= m <= kSkMaxRows, k % 32 == 0
    const uint8_t* qs;     // Q8_0 weights [n][k], byte = q + 128
    const uint16_t* d;     // fp16 scales [n][k/32]
    const float* norm_w;   // fused RMSNorm weights [k], or nullptr
    float eps;
    float* y;              // [m][ldy]
    int ldy;
    const float* bias;     // EPI_BIAS: [n]
};

// Device workspace of one stream's few-row matmuls (reused launch after launch).
struct SkinnyWork {
    float* part;           // split-K partial sums, skinny_part_floats(n, k) at least
    unsigned int* cnt;     // arrival counters, skinny_counters(n) at least, zero at rest
    float* sc;             // kSkMaxRows RMSNorm scales
};

size_t skinny_part_floats(int n, int k);
size_t skinny_counters(int n);
// Launches the RMSNorm scale kernel (when norm_w is set) and the matmul.
// epi: EPI_STORE, EPI_BIAS, EPI_RESID or EPI_SWIGLU (rows 2j, 2j+1 = gate_j, up_j).
int launch_skinny(const SkinnyGemm& g, int epi, const SkinnyWork& w, cudaStream_t s);
int prepare_skinny_kernels();

}  // namespace jyc
