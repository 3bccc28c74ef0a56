// kquant.cu — matmul over K-quant weights (Q4_K, Q5_K, Q6_K super-blocks of
// 256 weights, the reference's block layouts read in place): y[t][r] =
// sum_k W[r][k] x[t][k] for up to 8 activation rows per launch.
//
// Reference: qmat::matmul_q with t = Q4K / Q5K / Q6K
// (libs/matmul_libs/matmul_q.h:134-162): every block is dequantised to fp32
// (Q4_K as file_libs/q4/q4_fma.txt does, w = fma(q, d*sc, -(dmin*mn)); Q5_K
// d1*q - n1, matmul_q.h:52-77; Q6_K (d*sc)*q, matmul_q.h:78-100) and dotted
// with x in fp32. Here the dequantised values are the same floats; only the
// summation order of the dot differs.
//
// One CTA per pair of consecutive weight rows (grid-stride), its 8 warps
// splitting the rows' super-blocks (block bl to warp bl % 8); lane l
// dequantises 8 of each super-block's 256 weights:
//   Q4_K / Q5_K: group g = l/8 of 64 weights, byte quad p = 4 (l%8): the low
//     nibbles are weights 64g+p..+3 (sub-block 2g), the high nibbles
//     64g+32+p..+3 (sub-block 2g+1);
//   Q6_K: position l of both 128-weight halves: weights 128h + l + 32j.
// Per-lane fp32 FMAs, a warp sum, then the 8 warps' sums in warp order.
// Rows whose bytes are a multiple of 16 are staged in shared memory first
// (kq_gemv_smem_kernel); others are read in place (kq_gemv_kernel).
#include <algorithm>

#include "kernels.cuh"

namespace jyc {

namespace {

constexpr int kKqWarps = 8;
constexpr int kKqMaxRows = 8;
// consecutive weight rows per CTA (bytes in flight, shared x loads; 4 rows
// measured slower: registers halve the resident CTAs)
constexpr int kKqRowsPerCta = 2;

__device__ __forceinline__ float kq_h2f(uint32_t bits) { return __half2float(__ushort_as_half((uint16_t)bits)); }

// 6-bit scale / min of sub-block j from the 12 scale bytes q
// (matmul_q.h:24-33 get_scale_min_k4)
__device__ __forceinline__ void kq_scale_min(int j, const uint8_t* q, unsigned& sc, unsigned& mn) {
    if (j < 4) {
        sc = q[j] & 63u;
        mn = q[j + 4] & 63u;
    } else {
        sc = (q[j + 4] & 0xFu) | ((unsigned)(q[j - 4] >> 6) << 4);
        mn = (unsigned)(q[j + 4] >> 4) | ((unsigned)(q[j] >> 6) << 4);
    }
}

// Small non-negative integers to exact floats without a conversion
// instruction: the float with bits 0x4B000000 | v is 2^23 + v.
__device__ __forceinline__ float kq_small_f32(unsigned v, float bias) {  // v < 2^23; bias = 2^23 + offset
    return __fsub_rn(__uint_as_float(0x4B000000u | v), bias);
}
__device__ __forceinline__ float kq_byte_f32(uint32_t w, int i) {  // byte i of w
    return __fsub_rn(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540u + i)), 8388608.0f);
}

template <int QT>
constexpr int kq_block_bytes() {
    return QT == JYC_Q4K ? 144 : QT == JYC_Q5K ? 176 : 210;
}

// The 8 dequantised weights of lane `lane` in super-block `b` and the
// offsets (within the block's 256) of the first four / last four of them
// (Q6_K: o0 only, its weights sit at 128h + o0 + 32j).
template <int QT>
__device__ __forceinline__ void kq_dequant(const uint8_t* b, int lane, float (&w)[8], int& o0, int& o1) {
    if (QT == JYC_Q6K) {
        // ql[128] | qh[64] | int8 scales[16] | fp16 d
        const float d = kq_h2f(*reinterpret_cast<const uint16_t*>(b + 208));
        const int8_t* sc = reinterpret_cast<const int8_t*>(b + 192);
        const int is = lane >> 4;
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const unsigned l0 = b[64 * h + lane], l1 = b[64 * h + lane + 32], hh = b[128 + 32 * h + lane];
            // 6-bit q as float minus 32: 2^23 + q - (2^23 + 32), exact
            const float q1 = kq_small_f32((l0 & 0xFu) | (((hh >> 0) & 3u) << 4), 8388640.0f);
            const float q2 = kq_small_f32((l1 & 0xFu) | (((hh >> 2) & 3u) << 4), 8388640.0f);
            const float q3 = kq_small_f32((l0 >> 4) | (((hh >> 4) & 3u) << 4), 8388640.0f);
            const float q4 = kq_small_f32((l1 >> 4) | (((hh >> 6) & 3u) << 4), 8388640.0f);
            const int s = 8 * h + is;
            w[4 * h + 0] = __fmul_rn(__fmul_rn(d, (float)sc[s]), q1);
            w[4 * h + 1] = __fmul_rn(__fmul_rn(d, (float)sc[s + 2]), q2);
            w[4 * h + 2] = __fmul_rn(__fmul_rn(d, (float)sc[s + 4]), q3);
            w[4 * h + 3] = __fmul_rn(__fmul_rn(d, (float)sc[s + 6]), q4);
        }
        o0 = lane;  // weights 128h + lane + 32j
        o1 = 0;
    } else {
        const uint32_t dd = *reinterpret_cast<const uint32_t*>(b);  // fp16 d | fp16 dmin
        const float d = kq_h2f(dd & 0xFFFFu), dmin = kq_h2f(dd >> 16);
        const int g = lane >> 3, p = 4 * (lane & 7);
        unsigned s0, m0, s1, m1;
        kq_scale_min(2 * g, b + 4, s0, m0);
        kq_scale_min(2 * g + 1, b + 4, s1, m1);
        const float d1 = __fmul_rn(d, (float)s0), n1 = __fmul_rn(dmin, (float)m0);
        const float d2 = __fmul_rn(d, (float)s1), n2 = __fmul_rn(dmin, (float)m1);
        const uint8_t* qs = b + (QT == JYC_Q4K ? 16 : 48) + 32 * g + p;
        const uint32_t q = *reinterpret_cast<const uint32_t*>(qs);
        uint32_t lo = q & 0x0F0F0F0Fu, hi = (q >> 4) & 0x0F0F0F0Fu;  // 4 quants per word, one per byte
        if (QT == JYC_Q5K) {  // + 16 where the high bit (bit 2g / 2g+1 of qh[l]) is set
            const uint32_t qh = *reinterpret_cast<const uint32_t*>(b + 16 + p);
            lo |= ((qh >> (2 * g)) & 0x01010101u) << 4;
            hi |= ((qh >> (2 * g + 1)) & 0x01010101u) << 4;
        }
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float fl = kq_byte_f32(lo, i), fh = kq_byte_f32(hi, i);
            if (QT == JYC_Q4K) {
                w[i] = __fmaf_rn(fl, d1, -n1);
                w[4 + i] = __fmaf_rn(fh, d2, -n2);
            } else {
                w[i] = __fsub_rn(__fmul_rn(d1, fl), n1);
                w[4 + i] = __fsub_rn(__fmul_rn(d2, fh), n2);
            }
        }
        o0 = 64 * g + p;       // w[0..3]
        o1 = 64 * g + 32 + p;  // w[4..7]
    }
}

// Q4_K / Q5_K, 16 weights per lane (l16 = 0..15 of a half warp): group
// g = l16/4, byte octet p = 8 (l16%4): low nibbles -> weights 64g+p..+7 (w[0..7],
// sub-block 2g), high nibbles -> 64g+32+p..+7 (w[8..15], sub-block 2g+1).
template <int QT>
__device__ __forceinline__ void kq_dequant16(const uint8_t* b, int l16, float (&w)[16], int& o0, int& o1) {
    const uint32_t dd = *reinterpret_cast<const uint32_t*>(b);  // fp16 d | fp16 dmin
    const float d = kq_h2f(dd & 0xFFFFu), dmin = kq_h2f(dd >> 16);
    const int g = l16 >> 2, p = 8 * (l16 & 3);
    unsigned s0, m0, s1, m1;
    kq_scale_min(2 * g, b + 4, s0, m0);
    kq_scale_min(2 * g + 1, b + 4, s1, m1);
    const float d1 = __fmul_rn(d, (float)s0), n1 = __fmul_rn(dmin, (float)m0);
    const float d2 = __fmul_rn(d, (float)s1), n2 = __fmul_rn(dmin, (float)m1);
    const uint2 q = *reinterpret_cast<const uint2*>(b + (QT == JYC_Q4K ? 16 : 48) + 32 * g + p);
    uint32_t lo[2] = {q.x & 0x0F0F0F0Fu, q.y & 0x0F0F0F0Fu};
    uint32_t hi[2] = {(q.x >> 4) & 0x0F0F0F0Fu, (q.y >> 4) & 0x0F0F0F0Fu};
    if (QT == JYC_Q5K) {  // + 16 where the high bit (bit 2g / 2g+1 of qh[l]) is set
        const uint2 qh = *reinterpret_cast<const uint2*>(b + 16 + p);
        lo[0] |= ((qh.x >> (2 * g)) & 0x01010101u) << 4;
        lo[1] |= ((qh.y >> (2 * g)) & 0x01010101u) << 4;
        hi[0] |= ((qh.x >> (2 * g + 1)) & 0x01010101u) << 4;
        hi[1] |= ((qh.y >> (2 * g + 1)) & 0x01010101u) << 4;
    }
#pragma unroll
    for (int h = 0; h < 2; h++)
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float fl = kq_byte_f32(lo[h], i), fh = kq_byte_f32(hi[h], i);
            if (QT == JYC_Q4K) {
                w[4 * h + i] = __fmaf_rn(fl, d1, -n1);
                w[8 + 4 * h + i] = __fmaf_rn(fh, d2, -n2);
            } else {
                w[4 * h + i] = __fsub_rn(__fmul_rn(d1, fl), n1);
                w[8 + 4 * h + i] = __fsub_rn(__fmul_rn(d2, fh), n2);
            }
        }
    o0 = 64 * g + p;
    o1 = 64 * g + 32 + p;
}

// Q6_K, 16 weights per lane (l16 = 0..15 of a half warp): positions
// pp = 2 l16 and pp + 1 of both 128-weight halves h; w[8h + 4e + j] is the
// weight at 128h + pp + e + 32j (its scale sc[8h + pp/16 + 2j] is shared by
// both positions).
__device__ __forceinline__ void kq_dequant16_q6(const uint8_t* b, int l16, float (&w)[16]) {
    const float d = kq_h2f(*reinterpret_cast<const uint16_t*>(b + 208));
    const int8_t* sc = reinterpret_cast<const int8_t*>(b + 192);
    const int pp = 2 * l16, is = l16 >> 3;
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const unsigned ql0 = *reinterpret_cast<const uint16_t*>(b + 64 * h + pp);
        const unsigned ql1 = *reinterpret_cast<const uint16_t*>(b + 64 * h + 32 + pp);
        const unsigned hh = *reinterpret_cast<const uint16_t*>(b + 128 + 32 * h + pp);
        float ds[4];
#pragma unroll
        for (int j = 0; j < 4; j++) ds[j] = __fmul_rn(d, (float)sc[8 * h + is + 2 * j]);
#pragma unroll
        for (int e = 0; e < 2; e++) {
            const unsigned l0 = (ql0 >> (8 * e)) & 0xFFu, l1 = (ql1 >> (8 * e)) & 0xFFu, hb = (hh >> (8 * e)) & 0xFFu;
            w[8 * h + 4 * e + 0] = __fmul_rn(ds[0], kq_small_f32((l0 & 0xFu) | ((hb & 3u) << 4), 8388640.0f));
            w[8 * h + 4 * e + 1] = __fmul_rn(ds[1], kq_small_f32((l1 & 0xFu) | (((hb >> 2) & 3u) << 4), 8388640.0f));
            w[8 * h + 4 * e + 2] = __fmul_rn(ds[2], kq_small_f32((l0 >> 4) | (((hb >> 4) & 3u) << 4), 8388640.0f));
            w[8 * h + 4 * e + 3] = __fmul_rn(ds[3], kq_small_f32((l1 >> 4) | (((hb >> 6) & 3u) << 4), 8388640.0f));
        }
    }
}

template <int QT, int MT>
__global__ void __launch_bounds__(kKqWarps * 32) kq_gemv_kernel(const float* __restrict__ x, int ldx, int m, int n,
                                                                int k, const uint8_t* __restrict__ wq,
                                                                float* __restrict__ y, int ldy) {
    constexpr int BB = kq_block_bytes<QT>();
    constexpr int R = kKqRowsPerCta;
    __shared__ float s_part[kKqWarps][MT][R];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nblk = k >> 8;
    const size_t rbytes = (size_t)nblk * BB;
    for (int row0 = blockIdx.x * R; row0 < n; row0 += gridDim.x * R) {
        const uint8_t* rp[R];
#pragma unroll
        for (int r = 0; r < R; r++) rp[r] = wq + (size_t)min(row0 + r, n - 1) * rbytes;  // a missing last row re-reads row n-1
        float acc[MT][R];
#pragma unroll
        for (int t = 0; t < MT; t++)
#pragma unroll
            for (int r = 0; r < R; r++) acc[t][r] = 0.0f;
        // warp w takes super-blocks w, w + kKqWarps, ... of the CTA's rows
#pragma unroll 2
        for (int bl = warp; bl < nblk; bl += kKqWarps) {
            float w[R][8];
            int o0 = 0, o1 = 0;
#pragma unroll
            for (int r = 0; r < R; r++) kq_dequant<QT>(rp[r] + (size_t)bl * BB, lane, w[r], o0, o1);
            const int base = bl * 256;
#pragma unroll
            for (int t = 0; t < MT; t++) {
                if (t >= m) continue;
                const float* xr = x + (size_t)t * ldx + base;
                float xv[8];
                if (QT == JYC_Q6K) {
#pragma unroll
                    for (int j = 0; j < 8; j++) xv[j] = __ldg(xr + 128 * (j >> 2) + o0 + 32 * (j & 3));
                } else {
                    const float4 xa = __ldg(reinterpret_cast<const float4*>(xr + o0));
                    const float4 xb = __ldg(reinterpret_cast<const float4*>(xr + o1));
                    xv[0] = xa.x; xv[1] = xa.y; xv[2] = xa.z; xv[3] = xa.w;
                    xv[4] = xb.x; xv[5] = xb.y; xv[6] = xb.z; xv[7] = xb.w;
                }
#pragma unroll
                for (int r = 0; r < R; r++)
#pragma unroll
                    for (int j = 0; j < 8; j++) acc[t][r] = __fmaf_rn(w[r][j], xv[j], acc[t][r]);
            }
        }
        // per warp, then the warps in order (fixed summation order)
#pragma unroll
        for (int t = 0; t < MT; t++)
#pragma unroll
            for (int r = 0; r < R; r++) {
                const float v = warp_sum(acc[t][r]);
                if (lane == 0) s_part[warp][t][r] = v;
            }
        __syncthreads();
        if (threadIdx.x < MT * R) {
            const int t = threadIdx.x / R, r = threadIdx.x % R;
            float v = 0.0f;
            for (int w2 = 0; w2 < kKqWarps; w2++) v = __fadd_rn(v, s_part[w2][t][r]);
            if (t < m && row0 + r < n) y[(size_t)t * ldy + row0 + r] = v;
        }
        __syncthreads();  // s_part is reused by the next rows
    }
}

// Rows staged in shared memory: a CTA copies R = 8 whole weight rows (row
// bytes a multiple of 16) with 16-byte cp.async, every copy in flight at
// once; then warp w dequantises row w's super-blocks from shared memory and
// writes its warp sum (one warp per row: nothing to select or merge). Lanes
// take 16 weights of a block (a half warp per block, two blocks per step).
__device__ __forceinline__ void kq_cp16(uint32_t dst, const void* src, int bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
}

template <int QT, int MT>
__global__ void __launch_bounds__(kKqWarps * 32) kq_gemv_smem_kernel(const float* __restrict__ x, int ldx, int m,
                                                                     int n, int k, const uint8_t* __restrict__ wq,
                                                                     float* __restrict__ y, int ldy) {
    constexpr int BB = kq_block_bytes<QT>();
    constexpr int R = kKqWarps;
    extern __shared__ __align__(16) unsigned char kq_sm[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nblk = k >> 8;
    const int rbytes = nblk * BB;  // a multiple of 16
    const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(kq_sm);
    for (int row0 = blockIdx.x * R; row0 < n; row0 += gridDim.x * R) {
        const int nr = min(R, n - row0);
        const uint8_t* src = wq + (size_t)row0 * rbytes;
        const int chunks = nr * (rbytes >> 4);
        for (int c = tid; c < chunks; c += kKqWarps * 32) kq_cp16(sbase + 16 * c, src + (size_t)16 * c, 16);
        asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
        __syncthreads();
        if (warp < nr) {
            const unsigned char* rowp = kq_sm + warp * rbytes;
            float acc[MT];
#pragma unroll
            for (int t = 0; t < MT; t++) acc[t] = 0.0f;
            if (QT == JYC_Q6K) {  // half warp hw takes blocks 2i + hw, 16 weights per lane
                const int hw = lane >> 4, l16 = lane & 15, pp = 2 * l16;
#pragma unroll 2
                for (int bl = hw; bl < nblk; bl += 2) {
                    float w[16];
                    kq_dequant16_q6(rowp + bl * BB, l16, w);
#pragma unroll
                    for (int t = 0; t < MT; t++) {
                        if (t >= m) continue;
                        const float* xr = x + (size_t)t * ldx + bl * 256 + pp;
#pragma unroll
                        for (int h = 0; h < 2; h++)
#pragma unroll
                            for (int j = 0; j < 4; j++) {
                                const float2 xv = __ldg(reinterpret_cast<const float2*>(xr + 128 * h + 32 * j));
                                acc[t] = __fmaf_rn(w[8 * h + j], xv.x, acc[t]);
                                acc[t] = __fmaf_rn(w[8 * h + 4 + j], xv.y, acc[t]);
                            }
                    }
                }
            } else {  // Q4_K / Q5_K: half warp h takes blocks 2i + h, 16 weights per lane
                const int h = lane >> 4, l16 = lane & 15;
#pragma unroll 2
                for (int bl = h; bl < nblk; bl += 2) {
                    float w[16];
                    int o0 = 0, o1 = 0;
                    kq_dequant16<QT>(rowp + bl * BB, l16, w, o0, o1);
#pragma unroll
                    for (int t = 0; t < MT; t++) {
                        if (t >= m) continue;
                        const float* xr = x + (size_t)t * ldx + bl * 256;
                        const float4 xa = __ldg(reinterpret_cast<const float4*>(xr + o0));
                        const float4 xb = __ldg(reinterpret_cast<const float4*>(xr + o0 + 4));
                        const float4 xc = __ldg(reinterpret_cast<const float4*>(xr + o1));
                        const float4 xd = __ldg(reinterpret_cast<const float4*>(xr + o1 + 4));
                        const float xv[16] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w,
                                              xc.x, xc.y, xc.z, xc.w, xd.x, xd.y, xd.z, xd.w};
#pragma unroll
                        for (int j = 0; j < 16; j++) acc[t] = __fmaf_rn(w[j], xv[j], acc[t]);
                    }
                }
            }
#pragma unroll
            for (int t = 0; t < MT; t++) {
                const float v = warp_sum(acc[t]);
                if (lane == 0 && t < m) y[(size_t)t * ldy + row0 + warp] = v;
            }
        }
        __syncthreads();  // the staged rows are reused by the next rows
    }
}

constexpr int kKqSmemMax = 96 * 1024;  // staged rows per CTA at most

template <int QT, int MT>
int kq_launch_t(const float* x, int ldx, int m, int n, int k, const uint8_t* wq, float* y, int ldy, cudaStream_t s) {
    constexpr int R = kKqWarps;
    const size_t rbytes = (size_t)(k >> 8) * kq_block_bytes<QT>();
    if (rbytes % 16 == 0 && ((uintptr_t)wq & 15) == 0 && (size_t)R * rbytes <= (size_t)kKqSmemMax) {
        // once per instantiation (thread-safe static initialisation)
        static const cudaError_t attr = cudaFuncSetAttribute(
            kq_gemv_smem_kernel<QT, MT>, cudaFuncAttributeMaxDynamicSharedMemorySize, kKqSmemMax);
        if (attr != cudaSuccess) return cuda_fail(attr, "cudaFuncSetAttribute");
        const int blocks = std::min((n + R - 1) / R, 148 * 8);
        kq_gemv_smem_kernel<QT, MT><<<blocks, kKqWarps * 32, R * rbytes, s>>>(x, ldx, m, n, k, wq, y, ldy);
        JYC_LAUNCHED();
        return JYC_OK;
    }
    const int blocks = std::min((n + kKqRowsPerCta - 1) / kKqRowsPerCta, 148 * 8);
    kq_gemv_kernel<QT, MT><<<blocks, kKqWarps * 32, 0, s>>>(x, ldx, m, n, k, wq, y, ldy);
    JYC_LAUNCHED();
    return JYC_OK;
}

template <int QT>
int kq_launch_qt(const float* x, int ldx, int m, int n, int k, const uint8_t* wq, float* y, int ldy, cudaStream_t s) {
    if (m == 1) return kq_launch_t<QT, 1>(x, ldx, m, n, k, wq, y, ldy, s);
    if (m <= 4) return kq_launch_t<QT, 4>(x, ldx, m, n, k, wq, y, ldy, s);
    return kq_launch_t<QT, 8>(x, ldx, m, n, k, wq, y, ldy, s);
}

// Dequantisation of whole rows into fp32 (the reference's dequant_block
// values), for models whose K-quant weights run on the fp32 matmul path:
// one warp per (row, super-block); row r lands at dst row row_off + r * row_stride.
template <int QT>
__global__ void __launch_bounds__(kKqWarps * 32) kq_dequant_rows_kernel(const uint8_t* __restrict__ blocks, int n,
                                                                        int k, float* __restrict__ dst, int row_off,
                                                                        int row_stride) {
    constexpr int BB = kq_block_bytes<QT>();
    const int lane = threadIdx.x & 31;
    const int nblk = k >> 8;
    const long long units = (long long)n * nblk;
    for (long long u = (long long)blockIdx.x * kKqWarps + (threadIdx.x >> 5); u < units;
         u += (long long)gridDim.x * kKqWarps) {
        const int r = (int)(u / nblk), bl = (int)(u % nblk);
        float w[8];
        int o0 = 0, o1 = 0;
        kq_dequant<QT>(blocks + (size_t)u * BB, lane, w, o0, o1);
        float* out = dst + ((size_t)row_off + (size_t)r * row_stride) * k + (size_t)bl * 256;
        if (QT == JYC_Q6K) {
#pragma unroll
            for (int j = 0; j < 8; j++) out[128 * (j >> 2) + o0 + 32 * (j & 3)] = w[j];
        } else {
#pragma unroll
            for (int i = 0; i < 4; i++) {
                out[o0 + i] = w[i];
                out[o1 + i] = w[4 + i];
            }
        }
    }
}

template <int QT>
int kq_dequant_launch(const uint8_t* blocks, int n, int k, float* dst, int row_off, int row_stride,
                      cudaStream_t s) {
    const long long units = (long long)n * (k >> 8);
    const int grid = (int)std::min<long long>((units + kKqWarps - 1) / kKqWarps, 148 * 16);
    kq_dequant_rows_kernel<QT><<<grid, kKqWarps * 32, 0, s>>>(blocks, n, k, dst, row_off, row_stride);
    JYC_LAUNCHED();
    return JYC_OK;
}

}  // namespace

int launch_kquant_matmul(const float* x, int m, int n, int k, const uint8_t* wq, int qtype, float* y,
                         cudaStream_t s) {
    if (qtype != JYC_Q4K && qtype != JYC_Q5K && qtype != JYC_Q6K)
        return arg_error("matmul_qk: qtype must be JYC_Q4K, JYC_Q5K or JYC_Q6K");
    if (m <= 0 || n <= 0 || k <= 0 || k % 256) return arg_error("matmul_qk: need m, n > 0 and k % 256 == 0");
    if (((uintptr_t)x & 15) || ((uintptr_t)wq & 3))
        return arg_error("matmul_qk: A must be 16-byte and the blocks 4-byte aligned");
    for (int r0 = 0; r0 < m; r0 += kKqMaxRows) {
        const int mr = std::min(kKqMaxRows, m - r0);
        const float* xr = x + (size_t)r0 * k;
        float* yr = y + (size_t)r0 * n;
        int r;
        if (qtype == JYC_Q4K) r = kq_launch_qt<JYC_Q4K>(xr, k, mr, n, k, wq, yr, n, s);
        else if (qtype == JYC_Q5K) r = kq_launch_qt<JYC_Q5K>(xr, k, mr, n, k, wq, yr, n, s);
        else r = kq_launch_qt<JYC_Q6K>(xr, k, mr, n, k, wq, yr, n, s);
        if (r != JYC_OK) return r;
    }
    return JYC_OK;
}

// The same with row strides (x rows ldx floats apart, y rows ldy apart): the
// K-quant model path writes Q, K and V side by side into one q|k|v row.
int launch_kquant_matmul_ld(const float* x, int ldx, int m, int n, int k, const uint8_t* wq, int qtype, float* y,
                            int ldy, cudaStream_t s) {
    if (qtype != JYC_Q4K && qtype != JYC_Q5K && qtype != JYC_Q6K)
        return arg_error("matmul_qk: qtype must be JYC_Q4K, JYC_Q5K or JYC_Q6K");
    if (m <= 0 || n <= 0 || k <= 0 || k % 256) return arg_error("matmul_qk: need m, n > 0 and k % 256 == 0");
    if (((uintptr_t)x & 15) || (ldx & 3) || ((uintptr_t)wq & 3) || ldx < k || ldy < n)
        return arg_error("matmul_qk: A rows must be 16-byte aligned and the blocks 4-byte aligned");
    for (int r0 = 0; r0 < m; r0 += kKqMaxRows) {
        const int mr = std::min(kKqMaxRows, m - r0);
        const float* xr = x + (size_t)r0 * ldx;
        float* yr = y + (size_t)r0 * ldy;
        int r;
        if (qtype == JYC_Q4K) r = kq_launch_qt<JYC_Q4K>(xr, ldx, mr, n, k, wq, yr, ldy, s);
        else if (qtype == JYC_Q5K) r = kq_launch_qt<JYC_Q5K>(xr, ldx, mr, n, k, wq, yr, ldy, s);
        else r = kq_launch_qt<JYC_Q6K>(xr, ldx, mr, n, k, wq, yr, ldy, s);
        if (r != JYC_OK) return r;
    }
    return JYC_OK;
}

int launch_kquant_dequant(const uint8_t* blocks, int n, int k, int qtype, float* dst, int row_off, int row_stride,
                          cudaStream_t s) {
    if (n <= 0 || k <= 0 || k % 256) return arg_error("K-quant weights need k % 256 == 0");
    if (((uintptr_t)blocks & 3)) return arg_error("K-quant blocks must be 4-byte aligned");
    if (qtype == JYC_Q4K) return kq_dequant_launch<JYC_Q4K>(blocks, n, k, dst, row_off, row_stride, s);
    if (qtype == JYC_Q5K) return kq_dequant_launch<JYC_Q5K>(blocks, n, k, dst, row_off, row_stride, s);
    if (qtype == JYC_Q6K) return kq_dequant_launch<JYC_Q6K>(blocks, n, k, dst, row_off, row_stride, s);
    return arg_error("unknown K-quant type");
}

size_t kquant_block_bytes(int qtype) {
    return qtype == JYC_Q4K ? 144 : qtype == JYC_Q5K ? 176 : qtype == JYC_Q6K ? 210 : 0;
}

}  // namespace jyc
