// mega.cu — the batch-1 decode step as ONE persistent cooperative kernel.
//
// One CTA per SM: 16 consumer warps + 1 producer warp. The producer streams
// every weight tile this CTA needs for the whole step (layer by layer: QKV,
// O, gate/up, down rows of its slice, then the LM-head slice) from HBM into a
// shared-memory ring with 1-D TMA bulk copies (cp.async.bulk, L2 evict-first,
// mbarrier completion). It never waits on activations, so it runs ahead across
// the grid barriers that separate the step's dependent phases; HBM keeps
// streaming while the consumers synchronise.
//
// Consumer phases per layer (reference: transformer_layer, transformer_layer.h:10-90):
//   QKV     x = RMSNorm(X) (layer 0: embedding row, wmat_row wmat_kernel.h:18-29)
//           -> Q|K|V rows (+ bias)                          [grid barrier]
//   ATTN    per (kv head, position split): RoPE + int8 quantisation of the
//           group's Q heads, K/V append at pos (owner split), int8 dot
//           scores, online softmax, PV -> split partials      [grid barrier]
//   O       x = merge of the split partials -> X += Wo x    [grid barrier]
//   GATE/UP x = RMSNorm(X) -> h = silu(gate) * up           [grid barrier]
//   DOWN    x = h -> X += W2 h                              [grid barrier]
// then the LM head on RMSNorm(X) with a per-CTA argmax -> one atomicMax,
// a last barrier, and CTA 0 appends the token and advances the step state
// (generate.h:57-86).
//
// Dequant-dot on the tensor cores (mma.sync m16n8k32 s8 -> s32): the input
// vector x is cut into 32-element blocks matching Q8_0's; per block
// N_i = rint(x_i * 2^20 / amax) is split into three signed 7-bit digits
// (N = 2^14 a + 2^7 b + c), the B operand's three columns. One mma gives, for
// 16 rows, the exact integer dots of the int8 weights with each digit; they
// recombine as 2^14 C_a + 2^7 C_b + C_c and scale by the block's fp16 d and
// amax/2^20. x keeps 21 bits per block (error <= 2^-21 of the block max), the
// weight products stay exact: the accuracy of fp32 FMA accumulation.
// Reference arithmetic being replaced: qmat::matmul_q / dot_row_avx2
// (libs/matmul_libs/matmul_q.h:101-143).
//
// Warp w of the consumers owns the 32-column Q8 block w of each 512-column
// tile for every 16-row group; partial row sums meet in shared memory in a
// fixed order (deterministic).
//
// Every wait is bounded (mbarrier waits and grid barriers give up after about
// a second of clock cycles and record an error word the host reads).
#include <algorithm>
#include <cmath>

#include "mega.cuh"
#include "ptx.cuh"

namespace jyc {

constexpr int kMegaThreads = (kMegaCW + 1) * 32;
constexpr int kASB = 128;  // attention positions per sub-block

// Error word of the device kernels (non-zero: a bounded wait gave up; the
// value tells which: 3 ring slot free, 4 ring slot full, 5 grid barrier).
__device__ int g_err_word;

int* device_error_word() {
    int* p = nullptr;
    if (cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_err_word) != cudaSuccess) return nullptr;
    return p;
}

static __device__ __forceinline__ void csync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kMegaCW * 32) : "memory");
}

// physical 16-byte chunk of logical chunk c in row r (nch chunks per row)
static __host__ __device__ __forceinline__ int swz_chunk(int c, int r, int nch) {
    return ((c | 7) < nch) ? ((c & ~7) | ((c ^ r) & 7)) : c;
}

// ---------------------------------------------------------------------------
// Tiled repack: reference blocks [n][k/32] x 34 B -> [cb][row][w_cb] layout.
__global__ void q8_repack_tiled_kernel(const uint8_t* blocks, size_t nblocks, int nb, int k, uint8_t* qs,
                                       uint16_t* d, int n_total, int row_off, int row_stride) {
    for (size_t b = blockIdx.x * (size_t)blockDim.x + threadIdx.x; b < nblocks;
         b += (size_t)gridDim.x * blockDim.x) {
        const size_t r = b / nb;
        const int bl = (int)(b % nb);
        const size_t R = (size_t)row_off + r * (size_t)row_stride;
        const int col0 = bl * 32, cb = col0 / kMegaCB, w = min(kMegaCB, k - cb * kMegaCB);
        const int c = (col0 - cb * kMegaCB) / 16;  // even: first of the block's two chunks
        const uint8_t* src = blocks + b * 34;
        d[(size_t)cb * n_total * (kMegaCB / 32) + R * (w / 32) + c / 2] = (uint16_t)src[0] | ((uint16_t)src[1] << 8);
        uint8_t* row = qs + (size_t)cb * n_total * kMegaCB + R * w;
        for (int h = 0; h < 2; h++) {
            uint32_t* q = reinterpret_cast<uint32_t*>(row + 16 * swz_chunk(c + h, (int)(R & 7), w / 16));
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const uint8_t* s4 = src + 2 + 16 * h + 4 * i;
                q[i] = (uint32_t)s4[0] | ((uint32_t)s4[1] << 8) | ((uint32_t)s4[2] << 16) | ((uint32_t)s4[3] << 24);
            }
        }
    }
}

int launch_q8_repack_tiled(const void* blocks, int n, int k, uint8_t* qs, uint16_t* d, int n_total,
                           int row_off, int row_stride, cudaStream_t s) {
    if (n <= 0 || k <= 0 || k % 32) return arg_error("q8_repack_tiled: k must be a positive multiple of 32");
    const size_t nb = (size_t)n * (k / 32);
    const int grid = (int)std::min<size_t>((nb + 255) / 256, 148 * 16);
    q8_repack_tiled_kernel<<<grid, 256, 0, s>>>(static_cast<const uint8_t*>(blocks), nb, k / 32, k, qs, d,
                                                n_total, row_off, row_stride);
    JYC_LAUNCHED();
    return JYC_OK;
}

// ---------------------------------------------------------------------------
// tile sequence of one matrix for CTA b (shared by producer and consumers)
static __device__ __forceinline__ int mat_tiles(const MegaMat& M, int b) {
    const int r0 = b * M.rpc, r1 = min(r0 + M.rpc, M.n);
    if (r1 <= r0) return 0;
    return ((r1 - r0 + M.rt - 1) / M.rt) * ((M.k + kMegaCB - 1) / kMegaCB);
}

static __device__ bool produce_mat(const MegaMat& M, int b, int& t, int ns, uint64_t* full, uint64_t* empty,
                                   unsigned char* ring, uint64_t pol, int* err) {
    const int r_begin = b * M.rpc, r_end = min(r_begin + M.rpc, M.n);
    const int ncb = (M.k + kMegaCB - 1) / kMegaCB;
    for (int r0 = r_begin; r0 < r_end; r0 += M.rt) {
        const int rows = min(M.rt, r_end - r0);
        for (int cb = 0; cb < ncb; cb++, t++) {
            const int s = t % ns, u = t / ns;
            if (u > 0 && !mbar_wait_err(&empty[s], (u - 1) & 1, err, 3)) return false;
            const int w = min(kMegaCB, M.k - cb * kMegaCB);
            unsigned char* slot = ring + (size_t)s * kMegaSlotBytes;
            const uint32_t qb = (uint32_t)(rows * w), db = (uint32_t)(rows * (w / 32) * 2);
            mbar_expect_tx(&full[s], qb + db);
            bulk_g2s(slot, M.qs + (size_t)cb * M.n * kMegaCB + (size_t)r0 * w, qb, &full[s], pol);
            bulk_g2s(slot + kMegaRT * kMegaCB, M.d + (size_t)cb * M.n * (kMegaCB / 32) + (size_t)r0 * (w / 32),
                     db, &full[s], pol);
        }
    }
    return true;
}

enum MegaEpi { ME_STORE = 0, ME_BIAS, ME_RESID, ME_SWIGLU, ME_ARGMAX };

static __device__ __forceinline__ void mma_s8(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                              uint32_t b1, int& c0, int& c1, int& c2, int& c3) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=r"(c0), "=r"(c1), "=r"(c2), "=r"(c3)
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

// y[rows of this CTA] = W . x for one matrix; x given as 3 int8 digit planes
// xd[0..2][k] and per-32 block scales xsc[k/32].
template <int EPI>
static __device__ bool consume_mat(const MegaMat& M, const int8_t* xd, const float* xsc, int& t, int ns,
                                   uint64_t* full, uint64_t* empty, const unsigned char* ring, float* s_part,
                                   float* s_res, float* y, const float* bias, unsigned long long* s_best,
                                   int* err) {
    const int b = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int g = lane >> 2, tq = lane & 3;
    const int r_begin = b * M.rpc, r_end = min(r_begin + M.rpc, M.n);
    const int ncb = (M.k + kMegaCB - 1) / kMegaCB;
    constexpr int NRG = kMegaRT / 16;
    for (int r0 = r_begin; r0 < r_end; r0 += M.rt) {
        const int rows = min(M.rt, r_end - r0), nrg = rows >> 4;
        float acc[NRG][2];
#pragma unroll
        for (int j = 0; j < NRG; j++) acc[j][0] = acc[j][1] = 0.0f;
        for (int cb = 0; cb < ncb; cb++, t++) {
            const int s = t % ns, u = t / ns;
            if (!mbar_wait_err(&full[s], u & 1, err, 4)) return false;
            const int w = min(kMegaCB, M.k - cb * kMegaCB), nblk = w >> 5, nch = w >> 4;
            if (warp < nblk) {
                const unsigned char* slot = ring + (size_t)s * kMegaSlotBytes;
                const uint16_t* sd = reinterpret_cast<const uint16_t*>(slot + kMegaRT * kMegaCB);
                const int col = cb * kMegaCB + 32 * warp + 8 * tq;
                uint2 bf = make_uint2(0u, 0u);
                if (g < 3) bf = *reinterpret_cast<const uint2*>(xd + (size_t)g * M.k + col);
                const float sx = xsc[cb * (kMegaCB / 32) + warp];
                const int c = 2 * warp + (tq >> 1), off = 8 * (tq & 1);
#pragma unroll
                for (int rg = 0; rg < NRG; rg++) {
                    if (rg < nrg) {
                        const int ra = rg * 16 + g, rb = ra + 8;
                        const uint2 A0 = *reinterpret_cast<const uint2*>(slot + ra * w + 16 * swz_chunk(c, ra, nch) + off);
                        const uint2 A1 = *reinterpret_cast<const uint2*>(slot + rb * w + 16 * swz_chunk(c, rb, nch) + off);
                        int c0, c1, c2, c3;
                        mma_s8(A0.x, A1.x, A0.y, A1.y, bf.x, bf.y, c0, c1, c2, c3);
                        // digit 2 (column 2) sits in the next lane of the quad
                        const int la = __shfl_down_sync(0xffffffffu, c0, 1);
                        const int lb = __shfl_down_sync(0xffffffffu, c2, 1);
                        if (tq == 0) {
                            const float da = h2f(sd[ra * nblk + warp]), db = h2f(sd[rb * nblk + warp]);
                            const float fa = __fmaf_rn(16384.0f, (float)c0, (float)(128 * c1 + la));
                            const float fb = __fmaf_rn(16384.0f, (float)c2, (float)(128 * c3 + lb));
                            acc[rg][0] = __fmaf_rn(fa, __fmul_rn(sx, da), acc[rg][0]);
                            acc[rg][1] = __fmaf_rn(fb, __fmul_rn(sx, db), acc[rg][1]);
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        if (tq == 0) {
#pragma unroll
            for (int rg = 0; rg < NRG; rg++)
                if (rg < nrg) {
                    s_part[warp * kMegaRT + rg * 16 + g] = acc[rg][0];
                    s_part[warp * kMegaRT + rg * 16 + g + 8] = acc[rg][1];
                }
        }
        csync();
        for (int e = tid; e < rows; e += kMegaCW * 32) {
            float v = 0.0f;
#pragma unroll
            for (int w2 = 0; w2 < kMegaCW; w2++) v = __fadd_rn(v, s_part[w2 * kMegaRT + e]);
            s_res[e] = v;
        }
        csync();
        if (EPI == ME_SWIGLU) {
            for (int e = tid; e < rows / 2; e += kMegaCW * 32)
                y[(r0 >> 1) + e] = __fmul_rn(silu_ref(s_res[2 * e]), s_res[2 * e + 1]);
        } else if (EPI == ME_ARGMAX) {
            unsigned long long best = 0ull;
            for (int e = tid; e < rows; e += kMegaCW * 32) {
                y[r0 + e] = s_res[e];
                const unsigned long long p = argmax_pack(s_res[e], r0 + e);
                best = p > best ? p : best;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const unsigned long long q = __shfl_xor_sync(0xffffffffu, best, o);
                best = q > best ? q : best;
            }
            if (lane == 0 && best) atomicMax(s_best, best);
        } else {
            for (int e = tid; e < rows; e += kMegaCW * 32) {
                float v = s_res[e];
                if (EPI == ME_BIAS) v = __fadd_rn(v, __ldg(bias + r0 + e));
                if (EPI == ME_RESID) v = __fadd_rn(__ldcg(y + r0 + e), v);
                y[r0 + e] = v;
            }
        }
        csync();
    }
    return true;
}

// x_s = RMSNorm(x_s) * w over k (sum of squares: per-thread FMA chains + warp/CTA tree)
static __device__ void x_norm(float* x_s, int k, const float* w, float eps, float* s_red) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    csync();
    float ss = 0.0f;
    for (int i = tid; i < k; i += kMegaCW * 32) ss = __fmaf_rn(x_s[i], x_s[i], ss);
    ss = warp_sum(ss);
    if (lane == 0) s_red[warp] = ss;
    csync();
    float tsum = 0.0f;
    for (int i = 0; i < kMegaCW; i++) tsum += s_red[i];
    const float den = __fadd_rn(__fdiv_rn(tsum, (float)k), eps);
    const float sc = den <= 0.0f ? 0.0f : __fdiv_rn(1.0f, __fsqrt_rn(den));
    for (int i = tid; i < k; i += kMegaCW * 32) x_s[i] = __fmul_rn(__fmul_rn(x_s[i], sc), __ldg(w + i));
    csync();
}

// x_s[0..k) = src (16-byte loads, all independent)
static __device__ void x_load(float* x_s, const float* src, int k) {
    const float4* s4 = reinterpret_cast<const float4*>(src);
    float4* d4 = reinterpret_cast<float4*>(x_s);
#pragma unroll 4
    for (int i = threadIdx.x; i < (k >> 2); i += kMegaCW * 32) d4[i] = __ldcg(s4 + i);
    csync();
}

// x_s (k floats) -> three int8 digit planes + per-32 block scales. A lane
// takes 4 consecutive elements, 8 lanes one 32-element block.
static __device__ void x_digitize(const float* x_s, int k, int8_t* xd, float* xsc) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int sub = lane & 7;  // lane within its block
    const int nblk = k >> 5;
    for (int base = warp * 4; base < nblk; base += kMegaCW * 4) {
        const int blk = base + (lane >> 3);
        const bool valid = blk < nblk;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (valid) v = reinterpret_cast<const float4*>(x_s + blk * 32)[sub];
        float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
        if (!valid) continue;
        const float inv = amax > 0.0f ? __fdiv_rn(1048576.0f, amax) : 0.0f;
        const float vv[4] = {v.x, v.y, v.z, v.w};
        uint32_t pa = 0, pb = 0, pc = 0;
#pragma unroll
        for (int e = 0; e < 4; e++) {
            int N = __float2int_rn(__fmul_rn(vv[e], inv));
            N = max(-1048576, min(1048576, N));
            const int c = ((N + 64) & 127) - 64;
            const int n1 = (N - c) >> 7;
            const int bd = ((n1 + 64) & 127) - 64;
            const int a = (n1 - bd) >> 7;
            pa |= (uint32_t)(a & 255) << (8 * e);
            pb |= (uint32_t)(bd & 255) << (8 * e);
            pc |= (uint32_t)(c & 255) << (8 * e);
        }
        reinterpret_cast<uint32_t*>(xd)[blk * 8 + sub] = pa;
        reinterpret_cast<uint32_t*>(xd + k)[blk * 8 + sub] = pb;
        reinterpret_cast<uint32_t*>(xd + 2 * k)[blk * 8 + sub] = pc;
        if (sub == 0) xsc[blk] = __fmul_rn(amax, 1.0f / 1048576.0f);  // exact: power of two
    }
    csync();
}

// Grid barrier over the consumer threads of every CTA (bounded spin).
static __device__ bool grid_barrier(unsigned int* ctr, unsigned int target, int* err, int* s_ok) {
    csync();
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(ctr, 1u);
        int ok = 1;
        if ((int)(ld_acquire_gpu(ctr) - target) < 0) {
            const long long t0 = clock64();
            while ((int)(ld_acquire_gpu(ctr) - target) < 0) {
                if (clock64() - t0 > (1LL << 31)) {
                    atomicExch(err, 5);
                    ok = 0;
                    break;
                }
            }
        }
        *s_ok = ok;
    }
    csync();
    return *s_ok != 0;
}

// RoPE (reference slot order) + kv_pack_q8 quantisation of one head by one warp.
static __device__ __forceinline__ void rq_warp(const float* src, int hd, const float* ct, const float* stb,
                                               int8_t* dst, float* scale_out, int lane) {
    constexpr int MAXP = 4;
    const int half = hd >> 1;
    float x0[MAXP], x1[MAXP];
    float amax = 0.0f;
#pragma unroll
    for (int tt = 0; tt < MAXP; tt++) {
        const int p = lane + 32 * tt;
        x0[tt] = 0.0f;
        x1[tt] = 0.0f;
        if (p < half) {
            float v0 = __ldcg(src + 2 * p), v1 = __ldcg(src + 2 * p + 1);
            if (ct) {
                const float c = ct[p], sn = stb[p];
                const float r0 = __fmaf_rn(v0, c, -__fmul_rn(v1, sn));
                const float r1 = __fmaf_rn(v0, sn, __fmul_rn(v1, c));
                v0 = r0;
                v1 = r1;
            }
            x0[tt] = v0;
            x1[tt] = v1;
            amax = fmaxf(amax, fmaxf(fabsf(v0), fabsf(v1)));
        }
    }
    amax = warp_max(amax);
    const float inv = q8_inv(amax);
    if (lane == 0) *scale_out = q8_scale(amax);
#pragma unroll
    for (int tt = 0; tt < MAXP; tt++) {
        const int p = lane + 32 * tt;
        if (p < half) {
            const int o = ct ? rope_slot(p, half) : p;
            dst[2 * o] = (int8_t)q8_round(x0[tt], inv);
            dst[2 * o + 1] = (int8_t)q8_round(x1[tt], inv);
        }
    }
}

static int attn_item_smem(int G, int hd) {
    // q8 [G][hd] | qsc, m, l, alpha [G] | o [G][hd] | w [G][ASB] | K tile [ASB][hd+4] (int8, padded) |
    // V tile [ASB][hd] (fp32) | ks, vs [ASB]
    return G * hd + 4 * G * 4 + G * hd * 4 + G * kASB * 4 + kASB * (hd + 4) + kASB * hd * 4 + 2 * kASB * 4;
}

// 16 signed bytes -> 16 exact floats (2^23 mantissa trick on b ^ 0x80 = b + 128)
static __device__ __forceinline__ void s8x16_to_f32(uint4 w, float* f) {
    u8x4_to_f32(w.x ^ 0x80808080u, f);
    u8x4_to_f32(w.y ^ 0x80808080u, f + 4);
    u8x4_to_f32(w.z ^ 0x80808080u, f + 8);
    u8x4_to_f32(w.w ^ 0x80808080u, f + 12);
}

// One (layer, kv head, position split) attention item with the consumer threads.
static __device__ void attn_item(const MegaArgs& a, int layer, int kvh, int split, int pos, unsigned char* sm) {
    const int G = a.H / a.KV, hd = a.hd, half = hd >> 1;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int nthr = kMegaCW * 32;
    const int c0 = split * a.chunk, c1 = min(c0 + a.chunk, pos + 1);
    int8_t* s_q8 = reinterpret_cast<int8_t*>(sm);
    float* s_qsc = reinterpret_cast<float*>(sm + G * hd);
    float* s_m = s_qsc + G;
    float* s_l = s_m + G;
    float* s_alpha = s_l + G;
    float* s_o = s_alpha + G;
    float* s_w = s_o + G * hd;
    int8_t* s_k = reinterpret_cast<int8_t*>(s_w + G * kASB);
    float* s_v = reinterpret_cast<float*>(s_k + kASB * (hd + 4));
    float* s_ks = s_v + kASB * hd;
    float* s_vs = s_ks + kASB;

    const size_t lh = (size_t)layer * a.KV + kvh;
    int8_t* kb = a.k8 + lh * a.max_seq * hd;
    int8_t* vb = a.v8 + lh * a.max_seq * hd;
    float* ksb = a.ks + lh * a.max_seq;
    float* vsb = a.vs + lh * a.max_seq;
    const float* ct = a.cos_t + (size_t)pos * half;
    const float* stb = a.sin_t + (size_t)pos * half;
    const int q_dim = a.H * hd, kv_dim = a.KV * hd;

    for (int gq = warp; gq < G; gq += kMegaCW)
        rq_warp(a.qkv + (size_t)(kvh * G + gq) * hd, hd, ct, stb, s_q8 + gq * hd, s_qsc + gq, lane);
    if (pos < c1) {  // owner of the new position: append K (roped) and V
        if (warp == kMegaCW - 1)
            rq_warp(a.qkv + q_dim + (size_t)kvh * hd, hd, ct, stb, kb + (size_t)pos * hd, ksb + pos, lane);
        else if (warp == kMegaCW - 2)
            rq_warp(a.qkv + q_dim + kv_dim + (size_t)kvh * hd, hd, nullptr, nullptr, vb + (size_t)pos * hd,
                    vsb + pos, lane);
        __threadfence();  // the appended row is read back below through L2
    }
    for (int e = tid; e < G * hd; e += nthr) s_o[e] = 0.0f;
    for (int gq = tid; gq < G; gq += nthr) {
        s_m[gq] = -INFINITY;
        s_l[gq] = 0.0f;
    }
    csync();
    const int hw = hd >> 2, hv = hd >> 4;
    for (int j0 = c0; j0 < c1; j0 += kASB) {
        const int nj = min(kASB, c1 - j0);
        for (int e = tid; e < nj * hv; e += nthr) {
            const int j = e / hv, vq = e - j * hv;
            const size_t off = (size_t)(j0 + j) * hd + 16 * vq;
            const uint4 kq = __ldcg(reinterpret_cast<const uint4*>(kb + off));
            const uint4 vq4 = __ldcg(reinterpret_cast<const uint4*>(vb + off));
            uint32_t* kd = reinterpret_cast<uint32_t*>(s_k + j * (hd + 4) + 16 * vq);
            kd[0] = kq.x; kd[1] = kq.y; kd[2] = kq.z; kd[3] = kq.w;
            float f[16];
            s8x16_to_f32(vq4, f);
            float4* vd = reinterpret_cast<float4*>(s_v + j * hd + 16 * vq);
            vd[0] = make_float4(f[0], f[1], f[2], f[3]);
            vd[1] = make_float4(f[4], f[5], f[6], f[7]);
            vd[2] = make_float4(f[8], f[9], f[10], f[11]);
            vd[3] = make_float4(f[12], f[13], f[14], f[15]);
        }
        for (int j = tid; j < nj; j += nthr) {
            s_ks[j] = __ldcg(ksb + j0 + j);
            s_vs[j] = __ldcg(vsb + j0 + j);
        }
        csync();
        for (int e = tid; e < G * kASB; e += nthr) {
            const int gq = e / kASB, j = e - gq * kASB;
            float sc = -INFINITY;
            if (j < nj) {
                const int* qw = reinterpret_cast<const int*>(s_q8 + gq * hd);
                const int* kw = reinterpret_cast<const int*>(s_k + j * (hd + 4));
                int dot = 0;
                for (int wd = 0; wd < hw; wd++) dot = __dp4a(qw[wd], kw[wd], dot);
                const float ksc = __fmul_rn(__fmul_rn(s_ks[j], s_qsc[gq]), a.scale);
                sc = __fmul_rn((float)dot, ksc);
            }
            s_w[e] = sc;
        }
        csync();
        for (int gq = warp; gq < G; gq += kMegaCW) {
            float mx = -INFINITY;
            for (int j = lane; j < kASB; j += 32) mx = fmaxf(mx, s_w[gq * kASB + j]);
            mx = warp_max(mx);
            const float m_old = s_m[gq], m_new = fmaxf(m_old, mx);
            float sum = 0.0f;
            for (int j = lane; j < kASB; j += 32) {
                const float sv = s_w[gq * kASB + j];
                const float e = (sv == -INFINITY) ? 0.0f : expf(sv - m_new);
                sum += e;
                s_w[gq * kASB + j] = e * s_vs[j < nj ? j : 0];
            }
            sum = warp_sum(sum);
            if (lane == 0) {
                const float alpha = (m_old == -INFINITY) ? 0.0f : expf(m_old - m_new);
                s_alpha[gq] = alpha;
                s_l[gq] = s_l[gq] * alpha + sum;
                s_m[gq] = m_new;
            }
        }
        csync();
        for (int e = tid; e < G * hd; e += nthr) {
            const int gq = e / hd, dd = e - gq * hd;
            float o = s_o[e] * s_alpha[gq];
            const float* wp = s_w + gq * kASB;
            const float* vp = s_v + dd;
#pragma unroll 4
            for (int j = 0; j < nj; j++) o = __fmaf_rn(wp[j], vp[j * hd], o);
            s_o[e] = o;
        }
        csync();
    }
    for (int e = tid; e < G * hd; e += nthr) {
        const int gq = e / hd, dd = e - gq * hd, h = kvh * G + gq;
        a.part_o[((size_t)h * a.nsplit + split) * hd + dd] = s_o[e];
    }
    for (int gq = tid; gq < G; gq += nthr) {
        const int h = kvh * G + gq;
        a.part_ml[((size_t)h * a.nsplit + split) * 2] = s_m[gq];
        a.part_ml[((size_t)h * a.nsplit + split) * 2 + 1] = s_l[gq];
    }
    csync();
}

// x_s = merge of the attention split partials (the attention output row):
// per (head, split) the merge weight exp(m_s - M) / L once, then every output
// element sums its splits with independent loads. `scr` holds H*nsplit floats.
static __device__ void x_combine(const MegaArgs& a, float* x_s, float* scr, int pos) {
    const int H = a.H, hd = a.hd, ns = a.nsplit;
    const int nvalid = min(pos / a.chunk + 1, ns);
    const int tid = threadIdx.x;
    for (int e = tid; e < H * nvalid; e += kMegaCW * 32) {
        const int h = e / nvalid, s2 = e - h * nvalid;
        scr[e] = __ldcg(a.part_ml + ((size_t)h * ns + s2) * 2);  // m
    }
    csync();
    for (int h = tid; h < H; h += kMegaCW * 32) {
        float M = -INFINITY;
        for (int s2 = 0; s2 < nvalid; s2++) M = fmaxf(M, scr[h * nvalid + s2]);
        float L = 0.0f;
        for (int s2 = 0; s2 < nvalid; s2++) {
            const float ms = scr[h * nvalid + s2];
            const float wgt = (ms == -INFINITY) ? 0.0f : expf(ms - M);
            L = __fmaf_rn(wgt, __ldcg(a.part_ml + ((size_t)h * ns + s2) * 2 + 1), L);
            scr[h * nvalid + s2] = wgt;
        }
        const float inv = 1.0f / L;
        for (int s2 = 0; s2 < nvalid; s2++) scr[h * nvalid + s2] *= inv;
    }
    csync();
    for (int e = tid; e < H * hd; e += kMegaCW * 32) {
        const int h = e / hd, dd = e - h * hd;
        const float* po = a.part_o + (size_t)h * ns * hd + dd;
        const float* wt = scr + h * nvalid;
        float O = 0.0f;
#pragma unroll 8
        for (int s2 = 0; s2 < nvalid; s2++) O = __fmaf_rn(wt[s2], __ldcg(po + (size_t)s2 * hd), O);
        x_s[e] = O;
    }
    csync();
}

__global__ void __launch_bounds__(kMegaThreads, 1) mega_step_kernel(MegaArgs a) {
    extern __shared__ __align__(128) unsigned char sm[];
    uint64_t* full = reinterpret_cast<uint64_t*>(sm);
    uint64_t* empty = full + kMegaMaxSlots;
    unsigned char* xs_region = sm + 128;
    float* x_s = reinterpret_cast<float*>(xs_region);
    int8_t* xd = reinterpret_cast<int8_t*>(xs_region + (size_t)a.kmax * 4);
    float* xsc = reinterpret_cast<float*>(xs_region + (size_t)a.kmax * 7);
    unsigned char* ring = sm + 128 + a.xs_bytes;
    __shared__ float s_part[kMegaCW * kMegaRT];
    __shared__ float s_res[kMegaRT];
    __shared__ float s_red[kMegaCW];
    __shared__ unsigned long long s_best;
    __shared__ int s_ok;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, b = blockIdx.x;
    const int ns = a.nslots;

    if (tid == 0) {
        for (int s = 0; s < ns; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kMegaCW);
        }
        mbar_fence_init();
    }
    __syncthreads();

    if (warp == kMegaCW) {  // ---- producer: the step's weight tiles, in consumer order
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            int t = 0;
            bool ok = true;
            for (int l = 0; l < a.L && ok; l++) {
                const MegaLayer& ly = a.layers[l];
                ok = produce_mat(ly.qkv, b, t, ns, full, empty, ring, pol, a.err) &&
                     produce_mat(ly.o, b, t, ns, full, empty, ring, pol, a.err) &&
                     produce_mat(ly.gu, b, t, ns, full, empty, ring, pol, a.err) &&
                     produce_mat(ly.dn, b, t, ns, full, empty, ring, pol, a.err);
            }
            if (ok) produce_mat(a.head, b, t, ns, full, empty, ring, pol, a.err);
        }
        return;
    }

    // ---- consumers ---------------------------------------------------------
    DevState* st = a.st;
    const int active = *(volatile const int*)&st->active;
    int t = 0;
    if (!active) {  // disabled step: take every tile off the ring, then leave
        int n = 0;
        for (int l = 0; l < a.L; l++) {
            const MegaLayer& ly = a.layers[l];
            n += mat_tiles(ly.qkv, b) + mat_tiles(ly.o, b) + mat_tiles(ly.gu, b) + mat_tiles(ly.dn, b);
        }
        n += mat_tiles(a.head, b);
        for (; t < n; t++) {
            const int s = t % ns;
            if (!mbar_wait_err(&full[s], (t / ns) & 1, a.err, 4)) return;
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        return;
    }
    const int pos = (*(volatile const int*)&st->len) - 1;
    const unsigned int base = *(volatile const unsigned int*)&st->bar_base;
    const unsigned int nct = gridDim.x;
    int bi = 0;
    bool ok = true;
    const int nvalid = min(pos / a.chunk + 1, a.nsplit);
#define TRACE(idx)                                                               \
    do {                                                                         \
        if (a.trace != nullptr && tid == 0) a.trace[(size_t)b * kMegaTracePts + (idx)] = clock64(); \
    } while (0)
    TRACE(0);

    for (int l = 0; l < a.L && ok; l++) {
        const MegaLayer& ly = a.layers[l];
        // QKV
        if (l == 0) {
            const int id = __ldcg(a.tokens + pos);
            for (int i = tid; i < a.D; i += kMegaCW * 32) {
                float v;
                if (a.ef) {
                    v = __ldg(a.ef + (size_t)id * a.D + i);
                } else {
                    const int cb = i / kMegaCB, w = min(kMegaCB, a.D - cb * kMegaCB), c = i - cb * kMegaCB;
                    const uint8_t* row = a.eqs + (size_t)cb * a.V * kMegaCB + (size_t)id * w;
                    const int8_t q = (int8_t)row[16 * swz_chunk(c >> 4, id & 7, w >> 4) + (c & 15)];
                    v = __fmul_rn((float)q, h2f(a.ed[(size_t)cb * a.V * (kMegaCB / 32) + (size_t)id * (w / 32) + c / 32]));
                }
                x_s[i] = v;
                if (b == 0) a.X[i] = v;
            }
        } else {
            x_load(x_s, a.X, a.D);
        }
        x_norm(x_s, a.D, ly.rms1, 1e-5f, s_red);
        x_digitize(x_s, a.D, xd, xsc);
        const int tb = 1 + l * kMegaTraceLayer;
        TRACE(tb + 0);
        ok = ly.bias ? consume_mat<ME_BIAS>(ly.qkv, xd, xsc, t, ns, full, empty, ring, s_part, s_res, a.qkv, ly.bias,
                                           &s_best, a.err)
                     : consume_mat<ME_STORE>(ly.qkv, xd, xsc, t, ns, full, empty, ring, s_part, s_res, a.qkv,
                                            nullptr, &s_best, a.err);
        TRACE(tb + 1);
        ok = ok && grid_barrier(a.bar, base + (++bi) * nct, a.err, &s_ok);
        TRACE(tb + 2);
        if (!ok) break;
        // attention items (kv head, split), round-robin over CTAs
        for (int it = b; it < a.KV * nvalid; it += nct) attn_item(a, l, it / nvalid, it % nvalid, pos, xs_region);
        TRACE(tb + 3);
        ok = grid_barrier(a.bar, base + (++bi) * nct, a.err, &s_ok);
        TRACE(tb + 4);
        if (!ok) break;
        // O projection + residual
        x_combine(a, x_s, reinterpret_cast<float*>(xd), pos);
        x_digitize(x_s, a.H * a.hd, xd, xsc);
        TRACE(tb + 5);
        ok = consume_mat<ME_RESID>(ly.o, xd, xsc, t, ns, full, empty, ring, s_part, s_res, a.X, nullptr, &s_best, a.err);
        TRACE(tb + 6);
        ok = ok && grid_barrier(a.bar, base + (++bi) * nct, a.err, &s_ok);
        TRACE(tb + 7);
        if (!ok) break;
        // gate/up + SwiGLU
        x_load(x_s, a.X, a.D);
        x_norm(x_s, a.D, ly.rms2, 1e-5f, s_red);
        x_digitize(x_s, a.D, xd, xsc);
        TRACE(tb + 8);
        ok = consume_mat<ME_SWIGLU>(ly.gu, xd, xsc, t, ns, full, empty, ring, s_part, s_res, a.h, nullptr, &s_best,
                                    a.err);
        TRACE(tb + 9);
        ok = ok && grid_barrier(a.bar, base + (++bi) * nct, a.err, &s_ok);
        TRACE(tb + 10);
        if (!ok) break;
        // down projection + residual
        x_load(x_s, a.h, a.F);
        x_digitize(x_s, a.F, xd, xsc);
        TRACE(tb + 11);
        ok = consume_mat<ME_RESID>(ly.dn, xd, xsc, t, ns, full, empty, ring, s_part, s_res, a.X, nullptr, &s_best,
                                   a.err);
        TRACE(tb + 12);
        ok = ok && grid_barrier(a.bar, base + (++bi) * nct, a.err, &s_ok);
        TRACE(tb + 13);
    }
    if (!ok) return;
    // LM head + argmax
    const int th = 1 + a.L * kMegaTraceLayer;
    x_load(x_s, a.X, a.D);
    if (tid == 0) s_best = 0ull;
    x_norm(x_s, a.D, a.final_norm, 1e-5f, s_red);
    x_digitize(x_s, a.D, xd, xsc);
    TRACE(th + 0);
    if (!consume_mat<ME_ARGMAX>(a.head, xd, xsc, t, ns, full, empty, ring, s_part, s_res, a.logits, nullptr, &s_best,
                                a.err))
        return;
    TRACE(th + 1);
    if (tid == 0 && s_best) atomicMax(&st->amax, s_best);
    if (!grid_barrier(a.bar, base + (++bi) * nct, a.err, &s_ok)) return;
    TRACE(th + 2);
    if (b == 0 && tid == 0) {
        const unsigned long long packed = atomicAdd(&st->amax, 0ull);
        const int next = argmax_index(packed);
        const int len = st->len;
        a.tokens[len] = next;
        const int nlen = len + 1, nsteps = st->steps + 1;
        bool stop = nlen >= st->max_len || nsteps >= st->max_new;
        for (int e = 0; e < st->n_eos; e++)
            if (next == st->eos[e]) stop = true;
        st->len = nlen;
        st->steps = nsteps;
        st->amax = 0ull;
        st->bar_base = base + (unsigned int)bi * nct;
        if (stop) st->active = 0;
        __threadfence();
    }
}

// ---------------------------------------------------------------------------
int mega_num_ctas() {
    static int n = 0;
    if (n == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    }
    return n;
}

int mega_plan(MegaMat& m, int nctas) {
    if (m.n <= 0 || m.n % 16 || m.k % 32 || m.k <= 0) return JYC_ERR_UNSUPPORTED;
    int rpc = (m.n + nctas - 1) / nctas;
    rpc = (rpc + 15) / 16 * 16;
    m.rpc = rpc;
    m.rt = std::min(kMegaRT, rpc);
    return JYC_OK;
}

// x (4 B) + three digit planes (3 B) + block scales (1/8 B) per element; the
// attention item's scratch and the split merge's weights (after x) share it.
int mega_xs_bytes(int kmax, int G, int hd, int merge_weights) {
    const int xk = std::max(kmax * 4 + kmax * 3 + (kmax / 32) * 4, kmax * 4 + merge_weights * 4);
    return (std::max(xk, attn_item_smem(G, hd)) + 127) / 128 * 128;
}

int mega_smem_bytes(const MegaArgs& a) { return 128 + a.xs_bytes + a.nslots * kMegaSlotBytes; }

int mega_static_smem() {
    cudaFuncAttributes fa{};
    if (cudaFuncGetAttributes(&fa, mega_step_kernel) != cudaSuccess) return -1;
    return (int)fa.sharedSizeBytes;
}

int prepare_mega_kernel(int smem) {
    JYC_CUDA(cudaFuncSetAttribute(mega_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    return JYC_OK;
}

int launch_mega_step(const MegaArgs& a, cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(mega_num_ctas());
    cfg.blockDim = dim3(kMegaThreads);
    cfg.dynamicSmemBytes = (size_t)mega_smem_bytes(a);
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeCooperative;  // all CTAs co-resident: the grid barriers need it
    at[0].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, mega_step_kernel, a);
    if (e != cudaSuccess) return cuda_fail(e, "mega_step launch");
    count_launch();
    return JYC_OK;
}

}  // namespace jyc
