// prefill.cu — batched-token Q8_0 matmuls for prompt prefill.
//
// Y[t][r] = sum_k W[r][k] x[t][k] for T tokens at once (reference: the seq > 1
// calls of qmat::matmul_q, libs/matmul_libs/matmul_q.h:101-143, made by
// forward_cached for the prompt). Same exact-integer scheme as the decode
// kernel: every 32-element block of a token row is cut into three signed
// 7-bit digit planes (N = rint(x 2^20 / amax) = 2^14 a + 2^7 b + c); the
// tensor cores (mma.sync m16n8k32 s8 -> s32) give, for 16 weight rows and 8
// tokens, the exact integer dot of each digit plane with the int8 weights;
// they recombine in fp32 and scale by the weight row's fp16 d and the token
// block's amax / 2^20.
//
// Layouts:
//  weights: the tiled copy of the decode kernel ([cb][n][w_cb], chunks
//           swizzled by row & 7; paired scales), read straight from global
//           memory (L2-resident across the token tiles of one row tile);
//  digits:  [token tile][cb][k-block 16][plane 3][64 tokens][32 bytes], so one
//           column block of a token tile (96 KB) is one TMA bulk copy and the
//           B fragments (lane g: token g of an octet, 8 bytes at 8 tq) are one
//           conflict-free 64-bit shared load;
//  scales:  [token tile][cb][k-block 16][64 tokens] fp32 (amax / 2^20).
// CTA tile 64 rows x 64 tokens, 8 warps (4 row groups x 2 token halves),
// column blocks double-buffered in shared memory.
#include <algorithm>

#include "mega.cuh"
#include "prefill.cuh"
#include "ptx.cuh"

namespace jyc {

namespace {

constexpr int kTok = kPfTok;                       // tokens per tile
constexpr int kPlane = kTok * 32;                  // one digit plane of one k-block (2 KB)
constexpr int kStageDig = 16 * 3 * kPlane;         // one column block of digits (96 KB)
constexpr int kStageSx = 16 * kTok * 4;            // its block scales (4 KB)
constexpr int kStage = kStageDig + kStageSx;
constexpr int kSmem = 128 + 2 * kStage;
constexpr int kThreads = 256;
constexpr int kOct = 4;  // token octets per warp (8 warps: 4 row groups x 2 token halves)

__device__ __forceinline__ float small_i2f(int c) {
    return __fadd_rn(__int_as_float(c + 0x4B400000), -12582912.0f);
}
__device__ __forceinline__ float d_lo(uint32_t w) { return __int_as_float((w << 13) & 0x0FFFE000u); }
__device__ __forceinline__ float d_hi(uint32_t w) { return __int_as_float((w >> 3) & 0x0FFFE000u); }
__device__ __forceinline__ void mma_s8(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1, int& c0, int& c1, int& c2, int& c3) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=r"(c0), "=r"(c1), "=r"(c2), "=r"(c3)
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}
__device__ __forceinline__ int swz(int c, int r, int nch) { return ((c | 7) < nch) ? ((c & ~7) | ((c ^ r) & 7)) : c; }

// One token row -> optional RMSNorm (weights w) -> digit planes + scales in
// the tile layout. Token rows t >= T (tile padding) are written as zeros.
__global__ void __launch_bounds__(256) pf_digitize_kernel(const float* x, int ldx, int T, int k, const float* w,
                                                          float eps, int8_t* dig, float* sx) {
    __shared__ float s_red[8];
    const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int ncb = (k + kMegaCB - 1) / kMegaCB, tt = t / kTok, ti = t % kTok;
    const float* xr = x + (size_t)t * ldx;
    const bool real = t < T;
    float sc = 1.0f;
    if (real && w) {
        float ss = 0.0f;
        for (int i = tid; i < k; i += 256) ss = __fmaf_rn(xr[i], xr[i], ss);
        ss = warp_sum(ss);
        if (lane == 0) s_red[warp] = ss;
        __syncthreads();
        float tsum = 0.0f;
        for (int i = 0; i < 8; i++) tsum += s_red[i];
        const float den = __fadd_rn(__fdiv_rn(tsum, (float)k), eps);
        sc = den <= 0.0f ? 0.0f : __fdiv_rn(1.0f, __fsqrt_rn(den));
    }
    // 8 lanes per 32-element block, 4 elements per lane
    const int sub = lane & 7, nblk = k >> 5;
    for (int base = warp * 4; base < nblk; base += 8 * 4) {
        const int blk = base + (lane >> 3);
        const bool valid = blk < nblk;
        float v[4] = {0.f, 0.f, 0.f, 0.f};
        if (valid && real) {
            const float4 q = *reinterpret_cast<const float4*>(xr + blk * 32 + 4 * sub);
            v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
            if (w) {
                const float4 wq = *reinterpret_cast<const float4*>(w + blk * 32 + 4 * sub);
                v[0] = __fmul_rn(__fmul_rn(v[0], sc), wq.x);
                v[1] = __fmul_rn(__fmul_rn(v[1], sc), wq.y);
                v[2] = __fmul_rn(__fmul_rn(v[2], sc), wq.z);
                v[3] = __fmul_rn(__fmul_rn(v[3], sc), wq.w);
            }
        }
        float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
        if (!valid) continue;
        const float inv = amax > 0.0f ? __fdiv_rn(1048576.0f, amax) : 0.0f;
        uint32_t pa = 0, pb = 0, pc = 0;
#pragma unroll
        for (int e = 0; e < 4; e++) {
            int N = __float2int_rn(__fmul_rn(v[e], inv));
            N = max(-1048576, min(1048576, N));
            const int c = ((N + 64) & 127) - 64;
            const int n1 = (N - c) >> 7;
            const int bd = ((n1 + 64) & 127) - 64;
            const int a = (n1 - bd) >> 7;
            pa |= (uint32_t)(a & 255) << (8 * e);
            pb |= (uint32_t)(bd & 255) << (8 * e);
            pc |= (uint32_t)(c & 255) << (8 * e);
        }
        const int cb = blk >> 4, kb = blk & 15;
        int8_t* dst = dig + ((size_t)(tt * ncb + cb) * 16 + kb) * (3 * kPlane) + ti * 32 + 4 * sub;
        *reinterpret_cast<uint32_t*>(dst) = pa;
        *reinterpret_cast<uint32_t*>(dst + kPlane) = pb;
        *reinterpret_cast<uint32_t*>(dst + 2 * kPlane) = pc;
        if (sub == 0) sx[((size_t)(tt * ncb + cb) * 16 + kb) * kTok + ti] = __fmul_rn(amax, 1.0f / 1048576.0f);
    }
}

template <int EPI>
__global__ void __launch_bounds__(kThreads, 1) pf_gemm_kernel(PfGemm p) {
    extern __shared__ __align__(128) unsigned char sm[];
    uint64_t* full = reinterpret_cast<uint64_t*>(sm);
    unsigned char* stage0 = sm + 128;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, tq = lane & 3;
    const int r0 = blockIdx.x * kPfRows, tt = blockIdx.y;
    const int ncb = (p.k + kMegaCB - 1) / kMegaCB;
    auto issue = [&](int cb) {
        unsigned char* st = stage0 + (cb & 1) * kStage;
        fence_proxy_async_smem();
        mbar_expect_tx(&full[cb & 1], kStage);
        const uint64_t pol = policy_evict_first();
        bulk_g2s(st, p.dig + (size_t)(tt * ncb + cb) * kStageDig, kStageDig, &full[cb & 1], pol);
        bulk_g2s(st + kStageDig, p.sx + (size_t)(tt * ncb + cb) * 16 * kTok, kStageSx, &full[cb & 1], pol);
    };
    if (tid == 0) {
        mbar_init(&full[0], 1);
        mbar_init(&full[1], 1);
        mbar_fence_init();
        issue(0);
        if (ncb > 1) issue(1);
    }
    __syncthreads();

    const int R0 = r0 + 16 * (warp & 3);  // this warp's 16 rows
    const int oc0 = kOct * (warp >> 2);   // its first token octet
    float acc[kOct][4];
#pragma unroll
    for (int o = 0; o < kOct; o++)
#pragma unroll
        for (int i = 0; i < 4; i++) acc[o][i] = 0.0f;

    for (int cb = 0; cb < ncb; cb++) {
        const int w = min(kMegaCB, p.k - cb * kMegaCB), nkb = w >> 5, nch = w >> 4;
        const unsigned char* qrow = p.qs + (size_t)cb * p.n * kMegaCB + (size_t)(R0 + g) * w + 8 * (tq & 1);
        const uint32_t* dpair = reinterpret_cast<const uint32_t*>(p.d + (size_t)cb * p.n * (kMegaCB / 32)) +
                                (size_t)(R0 >> 4) * nkb * 8 + g;
        auto lda = [&](int kb, uint2& a0, uint2& a1, uint32_t& dw) {
            const int off = 16 * swz(2 * kb + (tq >> 1), g, nch);
            a0 = __ldg(reinterpret_cast<const uint2*>(qrow + off));
            a1 = __ldg(reinterpret_cast<const uint2*>(qrow + 8 * w + off));
            dw = __ldg(dpair + kb * 8);
        };
        uint2 A0, A1, nA0, nA1;
        uint32_t dw, ndw;
        lda(0, A0, A1, dw);
        // every thread waits (bounded); all leave together if any gave up
        if (__syncthreads_or(!mbar_wait_err(&full[cb & 1], (cb >> 1) & 1, p.err, 7))) return;
        const unsigned char* st = stage0 + (cb & 1) * kStage;
        const float* ssx = reinterpret_cast<const float*>(st + kStageDig);
        for (int kb = 0; kb < nkb; kb++) {
            if (kb + 1 < nkb) lda(kb + 1, nA0, nA1, ndw);
            const float dl = d_lo(dw), dh = d_hi(dw);  // row scales * 2^-112
#pragma unroll
            for (int o = 0; o < kOct; o++) {
                const int oc = oc0 + o;
                int C[3][4];
#pragma unroll
                for (int dd = 0; dd < 3; dd++) {
                    const uint2 bf = *reinterpret_cast<const uint2*>(st + (kb * 3 + dd) * kPlane + (oc * 8 + g) * 32 + 8 * tq);
                    mma_s8(A0.x, A1.x, A0.y, A1.y, bf.x, bf.y, C[dd][0], C[dd][1], C[dd][2], C[dd][3]);
                }
                const float2 sp = *reinterpret_cast<const float2*>(ssx + kb * kTok + oc * 8 + 2 * tq);
                const float s0 = __fmul_rn(sp.x, 0x1p84f), s1 = __fmul_rn(sp.y, 0x1p84f);
                const float sc[4] = {__fmul_rn(dl, s0), __fmul_rn(dl, s1), __fmul_rn(dh, s0), __fmul_rn(dh, s1)};
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const float v = __fmaf_rn(128.0f, __fmaf_rn(128.0f, small_i2f(C[0][i]), small_i2f(C[1][i])),
                                              small_i2f(C[2][i]));
                    acc[o][i] = __fmaf_rn(v, sc[i], acc[o][i]);
                }
            }
            A0 = nA0;
            A1 = nA1;
            dw = ndw;
        }
        __syncthreads();  // every warp is done with this stage
        if (tid == 0 && cb + 2 < ncb) issue(cb + 2);
    }

    // epilogue: acc[o][i] = (row R0 + g + 8 (i >> 1), token 8 (oc0 + o) + 2 tq + (i & 1)) * 2^-28
#pragma unroll
    for (int o = 0; o < kOct; o++) {
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int row = R0 + g + 8 * (i >> 1);
            const int tok = tt * kTok + 8 * (oc0 + o) + 2 * tq + (i & 1);
            const float val = __fmul_rn(acc[o][i], 0x1p28f);
            if (EPI == PF_SWIGLU) {
                // rows 2j (gate) and 2j+1 (up) sit in lanes g and g+1 (lane + 4)
                const float up = __shfl_down_sync(0xffffffffu, val, 4);
                if ((g & 1) == 0 && tok < p.T) p.y[(size_t)tok * p.ldy + (row >> 1)] = __fmul_rn(silu_ref(val), up);
            } else if (tok < p.T) {
                float* yp = p.y + (size_t)tok * p.ldy + row;
                if (EPI == PF_STORE) *yp = val;
                if (EPI == PF_BIAS) *yp = __fadd_rn(val, __ldg(p.bias + row));
                if (EPI == PF_RESID) *yp = __fadd_rn(*yp, val);
            }
        }
    }
}

}  // namespace

int prepare_pf_attention();

size_t pf_digit_bytes(int T, int k) {
    const size_t ntt = (T + kTok - 1) / kTok, ncb = (k + kMegaCB - 1) / kMegaCB;
    return ntt * ncb * kStageDig;
}
size_t pf_scale_floats(int T, int k) {
    const size_t ntt = (T + kTok - 1) / kTok, ncb = (k + kMegaCB - 1) / kMegaCB;
    return ntt * ncb * 16 * kTok;
}

int launch_pf_digitize(const float* x, int ldx, int T, int k, const float* w, float eps, int8_t* dig, float* sx,
                       cudaStream_t s) {
    if (T <= 0 || k <= 0 || k % 32) return arg_error("pf_digitize: k must be a positive multiple of 32");
    const int rows = (T + kTok - 1) / kTok * kTok;
    pf_digitize_kernel<<<rows, 256, 0, s>>>(x, ldx, T, k, w, eps, dig, sx);
    JYC_LAUNCHED();
    return JYC_OK;
}

int prepare_pf_kernels() {
    JYC_CUDA(cudaFuncSetAttribute(pf_gemm_kernel<PF_STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
    JYC_CUDA(cudaFuncSetAttribute(pf_gemm_kernel<PF_BIAS>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
    JYC_CUDA(cudaFuncSetAttribute(pf_gemm_kernel<PF_RESID>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
    JYC_CUDA(cudaFuncSetAttribute(pf_gemm_kernel<PF_SWIGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
    return prepare_pf_attention();
}

int launch_pf_gemm(const PfGemm& p, int epi, cudaStream_t s) {
    if (p.n % kPfRows || p.k % 32 || p.T <= 0) return arg_error("pf_gemm: n % 64 or k % 32");
    const dim3 grid(p.n / kPfRows, (p.T + kTok - 1) / kTok);
    switch (epi) {
        case PF_STORE: pf_gemm_kernel<PF_STORE><<<grid, kThreads, kSmem, s>>>(p); break;
        case PF_BIAS: pf_gemm_kernel<PF_BIAS><<<grid, kThreads, kSmem, s>>>(p); break;
        case PF_RESID: pf_gemm_kernel<PF_RESID><<<grid, kThreads, kSmem, s>>>(p); break;
        case PF_SWIGLU: pf_gemm_kernel<PF_SWIGLU><<<grid, kThreads, kSmem, s>>>(p); break;
        default: return arg_error("pf_gemm: epilogue");
    }
    JYC_LAUNCHED();
    return JYC_OK;
}

// ---------------------------------------------------------------------------
// Causal attention of a prompt chunk over the int8 cache (reference: the
// attention of transformer_layer for seq > 1, transformer_layer.h:35-70).
// CTA = (kv head, 16 query tokens); warp w takes tokens 2w, 2w+1 with all G
// query heads of the kv head (RW = 2G rows). Per block of 64 keys: K/V rows
// into shared memory, scores with int8 dots (dp4a, rotated word order:
// conflict-free), online softmax per row in registers, P.V with the V scale
// folded into P (as the decode path).
namespace {

constexpr int kKB = 64;

template <int HD, int MAXR>
__global__ void __launch_bounds__(256) pf_attention_kernel(PfAttn a) {
    constexpr int HW = HD / 4, DPL = HD / 32;  // words per row, dims per lane
    extern __shared__ __align__(16) unsigned char pf_sm[];
    const int G = a.H / a.KV, RW = 2 * G;
    int8_t* s_k = reinterpret_cast<int8_t*>(pf_sm);                 // [kKB][HD]
    int8_t* s_v = s_k + kKB * HD;                                    // [kKB][HD]
    float* s_ks = reinterpret_cast<float*>(s_v + kKB * HD);          // [kKB]
    float* s_vs = s_ks + kKB;                                        // [kKB]
    float* s_pb = s_vs + kKB;                                        // [8][MAXR][kKB]
    int8_t* s_q = reinterpret_cast<int8_t*>(s_pb + 8 * MAXR * kKB);  // [16 * G][HD]
    auto s_p = [&](int w, int r, int j) -> float& { return s_pb[(w * MAXR + r) * kKB + j]; };
    const int kvh = blockIdx.x, t0 = blockIdx.y * kPfQT;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int q_dim = a.H * HD;
    const int nt = min(kPfQT, a.T - t0);
    // queries of this CTA: row r = t * G + gq
    for (int e = tid; e < nt * G * HW; e += 256) {
        const int r = e / HW, wd = e - r * HW, t = r / G, gq = r - t * G;
        reinterpret_cast<uint32_t*>(s_q)[e] =
            __ldg(reinterpret_cast<const uint32_t*>(a.q8 + (size_t)(t0 + t) * q_dim + (kvh * G + gq) * HD) + wd);
    }
    const int8_t* kb = a.k8 + (size_t)kvh * a.max_seq * HD;
    const int8_t* vb = a.v8 + (size_t)kvh * a.max_seq * HD;
    const float* ksb = a.ks + (size_t)kvh * a.max_seq;
    const float* vsb = a.vs + (size_t)kvh * a.max_seq;
    const int kend = a.pos0 + t0 + nt;  // keys 0 .. kend-1 (the last query's position + 1)

    float acc[MAXR][DPL], m_r[MAXR], l_r[MAXR], qs_r[MAXR];
    int pos_r[MAXR];
#pragma unroll
    for (int r = 0; r < MAXR; r++) {
        m_r[r] = -INFINITY;
        l_r[r] = 0.0f;
#pragma unroll
        for (int i = 0; i < DPL; i++) acc[r][i] = 0.0f;
        const int rr = warp * RW + r, t = rr / G;
        pos_r[r] = (r < RW && t < nt) ? a.pos0 + t0 + t : -1;  // -1: no query row
        qs_r[r] = (r < RW && t < nt) ? __ldg(a.qsc + (size_t)(t0 + t) * a.H + kvh * G + (rr - t * G)) : 0.0f;
    }
    for (int j0 = 0; j0 < kend; j0 += kKB) {
        const int nk = min(kKB, kend - j0);
        __syncthreads();  // previous block fully used
        for (int e = tid; e < nk * (HD / 16); e += 256) {
            const int j = e / (HD / 16), c = e - j * (HD / 16);
            reinterpret_cast<uint4*>(s_k + j * HD)[c] = __ldcg(reinterpret_cast<const uint4*>(kb + (size_t)(j0 + j) * HD) + c);
            reinterpret_cast<uint4*>(s_v + j * HD)[c] = __ldcg(reinterpret_cast<const uint4*>(vb + (size_t)(j0 + j) * HD) + c);
        }
        for (int j = tid; j < nk; j += 256) {
            s_ks[j] = __ldcg(ksb + j0 + j);
            s_vs[j] = __ldcg(vsb + j0 + j);
        }
        __syncthreads();
#pragma unroll
        for (int r = 0; r < MAXR; r++) {
            if (r >= RW || pos_r[r] < 0) continue;  // warp-uniform
            const uint32_t* qw = reinterpret_cast<const uint32_t*>(s_q + (warp * RW + r) * HD);
            float sc[2];
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int j = 32 * h + lane;
                sc[h] = -INFINITY;
                if (j < nk && j0 + j <= pos_r[r]) {
                    const uint32_t* kw = reinterpret_cast<const uint32_t*>(s_k + j * HD);
                    int dot = 0;
#pragma unroll
                    for (int w = 0; w < HW; w++) {
                        const int i = (w + j) & (HW - 1);
                        dot = __dp4a((int)qw[i], (int)kw[i], dot);
                    }
                    sc[h] = __fmul_rn((float)dot, __fmul_rn(__fmul_rn(s_ks[j], qs_r[r]), a.scale));
                }
            }
            const float mb = warp_max(fmaxf(sc[0], sc[1]));
            const float m_new = fmaxf(m_r[r], mb);
            float ps = 0.0f;
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int j = 32 * h + lane;
                const float e = sc[h] == -INFINITY ? 0.0f : expf(sc[h] - m_new);
                ps += e;
                s_p(warp, r, j) = e * (j < nk ? s_vs[j] : 0.0f);
            }
            ps = warp_sum(ps);
            const float alpha = m_r[r] == -INFINITY ? 0.0f : expf(m_r[r] - m_new);
            l_r[r] = l_r[r] * alpha + ps;
            m_r[r] = m_new;
#pragma unroll
            for (int i = 0; i < DPL; i++) acc[r][i] = __fmul_rn(acc[r][i], alpha);
        }
        __syncwarp();
        for (int j = 0; j < nk; j++) {
            float f[4];
            if (DPL == 4) {
                u8x4_to_f32(*reinterpret_cast<const uint32_t*>(s_v + j * HD + 4 * lane) ^ 0x80808080u, f);
            } else {
                const uint32_t w2 = *reinterpret_cast<const uint16_t*>(s_v + j * HD + 2 * lane);
                u8x4_to_f32(w2 ^ 0x80808080u, f);
            }
#pragma unroll
            for (int r = 0; r < MAXR; r++) {
                if (r >= RW) continue;
                const float p = s_p(warp, r, j);
#pragma unroll
                for (int i = 0; i < DPL; i++) acc[r][i] = __fmaf_rn(p, f[i], acc[r][i]);
            }
        }
    }
#pragma unroll
    for (int r = 0; r < MAXR; r++) {
        if (r >= RW || pos_r[r] < 0) continue;
        const int rr = warp * RW + r, t = rr / G, gq = rr - t * G;
        const float inv = 1.0f / l_r[r];
        float* o = a.out + (size_t)(t0 + t) * q_dim + (kvh * G + gq) * HD + DPL * lane;
#pragma unroll
        for (int i = 0; i < DPL; i++) o[i] = __fmul_rn(acc[r][i], inv);
    }
}

}  // namespace

bool pf_attention_supported(int H, int KV, int hd) {
    const int G = KV > 0 ? H / KV : 0;
    return (hd == 64 || hd == 128) && G >= 1 && G <= 8 && H % KV == 0;
}

static int pf_attn_smem(int hd, int G, int maxr) { return 2 * kKB * hd + 2 * kKB * 4 + 8 * maxr * kKB * 4 + kPfQT * G * hd; }

int launch_pf_attention(const PfAttn& a, cudaStream_t s) {
    if (!pf_attention_supported(a.H, a.KV, a.hd)) return arg_error("pf_attention: unsupported head shape");
    const int G = a.H / a.KV;
    const dim3 grid(a.KV, (a.T + kPfQT - 1) / kPfQT);
    const int maxr = G <= 2 ? 4 : G <= 4 ? 8 : 16;
    const int smem = pf_attn_smem(a.hd, G, maxr);
    if (a.hd == 64) {
        if (maxr == 4) pf_attention_kernel<64, 4><<<grid, 256, smem, s>>>(a);
        else if (maxr == 8) pf_attention_kernel<64, 8><<<grid, 256, smem, s>>>(a);
        else pf_attention_kernel<64, 16><<<grid, 256, smem, s>>>(a);
    } else {
        if (maxr == 4) pf_attention_kernel<128, 4><<<grid, 256, smem, s>>>(a);
        else if (maxr == 8) pf_attention_kernel<128, 8><<<grid, 256, smem, s>>>(a);
        else pf_attention_kernel<128, 16><<<grid, 256, smem, s>>>(a);
    }
    JYC_LAUNCHED();
    return JYC_OK;
}

int prepare_pf_attention() {
    const int big = pf_attn_smem(128, 8, 16);
    JYC_CUDA(cudaFuncSetAttribute(pf_attention_kernel<64, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, big));
    JYC_CUDA(cudaFuncSetAttribute(pf_attention_kernel<64, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize, big));
    JYC_CUDA(cudaFuncSetAttribute(pf_attention_kernel<64, 16>, cudaFuncAttributeMaxDynamicSharedMemorySize, big));
    JYC_CUDA(cudaFuncSetAttribute(pf_attention_kernel<128, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, big));
    JYC_CUDA(cudaFuncSetAttribute(pf_attention_kernel<128, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize, big));
    JYC_CUDA(cudaFuncSetAttribute(pf_attention_kernel<128, 16>, cudaFuncAttributeMaxDynamicSharedMemorySize, big));
    return JYC_OK;
}

}  // namespace jyc
