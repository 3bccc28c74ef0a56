// kernels.cu — sm_100a kernels of the batch-1 decode path.
//
// Reference behaviour each kernel reproduces (paths relative to the jieyu tree):
//   gemv (Q8_0)      qmat::matmul_q / dot_row_avx2      libs/matmul_libs/matmul_q.h:101-162
//   gemv (fp32)      matmul                             libs/matmul_libs/matmul.h:7-76
//   fused RMSNorm    rmsnorm                            libs/model_libs/rmsnorm/x86/x86_classic.txt:1-27
//   SwiGLU epilogue  ffn + silu                         libs/model_libs/ffn/ffn.h:7-19, silu/x86/x86_classic.txt
//   rope_quant       rope_pos + kv_pack_q8 + Q quant    rope/x86/x86_classic.txt, attention_q8.h:20-37, 141-153
//   attention        attention_q8 score/softmax/PV      attention/x86/x86_classic.txt:9-74
//   argmax epilogue  greedy loop                        libs/model_libs/generate.h:57-60
//   embed            wmat_row                           libs/model_libs/wmat_kernel.h:18-29
#include "kernels.cuh"
#include "sample.cuh"

#include <algorithm>

namespace jyc {

// ---------------------------------------------------------------------------
// RMSNorm scale of row x[0..n): 1/sqrtf(sum(x^2)/n + eps) (0 when den <= 0),
// computed by the whole block. Same float operations as the reference after
// the sum of squares (whose summation order differs: tree vs 8-lane chains).
__device__ __forceinline__ float block_rms_scale(const float* x, int n, float eps, float* red) {
    float ss = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss = __fmaf_rn(x[i], x[i], ss);
    ss = warp_sum(ss);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (l == 0) red[w] = ss;
    __syncthreads();
    float t = 0.0f;
    for (int i = 0; i < nw; i++) t += red[i];
    const float den = __fadd_rn(__fdiv_rn(t, (float)n), eps);
    return den <= 0.0f ? 0.0f : __fdiv_rn(1.0f, __fsqrt_rn(den));
}

__device__ __forceinline__ uint4 ldg_stream(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// ---------------------------------------------------------------------------
// GEMV / skinny GEMM: y[mt][row] = sum_k xhat[mt][k] * W[row][k], mt < m <= MT.
// One warp owns RPW consecutive rows; lanes stride the row in 16-byte vectors
// (16 Q8 weights or 4x2 fp32 weights per lane and step); the next step's
// weight vectors are loaded before the current ones are used. Warps walk the
// rows grid-stride. Per-lane partials are reduced with xor shuffles.
template <int WT, int MT, int RPW, int EPI>
__global__ void __launch_bounds__(128) gemv_kernel(GemvArgs a) {
    if (a.st != nullptr && *(volatile const int*)&a.st->active == 0) return;
    __shared__ float s_red[8];
    __shared__ float s_scale[MT];
    __shared__ unsigned long long s_best;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarp = blockDim.x >> 5;
    const int m = a.m, k = a.k;

    // Fused RMSNorm prologue: per activation row, the scale 1/rms.
    if (a.norm_w != nullptr) {
        for (int mt = 0; mt < m; mt++) {
            const float sc = block_rms_scale(a.x + (size_t)mt * a.ldx, k, a.eps, s_red);
            if (threadIdx.x == 0) s_scale[mt] = sc;
        }
    }
    if (EPI == EPI_ARGMAX && threadIdx.x == 0) s_best = 0ull;
    __syncthreads();

    constexpr int EPC = (WT == W_Q8) ? 16 : 8;  // elements per lane-step
    const int nch = k / EPC;
    const int ngroups = (a.n + RPW - 1) / RPW;
    unsigned long long best = 0ull;

    for (int g = blockIdx.x * nwarp + warp; g < ngroups; g += gridDim.x * nwarp) {
        const int row0 = g * RPW;
        float acc[MT][RPW];
#pragma unroll
        for (int mt = 0; mt < MT; mt++)
#pragma unroll
            for (int r = 0; r < RPW; r++) acc[mt][r] = 0.0f;

        constexpr int NV = (WT == W_F32) ? 2 : 1;  // 16-byte vectors per row and lane-step
        // weight fetch for lane-step c
        auto fetch = [&](int c, uint4 (&w)[RPW][NV], float (&dsc)[RPW]) {
#pragma unroll
            for (int r = 0; r < RPW; r++) {
                const int row = min(row0 + r, a.n - 1);
                if (WT == W_Q8) {
                    w[r][0] = ldg_stream(a.qs + (size_t)row * k + (size_t)c * 16);
                    dsc[r] = h2f(__ldg(a.d + (size_t)row * (k >> 5) + (c >> 1)));
                } else if (WT == W_F16) {
                    w[r][0] = ldg_stream(a.wh + (size_t)row * k + (size_t)c * 8);
                    dsc[r] = 1.0f;
                } else {
                    const float* p = a.wt + (size_t)row * k + (size_t)c * 8;
                    w[r][0] = ldg_stream(p);
                    w[r][1] = ldg_stream(p + 4);
                    dsc[r] = 1.0f;
                }
            }
        };
        uint4 wc[RPW][NV], wn[RPW][NV];
        float dc[RPW], dn[RPW];
        int c = lane;
        if (c < nch) fetch(c, wc, dc);
        for (; c < nch; c += 32) {
            if (c + 32 < nch) fetch(c + 32, wn, dn);
            // weights of this step as floats
            float wf[RPW][EPC];
#pragma unroll
            for (int r = 0; r < RPW; r++) {
                if (WT == W_Q8) {
                    u8x4_to_f32(wc[r][0].x, &wf[r][0]);
                    u8x4_to_f32(wc[r][0].y, &wf[r][4]);
                    u8x4_to_f32(wc[r][0].z, &wf[r][8]);
                    u8x4_to_f32(wc[r][0].w, &wf[r][12]);
                } else if (WT == W_F16) {  // exact: every half is a float
                    const uint32_t hw[4] = {wc[r][0].x, wc[r][0].y, wc[r][0].z, wc[r][0].w};
#pragma unroll
                    for (int v = 0; v < 4; v++) {
                        wf[r][2 * v] = h2f((uint16_t)(hw[v] & 0xffffu));
                        wf[r][2 * v + 1] = h2f((uint16_t)(hw[v] >> 16));
                    }
                } else {
#pragma unroll
                    for (int v = 0; v < NV; v++) {
                        wf[r][v * 4 + 0] = __uint_as_float(wc[r][v].x);
                        wf[r][v * 4 + 1] = __uint_as_float(wc[r][v].y);
                        wf[r][v * 4 + 2] = __uint_as_float(wc[r][v].z);
                        wf[r][v * 4 + 3] = __uint_as_float(wc[r][v].w);
                    }
                }
            }
            const int k0 = c * EPC;
#pragma unroll
            for (int mt = 0; mt < MT; mt++) {
                if (mt < m) {
                    float xv[EPC];
                    const float4* xp = reinterpret_cast<const float4*>(a.x + (size_t)mt * a.ldx + k0);
#pragma unroll
                    for (int v = 0; v < EPC / 4; v++) {
                        const float4 t = __ldg(xp + v);
                        xv[v * 4 + 0] = t.x; xv[v * 4 + 1] = t.y;
                        xv[v * 4 + 2] = t.z; xv[v * 4 + 3] = t.w;
                    }
                    if (a.norm_w != nullptr) {
                        const float sc = s_scale[mt];
                        const float4* np = reinterpret_cast<const float4*>(a.norm_w + k0);
#pragma unroll
                        for (int v = 0; v < EPC / 4; v++) {
                            const float4 t = __ldg(np + v);
                            xv[v * 4 + 0] = __fmul_rn(__fmul_rn(xv[v * 4 + 0], sc), t.x);
                            xv[v * 4 + 1] = __fmul_rn(__fmul_rn(xv[v * 4 + 1], sc), t.y);
                            xv[v * 4 + 2] = __fmul_rn(__fmul_rn(xv[v * 4 + 2], sc), t.z);
                            xv[v * 4 + 3] = __fmul_rn(__fmul_rn(xv[v * 4 + 3], sc), t.w);
                        }
                    }
#pragma unroll
                    for (int r = 0; r < RPW; r++) {
                        float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
                        for (int i = 0; i < EPC; i += 2) {
                            s0 = __fmaf_rn(wf[r][i], xv[i], s0);
                            s1 = __fmaf_rn(wf[r][i + 1], xv[i + 1], s1);
                        }
                        acc[mt][r] = __fmaf_rn(__fadd_rn(s0, s1), dc[r], acc[mt][r]);
                    }
                }
            }
#pragma unroll
            for (int r = 0; r < RPW; r++) {
#pragma unroll
                for (int v = 0; v < NV; v++) wc[r][v] = wn[r][v];
                dc[r] = dn[r];
            }
        }
#pragma unroll
        for (int mt = 0; mt < MT; mt++)
#pragma unroll
            for (int r = 0; r < RPW; r++) acc[mt][r] = warp_sum(acc[mt][r]);

        if (lane == 0) {
#pragma unroll
            for (int mt = 0; mt < MT; mt++) {
                if (mt >= m) continue;
                if (EPI == EPI_SWIGLU) {
                    // rows (2j, 2j+1) = (gate_j, up_j): h_j = silu(gate_j) * up_j
#pragma unroll
                    for (int r = 0; r + 1 < RPW; r += 2) {
                        const int row = row0 + r;
                        if (row + 1 < a.n)
                            a.y[(size_t)mt * a.ldy + (row >> 1)] =
                                __fmul_rn(silu_ref(acc[mt][r]), acc[mt][r + 1]);
                    }
                } else {
#pragma unroll
                    for (int r = 0; r < RPW; r++) {
                        const int row = row0 + r;
                        if (row >= a.n) continue;
                        float v = acc[mt][r];
                        float* yp = a.y + (size_t)mt * a.ldy + row;
                        if (EPI == EPI_BIAS) v = __fadd_rn(v, a.bias[row]);
                        if (EPI == EPI_RESID) v = __fadd_rn(*yp, v);
                        *yp = v;
                        if (EPI == EPI_ARGMAX) {
                            const unsigned long long p = argmax_pack(v, row);
                            best = p > best ? p : best;
                        }
                    }
                }
            }
        }
    }

    if (EPI == EPI_ARGMAX) {
        // CTA max -> one 64-bit atomicMax; the last CTA to arrive publishes the token.
        if (lane == 0 && best) atomicMax(&s_best, best);
        __syncthreads();
        if (threadIdx.x == 0) {
            if (s_best) atomicMax(&a.st->amax, s_best);
            __threadfence();
            const unsigned int prev = atomicAdd(&a.st->head_arrive, 1u);
            if (prev == gridDim.x - 1) {
                __threadfence();
                DevState* st = a.st;
                const unsigned long long packed = atomicAdd(&st->amax, 0ull);
                const int next = argmax_index(packed);
                const int len = st->len;
                a.tokens[len] = next;
                const int nlen = len + 1;
                const int nsteps = st->steps + 1;
                bool stop = nlen >= st->max_len || nsteps >= st->max_new;
                for (int e = 0; e < st->n_eos; e++)
                    if (next == st->eos[e]) stop = true;
                st->len = nlen;
                st->steps = nsteps;
                st->amax = 0ull;
                st->head_arrive = 0u;
                st->fresh = 1;
                if (stop) st->active = 0;
                __threadfence();
            }
        }
    }
}

template <int WT, int MT, int RPW, int EPI>
static int launch_gemv_t(const GemvArgs& a, cudaStream_t s) {
    const int ngroups = (a.n + RPW - 1) / RPW;
    const int warps = 4;
    int blocks = (ngroups + warps - 1) / warps;
    int cap = 148 * 8;
    if (EPI == EPI_ARGMAX) cap = 148 * 4;
    blocks = std::min(blocks, cap);
    gemv_kernel<WT, MT, RPW, EPI><<<blocks, warps * 32, 0, s>>>(a);
    JYC_LAUNCHED();
    return JYC_OK;
}

template <int WT, int MT, int EPI>
static int launch_gemv_rpw(const GemvArgs& a, cudaStream_t s) {
    // Enough row groups for ~2 waves of 4-warp CTAs on 148 SMs, but more rows
    // per warp (the activation loads shared by more weight rows) when the
    // matrix is tall; 8 activation rows keep one or two weight rows per warp
    // (registers).
    if (EPI == EPI_SWIGLU) {
        if (MT <= 4 && a.n >= 148 * 4 * 4 * 2) return launch_gemv_t<WT, MT, 4, EPI>(a, s);
        return launch_gemv_t<WT, MT, 2, EPI>(a, s);
    }
    if (MT == 8) {
        if (a.n >= 148 * 4 * 2 * 2) return launch_gemv_t<WT, MT, 2, EPI>(a, s);
        return launch_gemv_t<WT, MT, 1, EPI>(a, s);
    }
    if (a.n >= 148 * 4 * 4 * 4) return launch_gemv_t<WT, MT, 4, EPI>(a, s);
    if (a.n >= 148 * 4 * 2 * 2) return launch_gemv_t<WT, MT, 2, EPI>(a, s);
    return launch_gemv_t<WT, MT, 1, EPI>(a, s);
}

template <int WT, int EPI>
static int launch_gemv_mt(const GemvArgs& a, cudaStream_t s) {
    if (a.m == 1) return launch_gemv_rpw<WT, 1, EPI>(a, s);
    if (a.m == 2) return launch_gemv_rpw<WT, 2, EPI>(a, s);
    if (a.m <= 4) return launch_gemv_rpw<WT, 4, EPI>(a, s);
    return launch_gemv_rpw<WT, 8, EPI>(a, s);
}

template <int WT>
static int launch_gemv_epi(const GemvArgs& a, int epi, cudaStream_t s) {
    switch (epi) {
        case EPI_STORE: return launch_gemv_mt<WT, EPI_STORE>(a, s);
        case EPI_BIAS: return launch_gemv_mt<WT, EPI_BIAS>(a, s);
        case EPI_RESID: return launch_gemv_mt<WT, EPI_RESID>(a, s);
        case EPI_SWIGLU: return launch_gemv_mt<WT, EPI_SWIGLU>(a, s);
        case EPI_ARGMAX:
            if (a.m != 1) return arg_error("gemv: argmax epilogue needs m == 1");
            return launch_gemv_rpw<WT, 1, EPI_ARGMAX>(a, s);
    }
    return arg_error("gemv: unknown epilogue");
}

int launch_gemv(const GemvArgs& a, int wtype, int epi, cudaStream_t s) {
    if (a.m < 1 || a.m > 8) return arg_error("gemv: m must be in [1, 8]");
    if (a.n <= 0 || a.k <= 0) return arg_error("gemv: empty shape");
    if (wtype == W_Q8) {
        if (a.k % 32) return arg_error("gemv: Q8_0 needs k % 32 == 0");
        return launch_gemv_epi<W_Q8>(a, epi, s);
    }
    if (a.k % 8) return arg_error("gemv: fp32 / fp16 paths need k % 8 == 0");
    if (wtype == W_F16) return launch_gemv_epi<W_F16>(a, epi, s);
    return launch_gemv_epi<W_F32>(a, epi, s);
}

// ---------------------------------------------------------------------------
// x[i] += p[i] (the residual add of a partial sum computed elsewhere).
__global__ void add_rows_kernel(float* x, const float* p, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        x[i] = __fadd_rn(x[i], p[i]);
}
int launch_add_rows(float* x, const float* p, size_t n, cudaStream_t s) {
    if (n == 0) return JYC_OK;
    const int blocks = (int)std::min<size_t>((n + 255) / 256, 148 * 8);
    add_rows_kernel<<<blocks, 256, 0, s>>>(x, p, n);
    JYC_LAUNCHED();
    return JYC_OK;
}

// ---------------------------------------------------------------------------
// Bias rows and the SwiGLU product (the K-quant model path's epilogues, the
// same arithmetic as the GEMV's EPI_BIAS and EPI_SWIGLU).
__global__ void bias_rows_kernel(float* y, int ldy, const float* bias, int n, int rows) {
    const size_t total = (size_t)rows * n;
    for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
        const int r = (int)(e / n), i = (int)(e - (size_t)r * n);
        float* p = y + (size_t)r * ldy + i;
        *p = __fadd_rn(*p, bias[i]);
    }
}
int launch_bias_rows(float* y, int ldy, const float* bias, int n, int rows, cudaStream_t s) {
    if (n <= 0 || rows <= 0) return JYC_OK;
    const size_t total = (size_t)rows * n;
    bias_rows_kernel<<<(int)std::min<size_t>((total + 255) / 256, 148 * 8), 256, 0, s>>>(y, ldy, bias, n, rows);
    JYC_LAUNCHED();
    return JYC_OK;
}
__global__ void swiglu_rows_kernel(const float* g, const float* u, float* h, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        h[i] = __fmul_rn(silu_ref(g[i]), u[i]);
}
int launch_swiglu_rows(const float* g, const float* u, float* h, size_t n, cudaStream_t s) {
    if (n == 0) return JYC_OK;
    swiglu_rows_kernel<<<(int)std::min<size_t>((n + 255) / 256, 148 * 8), 256, 0, s>>>(g, u, h, n);
    JYC_LAUNCHED();
    return JYC_OK;
}

// ---------------------------------------------------------------------------
// Standalone RMSNorm rows (op entry point).
__global__ void rmsnorm_kernel(const float* x, float* y, const float* w, int n, float eps) {
    __shared__ float red[32];
    const float* xr = x + (size_t)blockIdx.x * n;
    float* yr = y + (size_t)blockIdx.x * n;
    const float sc = block_rms_scale(xr, n, eps, red);
    for (int i = threadIdx.x; i < n; i += blockDim.x) yr[i] = __fmul_rn(__fmul_rn(xr[i], sc), w[i]);
}
int launch_rmsnorm(const float* x, float* y, const float* w, int rows, int n, float eps,
                   cudaStream_t s) {
    if (rows <= 0 || n <= 0) return arg_error("rmsnorm: empty shape");
    rmsnorm_kernel<<<rows, 256, 0, s>>>(x, y, w, n, eps);
    JYC_LAUNCHED();
    return JYC_OK;
}

// ---------------------------------------------------------------------------
// RoPE + int8 quantisation. One warp per (row, head); lane owns pairs p, p+32..
// Q heads: roped, quantised into q8/qsc. K heads: roped, quantised into the
// cache at pos. V heads: quantised into the cache.
__global__ void rope_quant_kernel(RopeQuantArgs a) {
    if (pos_inactive(a.pos)) return;
    const int lane = threadIdx.x & 31;
    const int unit = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int nh = a.H + 2 * a.KV;
    if (unit >= a.rows * nh) return;
    const int i = unit / nh, h = unit % nh;
    const int pos = a.row_len ? a.row_len[i] - 1 : pos_first(a.pos) + i;
    const int hd = a.hd, half = hd >> 1;
    const bool is_q = h < a.H, is_k = !is_q && h < a.H + a.KV;
    const float* src = is_q ? a.q + (size_t)i * a.ldq + (size_t)h * hd
                     : is_k ? a.k + (size_t)i * a.ldq + (size_t)(h - a.H) * hd
                            : a.v + (size_t)i * a.ldq + (size_t)(h - a.H - a.KV) * hd;
    const bool rot = a.cos_t != nullptr && (is_q || is_k);
    const float* ct = rot ? a.cos_t + (size_t)pos * half : nullptr;
    const float* stb = rot ? a.sin_t + (size_t)pos * half : nullptr;

    constexpr int MAXP = 4;  // pairs per lane (head_dim <= 256)
    float x0[MAXP], x1[MAXP];
    float amax = 0.0f;
#pragma unroll
    for (int t = 0; t < MAXP; t++) {
        const int p = lane + 32 * t;
        x0[t] = 0.0f; x1[t] = 0.0f;
        if (p < half) {
            float v0 = src[2 * p], v1 = src[2 * p + 1];
            if (rot) {
                const float c = ct[p], sn = stb[p];
                const float r0 = __fmaf_rn(v0, c, -__fmul_rn(v1, sn));
                const float r1 = __fmaf_rn(v0, sn, __fmul_rn(v1, c));
                v0 = r0; v1 = r1;
            }
            x0[t] = v0; x1[t] = v1;
            amax = fmaxf(amax, fmaxf(fabsf(v0), fabsf(v1)));
        }
    }
    amax = warp_max(amax);
    const float inv = q8_inv(amax), sc = q8_scale(amax);
    int8_t* dst;
    if (is_q) {
        dst = a.q8 + ((size_t)i * a.H + h) * hd;
        if (lane == 0) a.qsc[(size_t)i * a.H + h] = sc;
        if (a.q_roped) {
            float* qr = a.q_roped + (size_t)i * a.H * hd + (size_t)h * hd;
            for (int t = 0; t < MAXP; t++) {
                const int p = lane + 32 * t;
                const int o = rot ? rope_slot(p, half) : p;
                if (p < half) { qr[2 * o] = x0[t]; qr[2 * o + 1] = x1[t]; }
            }
        }
    } else {
        const int kvh = is_k ? h - a.H : h - a.H - a.KV;
        if (pos >= a.kv.cap) return;  // host checks capacity; never write past the cache
        int8_t* base = (is_k ? a.kv.k : a.kv.v) + (a.row_len ? (size_t)i * a.kv_row_stride : 0);
        float* sbase = (is_k ? a.kv.ks : a.kv.vs) + (a.row_len ? (size_t)i * a.skv_row_stride : 0);
        dst = base + (size_t)pos * a.kv.pos_stride + (size_t)kvh * a.kv.head_stride;
        if (lane == 0) sbase[(size_t)pos * a.kv.spos_stride + (size_t)kvh * a.kv.shead_stride] = sc;
        if (is_k && a.k_roped) {
            float* kr = a.k_roped + (size_t)i * a.KV * hd + (size_t)kvh * hd;
            for (int t = 0; t < MAXP; t++) {
                const int p = lane + 32 * t;
                const int o = rot ? rope_slot(p, half) : p;
                if (p < half) { kr[2 * o] = x0[t]; kr[2 * o + 1] = x1[t]; }
            }
        }
    }
#pragma unroll
    for (int t = 0; t < MAXP; t++) {
        const int p = lane + 32 * t;
        if (p < half) {
            const int o = rot ? rope_slot(p, half) : p;  // reference store order
            dst[2 * o] = (int8_t)q8_round(x0[t], inv);
            dst[2 * o + 1] = (int8_t)q8_round(x1[t], inv);
        }
    }
}
// In-place RoPE (rope_pos), one warp per (row, head), lane owns pairs; the
// rotated pairs are stored in the reference's slot order (rope_slot).
__global__ void rope_kernel(float* q, int seq, int start_pos, int heads, int hd,
                            const float* cos_t, const float* sin_t) {
    const int lane = threadIdx.x & 31;
    const int unit = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (unit >= seq * heads) return;
    const int i = unit / heads, half = hd >> 1;
    float* x = q + (size_t)unit * hd;
    const float* ct = cos_t + (size_t)(start_pos + i) * half;
    const float* st = sin_t + (size_t)(start_pos + i) * half;
    constexpr int MAXP = 4;  // head_dim <= 256
    float r0[MAXP], r1[MAXP];
#pragma unroll
    for (int t = 0; t < MAXP; t++) {
        const int p = lane + 32 * t;
        if (p < half) {
            const float v0 = x[2 * p], v1 = x[2 * p + 1], c = ct[p], sn = st[p];
            r0[t] = __fmaf_rn(v0, c, -__fmul_rn(v1, sn));
            r1[t] = __fmaf_rn(v0, sn, __fmul_rn(v1, c));
        }
    }
    __syncwarp();  // every pair is read before any slot is overwritten
#pragma unroll
    for (int t = 0; t < MAXP; t++) {
        const int p = lane + 32 * t;
        if (p < half) {
            const int o = rope_slot(p, half);
            x[2 * o] = r0[t];
            x[2 * o + 1] = r1[t];
        }
    }
}
int launch_rope(float* q, int seq, int start_pos, int heads, int hd, const float* cos_t,
                const float* sin_t, cudaStream_t s) {
    if ((hd & 1) || hd > 256) return arg_error("rope_pos: head_dim must be even and <= 256");
    const int units = seq * heads;
    if (units <= 0) return JYC_OK;
    rope_kernel<<<(units + 3) / 4, 128, 0, s>>>(q, seq, start_pos, heads, hd, cos_t, sin_t);
    JYC_LAUNCHED();
    return JYC_OK;
}

int launch_rope_quant(const RopeQuantArgs& a, cudaStream_t s) {
    if (a.hd > 256 || (a.hd & 1)) return arg_error("rope_quant: head_dim must be even and <= 256");
    const int units = a.rows * (a.H + 2 * a.KV);
    const int wpb = 4;
    rope_quant_kernel<<<(units + wpb - 1) / wpb, wpb * 32, 0, s>>>(a);
    JYC_LAUNCHED();
    return JYC_OK;
}

// ---------------------------------------------------------------------------
// Split-K flash-decoding over the int8 KV cache. CTA = (split, kv_head); it
// serves every (row, query head of the group) pair. Per sub-block of 64
// positions: int8 K/V tiles -> shared memory, int32 dp4a scores scaled
// exactly as the reference ((ks*qs)*scale), online softmax in fp32, PV
// accumulate. Partials (m, l, o) go to scratch; the last CTA of each kv head
// (arrival counter) merges the splits into `out`.
constexpr int SB = 64;

int attn_smem_bytes(int rows, int H, int KV, int hd) {
    const int P = rows * (H / KV);
    return P * hd                 // q8
           + P * 4 * 4            // qsc, m, l, alpha
           + P * hd * 4           // o accumulators
           + P * SB * 4           // scores / weights
           + SB * (hd + 4)        // k tile (rows padded one word: conflict-free dp4a reads)
           + SB * hd              // v tile
           + 2 * SB * 4;          // ks, vs
}

__global__ void __launch_bounds__(128) attention_kernel(AttnArgs a) {
    if (pos_inactive(a.pos)) return;
    extern __shared__ __align__(16) unsigned char smem[];
    const int G = a.H / a.KV, P = a.rows * G, hd = a.hd;
    const int kvh = blockIdx.y, split = blockIdx.x;
    const int pos0 = pos_first(a.pos);
    const int8_t* q8 = a.q8;
    const float* qsc = a.qsc;
    const int8_t* kbase = a.kv.k;
    const int8_t* vbase = a.kv.v;
    const float* ksbase = a.kv.ks;
    const float* vsbase = a.kv.vs;
    float* part_o = a.part_o;
    float* part_ml = a.part_ml;
    unsigned int* arrive = a.arrive;
    float* out = a.out;
    const int pos_last = pos0 + a.rows - 1;
    const int c0 = split * a.chunk;
    const int c1 = min(c0 + a.chunk, pos_last + 1);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nthr = blockDim.x;

    if (c0 <= pos_last) {
        int8_t* s_q8 = reinterpret_cast<int8_t*>(smem);
        float* s_qsc = reinterpret_cast<float*>(smem + P * hd);
        float* s_m = s_qsc + P;
        float* s_l = s_m + P;
        float* s_alpha = s_l + P;
        float* s_o = s_alpha + P;
        float* s_w = s_o + P * hd;
        int8_t* s_k = reinterpret_cast<int8_t*>(s_w + P * SB);
        int8_t* s_v = s_k + SB * (hd + 4);
        float* s_ks = reinterpret_cast<float*>(s_v + SB * hd);
        float* s_vs = s_ks + SB;

        // pair p = (row i, group head g) -> query head h = kvh*G + g
        for (int e = tid; e < P * hd; e += nthr) {
            const int p = e / hd, dd = e % hd, i = p / G, g = p % G;
            s_q8[e] = q8[((size_t)i * a.H + kvh * G + g) * hd + dd];
            s_o[e] = 0.0f;
        }
        for (int p = tid; p < P; p += nthr) {
            const int i = p / G, g = p % G;
            s_qsc[p] = qsc[(size_t)i * a.H + kvh * G + g];
            s_m[p] = -INFINITY;
            s_l[p] = 0.0f;
        }
        __syncthreads();

        const int8_t* kb = kbase + (size_t)kvh * a.kv.head_stride;
        const int8_t* vb = vbase + (size_t)kvh * a.kv.head_stride;
        const float* ksb = ksbase + (size_t)kvh * a.kv.shead_stride;
        const float* vsb = vsbase + (size_t)kvh * a.kv.shead_stride;
        const int hw = hd >> 2;  // 32-bit words per head row

        for (int j0 = c0; j0 < c1; j0 += SB) {
            const int nj = min(SB, c1 - j0);
            // tiles (4-byte granules; head_dim % 4 == 0)
            for (int e = tid; e < nj * hw; e += nthr) {
                const int j = e / hw, wd = e % hw;
                const size_t off = (size_t)(j0 + j) * a.kv.pos_stride;
                reinterpret_cast<uint32_t*>(s_k)[j * (hw + 1) + wd] =
                    __ldg(reinterpret_cast<const uint32_t*>(kb + off) + wd);
                reinterpret_cast<uint32_t*>(s_v)[j * hw + wd] =
                    __ldg(reinterpret_cast<const uint32_t*>(vb + off) + wd);
            }
            for (int j = tid; j < nj; j += nthr) {
                s_ks[j] = __ldg(ksb + (size_t)(j0 + j) * a.kv.spos_stride);
                s_vs[j] = __ldg(vsb + (size_t)(j0 + j) * a.kv.spos_stride);
            }
            __syncthreads();
            // scores
            for (int e = tid; e < P * SB; e += nthr) {
                const int p = e / SB, j = e % SB, i = p / G;
                float sc = -INFINITY;
                if (j < nj && j0 + j <= pos0 + i) {
                    const int* qw = reinterpret_cast<const int*>(s_q8 + p * hd);
                    const int* kw = reinterpret_cast<const int*>(s_k + j * (hd + 4));
                    int dot = 0;
                    for (int wd = 0; wd < hw; wd++) dot = __dp4a(qw[wd], kw[wd], dot);
                    const float ksc = __fmul_rn(__fmul_rn(s_ks[j], s_qsc[p]), a.scale);
                    sc = __fmul_rn((float)dot, ksc);
                }
                s_w[e] = sc;
            }
            __syncthreads();
            // online softmax per pair (one warp per pair)
            for (int p = warp; p < P; p += nthr >> 5) {
                float mx = -INFINITY;
                for (int j = lane; j < SB; j += 32) mx = fmaxf(mx, s_w[p * SB + j]);
                mx = warp_max(mx);
                const float m_old = s_m[p];
                const float m_new = fmaxf(m_old, mx);
                float sum = 0.0f;
                for (int j = lane; j < SB; j += 32) {
                    const float sv = s_w[p * SB + j];
                    const float e = (sv == -INFINITY) ? 0.0f : expf(sv - m_new);
                    sum += e;
                    s_w[p * SB + j] = e * s_vs[j < nj ? j : 0];
                }
                sum = warp_sum(sum);
                if (lane == 0) {
                    const float alpha = (m_old == -INFINITY) ? 0.0f : expf(m_old - m_new);
                    s_alpha[p] = alpha;
                    s_l[p] = s_l[p] * alpha + sum;
                    s_m[p] = m_new;
                }
            }
            __syncthreads();
            // o = o*alpha + sum_j w_j * v_j
            for (int e = tid; e < P * hd; e += nthr) {
                const int p = e / hd, dd = e % hd;
                float o = s_o[e] * s_alpha[p];
                const float* wp = s_w + p * SB;
                for (int j = 0; j < nj; j++) o = __fmaf_rn(wp[j], (float)s_v[j * hd + dd], o);
                s_o[e] = o;
            }
            __syncthreads();
        }
        // write partials
        for (int e = tid; e < P * hd; e += nthr) {
            const int p = e / hd, dd = e % hd, i = p / G, g = p % G;
            const int h = kvh * G + g;
            part_o[(((size_t)i * a.H + h) * a.nsplit + split) * hd + dd] = s_o[e];
        }
        for (int p = tid; p < P; p += nthr) {
            const int i = p / G, g = p % G, h = kvh * G + g;
            float* ml = part_ml + (((size_t)i * a.H + h) * a.nsplit + split) * 2;
            ml[0] = s_m[p];
            ml[1] = s_l[p];
        }
    }

    // arrival; the last CTA of this kv head merges the splits
    __shared__ unsigned int s_last;
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const unsigned int prev = atomicAdd(&arrive[kvh], 1u);
        s_last = (prev == gridDim.x - 1) ? 1u : 0u;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const int nvalid = pos_last / a.chunk + 1;
    for (int e = tid; e < P * hd; e += nthr) {
        const int p = e / hd, dd = e % hd, i = p / G, g = p % G, h = kvh * G + g;
        const size_t base = ((size_t)i * a.H + h) * a.nsplit;
        float M = -INFINITY;
        for (int s2 = 0; s2 < nvalid; s2++) M = fmaxf(M, __ldcg(part_ml + (base + s2) * 2));
        float L = 0.0f, O = 0.0f;
        for (int s2 = 0; s2 < nvalid; s2++) {
            const float ms = __ldcg(part_ml + (base + s2) * 2);
            if (ms == -INFINITY) continue;
            const float wgt = expf(ms - M);
            L = __fmaf_rn(wgt, __ldcg(part_ml + (base + s2) * 2 + 1), L);
            O = __fmaf_rn(wgt, __ldcg(part_o + (base + s2) * hd + dd), O);
        }
        out[(size_t)i * a.ldo + (size_t)h * hd + dd] = O / L;
    }
    if (tid == 0) arrive[kvh] = 0u;
}

// One-time kernel attributes (called at model creation, outside any capture).
int prepare_kernels() {
    // once per process (thread-safe static initialisation)
    static const cudaError_t e =
        cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    return e == cudaSuccess ? JYC_OK : cuda_fail(e, "cudaFuncSetAttribute");
}
#define TRY_PREPARE()                          \
    do {                                       \
        const int _r = prepare_kernels();      \
        if (_r != JYC_OK) return _r;           \
    } while (0)

int launch_attention(const AttnArgs& a, cudaStream_t s) {
    if (a.KV <= 0 || a.H % a.KV) return arg_error("attention: num_heads must be a multiple of num_kv_heads");
    if (a.hd % 4) return arg_error("attention: head_dim must be a multiple of 4");
    const int smem = attn_smem_bytes(a.rows, a.H, a.KV, a.hd);
    if (smem > 200 * 1024) return arg_error("attention: group too large for shared memory");
    TRY_PREPARE();
    dim3 grid(a.nsplit, a.KV);
    attention_kernel<<<grid, 128, smem, s>>>(a);
    JYC_LAUNCHED();
    return JYC_OK;
}

// ---------------------------------------------------------------------------
// Embedding rows: X[i] = embed[token[pos0+i]] (fp32 copy or exact Q8 dequant).
__global__ void embed_kernel(const int* tokens, PosSrc pos, const float* ef, const uint8_t* eqs,
                             const uint16_t* ed, int hidden, float* X) {
    if (pos_inactive(pos)) return;
    const int i = blockIdx.x;
    const int id = tokens[pos_first(pos) + i];
    float* xr = X + (size_t)i * hidden;
    for (int c = threadIdx.x; c < hidden; c += blockDim.x) {
        if (ef) {
            xr[c] = ef[(size_t)id * hidden + c];
        } else {
            const float q = (float)((int)eqs[(size_t)id * hidden + c] - 128);
            xr[c] = __fmul_rn(q, h2f(ed[(size_t)id * (hidden >> 5) + (c >> 5)]));
        }
    }
}
int launch_embed(const int* tokens, PosSrc pos, int rows, const float* ef, const uint8_t* eqs,
                 const uint16_t* ed, int hidden, float* X, cudaStream_t s) {
    embed_kernel<<<rows, 256, 0, s>>>(tokens, pos, ef, eqs, ed, hidden, X);
    JYC_LAUNCHED();
    return JYC_OK;
}

// ---------------------------------------------------------------------------
// Reference Q8_0 blocks [n][k/32] x (fp16 d, 32 x int8) -> device layout.
// Source row r lands in destination row row_off + r*row_stride (fused QKV and
// interleaved gate/up matrices are assembled this way).
__global__ void q8_repack_kernel(const uint8_t* blocks, size_t nblocks, int nb, uint8_t* qs,
                                 uint16_t* d, int row_off, int row_stride) {
    for (size_t b = blockIdx.x * (size_t)blockDim.x + threadIdx.x; b < nblocks;
         b += (size_t)gridDim.x * blockDim.x) {
        const size_t r = b / nb, bl = b % nb;
        const size_t db = ((size_t)row_off + r * (size_t)row_stride) * nb + bl;
        const uint8_t* src = blocks + b * 34;
        d[db] = (uint16_t)src[0] | ((uint16_t)src[1] << 8);
        uint32_t* q = reinterpret_cast<uint32_t*>(qs + db * 32);
#pragma unroll
        for (int w = 0; w < 8; w++) {
            uint32_t v = (uint32_t)src[2 + 4 * w] | ((uint32_t)src[3 + 4 * w] << 8) |
                         ((uint32_t)src[4 + 4 * w] << 16) | ((uint32_t)src[5 + 4 * w] << 24);
            q[w] = v ^ 0x80808080u;  // q -> q+128
        }
    }
}
int launch_q8_repack(const void* blocks, int n, int k, uint8_t* qs, uint16_t* d, int row_off,
                     int row_stride, cudaStream_t s) {
    if (n <= 0 || k <= 0 || k % 32) return arg_error("q8_repack: k must be a positive multiple of 32");
    const size_t nb = (size_t)n * (k / 32);
    const int blocks_n = (int)std::min<size_t>((nb + 255) / 256, 148 * 16);
    q8_repack_kernel<<<blocks_n, 256, 0, s>>>(static_cast<const uint8_t*>(blocks), nb, k / 32, qs, d,
                                              row_off, row_stride);
    JYC_LAUNCHED();
    return JYC_OK;
}

// B [k][n] -> Bt rows: source column c lands in row row_off + c*row_stride of Bt [.][k].
template <typename T>
__global__ void transpose_kernel(const T* B, T* Bt, int k, int n, int row_off, int row_stride) {
    __shared__ T tile[32][33];
    const int bx = blockIdx.x * 32, by = blockIdx.y * 32;
    for (int j = threadIdx.y; j < 32; j += blockDim.y) {
        const int r = by + j, c = bx + threadIdx.x;
        if (r < k && c < n) tile[j][threadIdx.x] = B[(size_t)r * n + c];
    }
    __syncthreads();
    for (int j = threadIdx.y; j < 32; j += blockDim.y) {
        const int col = bx + j, p = by + threadIdx.x;  // Bt[col][p] = B[p][col]
        if (col < n && p < k)
            Bt[((size_t)row_off + (size_t)col * row_stride) * k + p] = tile[threadIdx.x][j];
    }
}
int launch_transpose(const float* B, float* Bt, int k, int n, int row_off, int row_stride,
                     cudaStream_t s) {
    if (k <= 0 || n <= 0) return arg_error("transpose: empty shape");
    dim3 grid((n + 31) / 32, (k + 31) / 32), block(32, 8);
    transpose_kernel<float><<<grid, block, 0, s>>>(B, Bt, k, n, row_off, row_stride);
    JYC_LAUNCHED();
    return JYC_OK;
}
int launch_transpose_h(const uint16_t* B, uint16_t* Bt, int k, int n, int row_off, int row_stride,
                       cudaStream_t s) {
    if (k <= 0 || n <= 0) return arg_error("transpose: empty shape");
    dim3 grid((n + 31) / 32, (k + 31) / 32), block(32, 8);
    transpose_kernel<uint16_t><<<grid, block, 0, s>>>(B, Bt, k, n, row_off, row_stride);
    JYC_LAUNCHED();
    return JYC_OK;
}

// fp16 -> fp32, exact (wmat::row_to_f32: the embedding of an fp16 model).
__global__ void h2f_kernel(const uint16_t* h, float* f, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        f[i] = h2f(h[i]);
}
int launch_h2f(const uint16_t* h, float* f, size_t n, cudaStream_t s) {
    if (n == 0) return JYC_OK;
    const int blocks = (int)std::min<size_t>((n + 255) / 256, 148 * 16);
    h2f_kernel<<<blocks, 256, 0, s>>>(h, f, n);
    JYC_LAUNCHED();
    return JYC_OK;
}

// ---------------------------------------------------------------------------
// SiLU: the reference vectorises n/8*8 elements with its own exp and finishes
// the tail with libm expf (silu/x86/x86_classic.txt:11-31).
__global__ void silu_kernel(const float* x, float* y, int n) {
    const int nv = n / 8 * 8;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float v = x[i];
        y[i] = i < nv ? silu_ref(v) : __fdiv_rn(v, __fadd_rn(1.0f, expf(-v)));
    }
}
int launch_silu(const float* x, float* y, int n, cudaStream_t s) {
    if (n <= 0) return JYC_OK;
    silu_kernel<<<std::min((n + 255) / 256, 148 * 8), 256, 0, s>>>(x, y, n);
    JYC_LAUNCHED();
    return JYC_OK;
}

// kv_pack_q8 over `n` rows x `heads` heads, contiguous [n][heads][hd].
__global__ void kv_pack_kernel(const float* src, int8_t* dst, float* sc, int heads, int hd, int units) {
    const int lane = threadIdx.x & 31;
    const int u = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (u >= units) return;
    const float* s = src + (size_t)u * hd;
    int8_t* d = dst + (size_t)u * hd;
    float amax = 0.0f;
    for (int e = lane; e < hd; e += 32) amax = fmaxf(amax, fabsf(s[e]));
    amax = warp_max(amax);
    const float inv = q8_inv(amax);
    if (lane == 0) sc[u] = q8_scale(amax);
    for (int e = lane; e < hd; e += 32) d[e] = (int8_t)q8_round(s[e], inv);
}
int launch_kv_pack(const float* src, int8_t* dst, float* sc, int heads, int hd, int n,
                   cudaStream_t s) {
    const int units = n * heads;
    if (units <= 0) return JYC_OK;
    kv_pack_kernel<<<(units + 3) / 4, 128, 0, s>>>(src, dst, sc, heads, hd, units);
    JYC_LAUNCHED();
    return JYC_OK;
}

// ---------------------------------------------------------------------------
__global__ void argmax_kernel(const float* v, int n, unsigned long long* slot) {
    unsigned long long best = 0ull;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const unsigned long long p = argmax_pack(v[i], i);
        best = p > best ? p : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long q = __shfl_xor_sync(0xffffffffu, best, o);
        best = q > best ? q : best;
    }
    if ((threadIdx.x & 31) == 0 && best) atomicMax(slot, best);
}
__global__ void argmax_finish_kernel(unsigned long long* slot, int* out) {
    const unsigned long long p = *slot;
    *out = p ? argmax_index(p) : 0;
    *slot = 0ull;
}
int launch_argmax(const float* v, int n, unsigned long long* slot, int* out, cudaStream_t s) {
    if (n <= 0) return arg_error("argmax: n must be positive");
    argmax_kernel<<<std::min((n + 255) / 256, 148 * 4), 256, 0, s>>>(v, n, slot);
    JYC_LAUNCHED();
    argmax_finish_kernel<<<1, 1, 0, s>>>(slot, out);
    JYC_LAUNCHED();
    return JYC_OK;
}

// ---------------------------------------------------------------------------
// General C = A . Bt^T for any shape, fp32 or fp16 weights (op entry points;
// the model path uses the GEMV kernel). 32x32 tiles, fp32 FMA.
static __device__ __forceinline__ float w_to_f32(float w) { return w; }
static __device__ __forceinline__ float w_to_f32(uint16_t w) { return h2f(w); }
template <typename T>
__global__ void matmul_f32_kernel(const float* A, const T* Bt, float* C, int m, int n, int k) {
    __shared__ float as[32][33], bs[32][33];
    const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
    const int row0 = blockIdx.y * 32, col0 = blockIdx.x * 32;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int p0 = 0; p0 < k; p0 += 32) {
        for (int j = ty; j < 32; j += 8) {
            const int r = row0 + j, p = p0 + tx;
            as[j][tx] = (r < m && p < k) ? A[(size_t)r * k + p] : 0.0f;
            const int c = col0 + j;
            bs[j][tx] = (c < n && p < k) ? w_to_f32(Bt[(size_t)c * k + p]) : 0.0f;
        }
        __syncthreads();
#pragma unroll 8
        for (int p = 0; p < 32; p++) {
            const float b = bs[tx][p];
#pragma unroll
            for (int q = 0; q < 4; q++) acc[q] = __fmaf_rn(as[ty + 8 * q][p], b, acc[q]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int q = 0; q < 4; q++) {
        const int r = row0 + ty + 8 * q, c = col0 + tx;
        if (r < m && c < n) C[(size_t)r * n + c] = acc[q];
    }
}
int launch_matmul_f32_generic(const float* A, const float* Bt, float* C, int m, int n, int k,
                              cudaStream_t s) {
    dim3 grid((n + 31) / 32, (m + 31) / 32), block(32, 8);
    matmul_f32_kernel<float><<<grid, block, 0, s>>>(A, Bt, C, m, n, k);
    JYC_LAUNCHED();
    return JYC_OK;
}
int launch_matmul_f16_generic(const float* A, const uint16_t* Bt, float* C, int m, int n, int k,
                              cudaStream_t s) {
    dim3 grid((n + 31) / 32, (m + 31) / 32), block(32, 8);
    matmul_f32_kernel<uint16_t><<<grid, block, 0, s>>>(A, Bt, C, m, n, k);
    JYC_LAUNCHED();
    return JYC_OK;
}

// ---------------------------------------------------------------------------
__global__ void set_state_kernel(DevState* st, int len, int max_new, int max_len, int n_eos,
                                 int e0, int e1, int e2, int e3, int e4, int e5, int e6, int e7) {
    st->len = len;
    st->steps = 0;
    st->max_new = max_new;
    st->max_len = max_len;
    st->active = 1;
    st->n_eos = n_eos;
    const int e[8] = {e0, e1, e2, e3, e4, e5, e6, e7};
    for (int i = 0; i < 8; i++) st->eos[i] = e[i];
    st->amax = 0ull;
    st->head_arrive = 0u;
    st->fresh = 0;
    st->temperature = 0.0f;  // greedy until generate asks for its sampler
    st->penalty = 1.0f;
    st->rng = 12345u;
    st->prompt_len = len;
}
__global__ void set_sampling_kernel(DevState* st, float temperature, float penalty, unsigned int rng,
                                    int prompt_len) {
    st->temperature = temperature;
    st->penalty = penalty;
    st->rng = rng;
    st->prompt_len = prompt_len;
}
int launch_set_sampling(DevState* st, float temperature, float penalty, unsigned int rng, int prompt_len,
                        cudaStream_t s) {
    set_sampling_kernel<<<1, 1, 0, s>>>(st, temperature, penalty, rng, prompt_len);
    JYC_LAUNCHED();
    return JYC_OK;
}

// Sampling on a path whose head picked greedily (prefill, the per-op decode
// step): pick the appended token again from the same logits (in place) with
// the step's sampler and redo the stop test (generate.h:78-86).
__global__ void __launch_bounds__(kSampleThreads) resample_last_kernel(DevState* st, float* logits,
                                                                       unsigned int* stag, int V, int* tokens) {
    __shared__ double scratch[kSampleThreads + 1];
    if (!st->fresh) return;  // the step appended no token
    const int len = st->len;  // the new token sits at len - 1
    unsigned int rng = st->rng;
    const int next = sample_block(logits, V, st->temperature, st->penalty, tokens, st->prompt_len, len - 1, &rng,
                                  scratch, stag);
    if (threadIdx.x == 0) {
        tokens[len - 1] = next;
        st->rng = rng;
        bool stop = len >= st->max_len || st->steps >= st->max_new;
        for (int e = 0; e < st->n_eos; e++)
            if (next == st->eos[e]) stop = true;
        st->active = stop ? 0 : 1;
        st->fresh = 0;
    }
}
int launch_resample_last(DevState* st, float* logits, unsigned int* stag, int V, int* tokens, cudaStream_t s) {
    resample_last_kernel<<<1, kSampleThreads, 0, s>>>(st, logits, stag, V, tokens);
    JYC_LAUNCHED();
    return JYC_OK;
}

__global__ void __launch_bounds__(kSampleThreads) sample_kernel(float* logits, int V, float temperature,
                                                                float penalty, const int* ids, int prompt_len,
                                                                int len, unsigned int* rng, int* out) {
    __shared__ double scratch[kSampleThreads + 1];
    unsigned int r = *rng;
    const int next = sample_block(logits, V, temperature, penalty, ids, prompt_len, len, &r, scratch, nullptr);
    if (threadIdx.x == 0) {
        *out = next;
        *rng = r;
    }
}
int launch_sample(float* logits, int V, float temperature, float penalty, const int* ids, int prompt_len, int len,
                  unsigned int* rng_dev, int* out_dev, cudaStream_t s) {
    sample_kernel<<<1, kSampleThreads, 0, s>>>(logits, V, temperature, penalty, ids, prompt_len, len, rng_dev,
                                               out_dev);
    JYC_LAUNCHED();
    return JYC_OK;
}

int launch_set_state(DevState* st, int len, int max_new, int max_len, const int* eos, int n_eos,
                     cudaStream_t s) {
    if (n_eos > 8) return arg_error("generate: at most 8 EOS ids are supported");
    int e[8] = {-1, -1, -1, -1, -1, -1, -1, -1};
    for (int i = 0; i < n_eos; i++) e[i] = eos[i];
    set_state_kernel<<<1, 1, 0, s>>>(st, len, max_new, max_len, n_eos, e[0], e[1], e[2], e[3], e[4],
                                     e[5], e[6], e[7]);
    JYC_LAUNCHED();
    return JYC_OK;
}

}  // namespace jyc
