// skinny.cu — Q8_0 matmul over 1..8 activation rows (see skinny.cuh).
#include <mutex>

#include "skinny.cuh"

namespace jyc {

namespace {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kSkMaxRW = 16;  // weight rows per warp unit at most
constexpr int kSkThreads = kSkWarps * 32;
constexpr int kSkSmemMax = kSkMaxRows * kSkSlice * 4 + kSkWarps * kSkMaxRW * (kSkSlice + 32);
static_assert(kSkThreads == kSkSlice / 4, "one 16-byte column group of the slice per thread");

__device__ __forceinline__ void sk_cp16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src)
                 : "memory");
}

// 4 bytes u = q+128 -> 4 exact floats q as two pairs (float bits
// 0x4B0000uu = 2^23 + uu, minus 2^23 + 128 with one packed add per pair)
__device__ __forceinline__ void sk_u8x4(uint32_t w, float2& a, float2& b) {
    const float2 bias = make_float2(-8388736.0f, -8388736.0f);  // -(2^23 + 128)
    a = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540u)),
                               __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7541u))), bias);
    b = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7542u)),
                               __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7543u))), bias);
}

// sc[t] = 1 / sqrt(mean(x[t]^2) + eps), the reference rmsnorm's scale
// (rmsnorm/x86/x86_classic.txt:1-27; the sum of squares is a tree here).
__global__ void __launch_bounds__(256) sk_rowscale_kernel(const float* x, int ldx, int k, float eps, float* sc) {
    __shared__ float red[8];
    const float* xr = x + (size_t)blockIdx.x * ldx;
    float ss = 0.0f;
#pragma unroll 4
    for (int i = threadIdx.x * 4; i < k; i += 256 * 4) {  // k % 32 == 0, rows 16-byte aligned
        const float4 v = __ldg(reinterpret_cast<const float4*>(xr + i));
        ss = __fmaf_rn(v.x, v.x, ss);
        ss = __fmaf_rn(v.y, v.y, ss);
        ss = __fmaf_rn(v.z, v.z, ss);
        ss = __fmaf_rn(v.w, v.w, ss);
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.0f;
        for (int i = 0; i < 8; i++) t += red[i];
        const float den = __fadd_rn(__fdiv_rn(t, (float)k), eps);
        sc[blockIdx.x] = den <= 0.0f ? 0.0f : __fdiv_rn(1.0f, __fsqrt_rn(den));
    }
}

// Output (row, t) of the matmul with its epilogue; lanes holding row+1 of the
// same activation row sit MT lanes higher (SwiGLU pairs rows 2j, 2j+1).
template <int MT, int EPI>
__device__ __forceinline__ void sk_store(const SkinnyGemm& g, int row, int t, bool even, float v) {
    if (EPI == EPI_SWIGLU) {
        const float up = __shfl_down_sync(kFull, v, MT);
        if (even && row + 1 < g.n && t < g.m) g.y[(size_t)t * g.ldy + (row >> 1)] = __fmul_rn(silu_ref(v), up);
    } else if (row < g.n && t < g.m) {
        float* yp = g.y + (size_t)t * g.ldy + row;
        if (EPI == EPI_BIAS) v = __fadd_rn(v, g.bias[row]);
        if (EPI == EPI_RESID) v = __fadd_rn(*yp, v);
        *yp = v;
    }
}

// grid (row units / kSkWarps, K slices); warp w of CTA (bx, slice) owns rows
// [(bx*kSkWarps + w)*RW, +RW) x columns [slice*512, +512).
template <int MT, int EPI>
__global__ void __launch_bounds__(kSkThreads, MT <= 4 ? 3 : 2)
    skinny_kernel(SkinnyGemm g, SkinnyWork w, int RW, int npad, int nslices) {
    constexpr int G = 32 / MT;  // weight rows per butterfly (G x MT = 32 sums)
    extern __shared__ __align__(16) unsigned char sk_smem[];
    float4* xs = reinterpret_cast<float4*>(sk_smem);                        // [MT][4 quads][32 lanes]
    uint8_t* wring = sk_smem + MT * kSkSlice * 4;                           // [warps][RW][512]
    uint16_t* sring = reinterpret_cast<uint16_t*>(wring + kSkWarps * RW * kSkSlice);  // [warps][RW][16]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int slice = blockIdx.y, c0 = slice * kSkSlice;
    const int unit = blockIdx.x * kSkWarps + warp;
    const int row0 = unit * RW;
    const int n = g.n, k = g.k;
    const bool cols = c0 + lane * 16 < k;  // k % 32 == 0: a lane's 16 columns all exist or none
    uint8_t* wr = wring + (size_t)warp * RW * kSkSlice;
    uint16_t* sr = sring + (size_t)warp * RW * 16;

    // 1. the warp's weight rows of the slice, in flight while the rest loads
    if (row0 < n && cols) {
        const uint8_t* src = g.qs + (size_t)row0 * k + c0 + lane * 16;
        const int rows = min(RW, n - row0);
        for (int r = 0; r < rows; r++) sk_cp16(wr + r * kSkSlice + lane * 16, src + (size_t)r * k);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    if (row0 < n) {  // scales [RW][16]: all of a lane's loads issued before the first store
        const int kb = k >> 5, b0 = c0 >> 5;
        uint16_t sv[kSkMaxRW / 2];
#pragma unroll
        for (int i = 0; i < kSkMaxRW / 2; i++) {
            const int e = lane + 32 * i, r = e >> 4, b = e & 15;
            sv[i] = (r < RW && row0 + r < n && b0 + b < kb) ? __ldg(g.d + (size_t)(row0 + r) * kb + b0 + b) : 0;
        }
#pragma unroll
        for (int i = 0; i < kSkMaxRW / 2; i++)
            if (lane + 32 * i < RW * 16) sr[lane + 32 * i] = sv[i];
    }
    // 2. the slice of every activation row (RMSNorm applied), lane-major
    // quads: thread f holds columns [4f, 4f+4) of the slice for every row
    {
        const int f = threadIdx.x, c = c0 + f * 4;
        const bool in = c < k;
        float4 v[MT];
#pragma unroll
        for (int t = 0; t < MT; t++)
            v[t] = (in && t < g.m) ? __ldg(reinterpret_cast<const float4*>(g.x + (size_t)t * g.ldx + c))
                                   : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (g.norm_w != nullptr && in) {
            const float4 nw = __ldg(reinterpret_cast<const float4*>(g.norm_w + c));
#pragma unroll
            for (int t = 0; t < MT; t++) {
                const float s = t < g.m ? w.sc[t] : 0.0f;
                v[t].x = __fmul_rn(__fmul_rn(v[t].x, s), nw.x);
                v[t].y = __fmul_rn(__fmul_rn(v[t].y, s), nw.y);
                v[t].z = __fmul_rn(__fmul_rn(v[t].z, s), nw.z);
                v[t].w = __fmul_rn(__fmul_rn(v[t].w, s), nw.w);
            }
        }
#pragma unroll
        for (int t = 0; t < MT; t++) xs[(t * 4 + (f & 3)) * 32 + (f >> 2)] = v[t];
    }
    __syncthreads();
    if (row0 >= n) return;

    float2 xv[MT][8];
#pragma unroll
    for (int t = 0; t < MT; t++)
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const float4 v = xs[(t * 4 + q) * 32 + lane];
            xv[t][q * 2 + 0] = make_float2(v.x, v.y);
            xv[t][q * 2 + 1] = make_float2(v.z, v.w);
        }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncwarp();

    const int nrows = min(RW, n - row0);
    for (int gi = 0; gi * G < nrows; gi++) {
        float a[32];  // a[gg * MT + t]: this lane's 16-column partial of row gi*G+gg, activation row t
#pragma unroll
        for (int gg = 0; gg < G; gg++) {
            const int r = gi * G + gg;
            const uint4 wq = *reinterpret_cast<const uint4*>(wr + r * kSkSlice + lane * 16);
            const float dsc = (cols && r < nrows) ? h2f(sr[r * 16 + (lane >> 1)]) : 0.0f;
            float2 wf[8];
            sk_u8x4(wq.x, wf[0], wf[1]);
            sk_u8x4(wq.y, wf[2], wf[3]);
            sk_u8x4(wq.z, wf[4], wf[5]);
            sk_u8x4(wq.w, wf[6], wf[7]);
#pragma unroll
            for (int t = 0; t < MT; t++) {
                float2 s2 = make_float2(0.0f, 0.0f);  // even / odd columns
#pragma unroll
                for (int i = 0; i < 8; i++) s2 = __ffma2_rn(wf[i], xv[t][i], s2);
                a[gg * MT + t] = __fmul_rn(__fadd_rn(s2.x, s2.y), dsc);
            }
        }
        // transposing butterfly: after it, lane l holds the warp sum of a[l]
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) {
            const bool up = (lane & o) != 0;
#pragma unroll
            for (int j = 0; j < o; j++) {
                const float send = up ? a[j] : a[j + o];
                const float keep = up ? a[j + o] : a[j];
                a[j] = __fadd_rn(keep, __shfl_xor_sync(kFull, send, o));
            }
        }
        const int gg = lane / MT, t = lane % MT;
        const int row = row0 + gi * G + gg;
        if (nslices == 1)
            sk_store<MT, EPI>(g, row, t, (gg & 1) == 0, a[0]);
        else
            w.part[((size_t)slice * npad + row) * MT + t] = a[0];
    }
    if (nslices == 1) return;

    // 3. the last slice to finish this row unit sums the slices in order
    __threadfence();
    __syncwarp();
    unsigned int prev = 0;
    if (lane == 0) prev = atomicAdd(&w.cnt[unit], 1u);
    prev = __shfl_sync(kFull, prev, 0);
    if (prev != (unsigned int)(nslices - 1)) return;
    __threadfence();
    for (int j0 = 0; j0 < RW * MT; j0 += 32) {
        const int j = j0 + lane;
        float acc = 0.0f;
        for (int s2 = 0; s2 < nslices; s2++)
            acc = __fadd_rn(acc, __ldcg(w.part + ((size_t)s2 * npad + row0) * MT + j));
        sk_store<MT, EPI>(g, row0 + j / MT, j % MT, ((j / MT) & 1) == 0, acc);
    }
    if (lane == 0) w.cnt[unit] = 0u;
}

template <int MT, int EPI>
int sk_prepare_one() {
    JYC_CUDA(cudaFuncSetAttribute(skinny_kernel<MT, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSkSmemMax));
    return JYC_OK;
}

template <int MT>
int sk_prepare_mt() {
    int r = sk_prepare_one<MT, EPI_STORE>();
    if (r == JYC_OK) r = sk_prepare_one<MT, EPI_BIAS>();
    if (r == JYC_OK) r = sk_prepare_one<MT, EPI_RESID>();
    if (r == JYC_OK) r = sk_prepare_one<MT, EPI_SWIGLU>();
    return r;
}

template <int MT>
int sk_launch_mt(const SkinnyGemm& g, int epi, const SkinnyWork& w, dim3 grid, size_t smem, int RW, int npad,
                 int nslices, cudaStream_t s) {
    switch (epi) {
        case EPI_STORE: skinny_kernel<MT, EPI_STORE><<<grid, kSkThreads, smem, s>>>(g, w, RW, npad, nslices); break;
        case EPI_BIAS: skinny_kernel<MT, EPI_BIAS><<<grid, kSkThreads, smem, s>>>(g, w, RW, npad, nslices); break;
        case EPI_RESID: skinny_kernel<MT, EPI_RESID><<<grid, kSkThreads, smem, s>>>(g, w, RW, npad, nslices); break;
        case EPI_SWIGLU: skinny_kernel<MT, EPI_SWIGLU><<<grid, kSkThreads, smem, s>>>(g, w, RW, npad, nslices); break;
        default: return arg_error("skinny: unsupported epilogue");
    }
    JYC_LAUNCHED();
    return JYC_OK;
}

}  // namespace

size_t skinny_part_floats(int n, int k) {
    const size_t nslices = (size_t)(k + kSkSlice - 1) / kSkSlice;
    return nslices > 1 ? nslices * (size_t)(n + kSkMaxRW) * kSkMaxRows : 1;
}

size_t skinny_counters(int n) { return (size_t)n / 4 + 2; }

int prepare_skinny_kernels() {
    static std::once_flag once;
    static int result = JYC_OK;
    std::call_once(once, [] {
        result = sk_prepare_mt<2>();
        if (result == JYC_OK) result = sk_prepare_mt<4>();
        if (result == JYC_OK) result = sk_prepare_mt<8>();
    });
    return result;
}

int launch_skinny(const SkinnyGemm& g, int epi, const SkinnyWork& w, cudaStream_t s) {
    if (g.m < 1 || g.m > kSkMaxRows) return arg_error("skinny: m must be in [1, 8]");
    if (g.n <= 0 || g.k <= 0 || g.k % 32) return arg_error("skinny: need n > 0, k > 0 and k % 32 == 0");
    if (!g.x || !g.qs || !g.d || !g.y) return arg_error("skinny: null pointer");
    if ((g.ldx & 3) || ((uintptr_t)g.x & 15) || (g.norm_w && ((uintptr_t)g.norm_w & 15)) || ((uintptr_t)g.qs & 15))
        return arg_error("skinny: activations, norm weights and weights must be 16-byte aligned rows");
    if (epi == EPI_BIAS && !g.bias) return arg_error("skinny: bias epilogue without bias");
    if (epi == EPI_SWIGLU && (g.n & 1)) return arg_error("skinny: SwiGLU needs an even row count");
    if (const int pr = prepare_skinny_kernels()) return pr;
    const int MT = g.m <= 2 ? 2 : g.m <= 4 ? 4 : 8;
    const int G = 32 / MT;
    const int nslices = (g.k + kSkSlice - 1) / kSkSlice;
    if (nslices > 1 && (!w.part || !w.cnt)) return arg_error("skinny: split-K workspace missing");
    if (g.norm_w && !w.sc) return arg_error("skinny: RMSNorm scale buffer missing");
    // the largest unit that still fills every SM's CTA slots (fewer rows per
    // unit on short matrices)
    const int slots = 148 * (MT <= 4 ? 3 : 2);
    int RW = G;
    for (int cand = kSkMaxRW; cand >= G; cand >>= 1) {
        const long long ctas = (long long)((g.n + kSkWarps * cand - 1) / (kSkWarps * cand)) * nslices;
        if (ctas >= slots) {
            RW = cand;
            break;
        }
    }
    const int units = (g.n + RW - 1) / RW;
    const dim3 grid((units + kSkWarps - 1) / kSkWarps, nslices);
    const size_t smem = (size_t)MT * kSkSlice * 4 + (size_t)kSkWarps * RW * (kSkSlice + 32);
    if (g.norm_w) {
        sk_rowscale_kernel<<<g.m, 256, 0, s>>>(g.x, g.ldx, g.k, g.eps, w.sc);
        JYC_LAUNCHED();
    }
    const int npad = units * RW;
    if (MT == 2) return sk_launch_mt<2>(g, epi, w, grid, smem, RW, npad, nslices, s);
    if (MT == 4) return sk_launch_mt<4>(g, epi, w, grid, smem, RW, npad, nslices, s);
    return sk_launch_mt<8>(g, epi, w, grid, smem, RW, npad, nslices, s);
}

}  // namespace jyc
