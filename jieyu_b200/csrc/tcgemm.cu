// tcgemm.cu — tcgen05 GEMM of Q8_0 weights over token tiles (prefill and
// batched decode), see tcgemm.cuh for the numerics.
//
// CTA = 128 weight rows x N tokens x one range of K, 10 warps:
//   warp 0     allocates the tensor-memory accumulator (N fp32 columns) and
//              streams the token operand: one 1-D bulk copy (TMA) per 64-wide
//              K chunk brings its hi and lo planes, already in the 128-byte
//              swizzled K-major layout the MMA reads;
//   warp 1     one thread issues the MMAs: per 16-wide K step
//              D += Whi.Xhi + Whi.Xlo + Wlo.Xhi (tcgen05.mma kind::f16, fp32
//              accumulate, M=128, N tokens), then tcgen05.commit frees the
//              stage; the last commit signals the accumulator;
//   warps 2-9  converters: each thread dequantises one 32-weight block of one
//              row per chunk (q * d * 2^S exactly in fp32, split into fp16 hi
//              and lo), stores both into the swizzled A planes of the stage
//              and arrives on the stage's barrier; loads run 3 chunks ahead
//              in registers. After the K loop they are the epilogue: lanes of
//              tensor memory = weight rows, columns = tokens (tcgen05.ld),
//              unscaled by 2^-S_row 2^-s_token, then stored (+ bias, residual
//              or SwiGLU of interleaved gate/up rows). With K split over CTAs
//              each writes its partial tile and the last to arrive sums the
//              partials in split order (deterministic) and runs the epilogue.
// Every wait is bounded and reports error word 9.
#include <algorithm>

#include "mega.cuh"
#include "ptx.cuh"
#include "tcgemm.cuh"

namespace jyc {

namespace {

constexpr int kThreads = 320;
constexpr int kPlaneA = kTcRows * 128;  // one A plane (hi or lo) of a chunk: 128 rows x 128 bytes
constexpr int kSmemBudget = 200 * 1024;
constexpr int kErrTc = 9;

template <int N>
struct TcCfg {
    static constexpr int kPlaneB = N * 128;
    static constexpr int kStage = 2 * kPlaneA + 2 * kPlaneB;
    static constexpr int kStages = (kSmemBudget / kStage) > 4 ? 4 : (kSmemBudget / kStage);
    static constexpr int kCols = N < 32 ? 32 : N;  // tensor-memory columns: a power of two >= 32
    // alignment slack + stages + barriers + tmem slot/flag + row maxima
    static constexpr int kSmem = 1024 + kStages * kStage + 8 * (3 * kStages + 1) + 16 + 4 * kTcRows;
};

// ---- tcgen05 / tensor-memory helpers ---------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// D[tmem] (+)= A[smem] . B[smem]^T, fp16 inputs, fp32 accumulator
__device__ __forceinline__ void tc_mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// arrives once on `bar` when every MMA this thread issued so far has completed
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
// 8 consecutive fp32 columns of this warp's 32 tensor-memory lanes
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float* v) {
    uint32_t r0, r1, r2, r3, r4, r5, r6, r7;
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3), "=r"(r4), "=r"(r5), "=r"(r6), "=r"(r7)
        : "r"(taddr)
        : "memory");
    v[0] = __uint_as_float(r0); v[1] = __uint_as_float(r1); v[2] = __uint_as_float(r2); v[3] = __uint_as_float(r3);
    v[4] = __uint_as_float(r4); v[5] = __uint_as_float(r5); v[6] = __uint_as_float(r6); v[7] = __uint_as_float(r7);
}
// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (stride byte offset), sm_100 descriptor version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) | ((uint64_t)(1024u >> 4) << 32) |
           ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}
// Instruction descriptor of kind::f16: fp32 accumulator, fp16 A and B, both
// K-major, M = 128, N tokens.
template <int N>
__device__ __forceinline__ constexpr uint32_t idesc_f16() {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(kTcRows >> 4) << 24);
}
__device__ __forceinline__ void named_sync_conv() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
// 2^e for e in [-126, 127], exactly
__device__ __forceinline__ float exp2i(int e) { return __int_as_float((e + 127) << 23); }
__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
// copy without an L2 hint (the token planes are re-read by every row tile)
__device__ __forceinline__ void bulk_g2s_keep(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
// 8 fp32 values (already scaled) -> 16 bytes of fp16 hi and 16 bytes of lo
__device__ __forceinline__ void split8(const float* f, uint4& hi, uint4& lo) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const __half2 hh = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
        const float2 hf = __half22float2(hh);
        h[i] = h2u(hh);
        l[i] = h2u(__floats2half2_rn(__fsub_rn(f[2 * i], hf.x), __fsub_rn(f[2 * i + 1], hf.y)));
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
}

template <int N, int EPI>
__global__ void __launch_bounds__(kThreads, 1) tc_gemm_kernel(TcGemm p) {
    using C = TcCfg<N>;
    extern __shared__ unsigned char tc_smraw[];
    // the 128-byte swizzle is a function of the address bits: 1024-byte aligned tiles
    unsigned char* sm = tc_smraw + ((1024u - (smem_u32(tc_smraw) & 1023u)) & 1023u);
    uint64_t* afull = reinterpret_cast<uint64_t*>(sm + C::kStages * C::kStage);  // converters done (256 arrivals)
    uint64_t* bfull = afull + C::kStages;                                         // token planes landed (tx)
    uint64_t* empty = bfull + C::kStages;                                         // MMAs of the stage done
    uint64_t* accf = empty + C::kStages;                                          // accumulator complete
    uint32_t* s_tmem = reinterpret_cast<uint32_t*>(accf + 1);
    unsigned int* s_flag = s_tmem + 1;
    unsigned int* s_rmax = s_tmem + 4;  // [128] max |d| (fp16 magnitude bits) per row

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int mt = blockIdx.x, tt = blockIdx.y, z = blockIdx.z;
    const int nkc = (p.k + kTcKC - 1) / kTcKC;
    const int per = (nkc + p.splits - 1) / p.splits;
    const int c0 = z * per, nch = min(nkc, c0 + per) - c0;  // the host plan leaves no split empty

    if (tid == 0) {
        for (int s = 0; s < C::kStages; s++) {
            mbar_init(&afull[s], 256);
            mbar_init(&bfull[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accf, 1);
        mbar_fence_init();
    }
    if (tid >= 64 && tid < 64 + kTcRows) s_rmax[tid - 64] = 0u;
    if (warp == 0) {
        __syncwarp();
        tmem_alloc(s_tmem, C::kCols);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *s_tmem;

    if (warp == 0) {
        if (lane == 0) {
            const unsigned char* src =
                reinterpret_cast<const unsigned char*>(p.xs) + ((size_t)tt * nkc + c0) * 2 * C::kPlaneB;
            int issued = 0;
            for (int j = 0; j < nch; j++) {
                const int s = j % C::kStages;
                if (j >= C::kStages && !mbar_wait_err(&empty[s], ((j / C::kStages) - 1) & 1, p.err, kErrTc)) break;
                mbar_expect_tx(&bfull[s], 2 * C::kPlaneB);
                bulk_g2s_keep(sm + s * C::kStage + 2 * kPlaneA, src + (size_t)j * 2 * C::kPlaneB, 2 * C::kPlaneB,
                              &bfull[s]);
                issued = j + 1;
            }
            // no copy may still be landing when the CTA exits (matters only after an error)
            for (int j = max(0, issued - C::kStages); j < issued; j++)
                mbar_wait_err(&bfull[j % C::kStages], (j / C::kStages) & 1, p.err, kErrTc);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16<N>();
            for (int j = 0; j < nch; j++) {
                const int s = j % C::kStages;
                const uint32_t ph = (j / C::kStages) & 1;
                if (!mbar_wait_err(&afull[s], ph, p.err, kErrTc) || !mbar_wait_err(&bfull[s], ph, p.err, kErrTc))
                    break;
                tc_fence_after();
                const uint32_t st = smem_u32(sm + s * C::kStage);
                const uint64_t ah = sw128_desc(st), al = sw128_desc(st + kPlaneA);
                const uint64_t bh = sw128_desc(st + 2 * kPlaneA), bl = sw128_desc(st + 2 * kPlaneA + C::kPlaneB);
#pragma unroll
                for (int ks = 0; ks < kTcKC / 16; ks++) {
                    const uint64_t o = 2 * ks;  // 32 bytes further along K, in 16-byte units
                    tc_mma_f16(tmem, ah + o, bh + o, idesc, (j | ks) != 0);
                    tc_mma_f16(tmem, ah + o, bl + o, idesc, 1u);
                    tc_mma_f16(tmem, al + o, bh + o, idesc, 1u);
                }
                tc_commit(&empty[s]);
            }
            tc_commit(accf);  // also after an error: the epilogue waits on it
        }
    } else {
        // ---------------- converters ----------------
        const int ct = tid - 64, cw = ct >> 5;
        const int r = 32 * (cw & 3) + lane, h = cw >> 2;  // tile row, which 32-block of the chunk
        const int R = mt * kTcRows + r;
        const bool rv = R < p.n;
        const int nb = p.k >> 5;
        const uint8_t* qrow = p.qs + (size_t)(rv ? R : 0) * p.k;
        const uint16_t* drow = p.d + (size_t)(rv ? R : 0) * nb;
        {
            unsigned int mx = 0u;
            if (rv) {
                const int bend = min(nb, 2 * (c0 + nch));
                for (int b = 2 * c0 + h; b < bend; b += 2) mx = max(mx, (unsigned int)(__ldg(drow + b) & 0x7FFFu));
            }
            atomicMax(&s_rmax[r], mx);
        }
        named_sync_conv();
        // rows scaled by 2^S with S = 22 - exponent field of max |d|: 127 max|d| 2^S < 2^15
        const float rup = exp2i(22 - (int)(s_rmax[r] >> 10));
        uint4 qa[4][2];
        uint16_t dd[4];
        auto load = [&](int j, uint4* q, uint16_t& dv) {
            const int kb = 2 * (c0 + j) + h;
            if (rv && kb < nb) {
                const uint4* src = reinterpret_cast<const uint4*>(qrow + (size_t)kb * 32);
                q[0] = __ldg(src);
                q[1] = __ldg(src + 1);
                dv = __ldg(drow + kb);
            } else {
                q[0] = q[1] = make_uint4(0x80808080u, 0x80808080u, 0x80808080u, 0x80808080u);
                dv = 0;
            }
        };
        bool ok = true;
        auto convert = [&](int j, const uint4* q, uint16_t dv) {
            const int s = j % C::kStages;
            if (j >= C::kStages && ok && !mbar_wait_err(&empty[s], ((j / C::kStages) - 1) & 1, p.err, kErrTc))
                ok = false;
            unsigned char* ah = sm + s * C::kStage + r * 128;
            const float ds = __fmul_rn(h2f(dv), rup);
            const uint32_t* w = reinterpret_cast<const uint32_t*>(q);
#pragma unroll
            for (int c = 0; c < 4; c++) {
                float f[8];
                u8x4_to_f32(w[2 * c], f);
                u8x4_to_f32(w[2 * c + 1], f + 4);
#pragma unroll
                for (int i = 0; i < 8; i++) f[i] = __fmul_rn(f[i], ds);
                uint4 hi, lo;
                split8(f, hi, lo);
                const int pos = ((4 * h + c) ^ (r & 7)) * 16;
                *reinterpret_cast<uint4*>(ah + pos) = hi;
                *reinterpret_cast<uint4*>(ah + kPlaneA + pos) = lo;
            }
            fence_proxy_async_smem();
            mbar_arrive(&afull[s]);
        };
        if (nch > 0) load(0, qa[0], dd[0]);
        if (nch > 1) load(1, qa[1], dd[1]);
        if (nch > 2) load(2, qa[2], dd[2]);
        for (int j0 = 0; j0 < nch; j0 += 4) {
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int j = j0 + u;
                if (j < nch) {
                    if (j + 3 < nch) load(j + 3, qa[(u + 3) & 3], dd[(u + 3) & 3]);
                    convert(j, qa[u], dd[u]);
                }
            }
        }

        // ---------------- epilogue ----------------
        mbar_wait_err(accf, 0, p.err, kErrTc);
        tc_fence_after();
        constexpr int CH = N / 2;  // columns (tokens) per warp: two warps share a lane quadrant
        const int q4 = warp & 3, half = (warp - 2) >> 2;
        const int re = 32 * q4 + lane, Re = mt * kTcRows + re;
        const bool rev = Re < p.n;
        const float rdown = exp2i((int)(s_rmax[re] >> 10) - 22);
        const int t0 = tt * N + half * CH;
        const uint32_t tq = tmem + ((uint32_t)(32 * q4) << 16) + (uint32_t)(half * CH);
        // final values of 8 columns -> output (bias / residual / SwiGLU)
        auto store8 = [&](int c, const float* v) {
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int t = t0 + c + i;
                const bool ok_t = t < p.T;
                if (EPI == TC_SWIGLU) {
                    // rows 2j (gate) and 2j+1 (up) sit in adjacent lanes
                    const float upv = __shfl_down_sync(0xffffffffu, v[i], 1);
                    if ((lane & 1) == 0 && rev && ok_t)
                        p.y[(size_t)t * p.ldy + (Re >> 1)] = __fmul_rn(silu_ref(v[i]), upv);
                } else if (rev && ok_t) {
                    float* yp = p.y + (size_t)t * p.ldy + Re;
                    if (EPI == TC_STORE) *yp = v[i];
                    if (EPI == TC_BIAS) *yp = __fadd_rn(v[i], __ldg(p.bias + Re));
                    if (EPI == TC_RESID) *yp = __fadd_rn(*yp, v[i]);
                }
            }
        };
        // accumulator columns c..c+7, unscaled by 2^-S_row 2^-s_token
        auto load8 = [&](int c, float* v) {
            tmem_ld8(tq + (uint32_t)c, v);
#pragma unroll
            for (int i = 0; i < 8; i++) v[i] = __fmul_rn(__fmul_rn(v[i], rdown), exp2i(-__ldg(p.xe + t0 + c + i)));
        };
        if (p.splits == 1) {
#pragma unroll 1
            for (int c = 0; c < CH; c += 8) {
                float v[8];
                load8(c, v);
                store8(c, v);
            }
        } else {
#pragma unroll 1
            for (int c = 0; c < CH; c += 8) {
                float v[8];
                load8(c, v);
#pragma unroll
                for (int i = 0; i < 8; i++)
                    if (rev && t0 + c + i < p.T) p.part[((size_t)z * p.T + t0 + c + i) * p.n + Re] = v[i];
            }
            __threadfence();
            named_sync_conv();
            if (ct == 0) {
                const unsigned int old = atomicAdd(&p.cnt[mt * gridDim.y + tt], 1u);
                *s_flag = (old == (unsigned int)(p.splits - 1)) ? 1u : 0u;
            }
            named_sync_conv();
            if (*s_flag != 0u) {  // last of the tile's splits: sum them in split order
                __threadfence();
#pragma unroll 1
                for (int c = 0; c < CH; c += 8) {
                    float v[8];
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        float sum = 0.0f;
                        if (rev && t0 + c + i < p.T)
                            for (int zz = 0; zz < p.splits; zz++)
                                sum = __fadd_rn(sum, __ldcg(p.part + ((size_t)zz * p.T + t0 + c + i) * p.n + Re));
                        v[i] = sum;
                    }
                    store8(c, v);
                }
                if (ct == 0) p.cnt[mt * gridDim.y + tt] = 0u;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, C::kCols);
    }
}

// One token row -> optional RMSNorm -> power-of-two scale -> fp16 hi/lo in the
// swizzled tile layout: [token tile][chunk][hi, lo][N tokens][64 halves], the
// 16-byte chunk c of token row i stored at chunk c ^ (i & 7). Rows t >= T
// (tile padding) and columns >= k are zeros.
__global__ void __launch_bounds__(256) tc_split_kernel(const float* x, int ldx, int T, int k, const float* w,
                                                       float eps, int N, __half* xs, int* xe) {
    __shared__ float s_red[8];
    const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int tt = t / N, ti = t - tt * N, nkc = (k + kTcKC - 1) / kTcKC;
    const bool real = t < T;
    const float* xr = x + (size_t)(real ? t : 0) * ldx;
    float sc = 1.0f;
    if (real && w) {  // the RMSNorm of the decode and prefill paths
        float ss = 0.0f;
        for (int i = tid; i < k; i += 256) ss = __fmaf_rn(xr[i], xr[i], ss);
        ss = warp_sum(ss);
        if (lane == 0) s_red[warp] = ss;
        __syncthreads();
        float tsum = 0.0f;
        for (int i = 0; i < 8; i++) tsum += s_red[i];
        const float den = __fadd_rn(__fdiv_rn(tsum, (float)k), eps);
        sc = den <= 0.0f ? 0.0f : __fdiv_rn(1.0f, __fsqrt_rn(den));
        __syncthreads();  // s_red is reused below
    }
    auto load8 = [&](int i0, float* f) {
        if (!real || i0 >= k) {
#pragma unroll
            for (int e = 0; e < 8; e++) f[e] = 0.0f;
            return;
        }
        const float4 a = *reinterpret_cast<const float4*>(xr + i0);
        const float4 b = *reinterpret_cast<const float4*>(xr + i0 + 4);
        f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
        if (w) {
            const float4 wa = *reinterpret_cast<const float4*>(w + i0);
            const float4 wb = *reinterpret_cast<const float4*>(w + i0 + 4);
            const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
            for (int e = 0; e < 8; e++) f[e] = __fmul_rn(__fmul_rn(f[e], sc), wv[e]);
        }
    };
    float am = 0.0f;
    for (int c8 = tid; c8 < k / 8; c8 += 256) {
        float f[8];
        load8(c8 * 8, f);
#pragma unroll
        for (int e = 0; e < 8; e++) am = fmaxf(am, fabsf(f[e]));
    }
    am = warp_max(am);
    if (lane == 0) s_red[warp] = am;
    __syncthreads();
    am = 0.0f;
    for (int i = 0; i < 8; i++) am = fmaxf(am, s_red[i]);
    // 2^s with amax 2^s < 2^15 (exponent field ex: amax < 2^(ex-126))
    const int ex = (__float_as_int(am) >> 23) & 255;
    const int sx = am > 0.0f ? max(-100, min(100, 141 - ex)) : 0;
    const float up = exp2i(sx);
    if (tid == 0) xe[t] = sx;
    __half* base = xs + (size_t)tt * nkc * 2 * N * 64;
    for (int c8 = tid; c8 < nkc * 8; c8 += 256) {
        const int kc = c8 >> 3, c = c8 & 7;
        float f[8];
        load8(c8 * 8, f);
#pragma unroll
        for (int e = 0; e < 8; e++) f[e] = __fmul_rn(f[e], up);
        uint4 hi, lo;
        split8(f, hi, lo);
        __half* dst = base + ((size_t)kc * 2 * N + ti) * 64 + ((c ^ (ti & 7)) * 8);
        *reinterpret_cast<uint4*>(dst) = hi;
        *reinterpret_cast<uint4*>(dst + (size_t)N * 64) = lo;
    }
}

template <int N>
int set_smem() {
    using C = TcCfg<N>;
    static_assert(C::kSmem <= 227 * 1024, "tc_gemm shared memory");
    JYC_CUDA(cudaFuncSetAttribute(tc_gemm_kernel<N, TC_STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem));
    JYC_CUDA(cudaFuncSetAttribute(tc_gemm_kernel<N, TC_BIAS>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem));
    JYC_CUDA(cudaFuncSetAttribute(tc_gemm_kernel<N, TC_RESID>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem));
    JYC_CUDA(cudaFuncSetAttribute(tc_gemm_kernel<N, TC_SWIGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem));
    return JYC_OK;
}

template <int N>
int launch_n(const TcGemm& p, int epi, cudaStream_t s) {
    const dim3 grid((p.n + kTcRows - 1) / kTcRows, (p.T + N - 1) / N, p.splits);
    const int smem = TcCfg<N>::kSmem;
    switch (epi) {
        case TC_STORE: tc_gemm_kernel<N, TC_STORE><<<grid, kThreads, smem, s>>>(p); break;
        case TC_BIAS: tc_gemm_kernel<N, TC_BIAS><<<grid, kThreads, smem, s>>>(p); break;
        case TC_RESID: tc_gemm_kernel<N, TC_RESID><<<grid, kThreads, smem, s>>>(p); break;
        case TC_SWIGLU: tc_gemm_kernel<N, TC_SWIGLU><<<grid, kThreads, smem, s>>>(p); break;
        default: return arg_error("tc_gemm: epilogue");
    }
    JYC_LAUNCHED();
    return JYC_OK;
}

}  // namespace

int tc_token_tile(int T) { return T <= 16 ? 16 : T <= 32 ? 32 : T <= 64 ? 64 : 128; }

int tc_padded_tokens(int T, int N) { return (T + N - 1) / N * N; }

size_t tc_split_halves(int T, int N, int k) {
    const size_t nkc = (k + kTcKC - 1) / kTcKC;
    return (size_t)tc_padded_tokens(T, N) * nkc * 2 * kTcKC;
}

int tc_plan_splits(int n, int k, int T, int N, int max_splits) {
    const int tiles = ((n + kTcRows - 1) / kTcRows) * ((T + N - 1) / N);
    const int nkc = (k + kTcKC - 1) / kTcKC;
    const int sms = mega_num_ctas();
    int best = 1;
    double best_cost = 1e30;
    for (int s = 1; s <= std::min(max_splits, nkc); s++) {
        const int per = (nkc + s - 1) / s;
        const int eff = (nkc + per - 1) / per;  // no empty split
        if (eff != s) continue;
        const int waves = (tiles * s + sms - 1) / sms;
        // chunks of the slowest SM + a per-CTA fixed cost (~2 chunks) + the partial-sum pass
        const double cost = (double)waves * (per + 2) + (s > 1 ? 1.0 + 0.1 * s : 0.0);
        if (cost < best_cost - 1e-9) {
            best_cost = cost;
            best = s;
        }
    }
    return best;
}

int launch_tc_split(const float* x, int ldx, int T, int k, const float* norm_w, float eps, int N, __half* xs,
                    int* xe, cudaStream_t s) {
    if (T <= 0 || k <= 0 || k % 32 || ldx % 4) return arg_error("tc_split: k % 32, ldx % 4");
    if (N != 16 && N != 32 && N != 64 && N != 128) return arg_error("tc_split: token tile");
    tc_split_kernel<<<tc_padded_tokens(T, N), 256, 0, s>>>(x, ldx, T, k, norm_w, eps, N, xs, xe);
    JYC_LAUNCHED();
    return JYC_OK;
}

int prepare_tc_kernels() {
    static bool done = false;
    if (done) return JYC_OK;
    int r = set_smem<16>();
    if (r == JYC_OK) r = set_smem<32>();
    if (r == JYC_OK) r = set_smem<64>();
    if (r == JYC_OK) r = set_smem<128>();
    done = r == JYC_OK;
    return r;
}

int launch_tc_gemm(const TcGemm& p, int epi, cudaStream_t s) {
    if (p.n <= 0 || p.k <= 0 || p.k % 32 || p.T <= 0) return arg_error("tc_gemm: need n, T > 0 and k % 32 == 0");
    if (epi == TC_SWIGLU && p.n % 2) return arg_error("tc_gemm: SwiGLU needs interleaved row pairs");
    const int nkc = (p.k + kTcKC - 1) / kTcKC;
    if (p.splits < 1 || p.splits > nkc) return arg_error("tc_gemm: splits");
    const int per = (nkc + p.splits - 1) / p.splits;
    if ((nkc + per - 1) / per != p.splits) return arg_error("tc_gemm: a K split would be empty");
    if (p.splits > 1 && (!p.part || !p.cnt)) return arg_error("tc_gemm: split-K needs partial buffers");
    const int pr = prepare_tc_kernels();
    if (pr != JYC_OK) return pr;
    switch (p.N) {
        case 16: return launch_n<16>(p, epi, s);
        case 32: return launch_n<32>(p, epi, s);
        case 64: return launch_n<64>(p, epi, s);
        case 128: return launch_n<128>(p, epi, s);
        default: return arg_error("tc_gemm: token tile must be 16, 32, 64 or 128");
    }
}

}  // namespace jyc
