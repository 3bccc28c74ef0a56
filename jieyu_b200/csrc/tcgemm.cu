// tcgemm.cu — tcgen05 GEMM of Q8_0 weights over token tiles (prefill and
// batched decode), see tcgemm.cuh for the numerics.
//
// CTA = 128 weight rows x N tokens x one range of K, 10 warps:
//   warp 0     allocates the tensor-memory accumulator (N fp32 columns) and
//              streams the token operand: one 1-D bulk copy (TMA) per 64-wide
//              K chunk brings its hi and lo planes, already in the 128-byte
//              swizzled K-major layout the MMA reads;
//   warp 1     one thread issues the MMAs: per 16-wide K step
//              [D | E] += Whi.[Xhi | Xlo] (one MMA of width 2N) and
//              E += Wlo.Xhi (tcgen05.mma kind::f16, fp32 accumulators in
//              tensor memory, M=128) into the accumulator set of the chunk's
//              group, then tcgen05.commit frees the stage and, after the
//              group's last chunk, signals the set;
//   warps 2-9  converters: each thread dequantises one 32-weight block of one
//              row per chunk (q * d * 2^S exactly in fp32, split into fp16 hi
//              and lo), stores both into the swizzled A planes of the stage
//              and arrives on the stage's barrier; loads run 3 chunks ahead
//              in registers. They also drain every finished chunk's
//              accumulator set (tcgen05.ld: lanes = weight rows, columns =
//              tokens) into fp32 registers, and after the K loop run the
//              epilogue: unscale by 2^-S_row 2^-s_token, then store (+ bias,
//              residual or SwiGLU of interleaved gate/up rows) through a
//              shared-memory tile in coalesced rows. With K split over CTAs
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
    // tensor-memory columns (a power of two >= 32): two accumulator sets of
    // [N hi.hi columns | N hi.lo + lo.hi columns]; the corrections accumulate
    // apart so the large accumulator takes one rounding per K step, not three
    static constexpr int kCols = 4 * N < 32 ? 32 : 4 * N;
    // alignment slack + stages + barriers + tmem slot/flags
    static constexpr int kSmem = 1024 + kStages * kStage + 8 * (3 * kStages + 4) + 16;
};

// Tensor-memory A variant (token tiles up to 64): the weight planes go to
// tensor memory (tcgen05.st), shared memory holds only the token operand.
constexpr int kGroup = 2;         // K chunks accumulated per tensor-memory set before the drain
constexpr int kTaStageCols = 64;  // one A stage: hi (32 columns) + lo (32 columns) of 128 rows x 64 K
constexpr int kTaDone = 32;       // group-completion barriers in the ring (> any waiter's lag in groups)
constexpr int kTaQRing = 8;       // chunks of weight bytes in flight per converter thread (cp.async)
template <int N>
struct TcCfgTa {
    static constexpr int kPlaneB = N * 128;
    static constexpr int kStage = 2 * kPlaneB;  // token hi + lo planes of a chunk
    // A bulk copy completes about every 600 cycles whatever its size up to
    // 32 KB, so the token planes of kCB consecutive chunks travel together
    static constexpr int kCB = kStage >= 32768 ? 1 : 32768 / kStage;
    static constexpr int kSlotsB = 4;                 // B slots of kCB chunks
    static constexpr int kStagesB = kSlotsB * kCB;    // chunks of B in shared memory
    static constexpr int kStagesA = 4;
    static constexpr int kAccCols = 4 * N;
    static constexpr int kCols = 512;  // 4N + 4 x 64 <= 512 for N <= 64
    static_assert(kAccCols + kStagesA * kTaStageCols <= kCols, "tensor memory");
    // the epilogue tile [N][128] floats reuses the token stages
    static_assert(kStagesB * kStage >= N * kTcRows * 4, "epilogue tile");
    static constexpr int kSmem =
        1024 + kStagesB * kStage + kTaQRing * 256 * 32 + 8 * (kStagesA + kSlotsB + kTaDone + 2) + 16;
    static_assert(kStagesA % kGroup == 0, "A stages hold whole groups");
    static_assert(kStagesB / kGroup + kStagesA < kTaDone, "group ring deeper than any waiter's lag");
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
// D[tmem] (+)= A[tmem] . B[smem]^T (A: lane = row, two fp16 of K per column)
__device__ __forceinline__ void tc_mma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// this warp's 32 lanes, 16 consecutive columns from registers
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
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
// 16 columns at ta and 16 at tb of this warp's 32 lanes, one wait for both
__device__ __forceinline__ void tmem_ld16x2(uint32_t ta, uint32_t tb, float* a, float* b) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%32];\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, "
        "[%33];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(ta), "r"(tb)
        : "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) {
        a[i] = __uint_as_float(r[i]);
        b[i] = __uint_as_float(r[16 + i]);
    }
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
// 16-byte asynchronous global -> shared copy (L2 only) and its commit groups
__device__ __forceinline__ void cp_async16_cg(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit_group() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_groups() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// non-blocking test of an mbarrier phase (no suspension when not yet complete)
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// 2^e for e in [-126, 127], exactly
__device__ __forceinline__ float exp2i(int e) { return __int_as_float((e + 127) << 23); }
__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }
// copy without an L2 hint (the token planes are re-read by every row tile)
__device__ __forceinline__ void bulk_g2s_keep(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
// 8 fp32 values (already scaled below 2^15) -> 16 bytes of fp16 hi and 16
// bytes of lo. Veltkamp's split (c = f (2^13 + 1), hi = c - (c - f)) rounds f
// to its leading 11 bits in fp32, so hi converts to fp16 exactly and
// lo = f - hi is exact in fp32 (the fp16 conversion of lo keeps 11 of its at
// most 13 bits: all of them for the 18-bit weight products).
__device__ __forceinline__ void split8(const float* f, uint4& hi, uint4& lo) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        float hv[2], lv[2];
#pragma unroll
        for (int e = 0; e < 2; e++) {
            const float x = f[2 * i + e];
            const float c = __fmul_rn(x, 8193.0f);
            hv[e] = __fsub_rn(c, __fsub_rn(c, x));
            lv[e] = __fsub_rn(x, hv[e]);
        }
        h[i] = h2u(__floats2half2_rn(hv[0], hv[1]));
        l[i] = h2u(__floats2half2_rn(lv[0], lv[1]));
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
}

template <int N, int EPI>
__global__ void __launch_bounds__(kThreads, 1) tc_gemm_kernel(TcGemm p) {
    using C = TcCfg<N>;
    constexpr int CH = N / 2;  // accumulator columns (tokens) per converter thread
    extern __shared__ unsigned char tc_smraw[];
    // the 128-byte swizzle is a function of the address bits: 1024-byte aligned tiles
    unsigned char* sm = tc_smraw + ((1024u - (smem_u32(tc_smraw) & 1023u)) & 1023u);
    uint64_t* afull = reinterpret_cast<uint64_t*>(sm + C::kStages * C::kStage);  // converters done (256 arrivals)
    uint64_t* bfull = afull + C::kStages;                                         // token planes landed (tx)
    uint64_t* empty = bfull + C::kStages;                                         // MMAs of the stage done
    uint64_t* accf = empty + C::kStages;   // [2] accumulator set b holds a finished chunk (MMA commit)
    uint64_t* accfree = accf + 2;          // [2] accumulator set b drained (256 arrivals)
    uint32_t* s_tmem = reinterpret_cast<uint32_t*>(accfree + 2);
    unsigned int* s_flag = s_tmem + 1;
    volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 2);  // a bounded wait gave up

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int mt = blockIdx.x, tt = blockIdx.y, z = blockIdx.z;
    const int nkc = (p.k + kTcKC - 1) / kTcKC;
    const int per = (nkc + p.splits - 1) / p.splits;
    const int c0 = z * per, nch = min(nkc, c0 + per) - c0;  // the host plan leaves no split empty
    // bounded wait; after any give-up in this CTA every later wait is skipped
    auto wait = [&](uint64_t* bar, uint32_t parity) -> bool {
        if (*s_abort) return false;
        if (mbar_wait_err(bar, parity, p.err, kErrTc)) return true;
        *s_abort = 1;
        return false;
    };

    if (tid == 0) {
        for (int s = 0; s < C::kStages; s++) {
            mbar_init(&afull[s], 256);
            mbar_init(&bfull[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&accf[b], 1);
            mbar_init(&accfree[b], 256);
        }
        *s_abort = 0;
        mbar_fence_init();
    }
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
                if (j >= C::kStages && !wait(&empty[s], ((j / C::kStages) - 1) & 1)) break;
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
            // B hi and lo planes are adjacent rows of one K-major tile: a single
            // MMA of width 2N gives Whi.Xhi (columns [0, N)) and Whi.Xlo
            // (columns [N, 2N)); Wlo.Xhi then accumulates into [N, 2N)
            constexpr uint32_t idesc2 = idesc_f16<2 * N>();
            constexpr uint32_t idesc = idesc_f16<N>();
            for (int j = 0; j < nch; j++) {
                const int s = j % C::kStages, g = j / kGroup, b = g & 1;
                const bool first = j % kGroup == 0;  // the group's first chunk overwrites the set
                const uint32_t ph = (j / C::kStages) & 1;
                if (first && g >= 2 && !wait(&accfree[b], ((g >> 1) - 1) & 1)) break;
                if (!wait(&afull[s], ph) || !wait(&bfull[s], ph)) break;
                tc_fence_after();
                const uint32_t st = smem_u32(sm + s * C::kStage);
                const uint64_t ah = sw128_desc(st), al = sw128_desc(st + kPlaneA);
                const uint64_t bh = sw128_desc(st + 2 * kPlaneA);
                const uint32_t dm = tmem + (uint32_t)(2 * N * b), dc = dm + N;
#pragma unroll
                for (int ks = 0; ks < kTcKC / 16; ks++) {
                    const uint64_t o = 2 * ks;  // 32 bytes further along K, in 16-byte units
                    tc_mma_f16(dm, ah + o, bh + o, idesc2, !first || ks != 0);
                    tc_mma_f16(dc, al + o, bh + o, idesc, 1u);
                }
                tc_commit(&empty[s]);
                if (j % kGroup == kGroup - 1 || j == nch - 1) tc_commit(&accf[b]);
            }
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
        // rows scaled by 2^S with S = 22 - exponent field of max |d|: 127 max|d| 2^S < 2^15
        const float rup = exp2i(22 - (rv ? (int)__ldg(p.rexp + R) : 0));
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
        auto convert = [&](int j, const uint4* q, uint16_t dv) {
            const int s = j % C::kStages;
            if (j >= C::kStages) wait(&empty[s], ((j / C::kStages) - 1) & 1);
            unsigned char* ah = sm + s * C::kStage + r * 128;
            // packed half2 arithmetic, two weights per instruction:
            // q = (0x6400 | u) - 1152 exactly (fp16 1024 + u, u = q + 128);
            // hi = fp16(q d_s) rounded to nearest; lo = fma(q, d_s, -hi) is the
            // exact residual (q d_s has at most 18 significant bits)
            const __half2 ds2 = __float2half2_rn(__fmul_rn(h2f(dv), rup));
            const __half2 off = __float2half2_rn(1152.0f);
            const uint32_t* w = reinterpret_cast<const uint32_t*>(q);
#pragma unroll
            for (int c = 0; c < 4; c++) {
                uint32_t hw[4], lw[4];
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const uint32_t pk = __byte_perm(w[2 * c + (i >> 1)], 0x64646464u, (i & 1) ? 0x4342u : 0x4140u);
                    const __half2 q2 = __hsub2(u2h(pk), off);
                    const __half2 h2 = __hmul2_rn(q2, ds2);
                    hw[i] = h2u(h2);
                    lw[i] = h2u(__hfma2(q2, ds2, __hneg2(h2)));
                }
                const int pos = ((4 * h + c) ^ (r & 7)) * 16;
                *reinterpret_cast<uint4*>(ah + pos) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                *reinterpret_cast<uint4*>(ah + kPlaneA + pos) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
            }
            fence_proxy_async_smem();
            mbar_arrive(&afull[s]);
        };
        // The tensor cores accumulate in fp32 with truncation; over a long K
        // that biases sums toward zero. Each group of kGroup chunks therefore
        // lands in one of two accumulator sets, and these threads add it into
        // fp32 registers (round to nearest) one group later, while the MMAs
        // fill the other set.
        const int q4 = warp & 3, half = (warp - 2) >> 2;  // lane quadrant, column half
        const int re = 32 * q4 + lane;
        const uint32_t tq = tmem + ((uint32_t)(32 * q4) << 16) + (uint32_t)(half * CH);
        float acc[CH];
#pragma unroll
        for (int c = 0; c < CH; c++) acc[c] = 0.0f;
        auto drain = [&](int g) {
            const int b = g & 1;
            wait(&accf[b], (g >> 1) & 1);
            tc_fence_after();
            const uint32_t ta = tq + (uint32_t)(2 * N * b);
            if (CH % 16 == 0) {
#pragma unroll
                for (int c = 0; c < CH; c += 16) {
                    float mv[16], cv[16];
                    tmem_ld16x2(ta + (uint32_t)c, ta + (uint32_t)(N + c), mv, cv);
#pragma unroll
                    for (int i = 0; i < 16; i++) acc[c + i] = __fadd_rn(acc[c + i], __fadd_rn(mv[i], cv[i]));
                }
            } else {
#pragma unroll
                for (int c = 0; c < CH; c += 8) {
                    float mv[8], cv[8];
                    tmem_ld8(ta + (uint32_t)c, mv);
                    tmem_ld8(ta + (uint32_t)(N + c), cv);
#pragma unroll
                    for (int i = 0; i < 8; i++) acc[c + i] = __fadd_rn(acc[c + i], __fadd_rn(mv[i], cv[i]));
                }
            }
            tc_fence_before();
            mbar_arrive(&accfree[b]);
        };
        if (nch > 0) load(0, qa[0], dd[0]);
        if (nch > 1) load(1, qa[1], dd[1]);
        if (nch > 2) load(2, qa[2], dd[2]);
        int drained = 0;  // next group to drain
        for (int j0 = 0; j0 < nch; j0 += 4) {
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int j = j0 + u;
                if (j < nch) {
                    if (j + 3 < nch) load(j + 3, qa[(u + 3) & 3], dd[(u + 3) & 3]);
                    convert(j, qa[u], dd[u]);
                    // a group's chunks are converted: drain the group before it
                    if (j % kGroup == kGroup - 1 && j >= kGroup) drain(drained++);
                }
            }
        }
        while (drained * kGroup < nch) drain(drained++);

        // ---------------- epilogue ----------------
        // 1. register accumulators (thread = row re, tokens of its column half)
        //    -> scaled fp32 tile [N tokens][128 rows] in the idle stage memory
        //    (every MMA has completed: the last drain waited for it)
        float* stile = reinterpret_cast<float*>(sm);
        {
            const int Re = mt * kTcRows + re;
            const float rdown = exp2i((Re < p.n ? (int)__ldg(p.rexp + Re) : 0) - 22);
#pragma unroll
            for (int c = 0; c < CH; c++) {
                const int tl = half * CH + c;
                stile[tl * kTcRows + re] = __fmul_rn(__fmul_rn(acc[c], rdown), exp2i(-__ldg(p.xe + tt * N + tl)));
            }
        }
        named_sync_conv();
        // 2. coalesced row-major passes: element e = ct + 256 i is (token e / 128,
        //    row e % 128); groups of 16 keep 16 loads in flight per thread
        constexpr int kPer = N * kTcRows / 256, kG = kPer < 16 ? kPer : 16;
        const int rl = ct & (kTcRows - 1), Rg = mt * kTcRows + rl;
        const bool rok = Rg < p.n;
        auto tok_of = [&](int i) { return tt * N + ((ct + 256 * i) >> 7); };
        auto epilogue = [&](int i0, const float* v) {
            if (EPI == TC_RESID) {
                float old[kG];
#pragma unroll
                for (int u = 0; u < kG; u++) {
                    const int t = tok_of(i0 + u);
                    old[u] = (rok && t < p.T) ? p.y[(size_t)t * p.ldy + Rg] : 0.0f;
                }
#pragma unroll
                for (int u = 0; u < kG; u++) {
                    const int t = tok_of(i0 + u);
                    if (rok && t < p.T) p.y[(size_t)t * p.ldy + Rg] = __fadd_rn(old[u], v[u]);
                }
            } else {
                const float b = (EPI == TC_BIAS && rok) ? __ldg(p.bias + Rg) : 0.0f;
#pragma unroll
                for (int u = 0; u < kG; u++) {
                    const int t = tok_of(i0 + u);
                    const bool ok_t = t < p.T;
                    if (EPI == TC_SWIGLU) {
                        // rows 2j (gate) and 2j+1 (up) sit in adjacent lanes
                        const float upv = __shfl_down_sync(0xffffffffu, v[u], 1);
                        if ((lane & 1) == 0 && rok && ok_t)
                            p.y[(size_t)t * p.ldy + (Rg >> 1)] = __fmul_rn(silu_ref(v[u]), upv);
                    } else if (rok && ok_t) {
                        p.y[(size_t)t * p.ldy + Rg] = EPI == TC_BIAS ? __fadd_rn(v[u], b) : v[u];
                    }
                }
            }
        };
        if (p.splits == 1 && EPI == TC_SWIGLU) {
            // thread = one (gate, up) row pair of tokens ct / 64 + 4 i: one silu per pair
            const int pr = ct & 63, R2 = mt * (kTcRows / 2) + pr;
            const bool pok = 2 * R2 < p.n;
#pragma unroll 4
            for (int tl = ct >> 6; tl < N; tl += 4) {
                const int t = tt * N + tl;
                const float2 gu = *reinterpret_cast<const float2*>(stile + tl * kTcRows + 2 * pr);
                if (pok && t < p.T) p.y[(size_t)t * p.ldy + R2] = __fmul_rn(silu_ref(gu.x), gu.y);
            }
        } else if (p.splits == 1) {
#pragma unroll 1
            for (int i0 = 0; i0 < kPer; i0 += kG) {
                float v[kG];
#pragma unroll
                for (int u = 0; u < kG; u++) v[u] = stile[ct + 256 * (i0 + u)];
                epilogue(i0, v);
            }
        } else {
            // partial tile of this K range; the last CTA of the tile to arrive
            // sums all of them in split order and runs the epilogue
#pragma unroll 1
            for (int i = 0; i < kPer; i++) {
                const int t = tok_of(i);
                if (rok && t < p.T) p.part[((size_t)z * p.T + t) * p.n + Rg] = stile[ct + 256 * i];
            }
            __threadfence();
            named_sync_conv();
            if (ct == 0) {
                const unsigned int old = atomicAdd(&p.cnt[mt * gridDim.y + tt], 1u);
                *s_flag = (old == (unsigned int)(p.splits - 1)) ? 1u : 0u;
            }
            named_sync_conv();
            if (*s_flag != 0u) {
                __threadfence();
#pragma unroll 1
                for (int i0 = 0; i0 < kPer; i0 += kG) {
                    float v[kG];
#pragma unroll
                    for (int u = 0; u < kG; u++) v[u] = 0.0f;
                    // per 8 elements: four splits' loads in flight before their in-order adds
#pragma unroll
                    for (int g0 = 0; g0 < kG; g0 += 8) {
                        constexpr int kR = kG < 8 ? kG : 8;
                        for (int z0 = 0; z0 < p.splits; z0 += 4) {
                            float ld[4][kR];
#pragma unroll
                            for (int zi = 0; zi < 4; zi++)
#pragma unroll
                                for (int u = 0; u < kR; u++) {
                                    const int t = tok_of(i0 + g0 + u);
                                    ld[zi][u] = (rok && t < p.T && z0 + zi < p.splits)
                                                    ? __ldcg(p.part + ((size_t)(z0 + zi) * p.T + t) * p.n + Rg)
                                                    : 0.0f;
                                }
#pragma unroll
                            for (int zi = 0; zi < 4; zi++)
#pragma unroll
                                for (int u = 0; u < kR; u++)
                                    if (z0 + zi < p.splits) v[g0 + u] = __fadd_rn(v[g0 + u], ld[zi][u]);
                        }
                    }
                    epilogue(i0, v);
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

template <int N, int EPI>
__global__ void __launch_bounds__(kThreads, 1) tc_gemm_ta_kernel(TcGemm p) {
    using C = TcCfgTa<N>;
    constexpr int CH = N / 2;  // accumulator columns (tokens) per converter thread
    extern __shared__ unsigned char tc_smraw[];
    // the 128-byte swizzle is a function of the address bits: 1024-byte aligned tiles
    unsigned char* sm = tc_smraw + ((1024u - (smem_u32(tc_smraw) & 1023u)) & 1023u);
    // One tcgen05.commit per group of kGroup chunks (a commit costs hundreds of
    // cycles): gdone[g % kTaDone] completes when group g's MMAs have, which
    // frees its A and B stages and lets its accumulator set be drained.
    // shared memory: token slots | weight-byte ring | barriers
    uint64_t* afull = reinterpret_cast<uint64_t*>(sm + C::kStagesB * C::kStage + kTaQRing * 256 * 32);  // A stage written (256 arrivals)
    uint64_t* bfull = afull + C::kStagesA;                                         // token slot landed (tx)
    uint64_t* gdone = bfull + C::kSlotsB;                                          // [kTaDone] group MMAs done
    uint64_t* accfree = gdone + kTaDone;   // [2] accumulator set b drained (256 arrivals)
    uint32_t* s_tmem = reinterpret_cast<uint32_t*>(accfree + 2);
    unsigned int* s_flag = s_tmem + 1;
    volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 2);  // a bounded wait gave up

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int mt = blockIdx.x, tt = blockIdx.y, z = blockIdx.z;
    const int nkc = (p.k + kTcKC - 1) / kTcKC;
    const int per = (nkc + p.splits - 1) / p.splits;
    const int c0 = z * per, nch = min(nkc, c0 + per) - c0;  // the host plan leaves no split empty
    // bounded wait; after any give-up in this CTA every later wait is skipped
    auto wait = [&](uint64_t* bar, uint32_t parity) -> bool {
        if (mbar_test(bar, parity)) return true;  // already complete: no suspend round trip
        if (*s_abort) return false;
        if (mbar_wait_err(bar, parity, p.err, kErrTc)) return true;
        *s_abort = 1;
        return false;
    };

    if (tid == 0) {
        for (int s = 0; s < C::kStagesA; s++) mbar_init(&afull[s], 256);
        for (int s = 0; s < C::kSlotsB; s++) mbar_init(&bfull[s], 1);
        for (int g = 0; g < kTaDone; g++) mbar_init(&gdone[g], 1);
        for (int b = 0; b < 2; b++) mbar_init(&accfree[b], 256);
        *s_abort = 0;
        mbar_fence_init();
    }
    if (warp == 0) {
        __syncwarp();
        tmem_alloc(s_tmem, C::kCols);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *s_tmem;
    // wait until group g's MMAs are complete
    auto wait_group = [&](int g) -> bool { return wait(&gdone[g % kTaDone], (g / kTaDone) & 1); };

    if (warp == 0) {
        if (lane == 0) {
            const unsigned char* src =
                reinterpret_cast<const unsigned char*>(p.xs) + ((size_t)tt * nkc + c0) * 2 * C::kPlaneB;
            // load u brings chunks [u kCB, u kCB + kCB) into slot u % kSlotsB, once
            // the MMAs of that slot's previous chunks are done
            const int nload = (nch + C::kCB - 1) / C::kCB;
            int issued = 0;
            for (int u = 0; u < nload; u++) {
                const int sl = u % C::kSlotsB, cj = u * C::kCB, cn = min(C::kCB, nch - cj);
                if (u >= C::kSlotsB && !wait_group((cj - C::kSlotsB * C::kCB + C::kCB - 1) / kGroup)) break;
                mbar_expect_tx(&bfull[sl], cn * C::kStage);
                bulk_g2s_keep(sm + sl * C::kCB * C::kStage, src + (size_t)cj * C::kStage, cn * C::kStage, &bfull[sl]);
                issued = u + 1;
            }
            // no copy may still be landing when the CTA exits (matters only after an error)
            for (int u = max(0, issued - C::kSlotsB); u < issued; u++)
                mbar_wait_err(&bfull[u % C::kSlotsB], (u / C::kSlotsB) & 1, p.err, kErrTc);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // B hi and lo planes are adjacent rows of one K-major tile: a single
            // MMA of width 2N gives Whi.Xhi (columns [0, N)) and Whi.Xlo
            // (columns [N, 2N)); Wlo.Xhi then accumulates into [N, 2N)
            constexpr uint32_t idesc2 = idesc_f16<2 * N>();
            constexpr uint32_t idesc = idesc_f16<N>();
            for (int j = 0; j < nch; j++) {
                const int sa = j % C::kStagesA, g = j / kGroup, b = g & 1;
                const int u = j / C::kCB, sl = u % C::kSlotsB;  // the token slot holding chunk j
                const bool first = j % kGroup == 0;  // the group's first chunk overwrites the set
                if (first && g >= 2 && !wait(&accfree[b], ((g >> 1) - 1) & 1)) break;
                if (!wait(&afull[sa], (j / C::kStagesA) & 1)) break;
                if (j % C::kCB == 0 && !wait(&bfull[sl], (u / C::kSlotsB) & 1)) break;  // slot entry
                tc_fence_after();
                const uint64_t bh = sw128_desc(smem_u32(sm + (sl * C::kCB + j % C::kCB) * C::kStage));
                const uint32_t ah = tmem + (uint32_t)(C::kAccCols + kTaStageCols * sa), al = ah + 32;
                const uint32_t dm = tmem + (uint32_t)(2 * N * b), dc = dm + N;
#pragma unroll
                for (int ks = 0; ks < kTcKC / 16; ks++) {
                    // A: 8 columns (16 fp16 of K) per step; B: 32 bytes further along K
                    tc_mma_f16_ts(dm, ah + 8 * ks, bh + 2 * ks, idesc2, !first || ks != 0);
                    tc_mma_f16_ts(dc, al + 8 * ks, bh + 2 * ks, idesc, 1u);
                }
                if (j % kGroup == kGroup - 1 || j == nch - 1) tc_commit(&gdone[g % kTaDone]);
            }
        }
    } else {
        // ---------------- converters ----------------
        const int ct = tid - 64, cw = ct >> 5;
        // a warp writes only its own tensor-memory lane quadrant: rows 32 (warp & 3) + lane
        const int r = 32 * (warp & 3) + lane, h = cw >> 2;  // tile row, which 32-block of the chunk
        const int R = mt * kTcRows + r;
        const bool rv = R < p.n;
        const int nb = p.k >> 5;
        const uint8_t* qrow = p.qs + (size_t)(rv ? R : 0) * p.k;
        const uint16_t* drow = p.d + (size_t)(rv ? R : 0) * nb;
        // rows scaled by 2^S with S = 22 - exponent field of max |d|: 127 max|d| 2^S < 2^15
        const float rup = exp2i(22 - (rv ? (int)__ldg(p.rexp + R) : 0));
        // weight bytes: each thread's 32 bytes per chunk land in its own slot
        // of a kTaQRing-deep cp.async ring (64 KB in flight per SM); the fp16
        // scales come 3 chunks ahead in registers
        unsigned char* qring = sm + C::kStagesB * C::kStage + (size_t)ct * 32;  // + slot * 256 * 32
        auto issue_q = [&](int j) {
            const int kb = 2 * (c0 + j) + h;
            if (j < nch && rv && kb < nb) {
                const unsigned char* src = qrow + (size_t)kb * 32;
                unsigned char* dst = qring + (size_t)(j % kTaQRing) * 256 * 32;
                cp_async16_cg(dst, src);
                cp_async16_cg(dst + 16, src + 16);
            }
            cp_async_commit_group();
        };
        uint16_t dd[4];
        auto load = [&](int j, uint4*, uint16_t& dv) {
            const int kb = 2 * (c0 + j) + h;
            dv = (rv && kb < nb) ? __ldg(drow + kb) : (uint16_t)0;
        };
        uint4 qa[4][2];  // (the weight bytes of chunk j, read from the ring)
        auto convert = [&](int j, const uint4* q, uint16_t dv) {
            const int sa = j % C::kStagesA;
            if (j >= C::kStagesA) wait_group((j - C::kStagesA) / kGroup);
            tc_fence_after();
            // hi and lo planes of this row's 32 weights: 16 columns each (two
            // fp16 of K per 32-bit column), the same exact half2 split as the
            // shared-memory variant
            const __half2 ds2 = __float2half2_rn(__fmul_rn(h2f(dv), rup));
            const __half2 off = __float2half2_rn(1152.0f);
            const uint32_t* w = reinterpret_cast<const uint32_t*>(q);
            uint32_t hw[16], lw[16];
#pragma unroll
            for (int i = 0; i < 16; i++) {
                const uint32_t pk = __byte_perm(w[i >> 1], 0x64646464u, (i & 1) ? 0x4342u : 0x4140u);
                const __half2 q2 = __hsub2(u2h(pk), off);
                const __half2 h2 = __hmul2_rn(q2, ds2);
                hw[i] = h2u(h2);
                lw[i] = h2u(__hfma2(q2, ds2, __hneg2(h2)));
            }
            const uint32_t ta = tmem + ((uint32_t)(32 * (warp & 3)) << 16) +
                                (uint32_t)(C::kAccCols + kTaStageCols * sa + 16 * h);
            tmem_st16(ta, hw);
            tmem_st16(ta + 32, lw);
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&afull[sa]);
        };
        // The tensor cores accumulate in fp32 with truncation; over a long K
        // that biases sums toward zero. Each group of kGroup chunks therefore
        // lands in one of two accumulator sets, and these threads add it into
        // fp32 registers (round to nearest) one group later, while the MMAs
        // fill the other set.
        const int q4 = warp & 3, half = (warp - 2) >> 2;  // lane quadrant, column half
        const int re = 32 * q4 + lane;
        const uint32_t tq = tmem + ((uint32_t)(32 * q4) << 16) + (uint32_t)(half * CH);
        float acc[CH];
#pragma unroll
        for (int c = 0; c < CH; c++) acc[c] = 0.0f;
        auto drain = [&](int g) {
            const int b = g & 1;
            wait_group(g);
            tc_fence_after();
            const uint32_t ta = tq + (uint32_t)(2 * N * b);
            if (CH % 16 == 0) {
#pragma unroll
                for (int c = 0; c < CH; c += 16) {
                    float mv[16], cv[16];
                    tmem_ld16x2(ta + (uint32_t)c, ta + (uint32_t)(N + c), mv, cv);
#pragma unroll
                    for (int i = 0; i < 16; i++) acc[c + i] = __fadd_rn(acc[c + i], __fadd_rn(mv[i], cv[i]));
                }
            } else {
#pragma unroll
                for (int c = 0; c < CH; c += 8) {
                    float mv[8], cv[8];
                    tmem_ld8(ta + (uint32_t)c, mv);
                    tmem_ld8(ta + (uint32_t)(N + c), cv);
#pragma unroll
                    for (int i = 0; i < 8; i++) acc[c + i] = __fadd_rn(acc[c + i], __fadd_rn(mv[i], cv[i]));
                }
            }
            tc_fence_before();
            mbar_arrive(&accfree[b]);
        };
        if (nch > 0) load(0, qa[0], dd[0]);
        if (nch > 1) load(1, qa[1], dd[1]);
        if (nch > 2) load(2, qa[2], dd[2]);
#pragma unroll
        for (int i = 0; i < kTaQRing - 1; i++) issue_q(i);
        int drained = 0;  // next group to drain
        for (int j0 = 0; j0 < nch; j0 += 4) {
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int j = j0 + u;
                if (j < nch) {
                    if (j + 3 < nch) load(j + 3, qa[(u + 3) & 3], dd[(u + 3) & 3]);
                    issue_q(j + kTaQRing - 1);
                    cp_async_wait_groups<kTaQRing - 1>();  // this thread's bytes of chunk j landed
                    {
                        const int kb = 2 * (c0 + j) + h;
                        if (rv && kb < nb) {
                            const uint4* q = reinterpret_cast<const uint4*>(qring + (size_t)(j % kTaQRing) * 256 * 32);
                            qa[u][0] = q[0];
                            qa[u][1] = q[1];
                        } else {
                            qa[u][0] = qa[u][1] = make_uint4(0x80808080u, 0x80808080u, 0x80808080u, 0x80808080u);
                        }
                    }
                    convert(j, qa[u], dd[u]);
                    // a group's chunks are converted: drain the group before it
                    if (j % kGroup == kGroup - 1 && j >= kGroup) drain(drained++);
                }
            }
        }
        while (drained * kGroup < nch) drain(drained++);

        // ---------------- epilogue ----------------
        // 1. register accumulators (thread = row re, tokens of its column half)
        //    -> scaled fp32 tile [N tokens][128 rows] in the idle stage memory
        //    (every MMA has completed: the last drain waited for it)
        float* stile = reinterpret_cast<float*>(sm);
        {
            const int Re = mt * kTcRows + re;
            const float rdown = exp2i((Re < p.n ? (int)__ldg(p.rexp + Re) : 0) - 22);
#pragma unroll
            for (int c = 0; c < CH; c++) {
                const int tl = half * CH + c;
                stile[tl * kTcRows + re] = __fmul_rn(__fmul_rn(acc[c], rdown), exp2i(-__ldg(p.xe + tt * N + tl)));
            }
        }
        named_sync_conv();
        // 2. coalesced row-major passes: element e = ct + 256 i is (token e / 128,
        //    row e % 128); groups of 16 keep 16 loads in flight per thread
        constexpr int kPer = N * kTcRows / 256, kG = kPer < 16 ? kPer : 16;
        const int rl = ct & (kTcRows - 1), Rg = mt * kTcRows + rl;
        const bool rok = Rg < p.n;
        auto tok_of = [&](int i) { return tt * N + ((ct + 256 * i) >> 7); };
        auto epilogue = [&](int i0, const float* v) {
            if (EPI == TC_RESID) {
                float old[kG];
#pragma unroll
                for (int u = 0; u < kG; u++) {
                    const int t = tok_of(i0 + u);
                    old[u] = (rok && t < p.T) ? p.y[(size_t)t * p.ldy + Rg] : 0.0f;
                }
#pragma unroll
                for (int u = 0; u < kG; u++) {
                    const int t = tok_of(i0 + u);
                    if (rok && t < p.T) p.y[(size_t)t * p.ldy + Rg] = __fadd_rn(old[u], v[u]);
                }
            } else {
                const float b = (EPI == TC_BIAS && rok) ? __ldg(p.bias + Rg) : 0.0f;
#pragma unroll
                for (int u = 0; u < kG; u++) {
                    const int t = tok_of(i0 + u);
                    const bool ok_t = t < p.T;
                    if (EPI == TC_SWIGLU) {
                        // rows 2j (gate) and 2j+1 (up) sit in adjacent lanes
                        const float upv = __shfl_down_sync(0xffffffffu, v[u], 1);
                        if ((lane & 1) == 0 && rok && ok_t)
                            p.y[(size_t)t * p.ldy + (Rg >> 1)] = __fmul_rn(silu_ref(v[u]), upv);
                    } else if (rok && ok_t) {
                        p.y[(size_t)t * p.ldy + Rg] = EPI == TC_BIAS ? __fadd_rn(v[u], b) : v[u];
                    }
                }
            }
        };
        if (p.splits == 1 && EPI == TC_SWIGLU) {
            // thread = one (gate, up) row pair of tokens ct / 64 + 4 i: one silu per pair
            const int pr = ct & 63, R2 = mt * (kTcRows / 2) + pr;
            const bool pok = 2 * R2 < p.n;
#pragma unroll 4
            for (int tl = ct >> 6; tl < N; tl += 4) {
                const int t = tt * N + tl;
                const float2 gu = *reinterpret_cast<const float2*>(stile + tl * kTcRows + 2 * pr);
                if (pok && t < p.T) p.y[(size_t)t * p.ldy + R2] = __fmul_rn(silu_ref(gu.x), gu.y);
            }
        } else if (p.splits == 1) {
#pragma unroll 1
            for (int i0 = 0; i0 < kPer; i0 += kG) {
                float v[kG];
#pragma unroll
                for (int u = 0; u < kG; u++) v[u] = stile[ct + 256 * (i0 + u)];
                epilogue(i0, v);
            }
        } else {
            // partial tile of this K range; the last CTA of the tile to arrive
            // sums all of them in split order and runs the epilogue
#pragma unroll 1
            for (int i = 0; i < kPer; i++) {
                const int t = tok_of(i);
                if (rok && t < p.T) p.part[((size_t)z * p.T + t) * p.n + Rg] = stile[ct + 256 * i];
            }
            __threadfence();
            named_sync_conv();
            if (ct == 0) {
                const unsigned int old = atomicAdd(&p.cnt[mt * gridDim.y + tt], 1u);
                *s_flag = (old == (unsigned int)(p.splits - 1)) ? 1u : 0u;
            }
            named_sync_conv();
            if (*s_flag != 0u) {
                __threadfence();
#pragma unroll 1
                for (int i0 = 0; i0 < kPer; i0 += kG) {
                    float v[kG];
#pragma unroll
                    for (int u = 0; u < kG; u++) v[u] = 0.0f;
                    // per 8 elements: four splits' loads in flight before their in-order adds
#pragma unroll
                    for (int g0 = 0; g0 < kG; g0 += 8) {
                        constexpr int kR = kG < 8 ? kG : 8;
                        for (int z0 = 0; z0 < p.splits; z0 += 4) {
                            float ld[4][kR];
#pragma unroll
                            for (int zi = 0; zi < 4; zi++)
#pragma unroll
                                for (int u = 0; u < kR; u++) {
                                    const int t = tok_of(i0 + g0 + u);
                                    ld[zi][u] = (rok && t < p.T && z0 + zi < p.splits)
                                                    ? __ldcg(p.part + ((size_t)(z0 + zi) * p.T + t) * p.n + Rg)
                                                    : 0.0f;
                                }
#pragma unroll
                            for (int zi = 0; zi < 4; zi++)
#pragma unroll
                                for (int u = 0; u < kR; u++)
                                    if (z0 + zi < p.splits) v[g0 + u] = __fadd_rn(v[g0 + u], ld[zi][u]);
                        }
                    }
                    epilogue(i0, v);
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

// Per weight row: the fp16 exponent field of max |d| over its scales (one
// warp per row).
__global__ void __launch_bounds__(256) tc_rowexp_kernel(const uint16_t* d, int n, int nb, uint8_t* rexp) {
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= n) return;
    unsigned int mx = 0u;
    for (int b = lane; b < nb; b += 32) mx = max(mx, (unsigned int)(__ldg(d + (size_t)row * nb + b) & 0x7FFFu));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) rexp[row] = (uint8_t)(mx >> 10);
}

// token tiles up to 64 take the tensor-memory-A kernel, 128 the shared-memory one
template <int N, int EPI>
constexpr auto tc_kernel() {
    if constexpr (N <= 64) return tc_gemm_ta_kernel<N, EPI>;
    else return tc_gemm_kernel<N, EPI>;
}
template <int N>
constexpr int tc_smem() {
    if constexpr (N <= 64) return TcCfgTa<N>::kSmem;
    else return TcCfg<N>::kSmem;
}

template <int N>
int set_smem() {
    constexpr int smem = tc_smem<N>();
    static_assert(smem <= 227 * 1024, "tc_gemm shared memory");
    JYC_CUDA(cudaFuncSetAttribute(tc_kernel<N, TC_STORE>(), cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    JYC_CUDA(cudaFuncSetAttribute(tc_kernel<N, TC_BIAS>(), cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    JYC_CUDA(cudaFuncSetAttribute(tc_kernel<N, TC_RESID>(), cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    JYC_CUDA(cudaFuncSetAttribute(tc_kernel<N, TC_SWIGLU>(), cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    return JYC_OK;
}

template <int N>
int launch_n(const TcGemm& p, int epi, cudaStream_t s) {
    const dim3 grid((p.n + kTcRows - 1) / kTcRows, (p.T + N - 1) / N, p.splits);
    constexpr int smem = tc_smem<N>();
    switch (epi) {
        case TC_STORE: tc_kernel<N, TC_STORE>()<<<grid, kThreads, smem, s>>>(p); break;
        case TC_BIAS: tc_kernel<N, TC_BIAS>()<<<grid, kThreads, smem, s>>>(p); break;
        case TC_RESID: tc_kernel<N, TC_RESID>()<<<grid, kThreads, smem, s>>>(p); break;
        case TC_SWIGLU: tc_kernel<N, TC_SWIGLU>()<<<grid, kThreads, smem, s>>>(p); break;
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

void tc_plan(int n, int k, int T, int max_splits, int* N_out, int* splits_out) {
    // Cost model in microseconds at ~1.9 GHz: a CTA pays a fixed ~3 us (tensor
    // memory, barriers, pipeline fill, epilogue) plus per 64-wide K chunk the
    // slower of its weight conversion + accumulator drain (~250 + 2.4 N
    // cycles) and its 12 MMAs (128 x N x 16 each, ~6.35 N cycles); K splits
    // add a partial-sum pass.
    const int nkc = (k + kTcKC - 1) / kTcKC, mtiles = (n + kTcRows - 1) / kTcRows;
    const int sms = mega_num_ctas();
    double best = 1e30;
    *N_out = tc_token_tile(T);
    *splits_out = 1;
    for (int N = 16; N <= tc_token_tile(T); N *= 2) {
        const double chunk_us = std::max(250.0 + 2.4 * N, 6.35 * N) / 1900.0;
        const int tiles = mtiles * ((T + N - 1) / N);
        for (int s = 1; s <= std::min(max_splits, nkc); s++) {
            const int per = (nkc + s - 1) / s;
            if ((nkc + per - 1) / per != s) continue;  // no empty split
            const int waves = (tiles * s + sms - 1) / sms;
            const double cost = waves * (3.0 + per * chunk_us) + (s > 1 ? 2.0 + 0.2 * s : 0.0);
            if (cost < best - 1e-9) {
                best = cost;
                *N_out = N;
                *splits_out = s;
            }
        }
    }
}

int launch_tc_rowexp(const uint16_t* d, int n, int k, uint8_t* rexp, cudaStream_t s) {
    if (n <= 0 || k <= 0 || k % 32) return arg_error("tc_rowexp: n > 0, k % 32 == 0");
    tc_rowexp_kernel<<<(n + 7) / 8, 256, 0, s>>>(d, n, k / 32, rexp);
    JYC_LAUNCHED();
    return JYC_OK;
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
    // once per process (thread-safe static initialisation)
    static const int r = [] {
        int rr = set_smem<16>();
        if (rr == JYC_OK) rr = set_smem<32>();
        if (rr == JYC_OK) rr = set_smem<64>();
        if (rr == JYC_OK) rr = set_smem<128>();
        return rr;
    }();
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
    if (!p.rexp) return arg_error("tc_gemm: row exponents missing");
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
