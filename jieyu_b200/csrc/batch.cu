// batch.cu — kernels of batched decode: embedding gather by per-sequence
// length, attention over per-sequence KV cache slots, per-sequence greedy
// argmax + append, length updates. The matmuls and the RoPE/KV append of a
// batched step are the model kernels run over B rows (tcgemm.cu, or the
// GEMV of kernels.cu; rope_quant with row_len).
#include <algorithm>

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

// ---------------------------------------------------------------------------
// Batched decode attention over int8 KV caches (the attention of
// transformer_layer for one new row per sequence, libs/model_libs/attention/
// attention_q8.h:38-184, with the reference's score scaling
// dot * ((ks * qs) * 1/sqrt(hd)), fp32 online softmax and the V scale folded
// into the weights). CTA = (position split, kv head, sequence), 8 warps; each
// warp owns a contiguous run of the split's positions and keeps its own
// online-softmax state, so the loop has no CTA-wide barrier. Per tile of 32
// positions: lane j's K and V rows arrive with 16-byte cp.async into the
// warp's double buffer (chunks rotated per row: conflict-free row reads);
// lane j scores position j against every query head of the kv head (dp4a);
// the weights go through shared memory and each lane accumulates P.V for its
// HD/32 dims of every head. The warps merge at the end; partials (m, l, o)
// per split, and the last CTA of (sequence, kv head) merges the splits.
namespace jyc {
namespace {


template <int HD>
__device__ __forceinline__ int bd_rot(int j) {
    return HD == 64 ? ((j >> 1) & 3) : (j & 7);  // 16-byte chunk rotation of row j
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Per-warp shared memory: K and V tiles [2 buffers][32 rows][HD] (16-byte
// chunks rotated by bd_rot) and the tile's weights [32][8 heads].
template <int HD>
constexpr int bd_warp_bytes() {
    return 4 * 32 * HD + 32 * 8 * 4;
}

template <int HD, int NW>
__global__ void __launch_bounds__(NW * 32) bd_attention_kernel(BdAttn a) {
    constexpr int NCH = HD / 16, DPL = HD / 32, MAXG = 8;
    extern __shared__ __align__(16) unsigned char bd_sm[];
    const int G = a.H / a.KV;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int8_t* sq = reinterpret_cast<int8_t*>(bd_sm);  // [G][HD] queries (<= 1 KB)
    float* sqs = reinterpret_cast<float*>(bd_sm + 1024);
    unsigned char* wb = bd_sm + 1024 + 64 + warp * bd_warp_bytes<HD>();
    int8_t* sk = reinterpret_cast<int8_t*>(wb);                // [2][32][HD]
    int8_t* sv = sk + 2 * 32 * HD;                             // [2][32][HD]
    float* sp = reinterpret_cast<float*>(sv + 2 * 32 * HD);   // [32][MAXG]

    const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int pos_last = a.lens[b] - 1;
    const int c0 = split * a.chunk, c1 = min(c0 + a.chunk, pos_last + 1);
    const size_t hq = (size_t)b * a.H + (size_t)kvh * G;  // first query head row of this CTA

    if (c0 <= pos_last) {
        for (int e = tid; e < G * HD / 16; e += NW * 32)
            reinterpret_cast<uint4*>(sq)[e] = __ldg(reinterpret_cast<const uint4*>(a.q8 + hq * HD) + e);
        if (tid < G) sqs[tid] = __ldg(a.qsc + hq + tid);
        __syncthreads();
        const int8_t* kb = a.k8 + (size_t)b * a.slot_q + (size_t)kvh * a.cap * HD;
        const int8_t* vb = a.v8 + (size_t)b * a.slot_q + (size_t)kvh * a.cap * HD;
        const float* ksb = a.ks + (size_t)b * a.slot_s + (size_t)kvh * a.cap;
        const float* vsb = a.vs + (size_t)b * a.slot_s + (size_t)kvh * a.cap;
        // this warp's positions [w0, w1)
        const int per = a.chunk / NW, w0 = c0 + warp * per, w1 = min(w0 + per, c1);
        const int ntile = w1 > w0 ? (w1 - w0 + 31) / 32 : 0;
        // lane j copies row j of tile t (one commit group per call, empty past the end)
        auto issue = [&](int t, int buf) {
            const int j = w0 + 32 * t + lane;
            if (t < ntile && j < w1) {
#pragma unroll
                for (int c = 0; c < NCH; c++) {
                    const int ph = ((c + bd_rot<HD>(lane)) & (NCH - 1)) * 16;
                    cp_async16(sk + (buf * 32 + lane) * HD + ph, kb + (size_t)j * HD + c * 16);
                    cp_async16(sv + (buf * 32 + lane) * HD + ph, vb + (size_t)j * HD + c * 16);
                }
            }
            cp_async_commit();
        };
        float m[MAXG], l[MAXG], o[MAXG][DPL];
#pragma unroll
        for (int g = 0; g < MAXG; g++) {
            m[g] = -INFINITY;
            l[g] = 0.0f;
#pragma unroll
            for (int i = 0; i < DPL; i++) o[g][i] = 0.0f;
        }
        issue(0, 0);
        float ksn = 0.0f, vsn = 0.0f;
        if (ntile > 0 && w0 + lane < w1) {
            ksn = __ldg(ksb + w0 + lane);
            vsn = __ldg(vsb + w0 + lane);
        }
        for (int t = 0; t < ntile; t++) {
            const int buf = t & 1, jt = w0 + 32 * t, nj = min(32, w1 - jt);
            issue(t + 1, buf ^ 1);
            const float ksc = ksn, vsc = vsn;
            if (t + 1 < ntile && jt + 32 + lane < w1) {
                ksn = __ldg(ksb + jt + 32 + lane);
                vsn = __ldg(vsb + jt + 32 + lane);
            }
            cp_async_wait<1>();
            __syncwarp();
            // scores of position jt + lane for every head, online softmax per head
            const uint4* krow = reinterpret_cast<const uint4*>(sk + (buf * 32 + lane) * HD);
            uint4 kr[NCH];
#pragma unroll
            for (int c = 0; c < NCH; c++) kr[c] = krow[(c + bd_rot<HD>(lane)) & (NCH - 1)];
            float pw[MAXG];
#pragma unroll
            for (int g = 0; g < MAXG; g++) {
                pw[g] = 0.0f;
                if (g >= G) continue;
                const uint4* qrow = reinterpret_cast<const uint4*>(sq + g * HD);
                int dot = 0;
#pragma unroll
                for (int c = 0; c < NCH; c++) {
                    const uint4 qw = qrow[c];
                    dot = __dp4a((int)qw.x, (int)kr[c].x, dot);
                    dot = __dp4a((int)qw.y, (int)kr[c].y, dot);
                    dot = __dp4a((int)qw.z, (int)kr[c].z, dot);
                    dot = __dp4a((int)qw.w, (int)kr[c].w, dot);
                }
                const float sc = lane < nj ? __fmul_rn((float)dot, __fmul_rn(__fmul_rn(ksc, sqs[g]), a.scale))
                                           : -INFINITY;
                const float mn = fmaxf(m[g], warp_max(sc));
                const float e = sc == -INFINITY ? 0.0f : expf(sc - mn);
                const float al = m[g] == -INFINITY ? 0.0f : expf(m[g] - mn);
                m[g] = mn;
                l[g] = l[g] * al + e;  // per-lane share, summed over lanes at the end
#pragma unroll
                for (int i = 0; i < DPL; i++) o[g][i] = __fmul_rn(o[g][i], al);
                pw[g] = e * vsc;
            }
            *reinterpret_cast<float4*>(sp + lane * MAXG) = make_float4(pw[0], pw[1], pw[2], pw[3]);
            if (G > 4) *reinterpret_cast<float4*>(sp + lane * MAXG + 4) = make_float4(pw[4], pw[5], pw[6], pw[7]);
            __syncwarp();
            // P.V: lane owns dims [DPL lane, DPL lane + DPL) of every head
            const int c = (DPL * lane) >> 4, off = (DPL * lane) & 15;
            for (int jj = 0; jj < nj; jj++) {
                const int8_t* vr = sv + (buf * 32 + jj) * HD + ((c + bd_rot<HD>(jj)) & (NCH - 1)) * 16 + off;
                float f[4];
                if (DPL == 4) {
                    u8x4_to_f32(*reinterpret_cast<const uint32_t*>(vr) ^ 0x80808080u, f);
                } else {
                    u8x4_to_f32((uint32_t)(*reinterpret_cast<const uint16_t*>(vr)) ^ 0x80808080u, f);
                }
                const float4 p0 = *reinterpret_cast<const float4*>(sp + jj * MAXG);
                const float pg[4] = {p0.x, p0.y, p0.z, p0.w};
#pragma unroll
                for (int g = 0; g < 4; g++)
#pragma unroll
                    for (int i = 0; i < DPL; i++) o[g][i] = __fmaf_rn(pg[g], f[i], o[g][i]);
                if (G > 4) {
                    const float4 p1 = *reinterpret_cast<const float4*>(sp + jj * MAXG + 4);
                    const float ph[4] = {p1.x, p1.y, p1.z, p1.w};
#pragma unroll
                    for (int g = 0; g < 4; g++)
#pragma unroll
                        for (int i = 0; i < DPL; i++) o[4 + g][i] = __fmaf_rn(ph[g], f[i], o[4 + g][i]);
                }
            }
            __syncwarp();  // the next iteration's copies overwrite this buffer
        }
        cp_async_wait<0>();
        // merge the warps: (m, l, o) per warp -> shared memory, then per head
#pragma unroll
        for (int g = 0; g < MAXG; g++) l[g] = warp_sum(l[g]);
        __syncthreads();  // every warp is done with its tiles: reuse the area
        float* mw = reinterpret_cast<float*>(bd_sm + 1024 + 64);  // [NW][MAXG]
        float* lw = mw + NW * MAXG;                                // [NW][MAXG]
        float* ow = lw + NW * MAXG;                                // [NW][G][HD]
        if (lane < MAXG) {
            float mv = m[0], lv = l[0];
#pragma unroll
            for (int g = 1; g < MAXG; g++)
                if (lane == g) {
                    mv = m[g];
                    lv = l[g];
                }
            mw[warp * MAXG + lane] = mv;
            lw[warp * MAXG + lane] = lv;
        }
#pragma unroll
        for (int g = 0; g < MAXG; g++)
            if (g < G)
#pragma unroll
                for (int i = 0; i < DPL; i++) ow[(warp * G + g) * HD + DPL * lane + i] = o[g][i];
        __syncthreads();
        for (int e = tid; e < G * HD; e += NW * 32) {
            const int g = e / HD, d = e % HD;
            float M = -INFINITY;
            for (int w = 0; w < NW; w++) M = fmaxf(M, mw[w * MAXG + g]);
            float L = 0.0f, O = 0.0f;
            for (int w = 0; w < NW; w++) {
                const float mv = mw[w * MAXG + g];
                if (mv == -INFINITY) continue;
                const float wgt = expf(mv - M);
                L = __fmaf_rn(wgt, lw[w * MAXG + g], L);
                O = __fmaf_rn(wgt, ow[(w * G + g) * HD + d], O);
            }
            a.part_o[((hq + g) * a.nsplit + split) * HD + d] = O;
            if (d == 0) {
                a.part_ml[((hq + g) * a.nsplit + split) * 2] = M;
                a.part_ml[((hq + g) * a.nsplit + split) * 2 + 1] = L;
            }
        }
    }

    // arrival; the last CTA of (sequence, kv head) merges the splits
    __shared__ unsigned int s_last;
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const unsigned int prev = atomicAdd(&a.arrive[(size_t)b * a.KV + kvh], 1u);
        s_last = (prev == gridDim.x - 1) ? 1u : 0u;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const int nvalid = pos_last / a.chunk + 1;
    for (int e = tid; e < G * HD; e += NW * 32) {
        const int g = e / HD, d = e % HD;
        const size_t base = (hq + g) * a.nsplit;
        float M = -INFINITY;
        for (int s2 = 0; s2 < nvalid; s2++) M = fmaxf(M, __ldcg(a.part_ml + (base + s2) * 2));
        float L = 0.0f, O = 0.0f;
        for (int s2 = 0; s2 < nvalid; s2++) {
            const float ms = __ldcg(a.part_ml + (base + s2) * 2);
            if (ms == -INFINITY) continue;
            const float wgt = expf(ms - M);
            L = __fmaf_rn(wgt, __ldcg(a.part_ml + (base + s2) * 2 + 1), L);
            O = __fmaf_rn(wgt, __ldcg(a.part_o + (base + s2) * HD + d), O);
        }
        a.out[(size_t)b * a.ldo + (size_t)(kvh * G + g) * HD + d] = O / L;
    }
    if (tid == 0) a.arrive[(size_t)b * a.KV + kvh] = 0u;
}

constexpr int kBdWarps = 8;  // warps per CTA

int bd_attn_smem(int hd) {
    const int warps = 1024 + 64 + kBdWarps * (hd == 64 ? bd_warp_bytes<64>() : bd_warp_bytes<128>());
    const int merge = 1024 + 64 + (2 * kBdWarps * 8 + kBdWarps * 8 * hd) * 4;
    return warps > merge ? warps : merge;
}

}  // namespace

bool bd_attention_supported(int H, int KV, int hd) {
    const int G = KV > 0 ? H / KV : 0;
    return (hd == 64 || hd == 128) && KV > 0 && H % KV == 0 && G >= 1 && G <= 8;
}

int bd_attention_chunk(int cap, int nseq, int KV) {
    // about three CTAs per SM over (split, kv head, sequence); a chunk is a
    // whole number of 32-position tiles for each of the kBdWarps warps
    constexpr int q = 32 * kBdWarps;
    const long long target = 3LL * 148;
    long long chunk = ((long long)cap * nseq * KV + target - 1) / target;
    chunk = (chunk + q - 1) / q * q;
    return (int)std::max<long long>(q, std::min<long long>(chunk, ((long long)cap + q - 1) / q * q));
}

int launch_bd_attention(const BdAttn& a, int nseq, cudaStream_t s) {
    if (!bd_attention_supported(a.H, a.KV, a.hd)) return arg_error("bd_attention: unsupported head shape");
    if (a.chunk % (32 * kBdWarps)) return arg_error("bd_attention: chunk must be a multiple of 256");
    // once per process (thread-safe static initialisation)
    static const cudaError_t attr = [] {
        cudaError_t e = cudaFuncSetAttribute(bd_attention_kernel<64, kBdWarps>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, bd_attn_smem(64));
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(bd_attention_kernel<128, kBdWarps>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     bd_attn_smem(128));
        return e;
    }();
    if (attr != cudaSuccess) return cuda_fail(attr, "cudaFuncSetAttribute");
    const dim3 grid(a.nsplit, a.KV, nseq);
    if (a.hd == 64) bd_attention_kernel<64, kBdWarps><<<grid, kBdWarps * 32, bd_attn_smem(64), s>>>(a);
    else bd_attention_kernel<128, kBdWarps><<<grid, kBdWarps * 32, bd_attn_smem(128), s>>>(a);
    JYC_LAUNCHED();
    return JYC_OK;
}

}  // namespace jyc
