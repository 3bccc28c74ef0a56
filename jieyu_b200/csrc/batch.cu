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
// into the weights). CTA = (position split, kv head, sequence), 256 threads.
// Per block of 128 positions: K and V rows arrive with 16-byte cp.async into
// a double buffer (16-byte chunks rotated per row so that row-parallel reads
// are free of bank conflicts); each thread scores one position against up to
// half the query heads (dp4a); one warp per head runs the online softmax; P.V
// gives each thread 4 output dims of one head over a share of the positions.
// Partials (m, l, o) per split; the last CTA of (sequence, kv head) merges.
namespace jyc {
namespace {

constexpr int kBdKB = 128;    // positions per block
constexpr int kBdStages = 3;  // blocks in the cp.async ring (two in flight while one is used)

template <int HD>
__device__ __forceinline__ int bd_rot(int j) {
    return HD == 64 ? ((j >> 1) & 3) : (j & 7);  // 16-byte chunk rotation of row j
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <int HD>
__global__ void __launch_bounds__(256) bd_attention_kernel(BdAttn a) {
    constexpr int KB = kBdKB, NCH = HD / 16;
    extern __shared__ __align__(16) unsigned char bd_sm[];
    const int G = a.H / a.KV;
    int8_t* sk = reinterpret_cast<int8_t*>(bd_sm);                    // [kBdStages][KB][HD]
    int8_t* sv = sk + kBdStages * KB * HD;                              // [kBdStages][KB][HD]
    float* sks = reinterpret_cast<float*>(sv + kBdStages * KB * HD);    // [kBdStages][KB]
    float* svs = sks + kBdStages * KB;                                  // [kBdStages][KB]
    float* sp = svs + kBdStages * KB;                                   // [G][KB] scores, then weights
    float* sred = sp + G * KB;                                  // [256 / NQ][G * HD] P.V partials
    int8_t* sq = reinterpret_cast<int8_t*>(sred + 256 * 4);     // [G][HD]
    float* sqs = reinterpret_cast<float*>(sq + G * HD);         // [G]
    float* s_m = sqs + G;
    float* s_l = s_m + G;
    float* s_al = s_l + G;

    const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z, tid = threadIdx.x, lane = tid & 31,
              warp = tid >> 5;
    const int pos_last = a.lens[b] - 1;
    const int c0 = split * a.chunk, c1 = min(c0 + a.chunk, pos_last + 1);
    const int NQ = G * HD / 4, NJG = 256 / NQ;  // output quads; position groups of P.V
    const int q = tid % NQ, jg = tid / NQ, g_pv = (4 * q) / HD, d0 = (4 * q) % HD;
    float o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    const size_t hq = (size_t)b * a.H + (size_t)kvh * G;  // first query head row of this CTA

    if (c0 <= pos_last) {
        for (int e = tid; e < G * HD / 16; e += 256)
            reinterpret_cast<uint4*>(sq)[e] = __ldg(reinterpret_cast<const uint4*>(a.q8 + hq * HD) + e);
        if (tid < G) {
            sqs[tid] = __ldg(a.qsc + hq + tid);
            s_m[tid] = -INFINITY;
            s_l[tid] = 0.0f;
        }
        const int8_t* kb = a.k8 + (size_t)b * a.slot_q + (size_t)kvh * a.cap * HD;
        const int8_t* vb = a.v8 + (size_t)b * a.slot_q + (size_t)kvh * a.cap * HD;
        const float* ksb = a.ks + (size_t)b * a.slot_s + (size_t)kvh * a.cap;
        const float* vsb = a.vs + (size_t)b * a.slot_s + (size_t)kvh * a.cap;
        // one commit group per call (empty past the end) keeps the group count uniform
        auto issue = [&](int j0, int buf) {
            const int nj = j0 < c1 ? min(KB, c1 - j0) : 0;
            for (int e = tid; e < nj * NCH; e += 256) {
                const int j = e / NCH, c = e % NCH, ph = ((c + bd_rot<HD>(j)) & (NCH - 1)) * 16;
                cp_async16(sk + (buf * KB + j) * HD + ph, kb + (size_t)(j0 + j) * HD + c * 16);
                cp_async16(sv + (buf * KB + j) * HD + ph, vb + (size_t)(j0 + j) * HD + c * 16);
            }
            for (int j = tid; j < nj; j += 256) {
                cp_async4(sks + buf * KB + j, ksb + j0 + j);
                cp_async4(svs + buf * KB + j, vsb + j0 + j);
            }
            cp_async_commit();
        };
#pragma unroll
        for (int st = 0; st < kBdStages - 1; st++) issue(c0 + st * KB, st);
        int buf = 0;
        for (int j0 = c0; j0 < c1; j0 += KB, buf = (buf + 1) % kBdStages) {
            const int nj = min(KB, c1 - j0);
            issue(j0 + (kBdStages - 1) * KB, (buf + kBdStages - 1) % kBdStages);
            cp_async_wait<kBdStages - 1>();  // block j0's group (and every older one) has landed
            __syncthreads();  // ... for every thread
            // scores: thread -> position j, heads hh, hh + 2, ...
            {
                const int j = tid & (KB - 1), hh = tid >> 7;
                const uint4* krow = reinterpret_cast<const uint4*>(sk + (buf * KB + j) * HD);
                for (int g = hh; g < G; g += 2) {
                    float sc = -INFINITY;
                    if (j < nj) {
                        const uint4* qrow = reinterpret_cast<const uint4*>(sq + g * HD);
                        int dot = 0;
#pragma unroll
                        for (int c = 0; c < NCH; c++) {
                            const uint4 kw = krow[(c + bd_rot<HD>(j)) & (NCH - 1)];
                            const uint4 qw = qrow[c];
                            dot = __dp4a((int)qw.x, (int)kw.x, dot);
                            dot = __dp4a((int)qw.y, (int)kw.y, dot);
                            dot = __dp4a((int)qw.z, (int)kw.z, dot);
                            dot = __dp4a((int)qw.w, (int)kw.w, dot);
                        }
                        sc = __fmul_rn((float)dot, __fmul_rn(__fmul_rn(sks[buf * KB + j], sqs[g]), a.scale));
                    }
                    sp[g * KB + j] = sc;
                }
            }
            __syncthreads();
            // online softmax: warp g takes head g
            for (int g = warp; g < G; g += 8) {
                float v[KB / 32];
                float mx = -INFINITY;
#pragma unroll
                for (int i = 0; i < KB / 32; i++) {
                    v[i] = sp[g * KB + 32 * i + lane];
                    mx = fmaxf(mx, v[i]);
                }
                mx = warp_max(mx);
                const float m_old = s_m[g], m_new = fmaxf(m_old, mx);
                float sum = 0.0f;
#pragma unroll
                for (int i = 0; i < KB / 32; i++) {
                    const int j = 32 * i + lane;
                    const float e = v[i] == -INFINITY ? 0.0f : expf(v[i] - m_new);
                    sum += e;
                    sp[g * KB + j] = e * (j < nj ? svs[buf * KB + j] : 0.0f);
                }
                sum = warp_sum(sum);
                if (lane == 0) {
                    const float al = m_old == -INFINITY ? 0.0f : expf(m_old - m_new);
                    s_al[g] = al;
                    s_l[g] = s_l[g] * al + sum;
                    s_m[g] = m_new;
                }
            }
            __syncthreads();
            // P.V: 4 dims of head g_pv over positions jg, jg + NJG, ...
            if (jg < NJG) {
                const float al = s_al[g_pv];
#pragma unroll
                for (int i = 0; i < 4; i++) o[i] = __fmul_rn(o[i], al);
                const int c = d0 >> 4, w4 = d0 & 15;
                for (int j = jg; j < nj; j += NJG) {
                    const int8_t* vr = sv + (buf * KB + j) * HD + ((c + bd_rot<HD>(j)) & (NCH - 1)) * 16 + w4;
                    float f[4];
                    u8x4_to_f32(*reinterpret_cast<const uint32_t*>(vr) ^ 0x80808080u, f);
                    const float p = sp[g_pv * KB + j];
#pragma unroll
                    for (int i = 0; i < 4; i++) o[i] = __fmaf_rn(p, f[i], o[i]);
                }
            }
            __syncthreads();  // buffers and weights are reused by the next block
        }
        // sum the position groups' P.V partials
        if (jg < NJG) *reinterpret_cast<float4*>(sred + jg * G * HD + 4 * q) = make_float4(o[0], o[1], o[2], o[3]);
        __syncthreads();
        for (int e = tid; e < G * HD; e += 256) {
            float acc = 0.0f;
            for (int z = 0; z < NJG; z++) acc += sred[z * G * HD + e];
            const int g = e / HD, d = e % HD;
            a.part_o[((hq + g) * a.nsplit + split) * HD + d] = acc;
        }
        if (tid < G) {
            a.part_ml[((hq + tid) * a.nsplit + split) * 2] = s_m[tid];
            a.part_ml[((hq + tid) * a.nsplit + split) * 2 + 1] = s_l[tid];
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
    for (int e = tid; e < G * HD; e += 256) {
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

int bd_attn_smem(int hd, int G) {
    return 2 * kBdStages * kBdKB * hd + 2 * kBdStages * kBdKB * 4 + G * kBdKB * 4 + 256 * 4 * 4 + G * hd + 4 * G * 4;
}

}  // namespace

bool bd_attention_supported(int H, int KV, int hd) {
    const int G = KV > 0 ? H / KV : 0;
    return (hd == 64 || hd == 128) && KV > 0 && H % KV == 0 && G >= 1 && G <= 8 && (G * hd) % 64 == 0;
}

int bd_attention_chunk(int cap, int nseq, int KV) {
    const long long target = 3LL * 148;
    long long chunk = ((long long)cap * nseq * KV + target - 1) / target;
    chunk = (chunk + kBdKB - 1) / kBdKB * kBdKB;
    return (int)std::max<long long>(kBdKB, std::min<long long>(chunk, ((long long)cap + kBdKB - 1) / kBdKB * kBdKB));
}

int launch_bd_attention(const BdAttn& a, int nseq, cudaStream_t s) {
    if (!bd_attention_supported(a.H, a.KV, a.hd)) return arg_error("bd_attention: unsupported head shape");
    if (a.chunk % kBdKB) return arg_error("bd_attention: chunk must be a multiple of 128");
    const int G = a.H / a.KV, smem = bd_attn_smem(a.hd, G);
    static bool attr = false;
    if (!attr) {
        JYC_CUDA(cudaFuncSetAttribute(bd_attention_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      bd_attn_smem(64, 8)));
        JYC_CUDA(cudaFuncSetAttribute(bd_attention_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      bd_attn_smem(128, 8)));
        attr = true;
    }
    const dim3 grid(a.nsplit, a.KV, nseq);
    if (a.hd == 64) bd_attention_kernel<64><<<grid, 256, smem, s>>>(a);
    else bd_attention_kernel<128><<<grid, 256, smem, s>>>(a);
    JYC_LAUNCHED();
    return JYC_OK;
}

}  // namespace jyc
