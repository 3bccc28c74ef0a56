// prefill.cu — causal attention of a prompt chunk for the batched prefill
// (the matmuls of prefill run on the tcgen05 tiles of tcgemm.cu).
#include <algorithm>

#include "mega.cuh"
#include "prefill.cuh"
#include "ptx.cuh"

namespace jyc {

int prepare_pf_attention();

int prepare_pf_kernels() { return prepare_pf_attention(); }

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
    // this CTA: query heads [g0, g0 + Gv) of kv head blockIdx.x (Gc per CTA)
    const int G = a.H / a.KV, Gc = a.gc, g0 = blockIdx.z * Gc, Gv = min(Gc, G - g0), RW = 2 * Gc;
    int8_t* s_k = reinterpret_cast<int8_t*>(pf_sm);                 // [kKB][HD]
    int8_t* s_v = s_k + kKB * HD;                                    // [kKB][HD]
    float* s_ks = reinterpret_cast<float*>(s_v + kKB * HD);          // [kKB]
    float* s_vs = s_ks + kKB;                                        // [kKB]
    float* s_pb = s_vs + kKB;                                        // [8][MAXR][kKB]
    int8_t* s_q = reinterpret_cast<int8_t*>(s_pb + 8 * MAXR * kKB);  // [16 * Gc][HD]
    auto s_p = [&](int w, int r, int j) -> float& { return s_pb[(w * MAXR + r) * kKB + j]; };
    const int kvh = blockIdx.x, t0 = blockIdx.y * kPfQT;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int q_dim = a.H * HD;
    const int nt = min(kPfQT, a.T - t0);
    // queries of this CTA: row r = t * Gc + gl (head g0 + gl)
    for (int e = tid; e < nt * Gc * HW; e += 256) {
        const int r = e / HW, wd = e - r * HW, t = r / Gc, gl = r - t * Gc;
        reinterpret_cast<uint32_t*>(s_q)[e] =
            gl < Gv ? __ldg(reinterpret_cast<const uint32_t*>(a.q8 + (size_t)(t0 + t) * q_dim +
                                                              (kvh * G + g0 + gl) * HD) + wd)
                    : 0u;
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
        const int rr = warp * RW + r, t = rr / Gc, gl = rr - t * Gc;
        const bool real = r < RW && t < nt && gl < Gv;
        pos_r[r] = real ? a.pos0 + t0 + t : -1;  // -1: no query row
        qs_r[r] = real ? __ldg(a.qsc + (size_t)(t0 + t) * a.H + kvh * G + g0 + gl) : 0.0f;
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
        const int rr = warp * RW + r, t = rr / Gc, gl = rr - t * Gc;
        const float inv = 1.0f / l_r[r];
        float* o = a.out + (size_t)(t0 + t) * q_dim + (kvh * G + g0 + gl) * HD + DPL * lane;
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

int launch_pf_attention(const PfAttn& a_in, cudaStream_t s) {
    if (!pf_attention_supported(a_in.H, a_in.KV, a_in.hd)) return arg_error("pf_attention: unsupported head shape");
    PfAttn a = a_in;
    const int G = a.H / a.KV, ntb = (a.T + kPfQT - 1) / kPfQT;
    // query heads per CTA: the most that still give two CTAs per SM (K/V rows
    // are read once per CTA), else one
    const int want = 2 * mega_num_ctas();
    a.gc = 1;
    for (int gc = G; gc >= 1; gc--)
        if (a.KV * ntb * ((G + gc - 1) / gc) >= want) {
            a.gc = gc;
            break;
        }
    const dim3 grid(a.KV, ntb, (G + a.gc - 1) / a.gc);
    const int maxr = a.gc <= 2 ? 4 : a.gc <= 4 ? 8 : 16;
    const int smem = pf_attn_smem(a.hd, a.gc, maxr);
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
