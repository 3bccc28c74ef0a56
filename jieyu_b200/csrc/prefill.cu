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
// attention of transformer_layer for seq > 1, transformer_layer.h:35-70;
// attention_q8.h:38-184 for the score scaling dot * ((ks * qs) * 1/sqrt(hd)),
// fp32 softmax, and P.V with the V scale folded into P), on the tensor cores.
// CTA = (kv head, 16 query tokens, a group of gc query heads); warp w takes
// query head g0 + w for the 16 tokens (the 16 rows of an m16 tile). Per block
// of 64 keys: K (int8, 16-byte chunks swizzled by key) and V (int8, turned
// into fp16 in shared memory for ldmatrix.trans) arrive once for all warps;
// scores Q.K^T with mma.m16n8k32 s8 (exact int32 dots, Q fragments held in
// registers for the whole kernel), online softmax per row in registers; the
// weights p * vs (scaled by 2^S per block so that fp16 keeps them normal)
// become the A fragments of mma.m16n8k16 f16 without leaving registers, as an
// exact hi + lo pair of fp16 (22 significant bits); V (int8) is exact in
// fp16. Each block's P.V product starts from zero and is added to the fp32
// output accumulators with round to nearest (the online rescale's fma), so
// the tensor cores' own accumulation spans at most one block.
namespace {

constexpr int kKB = 64;  // keys per block

__device__ __forceinline__ void mma_s8_16832(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                             uint32_t b1, int (&c)[4]) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_f16_16816(const uint32_t (&a)[4], uint32_t b0, uint32_t b1, float (&c)[4]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4_trans(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void cp16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
// fp32 x -> fp16 hi + lo with hi + lo = x to 22 bits (lo: the rounded residual)
__device__ __forceinline__ void split_f16(float x, __half& hi, __half& lo) {
    hi = __float2half_rn(x);
    lo = __float2half_rn(__fsub_rn(x, __half2float(hi)));
}
__device__ __forceinline__ uint32_t pack_h2(__half a, __half b) {
    return (uint32_t)__half_as_ushort(a) | ((uint32_t)__half_as_ushort(b) << 16);
}

// 16-byte chunk c of key row j: K rows hold HD/16 chunks, V (fp16) rows HD/8
template <int NCH>
__device__ __forceinline__ int swz(int c, int j) {
    return NCH >= 8 ? (c ^ (j & 7)) : (c ^ ((j >> 1) & (NCH - 1)));
}

template <int HD>
constexpr int pf_smem_bytes() {
    return kKB * HD /* K */ + kKB * HD /* V int8 staging */ + kKB * HD * 2 /* V fp16 */ + 2 * kKB * 4;
}

template <int HD>
__global__ void __launch_bounds__(256) pf_attention_kernel(PfAttn a) {
    constexpr int NKS = HD / 32;   // int8 k-steps of Q.K^T
    constexpr int KCH = HD / 16;   // 16-byte chunks of a K row
    constexpr int VCH = HD / 8;    // 16-byte chunks of an fp16 V row
    constexpr int NDT = HD / 8;    // n8 tiles of output dims
    extern __shared__ __align__(128) unsigned char pf_sm[];
    int8_t* s_k = reinterpret_cast<int8_t*>(pf_sm);                      // [kKB][HD]
    int8_t* s_vr = s_k + kKB * HD;                                        // [kKB][HD] int8
    __half* s_v = reinterpret_cast<__half*>(s_vr + kKB * HD);             // [kKB][HD] fp16
    float* s_ks = reinterpret_cast<float*>(s_v + kKB * HD);               // [kKB]
    float* s_vs = s_ks + kKB;                                             // [kKB]

    const int G = a.H / a.KV, g0 = blockIdx.z * a.gc;
    const int kvh = blockIdx.x, t0 = blockIdx.y * kPfQT;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nthr = blockDim.x;
    const int gq = lane >> 2, tq = lane & 3;
    const int q_dim = a.H * HD;
    const int nt = min(kPfQT, a.T - t0);
    const int hl = g0 + warp;                 // this warp's query head within the kv head
    const bool hv = hl < G;
    const int h = kvh * G + (hv ? hl : 0);
    // rows gq and gq + 8 of the tile = tokens t0 + gq, t0 + gq + 8
    const bool r0v = hv && gq < nt, r1v = hv && gq + 8 < nt;
    const int p0 = a.pos0 + t0 + gq, p1 = p0 + 8;
    uint32_t qa[NKS][4];
    {
        const int8_t* q0 = a.q8 + (size_t)(t0 + gq) * q_dim + (size_t)h * HD;
        const int8_t* q1 = q0 + (size_t)8 * q_dim;
#pragma unroll
        for (int ks = 0; ks < NKS; ks++) {
            qa[ks][0] = r0v ? __ldg(reinterpret_cast<const uint32_t*>(q0 + ks * 32 + 4 * tq)) : 0u;
            qa[ks][1] = r1v ? __ldg(reinterpret_cast<const uint32_t*>(q1 + ks * 32 + 4 * tq)) : 0u;
            qa[ks][2] = r0v ? __ldg(reinterpret_cast<const uint32_t*>(q0 + ks * 32 + 16 + 4 * tq)) : 0u;
            qa[ks][3] = r1v ? __ldg(reinterpret_cast<const uint32_t*>(q1 + ks * 32 + 16 + 4 * tq)) : 0u;
        }
    }
    const float qs0 = r0v ? __ldg(a.qsc + (size_t)(t0 + gq) * a.H + h) : 0.0f;
    const float qs1 = r1v ? __ldg(a.qsc + (size_t)(t0 + gq + 8) * a.H + h) : 0.0f;
    const int8_t* kb = a.k8 + (size_t)kvh * a.max_seq * HD;
    const int8_t* vb = a.v8 + (size_t)kvh * a.max_seq * HD;
    const float* ksb = a.ks + (size_t)kvh * a.max_seq;
    const float* vsb = a.vs + (size_t)kvh * a.max_seq;
    const int kend = a.pos0 + t0 + nt;  // keys 0 .. kend-1

    float o[NDT][4];
#pragma unroll
    for (int d = 0; d < NDT; d++) o[d][0] = o[d][1] = o[d][2] = o[d][3] = 0.0f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;  // l: this lane's share of the row sums

    for (int j0 = 0; j0 < kend; j0 += kKB) {
        const int nk = min(kKB, kend - j0);
        __syncthreads();  // every warp is done with the previous block
        for (int e = tid; e < nk * KCH; e += nthr) {
            const int j = e / KCH, c = e - j * KCH;
            cp16(s_k + j * HD + swz<KCH>(c, j) * 16, kb + (size_t)(j0 + j) * HD + c * 16);
            cp16(s_vr + j * HD + c * 16, vb + (size_t)(j0 + j) * HD + c * 16);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
        for (int j = tid; j < kKB; j += nthr) {
            s_ks[j] = j < nk ? __ldcg(ksb + j0 + j) : 0.0f;
            s_vs[j] = j < nk ? __ldcg(vsb + j0 + j) : 0.0f;
        }
        asm volatile("cp.async.wait_group 0;" ::: "memory");
        __syncthreads();
        // V to fp16 (exact), 8 values per thread and step; rows past nk are zero
        for (int e = tid; e < kKB * VCH; e += nthr) {
            const int j = e / VCH, c = e - j * VCH;
            uint4 out = make_uint4(0u, 0u, 0u, 0u);
            if (j < nk) {
                const uint2 w = *reinterpret_cast<const uint2*>(s_vr + j * HD + c * 8);
                float f[8];
                u8x4_to_f32(w.x ^ 0x80808080u, f);
                u8x4_to_f32(w.y ^ 0x80808080u, f + 4);
                out.x = pack_h2(__float2half_rn(f[0]), __float2half_rn(f[1]));
                out.y = pack_h2(__float2half_rn(f[2]), __float2half_rn(f[3]));
                out.z = pack_h2(__float2half_rn(f[4]), __float2half_rn(f[5]));
                out.w = pack_h2(__float2half_rn(f[6]), __float2half_rn(f[7]));
            }
            *reinterpret_cast<uint4*>(s_v + j * HD + swz<VCH>(c, j) * 8) = out;
        }
        __syncthreads();
        if (!hv) continue;
        // block scale 2^S: max(vs) * 2^S in [2^13, 2^14) keeps every weight p * vs * 2^S
        // (p <= 1) below fp16's maximum and normal down to 2^-27 of the largest
        float vmax = fmaxf(s_vs[lane], s_vs[lane + 32]);
        vmax = warp_max(vmax);
        const int S = vmax > 0.0f ? 13 - ilogbf(vmax) : 0;
        const float up = ldexpf(1.0f, S), down = ldexpf(1.0f, -S);

        // scores: 8 tiles of 8 keys; the causal edge masks keys past a row's position
        float sc[8][4];
        const int last_key = min(p1, kend - 1);  // the largest key any row of this warp may see
#pragma unroll
        for (int nt8 = 0; nt8 < 8; nt8++) {
            const int n0 = nt8 * 8;
            int c[4] = {0, 0, 0, 0};
            if (j0 + n0 <= last_key && n0 < nk) {
                const int8_t* krow = s_k + (n0 + gq) * HD;
#pragma unroll
                for (int ks = 0; ks < NKS; ks++) {
                    const uint32_t b0 = *reinterpret_cast<const uint32_t*>(krow + swz<KCH>(2 * ks, n0 + gq) * 16 + 4 * tq);
                    const uint32_t b1 =
                        *reinterpret_cast<const uint32_t*>(krow + swz<KCH>(2 * ks + 1, n0 + gq) * 16 + 4 * tq);
                    mma_s8_16832(qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b0, b1, c);
                }
            }
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int kj = n0 + 2 * tq + (e & 1), key = j0 + kj;
                const bool lo_row = e < 2;
                const int pr = lo_row ? p0 : p1;
                const bool ok = (lo_row ? r0v : r1v) && kj < nk && key <= pr;
                sc[nt8][e] = ok ? __fmul_rn((float)c[e], __fmul_rn(__fmul_rn(s_ks[kj], lo_row ? qs0 : qs1), a.scale))
                                : -INFINITY;
            }
        }
        // online softmax per row (a row's 64 scores live in the 4 lanes of its quad)
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int nt8 = 0; nt8 < 8; nt8++) {
            mx0 = fmaxf(mx0, fmaxf(sc[nt8][0], sc[nt8][1]));
            mx1 = fmaxf(mx1, fmaxf(sc[nt8][2], sc[nt8][3]));
        }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
        const float al0 = (m0 == -INFINITY) ? 0.0f : expf(m0 - mn0);
        const float al1 = (m1 == -INFINITY) ? 0.0f : expf(m1 - mn1);
        m0 = mn0;
        m1 = mn1;
        // weights -> A fragments (hi, lo) of the four 16-key steps
        uint32_t ph[4][4], pl[4][4];
        float ps0 = 0.0f, ps1 = 0.0f;
#pragma unroll
        for (int nt8 = 0; nt8 < 8; nt8++) {
            __half hi[4], lo[4];
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const float sv = sc[nt8][e];
                const float pe = sv == -INFINITY ? 0.0f : expf(sv - (e < 2 ? mn0 : mn1));
                if (e < 2)
                    ps0 += pe;
                else
                    ps1 += pe;
                const float w = __fmul_rn(__fmul_rn(pe, s_vs[nt8 * 8 + 2 * tq + (e & 1)]), up);
                split_f16(w, hi[e], lo[e]);
            }
            const int ks16 = nt8 >> 1, hf = nt8 & 1;  // tile 2i -> a0, a1; tile 2i+1 -> a2, a3
            ph[ks16][2 * hf] = pack_h2(hi[0], hi[1]);
            ph[ks16][2 * hf + 1] = pack_h2(hi[2], hi[3]);
            pl[ks16][2 * hf] = pack_h2(lo[0], lo[1]);
            pl[ks16][2 * hf + 1] = pack_h2(lo[2], lo[3]);
        }
        l0 = __fmaf_rn(l0, al0, ps0);
        l1 = __fmaf_rn(l1, al1, ps1);
        // P.V per pair of 8-dim tiles: B fragments by ldmatrix.trans from the fp16 V rows
#pragma unroll
        for (int d = 0; d < NDT; d += 2) {
            float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int ks16 = 0; ks16 < 4; ks16++) {
                if (j0 + 16 * ks16 > last_key) break;  // every weight of this step is zero
                // lanes 0-7: keys 16 ks16 + 0..7, dims of tile d; 8-15: keys + 8..15;
                // 16-23: keys 0..7, tile d + 1; 24-31: keys 8..15, tile d + 1
                const int key = 16 * ks16 + (lane & 7) + ((lane >> 3) & 1) * 8;
                const int ch = d + (lane >> 4);
                uint32_t b0, b1, b2, b3;
                ldsm_x4_trans(s_v + key * HD + swz<VCH>(ch, key) * 8, b0, b1, b2, b3);
                mma_f16_16816(ph[ks16], b0, b1, c0);
                mma_f16_16816(pl[ks16], b0, b1, c0);
                mma_f16_16816(ph[ks16], b2, b3, c1);
                mma_f16_16816(pl[ks16], b2, b3, c1);
            }
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const float al = e < 2 ? al0 : al1;
                o[d][e] = __fmaf_rn(o[d][e], al, __fmul_rn(c0[e], down));
                o[d + 1][e] = __fmaf_rn(o[d + 1][e], al, __fmul_rn(c1[e], down));
            }
        }
    }
    if (!hv) return;
    // row sums over the quad, then out = o / l
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    const float i0 = r0v ? 1.0f / l0 : 0.0f, i1 = r1v ? 1.0f / l1 : 0.0f;
    float* out0 = a.out + (size_t)(t0 + gq) * q_dim + (size_t)h * HD + 2 * tq;
    float* out1 = out0 + (size_t)8 * q_dim;
#pragma unroll
    for (int d = 0; d < NDT; d++) {
        if (r0v) *reinterpret_cast<float2*>(out0 + 8 * d) = make_float2(__fmul_rn(o[d][0], i0), __fmul_rn(o[d][1], i0));
        if (r1v) *reinterpret_cast<float2*>(out1 + 8 * d) = make_float2(__fmul_rn(o[d][2], i1), __fmul_rn(o[d][3], i1));
    }
}

}  // namespace

bool pf_attention_supported(int H, int KV, int hd) {
    const int G = KV > 0 ? H / KV : 0;
    return (hd == 64 || hd == 128) && G >= 1 && G <= 8 && H % KV == 0;
}

int launch_pf_attention(const PfAttn& a_in, cudaStream_t s) {
    if (!pf_attention_supported(a_in.H, a_in.KV, a_in.hd)) return arg_error("pf_attention: unsupported head shape");
    PfAttn a = a_in;
    const int G = a.H / a.KV, ntb = (a.T + kPfQT - 1) / kPfQT;
    // query heads (warps) per CTA: all of the kv head's when that gives a
    // wave of CTAs (K/V blocks are read once per CTA), fewer otherwise
    a.gc = 1;
    for (int gc = G; gc >= 1; gc--)
        if (a.KV * ntb * ((G + gc - 1) / gc) >= mega_num_ctas()) {
            a.gc = gc;
            break;
        }
    const dim3 grid(a.KV, ntb, (G + a.gc - 1) / a.gc);
    if (a.hd == 64)
        pf_attention_kernel<64><<<grid, 32 * a.gc, pf_smem_bytes<64>(), s>>>(a);
    else
        pf_attention_kernel<128><<<grid, 32 * a.gc, pf_smem_bytes<128>(), s>>>(a);
    JYC_LAUNCHED();
    return JYC_OK;
}

int prepare_pf_attention() {
    JYC_CUDA(cudaFuncSetAttribute(pf_attention_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  pf_smem_bytes<64>()));
    JYC_CUDA(cudaFuncSetAttribute(pf_attention_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  pf_smem_bytes<128>()));
    return JYC_OK;
}

}  // namespace jyc
