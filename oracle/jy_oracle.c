/*
 * jy_oracle.c — TEST INFRASTRUCTURE ONLY: CPU restatement of the jieyu
 * reference decode path, used as the checker of the B200 kernels (tests/,
 * __graft_entry__.smoke()) and as the "port" CPU baseline. Never linked into
 * or called by the product library.
 *
 * Each function restates the reference's JIEYU_ISA=fma path (AVX2 + FMA
 * 8-lane code; AVX-VNNI off, which check_cpu.h:54-68 allows). Lane structure
 * and operation order follow the SIMD sources so results are bit-identical
 * to the reference on the same host (libm expf/powf/cosf/sinf are the host's,
 * as in the reference). Built with -ffp-contract=off: only explicit fmaf()
 * calls fuse, mirroring _mm256_fmadd_ps / _mm256_fmsub_ps.
 *
 * Citations: paths inside the jieyu source tree.
 */
#include "jy_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

void jyo_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* wmat::to_f32 (libs/date_libs/wmat.h:8-24): exact binary16 -> binary32. */
static float f16_to_f32(uint16_t h) {
    const uint32_t s = (h >> 15) & 1u, e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = s << 31;
        } else {
            uint32_t mm = m;
            int k = 0;
            while ((mm & 0x400u) == 0) { mm <<= 1; k++; }
            bits = (s << 31) | ((uint32_t)(113 - k) << 23) | ((mm & 0x3FFu) << 13);
        }
    } else if (e == 31) {
        bits = (s << 31) | 0x7F800000u | (m << 13);
    } else {
        bits = (s << 31) | ((e + 112u) << 23) | (m << 13);
    }
    float v;
    memcpy(&v, &bits, 4);
    return v;
}

/* Q8_0 block dequant (matmul_q.h:101-105): d * (float)q, exact in fp32. */
static void dequant_q8(const uint8_t* b, float* dst) {
    uint16_t dh;
    memcpy(&dh, b, 2);
    const float d = f16_to_f32(dh);
    for (int l = 0; l < 32; l++) dst[l] = (float)(int8_t)b[2 + l] * d;
}

/* 8-lane horizontal sum of rmsnorm's SIMD_HSUM / matmul_q's tail:
 * (lo128 + hi128) then two hadds -> (a0+a1)+(a2+a3). */
static float hsum8(const float* v) {
    float a[4];
    for (int i = 0; i < 4; i++) a[i] = v[i] + v[4 + i];
    return (a[0] + a[1]) + (a[2] + a[3]);
}

/* dot_row_avx2 (matmul_q.h:111-132): four 8-lane FMA accumulators s0..s3 over
 * 32-element blocks, then (s0+s1)+(s2+s3) and hsum8. */
static float dot_row_q8(const float* a, const uint8_t* row, int k) {
    float acc[32], blk[32];
    for (int l = 0; l < 32; l++) acc[l] = 0.0f;
    const int nb = k / 32;
    for (int b = 0; b < nb; b++) {
        dequant_q8(row + (size_t)b * 34, blk);
        const float* av = a + (size_t)b * 32;
        for (int l = 0; l < 32; l++) acc[l] = fmaf(av[l], blk[l], acc[l]);
    }
    float t[8];
    for (int i = 0; i < 8; i++) t[i] = (acc[i] + acc[8 + i]) + (acc[16 + i] + acc[24 + i]);
    return hsum8(t);
}

void jyo_matmul_q8(const float* a, const void* b, float* c, int m, int n, int k) {
    const uint8_t* base = (const uint8_t*)b;
    const size_t rbytes = (size_t)(k / 32) * 34;
    if (m == 1) {
#pragma omp parallel for schedule(static)
        for (int j = 0; j < n; j++) c[j] = dot_row_q8(a, base + (size_t)j * rbytes, k);
        return;
    }
    /* m > 1: scalar dequant + triple loop (matmul_q.h:145-161); compiled for
     * baseline x86-64 in the reference, so acc += a*w is a separate mul and add. */
#pragma omp parallel for schedule(static)
    for (int j = 0; j < n; j++) {
        float blk[32];
        float* acc = (float*)malloc(sizeof(float) * (size_t)m);
        for (int i = 0; i < m; i++) acc[i] = 0.0f;
        const uint8_t* row = base + (size_t)j * rbytes;
        for (int bl = 0; bl < k / 32; bl++) {
            dequant_q8(row + (size_t)bl * 34, blk);
            const size_t off = (size_t)bl * 32;
            for (int l = 0; l < 32; l++) {
                const float bv = blk[l];
                for (int i = 0; i < m; i++) acc[i] = acc[i] + a[(size_t)i * k + off + l] * bv;
            }
        }
        for (int i = 0; i < m; i++) c[(size_t)i * n + j] = acc[i];
        free(acc);
    }
}

/* 6-bit scale and min of sub-block j of a Q4_K / Q5_K super-block
 * (matmul_q.h:24-33 get_scale_min_k4). */
static void kq_scale_min(int j, const uint8_t* q, unsigned* sc, unsigned* mn) {
    if (j < 4) {
        *sc = q[j] & 63u;
        *mn = q[j + 4] & 63u;
    } else {
        *sc = (q[j + 4] & 0xFu) | ((unsigned)(q[j - 4] >> 6) << 4);
        *mn = (unsigned)(q[j + 4] >> 4) | ((unsigned)(q[j] >> 6) << 4);
    }
}

static float kq_f16(const uint8_t* p) {
    uint16_t h;
    memcpy(&h, p, 2);
    return f16_to_f32(h);
}

/* Q4_K (144 B / 256): the AVX2+FMA dequant of file_libs/q4/q4_fma.txt,
 * w = fma((float)q, d*sc, -(dmin*mn)) per 32-weight sub-block. */
static void dequant_q4k(const uint8_t* b, float* dst) {
    const float d = kq_f16(b), dmin = kq_f16(b + 2);
    const uint8_t* scp = b + 4;
    const uint8_t* qs = b + 16;
    for (int g = 0; g < 4; g++) {
        unsigned s0, m0, s1, m1;
        kq_scale_min(2 * g, scp, &s0, &m0);
        kq_scale_min(2 * g + 1, scp, &s1, &m1);
        const float d1 = d * (float)s0, n1 = -(dmin * (float)m0);
        const float d2 = d * (float)s1, n2 = -(dmin * (float)m1);
        for (int l = 0; l < 32; l++) dst[g * 64 + l] = fmaf((float)(qs[l] & 0xF), d1, n1);
        for (int l = 0; l < 32; l++) dst[g * 64 + 32 + l] = fmaf((float)(qs[l] >> 4), d2, n2);
        qs += 32;
    }
}

/* Q5_K (176 B / 256): matmul_q.h:52-77, d1*q - n1 as a separate multiply and
 * subtract (generic code, baseline x86-64). */
static void dequant_q5k(const uint8_t* b, float* dst) {
    const float d = kq_f16(b), dmin = kq_f16(b + 2);
    const uint8_t* sc = b + 4;
    const uint8_t* qh = b + 16;
    const uint8_t* qs = b + 48;
    unsigned u1 = 1, u2 = 2;
    for (int g = 0; g < 4; g++) {
        unsigned s0, m0, s1, m1;
        kq_scale_min(2 * g, sc, &s0, &m0);
        kq_scale_min(2 * g + 1, sc, &s1, &m1);
        const float d1 = d * (float)s0, n1 = dmin * (float)m0;
        const float d2 = d * (float)s1, n2 = dmin * (float)m1;
        for (int l = 0; l < 32; l++) {
            const float w = d1 * (float)((qs[l] & 0xF) + ((qh[l] & u1) ? 16 : 0));
            dst[g * 64 + l] = w - n1;
        }
        for (int l = 0; l < 32; l++) {
            const float w = d2 * (float)((qs[l] >> 4) + ((qh[l] & u2) ? 16 : 0));
            dst[g * 64 + 32 + l] = w - n2;
        }
        qs += 32;
        u1 <<= 2;
        u2 <<= 2;
    }
}

/* Q6_K (210 B / 256): matmul_q.h:78-100, (d * sc) * q (exact in fp32). */
static void dequant_q6k(const uint8_t* b, float* dst) {
    const uint8_t* ql = b;
    const uint8_t* qh = b + 128;
    const int8_t* sc = (const int8_t*)(b + 192);
    const float d = kq_f16(b + 208);
    for (int nn = 0; nn < 2; nn++) {
        for (int l = 0; l < 32; l++) {
            const int is = l / 16;
            const int q1 = (int)((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
            const int q2 = (int)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
            const int q3 = (int)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
            const int q4 = (int)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
            dst[nn * 128 + l] = d * (float)sc[is] * (float)q1;
            dst[nn * 128 + l + 32] = d * (float)sc[is + 2] * (float)q2;
            dst[nn * 128 + l + 64] = d * (float)sc[is + 4] * (float)q3;
            dst[nn * 128 + l + 96] = d * (float)sc[is + 6] * (float)q4;
        }
        ql += 64;
        qh += 32;
        sc += 8;
    }
}

static int kq_bytes(int t) { return t == JYC_Q4K ? 144 : t == JYC_Q5K ? 176 : t == JYC_Q6K ? 210 : 0; }

static void kq_dequant(int t, const uint8_t* b, float* dst) {
    if (t == JYC_Q4K) dequant_q4k(b, dst);
    else if (t == JYC_Q5K) dequant_q5k(b, dst);
    else dequant_q6k(b, dst);
}

/* qmat::matmul_q for the K-quants (matmul_q.h:134-162): m == 1 is
 * dot_row_avx2 (four 8-lane FMA accumulators = acc[l % 32], then the same
 * tail as Q8_0), m > 1 the scalar triple loop. Returns -1 for another t. */
int jyo_matmul_qk(const float* a, const void* b, float* c, int m, int n, int k, int t) {
    const int bb = kq_bytes(t);
    if (bb == 0 || k % 256) return -1;
    const uint8_t* base = (const uint8_t*)b;
    const size_t rbytes = (size_t)(k / 256) * bb;
#pragma omp parallel for schedule(static)
    for (int j = 0; j < n; j++) {
        float blk[256];
        const uint8_t* row = base + (size_t)j * rbytes;
        if (m == 1) {
            float acc[32];
            for (int l = 0; l < 32; l++) acc[l] = 0.0f;
            for (int bl = 0; bl < k / 256; bl++) {
                kq_dequant(t, row + (size_t)bl * bb, blk);
                const float* av = a + (size_t)bl * 256;
                for (int l = 0; l < 256; l++) acc[l & 31] = fmaf(av[l], blk[l], acc[l & 31]);
            }
            float tt[8];
            for (int i = 0; i < 8; i++) tt[i] = (acc[i] + acc[8 + i]) + (acc[16 + i] + acc[24 + i]);
            c[j] = hsum8(tt);
        } else {
            float* acc = (float*)malloc(sizeof(float) * (size_t)m);
            for (int i = 0; i < m; i++) acc[i] = 0.0f;
            for (int bl = 0; bl < k / 256; bl++) {
                kq_dequant(t, row + (size_t)bl * bb, blk);
                const size_t off = (size_t)bl * 256;
                for (int l = 0; l < 256; l++) {
                    const float bv = blk[l];
                    for (int i = 0; i < m; i++) acc[i] = acc[i] + a[(size_t)i * k + off + l] * bv;
                }
            }
            for (int i = 0; i < m; i++) c[(size_t)i * n + j] = acc[i];
            free(acc);
        }
    }
    return 0;
}

/* matmul x86_classic.txt:1-16: crow[j] = fma(a[p], B[p][j], crow[j]) for p in order. */
void jyo_matmul_f32(int m, int n, int k, const float* A, const float* B, float* C) {
#pragma omp parallel for schedule(static)
    for (int i = 0; i < m; i++) {
        float* crow = C + (size_t)i * n;
        const float* arow = A + (size_t)i * k;
        for (int j = 0; j < n; j++) crow[j] = 0.0f;
        for (int p = 0; p < k; p++) {
            const float va = arow[p];
            const float* brow = B + (size_t)p * n;
            for (int j = 0; j < n; j++) crow[j] = fmaf(va, brow[j], crow[j]);
        }
    }
}

/* matmul_f16_avx_fma (matmul_f16.h:19-41): C = 0, then per row i and input
 * index p in order, every output j += a[i][p] * f32(b[p][j]) as one fused
 * multiply-add: _mm256_fmadd_ps over the 8-wide column groups (:33-35), and
 * the scalar n % 8 tail (:37), which the compiler contracts to an FMA inside
 * that avx2/fma target function (checked bit for bit against the compiled
 * reference). */
void jyo_matmul_f16(const float* a, const uint16_t* b, float* c, int m, int n, int k) {
#pragma omp parallel for schedule(static)
    for (int i = 0; i < m; i++) {
        float* crow = c + (size_t)i * n;
        const float* arow = a + (size_t)i * k;
        for (int j = 0; j < n; j++) crow[j] = 0.0f;
        for (int p = 0; p < k; p++) {
            const float va = arow[p];
            const uint16_t* brow = b + (size_t)p * n;
            for (int j = 0; j < n; j++) crow[j] = fmaf(va, f16_to_f32(brow[j]), crow[j]);
        }
    }
}

/* rmsnorm x86_classic.txt:1-27: two 8-lane FMA sums (16-wide steps, then one
 * 8-wide step), hsum, scalar tail; y = (x*scale)*w. */
void jyo_rmsnorm(const float* x, float* y, const float* w, int n, float eps) {
    float s0[8] = {0}, s1[8] = {0};
    int i = 0;
    for (; i + 16 <= n; i += 16)
        for (int l = 0; l < 8; l++) {
            s0[l] = fmaf(x[i + l], x[i + l], s0[l]);
            s1[l] = fmaf(x[i + 8 + l], x[i + 8 + l], s1[l]);
        }
    for (; i + 8 <= n; i += 8)
        for (int l = 0; l < 8; l++) s0[l] = fmaf(x[i + l], x[i + l], s0[l]);
    float v[8];
    for (int l = 0; l < 8; l++) v[l] = s0[l] + s1[l];
    float ss = hsum8(v);
    for (; i < n; i++) ss = fmaf(x[i], x[i], ss);
    const float den = ss / (float)n + eps;
    if (den <= 0.0f) {
        for (int t = 0; t < n; t++) y[t] = 0.0f;
        return;
    }
    const float scale = 1.0f / sqrtf(den);
    for (int t = 0; t < n; t++) y[t] = (x[t] * scale) * w[t];
}

/* RoPETable::init (date.h:52-66). */
void jyo_rope_table(int max_seq, int head_dim, float theta, float* cos_out, float* sin_out) {
    const int half = head_dim / 2;
    for (int i = 0; i < max_seq; i++)
        for (int j = 0; j < half; j++) {
            float freq = 1.0f / powf(theta, 2.0f * j / head_dim);
            float angle = i * freq;
            cos_out[(size_t)i * half + j] = cosf(angle);
            sin_out[(size_t)i * half + j] = sinf(angle);
        }
}

/* Output pair slot of rotated pair p in rope x86_classic.txt:10-28. The 8-pair
 * vector body de-interleaves with _mm256_shuffle_ps (lanes hold pairs
 * 0,1,4,5 | 2,3,6,7), re-interleaves with unpacklo/unpackhi and stores the
 * four 128-bit halves at +0, +4, +8, +12 floats; as a result pairs 2,3 land in
 * slots 4,5 and pairs 4,5 in slots 2,3 of every full 8-pair group. The scalar
 * tail (half % 8 pairs) stores in place. Q and K get the same permutation, so
 * q.k dot products are unchanged; the stored K bytes carry it. */
static int rope_slot(int p, int half) {
    const int g = p >> 3;
    if ((g + 1) * 8 > half) return p;
    int j = p & 7;
    if (j == 2 || j == 3) j += 2;
    else if (j == 4 || j == 5) j -= 2;
    return g * 8 + j;
}

/* rope x86_classic.txt:1-39: r0 = fmsub(x0, c, x1*s), r1 = fma(x0, s, x1*c). */
void jyo_rope_pos(float* q, int seq, int start_pos, int heads, int hd, const float* cos_t,
                  const float* sin_t) {
    const int half = hd / 2;
    float* tmp = (float*)malloc(sizeof(float) * (size_t)hd);
    for (int pos = 0; pos < seq; pos++) {
        const float* c = cos_t + (size_t)(start_pos + pos) * half;
        const float* s = sin_t + (size_t)(start_pos + pos) * half;
        for (int h = 0; h < heads; h++) {
            float* qh = q + ((size_t)pos * heads + h) * hd;
            for (int i = 0; i < half; i++) {
                const float x0 = qh[2 * i], x1 = qh[2 * i + 1];
                const int o = rope_slot(i, half);
                tmp[2 * o] = fmaf(x0, c[i], -(x1 * s[i]));
                tmp[2 * o + 1] = fmaf(x0, s[i], x1 * c[i]);
            }
            memcpy(qh, tmp, sizeof(float) * (size_t)(2 * half));
        }
    }
    free(tmp);
}

/* kv_pack_q8 (attention_q8.h:20-37). */
static void quant_row(const float* s, int8_t* d, float* sc, int hd) {
    float amax = 0.0f;
    for (int k = 0; k < hd; k++) {
        const float a = fabsf(s[k]);
        if (a > amax) amax = a;
    }
    const float inv = amax > 1e-8f ? 127.0f / amax : 0.0f;
    *sc = amax > 1e-8f ? amax / 127.0f : 0.0f;
    for (int k = 0; k < hd; k++) {
        float x = s[k] * inv;
        x = x > 127.0f ? 127.0f : (x < -127.0f ? -127.0f : x);
        d[k] = (int8_t)lrintf(x);
    }
}

void jyo_kv_pack_q8(const float* src, int8_t* dst, float* sc, int heads, int hd, int n) {
    for (int i = 0; i < n; i++)
        for (int h = 0; h < heads; h++)
            quant_row(src + ((size_t)i * heads + h) * hd, dst + ((size_t)i * heads + h) * hd,
                      sc + (size_t)i * heads + h, hd);
}

/* attention x86_classic.txt:1-75 (the avx2+fma body; its int8 dot is exact). */
int jyo_attention_q8(const float* Q, const float* K, const float* V, float* out, int seq,
                     int start_pos, int H, int KV, int hd, int8_t* kc, float* ks, int8_t* vc,
                     float* vs, int cap) {
    if (KV <= 0 || H % KV != 0 || seq <= 0 || start_pos < 0) return -1;
    if (!kc || !ks || !vc || !vs || cap <= 0) return -1;
    if ((size_t)start_pos + (size_t)seq > (size_t)cap) return -1;
    const int kv_dim = KV * hd;
    jyo_kv_pack_q8(K, kc + (size_t)start_pos * kv_dim, ks + (size_t)start_pos * KV, KV, hd, seq);
    jyo_kv_pack_q8(V, vc + (size_t)start_pos * kv_dim, vs + (size_t)start_pos * KV, KV, hd, seq);
    const int group = H / KV;
    const float scale = 1.0f / sqrtf((float)hd);
#pragma omp parallel for schedule(static)
    for (int h = 0; h < H; h++) {
        float* scores = (float*)malloc(sizeof(float) * (size_t)(start_pos + seq));
        int8_t* q8 = (int8_t*)malloc((size_t)hd);
        float qsc;
        const int kv_h = h / group;
        for (int i = 0; i < seq; i++) {
            const int p = start_pos + i;
            quant_row(Q + ((size_t)i * H + h) * hd, q8, &qsc, hd);
            float mxs = -1e30f;
            for (int j = 0; j <= p; j++) {
                const int8_t* k = kc + ((size_t)j * KV + kv_h) * hd;
                const float ksc = ks[(size_t)j * KV + kv_h] * qsc * scale;
                int32_t dot = 0;
                for (int d = 0; d < hd; d++) dot += (int32_t)q8[d] * (int32_t)k[d];
                const float dt = (float)dot * ksc;
                scores[j] = dt;
                if (dt > mxs) mxs = dt;
            }
            float sum = 0.0f;
            for (int j = 0; j <= p; j++) {
                scores[j] = expf(scores[j] - mxs);
                sum += scores[j];
            }
            const float inv_sum = 1.0f / sum;
            for (int j = 0; j <= p; j++) scores[j] *= inv_sum;
            float* o = out + ((size_t)i * H + h) * hd;
            for (int d = 0; d < hd; d++) o[d] = 0.0f;
            for (int j = 0; j <= p; j++) {
                const int8_t* v = vc + ((size_t)j * KV + kv_h) * hd;
                const float pr = scores[j] * vs[(size_t)j * KV + kv_h];
                for (int d = 0; d < hd; d++) o[d] = fmaf(pr, (float)v[d], o[d]);
            }
        }
        free(scores);
        free(q8);
    }
    return 0;
}

/* silu x86_classic.txt:1-32: the reference's Cody-Waite + degree-6 Taylor exp
 * on n/8*8 elements, libm expf on the tail. */
void jyo_silu(const float* x, float* y, int n) {
    const float lg2e = 1.44269504088896341f, ln2h = 0.693359375f, ln2l = -2.12194440e-4f;
    const float q1 = 1.0f / 720.0f, q2 = 1.0f / 120.0f, q3 = 1.0f / 24.0f, q4 = 1.0f / 6.0f,
                q5 = 0.5f;
    const int nv = n / 8 * 8;
#pragma omp parallel for schedule(static) if (n >= 8192)
    for (int i = 0; i < nv; i++) {
        const float vx = x[i];
        float xa = 0.0f - vx;
        xa = fminf(fmaxf(xa, -87.0f), 88.0f);
        const float nf = rintf(xa * lg2e);
        const float r = (xa - nf * ln2h) - nf * ln2l;
        float p = fmaf(q1, r, q2);
        p = fmaf(p, r, q3);
        p = fmaf(p, r, q4);
        p = fmaf(p, r, q5);
        p = fmaf(p, r, 1.0f);
        p = fmaf(p, r, 1.0f);
        const int e = ((int)nf + 127) << 23;
        float s;
        memcpy(&s, &e, 4);
        y[i] = vx / (1.0f + p * s);
    }
    for (int i = nv; i < n; i++) y[i] = x[i] / (1.0f + expf(-x[i]));
}

/* ---------------------------------------------------------------------- */
typedef struct {
    int L, max_seq, KV, hd;
    int8_t *k, *v;
    float *ks, *vs;
} jyo_cache;

void* jyo_cache_create(int L, int max_seq, int KV, int hd) {
    jyo_cache* c = (jyo_cache*)calloc(1, sizeof(jyo_cache));
    c->L = L; c->max_seq = max_seq; c->KV = KV; c->hd = hd;
    const size_t n = (size_t)L * max_seq * KV;
    c->k = (int8_t*)calloc(n * hd, 1);
    c->v = (int8_t*)calloc(n * hd, 1);
    c->ks = (float*)calloc(n, sizeof(float));
    c->vs = (float*)calloc(n, sizeof(float));
    return c;
}

void jyo_cache_free(void* p) {
    jyo_cache* c = (jyo_cache*)p;
    if (!c) return;
    free(c->k); free(c->v); free(c->ks); free(c->vs); free(c);
}

void jyo_cache_read(void* p, int layer, int npos, int8_t* k, float* ks, int8_t* v, float* vs) {
    jyo_cache* c = (jyo_cache*)p;
    const size_t row = (size_t)c->KV * c->hd, lay = (size_t)layer * c->max_seq;
    memcpy(k, c->k + lay * row, (size_t)npos * row);
    memcpy(v, c->v + lay * row, (size_t)npos * row);
    memcpy(ks, c->ks + lay * c->KV, (size_t)npos * c->KV * sizeof(float));
    memcpy(vs, c->vs + lay * c->KV, (size_t)npos * c->KV * sizeof(float));
}

/* Writes one layer's first npos positions (the inverse of jyo_cache_read). */
void jyo_cache_write(void* p, int layer, int npos, const int8_t* k, const float* ks, const int8_t* v,
                     const float* vs) {
    jyo_cache* c = (jyo_cache*)p;
    const size_t row = (size_t)c->KV * c->hd, lay = (size_t)layer * c->max_seq;
    memcpy(c->k + lay * row, k, (size_t)npos * row);
    memcpy(c->v + lay * row, v, (size_t)npos * row);
    memcpy(c->ks + lay * c->KV, ks, (size_t)npos * c->KV * sizeof(float));
    memcpy(c->vs + lay * c->KV, vs, (size_t)npos * c->KV * sizeof(float));
}

/* matmul_w (wmat_kernel.h:9-16): fp32 [k][n] -> matmul, fp16 [k][n] -> matmul_f16, Q8_0 / K-quant
 * [n][k] -> matmul_q. */
static int matmul_w(const jyc_wmat* w, int m, int n, int k, const float* A, float* Cc) {
    if (w->f) { jyo_matmul_f32(m, n, k, A, w->f, Cc); return 0; }
    if (w->h && !w->q) { jyo_matmul_f16(A, w->h, Cc, m, n, k); return 0; }
    if (w->q && w->qt == JYC_Q8_0) { jyo_matmul_q8(A, w->q, Cc, m, n, k); return 0; }
    if (w->q && kq_bytes(w->qt)) return jyo_matmul_qk(A, w->q, Cc, m, n, k, w->qt);
    return -1;
}

/* wmat_row (wmat_kernel.h:18-29). */
static int wmat_row(const jyc_wmat* w, size_t id, int width, float* dst) {
    if (w->f) { memcpy(dst, w->f + id * (size_t)width, (size_t)width * sizeof(float)); return 0; }
    if (w->h) {  /* wmat::row_to_f32: exact */
        for (int t = 0; t < width; t++) dst[t] = f16_to_f32(w->h[id * (size_t)width + t]);
        return 0;
    }
    if (w->q && w->qt == JYC_Q8_0) {
        const uint8_t* row = (const uint8_t*)w->q + id * (size_t)(width / 32) * 34;
        for (int bl = 0; bl < width / 32; bl++) dequant_q8(row + (size_t)bl * 34, dst + bl * 32);
        return 0;
    }
    if (w->q && kq_bytes(w->qt) && width % 256 == 0) {  /* dequant_block per super-block */
        const int bb = kq_bytes(w->qt);
        const uint8_t* row = (const uint8_t*)w->q + id * (size_t)(width / 256) * bb;
        for (int bl = 0; bl < width / 256; bl++) kq_dequant(w->qt, row + (size_t)bl * bb, dst + bl * 256);
        return 0;
    }
    return -1;
}

/* ffn (ffn.h:7-19). */
static int ffn(const float* x, const jyc_wmat* w1, const jyc_wmat* w2, const jyc_wmat* w3,
               float* out, int seq, int hidden, int inter) {
    const size_t n = (size_t)seq * inter;
    float* gate = (float*)malloc(n * sizeof(float));
    float* up = (float*)malloc(n * sizeof(float));
    int r = matmul_w(w1, seq, inter, hidden, x, gate);
    r |= matmul_w(w3, seq, inter, hidden, x, up);
    jyo_silu(gate, gate, (int)n);
    for (size_t i = 0; i < n; i++) gate[i] = gate[i] * up[i];
    r |= matmul_w(w2, seq, hidden, inter, gate, out);
    free(gate);
    free(up);
    return r;
}

/* transformer_layer KV overload (transformer_layer.h:10-90). */
static int transformer_layer(float* X, const jyc_layer_weights* w, const float* cos_t,
                             const float* sin_t, int seq, int D, int H, int KV, int hd, int F,
                             int start_pos, jyo_cache* c, int layer) {
    const int q_dim = H * hd, kv_dim = KV * hd;
    const float eps = 1e-5f;
    float* xn = (float*)malloc((size_t)seq * D * sizeof(float));
    float* Q = (float*)malloc((size_t)seq * q_dim * sizeof(float));
    float* Kb = (float*)malloc((size_t)seq * kv_dim * sizeof(float));
    float* Vb = (float*)malloc((size_t)seq * kv_dim * sizeof(float));
    float* attn = (float*)malloc((size_t)seq * q_dim * sizeof(float));
    float* proj = (float*)malloc((size_t)seq * D * sizeof(float));
    int r = 0;
    for (int i = 0; i < seq; i++)
        jyo_rmsnorm(X + (size_t)i * D, xn + (size_t)i * D, w->rms1_weight, D, eps);
    r |= matmul_w(&w->Wq, seq, q_dim, D, xn, Q);
    r |= matmul_w(&w->Wk, seq, kv_dim, D, xn, Kb);
    r |= matmul_w(&w->Wv, seq, kv_dim, D, xn, Vb);
    if (w->bq) for (int i = 0; i < seq; i++) for (int j = 0; j < q_dim; j++) Q[(size_t)i * q_dim + j] += w->bq[j];
    if (w->bk) for (int i = 0; i < seq; i++) for (int j = 0; j < kv_dim; j++) Kb[(size_t)i * kv_dim + j] += w->bk[j];
    if (w->bv) for (int i = 0; i < seq; i++) for (int j = 0; j < kv_dim; j++) Vb[(size_t)i * kv_dim + j] += w->bv[j];
    jyo_rope_pos(Q, seq, start_pos, H, hd, cos_t, sin_t);
    jyo_rope_pos(Kb, seq, start_pos, KV, hd, cos_t, sin_t);
    const size_t lay = (size_t)layer * c->max_seq;
    r |= jyo_attention_q8(Q, Kb, Vb, attn, seq, start_pos, H, KV, hd, c->k + lay * kv_dim,
                          c->ks + lay * KV, c->v + lay * kv_dim, c->vs + lay * KV, c->max_seq);
    r |= matmul_w(&w->Wo, seq, D, q_dim, attn, proj);
    for (size_t i = 0; i < (size_t)seq * D; i++) X[i] += proj[i];
    for (int i = 0; i < seq; i++)
        jyo_rmsnorm(X + (size_t)i * D, xn + (size_t)i * D, w->rms2_weight, D, eps);
    r |= ffn(xn, &w->W1, &w->W2, &w->W3, proj, seq, D, F);
    for (size_t i = 0; i < (size_t)seq * D; i++) X[i] += proj[i];
    free(xn); free(Q); free(Kb); free(Vb); free(attn); free(proj);
    return r;
}

/* forward_cached (forward.h:47-96) on X [seq][D]. */
static int forward_cached(const jyc_model_desc* d, float* X, int seq, int start_pos, jyo_cache* c) {
    if (start_pos < 0 || start_pos + seq > c->max_seq) return -1;
    int r = 0;
    for (int l = 0; l < d->num_layers; l++)
        r |= transformer_layer(X, &d->layers[l], d->cos_table, d->sin_table, seq, d->hidden,
                               d->num_heads, d->num_kv_heads, d->head_dim, d->intermediate,
                               start_pos, c, l);
    float* xn = (float*)malloc((size_t)d->hidden * sizeof(float));
    for (int i = 0; i < seq; i++) {
        jyo_rmsnorm(X + (size_t)i * d->hidden, xn, d->final_rms_weight, d->hidden, 1e-5f);
        memcpy(X + (size_t)i * d->hidden, xn, (size_t)d->hidden * sizeof(float));
    }
    free(xn);
    return r;
}

int jyo_forward_logits(const jyc_model_desc* d, void* cache, const int* ids, int seq,
                       int start_pos, float* logits, float* hidden_out) {
    jyo_cache* c = (jyo_cache*)cache;
    float* X = (float*)malloc((size_t)seq * d->hidden * sizeof(float));
    int r = 0;
    for (int i = 0; i < seq; i++) r |= wmat_row(&d->embed, (size_t)ids[i], d->hidden, X + (size_t)i * d->hidden);
    r |= forward_cached(d, X, seq, start_pos, c);
    const float* last = X + (size_t)(seq - 1) * d->hidden;
    if (hidden_out) memcpy(hidden_out, last, (size_t)d->hidden * sizeof(float));
    if (logits) r |= matmul_w(&d->lm_head, 1, d->vocab_size, d->hidden, last, logits);
    free(X);
    return r ? -1 : 0;
}

/* The token pick of one generate step (generate.h:50-77): repetition penalty
 * over the ids generated so far (out_ids[prompt_len..len)), then greedy
 * (first index of the maximum) or, with temperature > 0, the reference's
 * sampler: expf((l - max) / T) written back, summed in double, one LCG step
 * (rng = rng * 1664525 + 1013904223), r = (rng >> 8) / 2^24 * sum, the first
 * v whose running r -= p_v reaches <= 0 (V - 1 if none). logits is modified
 * in place as in the reference. */
int jyo_sample(float* logits, int V, float temperature, float rep_penalty, const int* out_ids,
               int prompt_len, int len, unsigned* rng) {
    if (rep_penalty != 1.0f)
        for (int i = prompt_len; i < len; i++) {
            const int id = out_ids[i];
            if (id >= 0 && id < V)
                logits[id] = (logits[id] > 0.0f) ? logits[id] / rep_penalty : logits[id] * rep_penalty;
        }
    int next = 0;
    if (temperature <= 0.0f) {
        for (int v = 1; v < V; v++)
            if (logits[v] > logits[next]) next = v;
        return next;
    }
    float mx = logits[0];
    for (int v = 1; v < V; v++)
        if (logits[v] > mx) mx = logits[v];
    double sum = 0.0;
    for (int v = 0; v < V; v++) {
        logits[v] = expf((logits[v] - mx) / temperature);
        sum += logits[v];
    }
    *rng = *rng * 1664525u + 1013904223u;
    double rr = (double)(*rng >> 8) / 16777216.0 * sum;
    next = V - 1;
    for (int v = 0; v < V; v++) {
        rr -= logits[v];
        if (rr <= 0.0) {
            next = v;
            break;
        }
    }
    return next;
}

/* generate + generate_cached (generate.h:9-112). */
int jyo_generate(const jyc_model_desc* d, const int* prompt, int prompt_len, const int* eos,
                 int num_eos, int max_new, float temperature, int* out_ids, float rep_penalty) {
    const int max_seq = d->max_seq, V = d->vocab_size, D = d->hidden;
    if (prompt_len <= 0 || prompt_len > max_seq) return 0;
    for (int i = 0; i < prompt_len; i++) out_ids[i] = prompt[i];
    if (max_new <= 0) return prompt_len;
    jyo_cache* c = (jyo_cache*)jyo_cache_create(d->num_layers, max_seq, d->num_kv_heads, d->head_dim);
    float* X = (float*)malloc((size_t)max_seq * D * sizeof(float));
    float* logits = (float*)calloc((size_t)V, sizeof(float));
    unsigned rng = 12345u;
    int len = prompt_len, seq = prompt_len, err = 0;
    for (int step = 0; step < max_new && len < max_seq; step++) {
        const int start_pos = len - seq;
        for (int i = 0; i < seq; i++) err |= wmat_row(&d->embed, (size_t)out_ids[start_pos + i], D, X + (size_t)i * D);
        err |= forward_cached(d, X, seq, start_pos, c);
        const float* last = X + (size_t)(seq - 1) * D;
        err |= matmul_w(&d->lm_head, 1, V, D, last, logits);
        if (err) break;
        const int next = jyo_sample(logits, V, temperature, rep_penalty, out_ids, prompt_len, len, &rng);
        out_ids[len++] = next;
        seq = 1;
        int stop = 0;
        if (eos)
            for (int e = 0; e < num_eos; e++)
                if (next == eos[e]) stop = 1;
        if (stop) break;
    }
    free(X);
    free(logits);
    jyo_cache_free(c);
    return err ? -1 : len;
}

/* ---- seeded synthetic inputs ----------------------------------------------
 * The counter-based generator that defines the synthetic weights and prompts
 * of the tests and benches (the same integer function as the library's
 * jyc_synth_*: splitmix64's finaliser over (seed, stream, index), a sum of
 * four 16-bit uniforms as a bell-shaped integer, the Q8_0 rule d =
 * fp16(amax/127), q = lrintf(x/d) clamped to +-127). Restated here so that
 * the CPU checker and the reference arm of the bench build their inputs
 * without the product library; a host test holds the two byte-identical. */
static uint64_t syn_mix(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
static uint64_t syn_base(uint64_t seed, uint64_t stream) {
    return syn_mix(syn_mix(seed) ^ (stream * 0xD1B54A32D192ED03ull));
}
static int syn_bell(uint64_t base, uint64_t idx) {
    const uint64_t r = syn_mix(base + idx);
    return (int)(r & 0xFFFFu) + (int)((r >> 16) & 0xFFFFu) + (int)((r >> 32) & 0xFFFFu) + (int)(r >> 48) -
           2 * 65535;
}
/* binary32 -> binary16, round to nearest even */
static uint16_t syn_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t mag = x & 0x7FFFFFFFu;
    if (mag >= 0x7F800000u) return (uint16_t)(sign | (mag > 0x7F800000u ? 0x7E00u : 0x7C00u));
    if (mag >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);
    if (mag < 0x38800000u) {
        if (mag < 0x33000000u) return (uint16_t)sign;
        const uint32_t e = mag >> 23, m = (mag & 0x7FFFFFu) | 0x800000u;
        const int shift = 126 - (int)e;
        const uint32_t q = m >> shift, rem = m & ((1u << shift) - 1u), half = 1u << (shift - 1);
        return (uint16_t)(sign | (q + ((rem > half || (rem == half && (q & 1u))) ? 1u : 0u)));
    }
    uint32_t h = (((mag >> 23) - 112u) << 10) | ((mag & 0x7FFFFFu) >> 13);
    const uint32_t rem = mag & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)(sign | h);
}

void jyo_synth_f32(uint64_t seed, uint64_t stream, float std_dev, float* out, size_t n) {
    const uint64_t base = syn_base(seed, stream);
    const float sc = std_dev / 37837.227f;
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)n; i++) out[i] = (float)syn_bell(base, (uint64_t)i) * sc;
}

void jyo_synth_q8_0(uint64_t seed, uint64_t stream, float std_dev, void* out_blocks, size_t rows, size_t k) {
    const uint64_t base = syn_base(seed, stream);
    const float sc = std_dev / 37837.227f;
    uint8_t* dst = (uint8_t*)out_blocks;
    const size_t nb = k / 32;
#pragma omp parallel for schedule(static)
    for (long long r = 0; r < (long long)rows; r++) {
        float x[32];
        for (size_t bl = 0; bl < nb; bl++) {
            const size_t i0 = (size_t)r * k + bl * 32;
            float amax = 0.0f;
            for (int i = 0; i < 32; i++) {
                x[i] = (float)syn_bell(base, i0 + i) * sc;
                amax = fmaxf(amax, fabsf(x[i]));
            }
            uint8_t* blk = dst + ((size_t)r * nb + bl) * 34;
            const uint16_t dh = syn_f16(amax / 127.0f);
            const float d = f16_to_f32(dh);
            const float id = d != 0.0f ? 1.0f / d : 0.0f;
            memcpy(blk, &dh, 2);
            for (int i = 0; i < 32; i++) {
                float v = x[i] * id;
                v = v > 127.0f ? 127.0f : (v < -127.0f ? -127.0f : v);
                blk[2 + i] = (uint8_t)(int8_t)lrintf(v);
            }
        }
    }
}

void jyo_synth_ids(uint64_t seed, uint64_t stream, int vocab, int* out, size_t n) {
    const uint64_t base = syn_base(seed, stream);
    for (size_t i = 0; i < n; i++) out[i] = (int)(((syn_mix(base + i) >> 32) * (uint64_t)vocab) >> 32);
}
