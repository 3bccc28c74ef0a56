// common.cuh — shared definitions of the jieyu B200 library (device + host).
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <string>

#include "jieyu_b200.h"

namespace jyc {

// ---- error plumbing (host) ------------------------------------------------
void set_error(const std::string& msg);
void clear_error();
int cuda_fail(cudaError_t e, const char* what);
void count_launch(int n = 1);

#define JYC_CUDA(call)                                                        \
    do {                                                                      \
        cudaError_t _e = (call);                                              \
        if (_e != cudaSuccess) return ::jyc::cuda_fail(_e, #call);            \
    } while (0)

// Checks the launch that was just issued and counts it.
#define JYC_LAUNCHED()                                                        \
    do {                                                                      \
        cudaError_t _e = cudaGetLastError();                                  \
        if (_e != cudaSuccess) return ::jyc::cuda_fail(_e, "kernel launch");  \
        ::jyc::count_launch();                                                \
    } while (0)

inline int arg_error(const std::string& msg) {
    set_error(msg);
    return JYC_ERR_ARG;
}

// ---- host numeric helpers (host.cpp) --------------------------------------
uint16_t f32_to_f16_rne(float f);
float f16_to_f32(uint16_t h);

// ---- device helpers -------------------------------------------------------
constexpr int kWarp = 32;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// 4 bytes u = q+128 (q int8) -> 4 exact floats q, via the 2^23 mantissa trick:
// float bits 0x4B0000uu == 2^23 + uu, minus (2^23 + 128) == q exactly.
__device__ __forceinline__ void u8x4_to_f32(uint32_t w, float* f) {
    const float bias = 8388736.0f;  // 2^23 + 128
    f[0] = __fsub_rn(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540u)), bias);
    f[1] = __fsub_rn(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7541u)), bias);
    f[2] = __fsub_rn(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7542u)), bias);
    f[3] = __fsub_rn(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7543u)), bias);
}

__device__ __forceinline__ float h2f(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}

// Order-preserving map of a float to u32 (larger float -> larger key); NaN maps
// below every number so it never wins an argmax (the reference's strict `>`
// comparison never selects NaN).
__device__ __forceinline__ uint32_t f32_order_key(float f) {
    if (f != f) return 0u;
    const uint32_t b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
// (value key << 32) | ~index : atomicMax picks the max value, ties -> lowest index.
__device__ __forceinline__ unsigned long long argmax_pack(float v, int idx) {
    return ((unsigned long long)f32_order_key(v) << 32) |
           (unsigned long long)(0xFFFFFFFFu - (uint32_t)idx);
}
__device__ __forceinline__ int argmax_index(unsigned long long p) {
    return (int)(0xFFFFFFFFu - (uint32_t)(p & 0xFFFFFFFFull));
}

// SiLU with the reference's vector exp (Cody-Waite reduction + degree-6 Taylor,
// libs/model_libs/silu/x86/x86_classic.txt:2-28). Explicit _rn intrinsics keep
// nvcc from contracting the separate multiplies/subtracts into FMAs, so for a
// given input the result equals the reference's AVX2+FMA lanes bit for bit.
__device__ __forceinline__ float silu_ref(float x) {
    const float lg2e = 1.44269504088896341f, ln2h = 0.693359375f, ln2l = -2.12194440e-4f;
    float xa = __fsub_rn(0.0f, x);
    xa = fminf(fmaxf(xa, -87.0f), 88.0f);
    const float nf = rintf(__fmul_rn(xa, lg2e));
    const float r = __fsub_rn(__fsub_rn(xa, __fmul_rn(nf, ln2h)), __fmul_rn(nf, ln2l));
    float p = __fmaf_rn(1.0f / 720.0f, r, 1.0f / 120.0f);
    p = __fmaf_rn(p, r, 1.0f / 24.0f);
    p = __fmaf_rn(p, r, 1.0f / 6.0f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    const float s = __int_as_float(((int)nf + 127) << 23);
    return __fdiv_rn(x, __fadd_rn(1.0f, __fmul_rn(p, s)));
}

// Output slot of rotated pair p (of `half` pairs) in the reference's AVX2 RoPE
// (libs/model_libs/rope/x86/x86_classic.txt:10-28): its shuffle/unpack/store
// sequence puts pairs 2,3 into slots 4,5 and pairs 4,5 into slots 2,3 of every
// full 8-pair group; the scalar tail (half % 8 pairs) stays in place. Q and K
// share the permutation, so attention scores are unchanged, but the cached K
// bytes carry it; reproducing it keeps the int8 KV cache bit-identical.
__host__ __device__ __forceinline__ int rope_slot(int p, int half) {
    const int g = p >> 3;
    if ((g + 1) * 8 > half) return p;
    int j = p & 7;
    if (j == 2 || j == 3) j += 2;
    else if (j == 4 || j == 5) j -= 2;
    return g * 8 + j;
}

// kv_pack_q8 quantisation rule (libs/model_libs/attention/attention_q8.h:24-35):
// inv = 127/amax, scale = amax/127 (0 when amax <= 1e-8), q = lrintf(clamp(x*inv)).
__device__ __forceinline__ float q8_inv(float amax) {
    return amax > 1e-8f ? __fdiv_rn(127.0f, amax) : 0.0f;
}
__device__ __forceinline__ float q8_scale(float amax) {
    return amax > 1e-8f ? __fdiv_rn(amax, 127.0f) : 0.0f;
}
__device__ __forceinline__ int q8_round(float x, float inv) {
    float v = __fmul_rn(x, inv);
    v = v > 127.0f ? 127.0f : (v < -127.0f ? -127.0f : v);
    return __float2int_rn(v);
}

}  // namespace jyc
