// host.cpp — host-side parts of the C ABI: errors, version, launch counter,
// RoPE tables, seeded synthetic data and the fp32 -> Q8_0 quantiser.
#include <atomic>
#include <cmath>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include <cuda_runtime.h>

#include "jieyu_b200.h"

namespace jyc {

static thread_local std::string g_error;
static std::atomic<long long> g_launches{0};

void set_error(const std::string& msg) { g_error = msg; }
void clear_error() { g_error.clear(); }
void count_launch(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

static int arg_error(const std::string& msg) {
    set_error(msg);
    return JYC_ERR_ARG;
}

int cuda_fail(cudaError_t e, const char* what) {
    set_error(std::string(what) + ": " + cudaGetErrorString(e));
    return JYC_ERR_CUDA;
}

// IEEE binary32 -> binary16, round to nearest even (subnormals, inf, NaN handled).
uint16_t f32_to_f16_rne(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t mag = x & 0x7FFFFFFFu;
    if (mag >= 0x7F800000u) return (uint16_t)(sign | (mag > 0x7F800000u ? 0x7E00u : 0x7C00u));
    if (mag >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);  // rounds to >= 65520 -> inf
    if (mag < 0x38800000u) {                                       // below 2^-14: subnormal half
        if (mag < 0x33000000u) return (uint16_t)sign;               // < 2^-25 rounds to 0
        const uint32_t e = mag >> 23;
        const uint32_t m = (mag & 0x7FFFFFu) | 0x800000u;
        const int shift = 126 - (int)e;                             // 14 + (127-e) - 10 ... into 10-bit field
        const uint32_t q = m >> (shift);
        const uint32_t rem = m & ((1u << shift) - 1u);
        const uint32_t half = 1u << (shift - 1);
        uint32_t r = q + ((rem > half || (rem == half && (q & 1u))) ? 1u : 0u);
        return (uint16_t)(sign | r);
    }
    // normal range
    const uint32_t e = (mag >> 23) - 112u;  // rebias 127 -> 15
    const uint32_t m = mag & 0x7FFFFFu;
    uint32_t h = (e << 10) | (m >> 13);
    const uint32_t rem = m & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)(sign | h);
}

float f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else {  // subnormal: value = m * 2^-24
            float v = (float)m * 5.9604644775390625e-8f;
            std::memcpy(&bits, &v, 4);
            bits |= sign;
        }
    } else if (e == 31) {
        bits = sign | 0x7F800000u | (m << 13);
    } else {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    }
    float out;
    std::memcpy(&out, &bits, 4);
    return out;
}

// ---- seeded counter-based generator --------------------------------------
// splitmix64 finaliser (Steele, Lea & Flood 2014; constants as published by Vigna).
static inline uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
static inline uint64_t stream_base(uint64_t seed, uint64_t stream) {
    return mix64(mix64(seed) ^ (stream * 0xD1B54A32D192ED03ull));
}
// Sum of four 16-bit uniforms, centred: integer in [-131070, 131070];
// std of the sum is 37837.227 (4 * (65536^2-1)/12, square-rooted).
static inline int bell_int(uint64_t base, uint64_t idx) {
    const uint64_t r = mix64(base + idx);
    const int s = (int)(r & 0xFFFFu) + (int)((r >> 16) & 0xFFFFu) + (int)((r >> 32) & 0xFFFFu) +
                  (int)(r >> 48);
    return s - 2 * 65535;
}
static inline float bell_scale(float std_dev) { return std_dev / 37837.227f; }

template <class F>
static void parallel_rows(size_t rows, F body) {
    unsigned nt = std::thread::hardware_concurrency();
    if (nt == 0) nt = 1;
    if (nt > 32) nt = 32;
    if (rows < 64 || nt == 1) {
        body(0, rows);
        return;
    }
    std::vector<std::thread> ts;
    for (unsigned t = 0; t < nt; t++) {
        const size_t a = rows * t / nt, b = rows * (t + 1) / nt;
        if (a < b) ts.emplace_back([=] { body(a, b); });
    }
    for (auto& t : ts) t.join();
}

// One Q8_0 block from 32 floats: d = fp16(amax/127), q = lrintf(x / d) clamped.
static inline void quant_block(const float* x, uint8_t* blk) {
    float amax = 0.0f;
    for (int i = 0; i < 32; i++) amax = std::fmax(amax, std::fabs(x[i]));
    const uint16_t dh = f32_to_f16_rne(amax / 127.0f);
    const float d = f16_to_f32(dh);
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    std::memcpy(blk, &dh, 2);
    for (int i = 0; i < 32; i++) {
        float v = x[i] * id;
        v = v > 127.0f ? 127.0f : (v < -127.0f ? -127.0f : v);
        blk[2 + i] = (uint8_t)(int8_t)std::lrintf(v);
    }
}

}  // namespace jyc

using namespace jyc;

extern "C" {

JYC_API const char* jyc_version(void) { return "jieyu-b200 0.1.0 (sm_100a)"; }
JYC_API const char* jyc_last_error(void) { return g_error.c_str(); }
JYC_API long long jyc_kernel_launches(void) { return g_launches.load(); }

JYC_API int jyc_rope_table(int max_seq, int head_dim, float theta, float* cos_out,
                           float* sin_out) {
    if (max_seq <= 0 || head_dim <= 0 || (head_dim & 1) || !cos_out || !sin_out)
        return arg_error("jyc_rope_table: bad arguments");
    const int half = head_dim / 2;
    // Same float expressions, in the same order, as RoPETable::init.
    for (int i = 0; i < max_seq; i++) {
        for (int j = 0; j < half; j++) {
            float freq = 1.0f / powf(theta, 2.0f * j / head_dim);
            float angle = i * freq;
            cos_out[(size_t)i * half + j] = cosf(angle);
            sin_out[(size_t)i * half + j] = sinf(angle);
        }
    }
    return JYC_OK;
}

JYC_API int jyc_synth_f32(uint64_t seed, uint64_t stream, float std_dev, float* out, size_t n) {
    if (!out && n) return arg_error("jyc_synth_f32: null output");
    const uint64_t base = stream_base(seed, stream);
    const float sc = bell_scale(std_dev);
    parallel_rows(n, [&](size_t a, size_t b) {
        for (size_t i = a; i < b; i++) out[i] = (float)bell_int(base, i) * sc;
    });
    return JYC_OK;
}

JYC_API int jyc_synth_q8_0(uint64_t seed, uint64_t stream, float std_dev, void* out_blocks,
                           size_t rows, size_t k) {
    if (k % 32 != 0) return arg_error("jyc_synth_q8_0: k must be a multiple of 32");
    if (!out_blocks && rows) return arg_error("jyc_synth_q8_0: null output");
    const uint64_t base = stream_base(seed, stream);
    const float sc = bell_scale(std_dev);
    uint8_t* dst = static_cast<uint8_t*>(out_blocks);
    const size_t nb = k / 32;
    parallel_rows(rows, [&](size_t a, size_t b) {
        float x[32];
        for (size_t r = a; r < b; r++) {
            for (size_t bl = 0; bl < nb; bl++) {
                const size_t i0 = r * k + bl * 32;
                for (int i = 0; i < 32; i++) x[i] = (float)bell_int(base, i0 + i) * sc;
                quant_block(x, dst + (r * nb + bl) * 34);
            }
        }
    });
    return JYC_OK;
}

JYC_API int jyc_synth_ids(uint64_t seed, uint64_t stream, int vocab, int* out, size_t n) {
    if (vocab <= 0 || (!out && n)) return arg_error("jyc_synth_ids: bad arguments");
    const uint64_t base = stream_base(seed, stream);
    for (size_t i = 0; i < n; i++)
        out[i] = (int)(((mix64(base + i) >> 32) * (uint64_t)vocab) >> 32);
    return JYC_OK;
}

JYC_API int jyc_quantize_q8_0(const float* x, void* out_blocks, size_t rows, size_t k) {
    if (k % 32 != 0) return arg_error("jyc_quantize_q8_0: k must be a multiple of 32");
    if ((!x || !out_blocks) && rows) return arg_error("jyc_quantize_q8_0: null pointer");
    uint8_t* dst = static_cast<uint8_t*>(out_blocks);
    const size_t nb = k / 32;
    parallel_rows(rows, [&](size_t a, size_t b) {
        for (size_t r = a; r < b; r++)
            for (size_t bl = 0; bl < nb; bl++)
                quant_block(x + r * k + bl * 32, dst + (r * nb + bl) * 34);
    });
    return JYC_OK;
}

}  // extern "C"
