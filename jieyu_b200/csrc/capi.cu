// capi.cu — operator-level C ABI over device pointers (one entry per reference
// operator; see include/jieyu_b200.h for the reference function each replaces).
#include <algorithm>
#include <cmath>
#include <mutex>
#include <vector>

#include "kernels.cuh"
#include "mega.cuh"
#include "tcgemm.cuh"
#include "skinny.cuh"

using namespace jyc;

namespace {

#define TRY(x)                          \
    do {                                \
        int _r = (x);                   \
        if (_r != JYC_OK) return _r;    \
    } while (0)

inline cudaStream_t S(void* s) { return static_cast<cudaStream_t>(s); }

// Stream-ordered scratch for one op call (freed in stream order).
struct Scratch {
    cudaStream_t s;
    std::vector<void*> ptrs;
    explicit Scratch(cudaStream_t st) : s(st) {}
    template <class T>
    int get(T** p, size_t count) {
        void* q = nullptr;
        cudaError_t e = cudaMallocAsync(&q, std::max<size_t>(count, 1) * sizeof(T), s);
        if (e != cudaSuccess) return cuda_fail(e, "cudaMallocAsync");
        ptrs.push_back(q);
        *p = static_cast<T*>(q);
        return JYC_OK;
    }
    ~Scratch() {
        for (void* q : ptrs) cudaFreeAsync(q, s);
    }
};

}  // namespace

extern "C" {

JYC_API int jyc_q8_repack(const void* blocks, int n, int k, uint8_t* qs, uint16_t* d, void* stream) {
    clear_error();
    if (!blocks || !qs || !d) return arg_error("q8_repack: null pointer");
    return launch_q8_repack(blocks, n, k, qs, d, 0, 1, S(stream));
}

JYC_API int jyc_matmul_q8(const float* A, const uint8_t* qs, const uint16_t* d, float* C, int m,
                          int n, int k, void* stream) {
    clear_error();
    if (!A || !qs || !d || !C) return arg_error("matmul_q8: null pointer");
    if (m <= 0 || n <= 0 || k <= 0 || k % 32) return arg_error("matmul_q8: need m,n > 0 and k % 32 == 0");
    if (m >= kTcMinRows) {
        // a real contraction: tcgen05 tiles of 128 weight rows x up to 128 rows of A
        cudaStream_t s = S(stream);
        int N = 0, splits = 1;
        tc_plan(n, k, m, kTcMaxSplits, &N, &splits);
        Scratch sc(s);
        __half* xs = nullptr;
        int* xe = nullptr;
        TRY(sc.get(&xs, tc_split_halves(m, N, k)));
        TRY(sc.get(&xe, (size_t)tc_padded_tokens(m, N)));
        uint8_t* rexp = nullptr;
        TRY(sc.get(&rexp, (size_t)n));
        TRY(launch_tc_rowexp(d, n, k, rexp, s));
        TRY(launch_tc_split(A, k, m, k, nullptr, 0.0f, N, xs, xe, s));
        TcGemm g{};
        g.qs = qs; g.d = d; g.rexp = rexp; g.n = n; g.k = k; g.xs = xs; g.xe = xe; g.T = m; g.N = N;
        g.y = C; g.ldy = n; g.err = device_error_word();
        g.splits = splits;
        if (g.splits > 1) {
            const size_t tiles = (size_t)((n + kTcRows - 1) / kTcRows) * ((m + N - 1) / N);
            TRY(sc.get(&g.part, (size_t)g.splits * m * n));
            TRY(sc.get(&g.cnt, tiles));
            JYC_CUDA(cudaMemsetAsync(g.cnt, 0, tiles * sizeof(unsigned int), s));
        }
        return launch_tc_gemm(g, TC_STORE, s);
    }
    if (m > 1 && ((uintptr_t)A & 15) == 0 && ((uintptr_t)qs & 15) == 0) {
        // a few rows: activations in registers, weights streamed once per 8 rows
        cudaStream_t s = S(stream);
        Scratch sc(s);
        SkinnyWork w{};
        const size_t cnt = skinny_counters(n);
        TRY(sc.get(&w.part, skinny_part_floats(n, k)));
        TRY(sc.get(&w.cnt, cnt));
        JYC_CUDA(cudaMemsetAsync(w.cnt, 0, cnt * sizeof(unsigned int), s));
        for (int r0 = 0; r0 < m; r0 += kSkMaxRows) {
            SkinnyGemm g{};
            g.x = A + (size_t)r0 * k; g.ldx = k; g.m = std::min(kSkMaxRows, m - r0); g.n = n; g.k = k;
            g.qs = qs; g.d = d; g.y = C + (size_t)r0 * n; g.ldy = n;
            TRY(launch_skinny(g, EPI_STORE, w, s));
        }
        return JYC_OK;
    }
    for (int r0 = 0; r0 < m; r0 += 8) {
        GemvArgs g{};
        g.x = A + (size_t)r0 * k; g.ldx = k; g.m = std::min(8, m - r0); g.n = n; g.k = k;
        g.qs = qs; g.d = d; g.y = C + (size_t)r0 * n; g.ldy = n;
        TRY(launch_gemv(g, W_Q8, EPI_STORE, S(stream)));
    }
    return JYC_OK;
}

JYC_API int jyc_matmul_qk(const float* A, const void* blocks, float* C, int m, int n, int k, int qtype,
                          void* stream) {
    clear_error();
    if (!A || !blocks || !C) return arg_error("matmul_qk: null pointer");
    return launch_kquant_matmul(A, m, n, k, static_cast<const uint8_t*>(blocks), qtype, C, S(stream));
}

JYC_API int jyc_f32_transpose(const float* B, float* Bt, int k, int n, void* stream) {
    clear_error();
    if (!B || !Bt) return arg_error("f32_transpose: null pointer");
    return launch_transpose(B, Bt, k, n, 0, 1, S(stream));
}

JYC_API int jyc_matmul_f32(const float* A, const float* Bt, float* C, int m, int n, int k,
                           void* stream) {
    clear_error();
    if (!A || !Bt || !C) return arg_error("matmul_f32: null pointer");
    if (m <= 0 || n <= 0 || k <= 0) return arg_error("matmul_f32: empty shape");
    if (k % 8 == 0 && m <= 8) {
        GemvArgs g{};
        g.x = A; g.ldx = k; g.m = m; g.n = n; g.k = k; g.wt = Bt; g.y = C; g.ldy = n;
        return launch_gemv(g, W_F32, EPI_STORE, S(stream));
    }
    return launch_matmul_f32_generic(A, Bt, C, m, n, k, S(stream));
}

JYC_API int jyc_f16_transpose(const uint16_t* B, uint16_t* Bt, int k, int n, void* stream) {
    clear_error();
    if (!B || !Bt) return arg_error("f16_transpose: null pointer");
    return launch_transpose_h(B, Bt, k, n, 0, 1, S(stream));
}

JYC_API int jyc_matmul_f16(const float* A, const uint16_t* Bt, float* C, int m, int n, int k,
                           void* stream) {
    clear_error();
    if (!A || !Bt || !C) return arg_error("matmul_f16: null pointer");
    if (m <= 0 || n <= 0 || k <= 0) return arg_error("matmul_f16: empty shape");
    if (k % 8 == 0 && m <= 8) {
        GemvArgs g{};
        g.x = A; g.ldx = k; g.m = m; g.n = n; g.k = k; g.wh = Bt; g.y = C; g.ldy = n;
        return launch_gemv(g, W_F16, EPI_STORE, S(stream));
    }
    return launch_matmul_f16_generic(A, Bt, C, m, n, k, S(stream));
}

JYC_API int jyc_rmsnorm(const float* x, float* y, const float* w, int rows, int n, float eps,
                        void* stream) {
    clear_error();
    if (!x || !y || !w) return arg_error("rmsnorm: null pointer");
    return launch_rmsnorm(x, y, w, rows, n, eps, S(stream));
}

JYC_API int jyc_rope_pos(float* q, int seq, int start_pos, int num_heads, int head_dim,
                         const float* cos_table, const float* sin_table, void* stream) {
    clear_error();
    if (!q || !cos_table || !sin_table) return arg_error("rope_pos: null pointer");
    if (seq < 0 || start_pos < 0 || num_heads <= 0 || head_dim <= 0) return arg_error("rope_pos: bad shape");
    return launch_rope(q, seq, start_pos, num_heads, head_dim, cos_table, sin_table, S(stream));
}

JYC_API int jyc_kv_pack_q8(const float* src, int8_t* dst, float* scale, int heads, int head_dim,
                           int n, void* stream) {
    clear_error();
    if (!src || !dst || !scale) return arg_error("kv_pack_q8: null pointer");
    if (heads <= 0 || head_dim <= 0 || n < 0) return arg_error("kv_pack_q8: bad shape");
    return launch_kv_pack(src, dst, scale, heads, head_dim, n, S(stream));
}

JYC_API int jyc_attention_q8(const float* Q, const float* K, const float* V, float* out, int seq,
                             int start_pos, int num_heads, int num_kv_heads, int head_dim,
                             int8_t* kc, float* ks, int8_t* vc, float* vs, int cap, void* stream) {
    clear_error();
    // argument checks of attention/x86/x86_classic.txt:2-8
    if (num_kv_heads <= 0 || num_heads % num_kv_heads != 0)
        return arg_error("attention_q8: num_heads must be a multiple of num_kv_heads");
    if (seq <= 0) return arg_error("attention_q8: seq must be positive");
    if (start_pos < 0) return arg_error("attention_q8: start_pos must not be negative");
    if (!kc || !ks || !vc || !vs || cap <= 0) return arg_error("attention_q8: KV cache pointers incomplete");
    if ((long long)start_pos + seq > cap) {
        set_error("attention_q8: KV cache capacity exceeded");
        return JYC_ERR_KV_OOM;
    }
    if (!Q || !K || !V || !out) return arg_error("attention_q8: null pointer");
    if (head_dim % 4 || head_dim > 256) return arg_error("attention_q8: head_dim must be a multiple of 4, <= 256");
    cudaStream_t s = S(stream);
    const int rows_max = 8;
    if (attn_smem_bytes(rows_max, num_heads, num_kv_heads, head_dim) > 200 * 1024)
        return arg_error("attention_q8: query-head group too large");
    KVView kv{kc, ks, vc, vs, (long long)num_kv_heads * head_dim, head_dim, num_kv_heads, 1, cap};
    const int maxpos = start_pos + seq;
    const int target = std::max(1, 296 / num_kv_heads);
    int chunk = (maxpos + target - 1) / target;
    chunk = std::max(64, (chunk + 63) / 64 * 64);
    const int nsplit = (maxpos + chunk - 1) / chunk;
    Scratch sc(s);
    int8_t* q8;
    float *qsc, *po, *pml;
    unsigned int* arrive;
    TRY(sc.get(&q8, (size_t)rows_max * num_heads * head_dim));
    TRY(sc.get(&qsc, (size_t)rows_max * num_heads));
    TRY(sc.get(&po, (size_t)rows_max * num_heads * nsplit * head_dim));
    TRY(sc.get(&pml, (size_t)rows_max * num_heads * nsplit * 2));
    TRY(sc.get(&arrive, (size_t)num_kv_heads));
    JYC_CUDA(cudaMemsetAsync(arrive, 0, num_kv_heads * sizeof(unsigned int), s));
    const int qd = num_heads * head_dim, kvd = num_kv_heads * head_dim;
    for (int r0 = 0; r0 < seq; r0 += rows_max) {
        const int rows = std::min(rows_max, seq - r0);
        // kv_pack_q8 of the new K,V rows into the cache + Q quantisation (inputs already roped)
        RopeQuantArgs rq{};
        rq.q = Q + (size_t)r0 * qd; rq.k = K + (size_t)r0 * kvd; rq.v = V + (size_t)r0 * kvd;
        rq.ldq = 0;  // set per array below
        rq.rows = rows; rq.H = num_heads; rq.KV = num_kv_heads; rq.hd = head_dim;
        rq.q8 = q8; rq.qsc = qsc; rq.kv = kv; rq.pos = PosSrc{nullptr, start_pos + r0};
        // Q, K, V have different row strides: run Q-only and K/V-only passes.
        {
            RopeQuantArgs a = rq;  // queries: H heads, stride qd
            a.KV = 0; a.ldq = qd;
            // with KV = 0 the kernel only visits query heads
            TRY(launch_rope_quant(a, s));
        }
        {
            RopeQuantArgs a = rq;  // keys and values: stride kvd, no query heads
            a.H = 0; a.ldq = kvd;
            a.q8 = nullptr; a.qsc = nullptr;
            TRY(launch_rope_quant(a, s));
        }
        AttnArgs at{};
        at.q8 = q8; at.qsc = qsc; at.kv = kv;
        at.rows = rows; at.H = num_heads; at.KV = num_kv_heads; at.hd = head_dim;
        at.chunk = chunk; at.nsplit = nsplit; at.scale = 1.0f / sqrtf((float)head_dim);
        at.part_o = po; at.part_ml = pml; at.arrive = arrive;
        at.out = out + (size_t)r0 * qd; at.ldo = qd; at.pos = PosSrc{nullptr, start_pos + r0};
        TRY(launch_attention(at, s));
    }
    return JYC_OK;
}

// ---------------------------------------------------------------------------
// jyc_attention_q8_noalloc: the same kernels with a fixed scratch array.
}  // extern "C"

namespace {

constexpr size_t kNaQ8 = 8 * 8192;        // int8 queries: 8 rows x num_heads*head_dim
constexpr size_t kNaQsc = 8 * 1024;       // floats: 8 rows x num_heads
constexpr size_t kNaPo = 1u << 20;        // floats: split partial outputs (4 MiB)
constexpr size_t kNaPml = 1u << 16;       // floats: split (max, sum) pairs
constexpr size_t kNaArrive = 256;         // uint32 arrival counters, one per kv head
constexpr size_t kNaBytes = kNaQ8 + (kNaQsc + kNaPo + kNaPml) * 4 + kNaArrive * 4;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNaBytes];

// address of the array on each device, resolved once with that device current
std::mutex g_na_mu;
std::vector<unsigned char*> g_na_addr;

int noalloc_scratch(unsigned char** out) {
    int dev = 0;
    JYC_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lk(g_na_mu);
    if ((int)g_na_addr.size() <= dev) g_na_addr.resize(dev + 1, nullptr);
    if (!g_na_addr[dev]) {
        void* p = nullptr;
        JYC_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
        g_na_addr[dev] = static_cast<unsigned char*>(p);
    }
    *out = g_na_addr[dev];
    return JYC_OK;
}

}  // namespace

extern "C" {

JYC_API int jyc_attention_q8_noalloc(const float* Q, const float* K, const float* V, float* out, int seq,
                                     int start_pos, int num_heads, int num_kv_heads, int head_dim,
                                     int8_t* kc, float* ks, int8_t* vc, float* vs, int cap, void* stream) {
    clear_error();
    if (num_kv_heads <= 0 || num_heads % num_kv_heads != 0)
        return arg_error("attention_q8_noalloc: num_heads must be a multiple of num_kv_heads");
    if (seq <= 0) return arg_error("attention_q8_noalloc: seq must be positive");
    if (start_pos < 0) return arg_error("attention_q8_noalloc: start_pos must not be negative");
    if (!kc || !ks || !vc || !vs || cap <= 0) return arg_error("attention_q8_noalloc: KV cache pointers incomplete");
    if ((long long)start_pos + seq > cap) {
        set_error("attention_q8_noalloc: KV cache capacity exceeded");
        return JYC_ERR_KV_OOM;
    }
    if (!Q || !K || !V || !out) return arg_error("attention_q8_noalloc: null pointer");
    if (head_dim % 4 || head_dim > 256)
        return arg_error("attention_q8_noalloc: head_dim must be a multiple of 4, <= 256");
    const int rows_max = 8;
    if (attn_smem_bytes(rows_max, num_heads, num_kv_heads, head_dim) > 200 * 1024)
        return arg_error("attention_q8_noalloc: query-head group too large");
    const int maxpos = start_pos + seq;
    const int target = std::max(1, 296 / num_kv_heads);
    int chunk = (maxpos + target - 1) / target;
    chunk = std::max(64, (chunk + 63) / 64 * 64);
    const int nsplit = (maxpos + chunk - 1) / chunk;
    const size_t need_q8 = (size_t)rows_max * num_heads * head_dim;
    const size_t need_qsc = (size_t)rows_max * num_heads;
    const size_t need_po = (size_t)rows_max * num_heads * nsplit * head_dim;
    const size_t need_pml = (size_t)rows_max * num_heads * nsplit * 2;
    if (need_q8 > kNaQ8 || need_qsc > kNaQsc || need_po > kNaPo || need_pml > kNaPml ||
        (size_t)num_kv_heads > kNaArrive)
        return arg_error("attention_q8_noalloc: call exceeds the fixed scratch (num_heads*head_dim <= 8192, "
                         "num_kv_heads <= 256, 8*num_heads*head_dim*splits <= 1048576 floats)");
    unsigned char* base = nullptr;
    TRY(noalloc_scratch(&base));
    int8_t* q8 = reinterpret_cast<int8_t*>(base);
    float* qsc = reinterpret_cast<float*>(base + kNaQ8);
    float* po = qsc + kNaQsc;
    float* pml = po + kNaPo;
    unsigned int* arrive = reinterpret_cast<unsigned int*>(pml + kNaPml);
    cudaStream_t s = S(stream);
    KVView kv{kc, ks, vc, vs, (long long)num_kv_heads * head_dim, head_dim, num_kv_heads, 1, cap};
    const int qd = num_heads * head_dim, kvd = num_kv_heads * head_dim;
    for (int r0 = 0; r0 < seq; r0 += rows_max) {
        const int rows = std::min(rows_max, seq - r0);
        RopeQuantArgs rq{};
        rq.q = Q + (size_t)r0 * qd; rq.k = K + (size_t)r0 * kvd; rq.v = V + (size_t)r0 * kvd;
        rq.rows = rows; rq.H = num_heads; rq.KV = num_kv_heads; rq.hd = head_dim;
        rq.q8 = q8; rq.qsc = qsc; rq.kv = kv; rq.pos = PosSrc{nullptr, start_pos + r0};
        {
            RopeQuantArgs a = rq;
            a.KV = 0; a.ldq = qd;
            TRY(launch_rope_quant(a, s));
        }
        {
            RopeQuantArgs a = rq;
            a.H = 0; a.ldq = kvd;
            a.q8 = nullptr; a.qsc = nullptr;
            TRY(launch_rope_quant(a, s));
        }
        AttnArgs at{};
        at.q8 = q8; at.qsc = qsc; at.kv = kv;
        at.rows = rows; at.H = num_heads; at.KV = num_kv_heads; at.hd = head_dim;
        at.chunk = chunk; at.nsplit = nsplit; at.scale = 1.0f / sqrtf((float)head_dim);
        at.part_o = po; at.part_ml = pml; at.arrive = arrive;
        at.out = out + (size_t)r0 * qd; at.ldo = qd; at.pos = PosSrc{nullptr, start_pos + r0};
        TRY(launch_attention(at, s));
    }
    return JYC_OK;
}

JYC_API int jyc_silu(const float* x, float* y, int n, void* stream) {
    clear_error();
    if ((!x || !y) && n > 0) return arg_error("silu: null pointer");
    return launch_silu(x, y, n, S(stream));
}

JYC_API int jyc_argmax(const float* logits, int n, int* out_index, void* stream) {
    clear_error();
    if (!logits || !out_index) return arg_error("argmax: null pointer");
    cudaStream_t s = S(stream);
    Scratch sc(s);
    unsigned long long* slot;
    TRY(sc.get(&slot, 1));
    JYC_CUDA(cudaMemsetAsync(slot, 0, sizeof(unsigned long long), s));
    return launch_argmax(logits, n, slot, out_index, s);
}

JYC_API int jyc_sample(float* logits, int vocab_size, float temperature, float repetition_penalty,
                       const int* out_ids, int prompt_len, int len, unsigned int* rng, int* next, void* stream) {
    clear_error();
    if (!logits || !rng || !next || vocab_size <= 0) return arg_error("sample: bad arguments");
    if (repetition_penalty != 1.0f && (!out_ids || prompt_len < 0 || len < prompt_len))
        return arg_error("sample: penalty needs out_ids[prompt_len..len)");
    return launch_sample(logits, vocab_size, temperature, repetition_penalty, out_ids, prompt_len, len, rng, next,
                         S(stream));
}

}  // extern "C"
