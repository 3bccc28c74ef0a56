// hostops.cu — the reference's operators with the reference's calling
// convention: HOST pointers in the reference's own layouts, synchronous,
// caller-owned buffers. Each call copies its operands to the device, runs
// the device entry point of capi.cu (the same kernels as every other path)
// and copies the result back. They exist so that a caller of the reference's
// free functions (qmat::matmul_q, matmul_w, rmsnorm, rope_pos, attention_q8,
// ffn, silu, kv_pack_q8; the C++ shim include/jieyu_b200_shim.hpp binds them
// under those names) reaches the GPU without changing a call; the
// throughput path keeps its weights resident (jyc_model_create).
#include <algorithm>
#include <cstring>
#include <vector>

#include "kernels.cuh"

using namespace jyc;

namespace {

#define TRY(x)                       \
    do {                             \
        int _r = (x);                \
        if (_r != JYC_OK) return _r; \
    } while (0)

// A device copy that frees itself (synchronous allocation: these entry
// points are not stream-ordered).
struct Dev {
    void* p = nullptr;
    ~Dev() {
        if (p) cudaFree(p);
    }
    int alloc(size_t bytes) {
        cudaError_t e = cudaMalloc(&p, std::max<size_t>(bytes, 16));
        if (e != cudaSuccess) {
            p = nullptr;
            return cuda_fail(e, "cudaMalloc");
        }
        return JYC_OK;
    }
    int up(const void* src, size_t bytes) {
        TRY(alloc(bytes));
        if (bytes) JYC_CUDA(cudaMemcpy(p, src, bytes, cudaMemcpyHostToDevice));
        return JYC_OK;
    }
    int down(void* dst, size_t bytes) const {
        if (bytes) JYC_CUDA(cudaMemcpy(dst, p, bytes, cudaMemcpyDeviceToHost));
        return JYC_OK;
    }
    template <class T>
    T* as() const { return static_cast<T*>(p); }
};

// Bytes of one quantised block and weights per block (qmat::block_bytes /
// block_elems, libs/matmul_libs/matmul_q.h:15-40).
bool block_shape(int qtype, size_t* bytes, size_t* elems) {
    switch (qtype) {
        case JYC_Q8_0: *bytes = 34; *elems = 32; return true;
        case JYC_Q4K: *bytes = 144; *elems = 256; return true;
        case JYC_Q5K: *bytes = 176; *elems = 256; return true;
        case JYC_Q6K: *bytes = 210; *elems = 256; return true;
        default: return false;
    }
}

// y[i] = g[i] * u[i] (ffn.h:14-17: the SwiGLU product after silu)
__global__ void mul_kernel(float* g, const float* u, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        g[i] = __fmul_rn(g[i], u[i]);
}

int matmul_q_dev(const float* dA, const void* hb, float* dC, int m, int n, int k, int qtype) {
    size_t bb = 0, be = 0;
    if (!block_shape(qtype, &bb, &be)) return arg_error("matmul_q: unknown block type");
    if (k % (int)be) return arg_error("matmul_q: k must be a multiple of the block size");
    Dev b;
    TRY(b.up(hb, (size_t)n * (k / be) * bb));
    if (qtype == JYC_Q8_0) {
        Dev qs, d;
        TRY(qs.alloc((size_t)n * k));
        TRY(d.alloc((size_t)n * (k / 32) * 2));
        TRY(jyc_q8_repack(b.p, n, k, qs.as<uint8_t>(), d.as<uint16_t>(), nullptr));
        TRY(jyc_matmul_q8(dA, qs.as<uint8_t>(), d.as<uint16_t>(), dC, m, n, k, nullptr));
        JYC_CUDA(cudaDeviceSynchronize());
        return JYC_OK;
    }
    TRY(jyc_matmul_qk(dA, b.p, dC, m, n, k, qtype, nullptr));
    JYC_CUDA(cudaDeviceSynchronize());
    return JYC_OK;
}

int matmul_f32_dev(const float* dA, const float* hB, float* dC, int m, int n, int k) {
    Dev b, bt;
    TRY(b.up(hB, (size_t)k * n * 4));
    TRY(bt.alloc((size_t)k * n * 4));
    TRY(jyc_f32_transpose(b.as<float>(), bt.as<float>(), k, n, nullptr));
    TRY(jyc_matmul_f32(dA, bt.as<float>(), dC, m, n, k, nullptr));
    JYC_CUDA(cudaDeviceSynchronize());
    return JYC_OK;
}

int matmul_f16_dev(const float* dA, const uint16_t* hB, float* dC, int m, int n, int k) {
    Dev b, bt;
    TRY(b.up(hB, (size_t)k * n * 2));
    TRY(bt.alloc((size_t)k * n * 2));
    TRY(jyc_f16_transpose(b.as<uint16_t>(), bt.as<uint16_t>(), k, n, nullptr));
    TRY(jyc_matmul_f16(dA, bt.as<uint16_t>(), dC, m, n, k, nullptr));
    JYC_CUDA(cudaDeviceSynchronize());
    return JYC_OK;
}

// matmul_w's dispatch (wmat_kernel.h:9-16) over a device A and C.
int matmul_w_dev(const jyc_wmat* B, int m, int n, int k, const float* dA, float* dC) {
    if (B->f) return matmul_f32_dev(dA, B->f, dC, m, n, k);
    if (B->q) return matmul_q_dev(dA, B->q, dC, m, n, k, B->qt);
    if (B->h) return matmul_f16_dev(dA, B->h, dC, m, n, k);
    JYC_CUDA(cudaMemset(dC, 0, (size_t)m * n * 4));  // an empty WMat: C = 0, as the reference
    return JYC_OK;
}

}  // namespace

extern "C" {

JYC_API int jyc_host_matmul_q(const float* a, const void* b, float* c, int m, int n, int k, int qtype) {
    clear_error();
    if (!a || !b || !c) return arg_error("matmul_q: null pointer");
    if (m <= 0 || n <= 0 || k <= 0) return arg_error("matmul_q: empty shape");
    Dev da, dc;
    TRY(da.up(a, (size_t)m * k * 4));
    TRY(dc.alloc((size_t)m * n * 4));
    TRY(matmul_q_dev(da.as<float>(), b, dc.as<float>(), m, n, k, qtype));
    return dc.down(c, (size_t)m * n * 4);
}

JYC_API int jyc_host_matmul_f32(int m, int n, int k, const float* A, const float* B, float* C) {
    clear_error();
    if (!A || !B || !C) return arg_error("matmul: null pointer");
    if (m <= 0 || n <= 0 || k <= 0) return arg_error("matmul: empty shape");
    Dev da, dc;
    TRY(da.up(A, (size_t)m * k * 4));
    TRY(dc.alloc((size_t)m * n * 4));
    TRY(matmul_f32_dev(da.as<float>(), B, dc.as<float>(), m, n, k));
    return dc.down(C, (size_t)m * n * 4);
}

JYC_API int jyc_host_matmul_f16(const float* a, const uint16_t* b, float* c, int m, int n, int k) {
    clear_error();
    if (!a || !b || !c) return arg_error("matmul_f16: null pointer");
    if (m <= 0 || n <= 0 || k <= 0) return arg_error("matmul_f16: empty shape");
    Dev da, dc;
    TRY(da.up(a, (size_t)m * k * 4));
    TRY(dc.alloc((size_t)m * n * 4));
    TRY(matmul_f16_dev(da.as<float>(), b, dc.as<float>(), m, n, k));
    return dc.down(c, (size_t)m * n * 4);
}

JYC_API int jyc_host_matmul_w(const jyc_wmat* B, int m, int n, int k, const float* A, float* C) {
    clear_error();
    if (!B || !A || !C) return arg_error("matmul_w: null pointer");
    if (m <= 0 || n <= 0 || k <= 0) return arg_error("matmul_w: empty shape");
    Dev da, dc;
    TRY(da.up(A, (size_t)m * k * 4));
    TRY(dc.alloc((size_t)m * n * 4));
    TRY(matmul_w_dev(B, m, n, k, da.as<float>(), dc.as<float>()));
    return dc.down(C, (size_t)m * n * 4);
}

JYC_API int jyc_host_rmsnorm(const float* x, float* y, const float* w, int n, float eps) {
    clear_error();
    if (!x || !y || !w) return arg_error("rmsnorm: null pointer");
    if (n <= 0) return arg_error("rmsnorm: n must be positive");
    Dev dx, dy, dw;
    TRY(dx.up(x, (size_t)n * 4));
    TRY(dw.up(w, (size_t)n * 4));
    TRY(dy.alloc((size_t)n * 4));
    TRY(jyc_rmsnorm(dx.as<float>(), dy.as<float>(), dw.as<float>(), 1, n, eps, nullptr));
    JYC_CUDA(cudaDeviceSynchronize());
    return dy.down(y, (size_t)n * 4);
}

JYC_API int jyc_host_rope_pos(float* q, int seq, int start_pos, int num_heads, int head_dim,
                              const float* cos_table, const float* sin_table) {
    clear_error();
    if (!q || !cos_table || !sin_table) return arg_error("rope_pos: null pointer");
    if (seq < 0 || start_pos < 0 || num_heads <= 0 || head_dim <= 0 || head_dim % 2)
        return arg_error("rope_pos: bad shape");
    if (seq == 0) return JYC_OK;
    const size_t half = (size_t)head_dim / 2, n = (size_t)seq * num_heads * head_dim;
    // only the table rows [start_pos, start_pos + seq) travel
    Dev dq, dc, ds;
    TRY(dq.up(q, n * 4));
    TRY(dc.up(cos_table + (size_t)start_pos * half, (size_t)seq * half * 4));
    TRY(ds.up(sin_table + (size_t)start_pos * half, (size_t)seq * half * 4));
    TRY(jyc_rope_pos(dq.as<float>(), seq, 0, num_heads, head_dim, dc.as<float>(), ds.as<float>(), nullptr));
    JYC_CUDA(cudaDeviceSynchronize());
    return dq.down(q, n * 4);
}

JYC_API int jyc_host_kv_pack_q8(const float* src, int8_t* dst, float* sc, int heads, int head_dim, int n) {
    clear_error();
    if (!src || !dst || !sc) return arg_error("kv_pack_q8: null pointer");
    if (heads <= 0 || head_dim <= 0 || n < 0) return arg_error("kv_pack_q8: bad shape");
    if (n == 0) return JYC_OK;
    const size_t e = (size_t)n * heads * head_dim, r = (size_t)n * heads;
    Dev ds, dd, dsc;
    TRY(ds.up(src, e * 4));
    TRY(dd.alloc(e));
    TRY(dsc.alloc(r * 4));
    TRY(jyc_kv_pack_q8(ds.as<float>(), dd.as<int8_t>(), dsc.as<float>(), heads, head_dim, n, nullptr));
    JYC_CUDA(cudaDeviceSynchronize());
    TRY(dd.down(dst, e));
    return dsc.down(sc, r * 4);
}

JYC_API int jyc_host_attention_q8(const float* Q, const float* K, const float* V, float* out, int seq,
                                  int start_pos, int num_heads, int num_kv_heads, int head_dim, int8_t* kc,
                                  float* ks, int8_t* vc, float* vs, int cap) {
    clear_error();
    if (num_kv_heads <= 0 || head_dim <= 0 || num_heads <= 0 || seq <= 0 || start_pos < 0)
        return jyc_attention_q8(Q, K, V, out, seq, start_pos, num_heads, num_kv_heads, head_dim, kc, ks, vc,
                                vs, cap, nullptr);  // the device entry reports the reference's message
    if (!Q || !K || !V || !out) return arg_error("attention_q8: null pointer");
    const size_t qd = (size_t)num_heads * head_dim, kvd = (size_t)num_kv_heads * head_dim;
    // no complete cache: a temporary one of seq rows at position 0, as the
    // reference does (attention_q8.h:40-46)
    const bool temp = !kc || !ks || !vc || !vs || cap <= 0;
    const int sp = temp ? 0 : start_pos, c = temp ? seq : cap;
    if ((long long)sp + seq > c) {
        set_error("attention_q8: KV cache capacity exceeded");
        return JYC_ERR_KV_OOM;
    }
    const size_t rows = (size_t)sp + seq;
    Dev dq, dk, dv, dout, k8, v8, kss, vss;
    TRY(dq.up(Q, (size_t)seq * qd * 4));
    TRY(dk.up(K, (size_t)seq * kvd * 4));
    TRY(dv.up(V, (size_t)seq * kvd * 4));
    TRY(dout.alloc((size_t)seq * qd * 4));
    TRY(k8.alloc(rows * kvd));
    TRY(v8.alloc(rows * kvd));
    TRY(kss.alloc(rows * num_kv_heads * 4));
    TRY(vss.alloc(rows * num_kv_heads * 4));
    if (!temp && sp > 0) {  // the cached positions [0, start_pos)
        JYC_CUDA(cudaMemcpy(k8.p, kc, (size_t)sp * kvd, cudaMemcpyHostToDevice));
        JYC_CUDA(cudaMemcpy(v8.p, vc, (size_t)sp * kvd, cudaMemcpyHostToDevice));
        JYC_CUDA(cudaMemcpy(kss.p, ks, (size_t)sp * num_kv_heads * 4, cudaMemcpyHostToDevice));
        JYC_CUDA(cudaMemcpy(vss.p, vs, (size_t)sp * num_kv_heads * 4, cudaMemcpyHostToDevice));
    }
    TRY(jyc_attention_q8(dq.as<float>(), dk.as<float>(), dv.as<float>(), dout.as<float>(), seq, sp, num_heads,
                         num_kv_heads, head_dim, k8.as<int8_t>(), kss.as<float>(), v8.as<int8_t>(),
                         vss.as<float>(), (int)rows, nullptr));
    JYC_CUDA(cudaDeviceSynchronize());
    TRY(dout.down(out, (size_t)seq * qd * 4));
    if (!temp) {  // the appended rows [start_pos, start_pos + seq) back into the caller's cache
        JYC_CUDA(cudaMemcpy(kc + (size_t)sp * kvd, k8.as<int8_t>() + (size_t)sp * kvd, (size_t)seq * kvd,
                            cudaMemcpyDeviceToHost));
        JYC_CUDA(cudaMemcpy(vc + (size_t)sp * kvd, v8.as<int8_t>() + (size_t)sp * kvd, (size_t)seq * kvd,
                            cudaMemcpyDeviceToHost));
        JYC_CUDA(cudaMemcpy(ks + (size_t)sp * num_kv_heads, kss.as<float>() + (size_t)sp * num_kv_heads,
                            (size_t)seq * num_kv_heads * 4, cudaMemcpyDeviceToHost));
        JYC_CUDA(cudaMemcpy(vs + (size_t)sp * num_kv_heads, vss.as<float>() + (size_t)sp * num_kv_heads,
                            (size_t)seq * num_kv_heads * 4, cudaMemcpyDeviceToHost));
    }
    return JYC_OK;
}

JYC_API int jyc_host_silu(const float* x, float* y, int n) {
    clear_error();
    if (n < 0) return arg_error("silu: negative n");
    if (n == 0) return JYC_OK;
    if (!x || !y) return arg_error("silu: null pointer");
    Dev dx, dy;
    TRY(dx.up(x, (size_t)n * 4));
    TRY(dy.alloc((size_t)n * 4));
    TRY(jyc_silu(dx.as<float>(), dy.as<float>(), n, nullptr));
    JYC_CUDA(cudaDeviceSynchronize());
    return dy.down(y, (size_t)n * 4);
}

JYC_API int jyc_host_ffn(const float* x, const jyc_wmat* w1, const jyc_wmat* w2, const jyc_wmat* w3, float* out,
                         int seq, int hidden, int intermediate) {
    clear_error();
    if (!x || !w1 || !w2 || !w3 || !out) return arg_error("ffn: null pointer");
    if (seq <= 0 || hidden <= 0 || intermediate <= 0) return arg_error("ffn: empty shape");
    const size_t nx = (size_t)seq * hidden, nf = (size_t)seq * intermediate;
    Dev dx, g, u, dout;
    TRY(dx.up(x, nx * 4));
    TRY(g.alloc(nf * 4));
    TRY(u.alloc(nf * 4));
    TRY(dout.alloc(nx * 4));
    // gate = W1 x, up = W3 x, gate = silu(gate) * up, out = W2 gate (ffn.h:7-19)
    TRY(matmul_w_dev(w1, seq, intermediate, hidden, dx.as<float>(), g.as<float>()));
    TRY(matmul_w_dev(w3, seq, intermediate, hidden, dx.as<float>(), u.as<float>()));
    TRY(jyc_silu(g.as<float>(), g.as<float>(), (int)nf, nullptr));
    mul_kernel<<<(unsigned)std::min<size_t>((nf + 255) / 256, 148 * 8), 256>>>(g.as<float>(), u.as<float>(), nf);
    JYC_LAUNCHED();
    TRY(matmul_w_dev(w2, seq, hidden, intermediate, g.as<float>(), dout.as<float>()));
    JYC_CUDA(cudaDeviceSynchronize());
    return dout.down(out, nx * 4);
}

}  // extern "C"
