// model.cu — the device-resident token loop behind jyc_model_* / jyc_generate.
//
// Mirrors the reference call stack
//   generate (generate.h:90-112) -> generate_cached (generate.h:9-89)
//     -> forward_cached (forward.h:47-96) -> transformer_layer (transformer_layer.h:10-90)
// with every weight uploaded once (the bind_model point, pipeline.h:63-153), a
// device KV cache, and token ids that stay on the device: the last phase of a
// step (LM head + argmax) appends the next id and clears `active` when the
// reference loop would stop (EOS, max_new, max_seq).
//
// Decode step: Q8_0 models run ONE persistent cooperative kernel per token
// (mega.cu); other models (fp32 weights) run the generic kernels replayed as a
// CUDA graph. Prompt rows go through the generic kernels in chunks of 8 rows.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "mega.cuh"
#include "prefill.cuh"
#include "tcgemm.cuh"
#include "skinny.cuh"
#include "batch.cuh"

using namespace jyc;

namespace {

constexpr int kMT = 8;  // activation rows per prefill chunk
constexpr int kMaxBatchSeqs = 256;  // sequences of one batched decode

struct DevMat {  // one weight matrix on the device, [n][k]
    uint8_t* qs = nullptr;   // Q8: row-major copy (generic kernels)
    uint16_t* d = nullptr;
    uint8_t* tq = nullptr;   // Q8: tiled copy (decode megakernel), when `tiled`
    uint16_t* td = nullptr;
    uint8_t* rexp = nullptr; // Q8: per-row exponent of the largest scale (tensor-core path)
    float* f = nullptr;
    uint16_t* h = nullptr;   // fp16 [n][k]
    uint8_t* kqb = nullptr;  // K-quant super-blocks as the reference holds them, [n][k/256], read in place
    int kqt = -1;            // their type (JYC_Q4K / JYC_Q5K / JYC_Q6K)
    int n = 0, k = 0;
    bool tiled = false;
    double bytes() const {
        return kqb ? (double)n * (k / 256) * kquant_block_bytes(kqt)
               : f ? 4.0 * n * k : h ? 2.0 * n * k : (double)n * k * 34.0 / 32.0;
    }
    int wtype() const { return f ? W_F32 : h ? W_F16 : W_Q8; }
};

// Kernel classes of one generic decode step (for per-kernel timing).
enum KClass { K_EMBED = 0, K_QKV, K_ROPEQ, K_ATTN, K_OPROJ, K_GATEUP, K_DOWN, K_HEAD, K_NCLASS };

// Event marks recorded after each launch while a profiling graph is captured.
struct Prof {
    std::vector<cudaEvent_t> ev;
    std::vector<int> cls;
    cudaStream_t s = nullptr;
    int mark(int c) {
        cudaEvent_t e;
        cudaError_t r = cudaEventCreate(&e);
        if (r != cudaSuccess) return cuda_fail(r, "cudaEventCreate");
        // external record: inside a stream capture this becomes an event-record
        // node, so the event is timestamped on every graph replay
        r = cudaEventRecordWithFlags(e, s, cudaEventRecordExternal);
        if (r != cudaSuccess) return cuda_fail(r, "cudaEventRecord");
        ev.push_back(e);
        cls.push_back(c);
        return JYC_OK;
    }
    ~Prof() {
        for (cudaEvent_t e : ev) cudaEventDestroy(e);
    }
};

struct DevLayer {
    float* rms1 = nullptr;
    float* rms2 = nullptr;
    float* bias = nullptr;  // fused q|k|v bias, or null
    DevMat qkv, o, gateup, down;
    DevMat kq[7];           // K-quant models: q, k, v, o, gate, up, down blocks read in place
};

}  // namespace

struct jyc_model {
    int L = 0, D = 0, H = 0, KV = 0, hd = 0, F = 0, V = 0, max_seq = 0;
    int Ve = 0;          // embedding rows (token ids); V = LM-head rows
    int vocab_off = 0;   // token id of LM-head row 0 (vocabulary-sharded head)
    int q_dim = 0, kv_dim = 0, nqkv = 0;
    int wtype = W_Q8;
    // K-quant models whose layer matrices are all K-quant: the blocks stay as
    // they are on the device and the per-op path reads them in place
    bool kq_path = false;
    float* kq_xn = nullptr;  // RMSNorm rows [kMT][D]
    float* kq_t = nullptr;   // O / down rows before the residual add [kMT][D]
    float* kq_g = nullptr;   // gate rows [kMT][F]
    float* kq_u = nullptr;   // up rows [kMT][F]
    bool tiled = false;  // Q8 matrices in the 512-column tiled layout (megakernel models)
    std::vector<DevLayer> layers;
    DevMat head;
    float* embed_f = nullptr;  // fp32 embedding [V][D], or
    DevMat embed_q;            // Q8 embedding (may alias head)
    float* final_norm = nullptr;
    float *cos_t = nullptr, *sin_t = nullptr;
    // KV cache [L][KV][max_seq][hd] int8, scales [L][KV][max_seq]
    int8_t *k8 = nullptr, *v8 = nullptr;
    float *ks = nullptr, *vs = nullptr;
    // activations / scratch
    float *X = nullptr, *qkv = nullptr, *attn = nullptr, *h = nullptr, *logits = nullptr;
    unsigned int* stag = nullptr;  // the sampler's penalty tags: first index [V], counts [V]
    float* tmp = nullptr;
    int8_t* q8 = nullptr;
    float* qsc = nullptr;
    float *part_o = nullptr, *part_ml = nullptr;
    unsigned int* arrive = nullptr;
    int chunk = 64, nsplit = 1;
    // megakernel decode
    bool mega = false;
    MegaArgs margs{};
    int pf_rows = 0;           // tokens per batched prefill pass (0: generic prefill)
    // tensor parallel inside the decode kernel: this rank's receive area and
    // the peers' areas mapped through CUDA IPC
    unsigned char* tp_region = nullptr;
    int tp_size = 0, tp_rank = 0, tp_so = 1, tp_sd = 1;
    std::vector<void*> tp_mapped;
    // batched prefill on the tensor cores: split activations, per-token
    // exponents, split-K partial sums and their arrival counters
    float* pf_part = nullptr;  // [pf_rows][D]: a shard's O / down partial rows (tensor-parallel prefill)
    __half* tc_xs = nullptr;
    int* tc_xe = nullptr;
    float* tc_part = nullptr;
    size_t tc_part_floats = 0;
    unsigned int* tc_cnt = nullptr;
    MegaLayer* d_mlayers = nullptr;
    DevState* st = nullptr;
    int* tokens = nullptr;  // [max_seq + 1]
    cudaStream_t stream = nullptr;
    cudaGraphExec_t step_exec = nullptr;
    cudaGraphExec_t prof_exec = nullptr;  // generic decode step with event marks
    Prof* prof = nullptr;                 // set while capturing prof_exec
    std::unique_ptr<Prof> prof_marks;
    std::vector<void*> allocs;
    double weight_bytes = 0.0;

    template <class T>
    int alloc(T** p, size_t count) {
        void* q = nullptr;
        if (count == 0) count = 1;
        cudaError_t e = cudaMalloc(&q, count * sizeof(T));
        if (e != cudaSuccess) {
            set_error(std::string("cudaMalloc: ") + cudaGetErrorString(e));
            return JYC_ERR_NOMEM;
        }
        allocs.push_back(q);
        *p = static_cast<T*>(q);
        return JYC_OK;
    }
    ~jyc_model() {
        for (void* p : tp_mapped) cudaIpcCloseMemHandle(p);
        if (step_exec) cudaGraphExecDestroy(step_exec);
        if (prof_exec) cudaGraphExecDestroy(prof_exec);
        prof_marks.reset();
        for (void* p : allocs) cudaFree(p);
        if (stream) cudaStreamDestroy(stream);
    }

    KVView kv_layer(int l) const {
        KVView v;
        const size_t lay = (size_t)KV * max_seq;
        v.k = k8 + (size_t)l * lay * hd;
        v.v = v8 + (size_t)l * lay * hd;
        v.ks = ks + (size_t)l * lay;
        v.vs = vs + (size_t)l * lay;
        v.pos_stride = hd;
        v.head_stride = (long long)max_seq * hd;
        v.spos_stride = 1;
        v.shead_stride = max_seq;
        v.cap = max_seq;
        return v;
    }
};

namespace {

#define TRY(x)                       \
    do {                             \
        int _r = (x);                \
        if (_r != JYC_OK) return _r; \
    } while (0)

// Uploads one reference weight (host, reference layout) into rows
// [row_off + r*row_stride] of `dst` (device layout, n_total rows x k).
int upload_wmat(jyc_model* m, const jyc_wmat& w, int n, int k, DevMat& dst, int n_total, int row_off,
                int row_stride, void* staging, size_t staging_bytes, int expect_type) {
    // fp16 weights ([in][out] halves, matmul_f16.h) stay fp16 on the device
    const bool f16 = w.h != nullptr && w.f == nullptr && w.q == nullptr;
    // K-quant blocks (Q4_K / Q5_K / Q6_K) are dequantised to the reference's
    // fp32 values here and then run on the fp32 path
    const bool kq = w.q != nullptr && w.f == nullptr && kquant_block_bytes(w.qt) != 0;
    const bool q8 = w.q != nullptr && !kq;
    if (q8 && w.qt != JYC_Q8_0) {
        set_error("quantised weights must be Q8_0, Q4_K, Q5_K or Q6_K (got type " + std::to_string((int)w.qt) + ")");
        return JYC_ERR_UNSUPPORTED;
    }
    if (!q8 && !kq && !f16 && w.f == nullptr) {
        set_error("missing weight tensor");
        return JYC_ERR_ARG;
    }
    if ((q8 ? W_Q8 : f16 ? W_F16 : W_F32) != expect_type) {
        set_error("linear weights must all be Q8_0, all fp16, or all fp32 / K-quant");
        return JYC_ERR_UNSUPPORTED;
    }
    if (kq && k % 256) return arg_error("K-quant weights need an input dimension that is a multiple of 256");
    if (dst.n == 0) {  // first piece: allocate the whole (fused) matrix
        dst.n = n_total;
        dst.k = k;
        dst.tiled = q8 && m->tiled;
        if (q8) {
            TRY(m->alloc(&dst.qs, (size_t)n_total * k));
            TRY(m->alloc(&dst.d, (size_t)n_total * (k / 32)));
            if (dst.tiled) {
                TRY(m->alloc(&dst.tq, (size_t)n_total * k));
                TRY(m->alloc(&dst.td, (size_t)n_total * (k / 32)));
            }
        } else if (f16) {
            TRY(m->alloc(&dst.h, (size_t)n_total * k));
        } else {
            TRY(m->alloc(&dst.f, (size_t)n_total * k));
        }
    }
    const size_t bytes = q8    ? (size_t)n * (k / 32) * 34
                         : kq  ? (size_t)n * (k / 256) * kquant_block_bytes(w.qt)
                         : f16 ? (size_t)n * k * 2
                               : (size_t)n * k * 4;
    if (bytes > staging_bytes) {
        set_error("internal: staging buffer too small");
        return JYC_ERR_ARG;
    }
    const void* src = w.f ? (const void*)w.f : f16 ? (const void*)w.h : w.q;
    JYC_CUDA(cudaMemcpyAsync(staging, src, bytes, cudaMemcpyHostToDevice, m->stream));
    if (q8) {
        TRY(launch_q8_repack(staging, n, k, dst.qs, dst.d, row_off, row_stride, m->stream));
        if (dst.tiled)
            TRY(launch_q8_repack_tiled(staging, n, k, dst.tq, dst.td, n_total, row_off, row_stride, m->stream));
    } else if (kq) {
        TRY(launch_kquant_dequant(static_cast<const uint8_t*>(staging), n, k, w.qt, dst.f, row_off, row_stride,
                                  m->stream));
    } else if (f16) {
        TRY(launch_transpose_h(static_cast<const uint16_t*>(staging), dst.h, k, n, row_off, row_stride, m->stream));
    } else
        TRY(launch_transpose(static_cast<const float*>(staging), dst.f, k, n, row_off, row_stride, m->stream));
    // the staging buffer is reused by the next upload: wait for this one
    JYC_CUDA(cudaStreamSynchronize(m->stream));
    return JYC_OK;
}

// A K-quant matrix kept as the reference holds it ([n][k/256] super-blocks):
// the in-place path's weights.
int upload_kq_raw(jyc_model* m, const jyc_wmat& w, int n, int k, DevMat& dst) {
    if (k % 256) return arg_error("K-quant weights need an input dimension that is a multiple of 256");
    const size_t bytes = (size_t)n * (k / 256) * kquant_block_bytes(w.qt);
    TRY(m->alloc(&dst.kqb, bytes));
    JYC_CUDA(cudaMemcpy(dst.kqb, w.q, bytes, cudaMemcpyHostToDevice));
    dst.kqt = w.qt;
    dst.n = n;
    dst.k = k;
    return JYC_OK;
}

int upload_f32(jyc_model* m, const float* src, size_t n, float** dst) {
    TRY(m->alloc(dst, n));
    JYC_CUDA(cudaMemcpy(*dst, src, n * sizeof(float), cudaMemcpyHostToDevice));
    return JYC_OK;
}

// Q8_0 models whose shapes fit the tiled layout decode with the megakernel.
bool mega_eligible(const jyc_model* m, const jyc_model_desc* d) {
    if (m->wtype != W_Q8 || d->lm_head.q == nullptr || d->lm_head.qt != JYC_Q8_0) return false;
    if (d->embed.f == nullptr && (d->embed.q == nullptr || d->embed.qt != JYC_Q8_0)) return false;
    const int n16[] = {m->nqkv, m->D, 2 * m->F, m->V, m->Ve};
    for (int n : n16)
        if (n % 16) return false;
    const int k32[] = {m->D, m->q_dim, m->F};
    for (int k : k32)
        if (k % 32) return false;
    // head_dim 64 or 128; query heads per kv head <= 8
    return (m->hd == 64 || m->hd == 128) && m->H / m->KV <= 8;
}

MegaMat mega_mat(const DevMat& w, int nctas, bool splittable, int only_cpg = 0) {
    MegaMat mm{};
    mm.qs = w.tq;
    mm.d = w.td;
    mm.n = w.n;
    mm.k = w.k;
    mega_plan(mm, nctas, splittable, only_cpg);
    return mm;
}

// Shared bytes an attention item's plan may take before its sub-chunk is
// halved (JYC_MEGA_ATTN_CAP in KB overrides: tuning of ring depth against
// attention copies).
static int mega_attn_cap() {
    int kb = 96;
    if (const char* e = std::getenv("JYC_MEGA_ATTN_CAP")) kb = std::max(8, std::atoi(e));
    return kb * 1024;
}

// Column blocks per group of the O projection: one (each group then waits
// only for the attention items of the kv heads inside its 512 columns and
// merges just those). JYC_MEGA_O_CPG overrides it (0: the cost model).
static int mega_o_cpg() {
    int c = 1;
    if (const char* e = std::getenv("JYC_MEGA_O_CPG")) c = std::max(0, std::atoi(e));
    return c;
}

int setup_mega(jyc_model* m) {
    m->mega = false;
    const int nctas = mega_num_ctas();
    MegaArgs& a = m->margs;
    a = MegaArgs{};
    std::vector<MegaLayer> ml(m->L);
    int sq = 1, so = 1, sd = 1;
    for (int l = 0; l < m->L; l++) {
        const DevLayer& ly = m->layers[l];
        // QKV, O and down may split K (their readers sum the partials);
        // gate/up (SwiGLU) and the LM head (argmax) need whole rows
        ml[l].qkv = mega_mat(ly.qkv, nctas, true);
        ml[l].o = mega_mat(ly.o, nctas, true, mega_o_cpg());
        ml[l].gu = mega_mat(ly.gateup, nctas, false);
        ml[l].dn = mega_mat(ly.down, nctas, true);
        sq = std::max(sq, ml[l].qkv.spl);
        so = std::max(so, ml[l].o.spl);
        sd = std::max(sd, ml[l].dn.spl);
        ml[l].rms1 = ly.rms1;
        ml[l].rms2 = ly.rms2;
        ml[l].bias = ly.bias;
    }
    TRY(m->alloc(&m->d_mlayers, (size_t)m->L));
    JYC_CUDA(cudaMemcpy(m->d_mlayers, ml.data(), sizeof(MegaLayer) * m->L, cudaMemcpyHostToDevice));
    a.layers = m->d_mlayers;
    a.L = m->L;
    a.head = mega_mat(m->head, nctas, false);
    MegaMat* hd_dev = nullptr;
    TRY(m->alloc(&hd_dev, 1));
    JYC_CUDA(cudaMemcpy(hd_dev, &a.head, sizeof(MegaMat), cudaMemcpyHostToDevice));
    a.head_dev = hd_dev;
    a.final_norm = m->final_norm;
    a.ef = m->embed_f;
    a.eqs = m->embed_q.tq;
    a.ed = m->embed_q.td;
    a.D = m->D; a.H = m->H; a.KV = m->KV; a.hd = m->hd; a.F = m->F; a.V = m->V;
    a.Ve = m->Ve; a.vocab_off = m->vocab_off;
    a.cos_t = m->cos_t;
    a.sin_t = m->sin_t;
    a.k8 = m->k8; a.v8 = m->v8; a.ks = m->ks; a.vs = m->vs;
    a.max_seq = m->max_seq;
    a.X = m->X; a.qkv = m->qkv; a.h = m->h; a.logits = m->logits; a.stag = m->stag;
    TRY(m->alloc(&a.Xb, (size_t)m->D));
    TRY(m->alloc(&a.pq, (size_t)sq * m->nqkv));
    TRY(m->alloc(&a.po, (size_t)so * m->D));
    TRY(m->alloc(&a.pd, (size_t)sd * m->D));
    TRY(m->alloc(&a.attn, (size_t)m->q_dim));
    // attention split plan: about one (kv head, split) item per CTA at the
    // step's context (the kernel sizes the splits from the position: at
    // least chunk_min positions, a multiple of 64; at most `chunk`, the
    // length at max_seq, which sizes the sub-chunk copies)
    const int per_head = std::max(1, nctas / m->KV);
    int chunk = (m->max_seq + per_head - 1) / per_head;
    chunk = std::max(128, (chunk + 63) / 64 * 64);  // >= 128: few splits to merge at short contexts
    a.chunk = chunk;
    a.chunk_min = 128;
    a.per_head = per_head;
    const int nsplit_max = (m->max_seq + chunk - 1) / chunk;  // splits at max_seq
    a.nsplit = std::max(nsplit_max, per_head);                // any step has at most per_head
    a.nsplit += a.nsplit & 1;  // even: a head's (m, l) pairs are whole 16-byte chunks
    TRY(m->alloc(&a.part_o, (size_t)m->H * a.nsplit * m->hd));
    TRY(m->alloc(&a.part_ml, (size_t)m->H * a.nsplit * 2));
    a.scale = 1.0f / sqrtf((float)m->hd);
    a.st = m->st;
    a.tokens = m->tokens;
    TRY(m->alloc(&a.bar, 1));
    JYC_CUDA(cudaMemset(a.bar, 0, sizeof(unsigned int)));
    a.err = device_error_word();
    a.kmax = std::max({m->D, m->q_dim, m->F});
    a.kx = std::max(m->D, m->q_dim);
    // attention items: one per (kv head, split) at long contexts; one per
    // (query head, split) when those fit the CTAs at full context (short
    // contexts: more parallelism, fewer splits to merge per item)
    a.gsz = (m->KV * (m->H / m->KV) * nsplit_max <= nctas) ? 1 : m->H / m->KV;
    a.att_nb = mega_attn_nb(a.kx, a.kmax, a.gsz, m->hd, a.chunk, mega_attn_cap());
    a.xs_bytes = mega_xs_bytes(a.kx, a.kmax, a.gsz, m->hd, a.att_nb);
    // the x region also stages one head's split partials behind the
    // attention rows, and a 16-byte slice of up to 8 x 8 partial rows (+ the
    // base row) behind the residual row
    a.xs_bytes = std::max({a.xs_bytes, 4 * (m->q_dim + a.nsplit * m->hd + 2 * a.nsplit),
                           4 * (m->D + (kMegaMaxTP * 8 + 1) * 4)});
    a.xs_bytes = (a.xs_bytes + 127) / 128 * 128;
    // attention arrival counters: [2][L][KV] (two steps' worth; see the kernel)
    TRY(m->alloc(&a.acnt, (size_t)2 * m->L * m->KV));
    JYC_CUDA(cudaMemset(a.acnt, 0, sizeof(unsigned int) * 2 * m->L * m->KV));
    // ring as deep as the shared memory allows (227 KB per CTA, at least 2 slots)
    const int st_smem = mega_static_smem(a.gsz, m->hd);
    if (st_smem < 0) return cuda_fail(cudaGetLastError(), "mega: kernel attributes");
    const int budget = 227 * 1024 - st_smem - 128 - a.xs_bytes;
    a.nslots = std::min(kMegaMaxSlots, budget / kMegaSlotBytes);
    a.win0 = 0;
    a.win1 = 2 * m->L + 1;  // the whole step
    if (a.nslots < 2) return JYC_OK;  // does not fit: generic decode
    const int smem = mega_smem_bytes(a);
    TRY(prepare_mega_kernel(smem, a.gsz, m->hd));
    m->mega = true;
    return JYC_OK;
}

int build_model(jyc_model* m, const jyc_model_desc* d) {
    if (!d || !d->layers || d->num_layers <= 0) return arg_error("model: no layers");
    if (d->hidden <= 0 || d->num_heads <= 0 || d->num_kv_heads <= 0 || d->head_dim <= 0 ||
        d->intermediate <= 0 || d->vocab_size <= 0 || d->max_seq <= 0)
        return arg_error("model: non-positive hyper-parameter");
    if (d->num_heads % d->num_kv_heads) return arg_error("model: num_heads % num_kv_heads != 0");
    if (d->head_dim % 4 || d->head_dim > 256) return arg_error("model: head_dim must be a multiple of 4, <= 256");
    if (!d->final_rms_weight || !d->cos_table || !d->sin_table)
        return arg_error("model: missing final norm or RoPE tables");
    m->L = d->num_layers; m->D = d->hidden; m->H = d->num_heads; m->KV = d->num_kv_heads;
    m->hd = d->head_dim; m->F = d->intermediate; m->V = d->vocab_size; m->max_seq = d->max_seq;
    m->Ve = d->embed_rows > 0 ? d->embed_rows : d->vocab_size;
    m->vocab_off = d->vocab_offset;
    if (m->vocab_off < 0 || (long long)m->vocab_off + m->V > m->Ve)
        return arg_error("model: LM-head rows must be a slice of the embedding's vocabulary");
    m->q_dim = m->H * m->hd; m->kv_dim = m->KV * m->hd; m->nqkv = m->q_dim + 2 * m->kv_dim;
    // K-quant: the fp32 path; fp16: halves on the device (generic kernels)
    m->wtype = (d->layers[0].Wq.q != nullptr && d->layers[0].Wq.qt == JYC_Q8_0) ? W_Q8
               : (d->layers[0].Wq.h != nullptr && d->layers[0].Wq.f == nullptr && d->layers[0].Wq.q == nullptr)
                   ? W_F16
                   : W_F32;
    // K-quant models (every layer matrix Q4_K / Q5_K / Q6_K, as the
    // reference's downloads are) keep their blocks and read them in place;
    // a mix with fp32 matrices runs every matrix as fp32. JYC_KQ_FP32=1
    // selects the fp32 path for all (a comparison switch).
    m->kq_path = m->wtype == W_F32;
    if (const char* e = std::getenv("JYC_KQ_FP32")) m->kq_path = m->kq_path && std::atoi(e) == 0;
    for (int l = 0; l < d->num_layers && m->kq_path; l++) {
        const jyc_layer_weights& w = d->layers[l];
        for (const jyc_wmat* x : {&w.Wq, &w.Wk, &w.Wv, &w.Wo, &w.W1, &w.W3, &w.W2})
            if (x->f != nullptr || x->q == nullptr || kquant_block_bytes(x->qt) == 0) m->kq_path = false;
    }
    const int kq = m->wtype == W_Q8 ? 32 : 8;
    if (m->D % kq || m->q_dim % kq || m->F % kq)
        return arg_error("model: hidden, heads*head_dim and intermediate must be multiples of " +
                         std::to_string(kq));
    if (attn_smem_bytes(kMT, m->H, m->KV, m->hd) > 200 * 1024)
        return arg_error("model: query-head group too large for the attention kernel");
    m->tiled = mega_eligible(m, d);
    if (m->tiled && mega_negative_scales(true) < 0) return cuda_fail(cudaGetLastError(), "mega: scale flag");

    JYC_CUDA(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking));
    TRY(prepare_kernels());

    // staging for uploads: the largest single host tensor
    auto tb = [&](int n, int k) { return m->wtype == W_Q8 ? (size_t)n * (k / 32) * 34 : (size_t)n * k * 4; };
    size_t stage = std::max({tb(m->q_dim, m->D), tb(m->kv_dim, m->D), tb(m->D, m->q_dim), tb(m->F, m->D),
                             tb(m->D, m->F)});
    const bool head_q8 = d->lm_head.q != nullptr && d->lm_head.qt == JYC_Q8_0;
    const size_t head_bytes = head_q8 ? (size_t)std::max(m->V, m->Ve) * (m->D / 32) * 34
                                      : (size_t)std::max(m->V, m->Ve) * m->D * 4;
    stage = std::max(stage, head_bytes);
    void* staging = nullptr;
    JYC_CUDA(cudaMalloc(&staging, stage));
    std::unique_ptr<void, void (*)(void*)> stage_guard(staging, [](void* p) { cudaFree(p); });

    m->layers.resize(m->L);
    for (int l = 0; l < m->L; l++) {
        const jyc_layer_weights& w = d->layers[l];
        DevLayer& dl = m->layers[l];
        if (!w.rms1_weight || !w.rms2_weight)
            return arg_error("model: missing RMSNorm weight in layer " + std::to_string(l));
        TRY(upload_f32(m, w.rms1_weight, m->D, &dl.rms1));
        TRY(upload_f32(m, w.rms2_weight, m->D, &dl.rms2));
        const int wt = m->wtype;
        if (m->kq_path) {
            const jyc_wmat* src[7] = {&w.Wq, &w.Wk, &w.Wv, &w.Wo, &w.W1, &w.W3, &w.W2};
            const int nn[7] = {m->q_dim, m->kv_dim, m->kv_dim, m->D, m->F, m->F, m->D};
            const int kk[7] = {m->D, m->D, m->D, m->q_dim, m->D, m->D, m->F};
            for (int i = 0; i < 7; i++) {
                TRY(upload_kq_raw(m, *src[i], nn[i], kk[i], dl.kq[i]));
                m->weight_bytes += dl.kq[i].bytes();
            }
        } else {
            TRY(upload_wmat(m, w.Wq, m->q_dim, m->D, dl.qkv, m->nqkv, 0, 1, staging, stage, wt));
            TRY(upload_wmat(m, w.Wk, m->kv_dim, m->D, dl.qkv, m->nqkv, m->q_dim, 1, staging, stage, wt));
            TRY(upload_wmat(m, w.Wv, m->kv_dim, m->D, dl.qkv, m->nqkv, m->q_dim + m->kv_dim, 1, staging, stage,
                            wt));
            TRY(upload_wmat(m, w.Wo, m->D, m->q_dim, dl.o, m->D, 0, 1, staging, stage, wt));
            TRY(upload_wmat(m, w.W1, m->F, m->D, dl.gateup, 2 * m->F, 0, 2, staging, stage, wt));
            TRY(upload_wmat(m, w.W3, m->F, m->D, dl.gateup, 2 * m->F, 1, 2, staging, stage, wt));
            TRY(upload_wmat(m, w.W2, m->D, m->F, dl.down, m->D, 0, 1, staging, stage, wt));
        }
        if (w.bq || w.bk || w.bv) {
            std::vector<float> b(m->nqkv, 0.0f);
            if (w.bq) std::memcpy(b.data(), w.bq, m->q_dim * 4);
            if (w.bk) std::memcpy(b.data() + m->q_dim, w.bk, m->kv_dim * 4);
            if (w.bv) std::memcpy(b.data() + m->q_dim + m->kv_dim, w.bv, m->kv_dim * 4);
            TRY(upload_f32(m, b.data(), b.size(), &dl.bias));
        }
        m->weight_bytes += dl.qkv.bytes() + dl.o.bytes() + dl.gateup.bytes() + dl.down.bytes() +
                           2.0 * m->D * 4 + (dl.bias ? m->nqkv * 4.0 : 0.0);
    }
    // LM head (Q8 [V][D] blocks, or fp32 [D][V]) and embedding
    const bool head_f16 = d->lm_head.h != nullptr && d->lm_head.f == nullptr && d->lm_head.q == nullptr;
    TRY(upload_wmat(m, d->lm_head, m->V, m->D, m->head, m->V, 0, 1, staging, stage,
                    head_q8 ? W_Q8 : head_f16 ? W_F16 : W_F32));
    m->weight_bytes += m->head.bytes();
    if (d->embed.f != nullptr) {
        TRY(upload_f32(m, d->embed.f, (size_t)m->Ve * m->D, &m->embed_f));
    } else if (d->embed.q != nullptr && d->embed.qt == JYC_Q8_0) {
        if (d->embed.q == d->lm_head.q && head_q8 && m->Ve == m->V) {
            m->embed_q = m->head;  // tied: one device copy
        } else {
            TRY(upload_wmat(m, d->embed, m->Ve, m->D, m->embed_q, m->Ve, 0, 1, staging, stage, W_Q8));
        }
    } else if (d->embed.q != nullptr && kquant_block_bytes(d->embed.qt) != 0) {
        // K-quant embedding rows (the reference's wmat_row dequantises them): fp32 rows
        if (m->D % 256) return arg_error("K-quant embedding needs hidden % 256 == 0");
        const size_t eb = (size_t)m->Ve * (m->D / 256) * kquant_block_bytes(d->embed.qt);
        if (eb > stage) {
            set_error("internal: staging buffer too small for the embedding");
            return JYC_ERR_ARG;
        }
        TRY(m->alloc(&m->embed_f, (size_t)m->Ve * m->D));
        JYC_CUDA(cudaMemcpyAsync(staging, d->embed.q, eb, cudaMemcpyHostToDevice, m->stream));
        TRY(launch_kquant_dequant(static_cast<const uint8_t*>(staging), m->Ve, m->D, d->embed.qt, m->embed_f, 0, 1,
                                  m->stream));
        JYC_CUDA(cudaStreamSynchronize(m->stream));
    } else if (d->embed.h != nullptr) {
        // fp16 embedding rows (wmat::row_to_f32, exact): fp32 rows
        const size_t eb = (size_t)m->Ve * m->D * 2;
        if (eb > stage) {
            set_error("internal: staging buffer too small for the embedding");
            return JYC_ERR_ARG;
        }
        TRY(m->alloc(&m->embed_f, (size_t)m->Ve * m->D));
        JYC_CUDA(cudaMemcpyAsync(staging, d->embed.h, eb, cudaMemcpyHostToDevice, m->stream));
        TRY(launch_h2f(static_cast<const uint16_t*>(staging), m->embed_f, (size_t)m->Ve * m->D, m->stream));
        JYC_CUDA(cudaStreamSynchronize(m->stream));
    } else {
        set_error("embedding must be fp32, fp16, Q8_0, Q4_K, Q5_K or Q6_K");
        return JYC_ERR_UNSUPPORTED;
    }
    m->weight_bytes += (m->embed_f ? 4.0 * m->D : m->D * 34.0 / 32.0) + 4.0 * m->D;  // row + final norm
    TRY(upload_f32(m, d->final_rms_weight, m->D, &m->final_norm));
    const size_t half = (size_t)m->max_seq * (m->hd / 2);
    TRY(upload_f32(m, d->cos_table, half, &m->cos_t));
    TRY(upload_f32(m, d->sin_table, half, &m->sin_t));

    // KV cache and scratch
    const size_t kvn = (size_t)m->L * m->KV * m->max_seq;
    TRY(m->alloc(&m->k8, kvn * m->hd));
    TRY(m->alloc(&m->v8, kvn * m->hd));
    TRY(m->alloc(&m->ks, kvn));
    TRY(m->alloc(&m->vs, kvn));
    JYC_CUDA(cudaMemsetAsync(m->k8, 0, kvn * m->hd, m->stream));
    JYC_CUDA(cudaMemsetAsync(m->v8, 0, kvn * m->hd, m->stream));
    JYC_CUDA(cudaMemsetAsync(m->ks, 0, kvn * 4, m->stream));
    JYC_CUDA(cudaMemsetAsync(m->vs, 0, kvn * 4, m->stream));
    // batched prefill (tcgen05 token tiles) for Q8_0 models
    const bool pf_ok = m->wtype == W_Q8 && pf_attention_supported(m->H, m->KV, m->hd);
    int pf_chunk = kPfChunk;  // JYC_PF_ROWS overrides the tokens per pass (tuning)
    if (const char* e = std::getenv("JYC_PF_ROWS")) pf_chunk = std::max(16, std::min(16384, std::atoi(e)));
    m->pf_rows = pf_ok ? std::min(pf_chunk, m->max_seq) : 0;
    const size_t arows = std::max(kMT, m->pf_rows);
    TRY(m->alloc(&m->X, arows * m->D));
    TRY(m->alloc(&m->qkv, arows * m->nqkv));
    TRY(m->alloc(&m->attn, arows * m->q_dim));
    TRY(m->alloc(&m->h, arows * m->F));
    TRY(m->alloc(&m->logits, (size_t)m->V));
    TRY(m->alloc(&m->stag, 2 * (size_t)m->V));
    TRY(m->alloc(&m->tmp, (size_t)m->D));
    TRY(m->alloc(&m->q8, arows * m->q_dim));
    TRY(m->alloc(&m->qsc, arows * m->H));
    if (m->kq_path) {
        TRY(m->alloc(&m->kq_xn, (size_t)kMT * m->D));
        TRY(m->alloc(&m->kq_t, (size_t)kMT * m->D));
        TRY(m->alloc(&m->kq_g, (size_t)kMT * m->F));
        TRY(m->alloc(&m->kq_u, (size_t)kMT * m->F));
    }
    if (m->pf_rows) {
        const int kmax = std::max({m->D, m->q_dim, m->F});
        const int nmax = std::max({m->nqkv, m->D, 2 * m->F, m->V});
        const int N = tc_token_tile(m->pf_rows);
        TRY(m->alloc(&m->tc_xs, tc_split_halves(m->pf_rows, N, kmax)));
        TRY(m->alloc(&m->tc_xe, (size_t)tc_padded_tokens(m->pf_rows, N)));
        m->tc_part_floats = (size_t)kTcMaxSplits * std::min(m->pf_rows, kPfPartRows) * std::max({m->nqkv, m->D});
        TRY(m->alloc(&m->tc_part, m->tc_part_floats));
        const size_t tiles = (size_t)((nmax + kTcRows - 1) / kTcRows) * ((m->pf_rows + 15) / 16);
        TRY(m->alloc(&m->tc_cnt, tiles));
        TRY(m->alloc(&m->pf_part, (size_t)m->pf_rows * m->D));
        JYC_CUDA(cudaMemsetAsync(m->tc_cnt, 0, tiles * sizeof(unsigned int), m->stream));
        TRY(prepare_pf_kernels());
        TRY(prepare_tc_kernels());
        // per-row scale exponents of every matrix the tensor-core path reads
        auto rowexp = [&](DevMat& w) -> int {
            TRY(m->alloc(&w.rexp, (size_t)w.n));
            return launch_tc_rowexp(w.d, w.n, w.k, w.rexp, m->stream);
        };
        for (DevLayer& ly : m->layers) {
            TRY(rowexp(ly.qkv));
            TRY(rowexp(ly.o));
            TRY(rowexp(ly.gateup));
            TRY(rowexp(ly.down));
        }
    }
    // split-K plan of the generic attention: ~2 CTAs per SM over the kv heads
    const int target = std::max(1, 296 / m->KV);
    int chunk = (m->max_seq + target - 1) / target;
    chunk = std::max(64, (chunk + 63) / 64 * 64);
    m->chunk = chunk;
    m->nsplit = (m->max_seq + chunk - 1) / chunk;
    TRY(m->alloc(&m->part_o, (size_t)kMT * m->H * m->nsplit * m->hd));
    TRY(m->alloc(&m->part_ml, (size_t)kMT * m->H * m->nsplit * 2));
    TRY(m->alloc(&m->arrive, (size_t)m->KV));
    JYC_CUDA(cudaMemsetAsync(m->arrive, 0, m->KV * sizeof(unsigned int), m->stream));
    TRY(m->alloc(&m->st, 1));
    JYC_CUDA(cudaMemsetAsync(m->st, 0, sizeof(DevState), m->stream));
    TRY(m->alloc(&m->tokens, (size_t)m->max_seq + 1));
    JYC_CUDA(cudaStreamSynchronize(m->stream));
    // the decode kernel reads scales as non-negative (every Q8_0 quantiser
    // writes d = amax / 127); a model with a negative one decodes generically
    if (m->tiled && mega_negative_scales(true) == 0) TRY(setup_mega(m));
    JYC_CUDA(cudaStreamSynchronize(m->stream));
    return JYC_OK;
}

#define MARK(c)                             \
    do {                                    \
        if (m->prof) TRY(m->prof->mark(c)); \
    } while (0)

// One transformer stack pass over `rows` (<= kMT) tokens at pos (host constant
// or device state) with the generic kernels. Layer order = transformer_layer.
int run_layers(jyc_model* m, int rows, PosSrc pos, cudaStream_t s) {
    DevState* guard = pos.st ? m->st : nullptr;
    TRY(launch_embed(m->tokens, pos, rows, m->embed_f, m->embed_q.qs, m->embed_q.d, m->D, m->X, s));
    MARK(K_EMBED);
    for (int l = 0; l < m->L; l++) {
        const DevLayer& ly = m->layers[l];
        if (m->kq_path) {  // RMSNorm -> Q, K, V from the K-quant blocks in place (+ bias)
            TRY(launch_rmsnorm(m->X, m->kq_xn, ly.rms1, rows, m->D, 1e-5f, s));
            TRY(launch_kquant_matmul_ld(m->kq_xn, m->D, rows, m->q_dim, m->D, ly.kq[0].kqb, ly.kq[0].kqt,
                                        m->qkv, m->nqkv, s));
            TRY(launch_kquant_matmul_ld(m->kq_xn, m->D, rows, m->kv_dim, m->D, ly.kq[1].kqb, ly.kq[1].kqt,
                                        m->qkv + m->q_dim, m->nqkv, s));
            TRY(launch_kquant_matmul_ld(m->kq_xn, m->D, rows, m->kv_dim, m->D, ly.kq[2].kqb, ly.kq[2].kqt,
                                        m->qkv + m->q_dim + m->kv_dim, m->nqkv, s));
            if (ly.bias) TRY(launch_bias_rows(m->qkv, m->nqkv, ly.bias, m->nqkv, rows, s));
            MARK(K_QKV);
        } else {  // RMSNorm -> fused Q|K|V GEMV (+ bias)
            GemvArgs g{};
            g.m = rows; g.eps = 1e-5f; g.st = guard;
            g.x = m->X; g.ldx = m->D; g.n = m->nqkv; g.k = m->D;
            g.qs = ly.qkv.qs; g.d = ly.qkv.d; g.wt = ly.qkv.f; g.wh = ly.qkv.h; g.norm_w = ly.rms1;
            g.y = m->qkv; g.ldy = m->nqkv; g.bias = ly.bias;
            TRY(launch_gemv(g, m->wtype, ly.bias ? EPI_BIAS : EPI_STORE, s));
            MARK(K_QKV);
        }
        // RoPE(Q,K) + int8 quantisation of Q, K, V; K/V appended to the cache
        RopeQuantArgs rq{};
        rq.q = m->qkv; rq.k = m->qkv + m->q_dim; rq.v = m->qkv + m->q_dim + m->kv_dim;
        rq.ldq = m->nqkv; rq.rows = rows; rq.H = m->H; rq.KV = m->KV; rq.hd = m->hd;
        rq.cos_t = m->cos_t; rq.sin_t = m->sin_t; rq.q8 = m->q8; rq.qsc = m->qsc;
        rq.kv = m->kv_layer(l); rq.pos = pos;
        TRY(launch_rope_quant(rq, s));
        MARK(K_ROPEQ);
        // int8-KV attention (split-K flash decoding)
        AttnArgs at{};
        at.q8 = m->q8; at.qsc = m->qsc; at.kv = m->kv_layer(l);
        at.rows = rows; at.H = m->H; at.KV = m->KV; at.hd = m->hd;
        at.chunk = m->chunk; at.nsplit = m->nsplit;
        at.scale = 1.0f / sqrtf((float)m->hd);
        at.part_o = m->part_o; at.part_ml = m->part_ml; at.arrive = m->arrive;
        at.out = m->attn; at.ldo = m->q_dim; at.pos = pos;
        TRY(launch_attention(at, s));
        MARK(K_ATTN);
        if (m->kq_path) {
            // O (+ residual), RMSNorm -> gate, up -> SwiGLU, down (+ residual)
            TRY(launch_kquant_matmul_ld(m->attn, m->q_dim, rows, m->D, m->q_dim, ly.kq[3].kqb, ly.kq[3].kqt,
                                        m->kq_t, m->D, s));
            TRY(launch_add_rows(m->X, m->kq_t, (size_t)rows * m->D, s));
            MARK(K_OPROJ);
            TRY(launch_rmsnorm(m->X, m->kq_xn, ly.rms2, rows, m->D, 1e-5f, s));
            TRY(launch_kquant_matmul_ld(m->kq_xn, m->D, rows, m->F, m->D, ly.kq[4].kqb, ly.kq[4].kqt, m->kq_g,
                                        m->F, s));
            TRY(launch_kquant_matmul_ld(m->kq_xn, m->D, rows, m->F, m->D, ly.kq[5].kqb, ly.kq[5].kqt, m->kq_u,
                                        m->F, s));
            TRY(launch_swiglu_rows(m->kq_g, m->kq_u, m->h, (size_t)rows * m->F, s));
            MARK(K_GATEUP);
            TRY(launch_kquant_matmul_ld(m->h, m->F, rows, m->D, m->F, ly.kq[6].kqb, ly.kq[6].kqt, m->kq_t, m->D,
                                        s));
            TRY(launch_add_rows(m->X, m->kq_t, (size_t)rows * m->D, s));
            MARK(K_DOWN);
            continue;
        }
        // O projection + residual
        GemvArgs g{};
        g.m = rows; g.eps = 1e-5f; g.st = guard;
        g.x = m->attn; g.ldx = m->q_dim; g.n = m->D; g.k = m->q_dim;
        g.qs = ly.o.qs; g.d = ly.o.d; g.wt = ly.o.f; g.wh = ly.o.h; g.y = m->X; g.ldy = m->D;
        TRY(launch_gemv(g, m->wtype, EPI_RESID, s));
        MARK(K_OPROJ);
        // RMSNorm -> gate|up GEMV -> SwiGLU
        g = GemvArgs{};
        g.m = rows; g.eps = 1e-5f; g.st = guard;
        g.x = m->X; g.ldx = m->D; g.n = 2 * m->F; g.k = m->D;
        g.qs = ly.gateup.qs; g.d = ly.gateup.d; g.wt = ly.gateup.f; g.wh = ly.gateup.h;
        g.norm_w = ly.rms2; g.y = m->h; g.ldy = m->F;
        TRY(launch_gemv(g, m->wtype, EPI_SWIGLU, s));
        MARK(K_GATEUP);
        // down projection + residual
        g = GemvArgs{};
        g.m = rows; g.eps = 1e-5f; g.st = guard;
        g.x = m->h; g.ldx = m->F; g.n = m->D; g.k = m->F;
        g.qs = ly.down.qs; g.d = ly.down.d; g.wt = ly.down.f; g.wh = ly.down.h; g.y = m->X; g.ldy = m->D;
        TRY(launch_gemv(g, m->wtype, EPI_RESID, s));
        MARK(K_DOWN);
    }
    return JYC_OK;
}

// Final RMSNorm of row `row` + LM head GEMV + argmax; the last CTA appends the
// token to the device buffer and advances the state.
int run_head(jyc_model* m, int row, cudaStream_t s) {
    GemvArgs g{};
    g.m = 1; g.eps = 1e-5f; g.st = m->st; g.tokens = m->tokens;
    g.x = m->X + (size_t)row * m->D; g.ldx = m->D; g.n = m->V; g.k = m->D;
    g.qs = m->head.qs; g.d = m->head.d; g.wt = m->head.f; g.wh = m->head.h; g.norm_w = m->final_norm;
    g.y = m->logits; g.ldy = m->V;
    TRY(launch_gemv(g, m->head.wtype(), EPI_ARGMAX, s));
    MARK(K_HEAD);
    return JYC_OK;
}

// Y = X . W^T over `rows` tokens on the tensor cores (split-K when the tiles
// alone do not fill the GPU): RMSNorm (norm != null) + fp16 hi/lo split of X,
// then the tcgen05 GEMM with the epilogue `epi`.
int run_tc_gemm(jyc_model* m, const DevMat& w, const float* x, int ldx, int rows, const float* norm, float* y,
                int ldy, const float* bias, int epi, int* err, cudaStream_t s) {
    const int cap = (int)std::min<size_t>(kTcMaxSplits, m->tc_part_floats / ((size_t)rows * w.n));
    int N = 0, splits = 1;
    tc_plan(w.n, w.k, rows, std::max(1, cap), &N, &splits);
    TRY(launch_tc_split(x, ldx, rows, w.k, norm, 1e-5f, N, m->tc_xs, m->tc_xe, s));
    TcGemm g{};
    g.qs = w.qs; g.d = w.d; g.rexp = w.rexp; g.n = w.n; g.k = w.k;
    g.xs = m->tc_xs; g.xe = m->tc_xe; g.T = rows; g.N = N;
    g.y = y; g.ldy = ldy; g.bias = bias; g.err = err;
    g.splits = splits;
    g.part = m->tc_part; g.cnt = m->tc_cnt;
    return launch_tc_gemm(g, epi, s);
}

// Forward of n tokens already in m->tokens[start..start+n) in chunks of kMT,
// then the head on the last row (state must hold len == start+n).
// Batched prefill of tokens [start, start + n) in passes of pf_rows tokens:
// per layer RMSNorm+digits -> QKV (tensor-core token tiles) -> RoPE/quant +
// cache append -> causal attention -> O + residual -> RMSNorm+digits ->
// gate/up + SwiGLU -> down + residual; then the LM head on the last token.
int run_prefill_batched(jyc_model* m, int start, int n, cudaStream_t s) {
    int last_rows = 0;
    int* err = device_error_word();
    for (int c = 0; c < n; c += m->pf_rows) {
        const int rows = std::min(m->pf_rows, n - c);
        TRY(launch_embed(m->tokens, PosSrc{nullptr, start + c}, rows, m->embed_f, m->embed_q.qs, m->embed_q.d,
                         m->D, m->X, s));
        auto gemm = [&](const DevMat& w, const float* x, int ldx, const float* norm, float* y, int ldy,
                        const float* bias, int epi) -> int {
            return run_tc_gemm(m, w, x, ldx, rows, norm, y, ldy, bias, epi, err, s);
        };
        for (int l = 0; l < m->L; l++) {
            const DevLayer& ly = m->layers[l];
            TRY(gemm(ly.qkv, m->X, m->D, ly.rms1, m->qkv, m->nqkv, ly.bias, ly.bias ? TC_BIAS : TC_STORE));
            RopeQuantArgs rq{};
            rq.q = m->qkv; rq.k = m->qkv + m->q_dim; rq.v = m->qkv + m->q_dim + m->kv_dim;
            rq.ldq = m->nqkv; rq.rows = rows; rq.H = m->H; rq.KV = m->KV; rq.hd = m->hd;
            rq.cos_t = m->cos_t; rq.sin_t = m->sin_t; rq.q8 = m->q8; rq.qsc = m->qsc;
            rq.kv = m->kv_layer(l); rq.pos = PosSrc{nullptr, start + c};
            TRY(launch_rope_quant(rq, s));
            const KVView kv = m->kv_layer(l);
            PfAttn at{};
            at.q8 = m->q8; at.qsc = m->qsc; at.k8 = kv.k; at.v8 = kv.v; at.ks = kv.ks; at.vs = kv.vs;
            at.max_seq = m->max_seq; at.H = m->H; at.KV = m->KV; at.hd = m->hd; at.T = rows;
            at.pos0 = start + c; at.scale = 1.0f / sqrtf((float)m->hd); at.out = m->attn;
            TRY(launch_pf_attention(at, s));
            TRY(gemm(ly.o, m->attn, m->q_dim, nullptr, m->X, m->D, nullptr, TC_RESID));
            TRY(gemm(ly.gateup, m->X, m->D, ly.rms2, m->h, m->F, nullptr, TC_SWIGLU));
            TRY(gemm(ly.down, m->h, m->F, nullptr, m->X, m->D, nullptr, TC_RESID));
        }
        last_rows = rows;
    }
    return run_head(m, last_rows - 1, s);
}

// Half-layer phases [first, last) of the batched prefill for token rows
// [start, start + rows) of a tensor-parallel shard: phase 2l = RMSNorm + QKV +
// RoPE/cache append + attention + O, phase 2l+1 = RMSNorm + gate/up + SwiGLU +
// down. O and down leave this shard's partial rows in pf_part (no residual
// add); the caller sums them over the ranks between windows and the next
// phase adds the sum into X. Phase 0 starts from the embedding.
int run_prefill_window(jyc_model* m, int start, int rows, int first, int last, cudaStream_t s) {
    int* err = device_error_word();
    for (int p = first; p < last; p++) {
        const int l = p >> 1;
        const DevLayer& ly = m->layers[l];
        if (p == 0)
            TRY(launch_embed(m->tokens, PosSrc{nullptr, start}, rows, m->embed_f, m->embed_q.qs, m->embed_q.d, m->D,
                             m->X, s));
        else
            TRY(launch_add_rows(m->X, m->pf_part, (size_t)rows * m->D, s));
        auto gemm = [&](const DevMat& w, const float* x, int ldx, const float* norm, float* y, int ldy,
                        const float* bias, int epi) -> int {
            return run_tc_gemm(m, w, x, ldx, rows, norm, y, ldy, bias, epi, err, s);
        };
        if ((p & 1) == 0) {
            TRY(gemm(ly.qkv, m->X, m->D, ly.rms1, m->qkv, m->nqkv, ly.bias, ly.bias ? TC_BIAS : TC_STORE));
            RopeQuantArgs rq{};
            rq.q = m->qkv; rq.k = m->qkv + m->q_dim; rq.v = m->qkv + m->q_dim + m->kv_dim;
            rq.ldq = m->nqkv; rq.rows = rows; rq.H = m->H; rq.KV = m->KV; rq.hd = m->hd;
            rq.cos_t = m->cos_t; rq.sin_t = m->sin_t; rq.q8 = m->q8; rq.qsc = m->qsc;
            rq.kv = m->kv_layer(l); rq.pos = PosSrc{nullptr, start};
            TRY(launch_rope_quant(rq, s));
            const KVView kv = m->kv_layer(l);
            PfAttn at{};
            at.q8 = m->q8; at.qsc = m->qsc; at.k8 = kv.k; at.v8 = kv.v; at.ks = kv.ks; at.vs = kv.vs;
            at.max_seq = m->max_seq; at.H = m->H; at.KV = m->KV; at.hd = m->hd; at.T = rows;
            at.pos0 = start; at.scale = 1.0f / sqrtf((float)m->hd); at.out = m->attn;
            TRY(launch_pf_attention(at, s));
            TRY(gemm(ly.o, m->attn, m->q_dim, nullptr, m->pf_part, m->D, nullptr, TC_STORE));
        } else {
            TRY(gemm(ly.gateup, m->X, m->D, ly.rms2, m->h, m->F, nullptr, TC_SWIGLU));
            TRY(gemm(ly.down, m->h, m->F, nullptr, m->pf_part, m->D, nullptr, TC_STORE));
        }
    }
    return JYC_OK;
}

int run_prefill(jyc_model* m, int start, int n, cudaStream_t s) {
    if (m->pf_rows) return run_prefill_batched(m, start, n, s);
    int last_rows = 0;
    for (int c = 0; c < n; c += kMT) {
        const int rows = std::min(kMT, n - c);
        TRY(run_layers(m, rows, PosSrc{nullptr, start + c}, s));
        last_rows = rows;
    }
    return run_head(m, last_rows - 1, s);
}

int ensure_step_graph(jyc_model* m) {
    if (m->mega || m->step_exec) return JYC_OK;
    cudaGraph_t graph = nullptr;
    const long long counted = jyc_kernel_launches();
    JYC_CUDA(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
    int r = run_layers(m, 1, PosSrc{m->st, 0}, m->stream);
    if (r == JYC_OK) r = run_head(m, 0, m->stream);
    cudaError_t e = cudaStreamEndCapture(m->stream, &graph);
    count_launch((int)(counted - jyc_kernel_launches()));  // captured, not launched
    if (r != JYC_OK) {
        if (graph) cudaGraphDestroy(graph);
        return r;
    }
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamEndCapture");
    e = cudaGraphInstantiate(&m->step_exec, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGraphInstantiate");
    return JYC_OK;
}

int kernels_per_step(const jyc_model* m) { return m->mega ? 1 : 1 + m->L * 6 + 1; }

// One decode step on stream s (token at len-1, guarded by the state).
int decode_step(jyc_model* m, cudaStream_t s) {
    if (m->mega) return launch_mega_step(m->margs, s);
    TRY(ensure_step_graph(m));
    JYC_CUDA(cudaGraphLaunch(m->step_exec, s));
    count_launch(kernels_per_step(m));
    return JYC_OK;
}

}  // namespace

extern "C" {

JYC_API jyc_model* jyc_model_create(const jyc_model_desc* desc) {
    clear_error();
    jyc_model* m = new (std::nothrow) jyc_model();
    if (!m) {
        set_error("out of host memory");
        return nullptr;
    }
    if (build_model(m, desc) != JYC_OK) {
        delete m;
        return nullptr;
    }
    return m;
}

JYC_API void jyc_model_free(jyc_model* m) { delete m; }

JYC_API double jyc_model_weight_bytes_per_token(const jyc_model* m) { return m ? m->weight_bytes : 0.0; }

JYC_API double jyc_model_kv_bytes_per_token(const jyc_model* m, int ctx) {
    if (!m) return 0.0;
    // int8 K and V rows + one fp32 scale each, per layer, kv head and position
    return (double)m->L * m->KV * ctx * (2.0 * m->hd + 8.0);
}

// (Re)starts the device step state; a decode-kernel model also clears its
// attention arrival counters (a step that gave up part-way leaves them dirty).
static int set_state(jyc_model* m, int len, int max_new, int max_len, const int* eos, int n_eos, cudaStream_t s) {
    if (m->mega && m->margs.acnt)
        JYC_CUDA(cudaMemsetAsync(m->margs.acnt, 0, sizeof(unsigned int) * 2 * m->L * m->KV, s));
    return launch_set_state(m->st, len, max_new, max_len, eos, n_eos, s);
}

JYC_API int jyc_forward_logits(jyc_model* m, const int* ids, int seq, int start_pos, float* logits,
                               float* hidden_out) {
    clear_error();
    if (!m || !ids || seq <= 0 || start_pos < 0) return arg_error("forward_logits: bad arguments");
    if ((long long)start_pos + seq > m->max_seq) {
        set_error("forward: KV cache capacity exceeded");
        return JYC_ERR_KV_OOM;
    }
    for (int i = 0; i < seq; i++)
        if (ids[i] < 0 || ids[i] >= m->Ve) return arg_error("forward_logits: token id out of range");
    cudaStream_t s = m->stream;
    JYC_CUDA(cudaMemcpyAsync(m->tokens + start_pos, ids, seq * sizeof(int), cudaMemcpyHostToDevice, s));
    TRY(set_state(m, start_pos + seq, 1 << 30, m->max_seq + 1, nullptr, 0, s));
    if (seq == 1 && m->mega) {
        // a single token goes through the decode kernel (the path generate's steps use)
        TRY(launch_mega_step(m->margs, s));
    } else {
        TRY(run_prefill(m, start_pos, seq, s));
    }
    if (hidden_out) {
        const int last = (seq == 1 && m->mega) ? 0 : (seq - 1) % (m->pf_rows ? m->pf_rows : kMT);
        TRY(launch_rmsnorm(m->X + (size_t)last * m->D, m->tmp, m->final_norm, 1, m->D, 1e-5f, s));
        JYC_CUDA(cudaMemcpyAsync(hidden_out, m->tmp, m->D * sizeof(float), cudaMemcpyDeviceToHost, s));
    }
    if (logits)
        JYC_CUDA(cudaMemcpyAsync(logits, m->logits, (size_t)m->V * sizeof(float), cudaMemcpyDeviceToHost, s));
    JYC_CUDA(cudaStreamSynchronize(s));
    return JYC_OK;
}

JYC_API int jyc_model_read_kv(jyc_model* m, int layer, int npos, int8_t* k, float* ks, int8_t* v, float* vs) {
    clear_error();
    if (!m || layer < 0 || layer >= m->L || npos < 0 || npos > m->max_seq) return arg_error("read_kv: bad arguments");
    JYC_CUDA(cudaStreamSynchronize(m->stream));
    const KVView kv = m->kv_layer(layer);
    std::vector<int8_t> kb((size_t)m->KV * m->max_seq * m->hd), vb(kb.size());
    std::vector<float> ksb((size_t)m->KV * m->max_seq), vsb(ksb.size());
    JYC_CUDA(cudaMemcpy(kb.data(), kv.k, kb.size(), cudaMemcpyDeviceToHost));
    JYC_CUDA(cudaMemcpy(vb.data(), kv.v, vb.size(), cudaMemcpyDeviceToHost));
    JYC_CUDA(cudaMemcpy(ksb.data(), kv.ks, ksb.size() * 4, cudaMemcpyDeviceToHost));
    JYC_CUDA(cudaMemcpy(vsb.data(), kv.vs, vsb.size() * 4, cudaMemcpyDeviceToHost));
    for (int p = 0; p < npos; p++)
        for (int h = 0; h < m->KV; h++) {
            const size_t src = ((size_t)h * m->max_seq + p);
            const size_t dst = (size_t)p * m->KV + h;
            std::memcpy(k + dst * m->hd, kb.data() + src * m->hd, m->hd);
            std::memcpy(v + dst * m->hd, vb.data() + src * m->hd, m->hd);
            ks[dst] = ksb[src];
            vs[dst] = vsb[src];
        }
    return JYC_OK;
}

JYC_API int jyc_model_write_kv(jyc_model* m, int layer, int npos, const int8_t* k, const float* ks, const int8_t* v,
                               const float* vs) {
    clear_error();
    if (!m || layer < 0 || layer >= m->L || npos < 0 || npos > m->max_seq || !k || !ks || !v || !vs)
        return arg_error("write_kv: bad arguments");
    if (npos == 0) return JYC_OK;
    JYC_CUDA(cudaStreamSynchronize(m->stream));
    const KVView kv = m->kv_layer(layer);
    // reference order [pos][kv head] -> the device's [kv head][pos], one copy per head
    std::vector<int8_t> kb((size_t)npos * m->hd), vb(kb.size());
    std::vector<float> ksb((size_t)npos), vsb(ksb.size());
    for (int h = 0; h < m->KV; h++) {
        for (int p = 0; p < npos; p++) {
            const size_t src = (size_t)p * m->KV + h;
            std::memcpy(kb.data() + (size_t)p * m->hd, k + src * m->hd, m->hd);
            std::memcpy(vb.data() + (size_t)p * m->hd, v + src * m->hd, m->hd);
            ksb[p] = ks[src];
            vsb[p] = vs[src];
        }
        const size_t row0 = (size_t)h * m->max_seq;
        JYC_CUDA(cudaMemcpy(kv.k + row0 * m->hd, kb.data(), kb.size(), cudaMemcpyHostToDevice));
        JYC_CUDA(cudaMemcpy(kv.v + row0 * m->hd, vb.data(), vb.size(), cudaMemcpyHostToDevice));
        JYC_CUDA(cudaMemcpy(kv.ks + row0, ksb.data(), ksb.size() * 4, cudaMemcpyHostToDevice));
        JYC_CUDA(cudaMemcpy(kv.vs + row0, vsb.data(), vsb.size() * 4, cudaMemcpyHostToDevice));
    }
    return JYC_OK;
}

JYC_API int jyc_generate(jyc_model* m, const int* prompt_ids, int prompt_len, const int* eos_ids, int num_eos,
                         int max_new_tokens, float temperature, int* out_ids, float repetition_penalty,
                         jyc_token_cb cb, void* cb_ud) {
    clear_error();
    if (!m || !out_ids) return arg_error("generate: null model or output");
    if (prompt_len <= 0 || prompt_len > m->max_seq || !prompt_ids) return 0;
    for (int i = 0; i < prompt_len; i++) out_ids[i] = prompt_ids[i];
    if (max_new_tokens <= 0) return prompt_len;
    const bool sampling = temperature > 0.0f || repetition_penalty != 1.0f;
    if (sampling && m->margs.tp > 1) {
        set_error("generate: sampling over a vocabulary-sliced (tensor-parallel) head is not built");
        return JYC_ERR_UNSUPPORTED;
    }
    if (num_eos < 0 || num_eos > 8 || (num_eos > 0 && !eos_ids)) return arg_error("generate: at most 8 EOS ids");
    for (int i = 0; i < prompt_len; i++)
        if (prompt_ids[i] < 0 || prompt_ids[i] >= m->Ve) return arg_error("generate: prompt id out of range");
    if (prompt_len >= m->max_seq) return prompt_len;  // the loop condition len < max_seq fails at once
    cudaStream_t s = m->stream;
    TRY(ensure_step_graph(m));
    JYC_CUDA(cudaMemcpyAsync(m->tokens, prompt_ids, prompt_len * sizeof(int), cudaMemcpyHostToDevice, s));
    TRY(set_state(m, prompt_len, max_new_tokens, m->max_seq, eos_ids, num_eos, s));
    // the reference's sampler state: LCG seed 12345 per call (generate.h:36)
    if (sampling) {
        TRY(launch_set_sampling(m->st, temperature, repetition_penalty, 12345u, prompt_len, s));
        JYC_CUDA(cudaMemsetAsync(m->stag, 0xFF, (size_t)m->V * sizeof(unsigned int), s));
        JYC_CUDA(cudaMemsetAsync(m->stag + m->V, 0, (size_t)m->V * sizeof(unsigned int), s));
    }
    TRY(run_prefill(m, 0, prompt_len, s));
    if (sampling) TRY(launch_resample_last(m->st, m->logits, m->stag, m->V, m->tokens, s));
    // decode: one step per token; the state guard turns surplus steps into no-ops
    // (the decode kernel samples in its head phase; the per-op step re-picks)
    auto step = [&]() -> int {
        TRY(decode_step(m, s));
        if (sampling && !m->mega) TRY(launch_resample_last(m->st, m->logits, m->stag, m->V, m->tokens, s));
        return JYC_OK;
    };
    const int max_steps = std::min(max_new_tokens, m->max_seq - prompt_len) - 1;
    int len = prompt_len;
    if (!cb) {
        for (int i = 0; i < max_steps; i++) TRY(step());
        DevState hs;
        JYC_CUDA(cudaMemcpyAsync(&hs, m->st, sizeof(DevState), cudaMemcpyDeviceToHost, s));
        JYC_CUDA(cudaStreamSynchronize(s));
        len = hs.len;
        JYC_CUDA(cudaMemcpy(out_ids + prompt_len, m->tokens + prompt_len, (size_t)(len - prompt_len) * sizeof(int),
                            cudaMemcpyDeviceToHost));
        return len;
    }
    // with a callback: run blocks of steps, hand each new token to cb in order,
    // stop (and drop any tokens computed past it) when cb asks to.
    int done_steps = 0;
    int block = 1;
    while (true) {
        DevState hs;
        JYC_CUDA(cudaMemcpyAsync(&hs, m->st, sizeof(DevState), cudaMemcpyDeviceToHost, s));
        JYC_CUDA(cudaStreamSynchronize(s));
        JYC_CUDA(cudaMemcpy(out_ids + len, m->tokens + len, (size_t)(hs.len - len) * sizeof(int),
                            cudaMemcpyDeviceToHost));
        for (int i = len; i < hs.len; i++) {
            if (cb(out_ids[i], cb_ud)) return i + 1;
            bool stop = false;
            for (int e = 0; e < num_eos; e++)
                if (out_ids[i] == eos_ids[e]) stop = true;
            if (stop) return i + 1;
        }
        len = hs.len;
        if (!hs.active || done_steps >= max_steps) return len;
        const int n = std::min(block, max_steps - done_steps);
        for (int i = 0; i < n; i++) TRY(step());
        done_steps += n;
        block = std::min(block * 2, 32);
    }
}

JYC_API int jyc_prefill_device(jyc_model* m, const int* prompt_ids_dev, int prompt_len, void* stream) {
    clear_error();
    if (!m || !prompt_ids_dev || prompt_len <= 0 || prompt_len >= m->max_seq)
        return arg_error("prefill_device: bad arguments");
    cudaStream_t s = (cudaStream_t)stream;  // as given: 0 is the legacy default stream
    JYC_CUDA(cudaMemcpyAsync(m->tokens, prompt_ids_dev, prompt_len * sizeof(int), cudaMemcpyDeviceToDevice, s));
    TRY(set_state(m, prompt_len, 1 << 30, m->max_seq, nullptr, 0, s));
    return run_prefill(m, 0, prompt_len, s);
}

JYC_API int jyc_model_prefill_window(jyc_model* m, int start, int rows, int first, int last, void* stream) {
    clear_error();
    if (!m) return arg_error("prefill_window: null model");
    if (!m->pf_rows) {
        set_error("prefill_window: the model has no batched prefill (Q8_0 weights, supported head shape)");
        return JYC_ERR_UNSUPPORTED;
    }
    if (rows <= 0 || rows > m->pf_rows || start < 0 || start + rows > m->max_seq)
        return arg_error("prefill_window: rows must be in [1, " + std::to_string(m->pf_rows) + "] within max_seq");
    if (first < 0 || last <= first || last > 2 * m->L) return arg_error("prefill_window: bad phase range");
    return run_prefill_window(m, start, rows, first, last, static_cast<cudaStream_t>(stream));
}

JYC_API int jyc_model_prefill_partial(jyc_model* m, float** part, int* max_rows) {
    clear_error();
    if (!m || !part || !max_rows) return arg_error("prefill_partial: null argument");
    if (!m->pf_rows) {
        set_error("prefill_partial: the model has no batched prefill");
        return JYC_ERR_UNSUPPORTED;
    }
    *part = m->pf_part;
    *max_rows = m->pf_rows;
    return JYC_OK;
}

JYC_API int jyc_model_rewind(jyc_model* m, int len, void* stream) {
    clear_error();
    if (!m || len <= 0 || len >= m->max_seq) return arg_error("rewind: bad length");
    cudaStream_t s = (cudaStream_t)stream;  // as given: 0 is the legacy default stream
    return set_state(m, len, 1 << 30, m->max_seq, nullptr, 0, s);
}

JYC_API int jyc_decode_device(jyc_model* m, int n_steps, void* stream) {
    clear_error();
    if (!m || n_steps < 0) return arg_error("decode_device: bad arguments");
    cudaStream_t s = (cudaStream_t)stream;  // as given: 0 is the legacy default stream
    for (int i = 0; i < n_steps; i++) TRY(decode_step(m, s));
    return JYC_OK;
}

JYC_API int jyc_model_kernels_per_step(const jyc_model* m) { return m ? kernels_per_step(m) : 0; }

JYC_API int jyc_model_decode_path(const jyc_model* m) { return m ? (m->mega ? 2 : 0) : -1; }

JYC_API int jyc_model_decode_window(jyc_model* m, int first, int last, void* stream) {
    clear_error();
    if (!m) return arg_error("decode_window: null model");
    if (!m->mega) {
        set_error("decode_window: the model does not use the decode kernel");
        return JYC_ERR_UNSUPPORTED;
    }
    if (first < 0 || last <= first || last > 2 * m->L + 1) return arg_error("decode_window: bad phase range");
    MegaArgs a = m->margs;
    a.win0 = first;
    a.win1 = last;
    return launch_mega_step(a, static_cast<cudaStream_t>(stream));
}

JYC_API int jyc_model_tp_open(jyc_model* m, int size, int rank, void* handle_out) {
    clear_error();
    if (!m || !handle_out || size < 2 || size > kMegaMaxTP || rank < 0 || rank >= size)
        return arg_error("tp_open: bad arguments (2 <= size <= 8, 0 <= rank < size)");
    if (!m->mega) {
        set_error("tp_open: the model does not use the decode kernel");
        return JYC_ERR_UNSUPPORTED;
    }
    if (m->tp_region) return arg_error("tp_open: already open");
    std::vector<MegaLayer> ml(m->L);
    JYC_CUDA(cudaMemcpy(ml.data(), m->d_mlayers, sizeof(MegaLayer) * m->L, cudaMemcpyDeviceToHost));
    for (const MegaLayer& x : ml) {
        m->tp_so = std::max(m->tp_so, x.o.spl);
        m->tp_sd = std::max(m->tp_sd, x.dn.spl);
    }
    for (const MegaLayer& x : ml)  // readers take the senders' groups as one contiguous list
        if (x.o.spl != m->tp_so || x.dn.spl != m->tp_sd) {
            set_error("tp_open: layers with different split plans are not supported");
            return JYC_ERR_UNSUPPORTED;
        }
    const size_t floats = (size_t)size * (m->tp_so + m->tp_sd) * m->D;
    const size_t bytes = floats * 4 + (size_t)4 * size * sizeof(unsigned int) + (size_t)size * 8;
    TRY(m->alloc(&m->tp_region, bytes));
    JYC_CUDA(cudaMemset(m->tp_region, 0, bytes));
    JYC_CUDA(cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle_out), m->tp_region));
    m->tp_size = size;
    m->tp_rank = rank;
    return JYC_OK;
}

JYC_API int jyc_model_tp_connect(jyc_model* m, const void* handles) {
    clear_error();
    if (!m || !handles || !m->tp_region) return arg_error("tp_connect: call tp_open first");
    MegaArgs& a = m->margs;
    const int t = m->tp_size;
    const size_t xo_f = (size_t)t * m->tp_so * m->D, xd_f = (size_t)t * m->tp_sd * m->D;
    for (int q = 0; q < t; q++) {
        unsigned char* base = m->tp_region;
        if (q != m->tp_rank) {
            cudaIpcMemHandle_t h;
            std::memcpy(&h, static_cast<const unsigned char*>(handles) + (size_t)q * sizeof(h), sizeof(h));
            void* p = nullptr;
            JYC_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
            m->tp_mapped.push_back(p);
            base = static_cast<unsigned char*>(p);
        }
        // layout: xo [t][so][D] | xdn [t][sd][D] | flags [3][t] (+1 pad) | xam [t] (8-byte aligned)
        float* f = reinterpret_cast<float*>(base);
        a.peer_xo[q] = f;
        a.peer_xdn[q] = f + xo_f;
        a.peer_xflag[q] = reinterpret_cast<unsigned int*>(f + xo_f + xd_f);
        a.peer_xam[q] = reinterpret_cast<unsigned long long*>(a.peer_xflag[q] + 4 * t);
    }
    float* own = reinterpret_cast<float*>(m->tp_region);
    a.xo = own;
    a.xdn = own + xo_f;
    a.xflag = reinterpret_cast<unsigned int*>(own + xo_f + xd_f);
    a.xam = reinterpret_cast<unsigned long long*>(a.xflag + 4 * t);
    a.xo_stride = m->tp_so * m->D;
    a.xdn_stride = m->tp_sd * m->D;
    a.tp = t;
    a.tp_rank = m->tp_rank;
    return JYC_OK;
}

JYC_API int jyc_model_partials(jyc_model* m, float** o_part, int* o_count, float** d_part, int* d_count) {
    clear_error();
    if (!m || !o_part || !o_count || !d_part || !d_count) return arg_error("model_partials: bad arguments");
    if (!m->mega) {
        set_error("model_partials: the model does not use the decode kernel");
        return JYC_ERR_UNSUPPORTED;
    }
    int so = 1, sd = 1;
    std::vector<MegaLayer> ml(m->L);
    JYC_CUDA(cudaMemcpy(ml.data(), m->d_mlayers, sizeof(MegaLayer) * m->L, cudaMemcpyDeviceToHost));
    for (const MegaLayer& x : ml) {
        so = std::max(so, x.o.spl);
        sd = std::max(sd, x.dn.spl);
    }
    *o_part = m->margs.po;
    *o_count = so * m->D;
    *d_part = m->margs.pd;
    *d_count = sd * m->D;
    return JYC_OK;
}

JYC_API int jyc_model_trace_points(const jyc_model* m) {
    if (!m || !m->mega) return 0;
    return 1 + m->L * kMegaTraceLayer + 4;
}

// One traced decode step (megakernel models): out receives, per CTA, the SM
// clock at each phase boundary ([ctas][trace_points] int64); returns the CTA count.
JYC_API int jyc_model_trace_decode(jyc_model* m, void* stream, long long* out, int cap) {
    clear_error();
    if (!m || !m->mega || !out) return arg_error("trace_decode: megakernel model and buffer required");
    const int nct = mega_num_ctas(), npts = jyc_model_trace_points(m);
    if (cap < nct * npts) return arg_error("trace_decode: buffer too small");
    cudaStream_t s = (cudaStream_t)stream;
    long long* d = nullptr;
    JYC_CUDA(cudaMalloc(&d, sizeof(long long) * nct * kMegaTracePts));
    JYC_CUDA(cudaMemsetAsync(d, 0, sizeof(long long) * nct * kMegaTracePts, s));
    MegaArgs a = m->margs;
    a.trace = d;
    int r = launch_mega_step(a, s);
    std::vector<long long> h((size_t)nct * kMegaTracePts);
    if (r == JYC_OK) {
        cudaError_t e = cudaMemcpyAsync(h.data(), d, h.size() * sizeof(long long), cudaMemcpyDeviceToHost, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) r = cuda_fail(e, "trace readback");
    }
    cudaFree(d);
    if (r != JYC_OK) return r;
    for (int b = 0; b < nct; b++)
        for (int i = 0; i < npts; i++) out[(size_t)b * npts + i] = h[(size_t)b * kMegaTracePts + i];
    return nct;
}

JYC_API int jyc_device_error(int reset) {
    int* p = device_error_word();
    if (!p) return 0;
    int v = 0;
    if (cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    if (reset && v) {
        const int z = 0;
        cudaMemcpy(p, &z, sizeof(int), cudaMemcpyHostToDevice);
    }
    return v;
}

// Per-kernel timing of decode. Megakernel models: one class (the whole step)
// timed with events around each launch. Generic models: the step graph is
// replayed with an event after every kernel. Returns per class the summed
// device milliseconds, the launch count and the algorithmic bytes of one
// launch at the context the first profiled step runs at.
JYC_API int jyc_model_profile_decode(jyc_model* m, int n_steps, void* stream, double* ms, int* launches,
                                     double* bytes) {
    clear_error();
    if (!m || n_steps <= 0 || !ms || !launches || !bytes) return arg_error("profile_decode: bad arguments");
    cudaStream_t s = (cudaStream_t)stream;
    for (int c = 0; c < K_NCLASS; c++) {
        ms[c] = 0.0;
        launches[c] = 0;
        bytes[c] = 0.0;
    }
    DevState hs;
    JYC_CUDA(cudaStreamSynchronize(s));
    JYC_CUDA(cudaMemcpy(&hs, m->st, sizeof(DevState), cudaMemcpyDeviceToHost));
    const int ctx = hs.len;  // positions the first profiled step attends to
    if (m->mega) {
        bytes[0] = m->weight_bytes + (double)m->L * m->KV * ctx * (2.0 * m->hd + 8.0);
        cudaEvent_t e0, e1;
        JYC_CUDA(cudaEventCreate(&e0));
        JYC_CUDA(cudaEventCreate(&e1));
        for (int it = 0; it < n_steps; it++) {
            JYC_CUDA(cudaEventRecord(e0, s));
            TRY(launch_mega_step(m->margs, s));
            JYC_CUDA(cudaEventRecord(e1, s));
            JYC_CUDA(cudaEventSynchronize(e1));
            float t = 0.0f;
            JYC_CUDA(cudaEventElapsedTime(&t, e0, e1));
            ms[0] += t;
            launches[0] += 1;
        }
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
        return JYC_OK;
    }
    if (!m->prof_exec) {
        m->prof_marks.reset(new Prof());
        m->prof_marks->s = m->stream;
        cudaGraph_t graph = nullptr;
        JYC_CUDA(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
        m->prof = m->prof_marks.get();
        int r = m->prof->mark(-1);
        if (r == JYC_OK) r = run_layers(m, 1, PosSrc{m->st, 0}, m->stream);
        if (r == JYC_OK) r = run_head(m, 0, m->stream);
        m->prof = nullptr;
        cudaError_t e = cudaStreamEndCapture(m->stream, &graph);
        if (r != JYC_OK) {
            if (graph) cudaGraphDestroy(graph);
            return r;
        }
        if (e != cudaSuccess) return cuda_fail(e, "cudaStreamEndCapture");
        e = cudaGraphInstantiate(&m->prof_exec, graph, 0);
        cudaGraphDestroy(graph);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGraphInstantiate");
    }
    const double wb = m->wtype == W_Q8 ? 34.0 / 32.0 : m->wtype == W_F16 ? 2.0 : 4.0;
    const double hb = m->head.f ? 4.0 : m->head.h ? 2.0 : 34.0 / 32.0;
    bytes[K_EMBED] = m->embed_f ? 4.0 * m->D : m->D * 34.0 / 32.0;
    bytes[K_QKV] = (double)m->nqkv * m->D * wb + 4.0 * m->D;
    bytes[K_ROPEQ] = 4.0 * m->nqkv;
    bytes[K_ATTN] = (double)m->KV * ctx * (2.0 * m->hd + 8.0);
    bytes[K_OPROJ] = (double)m->D * m->q_dim * wb;
    bytes[K_GATEUP] = 2.0 * m->F * m->D * wb + 4.0 * m->D;
    bytes[K_DOWN] = (double)m->D * m->F * wb;
    bytes[K_HEAD] = (double)m->V * m->D * hb + 4.0 * m->D;
    if (m->kq_path) {  // the K-quant blocks each class reads, per layer (types may differ by layer)
        double q = 0.0, o = 0.0, gu = 0.0, dn = 0.0;
        for (const DevLayer& ly : m->layers) {
            q += ly.kq[0].bytes() + ly.kq[1].bytes() + ly.kq[2].bytes();
            o += ly.kq[3].bytes();
            gu += ly.kq[4].bytes() + ly.kq[5].bytes();
            dn += ly.kq[6].bytes();
        }
        bytes[K_QKV] = q / m->L + 4.0 * m->D;
        bytes[K_OPROJ] = o / m->L;
        bytes[K_GATEUP] = gu / m->L + 4.0 * m->D;
        bytes[K_DOWN] = dn / m->L;
    }
    Prof* p = m->prof_marks.get();
    for (int it = 0; it < n_steps; it++) {
        JYC_CUDA(cudaGraphLaunch(m->prof_exec, s));
        count_launch(kernels_per_step(m));
        JYC_CUDA(cudaStreamSynchronize(s));
        for (size_t i = 1; i < p->ev.size(); i++) {
            float t = 0.0f;
            JYC_CUDA(cudaEventElapsedTime(&t, p->ev[i - 1], p->ev[i]));
            ms[p->cls[i]] += t;
            launches[p->cls[i]] += 1;
        }
    }
    return JYC_OK;
}

JYC_API int* jyc_model_tokens_device(jyc_model* m) { return m ? m->tokens : nullptr; }

JYC_API int jyc_model_length(jyc_model* m, void* stream) {
    if (!m) return arg_error("model_length: null model");
    cudaStream_t s = (cudaStream_t)stream;
    DevState hs;
    JYC_CUDA(cudaMemcpyAsync(&hs, m->st, sizeof(DevState), cudaMemcpyDeviceToHost, s));
    JYC_CUDA(cudaStreamSynchronize(s));
    return hs.len;
}

}  // extern "C"

// ===========================================================================
// Batched decode: B independent sequences over one model, each with its own
// int8 KV cache slot (the model's cache layout, [slot][layer][kv head][pos][hd])
// and length; one step appends one greedy token to every sequence. The
// matmuls run over the B rows together: the few-row CUDA-core matmul up to
// kSkMaxRows (8) sequences, tcgen05 token tiles from 9 on.
// ===========================================================================
struct jyc_batch {
    jyc_model* m = nullptr;
    int B = 0, cap = 0;
    int8_t *k8 = nullptr, *v8 = nullptr;
    float *ks = nullptr, *vs = nullptr;
    long long slot_q = 0, slot_s = 0;  // int8 / scale elements per slot
    int* tokens = nullptr;             // [B][cap + 1]
    int* lens = nullptr;               // [B]
    float* logits = nullptr;           // [B][V]
    unsigned long long* slots = nullptr;
    SkinnyWork sk{};                   // workspace of the few-row matmuls (up to 8 sequences)
    float *part_o = nullptr, *part_ml = nullptr;
    unsigned int* arrive = nullptr;
    int chunk = 64, nsplit = 1;
    bool tc = false;
    cudaGraphExec_t step_exec = nullptr;
    std::vector<void*> allocs;

    template <class T>
    int alloc(T** p, size_t count) {
        void* q = nullptr;
        cudaError_t e = cudaMalloc(&q, std::max<size_t>(count, 1) * sizeof(T));
        if (e != cudaSuccess) {
            set_error(std::string("cudaMalloc: ") + cudaGetErrorString(e));
            return JYC_ERR_NOMEM;
        }
        allocs.push_back(q);
        *p = static_cast<T*>(q);
        return JYC_OK;
    }
    ~jyc_batch() {
        if (step_exec) cudaGraphExecDestroy(step_exec);
        for (void* p : allocs) cudaFree(p);
    }
    KVView kv_layer(int l) const {
        KVView v = m->kv_layer(l);
        const size_t lay = (size_t)m->KV * m->max_seq;
        v.k = k8 + (size_t)l * lay * m->hd;
        v.v = v8 + (size_t)l * lay * m->hd;
        v.ks = ks + (size_t)l * lay;
        v.vs = vs + (size_t)l * lay;
        return v;
    }
};

namespace {

// Y[rows] = X[rows] . W^T (+ epilogue) over the batch's rows
int batch_gemm(jyc_batch* bt, const DevMat& w, const float* x, int ldx, const float* norm, float* y, int ldy,
               const float* bias, int epi, cudaStream_t s) {
    jyc_model* m = bt->m;
    if (bt->tc) {
        const int tepi = epi == EPI_BIAS ? TC_BIAS : epi == EPI_RESID ? TC_RESID : epi == EPI_SWIGLU ? TC_SWIGLU : TC_STORE;
        return run_tc_gemm(m, w, x, ldx, bt->B, norm, y, ldy, bias, tepi, device_error_word(), s);
    }
    // up to kSkMaxRows sequences per launch, RMSNorm fused
    for (int r0 = 0; r0 < bt->B; r0 += kSkMaxRows) {
        SkinnyGemm g{};
        g.x = x + (size_t)r0 * ldx; g.ldx = ldx; g.m = std::min(kSkMaxRows, bt->B - r0);
        g.n = w.n; g.k = w.k; g.qs = w.qs; g.d = w.d;
        g.norm_w = norm; g.eps = 1e-5f;
        g.y = y + (size_t)r0 * ldy; g.ldy = ldy; g.bias = bias;
        TRY(launch_skinny(g, epi, bt->sk, s));
    }
    return JYC_OK;
}

// One batched step: every sequence's last token through the stack, LM head,
// greedy pick appended (lengths advance on the device).
int batch_step(jyc_batch* bt, cudaStream_t s) {
    jyc_model* m = bt->m;
    const int B = bt->B;
    TRY(launch_bd_embed(bt->tokens, bt->cap + 1, bt->lens, B, m->embed_f, m->embed_q.qs, m->embed_q.d, m->D, m->X,
                        s));
    for (int l = 0; l < m->L; l++) {
        const DevLayer& ly = m->layers[l];
        TRY(batch_gemm(bt, ly.qkv, m->X, m->D, ly.rms1, m->qkv, m->nqkv, ly.bias, ly.bias ? EPI_BIAS : EPI_STORE, s));
        const KVView kv = bt->kv_layer(l);
        RopeQuantArgs rq{};
        rq.q = m->qkv; rq.k = m->qkv + m->q_dim; rq.v = m->qkv + m->q_dim + m->kv_dim;
        rq.ldq = m->nqkv; rq.rows = B; rq.H = m->H; rq.KV = m->KV; rq.hd = m->hd;
        rq.cos_t = m->cos_t; rq.sin_t = m->sin_t; rq.q8 = m->q8; rq.qsc = m->qsc;
        rq.kv = kv; rq.pos = PosSrc{nullptr, 0};
        rq.row_len = bt->lens; rq.kv_row_stride = bt->slot_q; rq.skv_row_stride = bt->slot_s;
        TRY(launch_rope_quant(rq, s));
        BdAttn at{};
        at.q8 = m->q8; at.qsc = m->qsc;
        at.k8 = kv.k; at.v8 = kv.v; at.ks = kv.ks; at.vs = kv.vs;
        at.slot_q = bt->slot_q; at.slot_s = bt->slot_s;
        at.cap = m->max_seq; at.H = m->H; at.KV = m->KV; at.hd = m->hd;
        at.chunk = bt->chunk; at.nsplit = bt->nsplit; at.lens = bt->lens;
        at.scale = 1.0f / sqrtf((float)m->hd);
        at.part_o = bt->part_o; at.part_ml = bt->part_ml; at.arrive = bt->arrive;
        at.out = m->attn; at.ldo = m->q_dim;
        TRY(launch_bd_attention(at, B, s));
        TRY(batch_gemm(bt, ly.o, m->attn, m->q_dim, nullptr, m->X, m->D, nullptr, EPI_RESID, s));
        TRY(batch_gemm(bt, ly.gateup, m->X, m->D, ly.rms2, m->h, m->F, nullptr, EPI_SWIGLU, s));
        TRY(batch_gemm(bt, ly.down, m->h, m->F, nullptr, m->X, m->D, nullptr, EPI_RESID, s));
    }
    TRY(batch_gemm(bt, m->head, m->X, m->D, m->final_norm, bt->logits, m->V, nullptr, EPI_STORE, s));
    return launch_bd_argmax(bt->logits, m->V, B, bt->slots, bt->tokens, bt->cap + 1, bt->lens, bt->cap, s);
}

int ensure_batch_graph(jyc_batch* bt) {
    if (bt->step_exec) return JYC_OK;
    cudaStream_t cs = bt->m->stream;
    cudaGraph_t graph = nullptr;
    const long long counted = jyc_kernel_launches();
    JYC_CUDA(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal));
    const int r = batch_step(bt, cs);
    cudaError_t e = cudaStreamEndCapture(cs, &graph);
    count_launch((int)(counted - jyc_kernel_launches()));  // captured, not launched
    if (r != JYC_OK) {
        if (graph) cudaGraphDestroy(graph);
        return r;
    }
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamEndCapture");
    e = cudaGraphInstantiate(&bt->step_exec, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGraphInstantiate");
    return JYC_OK;
}

int kernels_per_batch_step(const jyc_batch* bt) {
    const jyc_model* m = bt->m;
    const int per_gemm = bt->tc ? 2 : 1;  // split + GEMM, or one few-row matmul
    const int norms = bt->tc ? 0 : 1;     // the few-row path computes RMSNorm scales in a kernel
    // embed; per layer 4 matmuls (2 normalised) + RoPE/KV append + attention; LM head; argmax + append
    return 1 + m->L * (4 * per_gemm + 2 * norms + 2) + per_gemm + norms + 2;
}

}  // namespace

extern "C" {

JYC_API jyc_batch* jyc_batch_create(jyc_model* m, int num_seqs) {
    clear_error();
    if (!m || num_seqs <= 0) {
        set_error("batch_create: bad arguments");
        return nullptr;
    }
    if (m->wtype != W_Q8 || !m->pf_rows || m->head.f) {
        set_error("batch_create: batched decode needs a Q8_0 model (layers and LM head) with the batched prefill");
        return nullptr;
    }
    if (num_seqs > m->pf_rows || num_seqs > kMaxBatchSeqs) {
        set_error("batch_create: at most " + std::to_string(std::min(m->pf_rows, kMaxBatchSeqs)) + " sequences");
        return nullptr;
    }
    jyc_batch* bt = new (std::nothrow) jyc_batch();
    if (!bt) {
        set_error("out of host memory");
        return nullptr;
    }
    bt->m = m;
    bt->B = num_seqs;
    bt->cap = m->max_seq;
    bt->tc = num_seqs > kSkMaxRows;  // 9+ sequences: one padded 16-row tile beats two few-row passes
    auto fail = [&](int) -> jyc_batch* {
        delete bt;
        return nullptr;
    };
    cudaStream_t s = m->stream;
    const size_t lay = (size_t)m->L * m->KV * m->max_seq;
    bt->slot_q = (long long)(lay * m->hd);
    bt->slot_s = (long long)lay;
    int r = JYC_OK;
    if (r == JYC_OK) r = bt->alloc(&bt->k8, (size_t)num_seqs * bt->slot_q);
    if (r == JYC_OK) r = bt->alloc(&bt->v8, (size_t)num_seqs * bt->slot_q);
    if (r == JYC_OK) r = bt->alloc(&bt->ks, (size_t)num_seqs * bt->slot_s);
    if (r == JYC_OK) r = bt->alloc(&bt->vs, (size_t)num_seqs * bt->slot_s);
    if (r == JYC_OK) r = bt->alloc(&bt->tokens, (size_t)num_seqs * (bt->cap + 1));
    if (r == JYC_OK) r = bt->alloc(&bt->lens, (size_t)num_seqs);
    if (r == JYC_OK) r = bt->alloc(&bt->logits, (size_t)num_seqs * m->V);
    if (r == JYC_OK) r = bt->alloc(&bt->slots, (size_t)num_seqs);
    if (r == JYC_OK && !bt->tc) {
        size_t part = 1, cnt = 1;
        auto need = [&](const DevMat& w) {
            part = std::max(part, skinny_part_floats(w.n, w.k));
            cnt = std::max(cnt, skinny_counters(w.n));
        };
        for (const DevLayer& ly : m->layers) {
            need(ly.qkv); need(ly.o); need(ly.gateup); need(ly.down);
        }
        need(m->head);
        r = prepare_skinny_kernels();
        if (r == JYC_OK) r = bt->alloc(&bt->sk.part, part);
        if (r == JYC_OK) r = bt->alloc(&bt->sk.cnt, cnt);
        if (r == JYC_OK) r = bt->alloc(&bt->sk.sc, (size_t)kSkMaxRows);
        if (r == JYC_OK) {
            const cudaError_t e = cudaMemsetAsync(bt->sk.cnt, 0, cnt * sizeof(unsigned int), s);
            if (e != cudaSuccess) r = cuda_fail(e, "cudaMemsetAsync");
        }
    }
    // attention split plan: about three CTAs per SM over (sequence, kv head, split)
    if (r == JYC_OK) {
        if (!bd_attention_supported(m->H, m->KV, m->hd))
            r = arg_error("batch_create: head_dim 64 or 128 and at most 8 query heads per kv head");
        bt->chunk = bd_attention_chunk(m->max_seq, num_seqs, m->KV);
        bt->nsplit = (m->max_seq + bt->chunk - 1) / bt->chunk;
    }
    if (r == JYC_OK) r = bt->alloc(&bt->part_o, (size_t)num_seqs * m->H * bt->nsplit * m->hd);
    if (r == JYC_OK) r = bt->alloc(&bt->part_ml, (size_t)num_seqs * m->H * bt->nsplit * 2);
    if (r == JYC_OK) r = bt->alloc(&bt->arrive, (size_t)num_seqs * m->KV);
    if (r == JYC_OK && bt->tc && !m->head.rexp) {  // the LM head on the tensor cores
        r = m->alloc(&m->head.rexp, (size_t)m->head.n);
        if (r == JYC_OK) r = launch_tc_rowexp(m->head.d, m->head.n, m->head.k, m->head.rexp, s);
    }
    if (r != JYC_OK) return fail(r);
    auto zero = [&](void* p, size_t bytes) -> int {
        const cudaError_t e = cudaMemsetAsync(p, 0, bytes, s);
        return e == cudaSuccess ? JYC_OK : cuda_fail(e, "cudaMemsetAsync");
    };
    if (r == JYC_OK) r = zero(bt->k8, (size_t)num_seqs * bt->slot_q);
    if (r == JYC_OK) r = zero(bt->v8, (size_t)num_seqs * bt->slot_q);
    if (r == JYC_OK) r = zero(bt->ks, (size_t)num_seqs * bt->slot_s * 4);
    if (r == JYC_OK) r = zero(bt->vs, (size_t)num_seqs * bt->slot_s * 4);
    if (r == JYC_OK) r = zero(bt->lens, (size_t)num_seqs * 4);
    if (r == JYC_OK) r = zero(bt->slots, (size_t)num_seqs * 8);
    if (r == JYC_OK) r = zero(bt->arrive, (size_t)num_seqs * m->KV * 4);
    if (r == JYC_OK) {
        const cudaError_t e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) r = cuda_fail(e, "cudaStreamSynchronize");
    }
    if (r != JYC_OK) return fail(r);
    return bt;
}

JYC_API void jyc_batch_free(jyc_batch* bt) { delete bt; }

JYC_API int jyc_batch_prefill(jyc_batch* bt, int seq, const int* prompt_ids, int prompt_len) {
    clear_error();
    if (!bt || seq < 0 || seq >= bt->B || !prompt_ids || prompt_len <= 0 || prompt_len >= bt->cap)
        return arg_error("batch_prefill: bad arguments");
    jyc_model* m = bt->m;
    cudaStream_t s = m->stream;
    int* tok = bt->tokens + (size_t)seq * (bt->cap + 1);
    JYC_CUDA(cudaMemcpyAsync(tok, prompt_ids, (size_t)prompt_len * sizeof(int), cudaMemcpyHostToDevice, s));
    // the model's own prefill, pointed at this sequence's cache slot and token
    // buffer (kernels take the pointers at launch; the model's are restored)
    int8_t* k8 = m->k8; int8_t* v8 = m->v8; float* ks = m->ks; float* vs = m->vs; int* tokens = m->tokens;
    m->k8 = bt->k8 + (size_t)seq * bt->slot_q;
    m->v8 = bt->v8 + (size_t)seq * bt->slot_q;
    m->ks = bt->ks + (size_t)seq * bt->slot_s;
    m->vs = bt->vs + (size_t)seq * bt->slot_s;
    m->tokens = tok;
    int r = set_state(m, prompt_len, 1 << 30, m->max_seq, nullptr, 0, s);
    if (r == JYC_OK) r = run_prefill(m, 0, prompt_len, s);
    m->k8 = k8; m->v8 = v8; m->ks = ks; m->vs = vs; m->tokens = tokens;
    TRY(r);
    TRY(launch_bd_take_len(m->st, bt->lens, seq, s));
    JYC_CUDA(cudaStreamSynchronize(s));
    return JYC_OK;
}

JYC_API int jyc_batch_decode(jyc_batch* bt, int n_steps, void* stream) {
    clear_error();
    if (!bt || n_steps < 0) return arg_error("batch_decode: bad arguments");
    TRY(ensure_batch_graph(bt));
    cudaStream_t s = (cudaStream_t)stream;  // as given: 0 is the legacy default stream
    for (int i = 0; i < n_steps; i++) {
        JYC_CUDA(cudaGraphLaunch(bt->step_exec, s));
        count_launch(kernels_per_batch_step(bt));
    }
    return JYC_OK;
}

JYC_API int jyc_batch_rewind(jyc_batch* bt, int len, void* stream) {
    clear_error();
    if (!bt || len <= 0 || len >= bt->cap) return arg_error("batch_rewind: bad length");
    return launch_bd_set_lens(bt->lens, bt->B, len, (cudaStream_t)stream);
}

JYC_API int jyc_batch_tokens(jyc_batch* bt, int seq, int* out_ids, int cap) {
    clear_error();
    if (!bt || seq < 0 || seq >= bt->B || !out_ids || cap <= 0) return arg_error("batch_tokens: bad arguments");
    int len = 0;
    JYC_CUDA(cudaStreamSynchronize(bt->m->stream));
    JYC_CUDA(cudaDeviceSynchronize());
    JYC_CUDA(cudaMemcpy(&len, bt->lens + seq, sizeof(int), cudaMemcpyDeviceToHost));
    const int n = std::min(len, cap);
    JYC_CUDA(cudaMemcpy(out_ids, bt->tokens + (size_t)seq * (bt->cap + 1), (size_t)n * sizeof(int),
                        cudaMemcpyDeviceToHost));
    return len;
}

JYC_API int jyc_batch_path(const jyc_batch* bt) { return bt ? (bt->tc ? 2 : 1) : -1; }

JYC_API int jyc_batch_kernels_per_step(const jyc_batch* bt) { return bt ? kernels_per_batch_step(bt) : 0; }

JYC_API double jyc_batch_kv_bytes_per_step(const jyc_batch* bt, int ctx) {
    return bt ? bt->B * jyc_model_kv_bytes_per_token(bt->m, ctx) : 0.0;
}

}  // extern "C"
