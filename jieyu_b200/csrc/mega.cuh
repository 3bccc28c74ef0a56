// mega.cuh — persistent decode-step kernel (one cooperative launch per token).
#pragma once
#include "kernels.cuh"

namespace jyc {

// Q8_0 weights in the tiled device layout read by the decode kernel: column
// blocks of 512 (the last one may be narrower, width w_cb), block-major, rows
// contiguous inside a block:
//   qs: [cb][n][w_cb] signed int8 q, the 16-byte chunks of row r permuted
//       within aligned groups of 8 chunks (chunk c -> c ^ (r & 7)) so that the
//       tensor-core fragment loads of 8 consecutive rows hit distinct banks;
//   d : [cb][n/16][w_cb/32][8][2] fp16 scales: per 16-row group and Q8 block,
//       the scales of rows g and g+8 side by side (one 32-bit load gives the
//       pair a tensor-core fragment row needs). Needs n % 16 == 0.
// A run of consecutive rows of one block is one contiguous byte range, so a
// tile (rows x one column block) arrives with two 1-D TMA bulk copies.
constexpr int kMegaCB = 512;
constexpr int kMegaRT = 48;       // rows per tile (multiple of 16)
constexpr int kMegaMaxSlots = 6;  // ring depth upper bound
constexpr int kMegaMaxTP = 8;       // most tensor-parallel ranks of the in-kernel exchange
constexpr int kMegaCW = 16;       // consumer warps (each takes 512 / 32 / kMegaCW column blocks of a tile)
constexpr int kMegaSlotBytes = kMegaRT * kMegaCB + kMegaRT * (kMegaCB / 32) * 2;

// index of row R, block j (of nblk in the column block) in the paired scale layout
__host__ __device__ __forceinline__ size_t mega_d_index(size_t R, int j, int nblk) {
    return (((R >> 4) * (size_t)nblk + j) * 8 + (R & 7)) * 2 + ((R >> 3) & 1);
}

// Work split of one matrix over the CTAs: CTA b takes row chunk b / spl (rpc
// rows) and column group b % spl (cpg column blocks). spl > 1 (split-K) writes
// per-group partial sums that the next reader adds up.
struct MegaMat {
    const uint8_t* qs;  // tiled copy (see above)
    const uint16_t* d;
    int n, k;
    int rpc;  // rows per CTA (multiple of 16)
    int rt;   // rows per tile (multiple of 16, <= kMegaRT)
    int spl;  // column groups
    int cpg;  // column blocks per group
};

struct MegaLayer {
    MegaMat qkv, o, gu, dn;
    const float* rms1;
    const float* rms2;
    const float* bias;  // fused q|k|v bias or null
};

struct MegaArgs {
    const MegaLayer* layers;  // device array [L]
    int L;
    MegaMat head;
    const MegaMat* head_dev;  // device copy of `head` (walked by the copy issuer)
    const float* final_norm;
    const float* ef;          // fp32 embedding [V][D], or
    const uint8_t* eqs;       // tiled Q8_0 embedding (n = V, k = D)
    const uint16_t* ed;
    int D, H, KV, hd, F, V;
    int Ve;                   // embedding rows (the head may hold a vocabulary slice)
    int vocab_off;            // token id of the head's row 0
    const float* cos_t;
    const float* sin_t;
    int8_t* k8;               // KV cache [L][KV][max_seq][hd]
    int8_t* v8;
    float* ks;                // [L][KV][max_seq]
    float* vs;
    int max_seq;
    float* X;                 // residual stream [D] after each layer's down projection (and the final one)
    float* Xb;                // residual stream [D] after each layer's O projection
    float* pq;                // QKV partial sums [qkv.spl][q|k|v] (bias added by the reader)
    float* po;                // O partial sums [o.spl][D]
    float* pd;                // down partial sums [dn.spl][D]
    float* attn;              // merged attention rows [H * hd]
    float* qkv;               // [q|k|v]
    float* h;                 // SwiGLU output [F]
    float* logits;            // [V]
    unsigned int* stag;       // the sampler's penalty tags [2 V]
    float* part_o;            // attention split partials [H][nsplit][hd]
    float* part_ml;           // [H][nsplit][2]
    int chunk, nsplit;        // largest split length (at max_seq), split stride of part_o / part_ml
    int per_head;             // splits per kv head a step aims at (positions per split follow the context)
    int chunk_min;            // shortest split length
    int att_nb;               // K/V tiles in flight per attention warp (1 or 2)
    int gsz;                  // query heads per attention item (a divisor of H / KV)
    unsigned int* acnt;       // [L][KV]: finished attention items of (layer, kv head) in this step
    float scale;              // 1/sqrtf(hd)
    DevState* st;
    int* tokens;
    unsigned int* bar;        // grid-barrier counter (monotonic)
    int* err;                 // device error word
    int kmax;                 // largest GEMV input length (digit buffers)
    int kx;                   // longest row kept as floats in shared memory (max(D, H hd))
    int xs_bytes;             // shared bytes of the x / digits / attention union
    int nslots;               // ring depth
    int win0, win1;           // phases of this launch: [win0, win1) of 2 l + h (h 0: QKV..O, 1: gate/up..down), 2 L = head
    long long* trace;         // optional: SM clock at each phase boundary, [CTA][kMegaTracePts]
    // tensor parallel inside the kernel (tp > 1): every CTA stores its O / down
    // partial rows into every rank's receive area (peer stores over NVLink) and
    // bumps that rank's arrival counter for it; readers wait for all counters
    int tp, tp_rank;
    float* xo;                       // this rank's receive area of O partials [tp][o.spl][D]
    float* xdn;                      // ... of down partials [tp][dn.spl][D]
    unsigned int* xflag;             // [3][tp] arrival counters (O, down, LM-head argmax) per sender
    unsigned long long* xam;         // [tp] packed argmax of each rank's vocabulary slice
    int xo_stride, xdn_stride;       // floats per sender slot (spl * D)
    float* peer_xo[kMegaMaxTP];      // every rank's xo (own included), mapped into this process
    float* peer_xdn[kMegaMaxTP];
    unsigned int* peer_xflag[kMegaMaxTP];
    unsigned long long* peer_xam[kMegaMaxTP];
};

// Phase boundaries recorded per CTA when tracing: per layer 14 phase points
// and 9 points inside the CTA's first attention item, then the head.
constexpr int kMegaTraceLayer = 23;
constexpr int kMegaTracePts = 1 + 64 * kMegaTraceLayer + 4;  // up to 64 layers

int launch_q8_repack_tiled(const void* blocks, int n, int k, uint8_t* qs, uint16_t* d, int n_total,
                           int row_off, int row_stride, cudaStream_t s);
int mega_plan(MegaMat& m, int nctas, bool splittable, int only_cpg = 0);
int mega_smem_bytes(const MegaArgs& a);
int mega_xs_bytes(int kx, int kmax, int gsz, int hd, int nb);
int mega_attn_nb(int kx, int kmax, int gsz, int hd, int chunk, int attn_cap);
int mega_num_ctas();
int launch_mega_step(const MegaArgs& a, cudaStream_t s);
int prepare_mega_kernel(int smem, int G, int hd);
int mega_static_smem(int G, int hd);  // -1 when the kernel image cannot be queried
int* device_error_word();
int mega_negative_scales(bool reset);  // 1 when a repacked Q8_0 scale was negative, -1 on error

}  // namespace jyc
