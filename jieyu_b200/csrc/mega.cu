// mega.cu — the batch-1 decode step as ONE persistent cooperative kernel.
//
// One CTA per SM: 16 consumer warps + 1 producer warp. The producer streams
// every weight tile this CTA needs for the whole step (layer by layer: QKV,
// O, gate/up, down rows of its slice, then the LM-head slice) from HBM into a
// shared-memory ring with 1-D TMA bulk copies (cp.async.bulk, L2 evict-first,
// mbarrier completion). It never waits on activations, so it runs ahead across
// the grid barriers that separate the step's dependent phases; HBM keeps
// streaming while the consumers synchronise.
//
// Consumer phases per layer (reference: transformer_layer, transformer_layer.h:10-90):
//   QKV     x = RMSNorm(X) (layer 0: embedding row, wmat_row wmat_kernel.h:18-29)
//           -> Q|K|V rows (+ bias)                          [grid barrier]
//   ATTN    per (kv head, position split): RoPE + int8 quantisation of the
//           group's Q heads, K/V append at pos (owner split), int8 dot
//           scores, online softmax, PV -> split partials, one arrival count
//           per item on its (layer, kv head) counter
//   O       (no grid barrier: each CTA waits for the kv heads its columns
//           read) x = merge of those heads' split partials -> X += Wo x
//                                                            [grid barrier]
//   GATE/UP x = RMSNorm(X) -> h = silu(gate) * up           [grid barrier]
//   DOWN    x = h -> X += W2 h                              [grid barrier]
// then the LM head on RMSNorm(X) with a per-CTA argmax -> one atomicMax,
// a last barrier, and CTA 0 appends the token and advances the step state
// (generate.h:57-86).
//
// Dequant-dot on the tensor cores (mma.sync m16n8k32 s8 -> s32): the input
// vector x is cut into 32-element blocks matching Q8_0's; per block
// N_i = rint(x_i * 2^20 / amax) is split into three signed 7-bit digits
// (N = 2^14 a + 2^7 b + c), the B operand's three columns. One mma gives, for
// 16 rows, the exact integer dots of the int8 weights with each digit; they
// recombine as 2^14 C_a + 2^7 C_b + C_c and scale by the block's fp16 d and
// amax/2^20. x keeps 21 bits per block (error <= 2^-21 of the block max), the
// weight products stay exact: the accuracy of fp32 FMA accumulation.
// Reference arithmetic being replaced: qmat::matmul_q / dot_row_avx2
// (libs/matmul_libs/matmul_q.h:101-143).
//
// Warp w of the consumers owns the 32-column Q8 block w of each 512-column
// tile for every 16-row group; partial row sums meet in shared memory in a
// fixed order (deterministic).
//
// Every wait is bounded (mbarrier waits and grid barriers give up after about
// a second of clock cycles and record an error word the host reads).
#include <algorithm>
#include <cmath>
#include <cstdlib>

#include "mega.cuh"
#include "sample.cuh"
#include "ptx.cuh"

namespace jyc {

// The residual sum is a separate function (not inlined): its registers are
// then allocated apart from the kernel body's, which cuts the spills of the
// GEMV phases' tile loop (measured: the configs[3] step 2.75 -> 2.64 ms).
// Out-of-line attention items, merges, norms or digitisers measured slower
// (their call frames outweigh what the body saves), so those stay inline.
#ifndef JYC_COLD
#define JYC_COLD __noinline__
#endif

constexpr int kMegaThreads = (kMegaCW + 1) * 32;  // consumer warps + one copy-issuing warp

// Error word of the device kernels (non-zero: a bounded wait gave up; the
// value tells which: 3 ring slot free, 4 ring slot full, 5 grid barrier,
// 7 prefill digit copy, 8 tensor-parallel exchange, 9 attention arrivals
// before the O projection).
__device__ int g_err_word;

int* device_error_word() {
    int* p = nullptr;
    if (cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_err_word) != cudaSuccess) return nullptr;
    return p;
}

static __device__ __forceinline__ void csync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kMegaCW * 32) : "memory");
}

// physical 16-byte chunk of logical chunk c in row r (nch chunks per row)
static __host__ __device__ __forceinline__ int swz_chunk(int c, int r, int nch) {
    return ((c | 7) < nch) ? ((c & ~7) | ((c ^ r) & 7)) : c;
}

// ---------------------------------------------------------------------------
// Tiled repack: reference blocks [n][k/32] x 34 B -> [cb][row][w_cb] q layout
// and the paired scale layout (see mega.cuh). Negative scales (no Q8_0
// quantiser writes them: d = amax / 127) are flagged in g_neg_scale.
__device__ int g_neg_scale;

__global__ void q8_repack_tiled_kernel(const uint8_t* blocks, size_t nblocks, int nb, int k, uint8_t* qs,
                                       uint16_t* d, int n_total, int row_off, int row_stride) {
    for (size_t b = blockIdx.x * (size_t)blockDim.x + threadIdx.x; b < nblocks;
         b += (size_t)gridDim.x * blockDim.x) {
        const size_t r = b / nb;
        const int bl = (int)(b % nb);
        const size_t R = (size_t)row_off + r * (size_t)row_stride;
        const int col0 = bl * 32, cb = col0 / kMegaCB, w = min(kMegaCB, k - cb * kMegaCB);
        const int c = (col0 - cb * kMegaCB) / 16;  // even: first of the block's two chunks
        const uint8_t* src = blocks + b * 34;
        const uint16_t dh = (uint16_t)src[0] | ((uint16_t)src[1] << 8);
        if ((dh & 0x8000u) && (dh & 0x7fffu)) atomicOr(&g_neg_scale, 1);
        d[(size_t)cb * n_total * (kMegaCB / 32) + mega_d_index(R, c / 2, w / 32)] = dh;
        uint8_t* row = qs + (size_t)cb * n_total * kMegaCB + R * w;
        for (int h = 0; h < 2; h++) {
            uint32_t* q = reinterpret_cast<uint32_t*>(row + 16 * swz_chunk(c + h, (int)(R & 7), w / 16));
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const uint8_t* s4 = src + 2 + 16 * h + 4 * i;
                q[i] = (uint32_t)s4[0] | ((uint32_t)s4[1] << 8) | ((uint32_t)s4[2] << 16) | ((uint32_t)s4[3] << 24);
            }
        }
    }
}

int mega_negative_scales(bool reset) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_neg_scale, sizeof(int)) != cudaSuccess) return -1;
    if (reset) {
        const int z = 0;
        if (cudaMemcpyToSymbol(g_neg_scale, &z, sizeof(int)) != cudaSuccess) return -1;
    }
    return v;
}

int launch_q8_repack_tiled(const void* blocks, int n, int k, uint8_t* qs, uint16_t* d, int n_total,
                           int row_off, int row_stride, cudaStream_t s) {
    if (n <= 0 || k <= 0 || k % 32) return arg_error("q8_repack_tiled: k must be a positive multiple of 32");
    const size_t nb = (size_t)n * (k / 32);
    const int grid = (int)std::min<size_t>((nb + 255) / 256, 148 * 16);
    q8_repack_tiled_kernel<<<grid, 256, 0, s>>>(static_cast<const uint8_t*>(blocks), nb, k / 32, k, qs, d,
                                                n_total, row_off, row_stride);
    JYC_LAUNCHED();
    return JYC_OK;
}

// ---------------------------------------------------------------------------
// tile sequence of one matrix for CTA b (shared by producer and consumers)
// rows [r0, r1) and column blocks [cb0, cb1) of CTA b (empty when r1 <= r0)
struct MatRange {
    int r0, r1, cb0, cb1, kg;
};

static __device__ __forceinline__ MatRange mat_range(const MegaMat& M, int b) {
    MatRange r;
    const int rb = b / M.spl;
    r.kg = b - rb * M.spl;
    r.r0 = rb * M.rpc;
    r.r1 = min(r.r0 + M.rpc, M.n);
    r.cb0 = r.kg * M.cpg;
    r.cb1 = min(r.cb0 + M.cpg, (M.k + kMegaCB - 1) / kMegaCB);
    if (r.cb1 <= r.cb0) r.r1 = r.r0;
    return r;
}

static __device__ __forceinline__ int mat_tiles(const MegaMat& M, int b) {
    const MatRange r = mat_range(M, b);
    if (r.r1 <= r.r0) return 0;
    return ((r.r1 - r.r0 + M.rt - 1) / M.rt) * (r.cb1 - r.cb0);
}

// Position in the ring: slot and the parity of its current fill.
struct RingPos {
    int s, ph;
    __device__ __forceinline__ void next(int ns) {
        if (++s == ns) {
            s = 0;
            ph ^= 1;
        }
    }
};

// One weight tile (rows r0.., column block cb) into ring slot `slot`: two 1-D
// bulk copies (q bytes, then the fp16 scales) completing on `bar`.
static __device__ __forceinline__ void load_tile(const MegaMat& M, int r0, int rows, int cb, unsigned char* slot,
                                                 uint64_t* bar, uint64_t pol) {
    const int w = min(kMegaCB, M.k - cb * kMegaCB);
    const uint32_t qb = (uint32_t)(rows * w), db = (uint32_t)(rows * (w / 32) * 2);
    mbar_expect_tx(bar, qb + db);
    bulk_g2s(slot, M.qs + (size_t)cb * M.n * kMegaCB + (size_t)r0 * w, qb, bar, pol);
    bulk_g2s(slot + kMegaRT * kMegaCB, M.d + (size_t)cb * M.n * (kMegaCB / 32) + (size_t)r0 * (w / 32), db, bar,
             pol);
}

// Walk over one CTA's tiles of the whole step, in consumer order: per layer
// QKV, O, gate/up, down, then the LM head (l == L). Row tiles outer, column
// blocks inner, as consume_mat takes them.
struct TileCursor {
    int l, m, r0, r_end, cb, cb0, cb1;
    const MegaMat* M;
};

// The matrices of one step in device memory: layers[0..L) then the LM head.
struct StepMats {
    const MegaLayer* layers;
    const MegaMat* head;  // device copy of the head's plan
    int L;
    int ord_end;          // walk matrices with 4 l + m < ord_end (the head counts as 4 L)
};

static __device__ __forceinline__ const MegaMat* cursor_mat(const StepMats& sm, int l, int m) {
    if (l >= sm.L) return sm.head;
    const MegaLayer& ly = sm.layers[l];
    return m == 0 ? &ly.qkv : m == 1 ? &ly.o : m == 2 ? &ly.gu : &ly.dn;
}

// positions c on the first tile of matrix (c.l, c.m) or later; false past the head
static __device__ bool cursor_enter(const StepMats& sm, TileCursor& c, int b) {
    while (c.l <= sm.L && (c.l < sm.L ? 4 * c.l + c.m : 4 * sm.L) < sm.ord_end) {
        c.M = cursor_mat(sm, c.l, c.m);
        const MatRange r = mat_range(*c.M, b);
        c.r0 = r.r0;
        c.r_end = r.r1;
        c.cb = c.cb0 = r.cb0;
        c.cb1 = r.cb1;
        if (c.r0 < c.r_end) return true;
        if (c.l == sm.L || ++c.m == 4) {
            c.m = 0;
            c.l++;
        }
    }
    return false;
}

static __device__ bool cursor_next(const StepMats& sm, TileCursor& c, int b) {
    if (++c.cb < c.cb1) return true;
    c.cb = c.cb0;
    c.r0 += c.M->rt;
    if (c.r0 < c.r_end) return true;
    if (c.l == sm.L || ++c.m == 4) {
        c.m = 0;
        c.l++;
    }
    return cursor_enter(sm, c, b);
}

// Producer (one thread): every tile of the step into the ring, in consumer
// order, a slot refilled as soon as every consumer warp released it. It never
// waits on activations, so weights keep streaming across the grid barriers.
static __device__ bool produce_step(const StepMats& smats, int l0, int m0, int b, int ns, uint64_t* full,
                                    uint64_t* empty, unsigned char* ring, int* err) {
    const uint64_t pol = policy_evict_first();
    TileCursor c{l0, m0, 0, 0, 0, 0, 0, nullptr};
    bool have = cursor_enter(smats, c, b);
    RingPos rp{0, 0};
    for (int t = 0; have; t++) {
        if (t >= ns && !mbar_wait_err(&empty[rp.s], rp.ph ^ 1, err, 3)) return false;
        load_tile(*c.M, c.r0, min(c.M->rt, c.r_end - c.r0), c.cb, ring + (size_t)rp.s * kMegaSlotBytes, &full[rp.s],
                  pol);
        rp.next(ns);
        have = cursor_next(smats, c, b);
    }
    return true;
}

// Ring context of the consumer warps, handed to consume_mat.
struct Ring {
    uint64_t* full;
    uint64_t* empty;
    unsigned char* ring;
    int ns;
    RingPos rp;  // next tile to consume
};

static __device__ __forceinline__ bool wait_tile(Ring& r, int* err) {
    return mbar_wait_err(&r.full[r.rp.s], r.rp.ph, err, 4);
}

// This warp is done with the current tile: release it and advance.
static __device__ __forceinline__ void release_tile(Ring& r, int lane) {
    __syncwarp();
    if (lane == 0) mbar_arrive(&r.empty[r.rp.s]);
    r.rp.next(r.ns);
}

enum MegaEpi { ME_PART = 0, ME_SWIGLU, ME_ARGMAX };  // ME_PART: y[kg * n + row] (kg = column group)

static __device__ __forceinline__ void mma_s8(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                              uint32_t b1, int& c0, int& c1, int& c2, int& c3) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=r"(c0), "=r"(c1), "=r"(c2), "=r"(c3)
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

// Scale pair (rows g, g+8 of a 16-row group, one Q8 block) -> both fp16
// values as fp32 (exact conversions).
static __device__ __forceinline__ float d_lo(uint32_t w) { return h2f((uint16_t)(w & 0xffffu)); }
static __device__ __forceinline__ float d_hi(uint32_t w) { return h2f((uint16_t)(w >> 16)); }

// Peer stores of partial rows (tensor parallel): row values of column group kg
// also go to dst[q][off + kg * n + row] for every rank q < n_dst.
struct PeerPush {
    float* const* dst;
    int n_dst;
    size_t off;
};

// One 16-row group of one Q8 block: the warp's mma and the scaled digit sums
// added to (acc0, acc1) (rows g, g+8). `ap` points at the lane's A bytes of
// row g, `stride8` is 8 rows of the tile, `dw` the scale pair.
static __device__ __forceinline__ void group_dot(const unsigned char* ap, int stride8, uint32_t dw, uint2 bf,
                                                 float kx, int im, float& acc0, float& acc1) {
    const uint2 A0 = *reinterpret_cast<const uint2*>(ap);
    const uint2 A1 = *reinterpret_cast<const uint2*>(ap + stride8);
    int c0, c1, c2, c3;
    mma_s8(A0.x, A1.x, A0.y, A1.y, bf.x, bf.y, c0, c1, c2, c3);
    // im * C0 + C1 is exact in int32 (|C| < 2^18); one rounding to fp32
    const float va = (float)(c0 * im + c1);
    const float vb = (float)(c2 * im + c3);
    acc0 = __fmaf_rn(va, __fmul_rn(d_lo(dw), kx), acc0);
    acc1 = __fmaf_rn(vb, __fmul_rn(d_hi(dw), kx), acc1);
}

// y[rows of this CTA] = W . x for one matrix; x given as 3 int8 digit planes
// xd[0..2][k] and per-32 block scales xsc[k/32].
//
// Fragment use of m16n8k32: B column j < 3 holds digit j of x (lanes g < 3
// load it), columns 3..7 are zero. Lane (g, tq) receives C columns 2tq, 2tq+1
// of rows g and g+8: lane tq=0 digit sums a, b, lane tq=1 digit sum c and a
// zero, lanes tq=2,3 zeros. Every lane forms u = im * C0 + C1 (im = 2^7 on
// tq=0, 1 elsewhere) and accumulates u * d * sx * m (m = 2^7 on tq=0), i.e.
// 2^14 a + 2^7 b on tq=0 and c on tq=1; the two meet once per row tile.
// Accumulators carry a 2^-28 factor (scale products stay normal for block
// maxima down to 2^-54 and finite up to 2^57), removed at the end.
//
// Cross-warp sums are deferred: after each row tile a warp stores its row
// sums in s_acc[warp][cap] (no CTA barrier); the 16 warps' rows are added in
// warp order (the same order for every row, deterministic) once the buffer
// holds `cap` rows or the matrix ends. Full tiles (rows kMegaRT, 512 columns)
// take a path with constant strides.
template <int EPI>
static __device__ __forceinline__ bool consume_mat(const MegaMat& M, const int8_t* xd, const float* xsc, Ring& rg_,
                                                   float* s_acc, int cap, float* y, unsigned long long* s_best,
                                                   int* err, PeerPush push = PeerPush{nullptr, 0, 0},
                                                   int idx_off = 0) {
    const int b = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int g = lane >> 2, tq = lane & 3;
    const int im = tq == 0 ? 128 : 1;
    const float km = tq == 0 ? 0x1p-21f : 0x1p-28f;  // 2^-28 * m
    const MatRange R = mat_range(M, b);
    const int r_begin = R.r0, r_end = R.r1, rt = M.rt;
    const int ncb = (M.k + kMegaCB - 1) / kMegaCB;
    const int wl = M.k - (ncb - 1) * kMegaCB;  // width of the last column block
    // Warp w takes the 32-column blocks w + i * kMegaCW (i < BPW) of each tile.
    // Per-lane A fragment offsets (rows g and g+8 of every 16-row group share
    // the swizzled chunk since row & 7 == g) for full and last column blocks.
    constexpr int BPW = (kMegaCB / 32) / kMegaCW;
    int a_full[BPW], a_last[BPW];
#pragma unroll
    for (int i = 0; i < BPW; i++) {
        const int bw = warp + i * kMegaCW, cf = 2 * bw + (tq >> 1), co = 8 * (tq & 1);
        a_full[i] = g * kMegaCB + 16 * swz_chunk(cf, g, kMegaCB / 16) + co;
        a_last[i] = g * wl + 16 * swz_chunk(cf, g, wl / 16) + co;
    }
    const int8_t* xb = xd + (size_t)min(g, 2) * M.k + 32 * warp + 8 * tq;
    constexpr int NRG = kMegaRT / 16;
    int rbase = r_begin;  // first row held in s_acc
    for (int r0 = r_begin; r0 < r_end; r0 += rt) {
        const int rows = min(rt, r_end - r0), nrg = rows >> 4;
        float acc[NRG][2];
#pragma unroll
        for (int j = 0; j < NRG; j++) acc[j][0] = acc[j][1] = 0.0f;
        for (int cb = R.cb0; cb < R.cb1; cb++) {
            if (!wait_tile(rg_, err)) return false;
            const bool lastb = cb == ncb - 1;
            const int w = lastb ? wl : kMegaCB, nblk = w >> 5;
            const unsigned char* slot = rg_.ring + (size_t)rg_.rp.s * kMegaSlotBytes;
            if (w == kMegaCB && nrg == NRG) {  // full tile: constant strides
#pragma unroll
                for (int i = 0; i < BPW; i++) {
                    const int bw = warp + i * kMegaCW;
                    const uint32_t* dp = reinterpret_cast<const uint32_t*>(slot + kMegaRT * kMegaCB) + bw * 8 + g;
                    uint2 bf = make_uint2(0u, 0u);
                    if (g < 3) bf = *reinterpret_cast<const uint2*>(xb + cb * kMegaCB + 32 * i * kMegaCW);
                    const float kx = __fmul_rn(xsc[cb * (kMegaCB / 32) + bw], km);
                    const unsigned char* ap = slot + a_full[i];
#pragma unroll
                    for (int rg = 0; rg < NRG; rg++)
                        group_dot(ap + rg * 16 * kMegaCB, 8 * kMegaCB, dp[rg * (kMegaCB / 32) * 8], bf, kx, im,
                                  acc[rg][0], acc[rg][1]);
                }
            } else {
#pragma unroll
                for (int i = 0; i < BPW; i++) {
                    const int bw = warp + i * kMegaCW;
                    if (bw < nblk) {
                        const uint32_t* dp =
                            reinterpret_cast<const uint32_t*>(slot + kMegaRT * kMegaCB) + bw * 8 + g;
                        uint2 bf = make_uint2(0u, 0u);
                        if (g < 3) bf = *reinterpret_cast<const uint2*>(xb + cb * kMegaCB + 32 * i * kMegaCW);
                        const float kx = __fmul_rn(xsc[cb * (kMegaCB / 32) + bw], km);
                        const unsigned char* ap = slot + (lastb ? a_last[i] : a_full[i]);
#pragma unroll
                        for (int rg = 0; rg < NRG; rg++)
                            if (rg < nrg)
                                group_dot(ap + rg * 16 * w, 8 * w, dp[rg * nblk * 8], bf, kx, im, acc[rg][0],
                                          acc[rg][1]);
                    }
                }
            }
            release_tile(rg_, lane);
        }
#pragma unroll
        for (int rg = 0; rg < NRG; rg++) {
            acc[rg][0] = __fadd_rn(acc[rg][0], __shfl_down_sync(0xffffffffu, acc[rg][0], 1));
            acc[rg][1] = __fadd_rn(acc[rg][1], __shfl_down_sync(0xffffffffu, acc[rg][1], 1));
        }
        const int ro = r0 - rbase;
        if (tq == 0) {
#pragma unroll
            for (int rg = 0; rg < NRG; rg++)
                if (rg < nrg) {
                    s_acc[warp * cap + ro + rg * 16 + g] = acc[rg][0];
                    s_acc[warp * cap + ro + rg * 16 + g + 8] = acc[rg][1];
                }
        }
        if (r0 + rt < r_end && ro + rows + rt <= cap) continue;  // room for the next row tile
        // rows [rbase, r0 + rows): every warp's sums, in warp order
        const int nr = ro + rows;
        csync();
        if (EPI == ME_SWIGLU) {
            for (int e = tid; e < nr / 2; e += kMegaCW * 32) {
                float v0 = 0.0f, v1 = 0.0f;
#pragma unroll
                for (int w2 = 0; w2 < kMegaCW; w2++) {
                    v0 = __fadd_rn(v0, s_acc[w2 * cap + 2 * e]);
                    v1 = __fadd_rn(v1, s_acc[w2 * cap + 2 * e + 1]);
                }
                y[(rbase >> 1) + e] = __fmul_rn(silu_ref(__fmul_rn(v0, 0x1p28f)), __fmul_rn(v1, 0x1p28f));
            }
        } else if (EPI == ME_ARGMAX) {
            unsigned long long best = 0ull;
            for (int e = tid; e < nr; e += kMegaCW * 32) {
                float v = 0.0f;
#pragma unroll
                for (int w2 = 0; w2 < kMegaCW; w2++) v = __fadd_rn(v, s_acc[w2 * cap + e]);
                v = __fmul_rn(v, 0x1p28f);
                y[rbase + e] = v;
                const unsigned long long p = argmax_pack(v, idx_off + rbase + e);
                best = p > best ? p : best;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const unsigned long long q = __shfl_xor_sync(0xffffffffu, best, o);
                best = q > best ? q : best;
            }
            if (lane == 0 && best) atomicMax(s_best, best);
        } else {
            for (int e = tid; e < nr; e += kMegaCW * 32) {
                float v = 0.0f;
#pragma unroll
                for (int w2 = 0; w2 < kMegaCW; w2++) v = __fadd_rn(v, s_acc[w2 * cap + e]);
                v = __fmul_rn(v, 0x1p28f);
                const size_t o = (size_t)R.kg * M.n + rbase + e;
                y[o] = v;
                for (int q = 0; q < push.n_dst; q++) push.dst[q][push.off + o] = v;
            }
        }
        csync();
        rbase = r0 + rt;
    }
    return true;
}

// x_s = RMSNorm(x_s) * w over k (sum of squares: per-thread FMA chains + warp/CTA tree).
// The weights of a thread's first kNormW elements are requested before the
// sum of squares, so their L2 round trip overlaps it.
constexpr int kNormW = 8;
static __device__ void x_norm(float* x_s, int k, const float* w, float eps, float* s_red) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int NT = kMegaCW * 32;
    float wr[kNormW];
#pragma unroll
    for (int j = 0; j < kNormW; j++) wr[j] = tid + j * NT < k ? __ldg(w + tid + j * NT) : 0.0f;
    csync();
    float ss = 0.0f;
    for (int i = tid; i < k; i += NT) ss = __fmaf_rn(x_s[i], x_s[i], ss);
    ss = warp_sum(ss);
    if (lane == 0) s_red[warp] = ss;
    csync();
    float tsum = 0.0f;
    for (int i = 0; i < kMegaCW; i++) tsum += s_red[i];
    const float den = __fadd_rn(__fdiv_rn(tsum, (float)k), eps);
    const float sc = den <= 0.0f ? 0.0f : __fdiv_rn(1.0f, __fsqrt_rn(den));
#pragma unroll
    for (int j = 0; j < kNormW; j++) {
        const int i = tid + j * NT;
        if (i < k) x_s[i] = __fmul_rn(__fmul_rn(x_s[i], sc), wr[j]);
    }
    for (int i = tid + kNormW * NT; i < k; i += NT) x_s[i] = __fmul_rn(__fmul_rn(x_s[i], sc), __ldg(w + i));
    csync();
}

// x_s[0..k) = base + sum of np partial rows (stride k), in that order; `out`
// (one CTA) also receives the sum. 16-byte loads, two partial rows issued
// ahead of their adds.
// (Eight rows in flight measured slower: more registers, more spills.)
constexpr int kMaxParts = 8;
static __device__ JYC_COLD void x_resid(float* x_s, const float* base, const float* parts, int np, int k,
                                        float* out) {
    constexpr int RB = 2;
    const float4* b4 = reinterpret_cast<const float4*>(base);
    const float4* p4 = reinterpret_cast<const float4*>(parts);
    float4* d4 = reinterpret_cast<float4*>(x_s);
    float4* o4 = reinterpret_cast<float4*>(out);
    const int k4 = k >> 2;
    for (int i = threadIdx.x; i < k4; i += kMegaCW * 32) {
        float4 v = __ldcg(b4 + i);
        for (int j0 = 0; j0 < np; j0 += RB) {  // RB partial rows in flight
            float4 q[RB];
#pragma unroll
            for (int j = 0; j < RB; j++)
                if (j0 + j < np) q[j] = __ldcg(p4 + (size_t)(j0 + j) * k4 + i);
#pragma unroll
            for (int j = 0; j < RB; j++)
                if (j0 + j < np) {
                    v.x = __fadd_rn(v.x, q[j].x);
                    v.y = __fadd_rn(v.y, q[j].y);
                    v.z = __fadd_rn(v.z, q[j].z);
                    v.w = __fadd_rn(v.w, q[j].w);
                }
        }
        d4[i] = v;
        if (out) o4[i] = v;
    }
    csync();
}

// Digits of one lane's 4 consecutive elements of a 32-element block whose 8
// lanes are lanes 8 q .. 8 q + 7 of the warp (all 32 lanes call; `valid`
// false contributes zeros and stores nothing). N = rint(x * 2^20 / amax)
// (round to nearest even: the 1.5 * 2^23 bias, exact for |N| < 2^22), split
// into three signed 7-bit digits N = 2^14 a + 2^7 b + c; the block scale
// amax / 2^20 is exact.
static __device__ __forceinline__ void digits4(float4 v, bool valid, int blk, int sub, int k, int8_t* xd,
                                               float* xsc) {
    float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
    if (!valid) return;
    // 2^20 * RN(1 / amax) == RN(2^20 / amax) (a power-of-two scaling of a
    // normal result)
    const float inv = amax > 0.0f ? __fmul_rn(__frcp_rn(amax), 1048576.0f) : 0.0f;
    const float vv[4] = {v.x, v.y, v.z, v.w};
    uint32_t pa = 0, pb = 0, pc = 0;
#pragma unroll
    for (int e = 0; e < 4; e++) {
        int N = __float_as_int(__fadd_rn(__fmul_rn(vv[e], inv), 12582912.0f)) - 0x4B400000;
        N = max(-1048576, min(1048576, N));
        const int c = ((N + 64) & 127) - 64;
        const int n1 = (N - c) >> 7;
        const int bd = ((n1 + 64) & 127) - 64;
        const int a = (n1 - bd) >> 7;
        pa |= (uint32_t)(a & 255) << (8 * e);
        pb |= (uint32_t)(bd & 255) << (8 * e);
        pc |= (uint32_t)(c & 255) << (8 * e);
    }
    reinterpret_cast<uint32_t*>(xd)[blk * 8 + sub] = pa;
    reinterpret_cast<uint32_t*>(xd + k)[blk * 8 + sub] = pb;
    reinterpret_cast<uint32_t*>(xd + 2 * k)[blk * 8 + sub] = pc;
    if (sub == 0) xsc[blk] = __fmul_rn(amax, 1.0f / 1048576.0f);  // exact: power of two
}

// x_s (k floats) -> three int8 digit planes + per-32 block scales, for the
// 32-element blocks [blk0, blk1) (default: all). A lane takes 4 consecutive
// elements, 8 lanes one block.
// GLOBAL: x is a global row written by other CTAs in this launch (read
// through L2 straight into the digits, no shared-memory copy); a lane's
// loads of up to kDigBatch passes are issued before their digits.
constexpr int kDigBatch = 8;
template <bool GLOBAL = false>
static __device__ void x_digitize(const float* x_s, int k, int8_t* xd, float* xsc, int blk0 = 0, int blk1 = -1) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int sub = lane & 7;  // lane within its block
    const int nblk = blk1 < 0 ? (k >> 5) : blk1;
    constexpr int NB = GLOBAL ? kDigBatch : 1;
    for (int base0 = blk0 + warp * 4; base0 < nblk; base0 += NB * kMegaCW * 4) {
        float4 v[NB];
#pragma unroll
        for (int u = 0; u < NB; u++) {
            const int blk = base0 + u * kMegaCW * 4 + (lane >> 3);
            v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (blk < nblk)
                v[u] = GLOBAL ? __ldcg(reinterpret_cast<const float4*>(x_s + blk * 32) + sub)
                              : reinterpret_cast<const float4*>(x_s + blk * 32)[sub];
        }
#pragma unroll
        for (int u = 0; u < NB; u++) {
            const int blk = base0 + u * kMegaCW * 4 + (lane >> 3);
            if (base0 + u * kMegaCW * 4 < nblk) digits4(v[u], blk < nblk, blk, sub, k, xd, xsc);
        }
    }
    csync();
}

// Tensor parallel: after this CTA's partial rows went to every rank, make
// them visible system-wide and count this CTA in every rank's counter for
// this sender (slot kind * tp + tp_rank).
static __device__ void xchg_arrive(const MegaArgs& a, int kind) {
    csync();
    if (threadIdx.x == 0) {
        __threadfence_system();
        for (int q = 0; q < a.tp; q++) atomicAdd_system(a.peer_xflag[q] + kind * a.tp + a.tp_rank, 1u);
    }
}

static __device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Wait (bounded) until every rank's CTAs delivered exchange number `target`
// (counts nct per exchange) of this kind; error word 8 on a timeout.
static __device__ bool xchg_wait(const MegaArgs& a, int kind, unsigned int target, int* s_ok) {
    if (threadIdx.x == 0) {
        int ok = 1;
        const long long t0 = clock64();
        for (int q = 0; q < a.tp && ok; q++) {
            const unsigned int* f = a.xflag + kind * a.tp + q;
            while ((int)(ld_acquire_sys(f) - target) < 0) {
                if (clock64() - t0 > (1LL << 31)) {
                    atomicExch(a.err, 8);
                    ok = 0;
                    break;
                }
                if (*(volatile int*)a.err != 0) {
                    ok = 0;
                    break;
                }
            }
        }
        *s_ok = ok;
    }
    csync();
    return *s_ok != 0;
}

// Grid barrier over the consumer threads of every CTA (bounded spin).
static __device__ bool grid_barrier(unsigned int* ctr, unsigned int target, int* err, int* s_ok) {
    csync();
    if (threadIdx.x == 0) {
        // arrive with a release reduction (no return trip to wait for); the
        // CTA barrier above orders every thread's writes before it
        asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(ctr), "r"(1u) : "memory");
        int ok = 1;
        if ((int)(ld_acquire_gpu(ctr) - target) < 0) {
            const long long t0 = clock64();
            while ((int)(ld_acquire_gpu(ctr) - target) < 0) {
                if (clock64() - t0 > (1LL << 31)) {
                    atomicExch(err, 5);
                    ok = 0;
                    break;
                }
                if (*(volatile int*)err != 0) {  // another CTA gave up: leave too
                    ok = 0;
                    break;
                }
            }
        }
        *s_ok = ok;
    }
    csync();
    return *s_ok != 0;
}

// Shared-memory plan of one attention item (byte offsets inside the x
// region): the quantised query heads, their scales, the new position's K and
// V rows (+ their two scales), then per consumer warp its K/V tiles
// ([nb][kAttTR][hd] each, 16-byte chunks rotated per row) and the tile's
// weights ([kAttTR][maxg]); after the tiles the same bytes hold the warps'
// (m, l, o) for the cross-warp merge.
constexpr int kAttTR = 16;  // positions per warp tile (two lanes per position)

struct AttnPlan {
    int q8, qsc, row, warps, wbytes, total;
};

static __host__ __device__ __forceinline__ AttnPlan attn_plan(int maxg, int hd, int nb) {
    AttnPlan p;
    int o = 0;
    p.q8 = o;
    o += (maxg * hd + 15) / 16 * 16;
    p.qsc = o;
    o += (maxg * 4 + 15) / 16 * 16;
    p.row = o;
    o += (2 * hd + 8 + 15) / 16 * 16;
    p.warps = o;
    p.wbytes = (nb * 2 * kAttTR * hd + kAttTR * maxg * 4 + 15) / 16 * 16;
    const int merge = kMegaCW * (2 * maxg + maxg * hd) * 4;
    o += max(kMegaCW * p.wbytes, merge);
    p.total = (o + 127) / 128 * 128;
    return p;
}

// physical 16-byte chunk of logical chunk c in tile row r (conflict-free
// reads of 16 rows by two lanes each)
template <int HD>
static __device__ __forceinline__ int att_chunk(int c, int r) {
    return HD == 128 ? ((c + r) & 7) : ((c + (r >> 1)) & 3);
}

// RoPE (when ct; rotated pairs stored in the reference's slot order) +
// kv_pack_q8 quantisation of one head row by a warp. The row is the sum of
// nsrc partial rows sstride apart (+ bias); it goes
// to dst/scale_out and, when dst2, also to dst2/scale2.
static __device__ __forceinline__ void rq_warp(const float* src, int nsrc, size_t sstride, const float* bias, int hd,
                                               const float* ct, const float* stb, int8_t* dst, float* scale_out,
                                               int lane, int8_t* dst2 = nullptr, float* scale2 = nullptr) {
    constexpr int MAXP = 4;
    const int half = hd >> 1;
    float x0[MAXP], x1[MAXP];
    float amax = 0.0f;
#pragma unroll
    for (int tt = 0; tt < MAXP; tt++) {
        const int p = lane + 32 * tt;
        x0[tt] = 0.0f;
        x1[tt] = 0.0f;
        if (p < half) {
            // RoPE factors and bias first (independent of the partials: their
            // round trips overlap)
            float c = 1.0f, sn = 0.0f, b0 = 0.0f, b1 = 0.0f;
            if (ct) {
                c = __ldg(ct + p);
                sn = __ldg(stb + p);
            }
            if (bias) {
                b0 = __ldg(bias + 2 * p);
                b1 = __ldg(bias + 2 * p + 1);
            }
            // the row = sum of the column groups' partials (+ bias), loaded
            // two groups at a time ahead of the adds
            float v0 = 0.0f, v1 = 0.0f;
            for (int k0 = 0; k0 < nsrc; k0 += 2) {
                float2 pv[2];
#pragma unroll
                for (int k = 0; k < 2; k++)
                    if (k0 + k < nsrc) pv[k] = __ldcg(reinterpret_cast<const float2*>(src + (k0 + k) * sstride + 2 * p));
#pragma unroll
                for (int k = 0; k < 2; k++)
                    if (k0 + k < nsrc) {
                        v0 = k0 + k == 0 ? pv[k].x : __fadd_rn(v0, pv[k].x);
                        v1 = k0 + k == 0 ? pv[k].y : __fadd_rn(v1, pv[k].y);
                    }
            }
            if (bias) {
                v0 = __fadd_rn(v0, b0);
                v1 = __fadd_rn(v1, b1);
            }
            if (ct) {
                const float r0 = __fmaf_rn(v0, c, -__fmul_rn(v1, sn));
                const float r1 = __fmaf_rn(v0, sn, __fmul_rn(v1, c));
                v0 = r0;
                v1 = r1;
            }
            x0[tt] = v0;
            x1[tt] = v1;
            amax = fmaxf(amax, fmaxf(fabsf(v0), fabsf(v1)));
        }
    }
    amax = warp_max(amax);
    const float inv = q8_inv(amax);
    if (lane == 0) {
        *scale_out = q8_scale(amax);
        if (scale2) *scale2 = q8_scale(amax);
    }
#pragma unroll
    for (int tt = 0; tt < MAXP; tt++) {
        const int p = lane + 32 * tt;
        if (p < half) {
            const int o = ct ? rope_slot(p, half) : p;
            const int8_t q0 = (int8_t)q8_round(x0[tt], inv), q1 = (int8_t)q8_round(x1[tt], inv);
            dst[2 * o] = q0;
            dst[2 * o + 1] = q1;
            if (dst2) {
                dst2[2 * o] = q0;
                dst2[2 * o + 1] = q1;
            }
        }
    }
}

// One (layer, kv head, query-head group, position split) attention item
// with the consumer warps (reference: attention over the int8 cache,
// attention_q8.h:38-184 with the score scaling dot * ((ks * qs) * 1/sqrt(hd)),
// fp32 softmax, the V scale folded into the weights). Each warp owns a
// contiguous run of the split's positions and keeps its own online-softmax
// state, so the position loop has no CTA-wide barrier: its K/V rows arrive by
// 16-byte cp.async into the warp's tiles (issued before the query heads are
// quantised, so the copies overlap that work; two tiles in flight when a warp
// has more than one); lanes (r, h) score half h of row r against every query
// head of the group (dp4a, halves added by one shuffle); each lane then
// accumulates P.V for hd/32 dims of every head. The new position's K and V
// (RoPE + kv_pack_q8 of the QKV rows, appended to the cache by the group-0
// item) come from shared memory. The warps merge at the end; the item writes
// its split partials (o, m, l) and counts itself in `cnt` (per kv head).
template <int MAXG, int HD>
static __device__ __forceinline__ bool attn_item(const MegaArgs& a, int layer, int kvh, int grp, int split,
                                                 int chunk, int pos, unsigned char* sm, unsigned int* cnt,
                                                 long long* tr) {
    constexpr int half = HD / 2, HC = HD / 16, HH = HC / 2, DPL = HD / 32;
    const int GA = a.H / a.KV, G = a.gsz, g0 = grp * G;
    const int nb = a.att_nb;
#define ATR(k)                                         \
    do {                                               \
        if (tr && threadIdx.x == 0) tr[k] = clock64(); \
    } while (0)
    ATR(0);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const AttnPlan P = attn_plan(MAXG, HD, nb);
    int8_t* s_q8 = reinterpret_cast<int8_t*>(sm + P.q8);
    float* s_qsc = reinterpret_cast<float*>(sm + P.qsc);
    int8_t* s_row = reinterpret_cast<int8_t*>(sm + P.row);  // new K row | V row | k scale | v scale
    float* s_rsc = reinterpret_cast<float*>(s_row + 2 * HD);
    unsigned char* wb = sm + P.warps + (size_t)warp * P.wbytes;
    int8_t* tk = reinterpret_cast<int8_t*>(wb);                     // [nb][TR][HD]
    int8_t* tv = tk + nb * kAttTR * HD;                             // [nb][TR][HD]
    float* sp = reinterpret_cast<float*>(tv + nb * kAttTR * HD);    // [TR][MAXG]

    const int c0 = split * chunk, c1 = min(c0 + chunk, pos + 1);
    const size_t lh = (size_t)layer * a.KV + kvh;
    int8_t* kb = a.k8 + lh * a.max_seq * HD;
    int8_t* vb = a.v8 + lh * a.max_seq * HD;
    float* ksb = a.ks + lh * a.max_seq;
    float* vsb = a.vs + lh * a.max_seq;
    const float* ct = a.cos_t + (size_t)pos * half;
    const float* stb = a.sin_t + (size_t)pos * half;
    const int q_dim = a.H * HD, kv_dim = a.KV * HD;
    const bool owner = pos < c1;

    // this warp's positions [w0, w1); rows below pos come from the cache
    const int per = (chunk + kMegaCW - 1) / kMegaCW;
    const int w0 = c0 + warp * per, w1 = min(w0 + per, c1), wc = min(w1, pos);
    const int ntile = w1 > w0 ? (w1 - w0 + kAttTR - 1) / kAttTR : 0;
    const int r = lane & (kAttTR - 1), hsel = lane >> 4;
    // lane (r, h) copies half h of K and V row r of tile t (one commit group per call)
    auto issue = [&](int t) {
        const int j = w0 + t * kAttTR + r;
        if (t < ntile && j < wc) {
            const int buf = nb == 2 ? (t & 1) : 0;
            int8_t* dk = tk + (buf * kAttTR + r) * HD;
            int8_t* dv = tv + (buf * kAttTR + r) * HD;
#pragma unroll
            for (int c = hsel * HH; c < (hsel + 1) * HH; c++) {
                const int ph = att_chunk<HD>(c, r) * 16;
                cp_async16_cg(dk + ph, kb + (size_t)j * HD + c * 16);
                cp_async16_cg(dv + ph, vb + (size_t)j * HD + c * 16);
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    issue(0);
    if (nb == 2) issue(1);
    // row scales of tile 0 (the cached rows; pos's come from s_row later)
    float ksr = 0.0f, vsr = 0.0f;
    {
        const int j = w0 + r;
        if (ntile > 0 && j < wc) {
            ksr = __ldcg(ksb + j);
            vsr = __ldcg(vsb + j);
        }
    }
    ATR(1);

    // RoPE + int8 quantisation of the group's query heads; the owner item
    // also forms the new K (roped) and V rows, and the group-0 item appends
    // them to the cache
    const MegaLayer& ly = a.layers[layer];
    const int nq = ly.qkv.spl;
    const size_t nqkv = (size_t)ly.qkv.n;
    const float* bq = ly.bias;
    for (int gq = warp; gq < G; gq += kMegaCW) {
        const size_t o = (size_t)(kvh * GA + g0 + gq) * HD;
        rq_warp(a.pq + o, nq, nqkv, bq ? bq + o : nullptr, HD, ct, stb, s_q8 + gq * HD, s_qsc + gq, lane);
    }
    if (owner) {
        const size_t ok = (size_t)q_dim + (size_t)kvh * HD, ov = ok + kv_dim;
        const bool app = g0 == 0;
        if (warp == kMegaCW - 1)
            rq_warp(a.pq + ok, nq, nqkv, bq ? bq + ok : nullptr, HD, ct, stb, app ? kb + (size_t)pos * HD : s_row,
                    app ? ksb + pos : s_rsc, lane, app ? s_row : nullptr, app ? s_rsc : nullptr);
        else if (warp == kMegaCW - 2)
            rq_warp(a.pq + ov, nq, nqkv, bq ? bq + ov : nullptr, HD, nullptr, nullptr,
                    app ? vb + (size_t)pos * HD : s_row + HD, app ? vsb + pos : s_rsc + 1, lane,
                    app ? s_row + HD : nullptr, app ? s_rsc + 1 : nullptr);
    }
    ATR(2);
    csync();
    ATR(3);

    float m[MAXG], l[MAXG], o[MAXG][DPL];
#pragma unroll
    for (int g = 0; g < MAXG; g++) {
        m[g] = -INFINITY;
        l[g] = 0.0f;
#pragma unroll
        for (int i = 0; i < DPL; i++) o[g][i] = 0.0f;
    }
    for (int t = 0; t < ntile; t++) {
        const int buf = nb == 2 ? (t & 1) : 0;
        const int jt = w0 + t * kAttTR, nj = min(kAttTR, w1 - jt);
        const float ksc = ksr, vsc = vsr;
        {
            ksr = vsr = 0.0f;  // the next tile's scales, loaded ahead
            const int j = jt + kAttTR + r;
            if (t + 1 < ntile && j < wc) {
                ksr = __ldcg(ksb + j);
                vsr = __ldcg(vsb + j);
            }
        }
        if (nb == 2)
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        else
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        __syncwarp();
        int8_t* rk = tk + buf * kAttTR * HD;
        int8_t* rv = tv + buf * kAttTR * HD;
        float ks_r = ksc, vs_r = vsc;
        if (pos >= jt && pos < jt + nj) {  // the new position: its rows from s_row
            const int rp = pos - jt;
            for (int c = lane; c < 2 * HC; c += 32) {
                const int cc = c < HC ? c : c - HC;
                int8_t* d = (c < HC ? rk : rv) + rp * HD + att_chunk<HD>(cc, rp) * 16;
                *reinterpret_cast<uint4*>(d) = reinterpret_cast<const uint4*>(s_row + (c < HC ? 0 : HD))[cc];
            }
            if (r == rp) {
                ks_r = s_rsc[0];
                vs_r = s_rsc[1];
            }
            __syncwarp();
        }
        if (t == 0) ATR(4);
        // scores of row r for every head: half hsel of the dot, halves added
        const bool valid = r < nj;
        uint4 kr[HH];
#pragma unroll
        for (int c = 0; c < HH; c++)
            kr[c] = *reinterpret_cast<const uint4*>(rk + r * HD + att_chunk<HD>(hsel * HH + c, r) * 16);
        // every head's dot first, then the reductions side by side (the
        // heads' shuffle chains overlap)
        float sc[MAXG], mx[MAXG];
#pragma unroll
        for (int g = 0; g < MAXG; g++) {
            int dot = 0;
            if (g < G) {
                const uint4* qrow = reinterpret_cast<const uint4*>(s_q8 + g * HD) + hsel * HH;
#pragma unroll
                for (int c = 0; c < HH; c++) {
                    const uint4 qw = qrow[c];
                    dot = __dp4a((int)qw.x, (int)kr[c].x, dot);
                    dot = __dp4a((int)qw.y, (int)kr[c].y, dot);
                    dot = __dp4a((int)qw.z, (int)kr[c].z, dot);
                    dot = __dp4a((int)qw.w, (int)kr[c].w, dot);
                }
            }
            sc[g] = (float)dot;
        }
#pragma unroll
        for (int g = 0; g < MAXG; g++) {
            const float d2 = sc[g] + __shfl_xor_sync(0xffffffffu, sc[g], 16);  // exact: integers below 2^24
            sc[g] = (valid && g < G) ? __fmul_rn(d2, __fmul_rn(__fmul_rn(ks_r, s_qsc[g]), a.scale)) : -INFINITY;
            mx[g] = sc[g];
        }
#pragma unroll
        for (int off = 8; off > 0; off >>= 1)  // rows live in lanes 0-15 and again in 16-31
#pragma unroll
            for (int g = 0; g < MAXG; g++) mx[g] = fmaxf(mx[g], __shfl_xor_sync(0xffffffffu, mx[g], off));
        float pw[MAXG];
#pragma unroll
        for (int g = 0; g < MAXG; g++) {
            pw[g] = 0.0f;
            if (g >= G) continue;
            const float mn = fmaxf(m[g], mx[g]);
            const float e = sc[g] == -INFINITY ? 0.0f : expf(sc[g] - mn);
            const float al = m[g] == -INFINITY ? 0.0f : expf(m[g] - mn);
            m[g] = mn;
            l[g] = __fmaf_rn(l[g], al, hsel == 0 ? e : 0.0f);  // each row counted once (lanes h = 0)
#pragma unroll
            for (int i = 0; i < DPL; i++) o[g][i] = __fmul_rn(o[g][i], al);
            pw[g] = __fmul_rn(e, vs_r);
        }
        if (hsel == 0) {
#pragma unroll
            for (int g = 0; g < MAXG; g++)
                if (g < G) sp[r * MAXG + g] = pw[g];
        }
        __syncwarp();
        // P.V: lane owns dims [DPL lane, DPL lane + DPL) of every head
        const int cl = (DPL * lane) >> 4, off = (DPL * lane) & 15;
        for (int jj = 0; jj < nj; jj++) {
            const int8_t* vr = rv + jj * HD + att_chunk<HD>(cl, jj) * 16 + off;
            float f[4];
            if (DPL == 4)
                u8x4_to_f32(*reinterpret_cast<const uint32_t*>(vr) ^ 0x80808080u, f);
            else
                u8x4_to_f32((uint32_t)(*reinterpret_cast<const uint16_t*>(vr)) ^ 0x80808080u, f);
            float pj[MAXG];
            if (MAXG >= 4) {  // the row's weights in 16-byte loads
#pragma unroll
                for (int g4 = 0; g4 < MAXG; g4 += 4) {
                    const float4 q4 = *reinterpret_cast<const float4*>(sp + jj * MAXG + g4);
                    pj[g4] = q4.x;
                    pj[g4 + 1] = q4.y;
                    pj[g4 + 2] = q4.z;
                    pj[g4 + 3] = q4.w;
                }
            } else {
#pragma unroll
                for (int g = 0; g < MAXG; g++) pj[g] = sp[jj * MAXG + g];
            }
#pragma unroll
            for (int g = 0; g < MAXG; g++)
                if (g < G) {
#pragma unroll
                    for (int i = 0; i < DPL; i++) o[g][i] = __fmaf_rn(pj[g], f[i], o[g][i]);
                }
        }
        __syncwarp();  // the next copies into this buffer come after every lane's reads
        if (nb == 2)
            issue(t + 2);
        else
            issue(t + 1);
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    ATR(5);
    // merge the warps: (m, l, o) per warp -> shared memory, then per head
#pragma unroll
    for (int g = 0; g < MAXG; g++) l[g] = warp_sum(l[g]);
    csync();  // every warp is done with its tiles: reuse the area
    float* mw = reinterpret_cast<float*>(sm + P.warps);  // [warps][MAXG]
    float* lw = mw + kMegaCW * MAXG;                     // [warps][MAXG]
    float* ow = lw + kMegaCW * MAXG;                     // [warps][G][HD]
    if (lane < MAXG) {
        float mv = m[0], lv = l[0];
#pragma unroll
        for (int g = 1; g < MAXG; g++)
            if (lane == g) {
                mv = m[g];
                lv = l[g];
            }
        mw[warp * MAXG + lane] = mv;
        lw[warp * MAXG + lane] = lv;
    }
#pragma unroll
    for (int g = 0; g < MAXG; g++)
        if (g < G)
#pragma unroll
            for (int i = 0; i < DPL; i++) ow[(warp * G + g) * HD + DPL * lane + i] = o[g][i];
    csync();
    // per head: the largest warp maximum M, each warp's weight exp(m_w - M)
    // (in place of m_w) and L = sum of weight * l_w; one warp per head
    for (int g = warp; g < G; g += kMegaCW) {
        const float mv = lane < kMegaCW ? mw[lane * MAXG + g] : -INFINITY;
        const float M = warp_max(mv);
        const float wgt = mv == -INFINITY ? 0.0f : expf(mv - M);
        const float L = warp_sum(lane < kMegaCW ? __fmul_rn(wgt, lw[lane * MAXG + g]) : 0.0f);
        __syncwarp();
        if (lane < kMegaCW) mw[lane * MAXG + g] = wgt;
        if (lane == 0) {
            const int h = kvh * GA + g0 + g;
            a.part_ml[((size_t)h * a.nsplit + split) * 2] = M;
            a.part_ml[((size_t)h * a.nsplit + split) * 2 + 1] = L;
        }
    }
    csync();
    for (int e = tid; e < G * HD; e += kMegaCW * 32) {
        const int g = e / HD, d = e - g * HD, h = kvh * GA + g0 + g;
        float O = 0.0f;
#pragma unroll 4
        for (int w = 0; w < kMegaCW; w++) O = __fmaf_rn(mw[w * MAXG + g], ow[(w * G + g) * HD + d], O);
        a.part_o[((size_t)h * a.nsplit + split) * HD + d] = O;
    }
    // arrival: the barrier orders the CTA's partial writes before thread 0's
    // fence and count
    csync();
    ATR(6);
    if (tid == 0)  // a release reduction: the CTA barrier above orders every thread's writes before it
        asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(cnt + kvh), "r"(1u) : "memory");
    ATR(7);
    ATR(8);
#undef ATR
    return true;
}

// Wait (bounded; error word 9) until every attention item of kv heads
// [kv0, kv1] arrived (cnt[kv] >= need).
static __device__ bool attn_wait(const unsigned int* cnt, int kv0, int kv1, unsigned int need, int* err, int* s_ok) {
    if (threadIdx.x == 0) {
        int ok = 1;
        const long long t0 = clock64();
        for (int kv = kv0; kv <= kv1 && ok; kv++) {
            while ((int)(ld_acquire_gpu(cnt + kv) - need) < 0) {
                if (clock64() - t0 > (1LL << 31)) {
                    atomicExch(err, 9);
                    ok = 0;
                    break;
                }
                if (*(volatile int*)err != 0) {
                    ok = 0;
                    break;
                }
            }
        }
        *s_ok = ok;
    }
    csync();
    return *s_ok != 0;
}

// x_s[e] for e in [c0, c1) = the attention row element e (head e / hd): its
// nv split partials (o, m, l) merged as sum_s w_s o_s, w_s = exp(m_s - M) / L
// (M the largest m_s, L = sum_s exp(m_s - M) l_s). The partials of the heads
// involved arrive in shared memory first (16-byte cp.async copies into the
// x region behind x_s[0, H hd), as many heads per round as fit): one L2
// round trip per round. part_ml's split stride (nsplit) is even, so a head's
// (m, l) pairs are whole 16-byte chunks.
static __device__ void attn_merge(const MegaArgs& a, float* x_s, int c0, int c1, int nv) {
    constexpr int nthr = kMegaCW * 32;
    const int tid = threadIdx.x, hd = a.hd, hd4 = hd >> 2, q_dim = a.H * hd;
    const int nv2 = (nv + 1) & ~1;  // (m, l) pairs staged per head
    float* stg = x_s + q_dim;
    const int per_head = nv * hd + 2 * nv2;
    const int hpr = max(1, (a.xs_bytes / 4 - q_dim) / per_head);
    const int h0 = c0 / hd, h1 = (c1 + hd - 1) / hd;
    for (int hb = h0; hb < h1; hb += hpr) {
        const int nh = min(h1 - hb, hpr);
        float* so = stg;                          // [nh][nv][hd]
        float* sml = stg + (size_t)nh * nv * hd;  // [nh][nv2][2]
        for (int idx = tid; idx < nh * nv * hd4; idx += nthr) {
            const int hh = idx / (nv * hd4), rem = idx - hh * nv * hd4, sp = rem / hd4, i = rem - sp * hd4;
            cp_async16_cg(so + ((size_t)hh * nv + sp) * hd + 4 * i,
                          a.part_o + ((size_t)(hb + hh) * a.nsplit + sp) * hd + 4 * i);
        }
        for (int idx = tid; idx < nh * (nv2 >> 1); idx += nthr) {
            const int hh = idx / (nv2 >> 1), c = idx - hh * (nv2 >> 1);
            cp_async16_cg(sml + ((size_t)hh * nv2 + 2 * c) * 2, a.part_ml + ((size_t)(hb + hh) * a.nsplit + 2 * c) * 2);
        }
        cp_async_wait_all();
        csync();
        // per (head, split): its weight exp(m_s - M) / L, M the head's largest
        // split maximum and L the weighted sum of the split sums (one warp per
        // head); the weights replace the (m, l) pairs in shared memory
        for (int hh = (int)(threadIdx.x >> 5); hh < nh; hh += kMegaCW) {
            const int lane = threadIdx.x & 31;
            float* ml = sml + (size_t)hh * nv2 * 2;
            float M = -INFINITY;
            for (int sp = lane; sp < nv; sp += 32) M = fmaxf(M, ml[2 * sp]);
            M = warp_max(M);
            float L = 0.0f;
            for (int sp = lane; sp < nv; sp += 32) {
                const float m = ml[2 * sp];
                L = __fmaf_rn(m == -INFINITY ? 0.0f : expf(m - M), ml[2 * sp + 1], L);
            }
            L = warp_sum(L);
            __syncwarp();
            for (int sp = lane; sp < nv; sp += 32) {
                const float m = ml[2 * sp];
                ml[2 * sp] = (m == -INFINITY || M == -INFINITY) ? 0.0f : __fdiv_rn(expf(m - M), L);
            }
        }
        csync();
        const int e0 = max(c0, hb * hd), e1 = min(c1, (hb + nh) * hd);
        for (int e = e0 + tid; e < e1; e += nthr) {
            const int hh = e / hd - hb, dd = e - (hb + hh) * hd;
            const float* wv = sml + (size_t)hh * nv2 * 2;
            const float* po = so + (size_t)hh * nv * hd + dd;
            float O = 0.0f;
            for (int sp = 0; sp < nv; sp++) O = __fmaf_rn(wv[2 * sp], po[(size_t)sp * hd], O);
            x_s[e] = O;
        }
        csync();
    }
}

// One instantiation per attention shape (query heads per kv head <= MAXG,
// head_dim HD) and per exchange mode (TP: in-kernel tensor-parallel
// exchange): each kernel carries only the code its model runs.
template <int MAXG, int HD, bool TP>
__global__ void __launch_bounds__(kMegaThreads, 1) mega_step_kernel(MegaArgs a) {
    extern __shared__ __align__(128) unsigned char sm[];
    uint64_t* full = reinterpret_cast<uint64_t*>(sm);
    uint64_t* empty = full + kMegaMaxSlots;
    static_assert(kMegaMaxSlots * 2 * 8 <= 128, "mbarriers exceed the shared-memory header");
    unsigned char* xs_region = sm + 128;
    float* x_s = reinterpret_cast<float*>(xs_region);  // kx floats, then the digits of up to kmax
    int8_t* xd = reinterpret_cast<int8_t*>(xs_region + (size_t)a.kx * 4);
    float* xsc = reinterpret_cast<float*>(xs_region + (size_t)a.kx * 4 + (size_t)a.kmax * 3);
    unsigned char* ring = sm + 128 + a.xs_bytes;
    __shared__ float s_part[kMegaCW * kMegaRT];
    // the GEMV phases' per-warp row sums: the float part of the x region (free
    // once x is digitised) when it holds a row tile per warp, else s_part
    const bool big = a.kx >= kMegaCW * kMegaRT;
    const int cap = big ? (a.kx / kMegaCW) & ~15 : kMegaRT;
    float* s_acc = big ? x_s : s_part;
    __shared__ float s_red[kMegaCW];
    __shared__ unsigned long long s_best;
    __shared__ int s_ok;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, b = blockIdx.x;
    const int ns = a.nslots;

    if (tid == 0) {
        for (int s = 0; s < ns; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kMegaCW);
        }
        mbar_fence_init();
    }
    __syncthreads();

    if (warp == kMegaCW) {  // ---- producer warp: the step's weight tiles, in consumer order
        if (lane == 0)
            produce_step(StepMats{a.layers, a.head_dev, a.L, 2 * a.win1}, a.win0 >> 1, (a.win0 & 1) * 2, b, ns,
                         full, empty, ring, a.err);
        return;
    }

    // ---- consumers ---------------------------------------------------------
    Ring rg{full, empty, ring, ns, RingPos{0, 0}};
    DevState* st = a.st;
    const int active = *(volatile const int*)&st->active;
    if (!active) {  // disabled step: take every tile off the ring, then leave
        int n = 0;
        for (int p = a.win0; p < a.win1; p++) {
            if (p >= 2 * a.L) {
                n += mat_tiles(*a.head_dev, b);
                continue;
            }
            const MegaLayer& ly = a.layers[p >> 1];
            n += (p & 1) ? mat_tiles(ly.gu, b) + mat_tiles(ly.dn, b) : mat_tiles(ly.qkv, b) + mat_tiles(ly.o, b);
        }
        for (int t = 0; t < n; t++) {
            if (!wait_tile(rg, a.err)) return;
            release_tile(rg, lane);
        }
        return;
    }
    const int pos = (*(volatile const int*)&st->len) - 1;
    const unsigned int base = *(volatile const unsigned int*)&st->bar_base;
    const unsigned int xb = *(volatile const unsigned int*)&st->xbase;  // tensor-parallel exchange epoch
    // attention arrival counters of this step: [apar][L][KV] (the other half,
    // the previous step's, is cleared layer by layer during this one)
    const unsigned int apar = *(volatile const unsigned int*)&st->apar & 1u;
    const unsigned int nct = gridDim.x;
    int bi = 0;
    bool ok = true;
    // positions per attention split at this context: about per_head splits
    // per kv head (at least chunk_min positions, a multiple of 64)
    int chunk = (pos + a.per_head) / a.per_head;
    chunk = max(a.chunk_min, (chunk + 63) / 64 * 64);
    const int nvalid = (pos + chunk) / chunk;
    const int ngrp = a.H / a.KV / a.gsz;  // query-head groups per kv head
#define TRACE(idx)                                                               \
    do {                                                                         \
        if (a.trace != nullptr && tid == 0) a.trace[(size_t)b * kMegaTracePts + (idx)] = clock64(); \
    } while (0)
    TRACE(0);

    // half-layer phases p = 2 l + h of this launch's window (h 0: QKV,
    // attention, O; h 1: gate/up, down); p = 2 L is the LM head
    for (int p = a.win0; p < a.win1 && p < 2 * a.L && ok; p++) {
        const int l = p >> 1;
        const MegaLayer& ly = a.layers[l];
        const int tb = 1 + l * kMegaTraceLayer;
        if ((p & 1) == 0) {
            // QKV
            if (l == 0) {
                const int id = __ldcg(a.tokens + pos);
                for (int i = tid; i < a.D; i += kMegaCW * 32) {
                    float v;
                    if (a.ef) {
                        v = __ldg(a.ef + (size_t)id * a.D + i);
                    } else {
                        const int cb = i / kMegaCB, w = min(kMegaCB, a.D - cb * kMegaCB), c = i - cb * kMegaCB;
                        const uint8_t* row = a.eqs + (size_t)cb * a.Ve * kMegaCB + (size_t)id * w;
                        const int8_t q = (int8_t)row[16 * swz_chunk(c >> 4, id & 7, w >> 4) + (c & 15)];
                        v = __fmul_rn((float)q, h2f(a.ed[(size_t)cb * a.Ve * (kMegaCB / 32) + mega_d_index(id, c / 32, w / 32)]));
                    }
                    x_s[i] = v;
                    if (b == 0) a.X[i] = v;
                }
            } else {  // X = X after O + the previous down projection's partials
                if (TP) {  // every rank's down partials of layer l-1, in rank order
                    ok = xchg_wait(a, 1, nct * (xb + (unsigned int)l), &s_ok);
                    if (!ok) break;
                    x_resid(x_s, a.Xb, a.xdn, a.tp * a.layers[l - 1].dn.spl, a.D, b == 0 ? a.X : nullptr);
                } else {
                    x_resid(x_s, a.Xb, a.pd, a.layers[l - 1].dn.spl, a.D, b == 0 ? a.X : nullptr);
                }
            }
            x_norm(x_s, a.D, ly.rms1, 1e-5f, s_red);
            x_digitize(x_s, a.D, xd, xsc);
            TRACE(tb + 0);
            ok = consume_mat<ME_PART>(ly.qkv, xd, xsc, rg, s_acc, cap, a.pq, &s_best,
                                      a.err);
            TRACE(tb + 1);
            ok = ok && grid_barrier(a.bar, base + (++bi) * nct, a.err, &s_ok);
            TRACE(tb + 2);
            if (!ok) break;
            // attention items (kv head, split), round-robin over CTAs
            unsigned int* acnt = a.acnt + ((size_t)apar * a.L + l) * a.KV;
            if (b == 0 && tid == 0)  // the previous step's counters of this layer: long read
                for (int kv = 0; kv < a.KV; kv++) a.acnt[((size_t)(apar ^ 1u) * a.L + l) * a.KV + kv] = 0u;
            for (int it = b; it < a.KV * ngrp * nvalid && ok; it += nct) {
                long long* tr = (a.trace && it == b) ? a.trace + (size_t)b * kMegaTracePts + tb + 14 : nullptr;
                const int kv_h = it / (ngrp * nvalid), rem = it - kv_h * ngrp * nvalid, gr = rem / nvalid;
                ok = attn_item<MAXG, HD>(a, l, kv_h, gr, rem - gr * nvalid, chunk, pos, xs_region, acnt, tr);
            }
            if (!ok) break;
            TRACE(tb + 3);
            // O projection (partials; the residual add happens in the next
            // reader). No grid barrier: a CTA waits for the attention items of
            // the kv heads whose query heads its columns hold, merges their
            // splits into its columns of the attention rows and digitises them.
            {
                const MatRange R = mat_range(ly.o, b);
                if (R.r1 > R.r0) {
                    const int c0 = R.cb0 * kMegaCB, c1 = min(R.cb1 * kMegaCB, a.H * a.hd);
                    const int gw = (a.H / a.KV) * a.hd;  // attention columns of one kv head
                    ok = attn_wait(acnt, c0 / gw, (c1 - 1) / gw, (unsigned int)(ngrp * nvalid), a.err, &s_ok);
                    if (!ok) break;
                    TRACE(tb + 4);
                    attn_merge(a, x_s, c0, c1, nvalid);
                    x_digitize(x_s, a.H * a.hd, xd, xsc, c0 >> 5, c1 >> 5);
                } else {
                    TRACE(tb + 4);
                }
            }
            TRACE(tb + 5);
            if (TP) {
                ok = consume_mat<ME_PART>(ly.o, xd, xsc, rg, s_acc, cap, a.po, &s_best, a.err,
                                          PeerPush{a.peer_xo, a.tp, (size_t)a.tp_rank * a.xo_stride});
                if (ok) xchg_arrive(a, 0);
            } else {
                ok = consume_mat<ME_PART>(ly.o, xd, xsc, rg, s_acc, cap, a.po, &s_best, a.err);
            }
            TRACE(tb + 6);
            // (tensor parallel: the readers' wait on every rank's arrival counts
            // this rank's CTAs too, which stands in for the grid barrier)
            if (!TP) ok = ok && grid_barrier(a.bar, base + (++bi) * nct, a.err, &s_ok);
            TRACE(tb + 7);
        } else {
            // gate/up + SwiGLU on RMSNorm(X + O partials); CTA 0 keeps that X in Xb
            if (TP) {  // every rank's O partials of layer l, in rank order
                ok = xchg_wait(a, 0, nct * (xb + (unsigned int)l + 1), &s_ok);
                if (!ok) break;
                x_resid(x_s, a.X, a.xo, a.tp * ly.o.spl, a.D, b == 0 ? a.Xb : nullptr);
            } else {
                x_resid(x_s, a.X, a.po, ly.o.spl, a.D, b == 0 ? a.Xb : nullptr);
            }
            // the down projection's column blocks of this CTA (its plan read
            // here: the round trip overlaps the norm, not the down prologue)
            int dn_b0 = 0, dn_b1 = 0;
            {
                const MatRange R = mat_range(ly.dn, b);
                if (R.r1 > R.r0) {
                    dn_b0 = R.cb0 * (kMegaCB / 32);
                    dn_b1 = min(R.cb1 * (kMegaCB / 32), a.F / 32);
                }
            }
            x_norm(x_s, a.D, ly.rms2, 1e-5f, s_red);
            x_digitize(x_s, a.D, xd, xsc);
            TRACE(tb + 8);
            ok = consume_mat<ME_SWIGLU>(ly.gu, xd, xsc, rg, s_acc, cap, a.h, &s_best,
                                        a.err);
            TRACE(tb + 9);
            ok = ok && grid_barrier(a.bar, base + (++bi) * nct, a.err, &s_ok);
            TRACE(tb + 10);
            if (!ok) break;
            // down projection + residual (SwiGLU rows digitised from L2: only
            // the column blocks this CTA's tiles read)
            if (dn_b1 > dn_b0) x_digitize<true>(a.h, a.F, xd, xsc, dn_b0, dn_b1);
            TRACE(tb + 11);
            if (TP) {
                ok = consume_mat<ME_PART>(ly.dn, xd, xsc, rg, s_acc, cap, a.pd, &s_best, a.err,
                                          PeerPush{a.peer_xdn, a.tp, (size_t)a.tp_rank * a.xdn_stride});
                if (ok) xchg_arrive(a, 1);
            } else {
                ok = consume_mat<ME_PART>(ly.dn, xd, xsc, rg, s_acc, cap, a.pd, &s_best, a.err);
            }
            TRACE(tb + 12);
            if (!TP) ok = ok && grid_barrier(a.bar, base + (++bi) * nct, a.err, &s_ok);
            TRACE(tb + 13);
        }
    }
    if (!ok) return;
    if (a.win1 <= 2 * a.L) {  // window without the head: hand the barrier epoch on
        if (b == 0 && tid == 0) st->bar_base = base + (unsigned int)bi * nct;
        return;
    }
    // LM head + argmax
    const int th = 1 + a.L * kMegaTraceLayer;
    if (TP) {
        if (!xchg_wait(a, 1, nct * (xb + (unsigned int)a.L), &s_ok)) return;
        x_resid(x_s, a.Xb, a.xdn, a.tp * a.layers[a.L - 1].dn.spl, a.D, b == 0 ? a.X : nullptr);  // final X
    } else {
        x_resid(x_s, a.Xb, a.pd, a.layers[a.L - 1].dn.spl, a.D, b == 0 ? a.X : nullptr);  // final X kept in X
    }
    if (tid == 0) s_best = 0ull;
    x_norm(x_s, a.D, a.final_norm, 1e-5f, s_red);
    x_digitize(x_s, a.D, xd, xsc);
    TRACE(th + 0);
    if (!consume_mat<ME_ARGMAX>(*a.head_dev, xd, xsc, rg, s_acc, cap, a.logits, &s_best,
                                a.err, PeerPush{nullptr, 0, 0}, a.vocab_off))
        return;
    TRACE(th + 1);
    if (tid == 0 && s_best) atomicMax(&st->amax, s_best);
    if (!grid_barrier(a.bar, base + (++bi) * nct, a.err, &s_ok)) return;
    TRACE(th + 2);
    if (b != 0) return;
    int next;
    if (!TP && (st->temperature > 0.0f || st->penalty != 1.0f)) {
        // sampler / repetition penalty over the whole logits row (CTA 0's consumers)
        unsigned int rng = st->rng;
        next = sample_block(a.logits, a.V, st->temperature, st->penalty, a.tokens, st->prompt_len, st->len, &rng,
                            reinterpret_cast<double*>(x_s), a.stag);
        if (tid == 0) st->rng = rng;
    } else {
        if (tid != 0) return;
        unsigned long long packed = atomicAdd(&st->amax, 0ull);
        if (TP) {  // every rank's argmax of its vocabulary slice -> the largest
            for (int q = 0; q < a.tp; q++) a.peer_xam[q][a.tp_rank] = packed;
            __threadfence_system();
            for (int q = 0; q < a.tp; q++) atomicAdd_system(a.peer_xflag[q] + 2 * a.tp + a.tp_rank, 1u);
            const unsigned int target = xb / (unsigned int)a.L + 1u;
            const long long t0 = clock64();
            for (int q = 0; q < a.tp; q++) {
                while ((int)(ld_acquire_sys(a.xflag + 2 * a.tp + q) - target) < 0) {
                    if (clock64() - t0 > (1LL << 31)) {
                        atomicExch(a.err, 8);
                        return;
                    }
                }
                const unsigned long long v = *(volatile unsigned long long*)(a.xam + q);
                packed = v > packed ? v : packed;
            }
        }
        next = argmax_index(packed);
    }
    if (tid == 0) {
        const int len = st->len;
        a.tokens[len] = next;
        const int nlen = len + 1, nsteps = st->steps + 1;
        bool stop = nlen >= st->max_len || nsteps >= st->max_new;
        for (int e = 0; e < st->n_eos; e++)
            if (next == st->eos[e]) stop = true;
        st->len = nlen;
        st->steps = nsteps;
        st->amax = 0ull;
        st->bar_base = base + (unsigned int)bi * nct;
        if (TP) st->xbase = xb + (unsigned int)a.L;
        st->apar = apar ^ 1u;
        st->fresh = 0;
        if (stop) st->active = 0;
        __threadfence();
    }
}

// ---------------------------------------------------------------------------
int mega_num_ctas() {
    static int n = 0;
    if (n == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    }
    return n;
}

// Work split of a matrix: for every column-group count (split-K only when
// `splittable`, at most kMaxParts groups) the least rows per CTA that fit the
// CTAs, costed as the bytes one CTA streams + a hand-off cost per tile + an
// epilogue cost per row tile + the readers' extra round trips; the cheapest
// wins (fewer groups on ties). only_cpg > 0 asks for that many column blocks
// per group instead (when the groups fit).
int mega_plan(MegaMat& m, int nctas, bool splittable, int only_cpg) {
    if (m.n <= 0 || m.n % 16 || m.k % 32 || m.k <= 0) return JYC_ERR_UNSUPPORTED;
    const int ncb = (m.k + kMegaCB - 1) / kMegaCB;
    if (only_cpg > 0 && (ncb + only_cpg - 1) / only_cpg <= std::min(nctas, kMaxParts)) {
        // the caller's split: only_cpg column blocks per group
        const int cpg = std::min(only_cpg, ncb), spl = (ncb + cpg - 1) / cpg;
        int rpc = (m.n + nctas / spl - 1) / (nctas / spl);
        rpc = (rpc + 15) / 16 * 16;
        m.rpc = rpc;
        m.rt = std::min(kMegaRT, rpc);
        m.spl = spl;
        m.cpg = cpg;
        return JYC_OK;
    }
    // readers sum the groups two at a time: every pair beyond the first costs
    // them one more L2 round trip
    const double kTileCost = 8192.0, kRowTileCost = 24576.0, kGroupCost = 2048.0, kTripCost = 24576.0;
    double best = 1e300;
    for (int cpg = ncb; cpg >= 1; cpg--) {
        const int spl = (ncb + cpg - 1) / cpg;
        if ((spl > 1 && !splittable) || spl > nctas || spl > kMaxParts) continue;
        const int chunks = nctas / spl;
        int rpc = (m.n + chunks - 1) / chunks;
        rpc = (rpc + 15) / 16 * 16;
        const int rt = std::min(kMegaRT, rpc);
        const int rtiles = (rpc + rt - 1) / rt, tiles = rtiles * cpg;
        const double cost = (double)rpc * cpg * kMegaCB + tiles * kTileCost + rtiles * kRowTileCost +
                            (spl - 1) * kGroupCost + ((spl + 1) / 2 - 1) * kTripCost;
        if (cost < best) {
            best = cost;
            m.rpc = rpc;
            m.rt = rt;
            m.spl = spl;
            m.cpg = cpg;
        }
    }
    return JYC_OK;
}

// x (4 B per element of the longest row kept in shared memory, kx) + three
// digit planes (3 B) + block scales (1/8 B) per element of the longest GEMV
// input (kmax); the attention item's plan (sub-chunks of S positions) shares
// the region.
static int mega_xk_bytes(int kx, int kmax) { return kx * 4 + kmax * 3 + (kmax / 32) * 4; }

// query heads an attention item instantiation holds (the kernel's MAXG)
static int mega_maxg(int gsz) { return gsz <= 1 ? 1 : gsz <= 4 ? 4 : 8; }

int mega_xs_bytes(int kx, int kmax, int gsz, int hd, int nb) {
    const int xk = mega_xk_bytes(kx, kmax);
    const int samp = (kSampleThreads + 1) * (int)sizeof(double);  // the sampler's scratch (head phase)
    return (std::max(std::max(xk, samp), attn_plan(mega_maxg(gsz), hd, nb).total) + 127) / 128 * 128;
}

// Tiles in flight per attention warp: two when a warp's share of the longest
// split spans more than one tile and the double tiles fit max(x region,
// attn_cap bytes), else one.
int mega_attn_nb(int kx, int kmax, int gsz, int hd, int chunk, int attn_cap) {
    const int per = (chunk + kMegaCW - 1) / kMegaCW;
    if (per <= kAttTR) return 1;
    const int cap = std::max(mega_xk_bytes(kx, kmax), attn_cap);
    return attn_plan(mega_maxg(gsz), hd, 2).total <= cap ? 2 : 1;
}

int mega_smem_bytes(const MegaArgs& a) { return 128 + a.xs_bytes + a.nslots * kMegaSlotBytes; }

// the kernel instantiation of a model's attention shape (query heads per
// attention item G, head_dim) and exchange mode
template <bool TP>
static const void* mega_kernel_tp(int G, int hd) {
    if (hd == 64)
        return G <= 1   ? (const void*)mega_step_kernel<1, 64, TP>
               : G <= 4 ? (const void*)mega_step_kernel<4, 64, TP>
                        : (const void*)mega_step_kernel<8, 64, TP>;
    return G <= 1   ? (const void*)mega_step_kernel<1, 128, TP>
           : G <= 4 ? (const void*)mega_step_kernel<4, 128, TP>
                    : (const void*)mega_step_kernel<8, 128, TP>;
}

static const void* mega_kernel_for(int G, int hd, bool tp) {
    return tp ? mega_kernel_tp<true>(G, hd) : mega_kernel_tp<false>(G, hd);
}

int mega_static_smem(int G, int hd) {
    int mx = 0;
    for (int tp = 0; tp < 2; tp++) {
        cudaFuncAttributes fa{};
        if (cudaFuncGetAttributes(&fa, mega_kernel_for(G, hd, tp != 0)) != cudaSuccess) return -1;
        mx = std::max(mx, (int)fa.sharedSizeBytes);
    }
    return mx;
}

int prepare_mega_kernel(int smem, int G, int hd) {
    for (int tp = 0; tp < 2; tp++)
        JYC_CUDA(cudaFuncSetAttribute(mega_kernel_for(G, hd, tp != 0), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      smem));
    return JYC_OK;
}

int launch_mega_step(const MegaArgs& a, cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(mega_num_ctas());
    cfg.blockDim = dim3(kMegaThreads);
    cfg.dynamicSmemBytes = (size_t)mega_smem_bytes(a);
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeCooperative;  // all CTAs co-resident: the grid barriers need it
    at[0].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    void* args[] = {const_cast<MegaArgs*>(&a)};
    cudaError_t e = cudaLaunchKernelExC(&cfg, mega_kernel_for(a.gsz, a.hd, a.tp > 1), args);
    if (e != cudaSuccess) return cuda_fail(e, "mega_step launch");
    count_launch();
    return JYC_OK;
}

}  // namespace jyc
