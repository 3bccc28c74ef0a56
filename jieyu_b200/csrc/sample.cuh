// sample.cuh — the token pick of one generate step on the device, for a CTA
// of kSampleThreads threads (named barrier 1): repetition penalty, then greedy
// or the reference's sampler (libs/model_libs/generate.h:50-77; restated in
// the oracle as jyo_sample).
#pragma once
#include "common.cuh"

namespace jyc {

constexpr int kSampleThreads = 512;

__device__ __forceinline__ void sample_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kSampleThreads) : "memory"); }

// scratch: kSampleThreads doubles + 2 words of shared memory.
// Repetition penalty: every id generated so far (ids[p0..len)) divides a
// positive logit by `pen` / multiplies a non-positive one, once per
// occurrence, in order: the thread of the id's first occurrence applies all
// k of them. With `tag` (2 V words: first index, then counts; all 0xFFFFFFFF
// / 0 on entry and again on return) first occurrences and counts come from
// atomics, O(len - p0); without it every thread scans the ids, O((len - p0)^2).
// Greedy (T <= 0): first index of the maximum (NaN never picked). Sampling:
// p_v = expf((l_v - max) / T) written back to logits, summed in double (per
// thread over a contiguous chunk, then the chunks in order), one LCG step of
// *rng, r = (rng >> 8) / 2^24 * sum, the first v where the running r -= p_v
// reaches <= 0 (V - 1 if none). Returns the pick in every thread.
static __device__ __noinline__ int sample_block(float* logits, int V, float T, float pen, const int* ids, int p0,
                                                int len, unsigned int* rng, double* scratch, unsigned int* tag) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int* s_pick = reinterpret_cast<int*>(scratch + kSampleThreads);
    if (pen != 1.0f) {
        if (tag != nullptr) {
            unsigned int* cnt = tag + V;
            for (int i = p0 + tid; i < len; i += kSampleThreads) {
                const int id = ids[i];
                if (id < 0 || id >= V) continue;
                atomicMin(tag + id, (unsigned int)i);
                atomicAdd(cnt + id, 1u);
            }
            __threadfence_block();
            sample_sync();
            for (int i = p0 + tid; i < len; i += kSampleThreads) {
                const int id = ids[i];
                if (id < 0 || id >= V || *(volatile unsigned int*)(tag + id) != (unsigned int)i) continue;
                const unsigned int k = *(volatile unsigned int*)(cnt + id);
                float l = logits[id];
                for (unsigned int r = 0; r < k; r++) l = (l > 0.0f) ? __fdiv_rn(l, pen) : __fmul_rn(l, pen);
                logits[id] = l;
                cnt[id] = 0u;  // only this thread reads them; others see the tag reset as "not first"
                tag[id] = 0xFFFFFFFFu;
            }
        } else {
            for (int i = p0 + tid; i < len; i += kSampleThreads) {
                const int id = ids[i];
                if (id < 0 || id >= V) continue;
                bool first = true;
                for (int j = p0; j < i && first; j++) first = ids[j] != id;
                if (!first) continue;
                int k = 0;
                for (int j = i; j < len; j++) k += ids[j] == id;
                float l = logits[id];
                for (int r = 0; r < k; r++) l = (l > 0.0f) ? __fdiv_rn(l, pen) : __fmul_rn(l, pen);
                logits[id] = l;
            }
        }
        __threadfence_block();
        sample_sync();
    }
    if (T <= 0.0f) {
        unsigned long long best = 0ull;
        for (int v = tid; v < V; v += kSampleThreads) {
            const unsigned long long p = argmax_pack(logits[v], v);
            best = p > best ? p : best;
        }
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long q = __shfl_xor_sync(0xffffffffu, best, o);
            best = q > best ? q : best;
        }
        unsigned long long* s_best = reinterpret_cast<unsigned long long*>(scratch);
        if (lane == 0) s_best[warp] = best;
        sample_sync();
        if (tid == 0) {
            unsigned long long b = 0ull;
            for (int w = 0; w < kSampleThreads / 32; w++) b = s_best[w] > b ? s_best[w] : b;
            *s_pick = argmax_index(b);
        }
        sample_sync();
        return *s_pick;
    }
    // maximum (NaN ignored)
    float mx = -INFINITY;
    for (int v = tid; v < V; v += kSampleThreads) mx = fmaxf(mx, logits[v]);
    mx = warp_max(mx);
    float* s_mx = reinterpret_cast<float*>(scratch);
    if (lane == 0) s_mx[warp] = mx;
    sample_sync();
    mx = s_mx[0];
    for (int w = 1; w < kSampleThreads / 32; w++) mx = fmaxf(mx, s_mx[w]);
    sample_sync();
    // probabilities and per-chunk double sums
    const int chunk = (V + kSampleThreads - 1) / kSampleThreads;
    const int v0 = min(V, tid * chunk), v1 = min(V, v0 + chunk);
    double ssum = 0.0;
    for (int v = v0; v < v1; v++) {
        const float p = expf(__fdiv_rn(__fsub_rn(logits[v], mx), T));
        logits[v] = p;
        ssum += (double)p;
    }
    scratch[tid] = ssum;
    __threadfence_block();
    sample_sync();
    if (tid == 0) {
        double total = 0.0;
        for (int t = 0; t < kSampleThreads; t++) total += scratch[t];
        const unsigned int rn = *rng * 1664525u + 1013904223u;
        *rng = rn;
        double r = (double)(rn >> 8) / 16777216.0 * total;
        int next = V - 1;
        for (int t = 0; t < kSampleThreads; t++) {
            if (r - scratch[t] > 0.0) {  // not inside this chunk
                r -= scratch[t];
                continue;
            }
            const int c0 = min(V, t * chunk), c1 = min(V, c0 + chunk);
            for (int v = c0; v < c1; v++) {
                r -= (double)logits[v];
                if (r <= 0.0) {
                    next = v;
                    break;
                }
            }
            if (next != V - 1 || r <= 0.0) break;
        }
        *s_pick = next;
    }
    sample_sync();
    return *s_pick;
}

}  // namespace jyc
