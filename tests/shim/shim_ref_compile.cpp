// Compiles include/jieyu_b200_shim.hpp in the same translation unit as the
// reference's own headers (the reference tree's libs/, include path given by
// tests/test_shim_host.py) and instantiates every shim entry point with the
// reference's real structs: WMat (libs/date_libs/wmat.h:32-44), LayerWeights
// and __KVcache (libs/date_libs/date.h:75-147), __KVq
// (libs/model_libs/attention/attention_q8.h:12-19). The shim's static_asserts
// check LayerWeights and WMat against the C ABI's layouts. main() then runs
// the argument-error paths, which return before any device work, so this
// needs no GPU: each must throw std::runtime_error as the reference's
// operators do on misuse.
#define JIEYU_HPP 1
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <exception>
#include <math.h>
#include <string>
#include <vector>
#if defined(_OPENMP)
#include <omp.h>
#endif

#include "date_libs/date.h"
#include "date_libs/check_cpu.h"
#include "date_libs/info.h"
#include "matmul_libs/matmul.h"
#include "matmul_libs/matmul_q.h"
#include "model_libs/wmat_kernel.h"
#include "model_libs/prefetch.h"
#include "model_libs/silu/silu.h"
#include "model_libs/rmsnorm/rmsnorm.h"
#include "model_libs/rope/rope.h"
#include "model_libs/attention/attention_q8.h"
#include "model_libs/ffn/ffn.h"
#include "model_libs/generate.h"

#include "jieyu_b200_shim.hpp"

template <class F>
static int throws(F f) {
    try {
        f();
    } catch (const std::runtime_error&) {
        return 1;
    }
    return 0;
}

// Every template instantiated with the reference's types (not called).
[[maybe_unused]] static void instantiate(const WMat& w, const LayerWeights* lw, const __KVq& kvq, __KVcache& cache,
                                         float* f, int* ids) {
    jieyu_b200::matmul_w(w, 1, 1, 32, f, f);
    jieyu_b200::attention_q8(f, f, f, f, 1, 0, 1, 1, 4, kvq);
    jieyu_b200::ffn(f, w, w, w, f, 1, 32, 32);
    jieyu_b200::generate(ids, 1, ids, 0, w, w, lw, 1, f, f, f, 8, 1, 0.0f, 8, 32, 1, 1, 32, 32, ids);
    jieyu_b200::generate_cached(ids, 1, ids, 0, w, w, lw, 1, f, f, f, 8, 1, 0.0f, 8, 32, 1, 1, 32, 32, cache, ids);
}

int main() {
    int ok = 0, total = 0;
    WMat none;
    __KVq kvq{nullptr, nullptr, nullptr, nullptr, 0};
    float x[4] = {0, 0, 0, 0};
    total++, ok += throws([] { jieyu_b200::qmat::matmul_q(nullptr, nullptr, nullptr, 1, 1, 32, 3); });
    total++, ok += throws([] { jieyu_b200::matmul(1, 1, 1, nullptr, nullptr, nullptr); });
    total++, ok += throws([&] { jieyu_b200::matmul_w(none, 0, 1, 1, x, x); });
    total++, ok += throws([] { jieyu_b200::rmsnorm(nullptr, nullptr, nullptr, 4, 1e-5f); });
    total++, ok += throws([] { jieyu_b200::rope_pos(nullptr, 1, 0, 1, 4, nullptr, nullptr); });
    total++, ok += throws([] { jieyu_b200::kv_pack_q8(nullptr, nullptr, nullptr, 1, 4, 1); });
    total++, ok += throws([&] { jieyu_b200::attention_q8(x, x, x, x, 1, 0, 3, 2, 4, kvq); });  // 3 % 2 != 0
    total++, ok += throws([&] { jieyu_b200::attention_q8(x, x, x, x, 0, 0, 2, 2, 4, kvq); });  // seq <= 0
    total++, ok += throws([] { jieyu_b200::silu(nullptr, nullptr, 4); });
    total++, ok += throws([&] { jieyu_b200::ffn(x, none, none, none, x, 0, 4, 4); });
    // generate's early returns (generate.h:25, 90-112): prompt_len <= 0 or > max_seq -> 0, no device work
    int ids[4] = {1, 2, 3, 4};
    LayerWeights lw{};
    total++, ok += jieyu_b200::generate(ids, 0, nullptr, 0, none, none, &lw, 1, x, x, x, 2, 4, 0.0f, 8, 4, 1, 1, 4,
                                        4, ids) == 0;
    total++, ok += jieyu_b200::generate(ids, 3, nullptr, 0, none, none, &lw, 1, x, x, x, 2, 4, 0.0f, 8, 4, 1, 1, 4,
                                        4, ids) == 0;
    __KVcache cache;
    cache.init(1, 2, 1, 4);
    // a cache of the wrong shape throws, as generate_cached does (generate.h:26-28)
    total++, ok += throws([&] {
        jieyu_b200::generate_cached(ids, 1, nullptr, 0, none, none, &lw, 1, x, x, x, 2, 4, 0.0f, 8, 4, 1, 2, 4, 4,
                                    cache, ids);
    });
    std::printf("shim: %d of %d misuse cases behaved as the reference\n", ok, total);
    return ok == total ? 0 : 1;
}
