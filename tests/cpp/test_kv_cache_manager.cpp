// The reference's KV cache tests (AICL-Lab/tiny-llm tests/test_kv_cache.cpp
// and the append round trip of tests/test_transformer.cu:141-194), written
// against this repository's tiny_llm::KVCacheManager facade. Without --gpu
// every test runs on the bookkeeping backend (no device needed) and the data
// round trip is skipped; with --gpu the CUDA backend is used throughout.
#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <functional>
#include <string>
#include <vector>

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "tiny_llm/kv_cache.h"

using namespace tiny_llm;

static bool g_gpu = false;
static int g_failed = 0, g_passed = 0;

#define EXPECT(cond)                                                                   \
    do {                                                                               \
        if (!(cond)) {                                                                 \
            std::fprintf(stderr, "  %s:%d: EXPECT failed: %s\n", __FILE__, __LINE__, #cond); \
            throw 1;                                                                   \
        }                                                                              \
    } while (0)

static PagedKVCacheConfig createConfig(int num_layers = 2, int num_heads = 4, int head_dim = 64,
                                  int max_seq_len = 128, int max_batch_size = 4) {
    PagedKVCacheConfig c;
    c.num_layers = num_layers;
    c.num_heads = num_heads;
    c.head_dim = head_dim;
    c.max_seq_len = max_seq_len;
    c.max_batch_size = max_batch_size;
    c.backend = g_gpu ? TL_BACKEND_CUDA : TL_BACKEND_HOST_BOOKKEEPING;
    return c;
}

static std::unique_ptr<KVCacheManager> createCache(const PagedKVCacheConfig &c) {
    auto r = KVCacheManager::create(c);
    if (r.isErr()) std::fprintf(stderr, "  create failed: %s\n", r.error().c_str());
    EXPECT(r.isOk());
    return std::move(r.value());
}

static void run(const char *name, const std::function<void()> &fn) {
    try {
        fn();
        ++g_passed;
        std::printf("[ OK ] %s\n", name);
    } catch (...) {
        ++g_failed;
        std::printf("[FAIL] %s\n", name);
    }
}

int main(int argc, char **argv) {
    for (int i = 1; i < argc; ++i)
        if (!std::strcmp(argv[i], "--gpu")) g_gpu = true;

    run("InitializationAllocatesMemory", [] {
        auto cache = createCache(createConfig());
        EXPECT(cache->getTotalMemory() > 0);
        EXPECT(cache->getUsedMemory() == 0);
        EXPECT(cache->getActiveSequenceCount() == 0);
    });
    run("AllocateSequenceReturnsValidId", [] {
        auto cache = createCache(createConfig());
        auto r = cache->allocateSequence(64);
        EXPECT(r.isOk());
        EXPECT(r.value() >= 0);
        EXPECT(cache->hasSequence(r.value()));
        EXPECT(cache->getSeqLen(r.value()) == 0);
    });
    run("AllocateMultipleSequences", [] {
        auto cache = createCache(createConfig(2, 4, 64, 128, 4));
        std::vector<int> ids;
        for (int i = 0; i < 4; ++i) {
            auto r = cache->allocateSequence(64);
            EXPECT(r.isOk());
            ids.push_back(r.value());
        }
        EXPECT(cache->getActiveSequenceCount() == 4);
        std::sort(ids.begin(), ids.end());
        EXPECT(std::unique(ids.begin(), ids.end()) == ids.end());
    });
    run("ExhaustionReturnsError", [] {
        auto cache = createCache(createConfig(2, 4, 64, 128, 2));
        EXPECT(cache->allocateSequence(64).isOk());
        EXPECT(cache->allocateSequence(64).isOk());
        auto r = cache->allocateSequence(64);
        EXPECT(r.isErr());
        EXPECT(r.error().find("exhausted") != std::string::npos);
    });
    run("ReleaseSequenceFreesSlot", [] {
        auto cache = createCache(createConfig(2, 4, 64, 128, 2));
        auto r1 = cache->allocateSequence(64);
        auto r2 = cache->allocateSequence(64);
        EXPECT(r1.isOk() && r2.isOk());
        EXPECT(cache->releaseSequence(r1.value()).isOk());
        EXPECT(!cache->hasSequence(r1.value()));
        EXPECT(cache->getActiveSequenceCount() == 1);
        EXPECT(cache->allocateSequence(64).isOk());
    });
    run("GetCacheReturnsValidPointers", [] {
        auto config = createConfig();
        auto cache = createCache(config);
        int id = cache->allocateSequence(64).value();
        for (int layer = 0; layer < config.num_layers; ++layer) {
            auto [k, v] = cache->getCache(id, layer);
            EXPECT(k != nullptr && v != nullptr && k != v);
        }
    });
    run("GetCacheForInvalidSequenceReturnsNull", [] {
        auto cache = createCache(createConfig());
        auto [k, v] = cache->getCache(999, 0);
        EXPECT(k == nullptr && v == nullptr);
    });
    run("InvalidMaxLenReturnsError", [] {
        auto cache = createCache(createConfig(2, 4, 64, 128, 4));
        EXPECT(cache->allocateSequence(0).isErr());
        EXPECT(cache->allocateSequence(-1).isErr());
        EXPECT(cache->allocateSequence(256).isErr());
    });
    run("MemoryAccountingIsCorrect", [] {
        auto cache = createCache(createConfig(2, 4, 64, 128, 4));
        size_t total = cache->getTotalMemory();
        EXPECT(cache->getFreeMemory() == total);
        EXPECT(cache->getUsedMemory() == 0);
        EXPECT(cache->allocateSequence(64).isOk());
        size_t one = cache->getUsedMemory();
        EXPECT(one > 0);
        EXPECT(cache->getFreeMemory() == total - one);
        EXPECT(cache->allocateSequence(64).isOk());
        EXPECT(cache->getUsedMemory() == one * 2);
    });
    run("InvalidLayerReturnsNullCachePointers", [] {
        auto cache = createCache(createConfig(2, 4, 8, 32, 2));
        int id = cache->allocateSequence(16).value();
        auto [k, v] = cache->getCache(id, -1);
        EXPECT(k == nullptr && v == nullptr);
        auto [k2, v2] = cache->getCache(id, 2);
        EXPECT(k2 == nullptr && v2 == nullptr);
    });
    run("InvalidAppendInputsDoNotAdvanceSequenceLength", [] {
        auto cache = createCache(createConfig(2, 4, 8, 32, 2));
        int id = cache->allocateSequence(16).value();
        EXPECT(cache->appendKV(id, -1, nullptr, nullptr, 0).isErr());
        EXPECT(cache->appendKV(id, 2, nullptr, nullptr, 1).isErr());
        EXPECT(cache->appendKV(id, 0, nullptr, nullptr, 1).isErr());
        EXPECT(cache->getSeqLen(id) == 0);
    });
    run("AdvanceSeqLenClampsToSequenceCapacity", [] {
        auto cache = createCache(createConfig(2, 4, 8, 32, 2));
        int id = cache->allocateSequence(5).value();
        cache->advanceSeqLen(id, 100);
        EXPECT(cache->getSeqLen(id) == 5);
    });
    run("AdvanceSeqLenIgnoresNonPositiveValues", [] {
        auto cache = createCache(createConfig(2, 4, 8, 32, 2));
        int id = cache->allocateSequence(5).value();
        EXPECT(cache->advanceSeqLen(id, 0).isErr());
        EXPECT(cache->advanceSeqLen(id, -3).isErr());
        EXPECT(cache->getSeqLen(id) == 0);
    });
    run("AppendDoesNotAdvanceVisibleSequenceLength", [] {
        auto config = createConfig(2, 4, 8, 32, 2);
        auto cache = createCache(config);
        int id = cache->allocateSequence(16).value();
        const int n = 3;
        const size_t elems = (size_t)n * config.num_heads * config.head_dim;
        if (g_gpu) {
            std::vector<half> hk(elems, __float2half(1.0f)), hv(elems, __float2half(2.0f));
            half *dk = nullptr, *dv = nullptr;
            EXPECT(cudaMalloc(&dk, elems * sizeof(half)) == cudaSuccess);
            EXPECT(cudaMalloc(&dv, elems * sizeof(half)) == cudaSuccess);
            cudaMemcpy(dk, hk.data(), elems * sizeof(half), cudaMemcpyHostToDevice);
            cudaMemcpy(dv, hv.data(), elems * sizeof(half), cudaMemcpyHostToDevice);
            EXPECT(cache->appendKV(id, 0, dk, dv, n).isOk());
            EXPECT(cache->syncCheck().isOk());
            cudaFree(dk);
            cudaFree(dv);
        }
        EXPECT(cache->getSeqLen(id) == 0);
        EXPECT(cache->advanceSeqLen(id, n).isOk());
        EXPECT(cache->getSeqLen(id) == n);
    });
    run("ProjectQKVAppendValidatesArguments", [] {  // the decode step's Q/K/V projection + append
        // every case here is refused before any device work (safe with --gpu)
        auto cache = createCache(createConfig(2, 4, 64, 32, 2));
        int id = cache->allocateSequence(2).value();
        auto H = [](uintptr_t a) { return reinterpret_cast<const half *>(a); };
        const int8_t *w = reinterpret_cast<const int8_t *>(uintptr_t(256));
        half *q = reinterpret_cast<half *>(uintptr_t(256));
        auto call = [&](int layer, const half *x, int hidden, const half *sk, int group, std::vector<int> ids) {
            return cache->projectQKVAppend(layer, x, hidden, w, H(256), w, sk, w, H(256), group, ids, q);
        };
        auto has = [](const Result<void> &r, const char *s) {
            return r.isErr() && r.error().find(s) != std::string::npos;
        };
        EXPECT(has(call(2, H(256), 256, H(256), 32, {id}), "Invalid layer_idx"));
        EXPECT(has(call(0, nullptr, 256, H(256), 32, {id}), "input is null"));
        EXPECT(has(call(0, H(256), 200, H(256), 32, {id}), "supported shapes"));
        EXPECT(has(call(0, H(256), 256, H(256), 8, {id}), "supported shapes"));
        EXPECT(has(call(0, H(256), 256, H(258), 32, {id}), "aligned"));
        EXPECT(has(call(0, H(256), 256, H(256), 32, {id + 7}), "not found"));
        EXPECT(has(call(0, H(256), 256, H(256), 32, {id, id}), "duplicate"));
        if (!g_gpu) EXPECT(has(call(0, H(256), 256, H(256), 32, {id}), "no CUDA device"));
        EXPECT(cache->getSeqLen(id) == 0);
        // the packed entry: the same checks under its own name
        auto packed = cache->projectQKVAppendPacked(0, H(256), 200, w, H(256), w, H(256), w, H(256), 32, {id}, q);
        EXPECT(has(packed, "projectQKVAppendPacked") && has(packed, "supported shapes"));
        EXPECT(has(KVCacheManager::packQKVWeight(nullptr, 256, 128, const_cast<int8_t *>(w)), "null"));
        EXPECT(has(KVCacheManager::packQKVWeight(w, 256, 96, reinterpret_cast<int8_t *>(uintptr_t(1) << 24)),
                   "multiples of 128"));
    });
    run("ResultMapAndFlatMap", [] {  // the reference's tests/test_cuda_utils.cpp:46,53 use them
        auto doubled = Result<int>::ok(21).map([](int x) { return 2 * x; });
        EXPECT(doubled.isOk() && doubled.value() == 42);
        auto failed = Result<int>::err("boom").map([](int x) { return x + 1; });
        EXPECT(failed.isErr() && failed.error() == "boom");
        auto chained = Result<int>::ok(5).flatMap([](int x) {
            return x > 3 ? Result<std::string>::ok(std::to_string(x)) : Result<std::string>::err("small");
        });
        EXPECT(chained.isOk() && chained.value() == "5");
        auto stopped = Result<int>::ok(1).flatMap([](int x) {
            return x > 3 ? Result<std::string>::ok("big") : Result<std::string>::err("small");
        });
        EXPECT(stopped.isErr() && stopped.error() == "small");
    });
    run("ReferenceConfigCreatesMhaPagedCache", [] {  // create(const KVCacheConfig &)
        KVCacheConfig base;
        base.num_layers = 2;
        base.num_heads = 4;
        base.head_dim = 64;
        base.max_seq_len = 100;
        base.max_batch_size = 3;
        PagedKVCacheConfig paged(base);
        paged.backend = g_gpu ? TL_BACKEND_CUDA : TL_BACKEND_HOST_BOOKKEEPING;
        auto cache = createCache(paged);
        EXPECT(cache->getConfig().num_heads == 4 && cache->getConfig().max_batch_size == 3);
        EXPECT(cache->getPagedConfig().block_size == 16 && !cache->getPagedConfig().rope_on_append);
        EXPECT(cache->getTotalMemory() > 0);
        if (g_gpu) {  // the five-field reference config alone: CUDA backend defaults
            auto r = KVCacheManager::create(base);
            EXPECT(r.isOk());
            EXPECT(r.value()->getPagedConfig().num_q_heads == 0);
        }
    });
    if (g_gpu) {
        run("KVCacheAppendRetrieve", [] {  // tests/test_transformer.cu:141-194
            auto config = createConfig(2, 4, 32, 64, 2);
            auto cache = createCache(config);
            int id = cache->allocateSequence(32).value();
            const int n = 4;
            const size_t elems = (size_t)n * config.num_heads * config.head_dim;
            std::vector<half> hk(elems), hv(elems);
            for (size_t i = 0; i < elems; ++i) {
                hk[i] = __float2half((float)((i * 37) % 101) / 50.0f - 1.0f);
                hv[i] = __float2half((float)((i * 53) % 97) / 48.0f - 1.0f);
            }
            half *dk = nullptr, *dv = nullptr;
            cudaMalloc(&dk, elems * sizeof(half));
            cudaMalloc(&dv, elems * sizeof(half));
            cudaMemcpy(dk, hk.data(), elems * sizeof(half), cudaMemcpyHostToDevice);
            cudaMemcpy(dv, hv.data(), elems * sizeof(half), cudaMemcpyHostToDevice);
            EXPECT(cache->appendKV(id, 0, dk, dv, n).isOk());
            EXPECT(cache->syncCheck().isOk());
            EXPECT(cache->getSeqLen(id) == 0);
            EXPECT(cache->advanceSeqLen(id, n).isOk());
            auto [kc, vc] = cache->getCache(id, 0);
            EXPECT(kc && vc);
            std::vector<half> rk(elems), rv(elems);
            cudaMemcpy(rk.data(), kc, elems * sizeof(half), cudaMemcpyDeviceToHost);
            cudaMemcpy(rv.data(), vc, elems * sizeof(half), cudaMemcpyDeviceToHost);
            EXPECT(std::memcmp(rk.data(), hk.data(), elems * sizeof(half)) == 0);
            EXPECT(std::memcmp(rv.data(), hv.data(), elems * sizeof(half)) == 0);
            cudaFree(dk);
            cudaFree(dv);
        });
    }
    std::printf("%d passed, %d failed (%s backend)\n", g_passed, g_failed,
                g_gpu ? "cuda" : "bookkeeping");
    return g_failed == 0 ? 0 : 1;
}
