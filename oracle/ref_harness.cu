// extern "C" harness over the REFERENCE's own public API, compiled together
// with the unmodified reference sources (src/kv_cache.cpp, src/logger.cpp,
// kernels/attention.cu, kernels/w8a16_matmul.cu) into
// oracle/_ref/libtllm_ref.so by Makefile.ref.
//
// TEST / BASELINE INFRASTRUCTURE ONLY: used to generate golden fixtures and
// to time the reference arm of bench.py. It calls, unchanged:
//   tiny_llm::KVCacheManager::create / allocateSequence / appendKV /
//   advanceSeqLen / getCache      (include/tiny_llm/kv_cache.h:24-111)
//   tiny_llm::kernels::attention_decode  (kernels/attention.cuh:15-18)
//   tiny_llm::kernels::w8a16_matmul      (kernels/w8a16_matmul.cuh:22-26)
#include <cuda_runtime.h>

#include <memory>
#include <string>

#include "attention.cuh"
#include "w8a16_matmul.cuh"
#include "tiny_llm/kv_cache.h"

namespace {
thread_local std::string g_err;
}

extern "C" {

const char *ref_last_error(void) { return g_err.c_str(); }

int ref_kv_create(int num_layers, int num_heads, int head_dim, int max_seq_len, int max_batch,
                  void **out) {
    tiny_llm::KVCacheConfig c;
    c.num_layers = num_layers;
    c.num_heads = num_heads;
    c.head_dim = head_dim;
    c.max_seq_len = max_seq_len;
    c.max_batch_size = max_batch;
    auto r = tiny_llm::KVCacheManager::create(c);
    if (r.isErr()) {
        g_err = r.error();
        return -1;
    }
    *out = r.value().release();
    return 0;
}

void ref_kv_destroy(void *h) { delete static_cast<tiny_llm::KVCacheManager *>(h); }

int ref_kv_allocate(void *h, int max_len, int *id) {
    auto r = static_cast<tiny_llm::KVCacheManager *>(h)->allocateSequence(max_len);
    if (r.isErr()) {
        g_err = r.error();
        return -1;
    }
    *id = r.value();
    return 0;
}

int ref_kv_append(void *h, int id, int layer, const void *k, const void *v, int n, void *stream) {
    try {
        auto r = static_cast<tiny_llm::KVCacheManager *>(h)->appendKV(
            id, layer, static_cast<const half *>(k), static_cast<const half *>(v), n,
            static_cast<cudaStream_t>(stream));
        if (r.isErr()) {
            g_err = r.error();
            return -1;
        }
    } catch (const std::exception &e) {  // CUDA_CHECK throws CudaException
        g_err = e.what();
        return -2;
    }
    return 0;
}

int ref_kv_advance(void *h, int id, int n) {
    auto r = static_cast<tiny_llm::KVCacheManager *>(h)->advanceSeqLen(id, n);
    if (r.isErr()) {
        g_err = r.error();
        return -1;
    }
    return 0;
}

int ref_kv_get_cache(void *h, int id, int layer, void **k, void **v) {
    auto p = static_cast<tiny_llm::KVCacheManager *>(h)->getCache(id, layer);
    *k = p.first;
    *v = p.second;
    return (p.first && p.second) ? 0 : -1;
}

// kernels::attention_decode followed by the launch check the reference omits.
int ref_attention_decode(const void *q, const void *k, const void *v, void *o, float scale,
                         int batch, int heads, int seq_len, int head_dim, void *stream) {
    tiny_llm::kernels::attention_decode(static_cast<const half *>(q), static_cast<const half *>(k),
                                        static_cast<const half *>(v), static_cast<half *>(o), scale,
                                        batch, heads, seq_len, head_dim,
                                        static_cast<cudaStream_t>(stream));
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        g_err = cudaGetErrorString(e);
        return (int)e;
    }
    return 0;
}

// kernels::attention_prefill (kernels/attention.cu:131-237) followed by the
// launch check the reference omits; q/k/v/o are [batch][heads][seq][dim].
int ref_attention_prefill(const void *q, const void *k, const void *v, void *o, float scale,
                          int batch, int heads, int seq_len, int head_dim, void *stream) {
    tiny_llm::kernels::attention_prefill(static_cast<const half *>(q), static_cast<const half *>(k),
                                         static_cast<const half *>(v), static_cast<half *>(o), scale,
                                         batch, heads, seq_len, head_dim,
                                         static_cast<cudaStream_t>(stream));
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        g_err = cudaGetErrorString(e);
        return (int)e;
    }
    return 0;
}

int ref_w8a16_matmul(const void *x, const void *w, const void *scales, void *out, int M, int N, int K,
                     int group, void *stream) {
    tiny_llm::kernels::w8a16_matmul(static_cast<const half *>(x), static_cast<const int8_t *>(w),
                                    static_cast<const half *>(scales), static_cast<half *>(out), M, N, K, group,
                                    static_cast<cudaStream_t>(stream));
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        g_err = cudaGetErrorString(e);
        return (int)e;
    }
    return 0;
}

}  // extern "C"
