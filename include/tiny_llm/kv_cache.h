// tiny_llm::KVCacheManager over the B200 paged KV cache (C-ABI tllm_kv.h).
//
// Drop-in for the reference header include/tiny_llm/kv_cache.h (AICL-Lab/
// tiny-llm, :24-111): every signature of the reference class (create /
// allocateSequence / releaseSequence / getCache / getCacheChecked / appendKV /
// advanceSeqLen / getSeqLen / hasSequence / memory statistics /
// getActiveSequenceCount / getConfig), its non-copyable, non-movable
// ownership and its error texts; plus the paged and fused entry points
// (reserve, appendKVAllLayers, decodeAttention, attentionStep,
// prefillAttention, projectQKVAppend, getBlockTable, getPoolStats).
//
// Two ways to build it:
//  - inside the tiny-llm tree (this directory ahead of the engine's include
//    directory, or this file in place of the engine's kv_cache.h): the
//    engine's tiny_llm/types.h supplies KVCacheConfig (types.h:122-128) and
//    its tiny_llm/result.h supplies Result<T>, so the engine's own sources
//    compile against this header unchanged;
//  - standalone (no tiny_llm/types.h on the include path, or
//    TLLM_KV_STANDALONE defined): tllm_result.h supplies Result<T> and the
//    five-field KVCacheConfig is declared here with the reference's defaults.
// Either way PagedKVCacheConfig extends KVCacheConfig with the pool and RoPE
// settings; create(const KVCacheConfig &) takes the paged defaults.
//
// Behavioural differences, by design:
//  - memory is a pool of fixed-size blocks; a sequence takes one block at
//    allocation and more as it grows, so getUsedMemory() counts blocks;
//  - getCache() points at the sequence's first block of the layer, which
//    (token-major layout) holds tokens 0..block_size-1 as [pos][Hkv][D];
//  - CUDA failures are returned as errors instead of thrown.
// The class is defined in tiny-llm_b200/csrc/kv_cache_manager.cpp, which the
// user compiles with the same include paths (the result and config types
// above belong to the user's build); it calls libtllm_kv.so's C-ABI.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <memory>
#include <utility>
#include <vector>

#if !defined(TLLM_KV_STANDALONE) && __has_include("tiny_llm/types.h")
#include "tiny_llm/types.h"  // the engine's KVCacheConfig and Result<T>
#if __has_include("tiny_llm/cuda_utils.h")
#include "tiny_llm/cuda_utils.h"  // included by the header this one replaces
#endif
#define TLLM_KV_ENGINE_TYPES 1
#else
#include "tllm_result.h"
#endif
#include "tllm_kv.h"

namespace tiny_llm {

#ifndef TLLM_KV_ENGINE_TYPES
// Reference KVCacheConfig (include/tiny_llm/types.h:122-128). num_heads is
// the KV-head count, as the reference engine passes it
// (src/inference_engine.cpp:59).
struct KVCacheConfig {
    int num_layers = 32;
    int num_heads = 32;
    int head_dim = 128;
    int max_seq_len = 2048;
    int max_batch_size = 1;
};
#endif

// KVCacheConfig plus the paged pool, query heads and RoPE settings.
struct PagedKVCacheConfig : KVCacheConfig {
    int block_size = 16;
    long long num_blocks = 0;  // 0: max_batch_size * ceil(max_seq_len / block_size)
    int num_q_heads = 0;       // 0: num_heads (MHA)
    float rope_theta = 10000.0f;
    bool rope_on_append = false;
    int layout = TL_LAYOUT_TOKEN_MAJOR;
    int backend = TL_BACKEND_CUDA;
    int device = -1;

    PagedKVCacheConfig() = default;
    explicit PagedKVCacheConfig(const KVCacheConfig &base) : KVCacheConfig(base) {}
};

class KVCacheManager {
  public:
    // The reference factory: a paged pool with the default block size, MHA
    // (query heads = config.num_heads) and no RoPE.
    static Result<std::unique_ptr<KVCacheManager>> create(const KVCacheConfig &config);
    static Result<std::unique_ptr<KVCacheManager>> create(const PagedKVCacheConfig &config);
    ~KVCacheManager();

    KVCacheManager(const KVCacheManager &) = delete;
    KVCacheManager &operator=(const KVCacheManager &) = delete;
    KVCacheManager(KVCacheManager &&) = delete;
    KVCacheManager &operator=(KVCacheManager &&) = delete;

    Result<int> allocateSequence(int max_len);
    Result<void> releaseSequence(int seq_id);
    std::pair<half *, half *> getCache(int seq_id, int layer_idx);
    Result<std::pair<half *, half *>> getCacheChecked(int seq_id, int layer_idx);
    Result<void> appendKV(int seq_id, int layer_idx, const half *new_k, const half *new_v,
                          int num_tokens, cudaStream_t stream = 0);
    Result<void> advanceSeqLen(int seq_id, int num_tokens);
    int getSeqLen(int seq_id) const noexcept;
    bool hasSequence(int seq_id) const noexcept;
    size_t getUsedMemory() const noexcept;
    size_t getTotalMemory() const noexcept;
    size_t getFreeMemory() const noexcept;
    int getActiveSequenceCount() const noexcept;
    const KVCacheConfig &getConfig() const noexcept { return config_; }
    const PagedKVCacheConfig &getPagedConfig() const noexcept { return config_; }

    // Paged / fused additions.
    Result<void> reserve(int seq_id, int new_len);
    Result<void> appendKVAllLayers(const std::vector<int> &seq_ids, const half *k, const half *v,
                                   cudaStream_t stream = 0);
    // Replacement of kernels::attention_decode for TransformerLayer::attention.
    Result<void> decodeAttention(int layer_idx, const half *q, half *out,
                                 const std::vector<int> &seq_ids, float scale = 0.0f,
                                 cudaStream_t stream = 0);
    // The decode branch of TransformerLayer::attention for a batch: appendKV
    // of each sequence's new token in layer_idx, then attention over len + 1
    // tokens (Q rotated like K when the cache rotates on append).
    Result<void> attentionStep(int layer_idx, const half *q, const half *k_new, const half *v_new,
                               half *out, const std::vector<int> &seq_ids, float scale = 0.0f,
                               cudaStream_t stream = 0);
    // Replacement of kernels::attention_prefill: causal attention of each
    // sequence's last num_tokens[i] written tokens over the paged cache.
    Result<void> prefillAttention(int layer_idx, const half *q, half *out, const std::vector<int> &seq_ids,
                                  const std::vector<int> &num_tokens, float scale = 0.0f,
                                  cudaStream_t stream = 0);
    // The decode step's Q/K/V projections (W8A16, weights in the reference's
    // [K][N] int8 + [K/group][N] fp16-scale layout) with K and V written
    // straight into the cache at each sequence's current length and Q into
    // q_out (rotated like K when the cache rotates on append).
    Result<void> projectQKVAppend(int layer_idx, const half *x, int hidden, const int8_t *wq, const half *sq,
                                  const int8_t *wk, const half *sk, const int8_t *wv, const half *sv,
                                  int group_size, const std::vector<int> &seq_ids, half *q_out,
                                  cudaStream_t stream = 0);
    // The same from weights repacked once by packQKVWeight (tile-blocked,
    // each 64-row block of a 128-column tile 8 KB contiguous).
    Result<void> projectQKVAppendPacked(int layer_idx, const half *x, int hidden, const int8_t *wq,
                                        const half *sq, const int8_t *wk, const half *sk, const int8_t *wv,
                                        const half *sv, int group_size, const std::vector<int> &seq_ids,
                                        half *q_out, cudaStream_t stream = 0);
    // Repacks one int8 weight [hidden][n] into `packed` (hidden * n bytes of
    // device memory) for projectQKVAppendPacked; asynchronous on `stream`.
    static Result<void> packQKVWeight(const int8_t *w, int hidden, int n, int8_t *packed, cudaStream_t stream = 0);
    Result<std::vector<int>> getBlockTable(int seq_id) const;
    tl_pool_stats getPoolStats() const noexcept;
    Result<void> syncCheck(cudaStream_t stream = 0);
    tl_cache *handle() noexcept { return h_; }

  private:
    explicit KVCacheManager(const PagedKVCacheConfig &config) : config_(config) {}
    Result<void> status(int code) const;

    PagedKVCacheConfig config_;
    tl_cache *h_ = nullptr;
};

}  // namespace tiny_llm
