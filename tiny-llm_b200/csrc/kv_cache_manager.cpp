// tiny_llm::KVCacheManager: the reference's C++ API
// (include/tiny_llm/kv_cache.h:24-111) as a thin layer over the C-ABI.
// Compiled by the user of the facade with the user's include paths, so that
// Result<T> and KVCacheConfig are the ones the rest of that build sees (the
// tiny-llm engine's own, or tllm_result.h's standalone); libtllm_kv.so
// carries only the C-ABI.
#include "tiny_llm/kv_cache.h"

namespace tiny_llm {

Result<std::unique_ptr<KVCacheManager>> KVCacheManager::create(const KVCacheConfig &config) {
    return create(PagedKVCacheConfig(config));
}

Result<std::unique_ptr<KVCacheManager>> KVCacheManager::create(const PagedKVCacheConfig &config) {
    tl_config c;
    tl_config_init(&c);
    c.num_layers = config.num_layers;
    c.num_kv_heads = config.num_heads;
    c.head_dim = config.head_dim;
    c.max_seq_len = config.max_seq_len;
    c.max_batch_size = config.max_batch_size;
    c.block_size = config.block_size;
    c.num_blocks = config.num_blocks;
    c.num_q_heads = config.num_q_heads;
    c.rope_theta = config.rope_theta;
    c.rope_on_append = config.rope_on_append ? 1 : 0;
    c.layout = config.layout;
    c.backend = config.backend;
    c.device = config.device;
    tl_cache *h = nullptr;
    const int st = tl_create(&c, &h);
    if (st != TL_OK) return Result<std::unique_ptr<KVCacheManager>>::err(tl_last_error(nullptr));
    std::unique_ptr<KVCacheManager> m(new KVCacheManager(config));
    m->h_ = h;
    return Result<std::unique_ptr<KVCacheManager>>::ok(std::move(m));
}

KVCacheManager::~KVCacheManager() { tl_destroy(h_); }

Result<void> KVCacheManager::status(int code) const {
    if (code == TL_OK) return Result<void>::ok();
    return Result<void>::err(tl_last_error(h_));
}

Result<int> KVCacheManager::allocateSequence(int max_len) {
    int id = -1;
    const int st = tl_allocate_sequence(h_, max_len, &id);
    if (st != TL_OK) return Result<int>::err(tl_last_error(h_));
    return Result<int>::ok(id);
}

Result<void> KVCacheManager::releaseSequence(int seq_id) { return status(tl_release_sequence(h_, seq_id)); }

Result<std::pair<half *, half *>> KVCacheManager::getCacheChecked(int seq_id, int layer_idx) {
    void *k = nullptr, *v = nullptr;
    const int st = tl_get_cache(h_, seq_id, layer_idx, &k, &v);
    if (st != TL_OK) return Result<std::pair<half *, half *>>::err(tl_last_error(h_));
    return Result<std::pair<half *, half *>>::ok({static_cast<half *>(k), static_cast<half *>(v)});
}

std::pair<half *, half *> KVCacheManager::getCache(int seq_id, int layer_idx) {
    auto r = getCacheChecked(seq_id, layer_idx);
    if (r.isErr()) return {nullptr, nullptr};
    return r.value();
}

Result<void> KVCacheManager::appendKV(int seq_id, int layer_idx, const half *new_k,
                                      const half *new_v, int num_tokens, cudaStream_t stream) {
    return status(tl_append_kv(h_, seq_id, layer_idx, new_k, new_v, num_tokens, stream));
}

Result<void> KVCacheManager::advanceSeqLen(int seq_id, int num_tokens) {
    return status(tl_advance_seq_len(h_, seq_id, num_tokens));
}

int KVCacheManager::getSeqLen(int seq_id) const noexcept { return tl_get_seq_len(h_, seq_id); }
bool KVCacheManager::hasSequence(int seq_id) const noexcept { return tl_has_sequence(h_, seq_id) != 0; }
size_t KVCacheManager::getUsedMemory() const noexcept { return tl_used_memory(h_); }
size_t KVCacheManager::getTotalMemory() const noexcept { return tl_total_memory(h_); }
size_t KVCacheManager::getFreeMemory() const noexcept { return tl_free_memory(h_); }
int KVCacheManager::getActiveSequenceCount() const noexcept { return tl_active_sequence_count(h_); }

Result<void> KVCacheManager::reserve(int seq_id, int new_len) { return status(tl_reserve(h_, seq_id, new_len)); }

Result<void> KVCacheManager::appendKVAllLayers(const std::vector<int> &seq_ids, const half *k,
                                               const half *v, cudaStream_t stream) {
    return status(tl_append_kv_all_layers(h_, seq_ids.data(), (int)seq_ids.size(), k, v, stream));
}

Result<void> KVCacheManager::decodeAttention(int layer_idx, const half *q, half *out,
                                             const std::vector<int> &seq_ids, float scale,
                                             cudaStream_t stream) {
    return status(tl_decode_attention(h_, layer_idx, q, out, seq_ids.data(), (int)seq_ids.size(),
                                      scale, stream));
}

Result<void> KVCacheManager::attentionStep(int layer_idx, const half *q, const half *k_new,
                                           const half *v_new, half *out, const std::vector<int> &seq_ids,
                                           float scale, cudaStream_t stream) {
    return status(tl_attention_step(h_, layer_idx, q, k_new, v_new, out, seq_ids.data(),
                                    (int)seq_ids.size(), scale, stream));
}

Result<void> KVCacheManager::prefillAttention(int layer_idx, const half *q, half *out,
                                              const std::vector<int> &seq_ids,
                                              const std::vector<int> &num_tokens, float scale,
                                              cudaStream_t stream) {
    if (seq_ids.size() != num_tokens.size())
        return Result<void>::err("prefillAttention: seq_ids and num_tokens differ in length");
    return status(tl_prefill_attention(h_, layer_idx, q, out, seq_ids.data(), num_tokens.data(),
                                       (int)seq_ids.size(), scale, stream));
}

Result<void> KVCacheManager::projectQKVAppend(int layer_idx, const half *x, int hidden, const int8_t *wq,
                                              const half *sq, const int8_t *wk, const half *sk,
                                              const int8_t *wv, const half *sv, int group_size,
                                              const std::vector<int> &seq_ids, half *q_out,
                                              cudaStream_t stream) {
    return status(tl_project_qkv_append(h_, layer_idx, x, hidden, wq, sq, wk, sk, wv, sv, group_size,
                                        seq_ids.data(), (int)seq_ids.size(), q_out, stream));
}

Result<void> KVCacheManager::projectQKVAppendPacked(int layer_idx, const half *x, int hidden, const int8_t *wq,
                                                    const half *sq, const int8_t *wk, const half *sk,
                                                    const int8_t *wv, const half *sv, int group_size,
                                                    const std::vector<int> &seq_ids, half *q_out,
                                                    cudaStream_t stream) {
    return status(tl_project_qkv_append_packed(h_, layer_idx, x, hidden, wq, sq, wk, sk, wv, sv, group_size,
                                               seq_ids.data(), (int)seq_ids.size(), q_out, stream));
}

Result<void> KVCacheManager::packQKVWeight(const int8_t *w, int hidden, int n, int8_t *packed,
                                           cudaStream_t stream) {
    if (tl_qkv_pack_weight(w, hidden, n, packed, stream) != TL_OK) return Result<void>::err(tl_last_error(nullptr));
    return Result<void>::ok();
}

Result<std::vector<int>> KVCacheManager::getBlockTable(int seq_id) const {
    int n = 0;
    if (tl_get_block_table(h_, seq_id, nullptr, 0, &n) != TL_OK)
        return Result<std::vector<int>>::err("Sequence not found: " + std::to_string(seq_id));
    std::vector<int> t((size_t)n);
    tl_get_block_table(h_, seq_id, t.data(), n, &n);
    return Result<std::vector<int>>::ok(std::move(t));
}

tl_pool_stats KVCacheManager::getPoolStats() const noexcept {
    tl_pool_stats s{};
    tl_get_pool_stats(h_, &s);
    return s;
}

Result<void> KVCacheManager::syncCheck(cudaStream_t stream) { return status(tl_sync_check(h_, stream)); }

}  // namespace tiny_llm
