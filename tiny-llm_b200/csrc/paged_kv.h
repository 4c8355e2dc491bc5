// Host side of the paged KV cache: block-pool allocator, sequences and their
// block tables, and the calls that launch the append / decode kernels.
//
// Replaces the reference's contiguous-slot KVCacheManager
// (src/kv_cache.cpp:8-297): instead of one max_seq_len region per slot, the
// pool is num_blocks fixed-size blocks shared by all sequences; a sequence
// owns a list of blocks (its block table) that grows as tokens are appended
// and returns to the free list on release.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <unordered_map>
#include <vector>

#include "kernels.h"
#include "tllm_kv.h"

namespace tllm {

// Free-list allocator of block ids. LIFO: a released block is the next one
// handed out, which keeps recently used (L2-warm) blocks in circulation.
class BlockPool {
  public:
    explicit BlockPool(long long num_blocks = 0);
    int allocate();               // -1 when empty
    bool release(int block);      // false on double free / out of range
    void permute(uint64_t seed);  // shuffle the free list (ragged benchmarks)
    long long capacity() const { return num_blocks_; }
    long long used() const { return num_blocks_ - (long long)free_.size(); }
    long long free_count() const { return (long long)free_.size(); }
    long long high_water() const { return high_water_; }

  private:
    long long num_blocks_ = 0;
    long long high_water_ = 0;
    std::vector<int> free_;
    std::vector<uint8_t> in_use_;
};

struct Sequence {
    int id = -1;
    int slot = -1;      // row of the device block table
    int max_len = 0;
    int len = 0;        // visible length (getSeqLen)
    int written = 0;    // tokens present: len + appended-but-not-advanced
    std::vector<int> blocks;
};

struct BlockDelta {
    int slot, idx, block;
};

}  // namespace tllm

// The opaque handle of the C-ABI.
struct tl_cache {
    tl_config cfg{};
    bool on_device = false;
    int device = -1;
    int num_sms = 0;

    // geometry
    int bs = 16;
    int max_blocks_per_seq = 0;
    long long block_elems = 0;   // halves in one (layer, K|V, block)
    long long block_bytes = 0;   // bytes of one block id over all layers, K and V
    size_t pool_elems = 0;
    int group = 1;

    // storage (device memory, or host memory for the bookkeeping backend)
    void *pool = nullptr;
    int *block_tables = nullptr;  // [max_batch][max_blocks_per_seq]
    int *err_word = nullptr;
    float *rope_cos = nullptr;
    float *rope_sin = nullptr;
    float *partial = nullptr;
    int *merge_counters = nullptr;  // [kMaxDecodeSeqs][Hkv], zero between launches
    // head-sharded peer gather (one process per GPU, CUDA IPC mappings)
    int peer_rank = -1, peer_world = 0;
    void *peer_region = nullptr;      // [flags (kPeerFlagBytes)][gathered outputs]
    size_t gather_bytes = 0;
    int *peer_done_counter = nullptr;
    void *peer_bases[tllm::kMaxPeers] = {};
    bool peer_opened[tllm::kMaxPeers] = {};
    bool peers_connected = false;
    unsigned long long peer_wait_ns = 0;  // 0: the kernel's built-in limit (10 s)
    size_t partial_floats = 0;
    // fused Q/K/V projection + append: split-K partials and per-tile counters
    float *qkv_partial = nullptr;
    size_t qkv_partial_floats = 0;
    int *qkv_counters = nullptr;
    int qkv_counter_n = 0;
    int max_workers = 0;
    alignas(64) unsigned char tmap[128];

    tllm::BlockPool blocks;
    std::vector<int> free_slots;
    std::unordered_map<int, tllm::Sequence> seqs;
    std::vector<tllm::BlockDelta> pending;
    int next_seq_id = 0;
    long long launches = 0;  // kernels launched by this handle
    std::string last_error;

    tllm::PoolGeom geom() const;
};

namespace tllm {

int set_error(tl_cache *c, int status, const std::string &msg);

}  // namespace tllm
