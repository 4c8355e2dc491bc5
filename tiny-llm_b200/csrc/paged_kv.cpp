// Host side of the paged KV cache and the extern "C" entry points of
// include/tllm_kv.h. Each entry point names the reference function it
// replaces; error texts keep the reference's substrings ("exhausted",
// "not found", "overflow", "Invalid max_len", "Invalid layer_idx", "is null",
// "must be positive") so callers that match on them keep working.
#include "paged_kv.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <numeric>
#include <random>
#include <unordered_set>

#include <cuda_runtime.h>

using tllm::BlockDelta;
using tllm::Sequence;

namespace {

thread_local std::string g_create_error;
int g_fail_alloc_countdown = 0;  // test hook: n-th allocation from now fails

constexpr const char *kVersion = "tllm_kv 0.1.0 (sm_100a)";

class DeviceGuard {
  public:
    explicit DeviceGuard(const tl_cache *c) {
        if (c && c->on_device && c->device >= 0) {
            if (cudaGetDevice(&prev_) == cudaSuccess && prev_ != c->device) {
                cudaSetDevice(c->device);
                restore_ = true;
            }
        }
    }
    ~DeviceGuard() {
        if (restore_) cudaSetDevice(prev_);
    }

  private:
    int prev_ = -1;
    bool restore_ = false;
};

bool injected_alloc_failure() {
    if (g_fail_alloc_countdown > 0) {
        if (--g_fail_alloc_countdown == 0) return true;
    }
    return false;
}

// Device allocation for the CUDA backend, host allocation for the
// bookkeeping backend. Returns a cudaError_t-like code (0 = ok).
int storage_alloc(tl_cache *c, void **p, size_t bytes, std::string *why) {
    *p = nullptr;
    if (bytes == 0) bytes = 16;
    if (injected_alloc_failure()) {
        *why = "injected allocation failure";
        return 1;
    }
    if (c->on_device) {
        cudaError_t e = cudaMalloc(p, bytes);
        if (e != cudaSuccess) {
            *why = cudaGetErrorString(e);
            cudaGetLastError();
            *p = nullptr;
            return 1;
        }
        e = cudaMemset(*p, 0, bytes);
        if (e != cudaSuccess) {
            *why = cudaGetErrorString(e);
            cudaFree(*p);
            *p = nullptr;
            return 1;
        }
        return 0;
    }
    *p = std::calloc(1, bytes);
    if (!*p) {
        *why = "host calloc failed";
        return 1;
    }
    return 0;
}

void storage_free(tl_cache *c, void *p) {
    if (!p) return;
    if (c->on_device)
        cudaFree(p);
    else
        std::free(p);
}

int ceil_div(long long a, long long b) { return (int)((a + b - 1) / b); }

bool decode_geometry_supported(const tl_cache *c) {
    int D = c->cfg.head_dim;
    return (D == 64 || D == 128 || D == 256) && (c->bs == 16 || c->bs == 32) && c->group >= 1 &&
           c->group <= 8;
}

}  // namespace

namespace tllm {

// ------------------------------------------------------------ BlockPool --

BlockPool::BlockPool(long long num_blocks) : num_blocks_(num_blocks) {
    free_.resize((size_t)num_blocks);
    // LIFO stack: pop_back hands out 0, 1, 2, ... on a fresh pool.
    for (long long i = 0; i < num_blocks; ++i) free_[(size_t)i] = (int)(num_blocks - 1 - i);
    in_use_.assign((size_t)num_blocks, 0);
}

int BlockPool::allocate() {
    if (free_.empty()) return -1;
    int b = free_.back();
    free_.pop_back();
    in_use_[(size_t)b] = 1;
    high_water_ = std::max(high_water_, used());
    return b;
}

bool BlockPool::release(int block) {
    if (block < 0 || block >= num_blocks_ || !in_use_[(size_t)block]) return false;
    in_use_[(size_t)block] = 0;
    free_.push_back(block);
    return true;
}

void BlockPool::permute(uint64_t seed) {
    std::mt19937_64 rng(seed);
    std::shuffle(free_.begin(), free_.end(), rng);
}

int set_error(tl_cache *c, int status, const std::string &msg) {
    if (c) c->last_error = msg;
    return status;
}

}  // namespace tllm

tllm::PoolGeom tl_cache::geom() const {
    tllm::PoolGeom g{};
    g.pool = pool;
    g.num_blocks = cfg.num_blocks;
    g.num_layers = cfg.num_layers;
    g.num_kv_heads = cfg.num_kv_heads;
    g.head_dim = cfg.head_dim;
    g.block_size = bs;
    g.head_major = cfg.layout == TL_LAYOUT_HEAD_MAJOR ? 1 : 0;
    g.bt_stride = max_blocks_per_seq;
    g.block_tables = block_tables;
    g.err = err_word;
    return g;
}

namespace {

using tllm::set_error;

Sequence *find_seq(tl_cache *c, int id) {
    auto it = c->seqs.find(id);
    return it == c->seqs.end() ? nullptr : &it->second;
}
const Sequence *find_seq(const tl_cache *c, int id) {
    auto it = c->seqs.find(id);
    return it == c->seqs.end() ? nullptr : &it->second;
}

std::string layer_error(const tl_cache *c, const char *ctx, int layer) {
    return std::string(ctx) + ": Invalid layer_idx: " + std::to_string(layer) +
           " (valid range: 0-" + std::to_string(c->cfg.num_layers - 1) + ")";
}

// Grows a sequence's block list to cover `ntokens` tokens. On failure the
// blocks taken by this call are returned and the queued table updates undone.
int ensure_blocks(tl_cache *c, Sequence &s, long long ntokens, size_t pending_mark,
                  std::vector<std::pair<Sequence *, int>> *undo) {
    int need = ceil_div(ntokens, c->bs);
    while ((int)s.blocks.size() < need) {
        int b = c->blocks.allocate();
        if (b < 0) {
            return set_error(c, TL_ERR_EXHAUSTED,
                             "KV cache exhausted: no free blocks available. Used: " +
                                 std::to_string(c->blocks.used() * c->block_bytes) +
                                 " bytes, Total: " +
                                 std::to_string(c->blocks.capacity() * c->block_bytes) + " bytes");
        }
        c->pending.push_back({s.slot, (int)s.blocks.size(), b});
        s.blocks.push_back(b);
        if (undo) undo->push_back({&s, b});
    }
    (void)pending_mark;
    return TL_OK;
}

void rollback(tl_cache *c, size_t pending_mark, std::vector<std::pair<Sequence *, int>> &undo) {
    for (auto it = undo.rbegin(); it != undo.rend(); ++it) {
        it->first->blocks.pop_back();
        c->blocks.release(it->second);
    }
    c->pending.resize(pending_mark);
    undo.clear();
}

// Moves up to kMaxDeltas queued block-table updates into the arrays of a
// launch argument block.
template <typename Args>
void take_deltas(tl_cache *c, Args &a, size_t &cursor) {
    int n = 0;
    while (cursor < c->pending.size() && n < tllm::kMaxDeltas) {
        const BlockDelta &d = c->pending[cursor++];
        a.delta_slot[n] = d.slot;
        a.delta_idx[n] = d.idx;
        a.delta_block[n] = d.block;
        ++n;
    }
    a.ndeltas = n;
}

int cuda_fail(tl_cache *c, cudaError_t e, const char *what) {
    cudaGetLastError();
    return set_error(c, TL_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

// Applies every queued block-table update with stand-alone kernels.
int flush_deltas(tl_cache *c, cudaStream_t stream) {
    size_t cursor = 0;
    while (cursor < c->pending.size()) {
        tllm::DeltaArgs a{};
        a.block_tables = c->block_tables;
        a.bt_stride = c->max_blocks_per_seq;
        take_deltas(c, a, cursor);
        cudaError_t e = tllm::launch_apply_deltas(a, stream);
        if (e != cudaSuccess) return cuda_fail(c, e, "block-table update launch failed");
        ++c->launches;
    }
    c->pending.clear();
    return TL_OK;
}

// Launches append kernels for rows [row_block, row_pos] over the given layers.
int launch_rows(tl_cache *c, const std::vector<int> &row_block, const std::vector<int> &row_pos,
                const void *k, const void *v, int layer0, int num_layers, long long layer_stride,
                long long row_stride, cudaStream_t stream) {
    size_t cursor = 0;
    const size_t nrows = row_block.size();
    for (size_t r0 = 0; r0 < nrows; r0 += tllm::kMaxAppendRows) {
        int n = (int)std::min<size_t>(tllm::kMaxAppendRows, nrows - r0);
        tllm::AppendArgs a{};
        a.g = c->geom();
        a.k = static_cast<const uint16_t *>(k) + r0 * row_stride;
        a.v = static_cast<const uint16_t *>(v) + r0 * row_stride;
        a.rope_cos = c->cfg.rope_on_append ? c->rope_cos : nullptr;
        a.rope_sin = c->cfg.rope_on_append ? c->rope_sin : nullptr;
        a.rope_max_pos = c->cfg.max_seq_len;
        a.layer0 = layer0;
        a.num_layers = num_layers;
        a.nrows = n;
        a.src_layer_stride = layer_stride;
        a.src_row_stride = row_stride;
        take_deltas(c, a, cursor);
        for (int j = 0; j < n; ++j) {
            a.row_block[j] = row_block[r0 + j];
            a.row_pos[j] = row_pos[r0 + j];
        }
        cudaError_t e = tllm::launch_append(a, stream);
        if (e != cudaSuccess) return cuda_fail(c, e, "append launch failed");
        ++c->launches;
    }
    // Updates that did not fit in the row launches.
    if (cursor < c->pending.size()) {
        c->pending.erase(c->pending.begin(), c->pending.begin() + (long)cursor);
        return flush_deltas(c, stream);
    }
    c->pending.clear();
    return TL_OK;
}

// One new token per sequence (at its current length) for layers
// [layer0, layer0 + num_layers): k/v are [num_layers][num_seqs][Hkv][D].
// Validates every sequence first; block growth is rolled back on failure.
int append_token_rows(tl_cache *c, const char *ctx, const int *seq_ids, int num_seqs, const void *k,
                      const void *v, int layer0, int num_layers, cudaStream_t stream) {
    if (num_seqs < 0) return set_error(c, TL_ERR_INVALID_ARG, std::string(ctx) + ": num_seqs must be >= 0");
    if (num_seqs == 0) return TL_OK;
    if (!seq_ids) return set_error(c, TL_ERR_INVALID_ARG, "seq_ids is null");
    if (!k) return set_error(c, TL_ERR_INVALID_ARG, "new_k is null");
    if (!v) return set_error(c, TL_ERR_INVALID_ARG, "new_v is null");
    std::vector<Sequence *> ss((size_t)num_seqs);
    std::unordered_set<int> seen;
    for (int i = 0; i < num_seqs; ++i) {
        Sequence *s = find_seq(c, seq_ids[i]);
        if (!s)
            return set_error(c, TL_ERR_NOT_FOUND,
                             std::string(ctx) + ": sequence not found: " + std::to_string(seq_ids[i]));
        if (!seen.insert(seq_ids[i]).second)
            return set_error(c, TL_ERR_INVALID_ARG,
                             std::string(ctx) + ": duplicate sequence id " + std::to_string(seq_ids[i]));
        if (s->len + 1 > s->max_len)
            return set_error(c, TL_ERR_OVERFLOW,
                             std::string(ctx) + ": cache overflow. seq " + std::to_string(seq_ids[i]) +
                                 " Current: " + std::to_string(s->len) +
                                 ", appending: 1, max: " + std::to_string(s->max_len));
        ss[(size_t)i] = s;
    }
    if (!c->on_device)
        return set_error(c, TL_ERR_NO_DEVICE, std::string(ctx) + ": handle has no CUDA device (bookkeeping backend)");
    DeviceGuard guard(c);
    std::vector<std::pair<Sequence *, int>> undo;
    size_t mark = c->pending.size();
    std::vector<int> rb((size_t)num_seqs), rp((size_t)num_seqs);
    for (int i = 0; i < num_seqs; ++i) {
        Sequence &s = *ss[(size_t)i];
        int st = ensure_blocks(c, s, (long long)s.len + 1, mark, &undo);
        if (st != TL_OK) {
            rollback(c, mark, undo);
            return st;
        }
        rp[(size_t)i] = s.len;
        rb[(size_t)i] = s.blocks[(size_t)(s.len / c->bs)];
    }
    const long long row = (long long)c->cfg.num_kv_heads * c->cfg.head_dim;
    int st = launch_rows(c, rb, rp, k, v, layer0, num_layers, row * num_seqs, row, stream);
    if (st != TL_OK) return st;
    for (Sequence *s : ss) s->written = std::max(s->written, s->len + 1);
    return TL_OK;
}

}  // namespace

extern "C" {

void tl_config_init(tl_config *cfg) {
    if (!cfg) return;
    std::memset(cfg, 0, sizeof(*cfg));
    cfg->num_layers = 32;
    cfg->num_kv_heads = 32;
    cfg->head_dim = 128;
    cfg->max_seq_len = 2048;
    cfg->max_batch_size = 1;
    cfg->block_size = 16;
    cfg->num_blocks = 0;
    cfg->num_q_heads = 0;
    cfg->rope_theta = 10000.0f;
    cfg->rope_on_append = 0;
    cfg->layout = TL_LAYOUT_TOKEN_MAJOR;
    cfg->backend = TL_BACKEND_CUDA;
    cfg->device = -1;
}

const char *tl_version(void) { return kVersion; }

const char *tl_status_name(int s) {
    switch (s) {
    case TL_OK: return "TL_OK";
    case TL_ERR_INVALID_ARG: return "TL_ERR_INVALID_ARG";
    case TL_ERR_NOT_FOUND: return "TL_ERR_NOT_FOUND";
    case TL_ERR_EXHAUSTED: return "TL_ERR_EXHAUSTED";
    case TL_ERR_OVERFLOW: return "TL_ERR_OVERFLOW";
    case TL_ERR_CUDA: return "TL_ERR_CUDA";
    case TL_ERR_NO_DEVICE: return "TL_ERR_NO_DEVICE";
    case TL_ERR_UNSUPPORTED: return "TL_ERR_UNSUPPORTED";
    case TL_ERR_DEVICE_FAULT: return "TL_ERR_DEVICE_FAULT";
    default: return "TL_ERR_UNKNOWN";
    }
}

const char *tl_last_error(const tl_cache *c) {
    return c ? c->last_error.c_str() : g_create_error.c_str();
}

int tl_debug_inject_alloc_failure(int nth) {
    g_fail_alloc_countdown = nth > 0 ? nth : 0;
    return TL_OK;
}

void tl_rope_table(float *cos_t, float *sin_t, int max_pos, int head_dim, float theta) {
    const int half = head_dim / 2;
    for (int i = 0; i < half; ++i) {
        const double freq = std::pow((double)theta, -2.0 * (double)i / (double)head_dim);
        for (int p = 0; p < max_pos; ++p) {
            const double a = (double)p * freq;
            cos_t[(size_t)p * half + i] = (float)std::cos(a);
            sin_t[(size_t)p * half + i] = (float)std::sin(a);
        }
    }
}

// KVCacheManager::create (reference src/kv_cache.cpp:8-59).
int tl_create(const tl_config *cfg_in, tl_cache **out) {
    g_create_error.clear();
    if (!out || !cfg_in) {
        g_create_error = "tl_create: null argument";
        return TL_ERR_INVALID_ARG;
    }
    *out = nullptr;
    tl_config cfg = *cfg_in;
    if (cfg.num_layers <= 0 || cfg.num_kv_heads <= 0 || cfg.head_dim <= 0 ||
        cfg.max_seq_len <= 0 || cfg.max_batch_size <= 0) {
        g_create_error = "KVCacheManager: invalid configuration parameters";
        return TL_ERR_INVALID_ARG;
    }
    if (cfg.block_size == 0) cfg.block_size = 16;
    if (cfg.block_size != 16 && cfg.block_size != 32) {
        g_create_error = "KVCacheManager: invalid configuration parameters (block_size must be 16 or 32)";
        return TL_ERR_INVALID_ARG;
    }
    if (cfg.num_q_heads == 0) cfg.num_q_heads = cfg.num_kv_heads;
    if (cfg.num_q_heads < cfg.num_kv_heads || cfg.num_q_heads % cfg.num_kv_heads != 0) {
        g_create_error = "KVCacheManager: invalid configuration parameters (num_q_heads must be a "
                         "multiple of num_kv_heads)";
        return TL_ERR_INVALID_ARG;
    }
    if (cfg.rope_on_append && (cfg.head_dim % 2 != 0 || !(cfg.rope_theta > 0.0f))) {
        g_create_error = "KVCacheManager: invalid configuration parameters (RoPE needs an even "
                         "head_dim and rope_theta > 0)";
        return TL_ERR_INVALID_ARG;
    }
    if (cfg.layout != TL_LAYOUT_TOKEN_MAJOR && cfg.layout != TL_LAYOUT_HEAD_MAJOR) {
        g_create_error = "KVCacheManager: invalid configuration parameters (layout)";
        return TL_ERR_INVALID_ARG;
    }
    if (cfg.backend != TL_BACKEND_CUDA && cfg.backend != TL_BACKEND_HOST_BOOKKEEPING) {
        g_create_error = "KVCacheManager: invalid configuration parameters (backend)";
        return TL_ERR_INVALID_ARG;
    }

    const int bs = cfg.block_size;
    const long long max_blocks_per_seq = ((long long)cfg.max_seq_len + bs - 1) / bs;
    if (cfg.num_blocks < 0) {
        g_create_error = "KVCacheManager: invalid configuration parameters (num_blocks)";
        return TL_ERR_INVALID_ARG;
    }
    if (cfg.num_blocks == 0) cfg.num_blocks = (long long)cfg.max_batch_size * max_blocks_per_seq;

    // Size arithmetic with overflow checks (reference kv_cache.cpp:19-34).
    const unsigned long long block_elems =
        (unsigned long long)bs * (unsigned long long)cfg.num_kv_heads * (unsigned long long)cfg.head_dim;
    const unsigned long long layers2 = 2ull * (unsigned long long)cfg.num_layers;
    const unsigned long long lim = (unsigned long long)SIZE_MAX / 2ull;
    if (block_elems == 0 || block_elems > lim / layers2 ||
        (unsigned long long)cfg.num_blocks > lim / (layers2 * block_elems) ||
        cfg.num_blocks > 0x7fffffffLL) {
        g_create_error = "KVCacheManager: memory size overflow";
        return TL_ERR_OVERFLOW;
    }
    // Row coordinates of the TMA tensor map are int32.
    const unsigned long long rows =
        layers2 * (unsigned long long)cfg.num_blocks *
        (unsigned long long)(cfg.layout == TL_LAYOUT_HEAD_MAJOR ? cfg.num_kv_heads : bs);
    if (rows >= 0x7fffffffull) {
        g_create_error = "KVCacheManager: pool size overflow (more than 2^31 rows)";
        return TL_ERR_OVERFLOW;
    }

    auto c = new tl_cache();
    c->cfg = cfg;
    c->bs = bs;
    c->max_blocks_per_seq = (int)max_blocks_per_seq;
    c->block_elems = (long long)block_elems;
    c->block_bytes = (long long)(block_elems * layers2 * 2ull);
    c->pool_elems = (size_t)(block_elems * layers2 * (unsigned long long)cfg.num_blocks);
    c->group = cfg.num_q_heads / cfg.num_kv_heads;
    c->on_device = cfg.backend == TL_BACKEND_CUDA;

    if (c->on_device) {
        int ndev = 0;
        cudaError_t e = cudaGetDeviceCount(&ndev);
        if (e != cudaSuccess || ndev == 0) {
            cudaGetLastError();
            g_create_error = std::string("KVCacheManager: no CUDA device available (") +
                             cudaGetErrorString(e) + ")";
            delete c;
            return TL_ERR_NO_DEVICE;
        }
        if (cfg.device >= 0) {
            if (cfg.device >= ndev || cudaSetDevice(cfg.device) != cudaSuccess) {
                cudaGetLastError();
                g_create_error = "KVCacheManager: invalid device ordinal " + std::to_string(cfg.device);
                delete c;
                return TL_ERR_INVALID_ARG;
            }
        }
        cudaGetDevice(&c->device);
        cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, c->device);
    }

    std::string why;
    auto fail = [&](int status, const std::string &msg) {
        g_create_error = msg;
        tl_destroy(c);
        return status;
    };
    if (storage_alloc(c, &c->pool, c->pool_elems * 2, &why))
        return fail(TL_ERR_CUDA, "KVCacheManager: cudaMalloc failed: " + why);
    void *p = nullptr;
    if (storage_alloc(c, &p, (size_t)cfg.max_batch_size * c->max_blocks_per_seq * sizeof(int), &why))
        return fail(TL_ERR_CUDA, "KVCacheManager: block-table allocation failed: " + why);
    c->block_tables = static_cast<int *>(p);
    if (storage_alloc(c, &p, 64, &why))
        return fail(TL_ERR_CUDA, "KVCacheManager: error-word allocation failed: " + why);
    c->err_word = static_cast<int *>(p);

    if (cfg.rope_on_append) {
        const size_t n = (size_t)cfg.max_seq_len * (cfg.head_dim / 2);
        std::vector<float> cs(n), sn(n);
        tl_rope_table(cs.data(), sn.data(), cfg.max_seq_len, cfg.head_dim, cfg.rope_theta);
        if (storage_alloc(c, &p, n * 4, &why))
            return fail(TL_ERR_CUDA, "KVCacheManager: RoPE table allocation failed: " + why);
        c->rope_cos = static_cast<float *>(p);
        if (storage_alloc(c, &p, n * 4, &why))
            return fail(TL_ERR_CUDA, "KVCacheManager: RoPE table allocation failed: " + why);
        c->rope_sin = static_cast<float *>(p);
        if (c->on_device) {
            if (cudaMemcpy(c->rope_cos, cs.data(), n * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
                cudaMemcpy(c->rope_sin, sn.data(), n * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
                cudaGetLastError();
                return fail(TL_ERR_CUDA, "KVCacheManager: RoPE table upload failed");
            }
        } else {
            std::memcpy(c->rope_cos, cs.data(), n * 4);
            std::memcpy(c->rope_sin, sn.data(), n * 4);
        }
    }

    if (c->on_device && decode_geometry_supported(c)) {
        c->max_workers = tllm::decode_max_workers(c->device, cfg.head_dim, bs);
        if (c->max_workers <= 0) return fail(TL_ERR_CUDA, "KVCacheManager: decode kernel occupancy query failed");
        c->partial_floats =
            (size_t)c->max_workers * 2 * (size_t)c->group * (size_t)tllm::partial_row_floats(cfg.head_dim);
        if (storage_alloc(c, &p, c->partial_floats * 4, &why))
            return fail(TL_ERR_CUDA, "KVCacheManager: split scratch allocation failed: " + why);
        c->partial = static_cast<float *>(p);
        if (storage_alloc(c, &p, (size_t)tllm::kMaxDecodeSeqs * cfg.num_kv_heads * sizeof(int), &why))
            return fail(TL_ERR_CUDA, "KVCacheManager: merge counter allocation failed: " + why);
        c->merge_counters = static_cast<int *>(p);
        cudaError_t e = tllm::encode_pool_tensor_map(c->geom(), c->tmap);
        if (e != cudaSuccess)
            return fail(TL_ERR_CUDA, std::string("KVCacheManager: tensor map encode failed: ") +
                                         cudaGetErrorString(e));
    }

    c->blocks = tllm::BlockPool(cfg.num_blocks);
    c->free_slots.resize((size_t)cfg.max_batch_size);
    for (int i = 0; i < cfg.max_batch_size; ++i) c->free_slots[(size_t)i] = cfg.max_batch_size - 1 - i;
    *out = c;
    return TL_OK;
}

void tl_destroy(tl_cache *c) {
    if (!c) return;
    {
        DeviceGuard guard(c);
        if (c->on_device) cudaDeviceSynchronize();
        storage_free(c, c->pool);
        storage_free(c, c->block_tables);
        storage_free(c, c->err_word);
        storage_free(c, c->rope_cos);
        storage_free(c, c->rope_sin);
        storage_free(c, c->partial);
        storage_free(c, c->merge_counters);
        storage_free(c, c->qkv_partial);
        storage_free(c, c->qkv_counters);
        for (int r = 0; r < tllm::kMaxPeers; ++r)
            if (c->peer_opened[r]) cudaIpcCloseMemHandle(c->peer_bases[r]);
        storage_free(c, c->peer_region);
        storage_free(c, c->peer_done_counter);
    }
    delete c;
}

// allocateSequence (reference src/kv_cache.cpp:91-119).
int tl_allocate_sequence(tl_cache *c, int max_len, int *seq_id) {
    if (!c || !seq_id) return set_error(c, TL_ERR_INVALID_ARG, "allocateSequence: null argument");
    if (max_len <= 0 || max_len > c->cfg.max_seq_len)
        return set_error(c, TL_ERR_INVALID_ARG,
                         "Invalid max_len: " + std::to_string(max_len) + " (must be 1-" +
                             std::to_string(c->cfg.max_seq_len) + ")");
    if (c->free_slots.empty())
        return set_error(c, TL_ERR_EXHAUSTED,
                         "KV cache exhausted: no free slots available. Used: " +
                             std::to_string(tl_used_memory(c)) + " bytes, Total: " +
                             std::to_string(tl_total_memory(c)) + " bytes");
    Sequence s;
    s.slot = c->free_slots.back();
    s.max_len = max_len;
    std::vector<std::pair<Sequence *, int>> undo;
    size_t mark = c->pending.size();
    int st = ensure_blocks(c, s, 1, mark, &undo);
    if (st != TL_OK) {
        rollback(c, mark, undo);
        return st;
    }
    c->free_slots.pop_back();
    s.id = c->next_seq_id++;
    *seq_id = s.id;
    c->seqs.emplace(s.id, std::move(s));
    return TL_OK;
}

// releaseSequence (reference src/kv_cache.cpp:121-137).
int tl_release_sequence(tl_cache *c, int seq_id) {
    if (!c) return TL_ERR_INVALID_ARG;
    auto it = c->seqs.find(seq_id);
    if (it == c->seqs.end())
        return set_error(c, TL_ERR_NOT_FOUND, "Sequence not found: " + std::to_string(seq_id));
    for (int b : it->second.blocks) c->blocks.release(b);
    c->free_slots.push_back(it->second.slot);
    c->seqs.erase(it);
    return TL_OK;
}

int tl_reserve(tl_cache *c, int seq_id, int new_len) {
    if (!c) return TL_ERR_INVALID_ARG;
    Sequence *s = find_seq(c, seq_id);
    if (!s) return set_error(c, TL_ERR_NOT_FOUND, "reserve: sequence not found: " + std::to_string(seq_id));
    if (new_len < 0 || new_len > s->max_len)
        return set_error(c, TL_ERR_OVERFLOW,
                         "reserve: cache overflow. Requested: " + std::to_string(new_len) +
                             ", max: " + std::to_string(s->max_len));
    std::vector<std::pair<Sequence *, int>> undo;
    size_t mark = c->pending.size();
    int st = ensure_blocks(c, *s, new_len, mark, &undo);
    if (st != TL_OK) rollback(c, mark, undo);
    return st;
}

// getCacheChecked (reference src/kv_cache.cpp:139-157).
int tl_get_cache(tl_cache *c, int seq_id, int layer, void **k, void **v) {
    if (k) *k = nullptr;
    if (v) *v = nullptr;
    if (!c || !k || !v) return set_error(c, TL_ERR_INVALID_ARG, "getCache: null argument");
    Sequence *s = find_seq(c, seq_id);
    if (!s) return set_error(c, TL_ERR_NOT_FOUND, "Sequence not found: " + std::to_string(seq_id));
    if (layer < 0 || layer >= c->cfg.num_layers)
        return set_error(c, TL_ERR_INVALID_ARG, layer_error(c, "getCache", layer));
    const long long nb = c->cfg.num_blocks;
    const long long b0 = s->blocks.empty() ? 0 : s->blocks[0];
    uint16_t *base = static_cast<uint16_t *>(c->pool);
    *k = base + (((long long)layer * 2 + 0) * nb + b0) * c->block_elems;
    *v = base + (((long long)layer * 2 + 1) * nb + b0) * c->block_elems;
    return TL_OK;
}

// appendKV (reference src/kv_cache.cpp:168-238): validation in the same order.
int tl_append_kv(tl_cache *c, int seq_id, int layer, const void *k, const void *v, int num_tokens,
                 tl_stream_t stream) {
    if (!c) return TL_ERR_INVALID_ARG;
    if (!k) return set_error(c, TL_ERR_INVALID_ARG, "new_k is null");
    if (!v) return set_error(c, TL_ERR_INVALID_ARG, "new_v is null");
    if (num_tokens <= 0)
        return set_error(c, TL_ERR_INVALID_ARG,
                         "appendKV: num_tokens must be positive: " + std::to_string(num_tokens));
    if (layer < 0 || layer >= c->cfg.num_layers)
        return set_error(c, TL_ERR_INVALID_ARG, layer_error(c, "appendKV", layer));
    Sequence *s = find_seq(c, seq_id);
    if (!s)
        return set_error(c, TL_ERR_NOT_FOUND, "appendKV: sequence not found: " + std::to_string(seq_id));
    const int pos = s->len;
    if ((long long)pos + num_tokens > s->max_len)
        return set_error(c, TL_ERR_OVERFLOW,
                         "appendKV: cache overflow. Current: " + std::to_string(pos) +
                             ", appending: " + std::to_string(num_tokens) +
                             ", max: " + std::to_string(s->max_len));
    if (!c->on_device)
        return set_error(c, TL_ERR_NO_DEVICE, "appendKV: handle has no CUDA device (bookkeeping backend)");
    DeviceGuard guard(c);
    std::vector<std::pair<Sequence *, int>> undo;
    size_t mark = c->pending.size();
    int st = ensure_blocks(c, *s, (long long)pos + num_tokens, mark, &undo);
    if (st != TL_OK) {
        rollback(c, mark, undo);
        return st;
    }
    std::vector<int> rb((size_t)num_tokens), rp((size_t)num_tokens);
    for (int j = 0; j < num_tokens; ++j) {
        rp[(size_t)j] = pos + j;
        rb[(size_t)j] = s->blocks[(size_t)((pos + j) / c->bs)];
    }
    const long long row = (long long)c->cfg.num_kv_heads * c->cfg.head_dim;
    st = launch_rows(c, rb, rp, k, v, layer, 1, 0, row, (cudaStream_t)stream);
    if (st != TL_OK) return st;
    s->written = std::max(s->written, pos + num_tokens);
    return TL_OK;
}

int tl_append_kv_all_layers(tl_cache *c, const int *seq_ids, int num_seqs, const void *k,
                            const void *v, tl_stream_t stream) {
    if (!c) return TL_ERR_INVALID_ARG;
    return append_token_rows(c, "appendKVAllLayers", seq_ids, num_seqs, k, v, 0, c->cfg.num_layers,
                             (cudaStream_t)stream);
}

// advanceSeqLen (reference src/kv_cache.cpp:240-259): clamps to max_len.
int tl_advance_seq_len(tl_cache *c, int seq_id, int num_tokens) {
    if (!c) return TL_ERR_INVALID_ARG;
    if (num_tokens <= 0)
        return set_error(c, TL_ERR_INVALID_ARG,
                         "advanceSeqLen: num_tokens must be positive: " + std::to_string(num_tokens));
    Sequence *s = find_seq(c, seq_id);
    if (!s)
        return set_error(c, TL_ERR_NOT_FOUND,
                         "advanceSeqLen: sequence not found: " + std::to_string(seq_id));
    const int new_len = (int)std::min<long long>((long long)s->len + num_tokens, s->max_len);
    std::vector<std::pair<Sequence *, int>> undo;
    size_t mark = c->pending.size();
    int st = ensure_blocks(c, *s, new_len, mark, &undo);
    if (st != TL_OK) {
        rollback(c, mark, undo);
        return st;
    }
    s->len = new_len;
    s->written = std::max(s->written, s->len);
    return TL_OK;
}

int tl_get_seq_len(const tl_cache *c, int seq_id) {
    const Sequence *s = c ? find_seq(c, seq_id) : nullptr;
    return s ? s->len : 0;
}

int tl_has_sequence(const tl_cache *c, int seq_id) { return c && find_seq(c, seq_id) ? 1 : 0; }

size_t tl_used_memory(const tl_cache *c) {
    return c ? (size_t)(c->blocks.used() * c->block_bytes) : 0;
}

size_t tl_total_memory(const tl_cache *c) {
    return c ? (size_t)(c->blocks.capacity() * c->block_bytes) : 0;
}

size_t tl_free_memory(const tl_cache *c) { return tl_total_memory(c) - tl_used_memory(c); }

int tl_active_sequence_count(const tl_cache *c) { return c ? (int)c->seqs.size() : 0; }

int tl_get_config(const tl_cache *c, tl_config *cfg) {
    if (!c || !cfg) return TL_ERR_INVALID_ARG;
    *cfg = c->cfg;
    return TL_OK;
}

int tl_get_block_table(const tl_cache *c, int seq_id, int *blocks, int cap, int *count) {
    if (!c || !count) return TL_ERR_INVALID_ARG;
    const Sequence *s = find_seq(c, seq_id);
    if (!s) return TL_ERR_NOT_FOUND;
    *count = (int)s->blocks.size();
    if (blocks)
        for (int i = 0; i < cap && i < (int)s->blocks.size(); ++i) blocks[i] = s->blocks[(size_t)i];
    return TL_OK;
}

int tl_get_pool_stats(const tl_cache *c, tl_pool_stats *st) {
    if (!c || !st) return TL_ERR_INVALID_ARG;
    st->num_blocks = c->blocks.capacity();
    st->used_blocks = c->blocks.used();
    st->free_blocks = c->blocks.free_count();
    st->high_water = c->blocks.high_water();
    st->block_bytes = c->block_bytes;
    st->active_sequences = (int)c->seqs.size();
    st->max_blocks_per_seq = c->max_blocks_per_seq;
    st->kernel_launches = c->launches;
    return TL_OK;
}

int tl_get_pool(const tl_cache *c, void **base, size_t *elements) {
    if (!c || !base || !elements) return TL_ERR_INVALID_ARG;
    *base = c->pool;
    *elements = c->pool_elems;
    return TL_OK;
}

int tl_permute_free_blocks(tl_cache *c, unsigned long long seed) {
    if (!c) return TL_ERR_INVALID_ARG;
    c->blocks.permute(seed);
    return TL_OK;
}

}  // extern "C"

namespace {

// Where a head-sharded (peer-mode) decode writes and whom it signals.
struct PeerSpec {
    size_t out_offset;  // bytes into every rank's gathered area
    unsigned epoch;
};

int decode_impl(tl_cache *c, const char *ctx, int layer, const void *q, void *o,
                const int *seq_ids, int num_seqs, float scale, cudaStream_t stream,
                const PeerSpec *peer, bool rope_q = false) {
    if (layer < 0 || layer >= c->cfg.num_layers)
        return set_error(c, TL_ERR_INVALID_ARG, layer_error(c, ctx, layer));
    if (num_seqs < 0) return set_error(c, TL_ERR_INVALID_ARG, std::string(ctx) + ": num_seqs must be >= 0");
    if (num_seqs == 0 && !peer) return TL_OK;
    if (!q) return set_error(c, TL_ERR_INVALID_ARG, "query is null");
    if (!o && !peer) return set_error(c, TL_ERR_INVALID_ARG, "output is null");
    if (!seq_ids && num_seqs > 0) return set_error(c, TL_ERR_INVALID_ARG, "seq_ids is null");
    if (((uintptr_t)q & 3u) || ((uintptr_t)o & 3u))
        return set_error(c, TL_ERR_INVALID_ARG, std::string(ctx) + ": q and o must be 4-byte aligned");
    std::vector<const Sequence *> ss((size_t)num_seqs);
    for (int i = 0; i < num_seqs; ++i) {
        ss[(size_t)i] = find_seq(c, seq_ids[i]);
        if (!ss[(size_t)i])
            return set_error(c, TL_ERR_NOT_FOUND,
                             std::string(ctx) + ": sequence not found: " + std::to_string(seq_ids[i]));
    }
    if (!decode_geometry_supported(c))
        return set_error(c, TL_ERR_UNSUPPORTED,
                         std::string(ctx) + ": supported shapes are head_dim 64/128/256, block_size "
                                            "16/32, query group 1..8");
    if (!c->on_device)
        return set_error(c, TL_ERR_NO_DEVICE, std::string(ctx) + ": handle has no CUDA device (bookkeeping backend)");
    const int D = c->cfg.head_dim, Hq = c->cfg.num_q_heads, Hkv = c->cfg.num_kv_heads;
    const long long row = (long long)Hq * D;
    if (peer) {
        if (!c->peers_connected)
            return set_error(c, TL_ERR_INVALID_ARG, std::string(ctx) + ": peers are not connected (tl_peer_connect)");
        if (num_seqs > tllm::kMaxDecodeSeqs)
            return set_error(c, TL_ERR_INVALID_ARG, std::string(ctx) + ": at most " +
                                                        std::to_string(tllm::kMaxDecodeSeqs) +
                                                        " sequences per peer-mode call");
        const size_t slice = (size_t)num_seqs * (size_t)row * 2;
        if ((peer->out_offset & 15u) ||
            peer->out_offset + (size_t)c->peer_world * slice > c->gather_bytes)
            return set_error(c, TL_ERR_INVALID_ARG,
                             std::string(ctx) + ": out_offset must be 16-byte aligned and the "
                                                "world's slices must fit the gather buffer");
    }
    DeviceGuard guard(c);
    if (!c->pending.empty()) {
        int st = flush_deltas(c, stream);
        if (st != TL_OK) return st;
    }
    if (!(scale > 0.0f)) scale = 1.0f / std::sqrt((float)D);
    for (int j0 = 0; j0 < num_seqs || (peer && j0 == 0); j0 += tllm::kMaxDecodeSeqs) {
        const int n = std::min(tllm::kMaxDecodeSeqs, num_seqs - j0);
        tllm::DecodeArgs a{};
        a.g = c->geom();
        a.q = static_cast<const uint16_t *>(q) + j0 * row;
        a.o = peer ? nullptr : static_cast<uint16_t *>(o) + j0 * row;
        a.partial = c->partial;
        a.counters = c->merge_counters;  // in-kernel merge of cut units
        a.layer = layer;
        a.group = c->group;
        a.scale_log2 = scale * 1.4426950408889634f;
        if (rope_q) {
            a.rope_cos = c->rope_cos;
            a.rope_sin = c->rope_sin;
            a.rope_max_pos = c->cfg.max_seq_len;
        }
        a.nseq = n;
        if (peer) {  // write this rank's slice locally, publish, pull the others
            const size_t slice = (size_t)n * (size_t)row * 2;
            unsigned char *base = static_cast<unsigned char *>(c->peer_region);
            a.ndst = 1;
            a.out_dst[0] = base + tllm::kPeerFlagBytes + peer->out_offset + (size_t)c->peer_rank * slice;
            a.flag_dst[0] = reinterpret_cast<unsigned *>(base) + c->peer_rank;
            a.epoch = peer->epoch;
            for (int r = 0; r < c->peer_world; ++r)
                a.peer_base[r] = static_cast<const unsigned char *>(c->peer_bases[r]);
            a.world = c->peer_world;
            a.rank = c->peer_rank;
            a.gather_off = tllm::kPeerFlagBytes + peer->out_offset;
            a.slice_bytes = slice;
            a.peer_wait_ns = c->peer_wait_ns;
        }
        long long real_tiles = 0;  // the per-unit overhead charge follows the tiles per worker
        for (int i = 0; i < n; ++i) real_tiles += ceil_div(ss[(size_t)(j0 + i)]->written, tllm::kDecodeTile);
        a.vslots = tllm::unit_overhead_slots((long long)Hkv * real_tiles, c->max_workers);
        a.prefix[0] = 0;
        for (int i = 0; i < n; ++i) {
            const Sequence *s = ss[(size_t)(j0 + i)];
            a.slot[i] = s->slot;
            a.len[i] = s->written;
            a.prefix[i + 1] = a.prefix[i] + tllm::unit_slots(ceil_div(s->written, tllm::kDecodeTile), a.vslots);
            if (s->written == 0) {  // nothing to attend: zeros, as documented
                const int ndst = peer ? a.ndst : 1;
                for (int r = 0; r < ndst; ++r) {
                    void *dst = peer ? static_cast<void *>(static_cast<uint16_t *>(a.out_dst[r]) + (long long)i * row)
                                     : static_cast<void *>(static_cast<uint16_t *>(a.o) + (long long)i * row);
                    cudaError_t e = cudaMemsetAsync(dst, 0, (size_t)row * 2, stream);
                    if (e != cudaSuccess) return cuda_fail(c, e, "decodeAttention: memset failed");
                }
            }
        }
        a.total_items = (long long)Hkv * a.prefix[n];
        if (a.total_items == 0 && !peer) continue;
        a.workers = (int)std::min<long long>(c->max_workers, std::max<long long>(a.total_items, 1));
        // Few long units cut into many pieces: merge them in a wide second
        // pass instead of by one warp inside the decode kernel.
        int max_tiles = 0;
        for (int i = 0; i < n; ++i) max_tiles = std::max(max_tiles, a.prefix[i + 1] - a.prefix[i]);
        const long long pieces =
            a.total_items ? (long long)max_tiles * a.workers / a.total_items + 2 : 0;
        // peer mode: the merge pass always runs, its last CTA publishes and gathers
        const bool two_pass = pieces > tllm::kInKernelMergeMaxPieces || a.total_items == 0 || peer;
        if (two_pass) a.counters = nullptr;
        cudaError_t e;
        if (a.total_items > 0) {
            tllm::DecodeArgs ad = a;
            ad.done_counter = nullptr;
            e = tllm::launch_decode(ad, c->tmap, stream);
            if (e != cudaSuccess) return cuda_fail(c, e, "decodeAttention: decode launch failed");
            ++c->launches;
        }
        if (two_pass) {
            tllm::DecodeArgs am = a;
            am.done_counter = peer ? c->peer_done_counter : nullptr;
            e = tllm::launch_merge(am, stream);
            if (e != cudaSuccess) return cuda_fail(c, e, "decodeAttention: merge launch failed");
            ++c->launches;
        }
        if (peer) break;
    }
    return TL_OK;
}

}  // namespace

extern "C" {

// Replacement for kernels::attention_decode (reference
// kernels/attention.cu:114-128) as called at src/transformer.cpp:230-237.
int tl_decode_attention(tl_cache *c, int layer, const void *q, void *o, const int *seq_ids,
                        int num_seqs, float scale, tl_stream_t stream) {
    if (!c) return TL_ERR_INVALID_ARG;
    return decode_impl(c, "decodeAttention", layer, q, o, seq_ids, num_seqs, scale,
                       (cudaStream_t)stream, nullptr);
}

// The decode branch of TransformerLayer::attention (reference
// src/transformer.cpp:222-237) for a batch: appendKV of each sequence's new
// token at its current length, then attention over len + 1 tokens, with Q
// rotated by the handle's RoPE table at that position when K is rotated on
// append.
int tl_attention_step(tl_cache *c, int layer, const void *q, const void *k_new, const void *v_new,
                      void *o, const int *seq_ids, int num_seqs, float scale, tl_stream_t stream) {
    if (!c) return TL_ERR_INVALID_ARG;
    if (layer < 0 || layer >= c->cfg.num_layers)
        return set_error(c, TL_ERR_INVALID_ARG, layer_error(c, "attentionStep", layer));
    if (num_seqs > 0 && (!q || !o))
        return set_error(c, TL_ERR_INVALID_ARG, !q ? "query is null" : "output is null");
    if (c->on_device && !decode_geometry_supported(c))
        return set_error(c, TL_ERR_UNSUPPORTED,
                         "attentionStep: supported shapes are head_dim 64/128/256, block_size 16/32, "
                         "query group 1..8");
    // The new token is each sequence's newest attended one (Q's position):
    // tokens appended past the length and not yet advanced are refused.
    for (int i = 0; i < num_seqs && seq_ids; ++i) {
        const Sequence *s = find_seq(c, seq_ids[i]);
        if (s && s->written > s->len + 1)
            return set_error(c, TL_ERR_INVALID_ARG,
                             "attentionStep: sequence " + std::to_string(seq_ids[i]) +
                                 " has tokens appended past its length; advance it first");
    }
    int st = append_token_rows(c, "attentionStep", seq_ids, num_seqs, k_new, v_new, layer, 1,
                               (cudaStream_t)stream);
    if (st != TL_OK) return st;
    return decode_impl(c, "attentionStep", layer, q, o, seq_ids, num_seqs, scale, (cudaStream_t)stream,
                       nullptr, c->cfg.rope_on_append != 0);
}

// Causal prefill attention over the paged cache (replaces
// kernels::attention_prefill, reference kernels/attention.cu:131-237, as
// called at src/transformer.cpp:238-242): sequence i's num_tokens[i] query
// rows are its last num_tokens[i] written tokens, each attending the tokens
// up to its own position.
int tl_prefill_attention(tl_cache *c, int layer, const void *q, void *o, const int *seq_ids,
                         const int *num_tokens, int num_seqs, float scale, tl_stream_t stream) {
    if (!c) return TL_ERR_INVALID_ARG;
    const char *ctx = "prefillAttention";
    if (layer < 0 || layer >= c->cfg.num_layers) return set_error(c, TL_ERR_INVALID_ARG, layer_error(c, ctx, layer));
    if (num_seqs < 0) return set_error(c, TL_ERR_INVALID_ARG, std::string(ctx) + ": num_seqs must be >= 0");
    if (num_seqs == 0) return TL_OK;
    if (!q) return set_error(c, TL_ERR_INVALID_ARG, "query is null");
    if (!o) return set_error(c, TL_ERR_INVALID_ARG, "output is null");
    if (!seq_ids || !num_tokens) return set_error(c, TL_ERR_INVALID_ARG, "seq_ids is null");
    if (((uintptr_t)q & 3u) || ((uintptr_t)o & 3u))
        return set_error(c, TL_ERR_INVALID_ARG, std::string(ctx) + ": q and o must be 4-byte aligned");
    std::vector<const Sequence *> ss((size_t)num_seqs);
    std::unordered_set<int> seen;
    for (int i = 0; i < num_seqs; ++i) {
        const Sequence *s = find_seq(c, seq_ids[i]);
        if (!s)
            return set_error(c, TL_ERR_NOT_FOUND,
                             std::string(ctx) + ": sequence not found: " + std::to_string(seq_ids[i]));
        if (!seen.insert(seq_ids[i]).second)
            return set_error(c, TL_ERR_INVALID_ARG,
                             std::string(ctx) + ": duplicate sequence id " + std::to_string(seq_ids[i]));
        ss[(size_t)i] = s;
    }
    for (int i = 0; i < num_seqs; ++i)
        if (num_tokens[i] <= 0 || num_tokens[i] > ss[(size_t)i]->written)
            return set_error(c, TL_ERR_INVALID_ARG,
                             std::string(ctx) + ": num_tokens must be in [1, written tokens] for seq " +
                                 std::to_string(seq_ids[i]) + ": " + std::to_string(num_tokens[i]));
    const int D = c->cfg.head_dim;
    if (!decode_geometry_supported(c) || (D != 64 && D != 128))
        return set_error(c, TL_ERR_UNSUPPORTED,
                         std::string(ctx) + ": supported shapes are head_dim 64/128, block_size 16/32, "
                                            "query group 1..8");
    if (!c->on_device)
        return set_error(c, TL_ERR_NO_DEVICE, std::string(ctx) + ": handle has no CUDA device (bookkeeping backend)");
    DeviceGuard guard(c);
    if (!c->pending.empty()) {
        int st = flush_deltas(c, (cudaStream_t)stream);
        if (st != TL_OK) return st;
    }
    if (!(scale > 0.0f)) scale = 1.0f / std::sqrt((float)D);
    int gp = 1;
    while (gp < c->group) gp <<= 1;
    const int qpb = tllm::prefill_tc_rows_per_cta() / gp;
    long long row = 0;
    for (int j0 = 0; j0 < num_seqs; j0 += tllm::kMaxPrefillSeqs) {
        const int n = std::min(tllm::kMaxPrefillSeqs, num_seqs - j0);
        tllm::PrefillArgs a{};
        a.g = c->geom();
        a.q = q;
        a.o = o;
        if (c->cfg.rope_on_append) {
            a.rope_cos = c->rope_cos;
            a.rope_sin = c->rope_sin;
            a.rope_max_pos = c->cfg.max_seq_len;
        }
        a.layer = layer;
        a.group = c->group;
        a.group_pad = gp;
        a.scale_log2 = scale * 1.4426950408889634f;
        a.nseq = n;
        a.cta_prefix[0] = 0;
        for (int i = 0; i < n; ++i) {
            const Sequence *s = ss[(size_t)(j0 + i)];
            const int nt = num_tokens[j0 + i];
            if (row + nt > INT32_MAX)
                return set_error(c, TL_ERR_INVALID_ARG, std::string(ctx) + ": too many query rows in one call");
            a.slot[i] = s->slot;
            a.written[i] = s->written;
            a.ntok[i] = nt;
            a.row_off[i] = (int)row;
            row += nt;
            a.cta_prefix[i + 1] = a.cta_prefix[i] + (nt + qpb - 1) / qpb;
        }
        cudaError_t e = tllm::launch_prefill_tc(a, c->tmap, (cudaStream_t)stream);
        if (e != cudaSuccess) return cuda_fail(c, e, "prefillAttention: launch failed");
        ++c->launches;
    }
    return TL_OK;
}

// Q/K/V projections (W8A16) of one decode token per sequence, with K and V
// appended at each sequence's current length (RoPE on Q and K when the
// handle rotates on append). Replaces the three kernels::w8a16_matmul calls
// and the appendKV of TransformerLayer::attention's decode step (reference
// src/transformer.cpp:209-226, kernels/w8a16_matmul.cu:119-235,
// src/kv_cache.cpp:206-233), batched over sequences.
static int project_qkv_append(tl_cache *c, int layer, const void *x, int hidden, const int8_t *wq, const void *sq,
                              const int8_t *wk, const void *sk, const int8_t *wv, const void *sv, int group_size,
                              const int *seq_ids, int num_seqs, void *q_out, tl_stream_t stream, bool packed) {
    const char *ctx = packed ? "projectQKVAppendPacked" : "projectQKVAppend";
    if (!c) return TL_ERR_INVALID_ARG;
    if (layer < 0 || layer >= c->cfg.num_layers)
        return set_error(c, TL_ERR_INVALID_ARG, layer_error(c, ctx, layer));
    if (num_seqs < 0) return set_error(c, TL_ERR_INVALID_ARG, std::string(ctx) + ": num_seqs must be >= 0");
    if (num_seqs == 0) return TL_OK;
    if (!seq_ids) return set_error(c, TL_ERR_INVALID_ARG, "seq_ids is null");
    if (!x || !q_out) return set_error(c, TL_ERR_INVALID_ARG, !x ? "input is null" : "q output is null");
    if (!wq || !wk || !wv || !sq || !sk || !sv)
        return set_error(c, TL_ERR_INVALID_ARG, std::string(ctx) + ": a weight or scale pointer is null");
    if (hidden <= 0 || group_size <= 0)
        return set_error(c, TL_ERR_INVALID_ARG, std::string(ctx) + ": hidden and group_size must be positive");
    const int D = c->cfg.head_dim;
    if ((D != 64 && D != 128) || hidden % tllm::qkv_k_block() != 0 ||
        (group_size != 16 && group_size != 32 && group_size != 64 && group_size != 128))
        return set_error(c, TL_ERR_UNSUPPORTED,
                         std::string(ctx) + ": supported shapes are head_dim 64/128, hidden a multiple of 128, "
                                            "group_size 16/32/64/128");
    auto mis = [](const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) != 0; };
    if (mis(x, 16) || mis(q_out, 16) || mis(sq, 16) || mis(sk, 16) || mis(sv, 16) || mis(wq, 4) || mis(wk, 4) ||
        mis(wv, 4))
        return set_error(c, TL_ERR_INVALID_ARG,
                         std::string(ctx) + ": input, q output and scales must be 16-byte aligned, weights 4-byte");
    std::vector<Sequence *> ss((size_t)num_seqs);
    std::unordered_set<int> seen;
    for (int i = 0; i < num_seqs; ++i) {
        Sequence *s = find_seq(c, seq_ids[i]);
        if (!s)
            return set_error(c, TL_ERR_NOT_FOUND,
                             std::string(ctx) + ": sequence not found: " + std::to_string(seq_ids[i]));
        if (!seen.insert(seq_ids[i]).second)
            return set_error(c, TL_ERR_INVALID_ARG,
                             std::string(ctx) + ": duplicate sequence id " + std::to_string(seq_ids[i]));
        if (s->len + 1 > s->max_len)
            return set_error(c, TL_ERR_OVERFLOW,
                             std::string(ctx) + ": cache overflow. seq " + std::to_string(seq_ids[i]) +
                                 " Current: " + std::to_string(s->len) +
                                 ", appending: 1, max: " + std::to_string(s->max_len));
        ss[(size_t)i] = s;
    }
    if (!c->on_device)
        return set_error(c, TL_ERR_NO_DEVICE, std::string(ctx) + ": handle has no CUDA device (bookkeeping backend)");
    DeviceGuard guard(c);
    const int Hkv = c->cfg.num_kv_heads, Hq = Hkv * c->group;
    const int tiles = Hq + 2 * Hkv;
    const int rows_max = std::min(num_seqs, tllm::kMaxQkvRows);
    // tcgen05 kernel where the columns come in tiles of 128 and the weights
    // allow 16-byte loads; the mma.sync kernel otherwise
    // (and a split of K whose group accumulators fit TMEM, for every
    // launch: a full one of rows_max rows and the last, shorter one)
    const int tiles128 = (Hq + 2 * Hkv) * D / 128;
    const int rows_last = num_seqs % tllm::kMaxQkvRows;
    auto tc_plan = [&](int n, int *ks_, int *kchunk_) {
        return tllm::qkv_tc_split(hidden, group_size, n, tiles128, c->num_sms, ks_, kchunk_);
    };
    int ks, kchunk;
    bool tc = tllm::qkv_tc_supported(D, group_size, Hq * D, Hkv * D, hidden) && !mis(wq, 16) &&
              !mis(wk, 16) && !mis(wv, 16) && tc_plan(rows_max, &ks, &kchunk);
    int ks_last = 0, kchunk_last = 0;
    if (tc && rows_last > 0 && num_seqs > tllm::kMaxQkvRows) tc = tc_plan(rows_last, &ks_last, &kchunk_last);
    if (packed && !tc)  // only the tcgen05 kernel reads the tile-blocked layout
        return set_error(c, TL_ERR_UNSUPPORTED,
                         std::string(ctx) + ": packed weights need Q, K and V widths in multiples of 128, "
                                            "group_size 32/64/128, 16-byte aligned weights and a split of "
                                            "hidden whose group accumulators fit TMEM");
    size_t need;
    if (tc) {
        // one fp32 accumulator per column tile
        need = ks > 1 ? (size_t)tiles128 * tllm::qkv_tc_rows_padded(rows_max) * 128 : 0;
        if (ks_last > 1)
            need = std::max(need, (size_t)tiles128 * tllm::qkv_tc_rows_padded(rows_last) * 128);
    } else {
        // split-K: about three CTAs per SM (2 and 4 measured slower); a chunk's
        // activations stay under ~100 KB of shared memory
        const int kblk = tllm::qkv_k_block(), nkb = hidden / kblk;
        const int rpad = tllm::qkv_rows_padded(rows_max);  // the largest launch's row tile
        const int kb_cap = std::max(1, (100 * 1024 / (2 * rpad) - 8) / kblk);
        ks = std::max(1, (3 * std::max(c->num_sms, 1) + tiles / 2) / tiles);
        ks = std::min(ks, nkb);
        const int kbc = std::min((nkb + ks - 1) / ks, kb_cap);
        ks = (nkb + kbc - 1) / kbc;
        kchunk = kbc * kblk;
        need = ks > 1 ? (size_t)tiles * rpad * D : 0;  // one fp32 accumulator per column tile
    }
    std::string why;
    if (need > c->qkv_partial_floats) {
        storage_free(c, c->qkv_partial);
        c->qkv_partial = nullptr;
        c->qkv_partial_floats = 0;
        void *p = nullptr;
        if (storage_alloc(c, &p, need * 4, &why))
            return set_error(c, TL_ERR_CUDA, std::string(ctx) + ": split-K scratch allocation failed: " + why);
        c->qkv_partial = static_cast<float *>(p);
        c->qkv_partial_floats = need;
    }
    if (tiles > c->qkv_counter_n) {
        storage_free(c, c->qkv_counters);
        c->qkv_counters = nullptr;
        c->qkv_counter_n = 0;
        void *p = nullptr;
        if (storage_alloc(c, &p, (size_t)tiles * sizeof(int), &why))
            return set_error(c, TL_ERR_CUDA, std::string(ctx) + ": counter allocation failed: " + why);
        c->qkv_counters = static_cast<int *>(p);
        c->qkv_counter_n = tiles;
    }
    std::vector<std::pair<Sequence *, int>> undo;
    size_t mark = c->pending.size();
    std::vector<int> rb((size_t)num_seqs), rp((size_t)num_seqs);
    for (int i = 0; i < num_seqs; ++i) {
        Sequence &s = *ss[(size_t)i];
        int st = ensure_blocks(c, s, (long long)s.len + 1, mark, &undo);
        if (st != TL_OK) {
            rollback(c, mark, undo);
            return st;
        }
        rp[(size_t)i] = s.len;
        rb[(size_t)i] = s.blocks[(size_t)(s.len / c->bs)];
    }
    if (!c->pending.empty()) {  // new blocks' table entries (the decode reads them)
        int st = flush_deltas(c, (cudaStream_t)stream);
        if (st != TL_OK) return st;
    }
    const long long nq = (long long)Hq * D;
    for (int r0 = 0; r0 < num_seqs; r0 += tllm::kMaxQkvRows) {
        const int n = std::min(tllm::kMaxQkvRows, num_seqs - r0);
        tllm::QkvArgs a{};
        a.g = c->geom();
        a.x = static_cast<const uint16_t *>(x) + (long long)r0 * hidden;
        a.w[0] = wq;
        a.w[1] = wk;
        a.w[2] = wv;
        a.w_packed = packed ? 1 : 0;
        a.sc[0] = sq;
        a.sc[1] = sk;
        a.sc[2] = sv;
        a.n[0] = Hq * D;
        a.n[1] = a.n[2] = Hkv * D;
        a.K = hidden;
        a.group = group_size;
        a.rows = n;
        a.num_q_heads = Hq;
        a.ksplit = ks;
        a.kchunk = kchunk;
        if (tc && n != rows_max) {  // the last, shorter launch has its own split
            a.ksplit = ks_last;
            a.kchunk = kchunk_last;
        }
        a.q_out = static_cast<uint16_t *>(q_out) + r0 * nq;
        if (c->cfg.rope_on_append) {
            a.rope_cos = c->rope_cos;
            a.rope_sin = c->rope_sin;
            a.rope_max_pos = c->cfg.max_seq_len;
        }
        a.layer = layer;
        a.partial = c->qkv_partial;
        a.counters = c->qkv_counters;
        for (int j = 0; j < n; ++j) {
            a.row_block[j] = rb[(size_t)(r0 + j)];
            a.row_pos[j] = rp[(size_t)(r0 + j)];
        }
        cudaError_t e = tc ? tllm::launch_qkv_append_tc(a, (cudaStream_t)stream)
                           : tllm::launch_qkv_append(a, (cudaStream_t)stream);
        if (e != cudaSuccess)
            return cuda_fail(c, e, packed ? "projectQKVAppendPacked: launch failed" : "projectQKVAppend: launch failed");
        ++c->launches;
    }
    for (Sequence *s : ss) s->written = std::max(s->written, s->len + 1);
    return TL_OK;
}

int tl_project_qkv_append(tl_cache *c, int layer, const void *x, int hidden, const int8_t *wq, const void *sq,
                          const int8_t *wk, const void *sk, const int8_t *wv, const void *sv, int group_size,
                          const int *seq_ids, int num_seqs, void *q_out, tl_stream_t stream) {
    return project_qkv_append(c, layer, x, hidden, wq, sq, wk, sk, wv, sv, group_size, seq_ids, num_seqs, q_out,
                              stream, false);
}

// The same projections from weights repacked once by tl_qkv_pack_weight: each
// CTA's weight blocks are then contiguous 8 KB copies instead of 64 row
// segments of 128 bytes.
int tl_project_qkv_append_packed(tl_cache *c, int layer, const void *x, int hidden, const int8_t *wq,
                                 const void *sq, const int8_t *wk, const void *sk, const int8_t *wv, const void *sv,
                                 int group_size, const int *seq_ids, int num_seqs, void *q_out, tl_stream_t stream) {
    return project_qkv_append(c, layer, x, hidden, wq, sq, wk, sk, wv, sv, group_size, seq_ids, num_seqs, q_out,
                              stream, true);
}

// Repacks one int8 weight [hidden][n] into the tile-blocked layout (once, at
// model load). No handle: errors are read back with tl_last_error(NULL).
int tl_qkv_pack_weight(const int8_t *w, int hidden, int n, int8_t *packed, tl_stream_t stream) {
    auto fail = [](int st, const std::string &m) {
        g_create_error = m;
        return st;
    };
    if (!w || !packed) return fail(TL_ERR_INVALID_ARG, "packQKVWeight: a weight pointer is null");
    if (hidden <= 0 || n <= 0 || hidden % 128 != 0 || n % 128 != 0)
        return fail(TL_ERR_UNSUPPORTED, "packQKVWeight: hidden and n must be positive multiples of 128");
    const uintptr_t a0 = reinterpret_cast<uintptr_t>(w), b0 = reinterpret_cast<uintptr_t>(packed);
    if ((a0 & 15) || (b0 & 15)) return fail(TL_ERR_INVALID_ARG, "packQKVWeight: weights must be 16-byte aligned");
    const uintptr_t bytes = (uintptr_t)hidden * (uintptr_t)n;
    if (a0 < b0 + bytes && b0 < a0 + bytes)
        return fail(TL_ERR_INVALID_ARG, "packQKVWeight: source and destination overlap");
    int devices = 0;
    if (cudaGetDeviceCount(&devices) != cudaSuccess || devices == 0) {
        cudaGetLastError();
        return fail(TL_ERR_NO_DEVICE, "packQKVWeight: no CUDA device");
    }
    cudaError_t e = tllm::launch_qkv_pack_weight(w, hidden, n, packed, (cudaStream_t)stream);
    if (e != cudaSuccess)
        return fail(TL_ERR_CUDA, std::string("packQKVWeight: launch failed: ") + cudaGetErrorString(e));
    return TL_OK;
}

// Token sampling on the device (reference src/inference_engine.cpp:296-307
// and the samplers of :330-490). No handle: errors are read back with
// tl_last_error(NULL).
int tl_sample_tokens(const void *logits, long long row_stride, int rows, int vocab, int do_sample,
                     float temperature, int top_k, float top_p, unsigned long long seed, unsigned long long step,
                     int *tokens_out, tl_stream_t stream) {
    auto fail = [](int st, const std::string &m) {
        g_create_error = m;
        return st;
    };
    if (rows < 0 || vocab <= 0) return fail(TL_ERR_INVALID_ARG, "sampleTokens: rows must be >= 0 and vocab > 0");
    if (vocab > tllm::sample_max_vocab() || rows > (1 << 27))
        return fail(TL_ERR_UNSUPPORTED, "sampleTokens: vocab above " + std::to_string(tllm::sample_max_vocab()) +
                                            " or more than 2^27 rows is not supported");
    if (rows == 0) return TL_OK;
    if (!logits || !tokens_out)
        return fail(TL_ERR_INVALID_ARG, !logits ? "sampleTokens: logits is null" : "sampleTokens: tokens is null");
    if (rows > 1 && row_stride < vocab && row_stride != 0)
        return fail(TL_ERR_INVALID_ARG, "sampleTokens: row_stride must be 0 (shared logits) or >= vocab");
    tllm::SampleArgs a{};
    a.logits = logits;
    a.row_stride = row_stride;
    a.rows = rows;
    a.vocab = vocab;
    a.temperature = std::max(temperature, 1e-5f);  // as the reference clamps
    a.seed = seed;
    a.step = step;
    a.tokens = tokens_out;
    if (!do_sample) {
        a.mode = 0;
    } else if (top_p < 1.0f) {
        a.mode = 2;
        a.top_p = std::min(std::max(top_p, 1e-5f), 1.0f);
    } else {
        a.mode = 1;
        a.top_k = top_k > 0 ? std::max(1, std::min(top_k, vocab)) : vocab;  // temperature: every token
    }
    cudaError_t e = tllm::launch_sample(a, (cudaStream_t)stream);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(TL_ERR_CUDA, std::string("sampleTokens: launch failed: ") + cudaGetErrorString(e));
    }
    return TL_OK;
}

int tl_peer_init(tl_cache *c, int rank, int world, size_t gather_bytes, void *ipc_handle) {
    if (!c) return TL_ERR_INVALID_ARG;
    if (world < 1 || world > tllm::kMaxPeers || rank < 0 || rank >= world || !ipc_handle)
        return set_error(c, TL_ERR_INVALID_ARG, "peerInit: need 1 <= world <= 8, 0 <= rank < world and a handle buffer");
    if (!c->on_device)
        return set_error(c, TL_ERR_NO_DEVICE, "peerInit: handle has no CUDA device (bookkeeping backend)");
    if (c->peer_region)
        return set_error(c, TL_ERR_INVALID_ARG, "peerInit: already initialised");
    DeviceGuard guard(c);
    const size_t bytes = tllm::kPeerFlagBytes + ((gather_bytes + 255) & ~size_t(255));
    void *p = nullptr;
    std::string why;
    if (storage_alloc(c, &p, bytes, &why))
        return set_error(c, TL_ERR_CUDA, "peerInit: allocation failed: " + why);
    void *ctr = nullptr;
    if (storage_alloc(c, &ctr, 256, &why)) {
        storage_free(c, p);
        return set_error(c, TL_ERR_CUDA, "peerInit: allocation failed: " + why);
    }
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        storage_free(c, p);
        storage_free(c, ctr);
        return cuda_fail(c, e, "peerInit: cudaIpcGetMemHandle failed");
    }
    std::memcpy(ipc_handle, &h, sizeof(h));
    c->peer_region = p;
    c->peer_done_counter = static_cast<int *>(ctr);
    c->gather_bytes = bytes - tllm::kPeerFlagBytes;
    c->peer_rank = rank;
    c->peer_world = world;
    return TL_OK;
}

int tl_peer_connect(tl_cache *c, const void *ipc_handles) {
    if (!c) return TL_ERR_INVALID_ARG;
    if (!c->peer_region || !ipc_handles)
        return set_error(c, TL_ERR_INVALID_ARG, "peerConnect: call tl_peer_init first and pass every rank's handle");
    DeviceGuard guard(c);
    const unsigned char *hs = static_cast<const unsigned char *>(ipc_handles);
    for (int r = 0; r < c->peer_world; ++r) {
        if (r == c->peer_rank) {
            c->peer_bases[r] = c->peer_region;
            continue;
        }
        cudaIpcMemHandle_t h;
        std::memcpy(&h, hs + (size_t)r * TL_IPC_HANDLE_BYTES, sizeof(h));
        void *p = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) return cuda_fail(c, e, "peerConnect: cudaIpcOpenMemHandle failed");
        c->peer_bases[r] = p;
        c->peer_opened[r] = true;
    }
    c->peers_connected = true;
    return TL_OK;
}

int tl_set_peer_wait_limit(tl_cache *c, double seconds) {
    if (!c) return TL_ERR_INVALID_ARG;
    if (!(seconds <= 600.0))
        return set_error(c, TL_ERR_INVALID_ARG, "setPeerWaitLimit: seconds must be at most 600 (<= 0: default)");
    c->peer_wait_ns = seconds > 0.0 ? (unsigned long long)(seconds * 1e9) : 0ull;
    if (seconds > 0.0 && c->peer_wait_ns == 0) c->peer_wait_ns = 1;
    return TL_OK;
}

int tl_debug_peer_attach(tl_cache *c, int rank, void *region) {
    if (!c) return TL_ERR_INVALID_ARG;
    if (!c->peer_region)
        return set_error(c, TL_ERR_INVALID_ARG, "peerAttach: call tl_peer_init first");
    if (rank < 0 || rank >= c->peer_world || rank == c->peer_rank || !region ||
        ((uintptr_t)region & 255u))
        return set_error(c, TL_ERR_INVALID_ARG,
                         "peerAttach: need another rank of the world and a 256-byte aligned region");
    if (c->peer_opened[rank]) {
        DeviceGuard guard(c);
        cudaIpcCloseMemHandle(c->peer_bases[rank]);
        c->peer_opened[rank] = false;
    }
    c->peer_bases[rank] = region;
    c->peer_bases[c->peer_rank] = c->peer_region;
    bool all = true;
    for (int r = 0; r < c->peer_world; ++r) all = all && c->peer_bases[r] != nullptr;
    c->peers_connected = all;
    return TL_OK;
}

int tl_peer_buffer(const tl_cache *c, void **gathered, size_t *bytes) {
    if (!c || !gathered || !c->peer_region) return TL_ERR_INVALID_ARG;
    *gathered = static_cast<unsigned char *>(c->peer_region) + tllm::kPeerFlagBytes;
    if (bytes) *bytes = c->gather_bytes;
    return TL_OK;
}

int tl_decode_attention_peer(tl_cache *c, int layer, const void *q, const int *seq_ids,
                             int num_seqs, float scale, size_t out_offset, unsigned epoch,
                             tl_stream_t stream) {
    if (!c) return TL_ERR_INVALID_ARG;
    PeerSpec ps{out_offset, epoch};
    return decode_impl(c, "decodeAttentionPeer", layer, q, nullptr, seq_ids, num_seqs, scale,
                       (cudaStream_t)stream, &ps);
}



int tl_sync_check(tl_cache *c, tl_stream_t stream) {
    if (!c) return TL_ERR_INVALID_ARG;
    if (!c->on_device) return TL_OK;
    DeviceGuard guard(c);
    cudaError_t e = cudaStreamSynchronize((cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(c, e, "sync: stream synchronize failed");
    int word = 0;
    e = cudaMemcpy(&word, c->err_word, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(c, e, "sync: error-word read failed");
    if (word != 0) {
        cudaMemset(c->err_word, 0, sizeof(int));
        // A worker that stopped early may have left merge tickets behind.
        if (c->merge_counters)
            cudaMemset(c->merge_counters, 0,
                       (size_t)tllm::kMaxDecodeSeqs * c->cfg.num_kv_heads * sizeof(int));
        // and a projection that stopped early, split-K sums and tickets
        if (c->qkv_partial) cudaMemset(c->qkv_partial, 0, c->qkv_partial_floats * sizeof(float));
        if (c->qkv_counters) cudaMemset(c->qkv_counters, 0, (size_t)c->qkv_counter_n * sizeof(int));
        std::string m = "device error word 0x" + [&] {
            char buf[16];
            std::snprintf(buf, sizeof buf, "%x", word);
            return std::string(buf);
        }() + ":";
        if (word & tllm::kErrBlockRange) m += " block id out of range;";
        if (word & tllm::kErrPosRange) m += " position out of range;";
        if (word & tllm::kErrWaitTimeout) m += " bounded wait timed out;";
        return set_error(c, TL_ERR_DEVICE_FAULT, m);
    }
    return TL_OK;
}

}  // extern "C"
