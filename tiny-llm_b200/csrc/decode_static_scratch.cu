// Allocation-free decode attention: tl_decode_attention_static.
//
// Who this is for. Some callers cannot call cudaMalloc at the point where
// they decode: an engine whose device memory all comes from its own arena or
// caching allocator (a raw cudaMalloc would fragment or bypass it), code that
// must not synchronize the device (cudaMalloc/cudaFree can), or a host path
// with hard latency limits. tl_decode_attention needs a handle, and creating
// a handle allocates the pool, block tables and split scratch. This entry
// point instead decodes over memory the caller already owns — pool, block
// tables, queries and outputs — and allocates nothing: its only scratch (the
// split-K partials and a fallback error word) lives in the file-scope array
// below, which is part of the loaded module, not a runtime allocation.
//
// Limits and sharing.
//  - The array is kStaticScratchBytes (8 MiB) on every GPU that loads this
//    library, held until the process exits.
//  - Every call uses the same array and leaves its contents behind. The
//    partials are always written before they are read; the fallback error
//    word is cleared (cudaMemsetAsync) at the start of each call.
//  - Calls whose work overlaps on the GPU (on different streams, or from
//    different host threads without ordering) race on the array. Order them
//    on one stream, or serialize them.
//  - The first call on each device looks the array's device address up with
//    cudaGetSymbolAddress (with that device current) and opts the decode
//    kernel into its shared-memory size; make that first call before any
//    stream capture.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <mutex>
#include <string>

#include "kernels.h"
#include "tllm_kv.h"

namespace {

constexpr size_t kStaticScratchBytes = size_t(8) << 20;  // 8 MiB
constexpr size_t kErrorSlotBytes = 256;                  // fallback error word
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_decode_scratch[kStaticScratchBytes];

std::mutex g_setup_mu;
void *g_scratch_ptr[kMaxDevices] = {};
int g_max_workers[kMaxDevices][3] = {};  // per device, per head_dim 64/128/256

int dim_index(int D) { return D == 64 ? 0 : (D == 128 ? 1 : 2); }

// Per-device set-up, run by the first call on that device (device current).
cudaError_t setup_device(int dev, int D, int bs, void **scratch, int *max_workers) {
    std::lock_guard<std::mutex> lock(g_setup_mu);
    if (!g_scratch_ptr[dev]) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_decode_scratch);
        if (e != cudaSuccess) return e;
        g_scratch_ptr[dev] = p;
    }
    int &mw = g_max_workers[dev][dim_index(D)];
    if (mw == 0) {
        mw = tllm::decode_max_workers(dev, D, bs);
        if (mw <= 0) {
            mw = 0;
            return cudaErrorInvalidConfiguration;
        }
    }
    *scratch = g_scratch_ptr[dev];
    *max_workers = mw;
    return cudaSuccess;
}

thread_local std::string g_static_error;

int fail(int status, const std::string &msg) {
    g_static_error = msg;
    return status;
}

}  // namespace

extern "C" int tl_decode_attention_static(const tl_paged_view *view, int layer, const void *q,
                                          void *o, const int *table_rows, const int *seq_lens,
                                          int num_seqs, float scale, tl_stream_t stream_,
                                          char *error_message, int error_message_size) {
    g_static_error.clear();
    auto ret = [&](int st) {
        if (st != TL_OK && error_message && error_message_size > 0) {
            const size_t n = std::min<size_t>(g_static_error.size(), (size_t)error_message_size - 1);
            std::copy(g_static_error.begin(), g_static_error.begin() + (long)n, error_message);
            error_message[n] = '\0';
        }
        return st;
    };
    if (!view) return ret(fail(TL_ERR_INVALID_ARG, "decodeAttentionStatic: view is null"));
    const tl_paged_view &v = *view;
    const int D = v.head_dim, Hkv = v.num_kv_heads, Hq = v.num_q_heads, bs = v.block_size;
    if (!(D == 64 || D == 128 || D == 256) || !(bs == 16 || bs == 32) || Hkv <= 0 || Hq <= 0 ||
        Hq % Hkv != 0 || Hq / Hkv > 8 || v.num_layers <= 0 || v.num_blocks <= 0 ||
        v.bt_stride <= 0 || v.num_rows <= 0 ||
        (v.layout != TL_LAYOUT_TOKEN_MAJOR && v.layout != TL_LAYOUT_HEAD_MAJOR))
        return ret(fail(TL_ERR_UNSUPPORTED,
                        "decodeAttentionStatic: supported shapes are head_dim 64/128/256, "
                        "block_size 16/32, query group 1..8, a valid layout, num_rows > 0"));
    if (layer < 0 || layer >= v.num_layers)
        return ret(fail(TL_ERR_INVALID_ARG, "decodeAttentionStatic: Invalid layer_idx: " +
                                                std::to_string(layer)));
    if (num_seqs < 0 || num_seqs > tllm::kMaxDecodeSeqs)
        return ret(fail(TL_ERR_INVALID_ARG,
                        "decodeAttentionStatic: num_seqs must be in 0.." +
                            std::to_string(tllm::kMaxDecodeSeqs)));
    if (num_seqs == 0) return ret(TL_OK);
    if (!v.pool || !v.block_tables || !q || !o || !table_rows || !seq_lens)
        return ret(fail(TL_ERR_INVALID_ARG, "decodeAttentionStatic: a pointer argument is null"));
    if (((uintptr_t)q & 3u) || ((uintptr_t)o & 3u) || ((uintptr_t)v.pool & 15u))
        return ret(fail(TL_ERR_INVALID_ARG,
                        "decodeAttentionStatic: q/o must be 4-byte and pool 16-byte aligned"));
    const unsigned long long rows = 2ull * v.num_layers * (unsigned long long)v.num_blocks *
                                    (unsigned long long)(v.layout == TL_LAYOUT_HEAD_MAJOR ? Hkv : bs);
    if (rows >= 0x7fffffffull)
        return ret(fail(TL_ERR_UNSUPPORTED, "decodeAttentionStatic: pool has more than 2^31 rows"));

    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return ret(fail(TL_ERR_CUDA, "decodeAttentionStatic: no usable current device"));
    void *scratch = nullptr;
    int max_workers = 0;
    e = setup_device(dev, D, bs, &scratch, &max_workers);
    if (e != cudaSuccess)
        return ret(fail(TL_ERR_CUDA, std::string("decodeAttentionStatic: set-up failed: ") +
                                         cudaGetErrorString(e)));

    const int G = Hq / Hkv;
    const size_t per_worker = 2ull * G * (size_t)tllm::partial_row_floats(D) * sizeof(float);
    const long long cap_workers = (long long)((kStaticScratchBytes - kErrorSlotBytes) / per_worker);

    tllm::DecodeArgs a{};
    a.g.pool = v.pool;
    a.g.num_blocks = v.num_blocks;
    a.g.num_layers = v.num_layers;
    a.g.num_kv_heads = Hkv;
    a.g.head_dim = D;
    a.g.block_size = bs;
    a.g.head_major = v.layout == TL_LAYOUT_HEAD_MAJOR ? 1 : 0;
    a.g.bt_stride = v.bt_stride;
    a.g.block_tables = const_cast<int *>(v.block_tables);
    a.g.err = v.error_word ? v.error_word : static_cast<int *>(scratch);
    a.q = q;
    a.o = o;
    a.partial = reinterpret_cast<float *>(static_cast<unsigned char *>(scratch) + kErrorSlotBytes);
    a.layer = layer;
    a.group = G;
    if (!(scale > 0.0f)) scale = 1.0f / std::sqrt((float)D);
    a.scale_log2 = scale * 1.4426950408889634f;
    a.nseq = num_seqs;
    a.prefix[0] = 0;
    cudaStream_t stream = (cudaStream_t)stream_;
    const long long row = (long long)Hq * D;
    for (int i = 0; i < num_seqs; ++i) {
        const int S = seq_lens[i];
        if (S < 0 || (long long)S > (long long)v.bt_stride * bs || table_rows[i] < 0 ||
            table_rows[i] >= v.num_rows)
            return ret(fail(TL_ERR_INVALID_ARG,
                            "decodeAttentionStatic: sequence " + std::to_string(i) +
                                " has a length outside 0..bt_stride*block_size or a table row outside "
                                "0..num_rows-1"));
        a.slot[i] = table_rows[i];
        a.len[i] = S;
    }
    long long real_tiles = 0;  // the per-unit overhead charge follows the tiles per worker
    for (int i = 0; i < num_seqs; ++i) real_tiles += (seq_lens[i] + tllm::kDecodeTile - 1) / tllm::kDecodeTile;
    a.vslots = tllm::unit_overhead_slots((long long)Hkv * real_tiles, std::min<long long>(max_workers, cap_workers));
    for (int i = 0; i < num_seqs; ++i)
        a.prefix[i + 1] = a.prefix[i] + tllm::unit_slots((seq_lens[i] + tllm::kDecodeTile - 1) / tllm::kDecodeTile, a.vslots);
    if (!v.error_word) {
        e = cudaMemsetAsync(scratch, 0, sizeof(int), stream);
        if (e != cudaSuccess)
            return ret(fail(TL_ERR_CUDA, std::string("decodeAttentionStatic: ") + cudaGetErrorString(e)));
    }
    for (int i = 0; i < num_seqs; ++i) {
        if (seq_lens[i] == 0) {
            e = cudaMemsetAsync(static_cast<uint16_t *>(o) + (long long)i * row, 0, (size_t)row * 2, stream);
            if (e != cudaSuccess)
                return ret(fail(TL_ERR_CUDA, std::string("decodeAttentionStatic: ") + cudaGetErrorString(e)));
        }
    }
    a.total_items = (long long)Hkv * a.prefix[num_seqs];
    if (a.total_items == 0) return ret(TL_OK);
    a.workers = (int)std::min<long long>({(long long)max_workers, a.total_items, cap_workers});
    if (a.workers < 1)
        return ret(fail(TL_ERR_UNSUPPORTED, "decodeAttentionStatic: split scratch too small for this shape"));

    alignas(64) unsigned char tmap[128];
    e = tllm::encode_pool_tensor_map(a.g, tmap);
    if (e != cudaSuccess)
        return ret(fail(TL_ERR_CUDA, "decodeAttentionStatic: tensor map encode failed"));
    e = tllm::launch_decode(a, tmap, stream);
    if (e != cudaSuccess)
        return ret(fail(TL_ERR_CUDA, std::string("decodeAttentionStatic: decode launch failed: ") +
                                         cudaGetErrorString(e)));
    if (a.workers > 1) {
        e = tllm::launch_merge(a, stream);
        if (e != cudaSuccess)
            return ret(fail(TL_ERR_CUDA, std::string("decodeAttentionStatic: merge launch failed: ") +
                                             cudaGetErrorString(e)));
    }
    return ret(TL_OK);
}
