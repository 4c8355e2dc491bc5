/*
 * tllm_kv.h — C-ABI of the B200 paged KV cache and GQA decode attention.
 *
 * This is the drop-in boundary for the hot path of AICL-Lab/tiny-llm:
 *   - the KVCacheManager API (include/tiny_llm/kv_cache.h:24-111 in the
 *     reference), re-implemented over a block pool with per-sequence block
 *     tables, and
 *   - the decode-attention call TransformerLayer::attention makes
 *     (kernels/attention.cuh:15-18, called at src/transformer.cpp:230-237).
 * The C++ facade tiny_llm::KVCacheManager (include/tiny_llm/kv_cache.h of
 * this repository) keeps the reference's C++ signatures on top of it.
 *
 * Conventions
 *   - Every function returns an int status (TL_OK = 0, negative = error) and
 *     never throws. The message of the last error on a handle is returned by
 *     tl_last_error(handle); tl_last_error(NULL) gives the last error of a
 *     failed tl_create on the calling thread.
 *   - Device pointers (K/V/Q/O) are owned by the caller; the pool, the block
 *     tables, the RoPE table and the split-K scratch are owned by the handle.
 *   - All device work is ordered on the caller's stream; no call blocks on
 *     the device except tl_sync_check and tl_destroy.
 *   - A handle is not thread-safe: one handle per GPU (per rank), driven from
 *     one host thread, as in the reference.
 *   - fp16 tensors are IEEE binary16 (the reference's `half`).
 */
#ifndef TLLM_KV_H
#define TLLM_KV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same type as cudaStream_t, without pulling in the CUDA headers. */
typedef struct CUstream_st *tl_stream_t;
typedef struct tl_cache tl_cache;

enum tl_status {
    TL_OK = 0,
    TL_ERR_INVALID_ARG = -1, /* bad pointer, size, layer index, ... */
    TL_ERR_NOT_FOUND = -2,   /* unknown sequence id ("not found") */
    TL_ERR_EXHAUSTED = -3,   /* no free sequence slot or no free block ("exhausted") */
    TL_ERR_OVERFLOW = -4,    /* append past the sequence's max_len ("overflow") */
    TL_ERR_CUDA = -5,        /* a CUDA runtime call failed */
    TL_ERR_NO_DEVICE = -6,   /* compute call on a handle without a CUDA device */
    TL_ERR_UNSUPPORTED = -7, /* shape outside what the kernels are built for */
    TL_ERR_DEVICE_FAULT = -8 /* a kernel reported a bounds/timeout error word */
};

enum tl_backend {
    TL_BACKEND_CUDA = 0,
    /* Bookkeeping only: the pool lives in host memory and every call that
     * would launch a kernel returns TL_ERR_NO_DEVICE. For testing the
     * allocator and the manager semantics on machines without a GPU. */
    TL_BACKEND_HOST_BOOKKEEPING = 1
};

enum tl_layout {
    /* block = [block_size][Hkv][D]: the first block of a layer holds tokens
     * 0..block_size-1 exactly as the reference's contiguous [pos][Hkv][D]
     * region (src/kv_cache.cpp:226), so tl_get_cache() readers keep working. */
    TL_LAYOUT_TOKEN_MAJOR = 0,
    /* block = [Hkv][block_size][D]: each (block, head) is one contiguous run. */
    TL_LAYOUT_HEAD_MAJOR = 1
};

/* Reference KVCacheConfig (include/tiny_llm/types.h:122-128) plus the paged
 * pool and RoPE fields. Zero-valued optional fields take the noted default. */
typedef struct {
    int num_layers;     /* L */
    int num_kv_heads;   /* Hkv (the reference's KVCacheConfig::num_heads) */
    int head_dim;       /* D: 64, 128 or 256 */
    int max_seq_len;    /* per-sequence cap on max_len */
    int max_batch_size; /* max concurrently allocated sequences */
    int block_size;     /* tokens per block; 0 -> 16. Must be 16 or 32 */
    long long num_blocks; /* pool blocks; 0 -> max_batch_size*ceil(max_seq_len/block_size) */
    int num_q_heads;    /* Hq for decode (multiple of Hkv); 0 -> num_kv_heads */
    float rope_theta;   /* RoPE base; used when rope_on_append != 0 */
    int rope_on_append; /* 1: rotate K (rotate-half) at its position while appending */
    int layout;         /* enum tl_layout */
    int backend;        /* enum tl_backend */
    int device;         /* CUDA device ordinal; -1 -> current device */
} tl_config;

typedef struct {
    long long num_blocks;      /* pool capacity in blocks */
    long long used_blocks;     /* blocks held by live sequences */
    long long free_blocks;     /* blocks on the free list */
    long long high_water;      /* max used_blocks seen */
    long long block_bytes;     /* bytes of one block over all layers, K and V */
    int active_sequences;
    int max_blocks_per_seq;
    long long kernel_launches; /* kernels this handle has launched so far */
} tl_pool_stats;

/* Fills *cfg with the defaults (reference KVCacheConfig defaults: 32 layers,
 * 32 heads, head_dim 128, max_seq_len 2048, batch 1; block 16; theta 1e4). */
void tl_config_init(tl_config *cfg);

/* KVCacheManager::create (reference include/tiny_llm/kv_cache.h:28,
 * src/kv_cache.cpp:8-59): validates, sizes and allocates the pool and zeroes
 * it. Errors: TL_ERR_INVALID_ARG ("invalid configuration"), TL_ERR_OVERFLOW
 * ("overflow"), TL_ERR_CUDA (allocation failed). */
int tl_create(const tl_config *cfg, tl_cache **out);
/* ~KVCacheManager (src/kv_cache.cpp:62-67). Synchronizes the device. */
void tl_destroy(tl_cache *cache);

const char *tl_last_error(const tl_cache *cache);
const char *tl_status_name(int status);

/* allocateSequence (kv_cache.h:42, kv_cache.cpp:91-119): max_len must be in
 * 1..max_seq_len ("Invalid max_len"); ids are monotonic and never reused.
 * Takes one block eagerly; more blocks are taken as the sequence grows. */
int tl_allocate_sequence(tl_cache *cache, int max_len, int *seq_id);
/* releaseSequence (kv_cache.h:46, kv_cache.cpp:121-137): returns the
 * sequence's blocks to the free list. */
int tl_release_sequence(tl_cache *cache, int seq_id);
/* Growth: makes sure blocks exist for the first new_len tokens (new_len <=
 * max_len). No reference counterpart; the reference reserves max_seq_len. */
int tl_reserve(tl_cache *cache, int seq_id, int new_len);

/* getCacheChecked (kv_cache.h:54, kv_cache.cpp:139-157): K and V base
 * pointers of the sequence's first block in layer `layer`. With the
 * token-major layout they address tokens 0..block_size-1 as [pos][Hkv][D]. */
int tl_get_cache(tl_cache *cache, int seq_id, int layer, void **k, void **v);

/* appendKV (kv_cache.h:61-62, kv_cache.cpp:168-238): writes num_tokens rows
 * k/v [num_tokens][Hkv][D] (device, fp16) of one layer at positions
 * current_len.. of the sequence, growing its block list as needed; K is
 * rotated by RoPE when the handle was created with rope_on_append. Does not
 * advance the visible length. Errors: "is null", "num_tokens must be
 * positive", "Invalid layer_idx", "not found", "overflow", "exhausted". */
int tl_append_kv(tl_cache *cache, int seq_id, int layer, const void *k, const void *v,
                 int num_tokens, tl_stream_t stream);

/* Fused decode append: one token per sequence for every layer in ONE kernel.
 * k/v: [L][num_seqs][Hkv][D] fp16 on the device; seq_ids: host array. Each
 * token goes to position current_len of its sequence. */
int tl_append_kv_all_layers(tl_cache *cache, const int *seq_ids, int num_seqs, const void *k,
                            const void *v, tl_stream_t stream);

/* advanceSeqLen (kv_cache.h:67, kv_cache.cpp:240-259): current_len =
 * min(current_len + n, max_len); n <= 0 is an error and changes nothing. */
int tl_advance_seq_len(tl_cache *cache, int seq_id, int num_tokens);

/* getSeqLen / hasSequence / memory statistics / getActiveSequenceCount
 * (kv_cache.h:70-84). Memory figures count whole blocks. */
int tl_get_seq_len(const tl_cache *cache, int seq_id);
int tl_has_sequence(const tl_cache *cache, int seq_id);
size_t tl_used_memory(const tl_cache *cache);
size_t tl_total_memory(const tl_cache *cache);
size_t tl_free_memory(const tl_cache *cache);
int tl_active_sequence_count(const tl_cache *cache);
int tl_get_config(const tl_cache *cache, tl_config *cfg);

/* Block table of a sequence (host copy): writes up to cap block ids. */
int tl_get_block_table(const tl_cache *cache, int seq_id, int *blocks, int cap, int *count);
int tl_get_pool_stats(const tl_cache *cache, tl_pool_stats *stats);

/* Device base of the pool [L][2][num_blocks][block] and the element count,
 * for inspection tools and tests. */
int tl_get_pool(const tl_cache *cache, void **base, size_t *elements);

/* Replacement for kernels::attention_decode (kernels/attention.cuh:15-18) as
 * called from TransformerLayer::attention (src/transformer.cpp:230-237):
 * GQA decode attention of layer `layer` for num_seqs sequences over their
 * paged K/V. q: [num_seqs][Hq][D] fp16 (device), o: [num_seqs][Hq][D] fp16
 * (device), seq_ids: host array. Each sequence attends to its written
 * tokens: current_len + the tokens appended since the last advance (the
 * reference's getSeqLen()+1 in decode). A sequence with no tokens gets
 * zeros. scale <= 0 -> 1/sqrt(D). Split-K with a merge pass over the
 * handle's scratch. */
int tl_decode_attention(tl_cache *cache, int layer, const void *q, void *o, const int *seq_ids,
                        int num_seqs, float scale, tl_stream_t stream);

/* The decode branch of TransformerLayer::attention (reference
 * src/transformer.cpp:222-237: appendKV, then attention_decode over
 * getSeqLen()+1 tokens) for a batch of sequences with one new token each:
 * appends k_new/v_new ([num_seqs][Hkv][D] fp16, device) at each sequence's
 * current length in `layer` (RoPE on K when the handle rotates on append),
 * then decodes q ([num_seqs][Hq][D]) into o over len + 1 tokens, with Q
 * rotated by the same table at the same position when K is. The caller
 * advances every sequence once after its last layer (tl_advance_seq_len).
 * Errors as tl_append_kv_all_layers and tl_decode_attention. */
int tl_attention_step(tl_cache *cache, int layer, const void *q, const void *k_new, const void *v_new,
                      void *o, const int *seq_ids, int num_seqs, float scale, tl_stream_t stream);

/* Causal prefill attention over the paged cache, replacing
 * kernels::attention_prefill (reference kernels/attention.cu:131-237, called
 * at src/transformer.cpp:238-242 over the prompt's own buffers): after the
 * prompt's K/V are appended (tl_append_kv, any number of tokens), sequence
 * i's num_tokens[i] query rows are its last num_tokens[i] written tokens;
 * each attends the sequence's tokens up to its own position (so a prompt
 * that continues a cached prefix sees the prefix), with Q rotated at its
 * position when K is rotated on append. q/o: [sum(num_tokens)][Hq][D] fp16,
 * sequence after sequence. head_dim 64 or 128. */
int tl_prefill_attention(tl_cache *cache, int layer, const void *q, void *o, const int *seq_ids,
                         const int *num_tokens, int num_seqs, float scale, tl_stream_t stream);

/* Q/K/V projections of one decode token per sequence with K and V written
 * straight into the cache, replacing the decode step's three
 * kernels::w8a16_matmul calls and its appendKV (reference
 * src/transformer.cpp:209-226; kernels/w8a16_matmul.cu:119-235;
 * src/kv_cache.cpp:206-233). x: [num_seqs][hidden] fp16 (row i = sequence
 * seq_ids[i]); wq/wk/wv: int8 [hidden][Hq*D] / [hidden][Hkv*D] row-major,
 * sq/sk/sv: fp16 [hidden/group_size][same columns] (the reference's
 * QuantizedWeight layout, include/tiny_llm/types.h:33-44). Each projection is
 * sum_k x[k] * w[k][n] * scale[k/group_size][n] accumulated in fp32 and
 * rounded to fp16; K and V rows are written at each sequence's current
 * length in `layer` (the length does not advance, as tl_append_kv), and
 * q_out ([num_seqs][Hq*D] fp16) receives Q; both Q and K are rotated at that
 * position when the handle rotates on append (then decode with
 * tl_decode_attention, which does not rotate Q). head_dim 64/128, hidden a
 * multiple of 128, group_size 16/32/64/128; x, q_out and the scales 16-byte
 * aligned, the weights 4-byte. Calls on different streams must not overlap
 * (they share the handle's split-K scratch). Errors as tl_append_kv. */
int tl_project_qkv_append(tl_cache *cache, int layer, const void *x, int hidden, const int8_t *wq,
                          const void *sq, const int8_t *wk, const void *sk, const int8_t *wv, const void *sv,
                          int group_size, const int *seq_ids, int num_seqs, void *q_out, tl_stream_t stream);

/* Weight repacking for tl_project_qkv_append_packed, done once at model load
 * (no reference counterpart: the reference reads QuantizedWeight as stored).
 * w: int8 [hidden][n] row-major as above; packed: a device buffer of the same
 * hidden * n bytes, not overlapping w. Layout: column tile t (128 columns),
 * 64-row block b is 8192 contiguous bytes at (t * hidden / 64 + b) * 8192,
 * its row r's 16-byte chunk c at r * 128 + (c ^ (r % 8)) * 16. hidden and n
 * multiples of 128, both pointers 16-byte aligned. Asynchronous on `stream`.
 * No handle: errors are read with tl_last_error(NULL). */
int tl_qkv_pack_weight(const int8_t *w, int hidden, int n, int8_t *packed, tl_stream_t stream);

/* tl_project_qkv_append with wq/wk/wv packed by tl_qkv_pack_weight (the
 * scales as before): the same outputs, bit for bit, with every weight read
 * a contiguous 8 KB copy. Only for the shapes the tcgen05 kernel takes: Q,
 * K and V widths multiples of 128, group_size 32/64/128; TL_ERR_UNSUPPORTED
 * otherwise. */
int tl_project_qkv_append_packed(tl_cache *cache, int layer, const void *x, int hidden, const int8_t *wq,
                                 const void *sq, const int8_t *wk, const void *sk, const int8_t *wv, const void *sv,
                                 int group_size, const int *seq_ids, int num_seqs, void *q_out, tl_stream_t stream);

/* Next-token sampling on the device for `rows` rows of fp16 logits
 * (row_stride elements apart; 0 shares one row), replacing the host round
 * trip of InferenceEngine::sampleFromHidden (reference
 * src/inference_engine.cpp:296-307: stream synchronize, logits copied to the
 * host, the host samplers of :330-490). The token ids go to tokens_out
 * (device int32 [rows]); nothing is synchronised. Strategy as the
 * reference's sample() (GenerationConfig, include/tiny_llm/types.h:96-102):
 * do_sample == 0: greedy (first index of the largest logit); otherwise
 * top_p < 1: top-p (p clamped to [1e-5, 1]); top_k > 0: top-k (k clamped to
 * [1, vocab]); else temperature; T clamped to >= 1e-5. The draw is an
 * inverse CDF over the candidates in descending logit order (ties by
 * ascending index) with a uniform of (seed, step, row) from splitmix64: the
 * same distribution as the reference's std::discrete_distribution, not the
 * same draws. No handle: errors are read with tl_last_error(NULL). */
int tl_sample_tokens(const void *logits, long long row_stride, int rows, int vocab, int do_sample,
                     float temperature, int top_k, float top_p, unsigned long long seed, unsigned long long step,
                     int *tokens_out, tl_stream_t stream);

/* ---- Head-sharded decode across the GPUs of one node -------------------
 * No reference counterpart (the reference is single-GPU). With KV heads
 * split over `world` ranks (one process per GPU), each rank's decode writes
 * its output slice into its own gather area; the last CTA of the launch
 * publishes an epoch in this rank's flag (one system-scope release) and then
 * pulls every other rank's slice over NVLink (CUDA IPC mappings, plain
 * loads) as soon as that rank's flag shows the epoch. Gather area layout, on
 * every rank: [world][num_seqs][Hq_local][D] fp16 at out_offset
 * (rank-major). */
#define TL_IPC_HANDLE_BYTES 64
/* Allocates this rank's gather region (gather_bytes of outputs plus flags)
 * and writes its IPC handle (TL_IPC_HANDLE_BYTES) to ipc_handle, for the
 * caller to exchange with the other ranks. */
int tl_peer_init(tl_cache *cache, int rank, int world, size_t gather_bytes, void *ipc_handle);
/* Opens every other rank's region from ipc_handles ([world][64] bytes). */
int tl_peer_connect(tl_cache *cache, const void *ipc_handles);
/* Device address and size of this rank's gathered-output area. */
int tl_peer_buffer(const tl_cache *cache, void **gathered, size_t *bytes);
/* Limit, in seconds, of each wait for a peer's flag in later
 * tl_decode_attention_peer calls (<= 0: the built-in 10 s; at most 600). A
 * wait that runs out stops the gather, leaves the other ranks' slices
 * unwritten and is reported by tl_sync_check as TL_ERR_DEVICE_FAULT ("bounded
 * wait timed out"); the handle stays usable. No reference counterpart. */
int tl_set_peer_wait_limit(tl_cache *cache, double seconds);
/* Testing hook: uses `region`, device memory of this process laid out as a
 * peer region ([flags 256 B][gathered outputs], 256-byte aligned), as rank
 * `rank`'s region instead of an IPC mapping, so the publish/pull protocol
 * (and a peer that never publishes) can be exercised on one GPU. Once every
 * rank of the world has a region the handle counts as connected. */
int tl_debug_peer_attach(tl_cache *cache, int rank, void *region);
/* tl_decode_attention for this rank's heads, all ranks calling it for the
 * same layer with the same out_offset, num_seqs and `epoch` (a value that
 * increases call to call). This rank's [num_seqs][Hq][D] slice lands at
 * out_offset + rank*slice of its gather area (16-byte aligned offset, at
 * most 256 sequences); when the call's kernels finish (stream order), the
 * area holds every rank's slice. Waits for peers are bounded (10 s; a
 * timeout is reported by tl_sync_check as TL_ERR_DEVICE_FAULT). */
int tl_decode_attention_peer(tl_cache *cache, int layer, const void *q, const int *seq_ids,
                             int num_seqs, float scale, size_t out_offset, unsigned epoch,
                             tl_stream_t stream);

/* A paged KV pool that lives in memory the caller owns, laid out as the
 * handle's pool: fp16 [num_layers][2 (K,V)][num_blocks][block], each block
 * [block_size][Hkv][D] (token-major) or [Hkv][block_size][D] (head-major);
 * block_tables is int32 [num_rows][bt_stride] on the device, entry j of a
 * row being the block that holds tokens j*block_size .. j*block_size+bs-1. */
typedef struct {
    void *pool;
    const int *block_tables;
    int *error_word;      /* optional device int: kernels OR error bits into it */
    long long num_blocks;
    int num_layers, num_kv_heads, num_q_heads, head_dim, block_size, layout, bt_stride;
    int num_rows;         /* rows of block_tables; every table row used must be below it */
} tl_paged_view;

/* Decode attention that allocates nothing. No counterpart in the reference:
 * it exists for callers that cannot call cudaMalloc when they decode — an
 * engine whose device memory all comes from its own arena or caching
 * allocator, or a path that must not risk the implicit device
 * synchronisation of cudaMalloc/cudaFree. Everything is the caller's:
 * the pool and block tables (`view`), q/o ([num_seqs][Hq][D] fp16, device),
 * and, on the host, table_rows[i] (the block-table row of sequence i, in
 * 0..num_rows-1) and seq_lens[i] (tokens it attends). The math and output are those of
 * tl_decode_attention. The split-K scratch is a file-scope device array of
 * 8 MiB inside this library, present on every GPU that loads it until the
 * process exits; num_seqs above 256, or a shape whose split partials cannot
 * fit it, are rejected with an error. All calls share that array: calls that
 * overlap on the GPU race, so order them on one stream. The first call on
 * each device does a one-time set-up (looks up the array's address, sets
 * the kernel's shared-memory limit); make it before any stream capture.
 * On error, a message is copied into error_message (if non-NULL). */
int tl_decode_attention_static(const tl_paged_view *view, int layer, const void *q, void *o,
                               const int *table_rows, const int *seq_lens, int num_seqs,
                               float scale, tl_stream_t stream, char *error_message,
                               int error_message_size);

/* Synchronizes `stream`, then reads and clears the handle's device error
 * word; returns TL_ERR_DEVICE_FAULT (with a message) if a kernel recorded
 * an out-of-range block/position or a wait that gave up. */
int tl_sync_check(tl_cache *cache, tl_stream_t stream);

/* Host-side RoPE table with the same math the handle uploads:
 * freq_i = theta^(-2i/D) in double, cos/sin(pos*freq_i) in double, rounded
 * to float; cos_t/sin_t are [max_pos][D/2]. Useful for rotating Q. */
void tl_rope_table(float *cos_t, float *sin_t, int max_pos, int head_dim, float theta);

/* Shuffles the free list so later allocations hand out blocks in a random
 * order (the ragged benchmark's "block tables randomly permuted over a
 * shared pool"). No reference counterpart. */
int tl_permute_free_blocks(tl_cache *cache, unsigned long long seed);

/* Testing hook: the nth storage allocation from now fails as if cudaMalloc
 * had failed (0 disables). Used by the failure-path tests. */
int tl_debug_inject_alloc_failure(int nth);

/* Library version string. */
const char *tl_version(void);

#ifdef __cplusplus
}
#endif
#endif
