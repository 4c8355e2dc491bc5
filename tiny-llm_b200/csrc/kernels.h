// Launch interface between the host manager (paged_kv.cpp) and the sm_100a
// kernels (kv_append.cu, paged_decode.cu). Argument blocks are passed to the
// kernels by value, so every per-call array here is bounded to keep a launch
// under the 4 KiB classic kernel-parameter limit; the host splits larger
// batches into several launches.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace tllm {

// Device error word bits (atomicOr'd by kernels, read by tl_sync_check).
enum DeviceErrorBits : int {
    kErrBlockRange = 1 << 0,   // a block id outside [0, num_blocks)
    kErrPosRange = 1 << 1,     // a position outside the RoPE table / sequence
    kErrWaitTimeout = 1 << 2,  // an mbarrier wait gave up (bounded spin)
};

constexpr int kMaxAppendRows = 256;
constexpr int kMaxDeltas = 96;
constexpr int kMaxDecodeSeqs = 256;
constexpr int kMaxPeers = 8;  // GPUs of one node in a head-sharded group
constexpr size_t kPeerFlagBytes = 256;  // flags area at the start of a peer region
// Decode work item: 16 tokens of one KV head (a block of 32 is two items).
constexpr int kDecodeTile = 16;
// Units cut into more pieces than this are merged by the wide merge pass.
constexpr int kInKernelMergeMaxPieces = 12;
// Work slots charged to each (sequence, kv_head) unit on top of its tiles:
// the unit's fixed cost (Q load, finalize, output) in tile-equivalents, so
// that the stream-K split balances time, not just tiles. A call with few
// tiles per worker (a batch split over many GPUs) charges more: there the
// fixed cost is a larger share of each worker's time.
constexpr int kUnitOverheadSlots = 2;
constexpr int kUnitOverheadSlotsFew = 4;
constexpr int kFewTilesPerWorker = 128;
inline int unit_overhead_slots(long long tiles, long long workers) {
    return tiles < kFewTilesPerWorker * workers ? kUnitOverheadSlotsFew : kUnitOverheadSlots;
}
inline int unit_slots(int tiles, int vslots) { return tiles > 0 ? tiles + vslots : 0; }

// Pool geometry shared by every kernel.
struct PoolGeom {
    void *pool;             // fp16 [L][2][num_blocks][block]
    long long num_blocks;   // NB
    int num_layers;         // L
    int num_kv_heads;       // Hkv
    int head_dim;           // D
    int block_size;         // bs
    int head_major;         // 0: block = [bs][Hkv][D]; 1: [Hkv][bs][D]
    int bt_stride;          // ints per block-table row (max blocks per sequence)
    int *block_tables;      // device [max_batch][bt_stride]
    int *err;               // device error word
};

// One append launch: `nrows` token rows for `num_layers` consecutive layers.
struct AppendArgs {
    PoolGeom g;
    const void *k;          // fp16 rows of [Hkv][D]
    const void *v;
    const float *rope_cos;  // [rope_max_pos][D/2] or nullptr (no RoPE)
    const float *rope_sin;
    int rope_max_pos;
    int layer0;             // first destination layer
    int num_layers;         // layers written (grid.y)
    int nrows;              // rows in this launch (grid.x)
    long long src_layer_stride;  // elements between layers in k/v
    long long src_row_stride;    // elements between rows in k/v
    int ndeltas;            // block-table updates applied by block (0,0)
    int delta_slot[kMaxDeltas];
    int delta_idx[kMaxDeltas];
    int delta_block[kMaxDeltas];
    int row_block[kMaxAppendRows];  // destination block of each row
    int row_pos[kMaxAppendRows];    // token position of each row
};

// Block-table updates alone (used when a decode finds updates pending).
struct DeltaArgs {
    int *block_tables;
    int bt_stride;
    int ndeltas;
    int delta_slot[kMaxDeltas];
    int delta_idx[kMaxDeltas];
    int delta_block[kMaxDeltas];
};

// One decode launch over up to kMaxDecodeSeqs sequences of one layer.
// Work = (sequence, kv_head, block) items ordered sequence-major, then
// kv_head, then block; worker w (one warp) owns the contiguous item range
// [w*W/V, (w+1)*W/V) (stream-K split), W = total items, V = workers.
struct DecodeArgs {
    PoolGeom g;
    const void *q;          // fp16 [nseq][Hq][D]
    void *o;                // fp16 [nseq][Hq][D]
    float *partial;         // [V][2][G][D+4] fp32 split partials (acc[D], m, l, pad)
    int *counters;          // [nseq][Hkv] zeroed tickets: the last worker of a cut
                            // unit merges it in-kernel; nullptr -> launch_merge pass
    // Head-sharded peer mode (ndst > 0): outputs go to out_dst[r] instead of
    // o (the host passes this rank's slice of its own gather area); the last
    // CTA of the merge pass stores `epoch` to flag_dst[r] (this rank's flag).
    // done_counter is a zeroed ticket, rearmed by the last CTA.
    int ndst;
    void *out_dst[kMaxPeers];
    unsigned *flag_dst[kMaxPeers];
    unsigned epoch;
    int *done_counter;
    // ... and the merge pass's last CTA then pulls the other ranks' slices:
    // peer_base[r] = rank r's region (this rank's own at [rank]); slices sit
    // at gather_off + r * slice_bytes in every region.
    const unsigned char *peer_base[kMaxPeers];
    int world, rank;
    unsigned long long gather_off, slice_bytes;
    unsigned long long peer_wait_ns;  // limit of each peer-flag wait; 0 -> the built-in 10 s
    int layer;
    int group;              // G = Hq / Hkv
    float scale_log2;       // softmax scale * log2(e)
    // Non-null: Q is rotated by this RoPE table ([rope_max_pos][D/2] fp32) at
    // each sequence's newest position (len - 1) before use, rounded as the
    // append kernel rounds K.
    const float *rope_cos;
    const float *rope_sin;
    int rope_max_pos;
    int nseq;
    long long total_items;  // W
    int workers;            // V
    int vslots;             // virtual slots per unit (unit_overhead_slots)
    int slot[kMaxDecodeSeqs];     // block-table row of each sequence
    int len[kMaxDecodeSeqs];      // attended tokens of each sequence
    int prefix[kMaxDecodeSeqs + 1];  // prefix sums of unit_slots(tiles) per sequence
};

// One causal prefill launch over up to kMaxPrefillSeqs sequences of one
// layer: sequence b's ntok[b] query rows (packed in q/o from row row_off[b],
// [rows][Hq][D] fp16) sit at positions [written[b] - ntok[b], written[b])
// and attend the sequence's tokens up to their own position. CTA x of the
// grid serves sequence b for cta_prefix[b] <= x < cta_prefix[b + 1], one CTA
// per 64 (query, head) rows (group padded to group_pad); grid.y = KV head.
constexpr int kMaxPrefillSeqs = 64;
struct PrefillArgs {
    PoolGeom g;
    const void *q;
    void *o;
    const float *rope_cos;  // non-null: Q rotated at each row's position
    const float *rope_sin;
    int rope_max_pos;
    int layer;
    int group, group_pad;
    float scale_log2;
    int nseq;
    int slot[kMaxPrefillSeqs];
    int written[kMaxPrefillSeqs];
    int ntok[kMaxPrefillSeqs];
    int row_off[kMaxPrefillSeqs];
    int cta_prefix[kMaxPrefillSeqs + 1];
};

// Sizes the kernels need from the host.
inline int partial_row_floats(int head_dim) { return head_dim + 4; }
int decode_workers_per_cta();
int decode_max_workers(int device, int head_dim, int block_size);

cudaError_t launch_append(const AppendArgs &a, cudaStream_t s);
cudaError_t launch_apply_deltas(const DeltaArgs &a, cudaStream_t s);
// Encodes the tensor map once per pool (stored opaque, 128 bytes).
cudaError_t encode_pool_tensor_map(const PoolGeom &g, void *tmap_out128);
// A 2-D tensor map (128-byte swizzle, zero fill out of bounds) over a
// row-major [outer][inner] array of uint8 or fp16 with rows row_bytes apart.
cudaError_t encode_tensor_map_2d(void *tmap_out128, bool fp16, const void *base, unsigned long long inner,
                                 unsigned long long outer, unsigned long long row_bytes, unsigned box_inner,
                                 unsigned box_outer);
cudaError_t launch_decode(const DecodeArgs &a, const void *tmap128, cudaStream_t s);
cudaError_t launch_merge(const DecodeArgs &a, cudaStream_t s);
// One fused Q/K/V projection + append launch (decode: one token per row).
constexpr int kMaxQkvRows = 64;
struct QkvArgs {
    PoolGeom g;
    const void *x;           // fp16 [rows][K] activations
    const int8_t *w[3];      // Q, K, V weights: int8 [K][n[i]] row-major, or
                             // tile-blocked (qkv_pack_weight) when w_packed
    int w_packed;            // tcgen05 kernel only
    const void *sc[3];       // fp16 scales [K / group][n[i]]
    int n[3];                // Hq*D, Hkv*D, Hkv*D
    int K, group, rows;
    int num_q_heads;
    int ksplit, kchunk;      // K split over ksplit CTAs of kchunk (a multiple of qkv_k_block())
    void *q_out;             // fp16 [rows][Hq*D]
    const float *rope_cos;   // RoPE on Q and K at each row's position, or nullptr
    const float *rope_sin;
    int rope_max_pos;
    int layer;
    float *partial;          // fp32 [Hq + 2 Hkv][qkv_rows_padded(rows)][D], zero between launches
    int *counters;           // [Hq + 2 Hkv], zero between launches
    int row_block[kMaxQkvRows];
    int row_pos[kMaxQkvRows];
};

// Token sampling, one cluster of CTAs per row of logits.
struct SampleArgs {
    const void *logits;       // fp16 [rows] rows of `vocab`, row_stride elements apart
    long long row_stride;
    int rows, vocab;
    int mode;                 // 0 greedy, 1 top-k (temperature: k = vocab), 2 top-p
    float temperature;        // clamped (>= 1e-5)
    int top_k;                // clamped to [1, vocab]
    float top_p;              // clamped to [1e-5, 1]
    unsigned long long seed, step;
    int *tokens;              // device [rows]
};
cudaError_t launch_sample(const SampleArgs &a, cudaStream_t s);
int sample_max_vocab();  // largest vocabulary a row may have

int prefill_tc_rows_per_cta();
cudaError_t launch_prefill_tc(const PrefillArgs &a, const void *tmap128, cudaStream_t s);
int qkv_k_block();
int qkv_rows_padded(int rows);  // the kernel's row tile for a launch of `rows` rows
cudaError_t launch_qkv_append(const QkvArgs &a, cudaStream_t s);
// The tcgen05 variant (qkv_append_tc.cu): weight columns in tiles of 128
// (Q, K and V each a multiple of 128 columns), group 32/64/128, weights
// 16-byte aligned, ksplit <= 16. partial: fp32 [columns / 128]
// [qkv_tc_rows_padded][128], counters: [columns / 128], both zero between
// launches (the last CTA of a tile zeroes what it read). qkv_tc_split picks the
// split of K for a launch of `rows` rows; false when no split keeps the
// group accumulators within TMEM (the mma.sync kernel runs instead).
bool qkv_tc_supported(int head_dim, int group, int nq, int nkv, int hidden);
int qkv_tc_rows_padded(int rows);
bool qkv_tc_split(int hidden, int group, int rows, int tiles, int num_sms, int *ksplit, int *kchunk);
cudaError_t launch_qkv_append_tc(const QkvArgs &a, cudaStream_t s);
// Tile-blocked copy of one int8 weight [K][n] (K a multiple of 64, n of 128,
// both pointers 16-byte aligned, not overlapping): column tile t, 64-row
// block b is 8192 contiguous bytes at (t * K / 64 + b) * 8192, row r's
// 16-byte chunk c at r * 128 + ((c ^ (r % 8)) * 16), the order in which a
// 2-D TMA load with 128-byte swizzle leaves the same tile in shared memory.
cudaError_t launch_qkv_pack_weight(const int8_t *w, int K, int n, int8_t *out, cudaStream_t s);


}  // namespace tllm
