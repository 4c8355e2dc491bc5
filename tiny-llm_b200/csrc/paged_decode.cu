// Split-K (flash-decoding) GQA decode attention over the paged KV pool, and
// the merge pass, for sm_100a.
//
// Replaces kernels::attention_decode (reference kernels/attention.cu:11-128),
// which runs one CTA per (batch, head) over a contiguous [H][S][D] cache,
// keeps every score in shared memory and re-reads K/V once per query head.
//
// Work decomposition (stream-K). The work of one call is the list of items
// (sequence b, kv_head h, tile t) in sequence-major order, one item = 16
// tokens of one KV head. Each WARP is an independent worker that owns one
// contiguous slice of that list, so every worker gets the same number of
// tiles whatever the sequence lengths (ragged batches stay balanced). A
// (sequence, kv_head) unit that a worker covers completely is finished in
// registers and written as fp16; a unit cut by a worker boundary leaves a
// partial (m, l, acc) in the split scratch, which the merge kernel combines.
//
// Data movement. Each worker owns a ring of NS stages in shared memory.
// Lane 0 issues TMA tile loads (cp.async.bulk.tensor, no multicast) for the
// K and V rows of the next tiles, addressed through the block table, with
// an evict-first L2 policy; an mbarrier per stage signals arrival. The tile
// is stored as 64-element (128-byte) half-rows with the 128-byte swizzle, so
// the ldmatrix reads below are bank-conflict free.
//
// Math (per 16-token tile, per warp). The query group (G <= 8 heads sharing
// one KV head) is the N=8 side of mma.sync m16n8k16:
//   S^T[t][g] = K[t][:] . Q[g][:]        (A = K from smem, B = Q in registers)
//   online softmax over t, per head g, in the exp2 domain (fp32)
//   O^T[d][g] += V^T[d][t] P^T[t][g]      (A = V^T via ldmatrix.trans,
//                                           B = P^T via movmatrix.trans)
// so each K/V tile is read from shared memory once for all G heads. fp16
// operands, fp32 accumulation, fp32 softmax state.
//
// Waits are bounded (globaltimer); a wait that gives up sets an error bit,
// drains the worker's own in-flight loads (bounded) and stops the worker.
#include <atomic>
#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include "kernels.h"
#include "ptx.cuh"

namespace tllm {
namespace {

constexpr int kTile = kDecodeTile;  // tokens per item
constexpr int kWarps = 4;          // workers per CTA
constexpr int kSmemBudget = 160 * 1024;
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s
// A peer rank may legitimately start a layer seconds later than this one
// (host-side skew at start-up); its flag wait gives up after 10 s.
constexpr uint64_t kPeerWaitLimitNs = 10000000000ull;
constexpr int kMergeThreads = 512;  // wide merge CTA: 2 per SM, so a grid fits one wave

template <int D>
struct Cfg {
    static constexpr int kNSub = D / 64;                  // 128-byte half-row tiles per row
    static constexpr int kSubBytes = kTile * 128;         // one [16][64] fp16 tile
    static constexpr int kStageBytes = 2 * kNSub * kSubBytes;  // K + V
    static constexpr int kNS0 = kSmemBudget / (kWarps * kStageBytes);
    static constexpr int kNS = kNS0 < 2 ? 2 : (kNS0 > 8 ? 8 : kNS0);
    static constexpr int kRingBytes = kNS * kStageBytes;
    static constexpr int kOutBytes = 8 * D * 2;           // one unit's fp16 output (G <= 8)
    static constexpr int kSmemBytes = kWarps * kRingBytes + kWarps * kOutBytes + kWarps * kNS * 8 + 1024;
    static constexpr int kKS = D / 16;                    // k-steps of the QK mma
};

// Floats per (worker, slot, head) partial row: acc[D], m, l, 2 pad, so rows
// start on 16-byte boundaries for the float4 reads of the merge.
template <int D>
constexpr int kPartialRow = D + 4;

// Position of a work slot. The work of a call is a list of slots in
// sequence-major, then kv-head order; unit (b, kvh) owns us =
// unit_slots(tiles of b) consecutive slots: vs = a.vslots virtual slots
// (no data: they stand for the unit's fixed cost — Q load, finalize — so
// that equal slot ranges mean equal time) followed by its real 16-token
// tiles. tile = slot - vs (< 0: virtual).
struct ItemPos {
    int b, kvh, slot, us, vs;
    long long unit_first;  // first slot of the unit (its virtual slots)
    __device__ __forceinline__ int tile() const { return slot - vs; }
    __device__ __forceinline__ int nb() const { return us - vs; }
    __device__ __forceinline__ long long real_first() const { return unit_first + vs; }
    __device__ __forceinline__ long long last() const { return unit_first + us - 1; }
};

// Output stores. Without peers the output goes to a.o; in the head-sharded
// peer mode every element is written to the same offset of each rank's
// gather buffer (this rank's slice), over NVLink for the remote ones.
__device__ __forceinline__ void store_out16(const DecodeArgs &a, long long off, uint4 v) {
    if (a.ndst == 0) {
        __half *p = static_cast<__half *>(a.o) + off;
        if ((reinterpret_cast<uintptr_t>(p) & 15) == 0) {
            *reinterpret_cast<uint4 *>(p) = v;
        } else {  // outputs are only promised 4-byte alignment
            uint32_t *q = reinterpret_cast<uint32_t *>(p);
            q[0] = v.x; q[1] = v.y; q[2] = v.z; q[3] = v.w;
        }
        return;
    }
    for (int r = 0; r < a.ndst; ++r) *reinterpret_cast<uint4 *>(static_cast<__half *>(a.out_dst[r]) + off) = v;
}

// 4 halves: one 8-byte store per peer (peer buffers are 16-byte aligned),
// two 4-byte stores locally (outputs are only promised 4-byte alignment).
__device__ __forceinline__ void store_out8(const DecodeArgs &a, long long off, __half2 lo, __half2 hi) {
    if (a.ndst == 0) {
        __half *p = static_cast<__half *>(a.o) + off;
        *reinterpret_cast<__half2 *>(p) = lo;
        *reinterpret_cast<__half2 *>(p + 2) = hi;
        return;
    }
    uint2 v;
    v.x = *reinterpret_cast<uint32_t *>(&lo);
    v.y = *reinterpret_cast<uint32_t *>(&hi);
    for (int r = 0; r < a.ndst; ++r) *reinterpret_cast<uint2 *>(static_cast<__half *>(a.out_dst[r]) + off) = v;
}

__device__ __forceinline__ void store_out4(const DecodeArgs &a, long long off, __half2 v) {
    if (a.ndst == 0) {
        *reinterpret_cast<__half2 *>(static_cast<__half *>(a.o) + off) = v;
        return;
    }
    for (int r = 0; r < a.ndst; ++r) *reinterpret_cast<__half2 *>(static_cast<__half *>(a.out_dst[r]) + off) = v;
}

// Raises this rank's flag on every peer once all of a launch's outputs are
// visible system-wide: called by each finishing participant; the last one
// (ticket == participants - 1) fences and publishes the epoch, then rearms.
__device__ __forceinline__ void fence_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// Publishes a launch's outputs in peer mode. Outputs are written to this
// GPU's own gather area; each participant (one thread, after a barrier that
// orders its outputs before it) takes a ticket with a gpu-scope release;
// the last one then performs ONE system-scope release store of the epoch
// into this rank's flag, so readers on other GPUs that acquire the flag see
// every participant's outputs (causality through the ticket chain).
__device__ __forceinline__ bool signal_peers(const DecodeArgs &a, int participants) {
    int old;
    asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], 1;" : "=r"(old) : "l"(a.done_counter) : "memory");
    if (old == participants - 1) {
        for (int r = 0; r < a.ndst; ++r)
            asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(a.flag_dst[r]), "r"(a.epoch) : "memory");
        *a.done_counter = 0;  // rearmed; the next launch is ordered after this one
        return true;
    }
    return false;
}

// After publishing, the last CTA gathers the other ranks' slices of the same
// call into this rank's gather area. Lanes of warp 0 poll one peer flag each
// over NVLink (relaxed polls, one acquire fence once every epoch is seen;
// bounded), then the whole CTA copies all peers' slices in one loop with
// independent 16-byte loads in flight. Publishing never waits, so two ranks
// can never wait on each other.
__device__ void pull_peer_slices(const DecodeArgs &a) {
    __shared__ int s_ok;
    constexpr int kBatch = 8;
    if (threadIdx.x < 32) {
        const int r = threadIdx.x;
        int ok = 1;
        if (r < a.world && r != a.rank) {
            const unsigned *flag = reinterpret_cast<const unsigned *>(a.peer_base[r]) + r;
            const uint64_t limit = a.peer_wait_ns ? a.peer_wait_ns : kPeerWaitLimitNs;
            const uint64_t t0 = ptx::globaltimer_ns();
            for (;;) {
                unsigned v;
                asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
                if ((int)(v - a.epoch) >= 0) break;
                if (ptx::globaltimer_ns() - t0 > limit) {
                    atomicOr(a.g.err, kErrWaitTimeout);
                    ok = 0;
                    break;
                }
                __nanosleep(64);
            }
        }
        ok = __all_sync(0xffffffffu, ok);
        if (threadIdx.x == 0) {
            asm volatile("fence.acq_rel.sys;" ::: "memory");
            s_ok = ok;
        }
    }
    __syncthreads();
    if (!s_ok) return;
    // all peers' slices as one index space of 16-byte chunks
    const size_t n16 = a.slice_bytes / 16;
    const size_t total = n16 * (size_t)(a.world - 1);
    const size_t stride = blockDim.x;
    unsigned char *local = const_cast<unsigned char *>(a.peer_base[a.rank]);
    for (size_t base = threadIdx.x; base < total; base += stride * kBatch) {
        uint4 v[kBatch];
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            const size_t i = base + j * stride;
            if (i < total) {
                int r = (int)(i / n16);
                r += r >= a.rank;  // skip this rank's own slice
                const size_t off = a.gather_off + (size_t)r * a.slice_bytes + (i % n16) * 16;
                v[j] = __ldcg(reinterpret_cast<const uint4 *>(a.peer_base[r] + off));
            }
        }
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            const size_t i = base + j * stride;
            if (i < total) {
                int r = (int)(i / n16);
                r += r >= a.rank;
                const size_t off = a.gather_off + (size_t)r * a.slice_bytes + (i % n16) * 16;
                *reinterpret_cast<uint4 *>(local + off) = v[j];
            }
        }
    }
}

// Rotates a lane's Q fragments by the RoPE table at position pos (rotate-half:
// element d pairs with d + D/2, which sits in k-step ks + D/32 of the same
// lane). Each product and sum is rounded separately (__fmul_rn, __fsub_rn,
// __fadd_rn) and the result converted to fp16 with round-to-nearest-even,
// the append kernel's sequence for K.
template <int D>
__device__ __forceinline__ void rope_q(uint32_t (&qf)[D / 16][2], const DecodeArgs &a, int pos, int tig) {
    constexpr int kKS = D / 16, kHalfD = D / 2;
    if (pos < 0 || pos >= a.rope_max_pos) {
        atomicOr(a.g.err, kErrPosRange);
        return;
    }
    const float *ct = a.rope_cos + (long long)pos * kHalfD;
    const float *st = a.rope_sin + (long long)pos * kHalfD;
#pragma unroll
    for (int ks = 0; ks < kKS / 2; ++ks) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int d = ks * 16 + j * 8 + 2 * tig;  // and d + 1, both < D/2
            const float2 c = *reinterpret_cast<const float2 *>(ct + d);
            const float2 sn = *reinterpret_cast<const float2 *>(st + d);
            const float2 x1 = __half22float2(*reinterpret_cast<const __half2 *>(&qf[ks][j]));
            const float2 x2 = __half22float2(*reinterpret_cast<const __half2 *>(&qf[ks + kKS / 2][j]));
            const __half2 r1 = __halves2half2(__float2half_rn(__fsub_rn(__fmul_rn(x1.x, c.x), __fmul_rn(x2.x, sn.x))),
                                              __float2half_rn(__fsub_rn(__fmul_rn(x1.y, c.y), __fmul_rn(x2.y, sn.y))));
            const __half2 r2 = __halves2half2(__float2half_rn(__fadd_rn(__fmul_rn(x2.x, c.x), __fmul_rn(x1.x, sn.x))),
                                              __float2half_rn(__fadd_rn(__fmul_rn(x2.y, c.y), __fmul_rn(x1.y, sn.y))));
            qf[ks][j] = *reinterpret_cast<const uint32_t *>(&r1);
            qf[ks + kKS / 2][j] = *reinterpret_cast<const uint32_t *>(&r2);
        }
    }
}

// Maps a flat item index to (sequence, kv_head, tile). prefix[] lives in the
// kernel's parameter space; the search is uniform across the warp.
__device__ __forceinline__ ItemPos locate(const DecodeArgs &a, long long w) {
    const int H = a.g.num_kv_heads;
    int lo = 0, hi = a.nseq - 1;
    while (lo < hi) {  // largest b with H*prefix[b] <= w
        const int mid = (lo + hi + 1) >> 1;
        if ((long long)H * a.prefix[mid] <= w) lo = mid;
        else hi = mid - 1;
    }
    ItemPos p;
    p.vs = a.vslots;
    p.b = lo;
    p.us = a.prefix[lo + 1] - a.prefix[lo];
    const int r = (int)(w - (long long)H * a.prefix[lo]);  // < H * us < 2^31
    p.kvh = r / p.us;
    p.slot = r - p.kvh * p.us;
    p.unit_first = (long long)H * a.prefix[lo] + (long long)p.kvh * p.us;
    return p;
}

__device__ __forceinline__ long long worker_start(long long v, long long W, long long V) {
    return v * W / V;
}

// Combines the partials of one cut unit (sequence b, kv head kvh) left by
// workers v_first..v_last and writes its fp16 output; one warp. A source
// stored the unit in slot 0 when the unit was its first piece (its range
// starts inside the unit), otherwise in slot 1. Lanes split the G heads
// (32/G' lanes per head, G' = G rounded up to a power of two) and each lane
// owns float4 chunks of D; sources are folded in with an online softmax
// merge, two per round with all their loads issued together, so the chain
// of L2 round trips is ~(number of sources)/2 long.
template <int D>
__device__ __forceinline__ void merge_unit(const DecodeArgs &a, long long unit_first, int b,
                                           int kvh, long long v_first, long long v_last,
                                           int lane) {
    constexpr int kRow = kPartialRow<D>;
    constexpr int kMaxChunks = D / 16;          // float4 chunks per lane at G' = 8
    constexpr int kPerRound = D <= 128 ? 2 : 1;  // sources per round (register budget)
    const long long W = a.total_items, V = a.workers;
    const int G = a.group, H = a.g.num_kv_heads, Hq = H * G;
    const int gp = G <= 1 ? 1 : (G <= 2 ? 2 : (G <= 4 ? 4 : 8));
    const int lpg = 32 / gp;                     // lanes per head
    const int g = lane / lpg, sub = lane % lpg;
    const int nchunks = (D / 4 + lpg - 1) / lpg;
    if (g >= G) return;
    float M = -INFINITY, L = 0.f;
    float4 O[kMaxChunks];
#pragma unroll
    for (int k = 0; k < kMaxChunks; ++k) O[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (long long v = v_first; v <= v_last; v += kPerRound) {
        float mv[kPerRound], lv[kPerRound];
        float4 xv[kPerRound][kMaxChunks];
#pragma unroll
        for (int r = 0; r < kPerRound; ++r) {
            const long long u = v + r;
            mv[r] = -INFINITY;
            lv[r] = 0.f;
            if (u <= v_last) {
                const int slot = worker_start(u, W, V) >= unit_first ? 0 : 1;
                const float *pb = a.partial + ((u * 2 + slot) * G + g) * (long long)kRow;
                mv[r] = __ldcg(pb + D);
                lv[r] = __ldcg(pb + D + 1);
#pragma unroll
                for (int k = 0; k < kMaxChunks; ++k) {
                    const int c = sub + k * lpg;
                    if (k < nchunks && c < D / 4) xv[r][k] = __ldcg(reinterpret_cast<const float4 *>(pb) + c);
                }
            }
        }
        float Mn = M;
#pragma unroll
        for (int r = 0; r < kPerRound; ++r) Mn = fmaxf(Mn, mv[r]);
        const float sc = ptx::ex2(M - Mn);
        float w[kPerRound];
#pragma unroll
        for (int r = 0; r < kPerRound; ++r) w[r] = (v + r <= v_last) ? ptx::ex2(mv[r] - Mn) : 0.f;
        L = L * sc;
#pragma unroll
        for (int r = 0; r < kPerRound; ++r) L += w[r] * lv[r];
#pragma unroll
        for (int k = 0; k < kMaxChunks; ++k) {
            if (k < nchunks) {
                float4 o = O[k];
                o.x *= sc; o.y *= sc; o.z *= sc; o.w *= sc;
#pragma unroll
                for (int r = 0; r < kPerRound; ++r) {
                    if (v + r <= v_last) {
                        o.x += w[r] * xv[r][k].x; o.y += w[r] * xv[r][k].y;
                        o.z += w[r] * xv[r][k].z; o.w += w[r] * xv[r][k].w;
                    }
                }
                O[k] = o;
            }
        }
        M = Mn;
    }
    const float inv = 1.f / L;
    const long long obase = ((long long)b * Hq + (long long)kvh * G + g) * D;
#pragma unroll
    for (int k = 0; k < kMaxChunks; ++k) {
        const int c = sub + k * lpg;
        if (k < nchunks && c < D / 4) {
            store_out8(a, obase + 4 * c, __floats2half2_rn(O[k].x * inv, O[k].y * inv),
                       __floats2half2_rn(O[k].z * inv, O[k].w * inv));
        }
    }
}

__device__ __forceinline__ long long worker_of_item(long long x, long long W, long long V) {
    return ((x + 1) * V + W - 1) / W - 1;  // largest v with worker_start(v) <= x
}

template <int D>
__global__ void __launch_bounds__(kWarps * 32, 1)
    paged_decode_kernel(const __grid_constant__ CUtensorMap tmap, const __grid_constant__ DecodeArgs a) {
    using C = Cfg<D>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int gid = lane >> 2, tig = lane & 3;
    const long long worker = (long long)blockIdx.x * kWarps + warp;
    if (worker >= a.workers) return;
    const long long W = a.total_items, V = a.workers;
    const long long ws = worker_start(worker, W, V);
    const long long we = worker_start(worker + 1, W, V);
    const int count = (int)(we - ws);
    if (count <= 0) return;

    const PoolGeom &g = a.g;
    const int H = g.num_kv_heads, G = a.group, Hq = H * G, BS = g.block_size;
    uint8_t *ring = smem + warp * C::kRingBytes;
    __half *ostage = reinterpret_cast<__half *>(smem + kWarps * C::kRingBytes + warp * C::kOutBytes);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kWarps * (C::kRingBytes + C::kOutBytes)) + warp * C::kNS;
    const uint32_t ring_u32 = ptx::smem_u32(ring);
    const uint32_t bar_u32 = ptx::smem_u32(bars);

    if (lane == 0) {
        ptx::prefetch_tensormap(&tmap);  // a launch parameter: safe before the wait below
        for (int s = 0; s < C::kNS; ++s) ptx::mbar_init(bar_u32 + 8 * s, 1);
        ptx::fence_barrier_init();
    }
    __syncwarp();
    // ---- producer side: lane j of a batch describes item (base + j) ------
    // The item positions come from the launch parameters alone, so the first
    // two batches are placed before the wait for the previous grid; their
    // block-table reads (which a previous kernel may have written) follow
    // the wait, both in flight together.
    struct BatchPos {
        long long bt_off;  // block-table entry of the item's tile
        int kvh, sub;
        bool real;         // this lane's slot is a real tile of the range
    };
    struct Batch {
        int bid, kvh, sub;
        unsigned real;  // ballot: lanes whose slot is a real tile of this range
    };
    auto place_batch = [&](long long base) {
        BatchPos r{0, 0, 0, false};
        const long long w = base + lane;
        if (w < we) {
            const ItemPos p = locate(a, w);
            if (p.tile() >= 0) {
                const int tok0 = p.tile() * kTile;
                r.real = true;
                r.bt_off = (long long)a.slot[p.b] * g.bt_stride + tok0 / BS;
                r.kvh = p.kvh;
                r.sub = tok0 % BS;
            }
        }
        return r;
    };
    auto finish_batch = [&](const BatchPos &pos, int bid) {
        Batch r{0, pos.kvh, pos.sub, 0u};
        if (pos.real) {
            if (bid < 0 || bid >= g.num_blocks) {
                atomicOr(g.err, kErrBlockRange);
                bid = 0;  // stay in bounds; the call reports the error
            }
            r.bid = bid;
        }
        r.real = __ballot_sync(0xffffffffu, pos.real);
        return r;
    };
    auto load_batch = [&](long long base) {
        const BatchPos pos = place_batch(base);
        return finish_batch(pos, pos.real ? __ldg(g.block_tables + pos.bt_off) : 0);
    };
    const BatchPos pos0 = place_batch(ws), pos1 = place_batch(ws + 32);

    // Programmatic dependent launch. With the in-kernel merge the dependent is
    // the next decode, whose CTAs only fit as ours retire: it may begin
    // launching now. With the merge pass the dependent is that pass, whose
    // CTAs would sit on our SMs and take issue slots while they wait: it is
    // released only once this CTA's loads are done. This kernel reads nothing
    // from global memory before the previous grid has completed (only the
    // parameter-only placement of its first items comes before the wait).
    const bool early_trigger = a.counters != nullptr;
    if (early_trigger) ptx::griddep_launch_dependents();
    ptx::griddep_wait();

    const uint64_t policy = ptx::l2_policy_evict_first();
    const long long layer_k_row = (long long)(a.layer * 2 + 0) * g.num_blocks;
    const long long layer_v_row = (long long)(a.layer * 2 + 1) * g.num_blocks;

    long long cur_base = ws;
    const int bid0 = pos0.real ? __ldg(g.block_tables + pos0.bt_off) : 0;
    const int bid1 = pos1.real ? __ldg(g.block_tables + pos1.bt_off) : 0;
    Batch cur = finish_batch(pos0, bid0);
    Batch nxt = finish_batch(pos1, bid1);
    int issued = 0;  // real tiles issued; stage = issued % kNS
    // Issues the next real tile of the range (uniform across the warp);
    // false when the range has none left.
    auto issue_one = [&]() -> bool {
        while (cur.real == 0u) {
            if (cur_base + 32 >= we) return false;
            cur_base += 32;
            cur = nxt;
            nxt = load_batch(cur_base + 32);
        }
        const int j = __ffs(cur.real) - 1;
        cur.real &= cur.real - 1u;
        const int bid = __shfl_sync(0xffffffffu, cur.bid, j);
        const int kvh = __shfl_sync(0xffffffffu, cur.kvh, j);
        const int sub = __shfl_sync(0xffffffffu, cur.sub, j);
        if (lane == 0) {
            const int stage = issued % C::kNS;
            const uint32_t bar = bar_u32 + 8 * stage;
            const uint32_t dst = ring_u32 + stage * C::kStageBytes;
            ptx::fence_proxy_async_smem();
            ptx::mbar_arrive_expect_tx(bar, C::kStageBytes);
#pragma unroll
            for (int kv = 0; kv < 2; ++kv) {
                const long long blk_row = (kv == 0 ? layer_k_row : layer_v_row) + bid;
                int y, z;
                if (g.head_major) {
                    y = sub;
                    z = (int)(blk_row * H + kvh);
                } else {
                    y = kvh;
                    z = (int)(blk_row * BS + sub);
                }
#pragma unroll
                for (int hs = 0; hs < C::kNSub; ++hs)
                    ptx::tma_load_3d(dst + (kv * C::kNSub + hs) * C::kSubBytes, &tmap, bar, hs * 64,
                                     y, z, policy);
            }
        }
        ++issued;
        return true;
    };

    for (int i = 0; i < C::kNS; ++i)
        if (!issue_one()) break;

    // ---- consumer state for the current (sequence, kv_head) unit ---------
    uint32_t qf[C::kKS][2];
    float acc[C::kKS][4];  // O^T tiles: d in [16*dm, 16*dm+16), g in {2tig, 2tig+1}
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    int ub = -1, ukvh = -1, uus = 0;
    long long ufirst = 0;
    bool first_piece = true;
    bool failed = false;
    bool wrote_remote = false;  // peer mode: this worker stored outputs to peers

    // Writes the finished unit (complete -> fp16 output; cut -> partial).
    auto finalize = [&]() {
        float lt0 = l0, lt1 = l1;
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
            lt0 += __shfl_xor_sync(0xffffffffu, lt0, off);
            lt1 += __shfl_xor_sync(0xffffffffu, lt1, off);
        }
        const bool complete = ufirst + a.vslots >= ws && ufirst + uus <= we;
        const int g0 = 2 * tig, g1 = 2 * tig + 1;
        if (complete) {
            // stage the unit's [G][D] fp16 output in shared memory, then
            // write it out as coalesced 16-byte chunks
            const float i0 = 1.f / lt0, i1 = 1.f / lt1;
#pragma unroll
            for (int dm = 0; dm < C::kKS; ++dm) {
                const int d = dm * 16 + gid;
                if (g0 < G) {
                    ostage[g0 * D + d] = __float2half_rn(acc[dm][0] * i0);
                    ostage[g0 * D + d + 8] = __float2half_rn(acc[dm][2] * i0);
                }
                if (g1 < G) {
                    ostage[g1 * D + d] = __float2half_rn(acc[dm][1] * i1);
                    ostage[g1 * D + d + 8] = __float2half_rn(acc[dm][3] * i1);
                }
            }
            __syncwarp();
            const long long obase = ((long long)ub * Hq + (long long)ukvh * G) * D;
            for (int ch = lane; ch < G * D / 8; ch += 32)
                store_out16(a, obase + ch * 8, reinterpret_cast<const uint4 *>(ostage)[ch]);
            __syncwarp();
            wrote_remote = a.ndst > 0;
        } else {
            const int slot = first_piece ? 0 : 1;
            float *pbase = a.partial + ((worker * 2 + slot) * G) * (long long)kPartialRow<D>;
#pragma unroll
            for (int dm = 0; dm < C::kKS; ++dm) {
                const int d = dm * 16 + gid;
                if (g0 < G) {
                    pbase[g0 * kPartialRow<D> + d] = acc[dm][0];
                    pbase[g0 * kPartialRow<D> + d + 8] = acc[dm][2];
                }
                if (g1 < G) {
                    pbase[g1 * kPartialRow<D> + d] = acc[dm][1];
                    pbase[g1 * kPartialRow<D> + d + 8] = acc[dm][3];
                }
            }
            if (gid == 0) {
                if (g0 < G) {
                    pbase[g0 * kPartialRow<D> + D] = m0;
                    pbase[g0 * kPartialRow<D> + D + 1] = lt0;
                }
                if (g1 < G) {
                    pbase[g1 * kPartialRow<D> + D] = m1;
                    pbase[g1 * kPartialRow<D> + D + 1] = lt1;
                }
            }
            if (a.counters) {
                // The last worker to finish a piece of this unit merges it:
                // an atomic ticket, no waiting on other workers.
                __threadfence();
                __syncwarp();
                const long long v_first = worker_of_item(ufirst + a.vslots, W, V);
                const long long v_last = worker_of_item(ufirst + uus - 1, W, V);
                int *ctr = a.counters + ((long long)ub * H + ukvh);
                int last = 0;
                if (lane == 0) last = atomicAdd(ctr, 1) == (int)(v_last - v_first);
                last = __shfl_sync(0xffffffffu, last, 0);
                if (last) {
                    __threadfence();
                    merge_unit<D>(a, ufirst, ub, ukvh, v_first, v_last, lane);
                    if (lane == 0) *ctr = 0;  // ready for the next launch
                }
            }
        }
        first_piece = false;
    };

    ItemPos p = locate(a, ws);
    long long w = ws;  // current slot; virtual slots are jumped over
    if (p.slot < p.vs) {
        w += p.vs - p.slot;
        p.slot = p.vs;
    }
    int fail_at = -1;
    int k = 0;  // real tiles consumed; stage = k % kNS
    for (; w < we; ++w) {
        if (p.slot == p.us) {  // next unit; its virtual slots are skipped
            p.unit_first += p.us;
            if (++p.kvh == H) {
                p.kvh = 0;
                do {
                    ++p.b;
                    p.us = a.prefix[p.b + 1] - a.prefix[p.b];
                } while (p.us == 0);
            }
            p.slot = p.vs;
            w += p.vs;
            if (w >= we) break;
        }
        if (p.b != ub || p.kvh != ukvh) {
            if (ub >= 0) finalize();
            ub = p.b;
            ukvh = p.kvh;
            uus = p.us;
            ufirst = p.unit_first;
            // Q fragments (B operand, col-major 16x8): rows d, cols g = gid.
            const __half *qrow = static_cast<const __half *>(a.q) +
                                 ((long long)p.b * Hq + (long long)p.kvh * G + gid) * D;
#pragma unroll
            for (int ks = 0; ks < C::kKS; ++ks) {
                if (gid < G) {
                    qf[ks][0] = __ldg(reinterpret_cast<const uint32_t *>(qrow + ks * 16 + 2 * tig));
                    qf[ks][1] = __ldg(reinterpret_cast<const uint32_t *>(qrow + ks * 16 + 8 + 2 * tig));
                } else {
                    qf[ks][0] = 0u;
                    qf[ks][1] = 0u;
                }
            }
            if (a.rope_cos != nullptr && gid < G) rope_q<D>(qf, a, a.len[p.b] - 1, tig);
#pragma unroll
            for (int dm = 0; dm < C::kKS; ++dm) acc[dm][0] = acc[dm][1] = acc[dm][2] = acc[dm][3] = 0.f;
            m0 = m1 = -INFINITY;
            l0 = l1 = 0.f;
        }

        const int stage = k % C::kNS;
        const uint32_t parity = (uint32_t)((k / C::kNS) & 1);
        if (!ptx::mbar_wait_bounded(bar_u32 + 8 * stage, parity, kWaitLimitNs)) {
            if (lane == 0) atomicOr(g.err, kErrWaitTimeout);
            failed = true;
            fail_at = k;
            break;
        }
        const uint32_t kbase = ring_u32 + stage * C::kStageBytes;
        const uint32_t vbase = kbase + C::kNSub * C::kSubBytes;
        const int nvalid = min(kTile, a.len[p.b] - p.tile() * kTile);

        // ---- S^T = K Q^T (two accumulators to shorten the mma chain) ----
        float s_even[4] = {0.f, 0.f, 0.f, 0.f}, s_odd[4] = {0.f, 0.f, 0.f, 0.f};
        {
            const int t = (lane & 7) + ((lane >> 3) & 1) * 8;
            const int dsel = (lane >> 4) & 1;  // +8 columns
#pragma unroll
            for (int ks = 0; ks < C::kKS; ++ks) {
                const int d = ks * 16 + dsel * 8;
                const uint32_t addr = kbase + (d >> 6) * C::kSubBytes + t * 128 +
                                      ((((d & 63) >> 3) ^ (t & 7)) << 4);
                uint32_t a0, a1, a2, a3;
                ptx::ldmatrix_x4(addr, a0, a1, a2, a3);
                if (ks & 1) ptx::mma_16816(s_odd, a0, a1, a2, a3, qf[ks][0], qf[ks][1]);
                else ptx::mma_16816(s_even, a0, a1, a2, a3, qf[ks][0], qf[ks][1]);
            }
        }
        // s[0],s[1]: token gid, heads 2tig, 2tig+1; s[2],s[3]: token gid+8.
        float s[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) s[r] = (s_even[r] + s_odd[r]) * a.scale_log2;
        if (gid >= nvalid) s[0] = s[1] = -INFINITY;
        if (gid + 8 >= nvalid) s[2] = s[3] = -INFINITY;

        // ---- online softmax (exp2 domain) ----
        float mx0 = fmaxf(s[0], s[2]), mx1 = fmaxf(s[1], s[3]);
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
        }
        const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
        const float al0 = ptx::ex2(m0 - mn0), al1 = ptx::ex2(m1 - mn1);
        m0 = mn0;
        m1 = mn1;
        const float p0 = ptx::ex2(s[0] - mn0), p1 = ptx::ex2(s[1] - mn1);
        const float p2 = ptx::ex2(s[2] - mn0), p3 = ptx::ex2(s[3] - mn1);
        l0 = l0 * al0 + p0 + p2;
        l1 = l1 * al1 + p1 + p3;
#pragma unroll
        for (int dm = 0; dm < C::kKS; ++dm) {
            acc[dm][0] *= al0;
            acc[dm][1] *= al1;
            acc[dm][2] *= al0;
            acc[dm][3] *= al1;
        }
        const uint32_t pb0 = ptx::movmatrix_trans(ptx::pack_half2(p0, p1));
        const uint32_t pb1 = ptx::movmatrix_trans(ptx::pack_half2(p2, p3));

        // Rows past the sequence end may hold stale data (even Inf/NaN bit
        // patterns); zero them so 0 * V stays 0.
        if (nvalid < kTile) {
            const int nz = (kTile - nvalid) * C::kNSub * 8;  // 16-byte chunks
            for (int c = lane; c < nz; c += 32) {
                const int sub = c / ((kTile - nvalid) * 8);
                const int rem = c % ((kTile - nvalid) * 8);
                const int t = nvalid + rem / 8, ch = rem % 8;
                uint4 *dst = reinterpret_cast<uint4 *>(ring + stage * C::kStageBytes +
                                                       C::kNSub * C::kSubBytes + sub * C::kSubBytes +
                                                       t * 128 + ch * 16);
                *dst = make_uint4(0u, 0u, 0u, 0u);
            }
            __syncwarp();
        }

        // ---- O^T += V^T P^T ----
        {
            const int t = (lane & 7) + ((lane >> 4) & 1) * 8;
            const int dsel = (lane >> 3) & 1;
#pragma unroll
            for (int dm = 0; dm < C::kKS; ++dm) {
                const int d = dm * 16 + dsel * 8;
                const uint32_t addr = vbase + (d >> 6) * C::kSubBytes + t * 128 +
                                      ((((d & 63) >> 3) ^ (t & 7)) << 4);
                uint32_t a0, a1, a2, a3;
                ptx::ldmatrix_x4_trans(addr, a0, a1, a2, a3);
                ptx::mma_16816(acc[dm], a0, a1, a2, a3, pb0, pb1);
            }
        }
        __syncwarp();
        ++k;
        ++p.slot;
        issue_one();
    }

    if (!early_trigger) ptx::griddep_launch_dependents();
    if (failed) {
        // Drain this worker's own loads still in flight (bounded) and stop.
        if (lane == 0) {
            const uint64_t t0 = ptx::globaltimer_ns();
            for (int it = fail_at; it < issued; ++it) {
                const int stage = it % C::kNS;
                const uint32_t parity = (uint32_t)((it / C::kNS) & 1);
                while (!ptx::mbar_try_wait(bar_u32 + 8 * stage, parity)) {
                    if (ptx::globaltimer_ns() - t0 > kWaitLimitNs) break;
                }
            }
        }
        __syncwarp();
        return;
    }
    if (ub >= 0) finalize();
    (void)wrote_remote;
}

// Second pass for launches without merge counters (and for units cut into
// many pieces, where one warp would have to read hundreds of KB of
// partials). One CTA per (unit, head): blockIdx.x = sequence*Hkv + kv_head,
// blockIdx.y = head g of the group. Its 512 threads are D/4 chunk lanes x
// (2048/D) source groups; each group folds every kGroups-th source with an
// online softmax merge, three sources per round with their loads issued
// together (the 64-register budget of two CTAs per SM), then the groups are
// combined in shared memory. Complete units (one worker) were written by the
// decode kernel and are skipped. Launched as a programmatic dependent of the
// decode kernel, which releases it once its loads are done: it waits for
// the decode grid before reading any partial.
template <int D>
__device__ __forceinline__ void merge_body(const DecodeArgs &a) {
    constexpr int kRow = kPartialRow<D>;
    constexpr int kChunks = D / 4;
    constexpr int kGroups = kMergeThreads / kChunks;
    __shared__ float s_m[kGroups][kChunks];
    __shared__ float s_l[kGroups][kChunks];
    __shared__ float4 s_o[kGroups][kChunks];
    const int H = a.g.num_kv_heads, G = a.group, Hq = H * G;
    const int b = blockIdx.x / H, kvh = blockIdx.x % H, g = blockIdx.y;
    if (b >= a.nseq || g >= G) return;
    const int us = a.prefix[b + 1] - a.prefix[b];
    if (us == 0) return;
    const long long W = a.total_items, V = a.workers;
    const long long unit_first = (long long)H * a.prefix[b] + (long long)kvh * us;
    const long long v_first = worker_of_item(unit_first + a.vslots, W, V);
    const long long v_last = worker_of_item(unit_first + us - 1, W, V);
    if (v_first == v_last) return;
    const int c = threadIdx.x % kChunks, sg = threadIdx.x / kChunks;
    float M = -INFINITY, L = 0.f;
    float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
    // Sources sg, sg + kGroups, ...: the loads of a batch are issued together.
    constexpr int kBatch = 3;
    for (long long u0 = v_first + sg; u0 <= v_last; u0 += (long long)kGroups * kBatch) {
        float mv[kBatch], lv[kBatch];
        float4 xv[kBatch];
#pragma unroll
        for (int r = 0; r < kBatch; ++r) {
            const long long u = u0 + (long long)r * kGroups;
            mv[r] = -INFINITY;
            lv[r] = 0.f;
            xv[r] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (u <= v_last) {
                const int slot = worker_start(u, W, V) >= unit_first ? 0 : 1;
                const float *pb = a.partial + ((u * 2 + slot) * G + g) * (long long)kRow;
                mv[r] = __ldcg(pb + D);
                lv[r] = __ldcg(pb + D + 1);
                xv[r] = __ldcg(reinterpret_cast<const float4 *>(pb) + c);
            }
        }
        float Mn = M;
#pragma unroll
        for (int r = 0; r < kBatch; ++r) Mn = fmaxf(Mn, mv[r]);  // finite: source u0 exists
        const float sc = ptx::ex2(M - Mn);  // M = -inf on the first batch: 0
        L *= sc;
        O.x *= sc;
        O.y *= sc;
        O.z *= sc;
        O.w *= sc;
#pragma unroll
        for (int r = 0; r < kBatch; ++r) {
            const float w = ptx::ex2(mv[r] - Mn);  // missing sources: -inf -> 0
            L += w * lv[r];
            O.x += w * xv[r].x;
            O.y += w * xv[r].y;
            O.z += w * xv[r].z;
            O.w += w * xv[r].w;
        }
        M = Mn;
    }
    s_m[sg][c] = M;
    s_l[sg][c] = L;
    s_o[sg][c] = O;
    __syncthreads();
    if (sg != 0) return;
    float Mf = -INFINITY;
    for (int j = 0; j < kGroups; ++j) Mf = fmaxf(Mf, s_m[j][c]);
    float Lf = 0.f;
    float4 Of = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < kGroups; ++j) {
        const float w = ptx::ex2(s_m[j][c] - Mf);  // empty groups: m = -inf -> 0
        const float4 x = s_o[j][c];
        Lf += w * s_l[j][c];
        Of.x += w * x.x;
        Of.y += w * x.y;
        Of.z += w * x.z;
        Of.w += w * x.w;
    }
    const float inv = 1.f / Lf;
    const long long off = ((long long)b * Hq + (long long)kvh * G + g) * D + 4 * c;
    store_out8(a, off, __floats2half2_rn(Of.x * inv, Of.y * inv), __floats2half2_rn(Of.z * inv, Of.w * inv));
}

template <int D>
__global__ void __launch_bounds__(kMergeThreads, 2) merge_kernel(const __grid_constant__ DecodeArgs a) {
    ptx::griddep_launch_dependents();
    ptx::griddep_wait();
    merge_body<D>(a);
    if (a.done_counter) {  // peer mode: the last CTA publishes, then gathers
        __shared__ int s_last;
        __syncthreads();
        if (threadIdx.x == 0) s_last = signal_peers(a, gridDim.x * gridDim.y) ? 1 : 0;
        __syncthreads();
        if (s_last) pull_peer_slices(a);
    }
}

// Opts the kernel into its dynamic shared memory size, once per device.
template <int D>
cudaError_t prepare() {
    static std::atomic<unsigned long long> done_mask{0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const unsigned long long bit = 1ull << (dev & 63);
    if (done_mask.load(std::memory_order_acquire) & bit) return cudaSuccess;
    e = cudaFuncSetAttribute(paged_decode_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Cfg<D>::kSmemBytes);
    if (e == cudaSuccess) done_mask.fetch_or(bit, std::memory_order_acq_rel);
    return e;
}

template <int D>
cudaError_t launch_decode_t(const DecodeArgs &a, const void *tmap128, cudaStream_t s) {
    cudaError_t e = prepare<D>();
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((a.workers + kWarps - 1) / kWarps);
    cfg.blockDim = dim3(kWarps * 32);
    cfg.dynamicSmemBytes = Cfg<D>::kSmemBytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, paged_decode_kernel<D>, *static_cast<const CUtensorMap *>(tmap128), a);
}

template <int D>
int max_workers_t(int device) {
    if (prepare<D>() != cudaSuccess) return 0;
    int per_sm = 0, sms = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, paged_decode_kernel<D>, kWarps * 32,
                                                      Cfg<D>::kSmemBytes) != cudaSuccess)
        return 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
    return per_sm * sms * kWarps;
}

}  // namespace

int decode_workers_per_cta() { return kWarps; }

int decode_max_workers(int device, int head_dim, int block_size) {
    (void)block_size;
    switch (head_dim) {
    case 64: return max_workers_t<64>(device);
    case 128: return max_workers_t<128>(device);
    case 256: return max_workers_t<256>(device);
    default: return 0;
    }
}

cudaError_t launch_decode(const DecodeArgs &a, const void *tmap128, cudaStream_t s) {
    switch (a.g.head_dim) {
    case 64: return launch_decode_t<64>(a, tmap128, s);
    case 128: return launch_decode_t<128>(a, tmap128, s);
    case 256: return launch_decode_t<256>(a, tmap128, s);
    default: return cudaErrorInvalidValue;
    }
}

template <int D>
cudaError_t launch_merge_t(const DecodeArgs &a, cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.nseq * a.g.num_kv_heads, a.group);
    cfg.blockDim = dim3(kMergeThreads);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, merge_kernel<D>, a);
}

cudaError_t launch_merge(const DecodeArgs &a, cudaStream_t s) {
    switch (a.g.head_dim) {
    case 64: return launch_merge_t<64>(a, s);
    case 128: return launch_merge_t<128>(a, s);
    case 256: return launch_merge_t<256>(a, s);
    default: return cudaErrorInvalidValue;
    }
}

// The driver's tensor-map encoder, resolved once by a thread-safe static
// initialiser (first calls may come from several host threads at once).
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static const PFN_cuTensorMapEncodeTiled_v12000 encode = [] {
        cudaDriverEntryPointQueryResult q;
        void *fn = nullptr;
        cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000,
                                                         cudaEnableDefault, &q);
        if (e != cudaSuccess || q != cudaDriverEntryPointSuccess) fn = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }();
    return encode;
}

cudaError_t encode_tensor_map_2d(void *tmap_out128, bool fp16, const void *base, unsigned long long inner,
                                 unsigned long long outer, unsigned long long row_bytes, unsigned box_inner,
                                 unsigned box_outer) {
    const PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
    if (!encode) return cudaErrorNotSupported;
    cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
    cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    cuuint32_t box[2] = {box_inner, box_outer}, estr[2] = {1, 1};
    CUresult r = encode(static_cast<CUtensorMap *>(tmap_out128),
                        fp16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
                        const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t encode_pool_tensor_map(const PoolGeom &g, void *tmap_out128) {
    const PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
    if (!encode) return cudaErrorNotSupported;
    const unsigned long long L2 = 2ull * g.num_layers;
    cuuint64_t dims[3], strides[2];
    cuuint32_t box[3], estr[3] = {1, 1, 1};
    dims[0] = (cuuint64_t)g.head_dim;
    if (g.head_major) {
        dims[1] = (cuuint64_t)g.block_size;
        dims[2] = (cuuint64_t)(L2 * (unsigned long long)g.num_blocks * g.num_kv_heads);
        strides[0] = (cuuint64_t)g.head_dim * 2;
        strides[1] = (cuuint64_t)g.block_size * g.head_dim * 2;
        box[0] = 64;
        box[1] = kTile;
        box[2] = 1;
    } else {
        dims[1] = (cuuint64_t)g.num_kv_heads;
        dims[2] = (cuuint64_t)(L2 * (unsigned long long)g.num_blocks * g.block_size);
        strides[0] = (cuuint64_t)g.head_dim * 2;
        strides[1] = (cuuint64_t)g.num_kv_heads * g.head_dim * 2;
        box[0] = 64;
        box[1] = 1;
        box[2] = kTile;
    }
    CUresult r = encode(static_cast<CUtensorMap *>(tmap_out128), CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                        g.pool, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

}  // namespace tllm
