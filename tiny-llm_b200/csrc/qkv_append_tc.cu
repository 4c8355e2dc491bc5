// Fused Q/K/V projection (W8A16) + KV append (+ RoPE on Q and K) on the
// 5th-generation tensor cores (tcgen05), sm_100a.
//
// Same operation and outputs as qkv_append.cu (the decode step's three
// kernels::w8a16_matmul calls of TransformerLayer::attention, reference
// src/transformer.cpp:209-226 and kernels/w8a16_matmul.cu:119-235, plus the
// appendKV copy, src/kv_cache.cpp:206-233), for the shapes where the weight
// columns come in tiles of 128 and the scale groups hold 32, 64 or 128 rows.
//
// The weights are the M side of one UMMA per 16 rows of K (M = 128 weight
// columns per CTA, A operand in TMEM, K-major), the batch rows the N side
// (N = 16, 32 or 64, K-major B operand in shared memory), so the tensor
// core reads every weight once
// and the math costs little next to the weight stream. Per CTA (a column
// tile x a K-chunk, split-K over the grid), in 64-row blocks:
//   warp 9     the producer: TMA loads of the block's int8 weight tile
//              (64 rows x 128 columns, 128-byte swizzle) and of its
//              activation tile (64 K x N rows: the B layout) into a deep
//              ring, completing on an mbarrier: the bytes in flight are the
//              ring's, with no registers held. From weights repacked by
//              qkv_pack_weight the tile is one contiguous 8 KB copy
//              (cp.async.bulk) of bytes already in the swizzled order, where
//              the row-major weights give 64 segments of 128 bytes;
//   warps 0-7  convert each int8 tile to fp16 (exact: the byte in the
//              mantissa of 1024.0, minus 1152) straight into TMEM, where the
//              UMMA reads its A operand: a transposing ldmatrix of 16 x 16
//              bytes hands every thread the bytes that tcgen05.st.16x256b
//              stores as fp16 pairs along K, so shared memory carries the
//              weights once (TMA in, ldmatrix out) and no fp16 copy of them;
//              afterwards they read the accumulators (one TMEM lane = one
//              weight column per thread; warps w and w + 4 split the rows);
//   warp 8     issues the UMMAs (one thread) and owns the TMEM allocation.
// Each scale group is summed by the tensor core into its own fp32 TMEM
// accumulator (fresh at the group's first k-step); the epilogue scales the
// groups and adds them, sum_g s_g * (sum_k a_k w_k), as qkv_append.cu does.
// Split-K: every CTA adds its fp32 partial sums into the tile's accumulator
// in L2 (one bulk reduction of its staged rows, cp.reduce.async.bulk
// .add.f32) and arrives on the tile's counter with release semantics; the
// last CTA to arrive (acquire) reads the total and zeroes the accumulator
// for the next launch, rounds to fp16, rotates
// Q and K pairs (d, d + D/2) by the RoPE table at the row's position (the
// append kernel's rounding) and writes Q to q_out and K/V into their block
// slots.
//
// Programmatic dependent launch: a CTA prefetches its weight tiles into L2
// at once and waits (griddepcontrol.wait) before any load, so it can start
// while the kernel before it finishes; it lets the next kernel start once
// its own loads are issued.
//
// No multicast anywhere: every TMA load reads this GPU's own memory. Every
// mbarrier wait is bounded (2 s); a wait that gives up records
// kErrWaitTimeout and the CTA finishes without its output.
#include <algorithm>
#include <cstdint>
#include <cuda_fp16.h>
#include <map>
#include <mutex>

#include "kernels.h"
#include "ptx.cuh"

namespace tllm {
namespace {

constexpr int kTcM = 128;         // weight columns per CTA (UMMA M)
constexpr int kBlk = 64;          // K rows per block (4 UMMA k-steps)
constexpr int kNW = 8;            // int8 weight + activation stages (TMA ring)
constexpr int kNA = 2;            // fp16 weight stages in TMEM (the UMMA A operand)
constexpr int kACols = kBlk / 2;  // TMEM columns of one A stage (fp16 pairs along K)
constexpr int kW8Bytes = kBlk * kTcM;            // [64 rows][128 B], swizzled
constexpr int kConvWarps = 8;
constexpr int kConvThreads = 32 * kConvWarps;
constexpr int kMmaWarp = kConvWarps, kProdWarp = kConvWarps + 1;
constexpr int kThreadsTc = kConvThreads + 64;     // + the MMA warp and the producer warp
constexpr int kMaxSplit = 16;                     // split-K CTAs of a tile
constexpr uint64_t kWaitNs = 2000000000ull;

// TMA descriptors of one launch: the three weight matrices and the
// activations (128 bytes each, opaque here).
struct alignas(64) QkvMaps {
    unsigned char w[3][128];
    unsigned char x[128];
};

// Scale groups one K-chunk of kchunk rows (a multiple of kBlk, starting at a
// multiple of kchunk) can touch: a chunk that is not a multiple of the group
// may start and end inside one.
__host__ __device__ constexpr int tc_max_groups(int kchunk, int group) {
    return kchunk % group == 0 ? kchunk / group : (kchunk - 1 + group - kBlk) / group + 1;
}

__device__ __forceinline__ uint32_t swz(int row, int chunk) { return row * 128 + (((chunk & 7) ^ (row & 7)) << 4); }

__device__ __forceinline__ long long pool_off(const PoolGeom &g, int layer, int kv, int block, int tok, int head) {
    const long long block_elems = (long long)g.block_size * g.num_kv_heads * g.head_dim;
    const long long base = ((long long)(layer * 2 + kv) * g.num_blocks + block) * block_elems;
    if (g.head_major) return base + ((long long)head * g.block_size + tok) * g.head_dim;
    return base + ((long long)tok * g.num_kv_heads + head) * g.head_dim;
}

// 4 int8 (one word) -> 4 fp16 (two words), exactly.
__device__ __forceinline__ void i8x4_to_h4(uint32_t w, uint32_t &lo, uint32_t &hi) {
    const uint32_t u = w ^ 0x80808080u;  // signed -> excess-128
    uint32_t a, b;
    asm("prmt.b32 %0, %1, %2, 0x5140;" : "=r"(a) : "r"(u), "r"(0x64646464u));
    asm("prmt.b32 %0, %1, %2, 0x7362;" : "=r"(b) : "r"(u), "r"(0x64646464u));
    const __half2 off = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1152
    const __half2 ha = __hsub2(*reinterpret_cast<const __half2 *>(&a), off);
    const __half2 hb = __hsub2(*reinterpret_cast<const __half2 *>(&b), off);
    lo = *reinterpret_cast<const uint32_t *>(&ha);
    hi = *reinterpret_cast<const uint32_t *>(&hb);
}

__device__ __forceinline__ void rope8(uint4 &x1v, uint4 &x2v, const float *c, const float *s) {
    __half *x1 = reinterpret_cast<__half *>(&x1v);
    __half *x2 = reinterpret_cast<__half *>(&x2v);
    const float4 c0 = __ldg(reinterpret_cast<const float4 *>(c)), c1 = __ldg(reinterpret_cast<const float4 *>(c) + 1);
    const float4 s0 = __ldg(reinterpret_cast<const float4 *>(s)), s1 = __ldg(reinterpret_cast<const float4 *>(s) + 1);
    const float cc[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    const float ss[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float a = __half2float(x1[i]), b = __half2float(x2[i]);
        x1[i] = __float2half_rn(__fsub_rn(__fmul_rn(a, cc[i]), __fmul_rn(b, ss[i])));
        x2[i] = __float2half_rn(__fadd_rn(__fmul_rn(b, cc[i]), __fmul_rn(a, ss[i])));
    }
}

// 16 columns of this thread's TMEM lane, without waiting: the registers are
// valid after tmem_wait_ld_into (which waits for every load in flight).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                   "=r"(r[15])
                 : "r"(taddr));
}
// Waits for this thread's TMEM loads; the registers are operands so that no
// use of them moves above the wait.
__device__ __forceinline__ void tmem_wait_ld_into(uint32_t (&r)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15])
                 :
                 : "memory");
}
// Orders later uses of r after the preceding (volatile) wait.
__device__ __forceinline__ void regs_after_wait(uint32_t (&r)[16]) {
    asm volatile(""
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15])
                 :
                 : "memory");
}

template <int NR>
struct TcLayout {
    static constexpr int kXBytes = kBlk * NR * 2;              // one block's activations [NR][128 B]
    static constexpr int kWStage = kW8Bytes + kXBytes;         // one TMA stage
    static constexpr int kRing = kNW * kWStage;
};

template <int D, int NR, int GS>
__global__ void __launch_bounds__(kThreadsTc, NR <= 32 ? 2 : 1) qkv_append_tc_kernel(const __grid_constant__ QkvArgs a,
                                                                   const __grid_constant__ QkvMaps maps) {
    static_assert(GS % 16 == 0 && (GS <= kBlk ? kBlk % GS == 0 : GS % kBlk == 0), "group size");
    using Lay = TcLayout<NR>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sw = smem;                                     // TMA ring [kNW][int8 weights | activations]
    const int maxg = tc_max_groups(a.kchunk, GS);
    __half *ssc = reinterpret_cast<__half *>(smem + Lay::kRing);  // the chunk's scales [groups][128]
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + Lay::kRing + maxg * kTcM * 2);
    uint32_t *tslot = reinterpret_cast<uint32_t *>(bars + 24);
    const uint32_t loaded_u = ptx::smem_u32(bars);          // [kNW] TMA stage landed
    const uint32_t wfree_u = loaded_u + 8 * kNW;            // [kNW] TMA stage consumed (MMAs done)
    const uint32_t afull_u = wfree_u + 8 * kNW;             // [kNA] fp16 stage in TMEM
    const uint32_t afree_u = afull_u + 8 * kNA;             // [kNA] fp16 stage consumed
    const uint32_t done_u = afree_u + 8 * kNA;              // every MMA complete

    const PoolGeom &g = a.g;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kc = blockIdx.x, tile = blockIdx.y;
    const int tq = a.n[0] / kTcM, tk = a.n[1] / kTcM;
    const int m = tile < tq ? 0 : (tile < tq + tk ? 1 : 2);  // Q, K or V
    const int col0 = kTcM * (tile - (m == 0 ? 0 : (m == 1 ? tq : tq + tk)));
    const int N = a.n[m];
    const int k0 = kc * a.kchunk;
    const int klen = min(a.kchunk, a.K - k0);  // a multiple of kBlk
    const int nblk = klen / kBlk;
    const int gfirst = k0 / GS;                          // the chunk's first scale group
    const int ngroups = (k0 + klen - 1) / GS - gfirst + 1;  // the first and last may be partial
    // tile-blocked weights: this CTA's blocks are nblk x 8 KB in a row
    const int8_t *wpk = a.w[m] + ((long long)(col0 / kTcM) * (a.K / kBlk) + k0 / kBlk) * kW8Bytes;
    // TMEM: the group accumulators [maxg][NR columns], then the A ring
    const uint32_t acol0 = (uint32_t)(maxg * NR);
    const uint32_t tneed = acol0 + kNA * kACols;
    const uint32_t tcols = tneed <= 32 ? 32u : tneed <= 64 ? 64u : tneed <= 128 ? 128u : tneed <= 256 ? 256u : 512u;

    if (warp == kProdWarp && lane == 0) {
        // The chunk's weight tiles head for L2 at once, while the kernel
        // before this one on the stream may still run (programmatic launch):
        // a prefetch only warms L2, the loads themselves come after
        // griddepcontrol.wait like every other read.
        ptx::prefetch_tensormap(&maps.x);
        if (a.w_packed) {
            ptx::bulk_prefetch_l2(wpk, (uint32_t)(nblk * kW8Bytes));
        } else {
            ptx::prefetch_tensormap(&maps.w[m]);
            for (int blk = 0; blk < nblk; ++blk) ptx::tma_prefetch_2d(&maps.w[m], col0, k0 + blk * kBlk);
        }
    }
    if (threadIdx.x == 0) {
        for (int s = 0; s < kNW; ++s) {
            ptx::mbar_init(loaded_u + 8 * s, 1);
            ptx::mbar_init(wfree_u + 8 * s, 1);
        }
        for (int s = 0; s < kNA; ++s) {
            ptx::mbar_init(afull_u + 8 * s, kConvWarps);
            ptx::mbar_init(afree_u + 8 * s, 1);
        }
        ptx::mbar_init(done_u, 1);
        ptx::fence_barrier_init();
    }
    if (warp == kMmaWarp) ptx::tmem_alloc(ptx::smem_u32(tslot), tcols);
    ptx::tc_fence_before_sync();
    __syncthreads();
    ptx::tc_fence_after_sync();
    const uint32_t tbase = *tslot;
    bool ok = true;
    ptx::griddep_wait();  // the preceding kernel's writes (activations, tables, scratch) are visible

    if (warp == kProdWarp) {
        // ---- producer: the weight and activation tiles of every block ----
        if (lane == 0) {
            const uint64_t stream = ptx::l2_policy_evict_first();  // weights: read once
            const uint64_t keep = ptx::l2_policy_evict_last();     // activations: every column tile reads them
            for (int blk = 0; blk < nblk; ++blk) {
                const int s = blk % kNW;
                if (blk >= kNW && !ptx::mbar_wait_bounded(wfree_u + 8 * s, (uint32_t)((blk / kNW - 1) & 1), kWaitNs)) {
                    atomicOr(g.err, kErrWaitTimeout);
                    break;
                }
                const uint32_t dst = ptx::smem_u32(sw + s * Lay::kWStage);
                ptx::mbar_arrive_expect_tx(loaded_u + 8 * s, (uint32_t)Lay::kWStage);
                if (a.w_packed)  // the same bytes, swizzled in memory: one contiguous copy
                    ptx::bulk_load(dst, wpk + (long long)blk * kW8Bytes, (uint32_t)kW8Bytes, loaded_u + 8 * s, stream);
                else
                    ptx::tma_load_2d(dst, maps.w[m], loaded_u + 8 * s, col0, k0 + blk * kBlk, stream);
                ptx::tma_load_2d(dst + kW8Bytes, maps.x, loaded_u + 8 * s, k0 + blk * kBlk, 0, keep);
            }
            ptx::griddep_launch_dependents();  // the next kernel may start prefetching its weights
        }
    } else if (warp < kConvWarps) {
        // ---- converters: the chunk's scales (cp.async), then int8 -> fp16 ----
        const int t = threadIdx.x;
        {
            const __half *S = static_cast<const __half *>(a.sc[m]) + (long long)gfirst * N + col0;
            const uint32_t ssc_u = ptx::smem_u32(ssc);
            for (int i = t; i < ngroups * (kTcM / 8); i += kConvThreads) {
                const int gi = i / (kTcM / 8), c8 = i % (kTcM / 8);
                ptx::cp_async16(ssc_u + (uint32_t)((gi * kTcM + 8 * c8) * 2), S + (long long)gi * N + 8 * c8, 16u);
            }
        }
        // warp w converts TMEM lanes 32 (w % 4) .. +31 (its weight columns)
        // for k-steps 2 (w / 4) and 2 (w / 4) + 1 of every block: per 16 x 16
        // tile one transposing ldmatrix gives thread (g, t) the bytes of rows
        // 4t..4t+3 of columns g and g + 8, which converted are exactly the
        // fp16 pairs tcgen05.st.16x256b puts at lanes g, g + 8, columns 2t,
        // 2t + 1: the K-major A operand, with no fp16 copy in shared memory
        const int q = warp & 3, kh = warp >> 2, r16 = lane & 15;
        for (int blk = 0; blk < nblk; ++blk) {
            const int s = blk % kNW, sa_i = blk % kNA;
            if (!ptx::mbar_wait_bounded(loaded_u + 8 * s, (uint32_t)((blk / kNW) & 1), kWaitNs)) ok = false;
            if (ok && blk >= kNA &&
                !ptx::mbar_wait_bounded(afree_u + 8 * sa_i, (uint32_t)((blk / kNA - 1) & 1), kWaitNs))
                ok = false;
            if (!__all_sync(0xffffffffu, ok)) {
                ok = false;
                break;
            }
            const uint32_t src = ptx::smem_u32(sw + s * Lay::kWStage);
            const uint32_t ta = tbase + ((uint32_t)(32 * q) << 16) + acol0 + (uint32_t)(sa_i * kACols);
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const int ks = 2 * kh + i;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    uint32_t b0, b1, v0, v1, v2, v3;
                    ptx::ldmatrix_m16n16_trans_b8(src + swz(16 * ks + r16, 2 * q + h), b0, b1);
                    i8x4_to_h4(b0, v0, v1);
                    i8x4_to_h4(b1, v2, v3);
                    ptx::tmem_st_16x256b(ta + ((uint32_t)(16 * h) << 16) + (uint32_t)(8 * ks), v0, v1, v2, v3);
                }
            }
            ptx::tmem_wait_st();
            ptx::tc_fence_before_sync();  // the stores before the MMA thread's wait on the barrier
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(afull_u + 8 * sa_i);
        }
        ptx::cp_async_wait_all();  // the scales (the epilogue reads them after a barrier)
        if (!ok && lane == 0) atomicOr(g.err, kErrWaitTimeout);
    } else if (lane == 0) {
        // ---- UMMA issue (one thread) ----
        // fp32 accumulate, fp16 A (TMEM) and B (shared memory), both K-major
        constexpr uint32_t idesc = (1u << 4) | ((uint32_t)(NR >> 3) << 17) | ((uint32_t)(kTcM >> 4) << 24);
        const uint32_t sw_u = ptx::smem_u32(sw);
        for (int blk = 0; blk < nblk && ok; ++blk) {
            const int s = blk % kNW, sa_i = blk % kNA;
            // the activation tile landed (its stage's TMA) and the fp16 weights are in place
            if (!ptx::mbar_wait_bounded(loaded_u + 8 * s, (uint32_t)((blk / kNW) & 1), kWaitNs) ||
                !ptx::mbar_wait_bounded(afull_u + 8 * sa_i, (uint32_t)((blk / kNA) & 1), kWaitNs)) {
                ok = false;
                break;
            }
            ptx::tc_fence_after_sync();
            const uint32_t xa = sw_u + s * Lay::kWStage + kW8Bytes;
#pragma unroll
            for (int ks = 0; ks < kBlk / 16; ++ks) {
                const int kk = blk * (kBlk / 16) + ks;  // k-step within the chunk
                const int ka = k0 + kk * 16;  // the k-step's first row
                const int grp = ka / GS - gfirst;
                const uint32_t at = tbase + acol0 + (uint32_t)(sa_i * kACols + 8 * ks);
                const uint64_t bd = ptx::umma_desc_sw128(xa + ks * 32, 16, 1024);
                ptx::umma_f16_ta(tbase + (uint32_t)(grp * NR), at, bd, idesc, (ka % GS && kk) ? 1u : 0u);
            }
            ptx::umma_commit(afree_u + 8 * sa_i);
            ptx::umma_commit(wfree_u + 8 * s);
        }
        if (!ok) atomicOr(g.err, kErrWaitTimeout);
        ptx::umma_commit(done_u);  // every MMA issued so far has completed
    }

    __syncwarp();  // the MMA and producer warps' lane 0 rejoins its warp

    // ---- epilogue: the converter warps read the group accumulators (thread
    // = weight column; 16 rows at a time, three groups' TMEM loads per wait,
    // warps w and w + 4 on alternate 16-row chunks) and sum
    // s_g * acc_g in group order into an fp32 [NR][128] tile in the TMA ring
    // (free: every load landed and every MMA completed) ----
    float *sf = reinterpret_cast<float *>(sw);
    __half *sy = reinterpret_cast<__half *>(sw + NR * kTcM * 4);  // fp16 rows [NR][128]
    static_assert(64 * kTcM * 6 <= kNW * TcLayout<16>::kWStage, "epilogue staging outgrows the ring");
    __shared__ int s_last;
    if (warp < kConvWarps) {
        ptx::named_barrier_sync(1, kConvThreads);  // every thread's scales landed
        const int nq4 = a.rows * (kTcM / 4);       // float4 chunks of the real rows
        {
            // warps w and w + 4 share TMEM lane quarter w % 4 (weight columns)
            // and take alternate 16-row chunks of it
            constexpr int RC = 16, GB = 3;
            const int q = warp & 3, rc0 = (warp >> 2) * RC;
            const int col = 32 * q + lane;
            bool done_ok = ptx::mbar_wait_bounded(done_u, 0u, kWaitNs);
            if (!done_ok && lane == 0) atomicOr(g.err, kErrWaitTimeout);
            done_ok = __all_sync(0xffffffffu, done_ok) && ok;
            ptx::tc_fence_after_sync();
            const uint32_t tl = tbase + ((uint32_t)(32 * q) << 16);
#pragma unroll
            for (int rc = rc0; rc < NR; rc += 2 * RC) {
                float acc[RC];
#pragma unroll
                for (int r = 0; r < RC; ++r) acc[r] = 0.f;
                if (done_ok) {
                    for (int g0 = 0; g0 < ngroups; g0 += GB) {
                        uint32_t v[GB][RC];
#pragma unroll
                        for (int u = 0; u < GB; ++u)
                            if (g0 + u < ngroups) tmem_ld16(tl + (uint32_t)((g0 + u) * NR + rc), v[u]);
                        tmem_wait_ld_into(v[0]);
#pragma unroll
                        for (int u = 1; u < GB; ++u) regs_after_wait(v[u]);
#pragma unroll
                        for (int u = 0; u < GB; ++u)
                            if (g0 + u < ngroups) {
                                const float sv = __half2float(ssc[(g0 + u) * kTcM + col]);
#pragma unroll
                                for (int r = 0; r < RC; ++r) acc[r] = fmaf(__uint_as_float(v[u][r]), sv, acc[r]);
                            }
                    }
                }
#pragma unroll
                for (int r = 0; r < RC; ++r) sf[(rc + r) * kTcM + col] = acc[r];
            }
        }
        ptx::named_barrier_sync(1, kConvThreads);
        if (a.ksplit > 1) {
            // add this CTA's sums into the tile's fp32 accumulator in L2 with
            // one bulk reduction of the staged rows (whole lines at L2, not
            // per-thread atomics), wait for it, then arrive on the tile's
            // counter: the arrival releases the adds; the last arrival
            // acquires them all, reads the total and leaves zeros behind
            float *tacc = a.partial + (long long)tile * NR * kTcM;
            ptx::fence_proxy_async_smem();  // sf's generic writes before the bulk copy reads them
            ptx::named_barrier_sync(1, kConvThreads);
            if (threadIdx.x == 0) {
                ptx::bulk_reduce_add_f32(tacc, ptx::smem_u32(sf), (uint32_t)(nq4 * 16));
                ptx::bulk_commit();
                ptx::bulk_wait_all();
                ptx::fence_proxy_async_global();
                const int prev = ptx::atom_add_acq_rel_gpu(&a.counters[tile], 1);
                s_last = prev == a.ksplit - 1;
                if (s_last) a.counters[tile] = 0;  // ready for the next launch
            }
            ptx::named_barrier_sync(1, kConvThreads);
            if (s_last) {
                constexpr int kPer = NR / 8;  // float4 chunks per thread (NR * 32 over 256 threads)
                float4 t[kPer];
#pragma unroll
                for (int j = 0; j < kPer; ++j) {
                    const int i = threadIdx.x + kConvThreads * j;
                    t[j] = i < nq4 ? __ldcg(reinterpret_cast<const float4 *>(tacc) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int j = 0; j < kPer; ++j) {
                    const int i = threadIdx.x + kConvThreads * j;
                    if (i < nq4) {
                        __stcg(reinterpret_cast<float4 *>(tacc) + i, make_float4(0.f, 0.f, 0.f, 0.f));
                        __half2 *dst = reinterpret_cast<__half2 *>(sy + 4 * i);
                        dst[0] = __floats2half2_rn(t[j].x, t[j].y);
                        dst[1] = __floats2half2_rn(t[j].z, t[j].w);
                    }
                }
            }
        } else {
            if (threadIdx.x == 0) s_last = 1;
            for (int i = threadIdx.x; i < nq4; i += kConvThreads) {
                const float4 v = *reinterpret_cast<const float4 *>(sf + 4 * i);
                __half2 *dst = reinterpret_cast<__half2 *>(sy + 4 * i);
                dst[0] = __floats2half2_rn(v.x, v.y);
                dst[1] = __floats2half2_rn(v.z, v.w);
            }
        }
        ptx::named_barrier_sync(1, kConvThreads);
        if (s_last) {
            // rotate and store the rows by 8-half chunks
            const bool rope = a.rope_cos != nullptr && m < 2;
            constexpr int kChunks = D / 16;  // 8-half chunks per half head
            constexpr int kHeads = kTcM / D;
            for (int i = threadIdx.x; i < a.rows * kHeads * kChunks; i += kConvThreads) {
                const int r = i / (kHeads * kChunks), hh = (i / kChunks) % kHeads, c = i % kChunks;
                const __half *src = sy + r * kTcM + hh * D;
                uint4 x1 = *reinterpret_cast<const uint4 *>(src + 8 * c);
                uint4 x2 = *reinterpret_cast<const uint4 *>(src + D / 2 + 8 * c);
                const int pos = a.row_pos[r];
                const int head = (col0 + hh * D) / D;
                if (rope) {
                    if (pos < 0 || pos >= a.rope_max_pos) {
                        atomicOr(g.err, kErrPosRange);
                        continue;
                    }
                    rope8(x1, x2, a.rope_cos + (long long)pos * (D / 2) + 8 * c,
                          a.rope_sin + (long long)pos * (D / 2) + 8 * c);
                }
                __half *dst;
                if (m == 0) {
                    dst = static_cast<__half *>(a.q_out) + (long long)r * N + head * D;
                } else {
                    const int block = a.row_block[r];
                    if (block < 0 || block >= g.num_blocks || pos < 0) {
                        atomicOr(g.err, kErrBlockRange);
                        continue;
                    }
                    dst = static_cast<__half *>(g.pool) + pool_off(g, a.layer, m - 1, block, pos % g.block_size, head);
                }
                *reinterpret_cast<uint4 *>(dst + 8 * c) = x1;
                *reinterpret_cast<uint4 *>(dst + D / 2 + 8 * c) = x2;
            }
        }
    }

    // ---- teardown: every MMA has completed (or its wait gave up); free TMEM
    ptx::tc_fence_before_sync();
    __syncthreads();
    if (warp == kMmaWarp) {
        ptx::tc_fence_after_sync();
        ptx::tmem_dealloc(tbase, tcols);
    }
}

// The TMA ring + the scales (kchunk / 32 groups at most) + barriers +
// alignment.
int tc_smem_bytes(int kchunk, int nr) {
    const int ring = nr <= 16 ? TcLayout<16>::kRing : (nr <= 32 ? TcLayout<32>::kRing : TcLayout<64>::kRing);
    return ring + (kchunk / 32) * kTcM * 2 + 256 + 1024;
}

template <int D, int NR, int GS>
cudaError_t launch_t(const QkvArgs &a, const QkvMaps &maps, cudaStream_t s) {
    const int smem = tc_smem_bytes(a.kchunk, NR);
    static std::mutex mu;
    static std::map<int, int> opted;  // device -> bytes, only ever raised
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    {
        std::lock_guard<std::mutex> lock(mu);
        int &cur = opted[dev];
        if (cur < smem) {
            e = cudaFuncSetAttribute(qkv_append_tc_kernel<D, NR, GS>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            if (e != cudaSuccess) return e;
            cur = smem;
        }
    }
    // programmatic launch: the CTAs may start (and prefetch their weight
    // tiles into L2) while the kernel before this one on the stream finishes
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.ksplit, (a.n[0] + a.n[1] + a.n[2]) / kTcM);
    cfg.blockDim = dim3(kThreadsTc);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, qkv_append_tc_kernel<D, NR, GS>, a, maps);
}

template <int D, int NR>
cudaError_t launch_nr(const QkvArgs &a, const QkvMaps &maps, cudaStream_t s) {
    switch (a.group) {
    case 32: return launch_t<D, NR, 32>(a, maps, s);
    case 64: return launch_t<D, NR, 64>(a, maps, s);
    case 128: return launch_t<D, NR, 128>(a, maps, s);
    default: return cudaErrorInvalidValue;
    }
}

template <int D>
cudaError_t launch_d(const QkvArgs &a, const QkvMaps &maps, cudaStream_t s) {
    switch (qkv_tc_rows_padded(a.rows)) {
    case 16: return launch_nr<D, 16>(a, maps, s);
    case 32: return launch_nr<D, 32>(a, maps, s);
    default: return launch_nr<D, 64>(a, maps, s);
    }
}

// One thread per 16-byte chunk of the tile-blocked layout: packed row
// (t * K / 64 + b) * 64 + r holds source row b * 64 + r, columns
// t * 128 .. t * 128 + 127, its chunk c at position c ^ (r % 8).
__global__ void qkv_pack_kernel(const int8_t *__restrict__ w, int K, int n, int8_t *__restrict__ out,
                                long long chunks) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= chunks) return;
    const int p = (int)(i & 7);
    const long long prow = i >> 3;
    const int r = (int)(prow & (kBlk - 1));
    const long long tb = prow / kBlk;
    const int kb = K / kBlk;
    const long long t = tb / kb, b = tb % kb;
    const int8_t *src = w + (b * kBlk + r) * (long long)n + t * kTcM + 16 * (p ^ (r & 7));
    *reinterpret_cast<uint4 *>(out + 16 * i) = __ldg(reinterpret_cast<const uint4 *>(src));
}

}  // namespace

cudaError_t launch_qkv_pack_weight(const int8_t *w, int K, int n, int8_t *out, cudaStream_t s) {
    if (K <= 0 || n <= 0 || K % kBlk != 0 || n % kTcM != 0 || (reinterpret_cast<uintptr_t>(w) & 15) ||
        (reinterpret_cast<uintptr_t>(out) & 15))
        return cudaErrorInvalidValue;
    const long long chunks = (long long)K * n / 16;
    const int threads = 256;
    const long long blocks = (chunks + threads - 1) / threads;
    if (blocks > 0x7fffffffLL) return cudaErrorInvalidValue;
    qkv_pack_kernel<<<(unsigned)blocks, threads, 0, s>>>(w, K, n, out, chunks);
    return cudaGetLastError();
}

int qkv_tc_rows_padded(int rows) { return rows <= 16 ? 16 : (rows <= 32 ? 32 : 64); }

bool qkv_tc_supported(int head_dim, int group, int nq, int nkv, int hidden) {
    return (head_dim == 64 || head_dim == 128) && (group == 32 || group == 64 || group == 128) &&
           nq % kTcM == 0 && nkv % kTcM == 0 && hidden % 128 == 0;
}

// TMEM columns one CTA may hold: two CTAs share an SM's 512 at up to 32
// rows, one CTA per SM at 64.
static int tc_tmem_budget(int nr) { return nr <= 32 ? 256 : 512; }

// K-chunk (a multiple of 64 rows) and split for a launch of `rows` rows:
// about one wave of CTAs (two per SM up to 32 rows, one at 64), at most
// kMaxSplit CTAs per tile, each chunk's group accumulators plus the A ring
// within the CTA's TMEM columns. Chunks need not hold whole scale groups, so
// 64 blocks of 64 rows split six ways are chunks of 11 blocks (the longest
// CTA streams 11 blocks, not the 12 of 128-row units).
bool qkv_tc_split(int hidden, int group, int rows, int tiles, int num_sms, int *ksplit, int *kchunk) {
    const int nr = qkv_tc_rows_padded(rows);
    const int blocks = hidden / kBlk;
    const int budget = tc_tmem_budget(nr) - kNA * kACols;  // accumulator columns
    if (blocks < 1) return false;
    const int per_sm = nr <= 32 ? 2 : 1;
    int ks = std::max(1, (per_sm * std::max(num_sms, 1)) / std::max(tiles, 1));
    ks = std::min({ks, blocks, kMaxSplit});
    int per = (blocks + ks - 1) / ks;  // blocks per chunk
    while (per > 0 && tc_max_groups(per * kBlk, group) * nr > budget) --per;
    if (per < 1 || (blocks + per - 1) / per > kMaxSplit) return false;
    *kchunk = per * kBlk;
    *ksplit = (blocks + per - 1) / per;
    return true;
}

cudaError_t launch_qkv_append_tc(const QkvArgs &a, cudaStream_t s) {
    if (a.rows <= 0) return cudaSuccess;
    if (a.rows > kMaxQkvRows || a.kchunk <= 0 || a.kchunk % kBlk != 0 || a.ksplit < 1 || a.ksplit > kMaxSplit ||
        (long long)(a.ksplit - 1) * a.kchunk >= a.K || (long long)a.ksplit * a.kchunk < a.K ||
        (a.group != 32 && a.group != 64 && a.group != 128) ||
        tc_max_groups(a.kchunk, a.group) * qkv_tc_rows_padded(a.rows) + kNA * kACols >
            tc_tmem_budget(qkv_tc_rows_padded(a.rows)))
        return cudaErrorInvalidValue;
    // tensor maps: each weight [K][n] int8 in 64-row x 128-column boxes; the
    // activations [rows][K] fp16 in 64 x (padded rows) boxes (rows past the
    // launch's read as zeros)
    QkvMaps maps = {};
    for (int i = 0; i < 3 && !a.w_packed; ++i) {
        cudaError_t e = encode_tensor_map_2d(maps.w[i], false, a.w[i], (unsigned long long)a.n[i],
                                             (unsigned long long)a.K, (unsigned long long)a.n[i], kTcM, kBlk);
        if (e != cudaSuccess) return e;
    }
    cudaError_t e = encode_tensor_map_2d(maps.x, true, a.x, (unsigned long long)a.K, (unsigned long long)a.rows,
                                         (unsigned long long)a.K * 2, 64, (unsigned)qkv_tc_rows_padded(a.rows));
    if (e != cudaSuccess) return e;
    switch (a.g.head_dim) {
    case 64: return launch_d<64>(a, maps, s);
    case 128: return launch_d<128>(a, maps, s);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace tllm
