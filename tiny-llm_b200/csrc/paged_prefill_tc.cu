// Causal prefill attention over the paged KV pool on the 5th-generation
// tensor cores (tcgen05 / TMEM), for sm_100a.
//
// Replaces kernels::attention_prefill (reference kernels/attention.cu:131-237,
// called at src/transformer.cpp:238-242), which runs one CTA per (query,
// head) over the prompt's own [H][S][D] buffers, keeps every score in shared
// memory and re-reads K/V per query and head. Here the prompt's K/V are
// already appended to the pool, and each query row attends the sequence's
// tokens up to its own position (a prompt continuing a cached prefix sees
// the prefix too).
//
// One CTA per (sequence, KV head, block of 256 (query, head) rows): two Q
// tiles of 128 rows (the M of one UMMA) that share every K/V tile the CTA
// loads, so a K/V byte feeds twice the math. The query group (G heads
// sharing the KV head, padded to a power of two G') is packed into the
// rows: row r = query r / G', head r % G'. Ten warps:
//   warps 0-7  softmax: warps 4t..4t+3 own Q tile t, thread = one row (its
//              TMEM lane). Each loads its Q row (RoPE at its position) into
//              shared memory once; per 64-key tile reads its S row from
//              TMEM, masks by position, keeps the running max and sum, and
//              writes its P row (fp16 pairs, two keys per packed fp32
//              instruction) back over the first 32 columns of that S.
//              O accumulates in TMEM across tiles; it is rescaled (TMEM
//              load, multiply, store) only when a row's max grows by more
//              than 2^8.
//   warp 8     producer: block ids (one per lane, a window of 8 tiles
//              loaded one window ahead) and the TMA loads of the K/V tiles
//              (4 boxes of 16 tokens x 64 halves per 64-column atom, 128-byte
//              swizzle, no multicast, evict-last: every query block of the
//              sequence reads them). Groups past the last token load from an
//              out-of-range coordinate and come back as zeros.
//   warp 9     MMA: one thread issues, per K/V tile, S = Q K^T for both Q
//              tiles (into one of two TMEM S buffers each, so the next
//              tile's S runs during this tile's softmax) and O += P V, and
//              commits to mbarriers; the warp owns the TMEM allocation (all
//              512 columns: per Q tile two 64-column S buffers and O).
// Operands: Q and K in shared memory (K-major), V in shared memory
// (MN-major, rows = keys), all with the 128-byte swizzle; P is the A
// operand of P V straight from TMEM. fp16 in, fp32 accumulate. CTAs are
// numbered KV head fastest, so the CTAs in flight spread over the heads
// instead of all reading one head's K/V, and query blocks last-first, so
// the launch ends on the blocks with the fewest keys. Every wait is
// bounded; TMEM is freed on every path.
#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>

#include "kernels.h"
#include "ptx.cuh"

namespace tllm {
namespace {

constexpr int kTcRows = 128;               // UMMA M: rows of one Q tile
constexpr int kQTiles = 2;                 // Q tiles per CTA, sharing each K/V tile
constexpr int kCtaRows = kQTiles * kTcRows;
constexpr int kTcKeys = 64;                // keys per tile (UMMA N of S, K of P V)
constexpr int kSoftWarps = 4 * kQTiles;    // one warp per 32 TMEM lanes of a Q tile
constexpr int kProdWarp = kSoftWarps, kMmaWarp = kSoftWarps + 1;
constexpr int kTcThreads = (kSoftWarps + 2) * 32;
constexpr uint64_t kTcWaitNs = 2000000000ull;

template <int D>
struct TcCfg {
    static constexpr int kAtoms = D / 64;                     // 64-half column atoms
    static constexpr int kQBytes = kAtoms * kTcRows * 128;    // one Q tile: [atom][128 rows][128 B]
    static constexpr int kAtomBytes = kTcKeys * 128;          // one atom of a K or V tile
    static constexpr int kKBytes = kAtoms * kAtomBytes;
    static constexpr int kStageBytes = 2 * kKBytes;           // K then V, each [atom][64 keys][128 B]
    static constexpr int kNS = D == 64 ? 8 : 5;               // K/V stages
    static constexpr int kBarBytes = 512;
    static constexpr int kSmemBytes = kQTiles * kQBytes + kNS * kStageBytes + kBarBytes + 1024;
    static_assert(kSmemBytes <= 227 * 1024, "prefill ring too large");
    static_assert(2 * kNS + 6 * kQTiles + 2 <= 32, "barriers overlap the TMEM address slot");
    // Q tile t: S buffers at 256t + {0, 64} (P of the tile over the first 32
    // columns of its S), O at 256t + 128
    static constexpr uint32_t kTmemCols = 512;
    // instruction descriptors: fp32 accumulate, fp16 A/B, A K-major, M = 128
    static constexpr uint32_t kIdescS = (1u << 4) | ((uint32_t)(kTcKeys >> 3) << 17) | ((uint32_t)(kTcRows >> 4) << 24);
    static constexpr uint32_t kIdescO =
        (1u << 4) | (1u << 16) | ((uint32_t)(D >> 3) << 17) | ((uint32_t)(kTcRows >> 4) << 24);  // B MN-major
};

// Byte offset of 16-byte chunk `chunk` of row `row` in a [rows][128 B] tile
// stored with the 128-byte swizzle (the TMA and UMMA layout).
__device__ __forceinline__ uint32_t swz(int row, int chunk) { return row * 128 + (((chunk & 7) ^ (row & 7)) << 4); }

// Rotates halves (x1[i], x2[i]) = (q[d], q[d + D/2]) by the RoPE table row,
// each product and sum rounded separately and the result rounded to nearest
// even, as the append kernel rotates K.
__device__ __forceinline__ void rope8(uint4 &x1, uint4 &x2, const float *ct, const float *st) {
    __half *h1 = reinterpret_cast<__half *>(&x1), *h2 = reinterpret_cast<__half *>(&x2);
    const float4 c0 = __ldg(reinterpret_cast<const float4 *>(ct)), c1 = __ldg(reinterpret_cast<const float4 *>(ct) + 1);
    const float4 s0 = __ldg(reinterpret_cast<const float4 *>(st)), s1 = __ldg(reinterpret_cast<const float4 *>(st) + 1);
    const float cv[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float u = __half2float(h1[i]), v = __half2float(h2[i]);
        const float c = cv[i], s = sv[i];
        h1[i] = __float2half_rn(__fsub_rn(__fmul_rn(u, c), __fmul_rn(v, s)));
        h2[i] = __float2half_rn(__fadd_rn(__fmul_rn(v, c), __fmul_rn(u, s)));
    }
}

// A row's running max only moves (and O in TMEM is only rescaled) once the
// tile max exceeds it by more than 2^8; until then P = 2^(s - m) <= 256,
// exact enough in fp16 and the final 1/l undoes the common factor.
constexpr float kRescaleLog2 = 8.0f;

template <int D>
__global__ void __launch_bounds__(kTcThreads, 1)
    paged_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmap, const __grid_constant__ PrefillArgs a) {
    using C = TcCfg<D>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sq = smem;                                   // Q[kQTiles]
    uint8_t *sstage = sq + kQTiles * C::kQBytes;          // K/V stages
    uint64_t *bars = reinterpret_cast<uint64_t *>(sstage + C::kNS * C::kStageBytes);
    uint32_t *tslot = reinterpret_cast<uint32_t *>(bars + 32);
    const uint32_t full_u = ptx::smem_u32(bars);          // [kNS] K/V tile landed
    const uint32_t empty_u = full_u + 8 * C::kNS;         // [kNS] K/V stage consumed
    const uint32_t sfull_u = empty_u + 8 * C::kNS;        // [t][2] S_t(kt) in TMEM, by kt & 1
    const uint32_t pfull_u = sfull_u + 16 * kQTiles;      // [t][2] P_t(kt) in TMEM, O_t rescaled
    const uint32_t ofull_u = pfull_u + 16 * kQTiles;      // [t][2] P V into O_t (kt) complete
    const uint32_t done_u = ofull_u + 16 * kQTiles;       // every MMA complete
    const uint32_t qfull_u = done_u + 8;                  // Q rows in smem

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const PoolGeom &g = a.g;
    const int H = g.num_kv_heads, G = a.group, Gp = a.group_pad, Hq = H * G, BS = g.block_size;
    const int lin = (int)(blockIdx.x + blockIdx.y * gridDim.x);
    // KV head fastest; query blocks from the last to the first, so that the
    // causal blocks with the most keys start first and the last wave holds
    // the lightest ones (a sequence's early query blocks)
    const int kvh = lin % H, xq = a.cta_prefix[a.nseq] - 1 - lin / H;

    int lo = 0, hi = a.nseq - 1;  // sequence of this CTA: largest b with cta_prefix[b] <= xq
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (a.cta_prefix[mid] <= xq) lo = mid;
        else hi = mid - 1;
    }
    const int b = lo;
    const int qpb = kCtaRows / Gp;
    const int q0 = (xq - a.cta_prefix[b]) * qpb;
    const int n = a.ntok[b], written = a.written[b];
    const int pos0 = written - n;
    const int q_last = min(n, q0 + qpb) - 1;
    const int ntiles = (pos0 + q_last) / kTcKeys + 1;  // keys [0, position of the last query]

    if (threadIdx.x == 0) {
        ptx::prefetch_tensormap(&tmap);
        for (int s = 0; s < C::kNS; ++s) {
            ptx::mbar_init(full_u + 8 * s, 1);
            ptx::mbar_init(empty_u + 8 * s, 1);
        }
        for (int i = 0; i < 2 * kQTiles; ++i) {
            ptx::mbar_init(sfull_u + 8 * i, 1);
            ptx::mbar_init(pfull_u + 8 * i, kTcRows);
            ptx::mbar_init(ofull_u + 8 * i, 1);
        }
        ptx::mbar_init(done_u, 1);
        ptx::mbar_init(qfull_u, kCtaRows);
        ptx::fence_barrier_init();
    }
    if (warp == kMmaWarp) ptx::tmem_alloc(ptx::smem_u32(tslot), C::kTmemCols);
    ptx::tc_fence_before_sync();
    __syncthreads();
    ptx::tc_fence_after_sync();
    const uint32_t tbase = *tslot;

    // ---- softmax threads: this row's Q (RoPE at its position) -> smem,
    // while the producer already loads the first K/V tiles ----
    const int qt = warp >> 2;                 // Q tile of a softmax warp
    const int r = (warp & 3) * 32 + lane;     // row within the Q tile = TMEM lane
    const int crow = qt * kTcRows + r;        // row within the CTA
    const int qr = q0 + crow / Gp, gr = crow % Gp;
    const bool row_valid = warp < kSoftWarps && qr <= q_last && gr < G;
    const int prow = pos0 + min(qr, q_last);
    if (warp < kSoftWarps) {
        const uint4 *src = reinterpret_cast<const uint4 *>(static_cast<const __half *>(a.q) +
                                                          ((long long)(a.row_off[b] + qr) * Hq + kvh * G + gr) * D);
        const bool rope = a.rope_cos != nullptr && prow < a.rope_max_pos;
        if (a.rope_cos != nullptr && !rope && row_valid) atomicOr(g.err, kErrPosRange);
        uint8_t *sqt = sq + qt * C::kQBytes;
        // the whole row in flight at once (one memory round trip), then
        // chunk c rotated with its partner c + D/16, the table rows read
        // four chunk pairs at a time
        uint4 x[D / 8];
#pragma unroll
        for (int c = 0; c < D / 8; ++c) x[c] = row_valid ? __ldg(src + c) : make_uint4(0u, 0u, 0u, 0u);
        if (rope && row_valid) {
            const float *ct = a.rope_cos + (long long)prow * (D / 2), *st = a.rope_sin + (long long)prow * (D / 2);
#pragma unroll
            for (int c0 = 0; c0 < D / 16; c0 += 4) {
#pragma unroll
                for (int c = c0; c < c0 + 4 && c < D / 16; ++c) rope8(x[c], x[c + D / 16], ct + 8 * c, st + 8 * c);
            }
        }
#pragma unroll
        for (int c = 0; c < D / 8; ++c)
            *reinterpret_cast<uint4 *>(sqt + (c >> 3) * (kTcRows * 128) + swz(r, c)) = x[c];
        ptx::fence_proxy_async_smem();
        ptx::mbar_arrive(qfull_u);
    }

    if (warp == kProdWarp) {
        // ---- producer (whole warp): lane i holds the block id of key group
        // i of an 8-tile window, loaded one window ahead; lane 0 issues ----
        const long long z_oob = 2ll * g.num_layers * g.num_blocks * (g.head_major ? H : BS);
        const int *bt = g.block_tables + (long long)a.slot[b] * g.bt_stride;
        auto load_ids = [&](int w) -> int {  // block id of key group 32 w + lane, -1 past the sequence
            const int key0 = (w * 32 + lane) * 16;
            if (key0 >= written) return -1;
            const int bid = __ldg(bt + key0 / BS);
            if (bid < 0 || bid >= g.num_blocks) {
                atomicOr(g.err, kErrBlockRange);
                return -1;
            }
            return bid;
        };
        const uint64_t policy = ptx::l2_policy_evict_last();  // every query block reads these K/V
        int ids = load_ids(0), ids_next = ntiles > 8 ? load_ids(1) : -1;
        for (int kt = 0; kt < ntiles; ++kt) {
            const int s = kt % C::kNS;
            if ((kt & 7) == 0 && kt > 0) {
                ids = ids_next;
                if (kt + 8 < ntiles) ids_next = load_ids((kt >> 3) + 1);
            }
            if (kt >= C::kNS && !__all_sync(0xffffffffu, ptx::mbar_wait_bounded(
                                                             empty_u + 8 * s, (uint32_t)(((kt / C::kNS) - 1) & 1),
                                                             kTcWaitNs))) {
                if (lane == 0) atomicOr(g.err, kErrWaitTimeout);
                break;
            }
            const uint32_t bar = full_u + 8 * s;
            const uint32_t dst0 = ptx::smem_u32(sstage + s * C::kStageBytes);
            if (lane == 0) ptx::mbar_arrive_expect_tx(bar, C::kStageBytes);
#pragma unroll
            for (int gi = 0; gi < kTcKeys / 16; ++gi) {
                const int bid = __shfl_sync(0xffffffffu, ids, (kt & 7) * 4 + gi);
                const int sub = (kt * kTcKeys + gi * 16) % BS;
                if (lane == 0) {
#pragma unroll
                    for (int kv = 0; kv < 2; ++kv) {
                        long long zz = z_oob;  // past the sequence (or a bad id): zero-filled
                        int y = 0;
                        if (bid >= 0) {
                            const long long row = (long long)(a.layer * 2 + kv) * g.num_blocks + bid;
                            if (g.head_major) {
                                y = sub;
                                zz = row * H + kvh;
                            } else {
                                y = kvh;
                                zz = row * BS + sub;
                            }
                        }
#pragma unroll
                        for (int hs = 0; hs < C::kAtoms; ++hs)
                            ptx::tma_load_3d(dst0 + kv * C::kKBytes + hs * C::kAtomBytes + gi * 2048, &tmap, bar,
                                             hs * 64, y, (int)zz, policy);
                    }
                }
            }
        }
    } else if (warp == kMmaWarp) {
        // ---- MMA issue (one thread) ----
        if (lane == 0) {
            const uint32_t q_u = ptx::smem_u32(sq);
            bool ok = true;
            auto issue_s = [&](int kt) -> bool {  // S_t(kt) = Q_t K^T into S buffer kt & 1 of each Q tile
                const int s = kt % C::kNS;
                if (!ptx::mbar_wait_bounded(full_u + 8 * s, (uint32_t)((kt / C::kNS) & 1), kTcWaitNs)) return false;
                ptx::tc_fence_after_sync();
                const uint32_t k_u = ptx::smem_u32(sstage + s * C::kStageBytes);
#pragma unroll
                for (int t = 0; t < kQTiles; ++t) {
                    const uint32_t d = tbase + (uint32_t)(t * 256 + (kt & 1) * kTcKeys);
#pragma unroll
                    for (int ks = 0; ks < D / 16; ++ks) {
                        const uint64_t ad = ptx::umma_desc_sw128(
                            q_u + t * C::kQBytes + (ks >> 2) * (kTcRows * 128) + (ks & 3) * 32, 16, 1024);
                        const uint64_t bd =
                            ptx::umma_desc_sw128(k_u + (ks >> 2) * C::kAtomBytes + (ks & 3) * 32, 16, 1024);
                        ptx::umma_f16(d, ad, bd, C::kIdescS, ks > 0 ? 1u : 0u);
                    }
                    ptx::umma_commit(sfull_u + 16 * t + 8 * (kt & 1));
                }
                return true;
            };
            ok = ptx::mbar_wait_bounded(qfull_u, 0u, kTcWaitNs) && issue_s(0);
            for (int kt = 0; kt < ntiles && ok; ++kt) {
                if (kt + 1 < ntiles && !issue_s(kt + 1)) {
                    ok = false;
                    break;
                }
                const uint32_t v_u = ptx::smem_u32(sstage + (kt % C::kNS) * C::kStageBytes + C::kKBytes);
#pragma unroll
                for (int t = 0; t < kQTiles; ++t) {
                    if (!ptx::mbar_wait_bounded(pfull_u + 16 * t + 8 * (kt & 1), (uint32_t)((kt >> 1) & 1),
                                                kTcWaitNs)) {
                        ok = false;
                        break;
                    }
                    ptx::tc_fence_after_sync();
#pragma unroll
                    for (int ks = 0; ks < kTcKeys / 16; ++ks) {
                        const uint32_t pa = tbase + (uint32_t)(t * 256 + (kt & 1) * kTcKeys + ks * 8);
                        const uint64_t bd = ptx::umma_desc_sw128(v_u + ks * 2048, C::kAtomBytes, 1024);
                        ptx::umma_f16_ta(tbase + (uint32_t)(t * 256 + 2 * kTcKeys), pa, bd, C::kIdescO,
                                         (kt > 0 || ks > 0) ? 1u : 0u);
                    }
                    ptx::umma_commit(ofull_u + 16 * t + 8 * (kt & 1));
                }
                if (!ok) break;
                ptx::umma_commit(empty_u + 8 * (kt % C::kNS));
            }
            if (!ok) atomicOr(g.err, kErrWaitTimeout);
            // every MMA issued has completed before TMEM is freed
            ptx::umma_commit(done_u);
            if (!ptx::mbar_wait_bounded(done_u, 0u, kTcWaitNs)) atomicOr(g.err, kErrWaitTimeout);
        }
    } else {
        // ---- softmax warps: one row per thread ----
        const uint32_t trow = tbase + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)(qt * 256);
        const uint32_t tmem_o = trow + 2 * kTcKeys;
        const uint32_t sfull_t = sfull_u + 16 * qt, pfull_t = pfull_u + 16 * qt, ofull_t = ofull_u + 16 * qt;
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        // waits agree across the warp: the TMEM loads and stores after them
        // are warp-collective
        auto wait_all = [&](uint32_t bar, uint32_t parity) -> bool {
            return __all_sync(0xffffffffu, ptx::mbar_wait_bounded(bar, parity, kTcWaitNs));
        };
        auto wait_pv = [&](int kt) -> bool {  // P V (kt) accumulated into this tile's O
            return wait_all(ofull_t + 8 * (kt & 1), (uint32_t)((kt >> 1) & 1));
        };
        for (int kt = 0; kt < ntiles; ++kt) {
            if (!wait_all(sfull_t + 8 * (kt & 1), (uint32_t)((kt >> 1) & 1))) {
                ok = false;
                break;
            }
            ptx::tc_fence_after_sync();
            float sv[kTcKeys];
            {
                uint32_t v0[32], v1[32];
                ptx::tmem_ld32(trow + (uint32_t)((kt & 1) * kTcKeys), v0);
                ptx::tmem_ld32(trow + (uint32_t)((kt & 1) * kTcKeys + 32), v1);
                ptx::tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    sv[j] = __uint_as_float(v0[j]);
                    sv[32 + j] = __uint_as_float(v1[j]);
                }
            }
            const int key0 = kt * kTcKeys;
            if (key0 + kTcKeys - 1 > prow) {  // keys past this row's position
#pragma unroll
                for (int j = 0; j < kTcKeys; ++j)
                    if (key0 + j > prow) sv[j] = -INFINITY;
            }
            // max of the raw scores, then scaled (the scale is positive and
            // rounding is monotonic, so this is the max of the scaled ones)
            float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};  // 4 independent chains
#pragma unroll
            for (int j = 0; j < kTcKeys; ++j) mx4[j & 3] = fmaxf(mx4[j & 3], sv[j]);
            const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * a.scale_log2;
            // The max moves on tile 0 (key 0 <= every position, so mx is
            // finite there) and when it rises past the threshold; O then
            // holds the earlier tiles at the old max and is rescaled once
            // P V (kt - 1) is complete.
            const bool grow = kt == 0 || mx > m + kRescaleLog2;
            if (kt > 0 && __any_sync(0xffffffffu, grow)) {
                if (!wait_pv(kt - 1)) {
                    ok = false;
                    break;
                }
                ptx::tc_fence_after_sync();
                const float mn = fmaxf(m, mx);
                const float alpha = ptx::ex2(m - mn);
                l *= alpha;
                m = mn;
#pragma unroll
                for (int c0 = 0; c0 < D; c0 += 32) {
                    uint32_t v[32];
                    ptx::tmem_ld32(tmem_o + c0, v);
                    ptx::tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(__uint_as_float(v[j]) * alpha);
                    ptx::tmem_st32(tmem_o + c0, v);
                }
                ptx::tmem_wait_st();
            } else if (kt == 0) {
                m = mx;
            }
            // P = 2^(s * scale - m), two keys per packed fp32 instruction,
            // as fp16 pairs over the first 32 columns of this tile's S
            const uint64_t sc2 = ptx::f2_pack(a.scale_log2, a.scale_log2), nm2 = ptx::f2_pack(-m, -m);
            uint64_t sum2[2] = {0ull, 0ull};  // two independent chains of pairs
            uint32_t pw[kTcKeys / 2];
#pragma unroll
            for (int j = 0; j < kTcKeys / 2; ++j) {
                float y0, y1;
                ptx::f2_unpack(ptx::f2_fma(ptx::f2_pack(sv[2 * j], sv[2 * j + 1]), sc2, nm2), y0, y1);
                const float p0 = ptx::ex2(y0), p1 = ptx::ex2(y1);
                sum2[j & 1] = ptx::f2_add(sum2[j & 1], ptx::f2_pack(p0, p1));
                const __half2 h = __floats2half2_rn(p0, p1);
                pw[j] = *reinterpret_cast<const uint32_t *>(&h);
            }
            ptx::tmem_st32(trow + (uint32_t)((kt & 1) * kTcKeys), pw);
            {
                float s0, s1, s2, s3;
                ptx::f2_unpack(sum2[0], s0, s1);
                ptx::f2_unpack(sum2[1], s2, s3);
                l += (s0 + s1) + (s2 + s3);
            }
            // The tile holding the sequence's last token: V rows past it
            // (stale data of the block) are zeroed so that 0 * V stays 0. Q
            // tile 0 does it; P V of tile 1 is issued after tile 0's P.
            if (qt == 0 && key0 + kTcKeys > written && written > key0) {
                uint8_t *vp = sstage + (kt % C::kNS) * C::kStageBytes + C::kKBytes;
                const int first_bad = written - key0;
                const int nchunks = (kTcKeys - first_bad) * C::kAtoms * 8;
                for (int i = r; i < nchunks; i += kTcRows) {
                    const int key = first_bad + i / (C::kAtoms * 8), rem = i % (C::kAtoms * 8);
                    *reinterpret_cast<uint4 *>(vp + (rem >> 3) * C::kAtomBytes + swz(key, rem & 7)) =
                        make_uint4(0u, 0u, 0u, 0u);
                }
                ptx::fence_proxy_async_smem();
            }
            ptx::tmem_wait_st();
            ptx::tc_fence_before_sync();
            ptx::mbar_arrive(pfull_t + 8 * (kt & 1));
        }
        if (ok && !wait_pv(ntiles - 1)) ok = false;
        if (!ok) {
            if (lane == 0) atomicOr(g.err, kErrWaitTimeout);
        } else {
            ptx::tc_fence_after_sync();
            const float inv = 1.f / l;
            uint4 *dst = reinterpret_cast<uint4 *>(static_cast<__half *>(a.o) +
                                                   ((long long)(a.row_off[b] + qr) * Hq + kvh * G + gr) * D);
            uint32_t v[D / 32][32];  // the whole O row, one TMEM wait
#pragma unroll
            for (int c0 = 0; c0 < D / 32; ++c0) ptx::tmem_ld32(tmem_o + 32 * c0, v[c0]);
            ptx::tmem_wait_ld();
            if (row_valid) {
#pragma unroll
                for (int c0 = 0; c0 < D / 32; ++c0) {
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        uint32_t w[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const __half2 h = __floats2half2_rn(__uint_as_float(v[c0][8 * c + 2 * e]) * inv,
                                                                __uint_as_float(v[c0][8 * c + 2 * e + 1]) * inv);
                            w[e] = *reinterpret_cast<const uint32_t *>(&h);
                        }
                        dst[4 * c0 + c] = make_uint4(w[0], w[1], w[2], w[3]);
                    }
                }
            }
        }
    }
    // ---- teardown: every MMA has completed (or its wait gave up); free TMEM ----
    ptx::tc_fence_before_sync();
    __syncthreads();
    if (warp == kMmaWarp) {
        ptx::tc_fence_after_sync();
        ptx::tmem_dealloc(tbase, C::kTmemCols);
    }
}

template <int D>
cudaError_t launch_prefill_tc_t(const PrefillArgs &a, const void *tmap128, cudaStream_t s) {
    cudaError_t e = cudaFuncSetAttribute(paged_prefill_tc_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         TcCfg<D>::kSmemBytes);
    if (e != cudaSuccess) return e;
    const int ctas = a.cta_prefix[a.nseq];
    if (ctas <= 0) return cudaSuccess;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ctas, a.g.num_kv_heads);
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = TcCfg<D>::kSmemBytes;
    cfg.stream = s;
    return cudaLaunchKernelEx(&cfg, paged_prefill_tc_kernel<D>, *static_cast<const CUtensorMap *>(tmap128), a);
}

}  // namespace

int prefill_tc_rows_per_cta() { return kCtaRows; }

cudaError_t launch_prefill_tc(const PrefillArgs &a, const void *tmap128, cudaStream_t s) {
    switch (a.g.head_dim) {
    case 64: return launch_prefill_tc_t<64>(a, tmap128, s);
    case 128: return launch_prefill_tc_t<128>(a, tmap128, s);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace tllm
