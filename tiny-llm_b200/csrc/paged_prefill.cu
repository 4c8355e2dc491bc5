// Causal prefill attention over the paged KV pool, for sm_100a.
//
// Replaces kernels::attention_prefill (reference kernels/attention.cu:131-237,
// called at src/transformer.cpp:238-242), which runs one CTA per (query,
// head) over the prompt's own [H][S][D] buffers, keeps every score in shared
// memory and re-reads K/V per query and head. Here the prompt's K/V are
// already appended to the pool, and each query row attends the sequence's
// tokens up to its own position (a prompt continuing a cached prefix sees
// the prefix too).
//
// Work: one CTA per (sequence, KV head, block of 64 (query, head) rows). The
// query group (G heads sharing the KV head, padded to a power of two G') is
// packed into the rows: row r = query r / G', head r % G'. Each of the four
// warps owns 16 rows (an mma.sync m16 tile) and keeps its Q fragments, its
// fp32 O accumulators and its softmax state in registers.
//
// Data movement: the CTA walks the keys in tiles of 64 (four 16-key groups,
// each a TMA box of the pool's tensor map: a block piece of 16 tokens x 64
// halves, 128-byte swizzle, no multicast) through a ring of stages. A fifth
// warp only produces: it reads the block ids and issues the loads, a full
// barrier per stage signals arrival, and an empty barrier (one arrival per
// compute warp) hands a stage back. (With the loads issued by a compute
// warp, which had to wait for the others before each refill, the kernel ran
// 40 % slower.) Groups past the sequence's last token are loaded from an
// out-of-range coordinate and come back as zeros. Every query block of a
// sequence reads the same K/V, so the loads ask L2 to keep them.
//
// Math per tile and warp: S = Q K^T (A = Q, B = K via ldmatrix), causal
// mask by position, online softmax in the exp2 domain, O += P V (A = P
// straight from the S accumulators, B = V via ldmatrix.trans). fp16
// operands, fp32 accumulation.
#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>

#include "kernels.h"
#include "ptx.cuh"

namespace tllm {
namespace {

constexpr int kPfWarps = 4;
constexpr int kPfRows = kPfWarps * 16;  // (query, head) rows per CTA
constexpr int kKeyTile = 64;            // keys per stage
constexpr int kKeyGroup = 16;           // keys per TMA box
constexpr uint64_t kPfWaitLimitNs = 2000000000ull;

template <int D>
struct PfCfg {
    static constexpr int kNSub = D / 64;                  // 64-half columns per row
    static constexpr int kSubBytes = kKeyGroup * 128;     // one [16][64] box
    static constexpr int kGroups = kKeyTile / kKeyGroup;  // boxes per tile, per K and V column
    static constexpr int kKBytes = kGroups * kNSub * kSubBytes;
    static constexpr int kStageBytes = 2 * kKBytes;       // K then V
    static constexpr int kNS = 3;
    static constexpr int kSmemBytes = kNS * kStageBytes + 2 * kNS * 8 + 1024;
    static constexpr int kKS = D / 16;  // k-steps of Q K^T
    static constexpr int kDN = D / 8;   // n-tiles of P V
};

// Byte offset of 16-byte chunk c (halves 8c .. 8c+7) of key row t in a
// [16][64] box with the 128-byte swizzle.
__device__ __forceinline__ uint32_t box_off(int t, int c) { return t * 128 + (((c & 7) ^ (t & 7)) << 4); }

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// Rotates two Q A-fragment registers (halves d, d+1 and their partners at
// d + D/2) by the RoPE table row (ct, st), each product and sum rounded
// separately and the result rounded to nearest even, as the append kernel
// rotates K.
__device__ __forceinline__ void rope_pair(uint32_t &lo, uint32_t &hi, const float *ct, const float *st, int d) {
    const float2 c = *reinterpret_cast<const float2 *>(ct + d);
    const float2 s = *reinterpret_cast<const float2 *>(st + d);
    const float2 x1 = __half22float2(*reinterpret_cast<const __half2 *>(&lo));
    const float2 x2 = __half22float2(*reinterpret_cast<const __half2 *>(&hi));
    const __half2 r1 = __halves2half2(__float2half_rn(__fsub_rn(__fmul_rn(x1.x, c.x), __fmul_rn(x2.x, s.x))),
                                      __float2half_rn(__fsub_rn(__fmul_rn(x1.y, c.y), __fmul_rn(x2.y, s.y))));
    const __half2 r2 = __halves2half2(__float2half_rn(__fadd_rn(__fmul_rn(x2.x, c.x), __fmul_rn(x1.x, s.x))),
                                      __float2half_rn(__fadd_rn(__fmul_rn(x2.y, c.y), __fmul_rn(x1.y, s.y))));
    lo = *reinterpret_cast<const uint32_t *>(&r1);
    hi = *reinterpret_cast<const uint32_t *>(&r2);
}

template <int D>
__global__ void __launch_bounds__((kPfWarps + 1) * 32, 2)
    paged_prefill_kernel(const __grid_constant__ CUtensorMap tmap, const __grid_constant__ PrefillArgs a) {
    using C = PfCfg<D>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::kNS * C::kStageBytes);  // full[kNS], empty[kNS]
    const uint32_t smem_u = ptx::smem_u32(smem);
    const uint32_t full_u = ptx::smem_u32(bars), empty_u = full_u + 8 * C::kNS;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gid = lane >> 2, tig = lane & 3;
    const PoolGeom &g = a.g;
    const int H = g.num_kv_heads, G = a.group, Gp = a.group_pad, Hq = H * G, BS = g.block_size;
    const int kvh = blockIdx.y;

    // sequence of this CTA: largest b with cta_prefix[b] <= blockIdx.x
    int lo = 0, hi = a.nseq - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (a.cta_prefix[mid] <= (int)blockIdx.x) lo = mid;
        else hi = mid - 1;
    }
    const int b = lo;
    const int qpb = kPfRows / Gp;                              // queries per CTA
    const int q0 = ((int)blockIdx.x - a.cta_prefix[b]) * qpb;  // first query of the CTA
    const int n = a.ntok[b], written = a.written[b];
    const int pos0 = written - n;                              // position of query 0
    const int q_last = min(n, q0 + qpb) - 1;
    const int ntiles = (pos0 + q_last) / kKeyTile + 1;         // keys [0, position of the last query]

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::kNS; ++s) {
            ptx::mbar_init(full_u + 8 * s, 1);
            ptx::mbar_init(empty_u + 8 * s, kPfWarps);
        }
        ptx::fence_barrier_init();
    }
    __syncthreads();

    // ---- producer: a tile = 4 groups x (K, V) x D/64 boxes ----
    const long long z_oob = 2ll * g.num_layers * g.num_blocks * (g.head_major ? H : BS);
    const int slot = a.slot[b];
    const uint64_t policy = ptx::l2_policy_evict_last();  // every query block reads these K/V
    auto issue_tile = [&](int kt) {
        const int s = kt % C::kNS;
        const uint32_t bar = full_u + 8 * s;
        ptx::fence_proxy_async_smem();
        ptx::mbar_arrive_expect_tx(bar, C::kStageBytes);
#pragma unroll
        for (int gi = 0; gi < C::kGroups; ++gi) {
            const int key0 = kt * kKeyTile + gi * kKeyGroup;
            int bid = -1, sub = 0;
            if (key0 < written) {
                bid = __ldg(g.block_tables + (long long)slot * g.bt_stride + key0 / BS);
                sub = key0 % BS;
                if (bid < 0 || bid >= g.num_blocks) {
                    atomicOr(g.err, kErrBlockRange);
                    bid = -1;
                }
            }
#pragma unroll
            for (int kv = 0; kv < 2; ++kv) {
                long long zz;
                int y;
                if (bid < 0) {  // past the sequence (or a bad id): zero-filled
                    zz = z_oob;
                    y = 0;
                } else {
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
                for (int hs = 0; hs < C::kNSub; ++hs)
                    ptx::tma_load_3d(smem_u + s * C::kStageBytes + kv * C::kKBytes +
                                         (gi * C::kNSub + hs) * C::kSubBytes,
                                     &tmap, bar, hs * 64, y, (int)zz, policy);
            }
        }
    };
    if (warp == kPfWarps) {  // the producer warp: refills each stage once every consumer is done
        if (lane == 0) {
            for (int kt = 0; kt < ntiles; ++kt) {
                if (kt >= C::kNS &&
                    !ptx::mbar_wait_bounded(empty_u + 8 * (kt % C::kNS), (uint32_t)(((kt / C::kNS) - 1) & 1),
                                            kPfWaitLimitNs)) {
                    atomicOr(g.err, kErrWaitTimeout);
                    break;
                }
                issue_tile(kt);
            }
        }
        return;
    }

    // ---- this warp's 16 rows: Q fragments (A operand) and positions ----
    const int rA = warp * 16 + gid, rB = rA + 8;  // CTA rows of this thread's two row slots
    const int qA = q0 + rA / Gp, qB = q0 + rB / Gp;
    const int gA = rA % Gp, gB = rB % Gp;
    const bool vA = qA <= q_last && gA < G, vB = qB <= q_last && gB < G;
    const int pA = pos0 + min(qA, q_last), pB = pos0 + min(qB, q_last);
    const __half *qrowA = static_cast<const __half *>(a.q) + ((long long)(a.row_off[b] + qA) * Hq + kvh * G + gA) * D;
    const __half *qrowB = static_cast<const __half *>(a.q) + ((long long)(a.row_off[b] + qB) * Hq + kvh * G + gB) * D;
    uint32_t qa[C::kKS][4];
#pragma unroll
    for (int ks = 0; ks < C::kKS; ++ks) {
        const int d = ks * 16 + 2 * tig;
        qa[ks][0] = vA ? __ldg(reinterpret_cast<const uint32_t *>(qrowA + d)) : 0u;
        qa[ks][1] = vB ? __ldg(reinterpret_cast<const uint32_t *>(qrowB + d)) : 0u;
        qa[ks][2] = vA ? __ldg(reinterpret_cast<const uint32_t *>(qrowA + d + 8)) : 0u;
        qa[ks][3] = vB ? __ldg(reinterpret_cast<const uint32_t *>(qrowB + d + 8)) : 0u;
    }
    if (a.rope_cos != nullptr) {
        if (pB >= a.rope_max_pos) {  // pA <= pB
            if (lane == 0) atomicOr(g.err, kErrPosRange);
        } else {
            const float *ctA = a.rope_cos + (long long)pA * (D / 2), *stA = a.rope_sin + (long long)pA * (D / 2);
            const float *ctB = a.rope_cos + (long long)pB * (D / 2), *stB = a.rope_sin + (long long)pB * (D / 2);
#pragma unroll
            for (int ks = 0; ks < C::kKS / 2; ++ks) {
                const int d = ks * 16 + 2 * tig;
                rope_pair(qa[ks][0], qa[ks + C::kKS / 2][0], ctA, stA, d);
                rope_pair(qa[ks][2], qa[ks + C::kKS / 2][2], ctA, stA, d + 8);
                rope_pair(qa[ks][1], qa[ks + C::kKS / 2][1], ctB, stB, d);
                rope_pair(qa[ks][3], qa[ks + C::kKS / 2][3], ctB, stB, d + 8);
            }
        }
    }

    float o[C::kDN][4];
#pragma unroll
    for (int j = 0; j < C::kDN; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float mA = -INFINITY, mB = -INFINITY, lA = 0.f, lB = 0.f;
    bool ok = true;

    // ldmatrix lane roles: K as the B operand of S = Q K^T (rows = keys),
    // V as the B operand of O += P V (transposed)
    const int k_key = (lane & 7) + ((lane >> 4) & 1) * 8, k_dsel = (lane >> 3) & 1;
    const int v_key = (lane & 7) + ((lane >> 3) & 1) * 8, v_dsel = (lane >> 4) & 1;

    for (int kt = 0; kt < ntiles; ++kt) {
        const int s = kt % C::kNS;
        const uint32_t parity = (uint32_t)((kt / C::kNS) & 1);
        if (!ptx::mbar_wait_bounded(full_u + 8 * s, parity, kPfWaitLimitNs)) {
            if (lane == 0) atomicOr(g.err, kErrWaitTimeout);
            ok = false;
        }
        const uint32_t kb = smem_u + s * C::kStageBytes, vb = kb + C::kKBytes;
        // The tile holding the sequence's last token: V rows past it (same
        // block, stale) are zeroed so that 0 * V stays 0.
        if ((kt + 1) * kKeyTile > written && written > kt * kKeyTile) {
            const int first_bad = written - kt * kKeyTile;  // 1..63
            uint8_t *vp = smem + s * C::kStageBytes + C::kKBytes;
            const int nchunks = (kKeyTile - first_bad) * C::kNSub * 8;
            for (int i = threadIdx.x; i < nchunks; i += kPfWarps * 32) {
                const int key = first_bad + i / (C::kNSub * 8), rem = i % (C::kNSub * 8);
                const int hs = rem / 8, c = rem % 8;
                const int gi = key / kKeyGroup, t = key % kKeyGroup;
                *reinterpret_cast<uint4 *>(vp + (gi * C::kNSub + hs) * C::kSubBytes + box_off(t, c)) =
                    make_uint4(0u, 0u, 0u, 0u);
            }
            ptx::named_barrier_sync(1, kPfWarps * 32);
        }

        // ---- S = Q K^T: 16 rows x 64 keys (8 n-tiles of 8 keys) ----
        float sc[8][4];
#pragma unroll
        for (int j = 0; j < 8; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
#pragma unroll
        for (int gi = 0; gi < C::kGroups; ++gi) {
#pragma unroll
            for (int ks = 0; ks < C::kKS; ++ks) {
                const int d = ks * 16 + k_dsel * 8;
                uint32_t b0, b1, b2, b3;
                ptx::ldmatrix_x4(kb + (gi * C::kNSub + (d >> 6)) * C::kSubBytes + box_off(k_key, (d & 63) >> 3),
                                 b0, b1, b2, b3);
                ptx::mma_16816(sc[2 * gi], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b0, b1);
                ptx::mma_16816(sc[2 * gi + 1], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b2, b3);
            }
        }
        // ---- causal mask, online softmax (exp2 domain) ----
        float mxA = -INFINITY, mxB = -INFINITY;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int key = kt * kKeyTile + j * 8 + 2 * tig;
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                sc[j][e] = key + e <= pA ? sc[j][e] * a.scale_log2 : -INFINITY;
                sc[j][2 + e] = key + e <= pB ? sc[j][2 + e] * a.scale_log2 : -INFINITY;
                mxA = fmaxf(mxA, sc[j][e]);
                mxB = fmaxf(mxB, sc[j][2 + e]);
            }
        }
#pragma unroll
        for (int off = 1; off < 4; off <<= 1) {
            mxA = fmaxf(mxA, __shfl_xor_sync(0xffffffffu, mxA, off));
            mxB = fmaxf(mxB, __shfl_xor_sync(0xffffffffu, mxB, off));
        }
        const float nA = fmaxf(mA, mxA), nB = fmaxf(mB, mxB);  // finite: key 0 <= every position
        const float alA = ptx::ex2(mA - nA), alB = ptx::ex2(mB - nB);
        mA = nA;
        mB = nB;
        float sumA = 0.f, sumB = 0.f;
        uint32_t pa[C::kGroups][4];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float p0 = ptx::ex2(sc[j][0] - nA), p1 = ptx::ex2(sc[j][1] - nA);
            const float p2 = ptx::ex2(sc[j][2] - nB), p3 = ptx::ex2(sc[j][3] - nB);
            sumA += p0 + p1;
            sumB += p2 + p3;
            pa[j >> 1][(j & 1) * 2 + 0] = pack2(p0, p1);  // row gid: keys 2tig (+8 for odd j)
            pa[j >> 1][(j & 1) * 2 + 1] = pack2(p2, p3);  // row gid + 8
        }
        lA = lA * alA + sumA;
        lB = lB * alB + sumB;
#pragma unroll
        for (int j = 0; j < C::kDN; ++j) {
            o[j][0] *= alA;
            o[j][1] *= alA;
            o[j][2] *= alB;
            o[j][3] *= alB;
        }
        // ---- O += P V: A = P (16 rows x 16 keys per group), B = V ----
#pragma unroll
        for (int gi = 0; gi < C::kGroups; ++gi) {
#pragma unroll
            for (int dp = 0; dp < D / 16; ++dp) {
                const int d = dp * 16 + v_dsel * 8;
                uint32_t b0, b1, b2, b3;
                ptx::ldmatrix_x4_trans(vb + (gi * C::kNSub + (d >> 6)) * C::kSubBytes + box_off(v_key, (d & 63) >> 3),
                                       b0, b1, b2, b3);
                ptx::mma_16816(o[2 * dp], pa[gi][0], pa[gi][1], pa[gi][2], pa[gi][3], b0, b1);
                ptx::mma_16816(o[2 * dp + 1], pa[gi][0], pa[gi][1], pa[gi][2], pa[gi][3], b2, b3);
            }
        }
        // ---- release the stage to the producer warp ----
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(empty_u + 8 * s);
        if (!__all_sync(0xffffffffu, ok)) break;
    }
    if (!ok) return;  // the call reports the error; no output written

    // ---- normalise and store this thread's rows ----
    float lsA = lA, lsB = lB;
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
        lsA += __shfl_xor_sync(0xffffffffu, lsA, off);
        lsB += __shfl_xor_sync(0xffffffffu, lsB, off);
    }
    const float iA = 1.f / lsA, iB = 1.f / lsB;
    __half *orowA = static_cast<__half *>(a.o) + ((long long)(a.row_off[b] + qA) * Hq + kvh * G + gA) * D;
    __half *orowB = static_cast<__half *>(a.o) + ((long long)(a.row_off[b] + qB) * Hq + kvh * G + gB) * D;
#pragma unroll
    for (int j = 0; j < C::kDN; ++j) {
        const int d = j * 8 + 2 * tig;
        if (vA) *reinterpret_cast<uint32_t *>(orowA + d) = pack2(o[j][0] * iA, o[j][1] * iA);
        if (vB) *reinterpret_cast<uint32_t *>(orowB + d) = pack2(o[j][2] * iB, o[j][3] * iB);
    }
}

template <int D>
cudaError_t launch_prefill_t(const PrefillArgs &a, const void *tmap128, cudaStream_t s) {
    static_assert(PfCfg<D>::kSmemBytes <= 227 * 1024, "prefill ring too large");
    cudaError_t e = cudaFuncSetAttribute(paged_prefill_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         PfCfg<D>::kSmemBytes);
    if (e != cudaSuccess) return e;
    const int ctas = a.cta_prefix[a.nseq];
    if (ctas <= 0) return cudaSuccess;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ctas, a.g.num_kv_heads);
    cfg.blockDim = dim3((kPfWarps + 1) * 32);
    cfg.dynamicSmemBytes = PfCfg<D>::kSmemBytes;
    cfg.stream = s;
    return cudaLaunchKernelEx(&cfg, paged_prefill_kernel<D>, *static_cast<const CUtensorMap *>(tmap128), a);
}

}  // namespace

int prefill_rows_per_cta() { return kPfRows; }

cudaError_t launch_prefill(const PrefillArgs &a, const void *tmap128, cudaStream_t s) {
    switch (a.g.head_dim) {
    case 64: return launch_prefill_t<64>(a, tmap128, s);
    case 128: return launch_prefill_t<128>(a, tmap128, s);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace tllm
