// Fused Q/K/V projection (W8A16) + KV append (+ RoPE on Q and K) into the
// paged pool, for one decode token per sequence, sm_100a.
//
// Replaces, for the decode step of TransformerLayer::attention
// (reference src/transformer.cpp:209-226), the three kernels::w8a16_matmul
// calls into q_buf_/k_buf_/v_buf_ (reference kernels/w8a16_matmul.cu:119-235,
// int8 weight [K][N] row-major, fp16 scale [K/group][N], fp32 accumulation,
// fp16 result) and the appendKV copy of k_buf_/v_buf_ into the cache
// (src/kv_cache.cpp:206-233): K and V rows go straight from the projection
// into their block slots, and Q comes out rotated for the decode kernel.
//
// The op streams the weights once (int8 + scales: HBM-bound), so the work is
// split over CTAs by column tile (one head of Q, K or V: D columns) and by
// K-chunk (split-K), about three CTAs per SM. In a CTA, warp w owns 32
// columns and thread (gid, tig) four adjacent columns 4*gid .. 4*gid+3: one
// 32-bit load of a weight row gives those four columns, and the n8 tile j of
// the m16n8k16 MMA is given column 4*gid + j, so byte permutes of two rows'
// words make the B fragments directly (int8 -> fp16 is exact: the byte
// lands in the mantissa of 1024.0 and 1152 is subtracted). With that
// column order each thread's accumulators are 8 adjacent columns, whose
// scales are one 16-byte load. Each group of K (group elements sharing a
// scale) is summed in its own fp32 accumulator by the MMA and then scaled
// into the running sum: sum_g s_g * (sum_k a_k w_k), the reference's sum of
// a_k * (w_k * s_g) with the products grouped. The batch rows are the M side
// (16 per MMA row tile, up to 64 rows per launch); activations of the CTA's
// K-chunk are staged in shared memory for ldmatrix.
//
// Split-K: every CTA adds its fp32 sums into the column tile's accumulator
// with vector reductions in L2 (so the order of the K-chunks' sums varies
// between runs, at fp32 rounding level); the last to finish the tile (a
// counter per tile, reset by that CTA) reads the total, zeroes the
// accumulator, rounds to fp16 like the reference's output, rotates Q and K
// pairs (d, d + D/2) by the RoPE table at the row's position exactly as the
// append kernel does, and writes Q to q_out and K/V into the pool.
#include <atomic>
#include <map>
#include <mutex>
#include <cstdint>
#include <cuda_fp16.h>

#include "kernels.h"
#include "ptx.cuh"

namespace tllm {
namespace {

constexpr int kQkvKBlock = 128;  // K per batch of weight loads (8 MMA k-steps)

__device__ __forceinline__ long long pool_off(const PoolGeom &g, int layer, int kv, int block, int tok, int head) {
    const long long block_elems = (long long)g.block_size * g.num_kv_heads * g.head_dim;
    const long long base = ((long long)(layer * 2 + kv) * g.num_blocks + block) * block_elems;
    if (g.head_major) return base + ((long long)head * g.block_size + tok) * g.head_dim;
    return base + ((long long)tok * g.num_kv_heads + head) * g.head_dim;
}

__device__ __forceinline__ uint32_t ldg_u32(const int8_t *p) {
    uint32_t r;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r) : "l"(p));
    return r;
}

// fp16 pair (lo = byte j of row word a, hi = byte j of row word b) from
// int8 words already XORed with 0x80 (signed -> excess-128).
template <int J>
__device__ __forceinline__ uint32_t i8x2_to_h2(uint32_t a, uint32_t b) {
    uint32_t t;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(t) : "r"(a), "r"(b), "n"(J | ((4 + J) << 8)));
    t = (t & 0x00FF00FFu) | 0x64006400u;  // 1024 + (x + 128) per half
    const __half2 h = __hsub2(*reinterpret_cast<const __half2 *>(&t), __halves2half2(__ushort_as_half(0x6480),
                                                                                     __ushort_as_half(0x6480)));
    return *reinterpret_cast<const uint32_t *>(&h);
}

// Four fp32 additions into global memory (L2 reduction, no return value).
__device__ __forceinline__ void red_add_v4(float *p, float x, float y, float z, float w) {
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(x), "f"(y), "f"(z), "f"(w)
                 : "memory");
}

// RoPE on 8 pairs, rounded as the append kernel rounds (kv_append.cu).
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

template <int D, int MT, int GS>
__global__ void __launch_bounds__(D) qkv_append_kernel(const __grid_constant__ QkvArgs a) {
    constexpr int R = 16 * MT;       // padded rows
    constexpr int SPG = GS / 16;     // MMA k-steps per scale group
    static_assert(GS % 16 == 0 && kQkvKBlock % GS == 0, "group size");
    extern __shared__ __align__(16) uint8_t smem[];
    const PoolGeom &g = a.g;
    const int kc = blockIdx.x, tile = blockIdx.y;
    const int Hq = a.num_q_heads, Hkv = g.num_kv_heads;
    const int m = tile < Hq ? 0 : (tile < Hq + Hkv ? 1 : 2);  // Q, K or V
    const int head = tile - (m == 0 ? 0 : (m == 1 ? Hq : Hq + Hkv));
    const int N = a.n[m];
    const int k0 = kc * a.kchunk;
    const int klen = min(a.kchunk, a.K - k0);  // a multiple of kQkvKBlock
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
    const int cw = head * D + 32 * warp;  // first column of this warp in matrix m

    const int8_t *W = a.w[m] + (long long)(k0 + 2 * tig) * N + cw + 4 * gid;
    const __half *S = static_cast<const __half *>(a.sc[m]) + cw + 8 * tig;
    // a block of 128 K: the weight words (rows 2tig, 2tig+1, 2tig+8, 2tig+9
    // of each of its 8 k-steps) and its scales
    struct Blk {
        uint32_t w[8][4];
        uint4 sc[kQkvKBlock / GS];
    };
    auto load = [&](Blk &bk, int kb) {
#pragma unroll
        for (int st = 0; st < 8; ++st) {
            const int8_t *p = W + (long long)(kb + 16 * st) * N;
            bk.w[st][0] = ldg_u32(p);
            bk.w[st][1] = ldg_u32(p + N);
            bk.w[st][2] = ldg_u32(p + 8 * (long long)N);
            bk.w[st][3] = ldg_u32(p + 9 * (long long)N);
        }
#pragma unroll
        for (int gi = 0; gi < kQkvKBlock / GS; ++gi)
            bk.sc[gi] = __ldg(reinterpret_cast<const uint4 *>(S + (long long)((k0 + kb) / GS + gi) * N));
    };
    Blk blk[2];
    load(blk[0], 0);  // in flight while the activations are staged

    // activations of this K-chunk: [R][ldx] fp16 (rows past a.rows are 0)
    const int ldx = a.kchunk + 8;
    __half *sx = reinterpret_cast<__half *>(smem);
    {  // asynchronous copies, all in flight at once (rows past a.rows zero-filled)
        const int cpr = klen / 8;
        const __half *x = static_cast<const __half *>(a.x);
        const uint32_t sx0 = ptx::smem_u32(sx);
        for (int i = threadIdx.x; i < R * cpr; i += D) {
            const int r = i / cpr, c = i % cpr;
            const bool in = r < a.rows;
            ptx::cp_async16(sx0 + (uint32_t)((r * ldx + c * 8) * 2), x + (in ? (long long)r * a.K + k0 + c * 8 : 0),
                            in ? 16u : 0u);
        }
        ptx::cp_async_wait_all();
    }
    __syncthreads();

    float acc[MT][4][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[mt][j][0] = acc[mt][j][1] = acc[mt][j][2] = acc[mt][j][3] = 0.f;

    const uint32_t sx_u = ptx::smem_u32(sx) + (uint32_t)(((lane & 15) * ldx + (lane >> 4) * 8) * 2);
    auto compute = [&](const Blk &bk, int kb) {
        float t[MT][4][4];
#pragma unroll
        for (int st = 0; st < 8; ++st) {
            if (st % SPG == 0) {
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                    for (int j = 0; j < 4; ++j) t[mt][j][0] = t[mt][j][1] = t[mt][j][2] = t[mt][j][3] = 0.f;
            }
            const uint32_t x0 = bk.w[st][0] ^ 0x80808080u, x1 = bk.w[st][1] ^ 0x80808080u;
            const uint32_t x8 = bk.w[st][2] ^ 0x80808080u, x9 = bk.w[st][3] ^ 0x80808080u;
            uint32_t b[4][2];
            b[0][0] = i8x2_to_h2<0>(x0, x1);
            b[0][1] = i8x2_to_h2<0>(x8, x9);
            b[1][0] = i8x2_to_h2<1>(x0, x1);
            b[1][1] = i8x2_to_h2<1>(x8, x9);
            b[2][0] = i8x2_to_h2<2>(x0, x1);
            b[2][1] = i8x2_to_h2<2>(x8, x9);
            b[3][0] = i8x2_to_h2<3>(x0, x1);
            b[3][1] = i8x2_to_h2<3>(x8, x9);
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                uint32_t a0, a1, a2, a3;
                ptx::ldmatrix_x4(sx_u + (uint32_t)((mt * 16 * ldx + kb + 16 * st) * 2), a0, a1, a2, a3);
#pragma unroll
                for (int j = 0; j < 4; ++j) ptx::mma_16816(t[mt][j], a0, a1, a2, a3, b[j][0], b[j][1]);
            }
            if (st % SPG == SPG - 1) {  // group complete: scale into the running sums
                const __half *sh = reinterpret_cast<const __half *>(&bk.sc[st / SPG]);
                float sv[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) sv[i] = __half2float(sh[i]);
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        acc[mt][j][0] = fmaf(t[mt][j][0], sv[j], acc[mt][j][0]);
                        acc[mt][j][1] = fmaf(t[mt][j][1], sv[4 + j], acc[mt][j][1]);
                        acc[mt][j][2] = fmaf(t[mt][j][2], sv[j], acc[mt][j][2]);
                        acc[mt][j][3] = fmaf(t[mt][j][3], sv[4 + j], acc[mt][j][3]);
                    }
            }
        }
    };
    // two blocks in registers: the next one's loads fly while this one's math runs
    for (int kb = 0; kb < klen; kb += 2 * kQkvKBlock) {
        const bool b1 = kb + kQkvKBlock < klen;
        if (b1) load(blk[1], kb + kQkvKBlock);
        compute(blk[0], kb);
        if (b1) {
            if (kb + 2 * kQkvKBlock < klen) load(blk[0], kb + 2 * kQkvKBlock);
            compute(blk[1], kb + kQkvKBlock);
        }
    }

    // this thread's sums: rows mt*16 + gid (+8), columns 32*warp + 8*tig + {j, 4 + j}
    const int ccol = 32 * warp + 8 * tig;
    if (a.ksplit > 1) {
        // every CTA adds its sums into the tile's fp32 accumulator (zero
        // between launches); the last to arrive reads the total back and
        // zeroes the accumulator for the next launch
        __shared__ int s_last;
        float *tacc = a.partial + (long long)tile * R * D;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                float *pr = tacc + (mt * 16 + gid + 8 * h) * D + ccol;
                red_add_v4(pr, acc[mt][0][2 * h], acc[mt][1][2 * h], acc[mt][2][2 * h], acc[mt][3][2 * h]);
                red_add_v4(pr + 4, acc[mt][0][2 * h + 1], acc[mt][1][2 * h + 1], acc[mt][2][2 * h + 1],
                           acc[mt][3][2 * h + 1]);
            }
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) {
            const int prev = atomicAdd(&a.counters[tile], 1);
            s_last = prev == a.ksplit - 1;
            if (s_last) a.counters[tile] = 0;  // ready for the next launch
        }
        __syncthreads();
        if (!s_last) return;
        __threadfence();
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                float4 *pr = reinterpret_cast<float4 *>(tacc + (mt * 16 + gid + 8 * h) * D + ccol);
                const float4 lo = __ldcg(pr), hi = __ldcg(pr + 1);
                __stcg(pr, make_float4(0.f, 0.f, 0.f, 0.f));
                __stcg(pr + 1, make_float4(0.f, 0.f, 0.f, 0.f));
                acc[mt][0][2 * h] = lo.x; acc[mt][1][2 * h] = lo.y; acc[mt][2][2 * h] = lo.z; acc[mt][3][2 * h] = lo.w;
                acc[mt][0][2 * h + 1] = hi.x; acc[mt][1][2 * h + 1] = hi.y;
                acc[mt][2][2 * h + 1] = hi.z; acc[mt][3][2 * h + 1] = hi.w;
            }
    }

    // fp16 rows of this head into shared memory, then rotate and store
    __syncthreads();  // sx is reused
    __half *sy = sx;  // [R][D]
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            __half *dst = sy + (mt * 16 + gid + 8 * h) * D + ccol;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                dst[j] = __float2half_rn(acc[mt][j][2 * h]);
                dst[4 + j] = __float2half_rn(acc[mt][j][2 * h + 1]);
            }
        }
    __syncthreads();
    const bool rope = a.rope_cos != nullptr && m < 2;
    constexpr int kChunks = D / 16;  // 8-half chunks per half row
    for (int i = threadIdx.x; i < a.rows * kChunks; i += D) {
        const int r = i / kChunks, c = i % kChunks;
        uint4 x1 = *reinterpret_cast<const uint4 *>(sy + r * D + 8 * c);
        uint4 x2 = *reinterpret_cast<const uint4 *>(sy + r * D + D / 2 + 8 * c);
        const int pos = a.row_pos[r];
        if (rope) {
            if (pos < 0 || pos >= a.rope_max_pos) {
                atomicOr(g.err, kErrPosRange);
                continue;
            }
            rope8(x1, x2, a.rope_cos + (long long)pos * (D / 2) + 8 * c, a.rope_sin + (long long)pos * (D / 2) + 8 * c);
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

// The row tile (16 * MT) for a launch of `rows` rows.
int mt_for(int rows) { return rows <= 16 ? 1 : (rows <= 32 ? 2 : 4); }

template <int D, int MT>
cudaError_t launch_mt(const QkvArgs &a, cudaStream_t s) {
    const int smem = max(16 * MT * (a.kchunk + 8), 16 * MT * D) * 2;
    const dim3 grid(a.ksplit, a.num_q_heads + 2 * a.g.num_kv_heads);
    cudaError_t e = cudaSuccess;
    auto go = [&](auto kern) {
        // the shared-memory opt-in of this kernel on this device, only ever
        // raised; the check, the set and the record happen under one lock so
        // host threads launching different chunk sizes cannot leave the
        // record above the attribute
        static std::mutex mu;
        static std::map<std::pair<int, const void *>, int> opted;  // (device, kernel) -> bytes
        int dev = 0;
        e = cudaGetDevice(&dev);
        if (e == cudaSuccess) {
            std::lock_guard<std::mutex> lock(mu);
            int &cur = opted[{dev, reinterpret_cast<const void *>(kern)}];
            if (cur < smem) {
                e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
                if (e == cudaSuccess) cur = smem;
            }
        }
        if (e == cudaSuccess) {
            kern<<<grid, D, smem, s>>>(a);
            e = cudaGetLastError();
        }
    };
    switch (a.group) {
    case 16: go(qkv_append_kernel<D, MT, 16>); break;
    case 32: go(qkv_append_kernel<D, MT, 32>); break;
    case 64: go(qkv_append_kernel<D, MT, 64>); break;
    case 128: go(qkv_append_kernel<D, MT, 128>); break;
    default: return cudaErrorInvalidValue;
    }
    return e;
}

template <int D>
cudaError_t launch_d(const QkvArgs &a, cudaStream_t s) {
    switch (mt_for(a.rows)) {
    case 1: return launch_mt<D, 1>(a, s);
    case 2: return launch_mt<D, 2>(a, s);
    default: return launch_mt<D, 4>(a, s);
    }
}

}  // namespace

int qkv_k_block() { return kQkvKBlock; }
int qkv_rows_padded(int rows) { return 16 * mt_for(rows); }

cudaError_t launch_qkv_append(const QkvArgs &a, cudaStream_t s) {
    if (a.rows <= 0) return cudaSuccess;
    if (a.rows > kMaxQkvRows) return cudaErrorInvalidValue;
    switch (a.g.head_dim) {
    case 64: return launch_d<64>(a, s);
    case 128: return launch_d<128>(a, s);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace tllm
