// Fused KV append (+ RoPE on K) into the paged pool, sm_100a.
//
// Replaces the reference's two cudaMemcpyAsync per (sequence, layer)
// (src/kv_cache.cpp:226-233): one launch writes every token row of every
// requested layer into its block slot. Grid = (rows, layers); each CTA moves
// one token row of one layer (Hkv x D halves of K and of V) with 16-byte
// vector loads/stores. With RoPE on, K pairs (i, i + D/2) are rotated by the
// host-built fp32 cos/sin table at the row's position; every product and sum
// is rounded separately (__fmul_rn / __fsub_rn / __fadd_rn), then converted
// with round-to-nearest-even, so results are bit-identical to the CPU
// restatement of the documented rotate-half math.
#include <cstdint>
#include <cuda_fp16.h>

#include "kernels.h"

namespace tllm {
namespace {

__device__ __forceinline__ long long pool_offset(const PoolGeom &g, int layer, int kv, int block,
                                                 int tok, int head) {
    const long long block_elems = (long long)g.block_size * g.num_kv_heads * g.head_dim;
    const long long base = ((long long)(layer * 2 + kv) * g.num_blocks + block) * block_elems;
    if (g.head_major) return base + ((long long)head * g.block_size + tok) * g.head_dim;
    return base + ((long long)tok * g.num_kv_heads + head) * g.head_dim;
}

__device__ __forceinline__ uint4 ld_stream(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ void rope8(const uint4 &x1v, const uint4 &x2v, const float *c,
                                      const float *s, uint4 &o1v, uint4 &o2v) {
    const __half *x1 = reinterpret_cast<const __half *>(&x1v);
    const __half *x2 = reinterpret_cast<const __half *>(&x2v);
    __half *o1 = reinterpret_cast<__half *>(&o1v);
    __half *o2 = reinterpret_cast<__half *>(&o2v);
    const float4 c0 = reinterpret_cast<const float4 *>(c)[0];
    const float4 c1 = reinterpret_cast<const float4 *>(c)[1];
    const float4 s0 = reinterpret_cast<const float4 *>(s)[0];
    const float4 s1 = reinterpret_cast<const float4 *>(s)[1];
    const float cc[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    const float ss[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float a = __half2float(x1[i]);
        const float b = __half2float(x2[i]);
        const float r1 = __fsub_rn(__fmul_rn(a, cc[i]), __fmul_rn(b, ss[i]));
        const float r2 = __fadd_rn(__fmul_rn(b, cc[i]), __fmul_rn(a, ss[i]));
        o1[i] = __float2half_rn(r1);
        o2[i] = __float2half_rn(r2);
    }
}

__global__ void __launch_bounds__(128) append_kernel(const __grid_constant__ AppendArgs a) {
    const PoolGeom &g = a.g;
    const int row = blockIdx.x;
    const int lyr = blockIdx.y;
    const int layer = a.layer0 + lyr;

    // Block-table updates queued by the host (new blocks of growing
    // sequences). Nothing in this kernel reads the tables.
    if (row == 0 && lyr == 0) {
        for (int i = threadIdx.x; i < a.ndeltas; i += blockDim.x)
            g.block_tables[(long long)a.delta_slot[i] * g.bt_stride + a.delta_idx[i]] =
                a.delta_block[i];
    }

    const int block = a.row_block[row];
    const int pos = a.row_pos[row];
    const bool rope = a.rope_cos != nullptr;
    if (block < 0 || block >= g.num_blocks || pos < 0) {
        if (threadIdx.x == 0) atomicOr(g.err, kErrBlockRange);
        return;
    }
    if (rope && pos >= a.rope_max_pos) {
        if (threadIdx.x == 0) atomicOr(g.err, kErrPosRange);
        return;
    }
    const int tok = pos % g.block_size;
    const int D = g.head_dim, H = g.num_kv_heads;
    const __half *ks = static_cast<const __half *>(a.k) + lyr * a.src_layer_stride + row * a.src_row_stride;
    const __half *vs = static_cast<const __half *>(a.v) + lyr * a.src_layer_stride + row * a.src_row_stride;
    __half *pool = static_cast<__half *>(g.pool);

    const bool vec = (D % 16 == 0) && ((reinterpret_cast<uintptr_t>(ks) | reinterpret_cast<uintptr_t>(vs)) & 15) == 0;
    if (vec) {
        const int cpr = D / 8;  // 16-byte chunks per head row
        for (int i = threadIdx.x; i < H * cpr; i += blockDim.x) {
            const int h = i / cpr, c = i % cpr;
            const uint4 val = ld_stream(vs + h * D + c * 8);
            *reinterpret_cast<uint4 *>(pool + pool_offset(g, layer, 1, block, tok, h) + c * 8) = val;
        }
        if (!rope) {
            for (int i = threadIdx.x; i < H * cpr; i += blockDim.x) {
                const int h = i / cpr, c = i % cpr;
                const uint4 val = ld_stream(ks + h * D + c * 8);
                *reinterpret_cast<uint4 *>(pool + pool_offset(g, layer, 0, block, tok, h) + c * 8) = val;
            }
        } else {
            const int hd = D / 2, cph = hd / 8;  // chunks per half row
            const float *ct = a.rope_cos + (long long)pos * hd;
            const float *st = a.rope_sin + (long long)pos * hd;
            for (int i = threadIdx.x; i < H * cph; i += blockDim.x) {
                const int h = i / cph, c = i % cph;
                const uint4 x1 = ld_stream(ks + h * D + c * 8);
                const uint4 x2 = ld_stream(ks + h * D + hd + c * 8);
                uint4 o1, o2;
                rope8(x1, x2, ct + c * 8, st + c * 8, o1, o2);
                __half *dst = pool + pool_offset(g, layer, 0, block, tok, h);
                *reinterpret_cast<uint4 *>(dst + c * 8) = o1;
                *reinterpret_cast<uint4 *>(dst + hd + c * 8) = o2;
            }
        }
    } else {
        // Any head_dim / alignment: element-wise.
        for (int i = threadIdx.x; i < H * D; i += blockDim.x) {
            const int h = i / D, d = i % D;
            pool[pool_offset(g, layer, 1, block, tok, h) + d] = vs[h * D + d];
        }
        if (!rope) {
            for (int i = threadIdx.x; i < H * D; i += blockDim.x) {
                const int h = i / D, d = i % D;
                pool[pool_offset(g, layer, 0, block, tok, h) + d] = ks[h * D + d];
            }
        } else {
            const int hd = D / 2;
            for (int i = threadIdx.x; i < H * hd; i += blockDim.x) {
                const int h = i / hd, d = i % hd;
                const float x1 = __half2float(ks[h * D + d]);
                const float x2 = __half2float(ks[h * D + hd + d]);
                const float c = a.rope_cos[(long long)pos * hd + d];
                const float s = a.rope_sin[(long long)pos * hd + d];
                __half *dst = pool + pool_offset(g, layer, 0, block, tok, h);
                dst[d] = __float2half_rn(__fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s)));
                dst[hd + d] = __float2half_rn(__fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s)));
            }
        }
    }
}

__global__ void apply_deltas_kernel(const __grid_constant__ DeltaArgs a) {
    for (int i = threadIdx.x; i < a.ndeltas; i += blockDim.x)
        a.block_tables[(long long)a.delta_slot[i] * a.bt_stride + a.delta_idx[i]] = a.delta_block[i];
}

}  // namespace

cudaError_t launch_append(const AppendArgs &a, cudaStream_t s) {
    if (a.nrows <= 0 || a.num_layers <= 0) return cudaSuccess;
    dim3 grid(a.nrows, a.num_layers);
    append_kernel<<<grid, 128, 0, s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_apply_deltas(const DeltaArgs &a, cudaStream_t s) {
    if (a.ndeltas <= 0) return cudaSuccess;
    apply_deltas_kernel<<<1, 128, 0, s>>>(a);
    return cudaGetLastError();
}

}  // namespace tllm
