// On-device token sampling from fp16 logits, sm_100a.
//
// Replaces the host round trip of InferenceEngine::sampleFromHidden
// (reference src/inference_engine.cpp:296-307: a stream synchronize, a
// device-to-host copy of the logits and the host samplers of :330-490) with
// one launch that leaves the token ids in device memory, for every row of a
// batch. The strategies keep the reference's definitions:
//   greedy       the first index of the largest logit (sampleGreedy);
//   temperature  softmax((l - max) / T) over the vocabulary;
//   top-k        softmax over the k largest logits;
//   top-p        softmax over all, then the smallest prefix of the logits in
//                descending order whose probability reaches p.
// (T clamped to >= 1e-5, k to [1, V], p to [1e-5, 1], as the reference
// does.) The draw is an inverse CDF over the candidates in descending logit
// order, equal logits by ascending index, with a counter-based uniform of
// (seed, step, row); the reference draws with std::mt19937 and
// std::discrete_distribution, so tokens match in distribution, not draw by
// draw.
//
// One CTA per row. fp16 logits map to 16-bit keys that order like the
// values (-0 folded into +0, NaN lowest), so thresholds and the draw are
// found with 256-bin histograms over the key's high byte, then its low byte
// within one bin (counts for top-k, probability mass for top-p and the
// draw), and the index among equal keys with one block-wide scan. Every pass
// reads the row again (from L2 after the first).
#include <cstdint>
#include <cuda_fp16.h>

#include "kernels.h"

namespace tllm {
namespace {

constexpr int kSampleThreads = 1024;

__device__ __forceinline__ uint32_t key_of(uint16_t h) {
    if ((h & 0x7C00u) == 0x7C00u && (h & 0x03FFu) != 0) return 0u;  // NaN: below everything
    if (h == 0x8000u) h = 0;                                         // -0 == +0
    return (h & 0x8000u) ? (~h & 0xFFFFu) : (h | 0x8000u);
}
__device__ __forceinline__ float value_of(uint32_t key) {
    const uint16_t h = (key & 0x8000u) ? (uint16_t)(key & 0x7FFFu) : (uint16_t)(~key & 0xFFFFu);
    return __half2float(__ushort_as_half(h));
}

// splitmix64: the uniform of (seed, step, row) in [0, 1), 24 bits.
__device__ __forceinline__ float uniform_of(unsigned long long seed, unsigned long long step, int row) {
    unsigned long long z = seed ^ (0x9E3779B97F4A7C15ull * (unsigned long long)(row + 1)) ^
                           (0xD1B54A32D192ED03ull * (step + 1));
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z ^= z >> 31;
    return (float)(z >> 40) * (1.0f / 16777216.0f);
}

template <typename T, typename Op>
__device__ T block_reduce(T v, Op op, T *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        v = red[lane];  // blockDim.x == 1024: 32 warps
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (lane == 0) red[0] = v;
    }
    __syncthreads();
    const T r = red[0];
    __syncthreads();
    return r;
}

// Scans a 256-bin histogram from the top bin down; returns the bin where the
// running total first exceeds `target` (or reaches it, when `reach`), and
// the total of the bins above it. -1 when it never does.
template <typename T>
__device__ int scan_down(const T *hist, T target, bool reach, T *above) {
    T run = 0;
    for (int b = 255; b >= 0; --b) {
        const T next = run + hist[b];
        if (reach ? next >= target : next > target) {
            *above = run;
            return b;
        }
        run = next;
    }
    *above = run;
    return -1;
}

__global__ void __launch_bounds__(kSampleThreads) sample_kernel(const __grid_constant__ SampleArgs a) {
    __shared__ float fh[256];
    __shared__ unsigned int ch[256];
    __shared__ unsigned long long red64[32];
    __shared__ float redf[32];
    __shared__ int s_bin, s_idx;
    __shared__ float s_f0, s_f1;
    __shared__ unsigned int s_u0;
    const int row = blockIdx.x, tid = threadIdx.x, V = a.vocab;
    const uint16_t *lg = static_cast<const uint16_t *>(a.logits) + (long long)row * a.row_stride;

    // largest key, first index: max of (key << 32 | ~index)
    unsigned long long best = 0;
    for (int i = tid; i < V; i += kSampleThreads) {
        const unsigned long long v = ((unsigned long long)key_of(lg[i]) << 32) | (0xFFFFFFFFu - (unsigned)i);
        best = v > best ? v : best;
    }
    best = block_reduce(best, [](unsigned long long x, unsigned long long y) { return x > y ? x : y; }, red64);
    const uint32_t kmax = (uint32_t)(best >> 32);
    const int argmax = (int)(0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFu));
    if (a.mode == 0 || kmax == 0u) {  // greedy (a NaN first logit wins in the reference's loop); all NaN: 0
        if (tid == 0) {
            const uint16_t h0 = lg[0];
            const bool nan0 = (h0 & 0x7C00u) == 0x7C00u && (h0 & 0x03FFu) != 0;
            a.tokens[row] = nan0 || kmax == 0u ? 0 : argmax;
        }
        return;
    }
    const float m = value_of(kmax);
    const float c = 1.4426950408889634f / a.temperature;  // exp((l - m) / T) = 2^((l - m) c)
    auto weight = [&](uint32_t key) { return key == 0u ? 0.f : exp2f((value_of(key) - m) * c); };  // NaN: 0
    if (tid == 0) a.tokens[row] = argmax;  // replaced below by the drawn token

    // ---- the candidate threshold: the lowest key kt of the candidates, the
    // count (top-k) or mass (top-p) above it, and how many of its ties join
    uint32_t kt;
    float mass_gt;   // probability mass of keys > kt (unnormalised)
    int need_eq;     // tokens with key == kt among the candidates (ascending index)
    auto clear = [&]() {
        for (int b = tid; b < 256; b += kSampleThreads) {
            fh[b] = 0.f;
            ch[b] = 0u;
        }
        __syncthreads();
    };
    if (a.mode == 1) {  // top-k (temperature: k = V)
        const unsigned int k = (unsigned int)a.top_k;
        clear();
        for (int i = tid; i < V; i += kSampleThreads) atomicAdd(&ch[key_of(lg[i]) >> 8], 1u);
        __syncthreads();
        if (tid == 0) {
            unsigned int above = 0;
            s_bin = scan_down<unsigned int>(ch, k, true, &above);
            s_u0 = above;
        }
        __syncthreads();
        const int bh = s_bin;
        const unsigned int c_above = s_u0;
        __syncthreads();
        clear();
        for (int i = tid; i < V; i += kSampleThreads) {
            const uint32_t key = key_of(lg[i]);
            if ((int)(key >> 8) == bh) atomicAdd(&ch[key & 0xFFu], 1u);
        }
        __syncthreads();
        if (tid == 0) {
            unsigned int above = 0;
            const int bl = scan_down<unsigned int>(ch, k - c_above, true, &above);
            s_bin = (bh << 8) | bl;
            s_u0 = k - c_above - above;  // ties of kt taken
        }
        __syncthreads();
        kt = (uint32_t)s_bin;
        need_eq = (int)s_u0;
        float ms = 0.f;
        for (int i = tid; i < V; i += kSampleThreads) {
            const uint32_t key = key_of(lg[i]);
            if (key > kt) ms += weight(key);
        }
        mass_gt = block_reduce(ms, [](float x, float y) { return x + y; }, redf);
    } else {  // top-p: the smallest descending prefix reaching p of the total
        clear();
        float z = 0.f;
        for (int i = tid; i < V; i += kSampleThreads) {
            const uint32_t key = key_of(lg[i]);
            const float w = weight(key);
            z += w;
            atomicAdd(&fh[key >> 8], w);
        }
        z = block_reduce(z, [](float x, float y) { return x + y; }, redf);
        const float target = a.top_p * z;
        if (tid == 0) {
            float above = 0.f;
            int b = scan_down<float>(fh, target, true, &above);
            if (b < 0) {  // rounding: everything
                b = 0;
                above = 0.f;
                while (b < 255 && fh[b] == 0.f) ++b;
                above = 0.f;
                for (int q = 255; q > b; --q) above += fh[q];
            }
            s_bin = b;
            s_f0 = above;
        }
        __syncthreads();
        const int bh = s_bin;
        const float m_above = s_f0;
        __syncthreads();
        clear();
        for (int i = tid; i < V; i += kSampleThreads) {
            const uint32_t key = key_of(lg[i]);
            if ((int)(key >> 8) == bh) {
                atomicAdd(&fh[key & 0xFFu], weight(key));
                atomicAdd(&ch[key & 0xFFu], 1u);
            }
        }
        __syncthreads();
        if (tid == 0) {
            float above = 0.f;
            int bl = scan_down<float>(fh, target - m_above, true, &above);
            if (bl < 0) {  // rounding: the lowest key of the bin
                bl = 0;
                while (bl < 255 && ch[bl] == 0u) ++bl;
                above = 0.f;
                for (int q = 255; q > bl; --q) above += fh[q];
            }
            const uint32_t key = ((uint32_t)bh << 8) | (uint32_t)bl;
            const float wt = weight(key);
            const float gt = m_above + above;
            int n = (int)ceilf((target - gt) / wt);
            n = max(1, min(n, (int)ch[bl]));
            s_bin = (int)key;
            s_u0 = (unsigned int)n;
            s_f1 = gt;
        }
        __syncthreads();
        kt = (uint32_t)s_bin;
        need_eq = (int)s_u0;
        mass_gt = s_f1;
    }

    // ---- the draw: target mass u * (mass above kt + its ties taken), walked
    // from the largest key down (equal keys by ascending index)
    const float wt = weight(kt);
    const float total = mass_gt + (float)need_eq * wt;
    const float target = uniform_of(a.seed, a.step, row) * total;
    uint32_t ks;      // the drawn key
    int j;            // which of its ties (ascending index)
    if (target >= mass_gt) {
        ks = kt;
        j = wt > 0.f ? min((int)((target - mass_gt) / wt), need_eq - 1) : 0;
    } else {
        clear();
        for (int i = tid; i < V; i += kSampleThreads) {
            const uint32_t key = key_of(lg[i]);
            if (key > kt) atomicAdd(&fh[key >> 8], weight(key));
        }
        __syncthreads();
        if (tid == 0) {
            float above = 0.f;
            int b = scan_down<float>(fh, target, false, &above);
            if (b < 0) {  // rounding: the lowest bin with mass
                b = 0;
                while (b < 255 && fh[b] == 0.f) ++b;
                above = 0.f;
                for (int q = 255; q > b; --q) above += fh[q];
            }
            s_bin = b;
            s_f0 = above;
        }
        __syncthreads();
        const int bh = s_bin;
        const float m_above = s_f0;
        __syncthreads();
        clear();
        for (int i = tid; i < V; i += kSampleThreads) {
            const uint32_t key = key_of(lg[i]);
            if (key > kt && (int)(key >> 8) == bh) {
                atomicAdd(&fh[key & 0xFFu], weight(key));
                atomicAdd(&ch[key & 0xFFu], 1u);
            }
        }
        __syncthreads();
        if (tid == 0) {
            float above = 0.f;
            int bl = scan_down<float>(fh, target - m_above, false, &above);
            if (bl < 0) {
                bl = 0;
                while (bl < 255 && ch[bl] == 0u) ++bl;
                above = 0.f;
                for (int q = 255; q > bl; --q) above += fh[q];
            }
            const uint32_t key = ((uint32_t)bh << 8) | (uint32_t)bl;
            const float wk = weight(key);
            s_bin = (int)key;
            s_idx = wk > 0.f ? min((int)((target - m_above - above) / wk), (int)ch[bl] - 1) : 0;
        }
        __syncthreads();
        ks = (uint32_t)s_bin;
        j = max(s_idx, 0);
    }

    // ---- the j-th index (ascending) holding key ks: per-thread counts over
    // contiguous chunks, an exclusive scan, then the owning thread's search
    const int chunk = (V + kSampleThreads - 1) / kSampleThreads;
    const int i0 = min(V, tid * chunk), i1 = min(V, i0 + chunk);
    int cnt = 0;
    for (int i = i0; i < i1; ++i) cnt += key_of(lg[i]) == ks;
    // inclusive scan of cnt over the block (warp shuffles, then warp totals)
    int incl = cnt;
    const int lane = tid & 31, warp = tid >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
    }
    __shared__ int wsum[32];
    if (lane == 31) wsum[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        int w = wsum[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += t;
        }
        wsum[lane] = w;  // inclusive over warps
    }
    __syncthreads();
    // j never passes the last index holding ks (wsum[31] of them): rounding
    // in the mass walk cannot leave the pre-set argmax standing in for a draw
    j = min(j, wsum[31] - 1);
    const int excl = incl - cnt + (warp > 0 ? wsum[warp - 1] : 0);
    if (j >= excl && j < excl + cnt) {
        int seen = excl;
        for (int i = i0; i < i1; ++i)
            if (key_of(lg[i]) == ks) {
                if (seen == j) {
                    a.tokens[row] = i;
                    break;
                }
                ++seen;
            }
    }
}

}  // namespace

cudaError_t launch_sample(const SampleArgs &a, cudaStream_t s) {
    if (a.rows <= 0) return cudaSuccess;
    sample_kernel<<<a.rows, kSampleThreads, 0, s>>>(a);
    return cudaGetLastError();
}

}  // namespace tllm
