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
// One thread-block cluster of kCtas CTAs per row. Each CTA owns a contiguous
// slice of the row, reads it from global memory once and keeps it in shared
// memory as 16-bit keys that order like the values (-0 folded into +0, NaN
// lowest and weightless). Thresholds and the draw are found with 256-bin
// histograms over the key's high byte, then its low byte within one bin
// (counts for top-k, probability mass for top-p and the draw). Masses are
// exact integers: each weight exp((l - max) / T) <= 1 in units of 2^-40, so
// histogram sums are associative and every CTA of the cluster derives the
// same thresholds. Every warp fills its own histogram copy (no atomics
// between warps; a mass bin is two 32-bit words, the low word's atomic add
// returning the carry into the high one, since 32-bit shared-memory atomics
// are far cheaper than 64-bit ones), the CTA sums its copies, every CTA sums the cluster's CTA
// histograms through distributed shared memory, and one warp turns the
// result into suffix sums and finds thresholds with ballots. Once the first
// pass has placed the threshold in a high-byte bin, every CTA lists the slice
// positions of its keys in that bin and above (up to 4096; more, and the
// later passes scan the whole slice as before), and the later passes (low
// bytes of one such bin, the drawn key's count) read only the list, their few
// keys into one CTA-wide histogram instead of one per warp. The index
// among equal keys comes from per-CTA counts, a prefix over the cluster's
// ranks (slices are in index order) and one block-wide scan in the CTA that
// holds it.
#include <cooperative_groups.h>
#include <cstdint>
#include <cuda_fp16.h>
#include <map>
#include <mutex>

#include "kernels.h"

namespace cg = cooperative_groups;

namespace tllm {
namespace {

constexpr int kCtas = 8;          // CTAs per row (one cluster)
constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxSlice = 65536;  // keys per CTA: vocabularies up to kCtas * kMaxSlice
constexpr float kFx = 1099511627776.0f;  // 2^40: the unit of an integer mass
constexpr int kCandCap = 4096;    // slice positions of the keys at or above the threshold bin

using u64 = unsigned long long;

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

// What every CTA publishes for the others to read. Double-buffered: a buffer
// is written again two reductions later, after the cluster barrier that
// follows every reader's use of it.
struct Pub {
    u64 mass[256];
    unsigned cnt[256];
    u64 best;
    unsigned count;
};

struct Shared {
    unsigned wlo[kWarps][256];  // per-warp mass histograms: low and high words
    unsigned whi[kWarps][256];
    unsigned wcnt[kWarps][256];
    u64 gmass[256];          // the cluster's histograms of the last pass
    unsigned gcnt[256];
    u64 amass[256];          // their suffix sums: bins above b
    unsigned acnt[256];
    u64 hmass1[256];         // the first pass's masses and suffix sums
    u64 amass1[256];
    Pub pub[2];
    u64 red64[kWarps];
    unsigned redu[kWarps];
    unsigned wpre[kWarps];
    u64 s_u[4];
    int s_int[4];
    unsigned ncand;
    uint16_t cand[kCandCap];  // the candidates' slice positions (any order)
};

__device__ __forceinline__ u64 warp_max64(u64 v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const u64 t = __shfl_xor_sync(0xffffffffu, v, o);
        v = t > v ? t : v;
    }
    return v;
}
__device__ __forceinline__ int warp_max_int(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ int warp_min_int(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ unsigned warp_sum(unsigned v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// One warp: above[b] = sum of h over the bins above b (lane l holds bins
// 8l .. 8l+7).
template <typename T>
__device__ __forceinline__ void suffix_warp(const T *h, T *above, int lane) {
    T s = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) s += h[8 * lane + i];
    T incl = s;  // sum over lanes >= this one
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const T t = __shfl_down_sync(0xffffffffu, incl, o);
        if (lane + o < 32) incl += t;
    }
    T run = incl - s;  // exact: integers
#pragma unroll
    for (int i = 7; i >= 0; --i) {
        above[8 * lane + i] = run;
        run += h[8 * lane + i];
    }
}

// One warp: the highest bin b >= lo where the running total from the top,
// above[b] + h[b], reaches `target` (reach) or exceeds it; -1 if none. The
// running total only grows downwards, so this is the first such bin from
// the top.
template <typename T>
__device__ __forceinline__ int find_top(const T *h, const T *above, T target, bool reach, int lo, int lane) {
    int best = -1;
    for (int b = lane; b < 256; b += 32) {
        if (b < lo) continue;
        const T v = above[b] + h[b];
        if (reach ? v >= target : v > target) best = max(best, b);
    }
    return warp_max_int(best);
}
// One warp: the lowest bin b >= lo with a nonzero count (256 if none).
__device__ __forceinline__ int lowest_nonzero(const unsigned *c, int lo, int lane) {
    int best = 256;
    for (int b = lane; b < 256; b += 32)
        if (b >= lo && c[b] != 0u) best = min(best, b);
    return warp_min_int(best);
}

__global__ void __cluster_dims__(kCtas, 1, 1) __launch_bounds__(kThreads)
    sample_kernel(const __grid_constant__ SampleArgs a) {
    extern __shared__ __align__(16) unsigned char dyn[];
    Shared &sh = *reinterpret_cast<Shared *>(dyn);
    uint16_t *skey = reinterpret_cast<uint16_t *>(dyn + sizeof(Shared));
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();
    const int row = blockIdx.x / kCtas, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int V = a.vocab;
    const int per = (V + kCtas - 1) / kCtas;
    const int start = min(V, rank * per), n = min(V, start + per) - start;
    const uint16_t *lg = static_cast<const uint16_t *>(a.logits) + (long long)row * a.row_stride;
    int stage = 0;  // the Pub buffer the next reduction writes

    // ---- the slice as keys in shared memory; the largest key, first index
    u64 best = 0;
    for (int i = tid; i < n; i += kThreads) {
        const uint32_t key = key_of(lg[start + i]);
        skey[i] = (uint16_t)key;
        const u64 v = ((u64)key << 32) | (0xFFFFFFFFu - (unsigned)(start + i));
        best = v > best ? v : best;
    }
    best = warp_max64(best);
    if (lane == 0) sh.red64[warp] = best;
    __syncthreads();
    if (warp == 0) {
        u64 b = warp_max64(lane < kWarps ? sh.red64[lane] : 0ull);
        if (lane == 0) sh.pub[stage].best = b;
    }
    cluster.sync();
    if (warp == 0) {
        const u64 o = lane < kCtas ? cluster.map_shared_rank(&sh.pub[stage], lane)->best : 0ull;
        const u64 b = warp_max64(o);
        if (lane == 0) sh.s_u[0] = b;
    }
    stage ^= 1;
    __syncthreads();
    const u64 gbest = sh.s_u[0];
    const uint32_t kmax = (uint32_t)(gbest >> 32);
    const int argmax = (int)(0xFFFFFFFFu - (uint32_t)(gbest & 0xFFFFFFFFu));
    if (a.mode == 0 || kmax == 0u) {  // greedy (a NaN first logit wins in the reference's loop); all NaN: 0
        if (rank == 0 && tid == 0) {
            const uint16_t h0 = lg[0];
            const bool nan0 = (h0 & 0x7C00u) == 0x7C00u && (h0 & 0x03FFu) != 0;
            a.tokens[row] = nan0 || kmax == 0u ? 0 : argmax;
        }
        cluster.sync();  // no CTA leaves while another may still read its shared memory
        return;
    }
    const float m = value_of(kmax);
    const float c = 1.4426950408889634f / a.temperature;  // exp((l - m) / T) = 2^((l - m) c)
    // integer mass of a key: its weight in units of 2^-40 (NaN: 0)
    auto fx = [&](uint32_t key) -> u64 {
        return key == 0u ? 0ull : (u64)__float2ull_rn(exp2f((value_of(key) - m) * c) * kFx);
    };

    bool use_list = false;  // set once the candidates are listed (after the first pass)
    int ncand = 0;
    // One histogram pass over the slice and its cluster reduction into
    // sh.gmass / sh.gcnt and their suffix sums: the keys with high byte ==
    // sel (sel < 0: every key), at their high byte (sel < 0) or low byte.
    auto histogram = [&](int sel) {
        // a later pass looks at one bin at or above the threshold bin: the
        // candidate list holds all of its keys when it did not overflow, and
        // its few keys share one histogram (copy 0) instead of one per warp
        const bool from_list = sel >= 0 && use_list;
        const int hw = from_list ? 0 : warp, ncopies = from_list ? 1 : kWarps;
        if (from_list) {
            for (int b = tid; b < 256; b += kThreads) {
                sh.wlo[0][b] = 0u;
                sh.whi[0][b] = 0u;
                sh.wcnt[0][b] = 0u;
            }
            __syncthreads();
        } else {
            for (int b = lane; b < 256; b += 32) {
                sh.wlo[warp][b] = 0u;
                sh.whi[warp][b] = 0u;
                sh.wcnt[warp][b] = 0u;
            }
            __syncwarp();
        }
        const int cnt_keys = from_list ? ncand : n;
        for (int c = tid; c < cnt_keys; c += kThreads) {
            const int i = from_list ? (int)sh.cand[c] : c;
            const uint32_t key = skey[i];
            if (sel < 0 || (int)(key >> 8) == sel) {
                const int b = sel < 0 ? (int)(key >> 8) : (int)(key & 0xFFu);
                // the 64-bit mass as two 32-bit words: the low word's add
                // returns the old value, whose wrap is the carry into the
                // high word (added only when nonzero: masses of 2^32 units
                // and more are the keys near the maximum)
                const u64 x = fx(key);
                const unsigned xlo = (unsigned)x;
                const unsigned old = atomicAdd(&sh.wlo[hw][b], xlo);
                const unsigned up = (unsigned)(x >> 32) + (old + xlo < old ? 1u : 0u);
                if (up) atomicAdd(&sh.whi[hw][b], up);
                atomicAdd(&sh.wcnt[hw][b], 1u);
            }
        }
        __syncthreads();
        Pub &p = sh.pub[stage];
        for (int b = tid; b < 256; b += kThreads) {
            u64 ms = 0ull;
            unsigned cs = 0u;
            for (int w = 0; w < ncopies; ++w) {
                ms += ((u64)sh.whi[w][b] << 32) + sh.wlo[w][b];
                cs += sh.wcnt[w][b];
            }
            p.mass[b] = ms;
            p.cnt[b] = cs;
        }
        cluster.sync();
        for (int b = tid; b < 256; b += kThreads) {
            u64 ms = 0ull;
            unsigned cs = 0u;
            for (int r = 0; r < kCtas; ++r) {
                const Pub *o = cluster.map_shared_rank(&p, r);
                ms += o->mass[b];
                cs += o->cnt[b];
            }
            sh.gmass[b] = ms;
            sh.gcnt[b] = cs;
        }
        stage ^= 1;
        __syncthreads();
        if (warp == 0) {
            suffix_warp<u64>(sh.gmass, sh.amass, lane);
            suffix_warp<unsigned>(sh.gcnt, sh.acnt, lane);
        }
        __syncthreads();
    };

    // ---- the candidate threshold kt (the lowest candidate key), the mass of
    // the keys above it and how many of its ties join (lowest indices first)
    histogram(-1);
    for (int b = tid; b < 256; b += kThreads) {
        sh.hmass1[b] = sh.gmass[b];
        sh.amass1[b] = sh.amass[b];
    }
    if (warp == 0) {
        const u64 z = sh.amass[0] + sh.gmass[0];
        int bh;
        unsigned c_above = 0u;
        u64 target = 0ull;
        if (a.mode == 1) {  // top-k (temperature: k = V)
            bh = find_top<unsigned>(sh.gcnt, sh.acnt, (unsigned)a.top_k, true, 0, lane);
            if (bh < 0) bh = 0;  // (cannot happen: k <= V)
            c_above = sh.acnt[bh];
        } else {  // top-p: the smallest descending prefix reaching p of the total
            target = (u64)((double)a.top_p * (double)z);
            if (target == 0ull) target = 1ull;
            bh = find_top<u64>(sh.gmass, sh.amass, target, true, 0, lane);
            if (bh < 0) bh = lowest_nonzero(sh.gcnt, 0, lane);  // rounding: everything
        }
        if (lane == 0) {
            sh.s_int[0] = bh;
            sh.s_int[1] = (int)c_above;
            sh.s_u[0] = target;
        }
    }
    __syncthreads();
    const int bh = sh.s_int[0];
    const unsigned c_above1 = (unsigned)sh.s_int[1];
    const u64 p_target = sh.s_u[0];
    const u64 m_above1 = sh.amass1[bh];
    // ---- list the slice positions of the keys in bin bh and above: every
    // later pass (the low bytes of a bin >= bh, the drawn key's count) reads
    // only them. One warp-aggregated shared-memory atomic per warp and round;
    // past kCandCap entries the passes scan the whole slice instead.
    if (tid == 0) sh.ncand = 0u;
    __syncthreads();
    for (int base = 0; base < n; base += kThreads) {
        const int i = base + tid;
        const bool take = i < n && (int)(skey[i] >> 8) >= bh;
        const unsigned mask = __ballot_sync(0xffffffffu, take);
        if (mask) {
            unsigned pos = 0u;
            if (lane == 0) pos = atomicAdd(&sh.ncand, (unsigned)__popc(mask));
            pos = __shfl_sync(0xffffffffu, pos, 0) + (unsigned)__popc(mask & ((1u << lane) - 1u));
            if (take && pos < (unsigned)kCandCap) sh.cand[pos] = (uint16_t)i;
        }
    }
    __syncthreads();
    ncand = (int)sh.ncand;
    use_list = ncand <= kCandCap;

    histogram(bh);  // the low bytes of bin bh
    if (warp == 0) {
        int bl, neq;
        if (a.mode == 1) {
            const unsigned need = (unsigned)a.top_k - c_above1;
            bl = find_top<unsigned>(sh.gcnt, sh.acnt, need, true, 0, lane);
            if (bl < 0) bl = 0;  // (cannot happen: bin bh holds the k-th key)
            neq = (int)(need - sh.acnt[bl]);
        } else {
            const u64 rest = p_target > m_above1 ? p_target - m_above1 : 0ull;
            bl = find_top<u64>(sh.gmass, sh.amass, rest, true, 0, lane);
            if (bl < 0) bl = lowest_nonzero(sh.gcnt, 0, lane);  // rounding: the lowest key of the bin
            if (bl > 255) bl = 255;
            const u64 gt = m_above1 + sh.amass[bl];
            const u64 wkt = sh.gcnt[bl] ? sh.gmass[bl] / sh.gcnt[bl] : 0ull;  // one key's mass
            const u64 need = p_target > gt ? p_target - gt : 0ull;
            neq = wkt ? (int)min((u64)sh.gcnt[bl], (need + wkt - 1) / wkt) : (int)sh.gcnt[bl];
            neq = max(1, neq);
        }
        if (lane == 0) {
            sh.s_int[0] = (int)(((uint32_t)bh << 8) | (uint32_t)bl);
            sh.s_int[1] = neq;
            sh.s_u[0] = m_above1 + sh.amass[bl];  // mass above kt
            sh.s_u[1] = sh.gcnt[bl] ? sh.gmass[bl] / sh.gcnt[bl] : 0ull;
        }
    }
    __syncthreads();
    const uint32_t kt = (uint32_t)sh.s_int[0];
    const int need_eq = sh.s_int[1];
    const u64 mass_gt = sh.s_u[0], wt = sh.s_u[1];
    __syncthreads();

    // ---- the draw: target mass u * (mass above kt + its ties taken), walked
    // from the largest key down (equal keys by ascending index)
    const u64 total = mass_gt + (u64)need_eq * wt;
    const u64 target = (u64)((double)uniform_of(a.seed, a.step, row) * (double)total);
    uint32_t ks;  // the drawn key
    int j;        // which of its ties (ascending index)
    if (target >= mass_gt) {
        ks = kt;
        j = wt ? (int)min((u64)(need_eq - 1), (target - mass_gt) / wt) : 0;
    } else {
        // the high byte: bins above bh from the first pass, else bin bh
        if (warp == 0) {
            int sel = find_top<u64>(sh.hmass1, sh.amass1, target, false, bh + 1, lane);
            if (sel < 0) sel = bh;
            if (lane == 0) sh.s_int[0] = sel;
        }
        __syncthreads();
        const int bsel = sh.s_int[0];
        const u64 m_above = sh.amass1[bsel];
        __syncthreads();
        // the low byte: bin bh's keys above kt are in the second pass's
        // histogram, another bin needs its own pass
        if (bsel != bh) histogram(bsel);
        if (warp == 0) {
            const int lo_min = bsel == bh ? (int)(kt & 0xFFu) + 1 : 0;  // keys above kt only
            const u64 rest = target > m_above ? target - m_above : 0ull;
            int bl = find_top<u64>(sh.gmass, sh.amass, rest, false, lo_min, lane);
            if (bl < 0) bl = min(255, lowest_nonzero(sh.gcnt, lo_min, lane));  // rounding: the lowest key
            const u64 wk = sh.gcnt[bl] ? sh.gmass[bl] / sh.gcnt[bl] : 0ull;
            const u64 in_bin = rest > sh.amass[bl] ? rest - sh.amass[bl] : 0ull;
            if (lane == 0) {
                sh.s_int[0] = (int)(((uint32_t)bsel << 8) | (uint32_t)bl);
                sh.s_int[1] = wk ? (int)min((u64)max((int)sh.gcnt[bl] - 1, 0), in_bin / wk) : 0;
            }
        }
        __syncthreads();
        ks = (uint32_t)sh.s_int[0];
        j = sh.s_int[1];
        __syncthreads();
    }

    // ---- the j-th index (ascending) holding key ks: per-CTA counts, a prefix
    // over the ranks, then a block-wide scan in the CTA that holds it
    const int chunk = (n + kThreads - 1) / kThreads;
    const int i0 = min(n, tid * chunk), i1 = min(n, i0 + chunk);
    unsigned cnt = 0;  // this thread's contiguous range (the scan below); the list when it serves
    if (use_list) {
        for (int c = tid; c < ncand; c += kThreads) cnt += skey[sh.cand[c]] == ks;
    } else {
        for (int i = i0; i < i1; ++i) cnt += skey[i] == ks;
    }
    const unsigned wcount = warp_sum(cnt);
    if (lane == 0) sh.redu[warp] = wcount;
    __syncthreads();
    if (warp == 0) {
        const unsigned t = warp_sum(lane < kWarps ? sh.redu[lane] : 0u);
        if (lane == 0) sh.pub[stage].count = t;
    }
    cluster.sync();
    if (warp == 0) {
        const unsigned cr = lane < kCtas ? cluster.map_shared_rank(&sh.pub[stage], lane)->count : 0u;
        const unsigned pre = warp_sum(lane < rank ? cr : 0u);
        const unsigned total_ks = warp_sum(cr);
        if (lane == 0) {
            // j never passes the last index holding ks: the row always gets
            // a drawn token
            const int jj = min(j, (int)total_ks - 1);
            const int local = jj - (int)pre;
            sh.s_int[0] = local;
            sh.s_int[1] = (int)total_ks;
            sh.s_int[2] = total_ks > 0 && local >= 0 && local < (int)sh.pub[stage].count;
        }
    }
    __syncthreads();
    const int jl = sh.s_int[0];
    if (sh.s_int[1] == 0 && rank == 0 && tid == 0) a.tokens[row] = argmax;  // (cannot happen)
    if (sh.s_int[2]) {  // this CTA holds the drawn index
        if (use_list) {  // the list is in no particular order: count the contiguous ranges
            cnt = 0;
            for (int i = i0; i < i1; ++i) cnt += skey[i] == ks;
        }
        unsigned incl = cnt;  // inclusive scan over the block: warp shuffles, then warp totals
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned t = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += t;
        }
        if (lane == 31) sh.wpre[warp] = incl;
        __syncthreads();
        if (tid == 0) {
            unsigned run = 0;
            for (int w = 0; w < kWarps; ++w) {
                const unsigned t = sh.wpre[w];
                sh.wpre[w] = run;
                run += t;
            }
        }
        __syncthreads();
        const int excl = (int)(incl - cnt + sh.wpre[warp]);
        if (jl >= excl && jl < excl + (int)cnt) {
            int seen = excl;
            for (int i = i0; i < i1; ++i)
                if (skey[i] == ks) {
                    if (seen == jl) {
                        a.tokens[row] = start + i;
                        break;
                    }
                    ++seen;
                }
        }
    }
    cluster.sync();  // no CTA leaves while another may still read its shared memory
}

}  // namespace

cudaError_t launch_sample(const SampleArgs &a, cudaStream_t s) {
    if (a.rows <= 0) return cudaSuccess;
    if (a.vocab > kCtas * kMaxSlice || a.rows > (1 << 27)) return cudaErrorInvalidValue;
    const int per = (a.vocab + kCtas - 1) / kCtas;
    const int dyn = (int)(sizeof(Shared) + ((((size_t)per * 2) + 15) & ~size_t(15)));
    // shared-memory opt-in per device, only ever raised (under one lock)
    static std::mutex mu;
    static std::map<int, int> opted;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    {
        std::lock_guard<std::mutex> lock(mu);
        int &cur = opted[dev];
        if (cur < dyn) {
            e = cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn);
            if (e != cudaSuccess) return e;
            cur = dyn;
        }
    }
    sample_kernel<<<a.rows * kCtas, kThreads, dyn, s>>>(a);
    return cudaGetLastError();
}

int sample_max_vocab() { return kCtas * kMaxSlice; }

}  // namespace tllm
