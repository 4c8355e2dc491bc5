/*
 * CPU oracle for the paged KV cache + GQA decode-attention path.
 * TEST INFRASTRUCTURE ONLY: the checker for tests/, smoke() and bench.py's
 * cpu_baseline leg; never linked into the product. See oracle.h for what each
 * function restates and the reference file:line it follows.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ---------------------------------------------------------------- fp16 --- */

uint16_t or_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    uint32_t ax = x & 0x7fffffffu;
    if (ax > 0x7f800000u) return (uint16_t)(sign | 0x7e00u); /* NaN -> quiet NaN */
    if (ax >= 0x47800000u) return (uint16_t)(sign | 0x7c00u); /* >= 2^16 (or inf) -> inf */
    if (ax >= 0x38800000u) { /* result is a normal half (>= 2^-14) */
        uint32_t mant = ax & 0x7fffffu;
        uint32_t e = (ax >> 23) - 127u + 15u;
        uint32_t h = (e << 10) | (mant >> 13);
        uint32_t rem = mant & 0x1fffu;
        if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++; /* may carry into inf */
        return (uint16_t)(sign | h);
    }
    if (ax < 0x33000000u) return sign; /* below half of the smallest subnormal */
    {
        /* subnormal result, in units of 2^-24: value = m * 2^(e-150) */
        uint32_t e = ax >> 23;
        uint32_t m = (ax & 0x7fffffu) | 0x800000u;
        uint32_t shift = 126u - e; /* 14..24 */
        uint32_t h = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t halfway = 1u << (shift - 1u);
        if (rem > halfway || (rem == halfway && (h & 1u))) h++;
        return (uint16_t)(sign | h);
    }
}

float or_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu;
    uint32_t m = h & 0x3ffu;
    uint32_t x;
    if (e == 0) {
        if (m == 0) {
            x = sign;
        } else {
            uint32_t shift = 0;
            while (!(m & 0x400u)) {
                m <<= 1;
                shift++;
            }
            m &= 0x3ffu;
            x = sign | ((113u - shift) << 23) | (m << 13);
        }
    } else if (e == 31) {
        x = sign | 0x7f800000u | (m << 13);
    } else {
        x = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

void or_f32_to_f16_array(const float *src, uint16_t *dst, size_t n) {
    for (size_t i = 0; i < n; ++i) dst[i] = or_f32_to_f16(src[i]);
}

void or_f16_to_f32_array(const uint16_t *src, float *dst, size_t n) {
    for (size_t i = 0; i < n; ++i) dst[i] = or_f16_to_f32(src[i]);
}

/* ----------------------------------------------------------------- RNG --- */

static uint64_t splitmix64(uint64_t *s) {
    uint64_t z = (*s += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

void or_fill_normal_f16(uint16_t *dst, size_t n, uint64_t seed) {
    uint64_t s = seed;
    const double two_pi = 6.283185307179586476925286766559;
    for (size_t i = 0; i < n; i += 2) {
        /* u1 in (0, 1], u2 in [0, 1) with 53-bit resolution */
        double u1 = ((double)(splitmix64(&s) >> 11) + 1.0) * (1.0 / 9007199254740992.0);
        double u2 = (double)(splitmix64(&s) >> 11) * (1.0 / 9007199254740992.0);
        double r = sqrt(-2.0 * log(u1));
        dst[i] = or_f32_to_f16((float)(r * cos(two_pi * u2)));
        if (i + 1 < n) dst[i + 1] = or_f32_to_f16((float)(r * sin(two_pi * u2)));
    }
}

/* ---------------------------------------------------------------- RoPE --- */

void or_rope_table(float *cos_t, float *sin_t, int max_pos, int head_dim, float theta) {
    int half = head_dim / 2;
    for (int i = 0; i < half; ++i) {
        double freq = pow((double)theta, -2.0 * (double)i / (double)head_dim);
        for (int p = 0; p < max_pos; ++p) {
            double a = (double)p * freq;
            cos_t[(size_t)p * half + i] = (float)cos(a);
            sin_t[(size_t)p * half + i] = (float)sin(a);
        }
    }
}

void or_rope_row(uint16_t *dst, const uint16_t *src, int num_kv_heads, int head_dim,
                 const float *cos_t, const float *sin_t, int pos) {
    int half = head_dim / 2;
    const float *c = cos_t + (size_t)pos * half;
    const float *s = sin_t + (size_t)pos * half;
    for (int h = 0; h < num_kv_heads; ++h) {
        const uint16_t *x = src + (size_t)h * head_dim;
        uint16_t *y = dst + (size_t)h * head_dim;
        for (int i = 0; i < half; ++i) {
            float x1 = or_f16_to_f32(x[i]);
            float x2 = or_f16_to_f32(x[i + half]);
            /* each product and sum rounded to fp32 (no contraction) */
            float a = x1 * c[i];
            float b = x2 * s[i];
            float o1 = a - b;
            float d = x2 * c[i];
            float e = x1 * s[i];
            float o2 = d + e;
            y[i] = or_f32_to_f16(o1);
            y[i + half] = or_f32_to_f16(o2);
        }
    }
}

/* ---------------------------------------------------------- paged pool --- */

size_t or_pool_offset(const or_pool_geom *g, int layer, int kv, int block, int tok, int head) {
    size_t block_elems = (size_t)g->block_size * g->num_kv_heads * g->head_dim;
    size_t base = (((size_t)layer * 2 + kv) * g->num_blocks + block) * block_elems;
    if (g->head_major)
        return base + ((size_t)head * g->block_size + tok) * g->head_dim;
    return base + ((size_t)tok * g->num_kv_heads + head) * g->head_dim;
}

void or_append(uint16_t *pool, const or_pool_geom *g, const int *bt, int layer, int pos0,
               int n, const uint16_t *k, const uint16_t *v, const float *cos_t,
               const float *sin_t) {
    size_t row = (size_t)g->num_kv_heads * g->head_dim;
    uint16_t *tmp = (uint16_t *)malloc(row * sizeof(uint16_t));
    for (int j = 0; j < n; ++j) {
        int pos = pos0 + j;
        int blk = bt[pos / g->block_size];
        int tok = pos % g->block_size;
        const uint16_t *krow = k + (size_t)j * row;
        const uint16_t *vrow = v + (size_t)j * row;
        if (cos_t) {
            or_rope_row(tmp, krow, g->num_kv_heads, g->head_dim, cos_t, sin_t, pos);
            krow = tmp;
        }
        for (int h = 0; h < g->num_kv_heads; ++h) {
            memcpy(pool + or_pool_offset(g, layer, 0, blk, tok, h), krow + (size_t)h * g->head_dim,
                   (size_t)g->head_dim * 2);
            memcpy(pool + or_pool_offset(g, layer, 1, blk, tok, h), vrow + (size_t)h * g->head_dim,
                   (size_t)g->head_dim * 2);
        }
    }
    free(tmp);
}

void or_gather(const uint16_t *pool, const or_pool_geom *g, const int *bt, int layer, int S,
               uint16_t *k_out, uint16_t *v_out) {
    size_t row = (size_t)g->num_kv_heads * g->head_dim;
    for (int pos = 0; pos < S; ++pos) {
        int blk = bt[pos / g->block_size];
        int tok = pos % g->block_size;
        for (int h = 0; h < g->num_kv_heads; ++h) {
            memcpy(k_out + pos * row + (size_t)h * g->head_dim,
                   pool + or_pool_offset(g, layer, 0, blk, tok, h), (size_t)g->head_dim * 2);
            memcpy(v_out + pos * row + (size_t)h * g->head_dim,
                   pool + or_pool_offset(g, layer, 1, blk, tok, h), (size_t)g->head_dim * 2);
        }
    }
}

/* ------------------------------------------------------ decode (fp64) --- */

void or_decode_one(const uint16_t *q, const uint16_t *k, const uint16_t *v, int S,
                   int num_q_heads, int num_kv_heads, int head_dim, float scale, double eps,
                   float *out) {
    int G = num_q_heads / num_kv_heads;
    size_t row = (size_t)num_kv_heads * head_dim;
    double *sc = (double *)malloc(sizeof(double) * (S > 0 ? S : 1));
    double *acc = (double *)malloc(sizeof(double) * head_dim);
    for (int hq = 0; hq < num_q_heads; ++hq) {
        int kvh = hq / G;
        const uint16_t *qh = q + (size_t)hq * head_dim;
        if (S <= 0) {
            for (int d = 0; d < head_dim; ++d) out[(size_t)hq * head_dim + d] = 0.0f;
            continue;
        }
        double m = -INFINITY;
        for (int t = 0; t < S; ++t) {
            const uint16_t *kt = k + t * row + (size_t)kvh * head_dim;
            double s = 0.0;
            for (int d = 0; d < head_dim; ++d)
                s += (double)or_f16_to_f32(qh[d]) * (double)or_f16_to_f32(kt[d]);
            s *= (double)scale;
            sc[t] = s;
            if (s > m) m = s;
        }
        double l = 0.0;
        for (int d = 0; d < head_dim; ++d) acc[d] = 0.0;
        for (int t = 0; t < S; ++t) {
            double p = exp(sc[t] - m);
            l += p;
            const uint16_t *vt = v + t * row + (size_t)kvh * head_dim;
            for (int d = 0; d < head_dim; ++d) acc[d] += p * (double)or_f16_to_f32(vt[d]);
        }
        for (int d = 0; d < head_dim; ++d)
            out[(size_t)hq * head_dim + d] = (float)(acc[d] / (l + eps));
    }
    free(sc);
    free(acc);
}

/* ------------------------------------------- timed CPU baseline (fp32) --- */

static void decode_unit_f32(const uint16_t *pool, const or_pool_geom *g, int layer,
                            const int *bt, int S, const uint16_t *q, int G, int kvh, float scale,
                            uint16_t *out, float *scores, float *qf, float *acc) {
    int D = g->head_dim;
    for (int gi = 0; gi < G; ++gi) {
        int hq = kvh * G + gi;
        for (int d = 0; d < D; ++d) qf[d] = or_f16_to_f32(q[(size_t)hq * D + d]);
        float m = -INFINITY;
        for (int t = 0; t < S; ++t) {
            const uint16_t *kt =
                pool + or_pool_offset(g, layer, 0, bt[t / g->block_size], t % g->block_size, kvh);
            float s = 0.0f;
            for (int d = 0; d < D; ++d) s += qf[d] * or_f16_to_f32(kt[d]);
            s *= scale;
            scores[t] = s;
            m = s > m ? s : m;
        }
        float l = 0.0f;
        for (int t = 0; t < S; ++t) {
            scores[t] = expf(scores[t] - m);
            l += scores[t];
        }
        float inv = 1.0f / (l + 1e-6f);
        for (int d = 0; d < D; ++d) acc[d] = 0.0f;
        for (int t = 0; t < S; ++t) {
            const uint16_t *vt =
                pool + or_pool_offset(g, layer, 1, bt[t / g->block_size], t % g->block_size, kvh);
            float p = scores[t] * inv;
            for (int d = 0; d < D; ++d) acc[d] += p * or_f16_to_f32(vt[d]);
        }
        for (int d = 0; d < D; ++d) out[(size_t)hq * D + d] = or_f32_to_f16(acc[d]);
    }
}

int or_decode_paged_f32(const uint16_t *pool, const or_pool_geom *g, int layer, int B,
                        const int *bt, int bt_stride, const int *lens, const uint16_t *q,
                        int num_q_heads, float scale, uint16_t *out, int threads) {
    int Hkv = g->num_kv_heads;
    int G = num_q_heads / Hkv;
    int D = g->head_dim;
    int maxS = 1;
    for (int b = 0; b < B; ++b) maxS = lens[b] > maxS ? lens[b] : maxS;
    int used = 1;
#ifdef _OPENMP
    if (threads < 1) threads = omp_get_max_threads();
    used = threads;
#pragma omp parallel num_threads(threads)
#endif
    {
        float *scores = (float *)malloc(sizeof(float) * maxS);
        float *qf = (float *)malloc(sizeof(float) * D);
        float *acc = (float *)malloc(sizeof(float) * D);
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
        for (int u = 0; u < B * Hkv; ++u) {
            int b = u / Hkv, kvh = u % Hkv;
            decode_unit_f32(pool, g, layer, bt + (size_t)b * bt_stride, lens[b],
                            q + (size_t)b * num_q_heads * D, G, kvh, scale,
                            out + (size_t)b * num_q_heads * D, scores, qf, acc);
        }
        free(scores);
        free(qf);
        free(acc);
    }
    return used;
}

/* kernels/w8a16_matmul.cu:71-93 (reference kernel) restated. */
void or_w8a16_matmul(const uint16_t *x, const int8_t *w, const uint16_t *scales, int M, int N, int K,
                     int group, float *out, int threads) {
    if (M <= 0 || N <= 0 || K <= 0 || group <= 0) return;
    const long long total = (long long)M * N;
#pragma omp parallel for schedule(static) num_threads(threads > 1 ? threads : 1)
    for (long long i = 0; i < total; ++i) {
        const int r = (int)(i / N), n = (int)(i % N);
        float sum = 0.0f;
        for (int k = 0; k < K; ++k) {
            const float a = or_f16_to_f32(x[(size_t)r * K + k]);
            const float s = or_f16_to_f32(scales[(size_t)(k / group) * N + n]);
            const float wk = (float)w[(size_t)k * N + n] * s;
            sum = fmaf(a, wk, sum);
        }
        out[i] = sum;
    }
}
